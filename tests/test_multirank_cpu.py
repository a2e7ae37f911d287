"""N > 1 host logic on CPU ranks (gloo, world_size 2).

1. Sequence partitioning (one pool per GPU, no collective): every rank computes the same LPT
   assignment, the shards cover every sequence once, and concatenating the ranks' oracle
   outputs reproduces the single-process batch.
2. Long-context split-KV: each rank attends its contiguous block range and produces
   partials (max, sum, acc); an all-gather plus a log-sum-exp merge reproduces the
   single-process result.  This is the exchange the multi-GPU cfg5 path performs.
"""
import math
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _partials(K, V, g, ids, n_tok, q, n_heads, scale):
    """(m, l, acc) of one rank's block range, in float64 (natural-log max)."""
    nkv = g.heads_kv
    grp = n_heads // nkv
    rows = [(ids[t // g.block_size], t % g.block_size) for t in range(n_tok)]
    m = np.full(n_heads, -np.inf)
    l = np.zeros(n_heads)
    acc = np.zeros((n_heads, g.v_head_dim))
    for h in range(n_heads):
        kv = h // grp
        if not rows:
            continue
        kk = np.stack([K[b, 0, kv, o] for b, o in rows]).astype(np.float64)
        vv = np.stack([V[b, 0, kv, o] for b, o in rows]).astype(np.float64)
        s = kk @ q[h].astype(np.float64) * scale
        m[h] = s.max()
        p = np.exp(s - m[h])
        l[h] = p.sum()
        acc[h] = p @ vv
    return m, l, acc


def _worker(rank, world, port, ret):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "glacier.serve_b200")]
    import torch
    import torch.distributed as dist

    import glacier_kv as G
    from oracle import pyoracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(77)  # same inputs on every rank
        nH, nKv, d, bs = 8, 2, 32, 16
        ctx = rng.integers(1, 200, size=13).astype(np.int32)
        total = int(sum((c + bs - 1) // bs for c in ctx)) + 2
        g = O.geom(total, 1, nKv, d, d, bs)
        K, V = O.new_arena(g)
        K[...] = rng.standard_normal(K.shape)
        V[...] = rng.standard_normal(V.shape)
        perm = rng.permutation(total).astype(np.int32)
        mb = int(max((c + bs - 1) // bs for c in ctx))
        tables = np.full((len(ctx), mb), -1, np.int32)
        at = 0
        for i, c in enumerate(ctx):
            n = (int(c) + bs - 1) // bs
            tables[i, :n] = perm[at:at + n]
            at += n
        q = rng.standard_normal((len(ctx), nH, d)).astype(np.float32)
        scale = 1 / math.sqrt(d)

        # 1. sequence partitioning
        assign = G.partition_lpt(ctx, world)
        gathered = [torch.zeros(len(ctx), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(assign))
        agree = all(torch.equal(x, gathered[0]) for x in gathered)
        mine = np.nonzero(assign == rank)[0]
        out = np.zeros((len(ctx), nH, d), np.float32)
        if mine.size:
            out[mine] = O.decode_batch(K, V, g, 0, tables[mine], ctx[mine], q[mine], nH, scale)
        t = torch.from_numpy(out)
        dist.all_reduce(t)  # shards are disjoint: the sum is the concatenation
        full = O.decode_batch(K, V, g, 0, tables, ctx, q, nH, scale)
        shard_err = float(np.abs(t.numpy() - full).max())

        # 2. split-KV over contiguous block ranges of one long sequence
        seq = int(np.argmax(ctx))
        nblk = (int(ctx[seq]) + bs - 1) // bs
        b0, b1 = G.split_block_range(nblk, world, rank)
        n_local = max(0, min(int(ctx[seq]), b1 * bs) - b0 * bs)
        m, l, acc = _partials(K, V, g, tables[seq, b0:b1], n_local, q[seq], nH, scale)
        payload = torch.from_numpy(np.concatenate([m[:, None], l[:, None], acc], 1))
        parts = [torch.zeros_like(payload) for _ in range(world)]
        dist.all_gather(parts, payload)
        P = torch.stack(parts).numpy()  # [world, nH, 2 + dv]
        M = P[:, :, 0].max(0)
        f = np.exp(P[:, :, 0] - M)
        f[~np.isfinite(f)] = 0.0
        merged = (P[:, :, 2:] * f[:, :, None]).sum(0) / (P[:, :, 1] * f).sum(0)[:, None]
        split_err = float(np.abs(merged - full[seq]).max())
        ret[rank] = (agree, shard_err, split_err, sorted(mine.tolist()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_split_kv():
    import torch.multiprocessing as mp

    port = _free_port()
    mgr = mp.Manager()
    ret = mgr.dict()
    mp.spawn(_worker, args=(2, port, ret), nprocs=2, join=True)
    r0, r1 = ret[0], ret[1]
    assert r0[0] and r1[0], "ranks disagree on the LPT assignment"
    assert r0[1] < 1e-6 and r1[1] < 1e-6
    assert r0[2] < 1e-5 and r1[2] < 1e-5
    assert sorted(r0[3] + r1[3]) == list(range(13)) and not set(r0[3]) & set(r1[3])
