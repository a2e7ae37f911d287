"""Long-context split-KV across ranks: per-range decode with log-sum-exp, the LSE merge, and
the NCCL exchange (2-GPU part skips on a 1-GPU box)."""
import math
import os
import socket

import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, geom_of, random_arena, random_tables
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _range_tables(tables, ctx, bs, world, rank):
    """Rank `rank`'s contiguous block range of every sequence (empty ranges allowed)."""
    B = len(ctx)
    nb = [(int(c) + bs - 1) // bs for c in ctx]
    rows, lens = [], []
    for b in range(B):
        b0, b1 = G.split_block_range(nb[b], world, rank)
        rows.append(tables[b, b0:b1])
        lens.append(max(0, min(int(ctx[b]), b1 * bs) - b0 * bs))
    mb = max(1, max(len(r) for r in rows))
    t = np.full((B, mb), -1, np.int32)
    for b, r in enumerate(rows):
        t[b, :len(r)] = r
    return t, np.array(lens, np.int32)


@pytest.mark.parametrize("dtype,nH,nKv", [("f32", 28, 4), ("bf16", 64, 8)])
def test_emulated_ranks_merge_to_full_decode(cuda, dtype, nH, nKv):
    import torch

    rng = np.random.default_rng(41)
    bs, d = 16, 128
    ctx = [4000, 31, 1500, 200]  # the short ones leave some ranks empty
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = G.PagedBlockPool(need + 3, 1, nKv, d, bs, dtype=dtype)
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, ctx, bs, need + 3)
    q = rng.standard_normal((len(ctx), nH, d)).astype(np.float32)
    qd = torch.from_numpy(q).to(cuda)
    world = 5
    rows = len(ctx) * nH
    parts = torch.empty((world, rows * (d + 1)), device=cuda)
    for r in range(world):
        t, lens = _range_tables(tables, ctx, bs, world, r)
        out_r = parts[r, : rows * d].view(len(ctx), nH, d)
        lse_r = parts[r, rows * d:].view(len(ctx), nH)
        lse_r.fill_(-math.inf)
        pool.upload_step(t, lens)
        pool.paged_decode_lse(0, qd, out_r, lse_r, nH, 1 / math.sqrt(d))
    sinks = torch.full((nH,), 0.4, device=cuda)
    for sk in (None, sinks):
        out = torch.zeros((len(ctx), nH, d), device=cuda)
        G.lse_merge(parts.view(-1), world, rows, d, out.view(-1), sinks=sk, n_heads=nH)
        torch.cuda.synchronize(cuda)
        ref = O.decode_batch(K, V, geom_of(pool), 0, tables, np.array(ctx, np.int32), q, nH, 1 / math.sqrt(d),
                             sink_logit=None if sk is None else 0.4)
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL[dtype], rtol=0)
    pool.close()


def test_lse_matches_the_softmax_denominator(cuda):
    import torch

    rng = np.random.default_rng(42)
    pool = G.PagedBlockPool(40, 1, 2, 64, 16)
    K, V = random_arena(pool, rng)
    ctx = [300, 9]
    tables = random_tables(rng, ctx, 16, 40)
    q = rng.standard_normal((2, 4, 64)).astype(np.float32)
    out = torch.zeros((2, 4, 64), device=cuda)
    lse = torch.zeros((2, 4), device=cuda)
    pool.upload_step(tables, np.array(ctx, np.int32))
    pool.paged_decode_lse(0, torch.from_numpy(q).to(cuda), out, lse, 4, 0.125)
    torch.cuda.synchronize(cuda)
    for b, c in enumerate(ctx):
        for h in range(4):
            kk = np.stack([K[tables[b, t // 16], 0, h // 2, t % 16] for t in range(c)]).astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) * 0.125
            ref = s.max() + math.log(np.exp(s - s.max()).sum())
            assert abs(float(lse[b, h]) - ref) < 1e-4
    pool.close()


def test_comm_init_times_out_when_a_peer_never_joins(cuda):
    """The failure is made on the host: rank 1 of 2 never calls init; rank 0's bounded wait
    must end with GKV_ETIMEDOUT (after aborting the communicator), not hang."""
    uid = G.Comm.unique_id()
    with pytest.raises(G.TimeoutError_):
        G.Comm(uid, 2, 0, 0, timeout_ms=3000)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dist_worker(rank, world, q_uid, ret):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "glacier.serve_b200"), os.path.join(root, "tests")]
    import torch

    import glacier_kv as G2
    from oracle import pyoracle as O2

    torch.cuda.set_device(rank)
    dev = torch.device(f"cuda:{rank}")
    rng = np.random.default_rng(43)  # identical full problem on every rank
    bs, d, nH, nKv = 16, 128, 64, 8
    ctx = np.array([6000, 2048, 100], np.int32)
    nb = [(int(c) + bs - 1) // bs for c in ctx]
    total = sum(nb)
    Kf = rng.standard_normal((total, 1, nKv, bs, d)).astype(np.float32)
    Vf = rng.standard_normal((total, 1, nKv, bs, d)).astype(np.float32)
    Kb, Vb = O2.f32_to_bf16_bits(Kf), O2.f32_to_bf16_bits(Vf)
    tables = np.full((3, max(nb)), -1, np.int32)
    at = 0
    for b, n in enumerate(nb):
        tables[b, :n] = np.arange(at, at + n)
        at += n
    q = rng.standard_normal((3, nH, d)).astype(np.float32)
    # this rank's pool holds only its block ranges, renumbered locally
    mine = []
    local = np.full((3, max(nb)), -1, np.int32)
    lens = np.zeros(3, np.int32)
    for b in range(3):
        b0, b1 = G2.split_block_range(nb[b], world, rank)
        for i, blk in enumerate(tables[b, b0:b1]):
            local[b, i] = len(mine)
            mine.append(int(blk))
        lens[b] = max(0, min(int(ctx[b]), b1 * bs) - b0 * bs)
    pool = G2.PagedBlockPool(max(1, len(mine)), 1, nKv, d, bs, dtype="bf16", device=rank)
    idx = np.array(mine, np.int64)
    kv = pool.key_view()
    kv.view(torch.int16).copy_(torch.from_numpy(Kb[idx].view(np.int16)))
    pool.value_view().view(torch.int16).copy_(torch.from_numpy(Vb[idx].view(np.int16)))
    uid = q_uid.get() if rank else None
    if rank == 0:
        uid = G2.Comm.unique_id()
        for _ in range(world - 1):
            q_uid.put(uid)
    comm = G2.Comm(uid, world, rank, rank, timeout_ms=60_000)
    pool.upload_step(local, lens)
    g = O2.geom(total, 1, nKv, d, d, bs, O2.BF16)
    err = 0.0
    # several decodes: the peer mailboxes alternate parity every call
    for step in range(4):
        qs = q if step == 0 else np.random.default_rng(100 + step).standard_normal(q.shape).astype(np.float32)
        out = torch.zeros((3, nH, d), device=dev)
        pool.paged_decode_splitkv_dist(comm, 0, torch.from_numpy(qs).to(dev), out, nH, 1 / math.sqrt(d))
        torch.cuda.synchronize(dev)
        ref = O2.decode_batch(np.ascontiguousarray(Kb), np.ascontiguousarray(Vb), g, 0, tables, ctx, qs, nH,
                              1 / math.sqrt(d))
        err = max(err, float(np.abs(out.cpu().numpy() - ref).max()))
    pool.sync()
    ret[rank] = err
    ret[f"kind{rank}"] = comm.exchange_kind
    comm.close()
    pool.close()


def test_two_gpu_nccl_split_kv(cuda):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    ret, q_uid = mgr.dict(), mgr.Queue()
    procs = [ctx.Process(target=_dist_worker, args=(r, 2, q_uid, ret)) for r in range(2)]
    [p.start() for p in procs]
    [p.join(timeout=300) for p in procs]
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert ret[0] < TOL["bf16"] and ret[1] < TOL["bf16"], dict(ret)
    # NVLink peers map each other's mailboxes: the exchange must not fall back to NCCL
    assert ret["kind0"] == 2 and ret["kind1"] == 2, dict(ret)


def test_one_rank_comm_runs_the_mailbox_exchange(cuda):
    """A one-rank communicator takes the peer-mailbox path on one GPU (the decode writes into
    its own mailbox slot, the merge kernel publishes, waits and merges): over calls of both
    parities, with and without sinks, it equals the oracle's decode; a sequence with no tokens
    (the lse fill path) merges to zeros."""
    import torch

    rng = np.random.default_rng(47)
    bs, d, nH, nKv = 16, 128, 64, 8
    ctx = [3000, 17, 0, 640]
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = G.PagedBlockPool(need + 2, 1, nKv, d, bs, dtype="bf16")
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, ctx, bs, need + 2)
    comm = G.Comm(G.Comm.unique_id(), 1, 0, cuda.index or 0, timeout_ms=60_000)
    pool.upload_step(tables, np.array(ctx, np.int32))
    live = [b for b, c in enumerate(ctx) if c > 0]
    for step in range(4):
        q = rng.standard_normal((len(ctx), nH, d)).astype(np.float32)
        sk = 0.3 if step == 3 else None
        sinks = None if sk is None else torch.full((nH,), sk, device=cuda)
        out = torch.full((len(ctx), nH, d), 7.0, device=cuda)
        pool.paged_decode_splitkv_dist(comm, 0, torch.from_numpy(q).to(cuda), out, nH, 1 / math.sqrt(d), sinks=sinks)
        pool.sync()
        got = out.cpu().numpy()
        ref = O.decode_batch(K, V, geom_of(pool), 0, tables, np.array(ctx, np.int32), q, nH, 1 / math.sqrt(d),
                             sink_logit=sk)
        np.testing.assert_allclose(got[live], ref[live], atol=TOL["bf16"], rtol=0)
        assert np.array_equal(got[2], np.zeros((nH, d), np.float32))
    assert comm.exchange_kind == 2
    comm.close()
    pool.close()
