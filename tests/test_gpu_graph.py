"""The static step layout (gkv_step_set_static): the per-layer kv_append + paged_decode launches
of a decode iteration captured ONCE in a CUDA graph and replayed every step after upload_step
(a CUDA-graph form of the decode iteration of CudaPagedTransformerRunner.ForwardBatch,
CudaPagedTransformerRunner.cs:307-364).  Every step changes the batch, the tables, the
context lengths and the appended slots; each replay must equal the oracle's Store + decode."""
import math

import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, arena_to_host, geom_of, random_arena
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _steps(rng, n_steps, max_batch, bs, total_blocks, max_ctx):
    """Per step: tables, ctx (including the appended token), slots of the appended tokens
    (one per sequence: its last position), distinct blocks per sequence."""
    out = []
    for _ in range(n_steps):
        batch = int(rng.integers(1, max_batch + 1))
        ctx = rng.integers(1, max_ctx + 1, size=batch).astype(np.int32)
        ctx[0] = max_ctx  # one long sequence: split over workers, merged by the merge kernel
        nb = (ctx + bs - 1) // bs
        perm = rng.permutation(total_blocks).astype(np.int32)
        mb = int(nb.max())
        tables = np.full((batch, mb), -1, np.int32)
        at = 0
        for b in range(batch):
            tables[b, :nb[b]] = perm[at:at + nb[b]]
            at += nb[b]
        pos = ctx - 1
        slots = (tables[np.arange(batch), pos // bs].astype(np.int64) * bs + pos % bs)
        out.append((tables, ctx, slots))
    return out


@pytest.mark.parametrize("dtype,nH,nKv", [("f32", 28, 4), ("bf16", 28, 4), ("f16", 16, 8), ("fp8", 28, 4)])
def test_graph_replayed_decode_iteration_matches_oracle(cuda, dtype, nH, nKv):
    import torch

    rng = np.random.default_rng(71)
    layers, bs, d = 3, 16, 128
    max_batch, max_ctx = 6, 2500
    max_blocks = (max_ctx + bs - 1) // bs
    nb_total = max_batch * max_blocks + 8
    pool = G.PagedBlockPool(nb_total, layers, nKv, d, bs, dtype=dtype)
    K, V = random_arena(pool, rng)
    pool.reserve_step(max_batch, max_blocks, max_batch, nH)
    pool.set_static_step(True)
    s = torch.cuda.Stream(cuda)
    # device inputs at fixed addresses, rewritten before every replay
    q = torch.zeros((layers, max_batch, nH, d), device=cuda)
    kn = torch.zeros((layers, max_batch, nKv, d), device=cuda)
    vn = torch.zeros((layers, max_batch, nKv, d), device=cuda)
    out = torch.zeros((layers, max_batch, nH, d), device=cuda)
    steps = _steps(rng, 5, max_batch, bs, nb_total, max_ctx)

    def iteration():
        for l in range(layers):
            pool.kv_append(l, kn[l], vn[l], stream=s)
            pool.paged_decode(l, q[l], out[l], nH, 1 / math.sqrt(d), stream=s)

    # warm-up (first-use kernel attributes) and capture, both after an upload of step 0
    tables, ctx, slots = steps[0]
    with torch.cuda.stream(s):
        pool.upload_step(tables, ctx, slots, stream=s)
        iteration()
    s.synchronize()
    K, V = arena_to_host(pool)  # the warm-up appended step 0's (zero) rows: start from there
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        iteration()
    g = geom_of(pool)
    for tables, ctx, slots in steps:
        batch = len(ctx)
        qs = rng.standard_normal((layers, batch, nH, d)).astype(np.float32)
        ks = rng.standard_normal((layers, batch, nKv, d)).astype(np.float32)
        vs = rng.standard_normal((layers, batch, nKv, d)).astype(np.float32)
        with torch.cuda.stream(s):
            q[:, :batch].copy_(torch.from_numpy(qs))
            kn[:, :batch].copy_(torch.from_numpy(ks))
            vn[:, :batch].copy_(torch.from_numpy(vs))
            out.fill_(7.0)
            pool.upload_step(tables, ctx, slots, stream=s)
            graph.replay()
        s.synchronize()
        pool.sync()
        got = out.cpu().numpy()
        for l in range(layers):
            assert O.store_many(K, V, g, l, slots, ks[l], vs[l]) == 0
            ref = O.decode_batch(K, V, g, l, tables, ctx, qs[l], nH, 1 / math.sqrt(d))
            np.testing.assert_allclose(got[l, :batch], ref, atol=TOL[dtype], rtol=0)
            assert (got[l, batch:] == 7.0).all()  # rows past the step's batch are left alone
        Kg, Vg = arena_to_host(pool)
        assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    pool.set_static_step(False)
    pool.close()


def test_static_layout_refusals(cuda):
    """Uploads beyond the reservation, another head count, the prefill, a second reservation
    and pending copy-on-write copies are refused while the layout is static."""
    import torch

    pool = G.PagedBlockPool(64, 1, 2, 64, 16)
    with pytest.raises(G.InvalidOperationError):
        pool.set_static_step(True)  # nothing reserved yet
    pool.reserve_step(2, 4, 2, 8)
    pool.set_static_step(True)
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.upload_step(np.zeros((3, 1), np.int32), np.ones(3, np.int32))
    with pytest.raises(G.InvalidOperationError):
        pool.reserve_step(4, 4, 4, 8)
    pool.upload_step(np.array([[0], [1]], np.int32), np.array([5, 9], np.int32))
    q = torch.zeros((2, 4, 64), device=cuda)
    out = torch.zeros((2, 4, 64), device=cuda)
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.paged_decode(0, q, out, 4, 0.125)
    with pytest.raises(G.InvalidOperationError):
        pool.paged_prefill(0, torch.zeros((1, 8, 64), device=cuda), torch.zeros((1, 8, 64), device=cuda),
                           np.array([0, 0], np.int32), np.array([1, 0], np.int32), 8, 0.125)
    ok, blk = pool.try_allocate_block()
    pool.retain_block(blk)  # shared: the fork allocates a new block and queues a copy
    ok2, fork = pool.try_fork_block(blk, 4)
    assert ok and ok2 and fork != blk and pool.pending_copies == 1
    with pytest.raises(G.InvalidOperationError):
        pool.paged_decode(0, torch.zeros((2, 8, 64), device=cuda), torch.zeros((2, 8, 64), device=cuda), 8, 0.125)
    pool.flush_copies()
    pool.paged_decode(0, torch.zeros((2, 8, 64), device=cuda), torch.zeros((2, 8, 64), device=cuda), 8, 0.125)
    pool.sync()
    pool.set_static_step(False)
    pool.close()
