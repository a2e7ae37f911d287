"""gkv_paged_decode_noalloc: the decode entry point for callers that cannot allocate device
memory on the decode path (hosts whose memory belongs to another allocator or to a fixed
budget, serving loops that cannot take a call that may synchronize the device).

It is checked through the C ABI against the CPU oracle (the restatement of the reference's
PagedAttentionKernel.ComputeAttention) and against the allocating path (gkv_upload_step +
gkv_paged_decode) on the same inputs, on two calls in a row with different batches, so that
contents the first call leaves in the shared static scratch cannot leak into the second; its
error word is read back through gkv_paged_decode_noalloc_status.  This file sorts last so that a
run stopping at the first failure has already run every other test; it also passes alone in a
fresh process.
"""
import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, geom_of, gpu_decode, random_arena, random_tables
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _buffers(pool, ctx, q_np, n_heads, cuda):
    import torch

    q = torch.from_numpy(np.ascontiguousarray(q_np, np.float32)).to(cuda)
    out = torch.zeros((len(ctx), n_heads, pool.value_head_dim), dtype=torch.float32, device=cuda)
    return q, out


def _noalloc(pool, tables, ctx, q, out, n_heads, scale, cuda):
    import torch

    out.zero_()
    G.paged_decode_noalloc(pool, 0, tables, np.asarray(ctx, np.int32), q, out, n_heads, scale)
    torch.cuda.synchronize(cuda)
    return out.cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_noalloc_matches_allocating_decode_on_two_calls(cuda, dtype):
    import torch

    rng = np.random.default_rng(31)
    pool = G.PagedBlockPool(3000, 1, 8, 128, 16, dtype=dtype)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    # call 1: many long sequences (most segments split over several warps -> partials)
    ctx1 = [2049] * 16 + [5, 1, 700]
    t1 = random_tables(rng, ctx1, 16, 3000)
    q1 = rng.standard_normal((len(ctx1), 32, 128)).astype(np.float32)
    # call 2: a different, smaller batch and head count
    ctx2 = [300, 17, 1200]
    t2 = random_tables(rng, ctx2, 16, 3000)
    q2 = rng.standard_normal((len(ctx2), 64, 128)).astype(np.float32)

    ora1 = O.decode_batch(K, V, g, 0, t1, np.asarray(ctx1, np.int32), q1, 32, 0.088)
    ora2 = O.decode_batch(K, V, g, 0, t2, np.asarray(ctx2, np.int32), q2, 64, 0.088)
    ref1 = gpu_decode(pool, 0, t1, ctx1, q1, 32, 0.088)
    ref2 = gpu_decode(pool, 0, t2, ctx2, q2, 64, 0.088)
    b1 = _buffers(pool, ctx1, q1, 32, cuda)
    b2 = _buffers(pool, ctx2, q2, 64, cuda)
    torch.cuda.synchronize(cuda)
    got1 = _noalloc(pool, t1, ctx1, *b1, 32, 0.088, cuda)
    free_after_first = torch.cuda.mem_get_info(cuda)[0]
    got2 = _noalloc(pool, t2, ctx2, *b2, 64, 0.088, cuda)
    G.paged_decode_noalloc_status(pool.device)  # no error bits from either call
    for got, ora, ref in ((got1, ora1, ref1), (got2, ora2, ref2)):
        np.testing.assert_allclose(got, ora, atol=TOL[dtype], rtol=0)  # the reference's arithmetic
        np.testing.assert_allclose(got, ref, atol=TOL[dtype], rtol=0)  # the allocating path
    # and once more with the first batch, after the second call overwrote the scratch
    got1b = _noalloc(pool, t1, ctx1, *b1, 32, 0.088, cuda)
    np.testing.assert_allclose(got1b, ora1, atol=TOL[dtype], rtol=0)
    np.testing.assert_allclose(got1b, ref1, atol=TOL[dtype], rtol=0)
    G.paged_decode_noalloc_status(pool.device)
    # the calls after the first one take no device memory
    assert torch.cuda.mem_get_info(cuda)[0] == free_after_first
    pool.close()


def test_noalloc_rejects_sizes_beyond_its_static_scratch(cuda):
    import torch

    pool = G.PagedBlockPool(64, 1, 1, 128, 16)
    ctx = [16] * 4
    q = torch.zeros((4, 1, 128), device=cuda)
    out = torch.zeros((4, 1, 128), device=cuda)
    huge = np.zeros((4, 300_000), np.int32)  # 4.8 MB of block table > the 4 MiB metadata part
    with pytest.raises(G.ArgumentOutOfRangeError, match="static scratch"):
        G.paged_decode_noalloc(pool, 0, huge, np.array(ctx, np.int32), q, out, 1, 1.0)
    with pytest.raises(G.ArgumentOutOfRangeError):
        G.paged_decode_noalloc(pool, 0, np.full((4, 1), 99, np.int32), np.array(ctx, np.int32), q, out, 1, 1.0)
    pool.close()


def test_noalloc_sees_a_fork_queued_on_the_pool(cuda):
    """A copy-on-write fork only queues its block copy on the pool; the Python wrapper issues it
    before the allocation-free decode, which reads the raw arena (TryForkBlock,
    PagedBlockPool.cs:332-342, then ComputeAttention over the forked table)."""
    import torch

    rng = np.random.default_rng(5)
    pool = G.PagedBlockPool(64, 1, 2, 128, 16)
    K, V = random_arena(pool, rng)
    src = 3
    ok, dst = pool.try_fork_block(src, 11)
    assert ok and pool.pending_copies == 1
    # the fork's destination holds the first 11 slots of src once the copy has run
    O.copy_block_data(K, V, geom_of(pool), src, dst, 11)
    tables = np.array([[dst]], np.int32)
    ctx = np.array([11], np.int32)
    q_np = rng.standard_normal((1, 4, 128)).astype(np.float32)
    q = torch.from_numpy(q_np).to(cuda)
    out = torch.zeros((1, 4, 128), device=cuda)
    G.paged_decode_noalloc(pool, 0, tables, ctx, q, out, 4, 0.088)
    G.paged_decode_noalloc_status(pool.device)
    assert pool.pending_copies == 0
    ora = O.decode_batch(K, V, geom_of(pool), 0, tables, ctx, q_np, 4, 0.088)
    np.testing.assert_allclose(out.cpu().numpy(), ora, atol=TOL["f32"], rtol=0)
    pool.close()


def test_noalloc_refuses_stream_capture(cuda):
    """Its table upload cannot be replayed by a CUDA graph, so a capturing stream is refused
    (GKV_ESTATE) before anything is enqueued; the static step layout is the capturable path."""
    import torch

    pool = G.PagedBlockPool(8, 1, 2, 128, 16, dtype="bf16")
    q = torch.zeros((1, 8, 128), device=cuda)
    out = torch.zeros((1, 8, 128), device=cuda)
    tables, ctx = np.array([[0]], np.int32), np.array([5], np.int32)
    G.paged_decode_noalloc(pool, 0, tables, ctx, q, out, 8, 0.125)  # resolves the scratch address
    torch.cuda.synchronize(cuda)
    s = torch.cuda.Stream(cuda)
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(G.InvalidOperationError):
        with torch.cuda.graph(graph, stream=s):
            G.paged_decode_noalloc(pool, 0, tables, ctx, q, out, 8, 0.125, stream=s)
    torch.cuda.synchronize(cuda)
    pool.close()
