"""gkv_paged_decode_noalloc: the decode entry point for callers that cannot allocate device
memory on the decode path (hosts whose memory belongs to another allocator or to a fixed
budget, serving loops that cannot take a call that may synchronize the device).

It is checked through the C ABI against the allocating path (gkv_upload_step +
gkv_paged_decode) on the same inputs, on two calls in a row with different batches, so
that contents the first call leaves in the shared static scratch cannot leak into the
second.  This file sorts last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, gpu_decode, random_arena, random_tables

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


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_noalloc_matches_allocating_decode_on_two_calls(cuda, dtype):
    import torch

    rng = np.random.default_rng(31)
    pool = G.PagedBlockPool(3000, 1, 8, 128, 16, dtype=dtype)
    random_arena(pool, rng)
    # call 1: many long sequences (most segments split over several warps -> partials)
    ctx1 = [2049] * 16 + [5, 1, 700]
    t1 = random_tables(rng, ctx1, 16, 3000)
    q1 = rng.standard_normal((len(ctx1), 32, 128)).astype(np.float32)
    # call 2: a different, smaller batch and head count
    ctx2 = [300, 17, 1200]
    t2 = random_tables(rng, ctx2, 16, 3000)
    q2 = rng.standard_normal((len(ctx2), 64, 128)).astype(np.float32)

    ref1 = gpu_decode(pool, 0, t1, ctx1, q1, 32, 0.088)
    ref2 = gpu_decode(pool, 0, t2, ctx2, q2, 64, 0.088)
    b1 = _buffers(pool, ctx1, q1, 32, cuda)
    b2 = _buffers(pool, ctx2, q2, 64, cuda)
    torch.cuda.synchronize(cuda)
    got1 = _noalloc(pool, t1, ctx1, *b1, 32, 0.088, cuda)
    free_after_first = torch.cuda.mem_get_info(cuda)[0]
    got2 = _noalloc(pool, t2, ctx2, *b2, 64, 0.088, cuda)
    np.testing.assert_allclose(got1, ref1, atol=TOL[dtype], rtol=0)
    np.testing.assert_allclose(got2, ref2, atol=TOL[dtype], rtol=0)
    # and once more with the first batch, after the second call overwrote the scratch
    got1b = _noalloc(pool, t1, ctx1, *b1, 32, 0.088, cuda)
    np.testing.assert_allclose(got1b, ref1, atol=TOL[dtype], rtol=0)
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
