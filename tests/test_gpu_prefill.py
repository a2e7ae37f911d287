"""Chunked causal prefill (gkv_paged_prefill) against the oracle's restatement of
PagedTransformerRunner.ForwardPrefillSubBatch (one ComputeAttention per chunk token,
PagedTransformerRunner.cs:424-471).  bf16 and fp16 pools with d = dv = 128 take the tcgen05
kernel; every other pool takes the decode kernel with one segment per query."""
import math

import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, geom_of, random_arena, random_tables
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _bf16_round(x):
    return O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.ascontiguousarray(x, np.float32)))


def _round(x, dtype):
    """x as the device sees it after rounding to `dtype` (fp16 saturating at +-65504)."""
    if dtype == "bf16":
        return _bf16_round(x)
    if dtype == "f16":
        return O.f16_bits_to_f32(O.f32_to_f16_bits(np.clip(x, -65504.0, 65504.0)))
    return np.ascontiguousarray(x, np.float32)


def _run(pool, rng, prefixes, q_lens, n_heads, layer=0, q_dtype="bf16", starts=None, toks=None,
         out_init=0.0, K=None, V=None):
    """Builds tables for token counts prefix + q_len (or `toks`), runs the GPU prefill and
    returns (gpu out, per-sequence oracle outs, q as the oracle saw it)."""
    import torch

    bs = pool.block_size
    B = len(q_lens)
    starts = list(prefixes) if starts is None else list(starts)
    toks = [p + l for p, l in zip(prefixes, q_lens)] if toks is None else list(toks)
    cap = [max(t, s + l) for t, s, l in zip(toks, starts, q_lens)]
    tables = random_tables(rng, cap, bs, pool.total_blocks)
    if K is None:
        K, V = random_arena(pool, rng)
    total_q = int(sum(q_lens))
    d = pool.head_dim
    q = _round(rng.standard_normal((total_q, n_heads, d)).astype(np.float32), q_dtype)
    dev = f"cuda:{pool.device}"
    qt = torch.from_numpy(q).to(dev)
    if q_dtype != "f32":
        qt = qt.to(torch.bfloat16 if q_dtype == "bf16" else torch.float16)  # exact: q is rounded already
    if pool.dtype in ("bf16", "f16") and d == 128:
        q = _round(q, pool.dtype)  # the tensor-core path computes with q in the arena's type
    out = torch.full((total_q, n_heads, pool.value_head_dim), out_init, dtype=torch.float32, device=dev)
    pool.upload_step(tables, np.asarray(toks, np.int32))
    scale = 1 / math.sqrt(d)
    pool.paged_prefill(layer, qt, out, np.asarray(starts, np.int32), np.asarray(q_lens, np.int32), n_heads, scale)
    pool.sync()
    got = out.cpu().numpy()
    refs, off = [], 0
    g = geom_of(pool)
    for b in range(B):
        n = q_lens[b]
        if n:
            ref = O.prefill_chunk(K, V, g, layer, tables[b], toks[b], starts[b], q[off:off + n], n_heads, scale)
            if toks[b] == 0:
                ref[...] = out_init
        else:
            ref = np.zeros((0, n_heads, pool.value_head_dim), np.float32)
        refs.append(ref)
        off += n
    return got, refs, q


def _assert_close(got, refs, tol):
    ref = np.concatenate(refs, axis=0) if refs else got
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, atol=tol, rtol=0)


@pytest.mark.parametrize("prefixes,q_lens,nH,nKv", [
    ([0], [1], 28, 4),                       # one query, one key
    ([0, 5], [128, 129], 28, 4),             # exact tile / one past
    ([37, 200, 0], [300, 17, 64], 28, 4),    # ragged prefixes and chunks
    ([130], [257], 8, 8),                    # MHA
    ([64, 1000], [191, 70], 32, 2),          # wide group
])
def test_tc_prefill_parity(cuda, prefixes, q_lens, nH, nKv):
    rng = np.random.default_rng(sum(prefixes) * 7 + sum(q_lens) + nH)
    need = sum((p + l + 15) // 16 for p, l in zip(prefixes, q_lens)) + 4
    pool = G.PagedBlockPool(need, 1, nKv, 128, 16, dtype="bf16")
    got, refs, _ = _run(pool, rng, prefixes, q_lens, nH)
    _assert_close(got, refs, TOL["bf16"])
    pool.close()


@pytest.mark.parametrize("q_dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("prefixes,q_lens,nH,nKv", [([0, 5], [128, 129], 28, 4), ([37, 200, 0], [300, 17, 64], 28, 4)])
def test_tc_prefill_f16_arena(cuda, prefixes, q_lens, nH, nKv, q_dtype):
    """fp16 storage (the reference GPU pools' precision): both MMA operands fp16, q converted to
    fp16 from whichever type it comes in."""
    rng = np.random.default_rng(sum(prefixes) + sum(q_lens) + len(q_dtype))
    need = sum((p + l + 15) // 16 for p, l in zip(prefixes, q_lens)) + 4
    pool = G.PagedBlockPool(need, 1, nKv, 128, 16, dtype="f16")
    got, refs, _ = _run(pool, rng, prefixes, q_lens, nH, q_dtype=q_dtype)
    _assert_close(got, refs, TOL["f16"])
    pool.close()


def test_tc_prefill_f32_q_is_rounded_to_bf16(cuda):
    rng = np.random.default_rng(3)
    pool = G.PagedBlockPool(40, 1, 4, 128, 16, dtype="bf16")
    got, refs, _ = _run(pool, rng, [100, 3], [150, 40], 28, q_dtype="f32")
    _assert_close(got, refs, TOL["bf16"])
    pool.close()


def test_tc_prefill_layer_and_block_size_8(cuda):
    rng = np.random.default_rng(4)
    pool = G.PagedBlockPool(120, 3, 2, 128, 8, dtype="bf16")
    got, refs, _ = _run(pool, rng, [77, 0], [200, 33], 14, layer=2)
    _assert_close(got, refs, TOL["bf16"])
    pool.close()


def test_tc_prefill_queries_before_the_end_and_past_token_count(cuda):
    """Queries at positions below token_count (later keys exist but are causally masked) and
    past it (every stored key visible)."""
    rng = np.random.default_rng(5)
    pool = G.PagedBlockPool(80, 1, 4, 128, 16, dtype="bf16")
    got, refs, _ = _run(pool, rng, [0, 0], [100, 90], 28, starts=[50, 300], toks=[400, 250])
    _assert_close(got, refs, TOL["bf16"])
    pool.close()


def test_tc_prefill_ignores_non_finite_unwritten_slots(cuda):
    """Slots past token_count in the last page hold NaN: masked keys and zeroed value rows keep
    them out of the result."""
    import torch

    rng = np.random.default_rng(6)
    pool = G.PagedBlockPool(30, 1, 4, 128, 16, dtype="bf16")
    K, V = random_arena(pool, rng)
    K[...] = 0x7FC0  # NaN everywhere; the test writes real values into the used slots
    V[...] = 0x7FC0
    toks = [77, 130]
    tables = random_tables(rng, toks, 16, 30)
    kf = O.f32_to_bf16_bits(rng.standard_normal(K.shape).astype(np.float32))
    vf = O.f32_to_bf16_bits(rng.standard_normal(V.shape).astype(np.float32))
    for b, t in enumerate(toks):
        for pos in range(t):
            blk, s = tables[b, pos // 16], pos % 16
            K[blk, :, :, s] = kf[blk, :, :, s]
            V[blk, :, :, s] = vf[blk, :, :, s]
    for view, arr in ((pool.key_view(), K), (pool.value_view(), V)):
        view.view(torch.int16).copy_(torch.from_numpy(arr.view(np.int16)))
    rng2 = np.random.default_rng(7)
    q = _bf16_round(rng2.standard_normal((2 * 60, 28, 128)).astype(np.float32))
    out = torch.zeros((120, 28, 128), device=cuda)
    pool.upload_step(tables, np.asarray(toks, np.int32))
    starts = np.array([17, 70], np.int32)
    pool.paged_prefill(0, torch.from_numpy(q).to(cuda).to(torch.bfloat16), out, starts,
                       np.array([60, 60], np.int32), 28, 1 / math.sqrt(128))
    pool.sync()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    g = geom_of(pool)
    for b in range(2):
        ref = O.prefill_chunk(K, V, g, 0, tables[b], toks[b], int(starts[b]), q[b * 60:(b + 1) * 60], 28,
                              1 / math.sqrt(128))
        np.testing.assert_allclose(got[b * 60:(b + 1) * 60], ref, atol=TOL["bf16"], rtol=0)
    pool.close()


@pytest.mark.parametrize("dtype,d,nH,nKv,q_dtype", [
    ("f32", 128, 28, 4, "f32"),
    ("f32", 64, 8, 2, "f32"),
    ("bf16", 64, 16, 4, "bf16"),
    ("bf16", 256, 8, 1, "f32"),
    ("f16", 64, 16, 4, "f16"),
    ("f16", 32, 8, 8, "f32"),
])
def test_decode_kernel_prefill_parity(cuda, dtype, d, nH, nKv, q_dtype):
    rng = np.random.default_rng(d + nH)
    prefixes, q_lens = [0, 45, 300], [70, 1, 33]
    need = sum((p + l + 15) // 16 for p, l in zip(prefixes, q_lens)) + 2
    pool = G.PagedBlockPool(need, 1, nKv, d, 16, dtype=dtype)
    got, refs, _ = _run(pool, rng, prefixes, q_lens, nH, q_dtype=q_dtype)
    _assert_close(got, refs, TOL[dtype])
    pool.close()


@pytest.mark.parametrize("dtype", ["bf16", "f32", "f16"])
def test_empty_sequences_leave_rows_untouched(cuda, dtype):
    rng = np.random.default_rng(8)
    pool = G.PagedBlockPool(20, 1, 4, 128, 16, dtype=dtype)
    got, refs, _ = _run(pool, rng, [0, 10, 0], [5, 0, 20], 28, q_dtype=dtype, toks=[0, 10, 20], out_init=7.5)
    assert (got[:5] == 7.5).all()
    _assert_close(got, refs, TOL[dtype])
    pool.close()


def test_prefill_argument_errors(cuda):
    import torch

    pool = G.PagedBlockPool(8, 1, 4, 128, 16, dtype="bf16")
    q = torch.zeros((4, 28, 128), device=cuda, dtype=torch.bfloat16)
    out = torch.zeros((4, 28, 128), device=cuda)
    with pytest.raises(G.InvalidOperationError):
        pool.paged_prefill(0, q, out, [0], [4], 28, 0.1)  # nothing uploaded
    pool.upload_step(np.array([[0, 1]], np.int32), np.array([20], np.int32))
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.paged_prefill(0, q, out, [30], [4], 28, 0.1)  # position 33 >= 2 blocks * 16
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.paged_prefill(0, q, out, [-1], [4], 28, 0.1)
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.paged_prefill(1, q, out, [0], [4], 28, 0.1)  # layer
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.paged_prefill(0, q, out, [0], [4], 27, 0.1)  # heads not a multiple of heads_kv
    pool.paged_prefill(0, q, out, [16], [4], 28, 0.1)
    pool.sync()
    assert pool.last_launch_count == 1
    pool.close()


def test_cfg4_shape_sampled_rows(cuda):
    """The cfg4 geometry (28/4 heads, d 128, bf16, prefix up to 4096, 2048-token chunks),
    two sequences, with the oracle run on the last 48 queries of each chunk (the heaviest
    rows) and on the first 16."""
    import torch

    rng = np.random.default_rng(9)
    prefixes, L = [4000, 1537], 2048
    toks = [p + L for p in prefixes]
    need = sum((t + 15) // 16 for t in toks) + 1
    pool = G.PagedBlockPool(need, 1, 4, 128, 16, dtype="bf16")
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, toks, 16, need)
    q = _bf16_round(rng.standard_normal((2 * L, 28, 128)).astype(np.float32))
    out = torch.zeros((2 * L, 28, 128), device=cuda)
    pool.upload_step(tables, np.asarray(toks, np.int32))
    scale = 1 / math.sqrt(128)
    pool.paged_prefill(0, torch.from_numpy(q).to(cuda).to(torch.bfloat16), out, np.asarray(prefixes, np.int32),
                       np.array([L, L], np.int32), 28, scale)
    pool.sync()
    got = out.cpu().numpy()
    g = geom_of(pool)
    for b in range(2):
        for t0, n in ((0, 16), (L - 48, 48)):
            rows = slice(b * L + t0, b * L + t0 + n)
            ref = O.prefill_chunk(K, V, g, 0, tables[b], toks[b], prefixes[b] + t0, q[rows], 28, scale)
            np.testing.assert_allclose(got[rows], ref, atol=TOL["bf16"], rtol=0)
    pool.close()
