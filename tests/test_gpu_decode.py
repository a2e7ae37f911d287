"""Parity of the sm_100a split-KV decode with the CPU oracle, through the C ABI.

Bars: max-abs 1e-4 for fp32 KV and 2e-2 for bf16 and fp16 KV storage (the oracle computes from
the same rounded values in fp32).
"""
import glob
import json
import math
import os
import zlib

import numpy as np
import pytest

import glacier_kv as G
from conftest import ROOT
from gpu_helpers import (TOL, arena_to_host, compact, geom_of, gpu_decode, host_to_arena, random_arena,
                         random_tables, scale_of)
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(ROOT, "tests", "golden")


def test_kat_closed_form_through_compute_attention(cuda):
    """PagedAttentionTests.cs:112-179 through the reference-shaped single-sequence call."""
    import torch

    kat = json.load(open(os.path.join(GOLD, "kat_compute_attention.json")))
    d, T, nH, nKv = kat["head_dim"], kat["tokens"], kat["n_heads"], kat["n_heads_kv"]
    pool = G.PagedBlockPool(8, 1, nKv, d, 16)
    table = G.BlockTable(pool)
    for t in range(T):
        ok, blk, off = table.append_token()
        assert ok
        k = torch.full((nKv * d,), kat["k_value_per_token"][t], dtype=torch.float32, device=cuda)
        v = torch.cat([torch.full((d,), c * (t + 1), dtype=torch.float32, device=cuda)
                       for c in kat["v_scale_per_kv_head"]])
        pool.store(blk, 0, off, k, v)
    q = torch.ones(nH * d, dtype=torch.float32, device=cuda)
    out = torch.zeros(nH * d, dtype=torch.float32, device=cuda)
    G.PagedAttentionKernel.compute_attention(0, 0, T - 1, q, out, table, pool, nH, nKv, d, d, kat["attn_scale"], T)
    pool.sync()
    o = out.view(nH, d).cpu().numpy()
    for h, e in enumerate(kat["expected_per_head"]):
        assert o[h].min() > 0
        np.testing.assert_allclose(o[h], e, atol=TOL["f32"] * 10, rtol=1e-5)
        np.testing.assert_allclose(o[h], o[h][0], atol=1e-5, rtol=0)  # precision 4 of the reference
    table.release_all()
    assert pool.free_blocks_count == 8


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "decode_small_*.npz"))))
def test_committed_fixtures(cuda, path):
    z = np.load(path)
    total, layers, nKv, d, dv, bs, dt = [int(x) for x in z["geom"]]
    dtype = "bf16" if dt == O.BF16 else "f32"
    pool = G.PagedBlockPool(total, layers, nKv, d, bs, dv, dtype=dtype)
    host_to_arena(pool, z["K"], z["V"])
    out = gpu_decode(pool, 0, z["tables"], z["ctx"], z["q"], int(z["n_heads"]), float(z["scale"]))
    np.testing.assert_allclose(out, z["out"], atol=TOL[dtype], rtol=0)


CASES = [
    # nH, nKv, d, dv, bs, dtype, ctx
    (28, 4, 128, 128, 16, "f32", [1, 7, 8, 9, 15, 16, 17, 31, 33, 127, 128, 129, 1000]),
    (32, 8, 128, 128, 16, "f32", [2049, 2049, 5, 2049]),
    (64, 8, 128, 128, 16, "bf16", [5000, 3, 640]),
    (28, 4, 128, 128, 16, "bf16", [1500, 16, 2, 333]),
    (2, 1, 32, 64, 8, "f32", [20, 7, 1]),
    (16, 1, 64, 64, 16, "bf16", [300, 45]),        # group 16: two head groups
    (12, 1, 128, 128, 16, "f32", [77, 400]),        # group 12: partial second head group
    (1, 1, 256, 256, 16, "f32", [65, 1]),
    (3, 3, 32, 32, 4, "f32", [13, 4, 1]),           # MHA, block size 4
    (8, 2, 128, 64, 12, "f32", [50, 12, 13]),       # block size 12: chunks of 8 + 4
    (4, 4, 64, 64, 16, "f32", [20000]),             # one long sequence split over many workers
    (16, 2, 128, 128, 8, "bf16", [37, 8, 1, 100]),  # tensor-core kernel, block size 8
    (8, 1, 128, 128, 24, "bf16", [50, 24, 25, 3]),  # tensor-core kernel, block size 24
    (56, 8, 128, 128, 16, "bf16", [9000, 17]),      # group 7, long sequence: fused merge
    # fp32 KV, wide groups, other block sizes
    (16, 2, 128, 128, 8, "f32", [37, 8, 1, 100]),   # block size 8
    (8, 1, 128, 128, 24, "f32", [50, 24, 25, 3]),   # block size 24: chunks of 8
    (40, 8, 128, 128, 16, "f32", [3000, 7, 129]),   # group 5: three idle heads of the pass
    (12, 4, 128, 128, 16, "f32", [2049, 300, 5, 17]),  # group 3: the padding slot compiled out
    # long and short splits in one batch: the merge gives the long ones a CTA, the others a warp
    (28, 4, 128, 128, 16, "f32", [12000, 700, 300, 90, 5]),
    (28, 4, 128, 128, 16, "bf16", [20000, 900, 64, 33]),
    # fp16 storage (the reference GPU pools' precision): tensor-core and CUDA-core kernels
    (28, 4, 128, 128, 16, "f16", [1500, 16, 2, 333, 4097]),
    (64, 8, 128, 128, 16, "f16", [5000, 3, 640]),
    (12, 1, 128, 128, 8, "f16", [77, 400]),         # tensor-core kernel, two head groups
    (32, 8, 128, 128, 16, "f16", [2049, 2049, 5]),  # group 4: CUDA-core kernel
    (2, 1, 32, 64, 8, "f16", [20, 7, 1]),
    (16, 1, 64, 64, 16, "f16", [300, 45]),
]


@pytest.mark.parametrize("case", CASES, ids=[f"h{c[0]}kv{c[1]}d{c[2]}-{c[3]}bs{c[4]}{c[5]}" for c in CASES])
def test_decode_parity(cuda, case):
    nH, nKv, d, dv, bs, dtype, ctx = case
    rng = np.random.default_rng(zlib.crc32(str(case).encode()))
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = G.PagedBlockPool(need + 5, 1, nKv, d, bs, dv, dtype=dtype)
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, ctx, bs, need + 5)
    q = rng.standard_normal((len(ctx), nH, d)).astype(np.float32)
    out = gpu_decode(pool, 0, tables, ctx, q, nH, scale_of(d))
    ref = O.decode_batch(K, V, geom_of(pool), 0, tables, np.array(ctx, np.int32), q, nH, scale_of(d))
    np.testing.assert_allclose(out, ref, atol=TOL[dtype], rtol=0)


@pytest.mark.parametrize("q_mag", [3e4, 1e-5])
def test_f16_tensor_core_decode_takes_any_fp32_q(cuda, q_mag):
    """The tensor-core decode of an fp16 arena splits q into fp16 hi + lo after a power-of-two
    scale, so q components far outside fp16's range (or far below its normal range) still
    give the oracle's result."""
    rng = np.random.default_rng(77)
    ctx = [700, 33]
    pool = G.PagedBlockPool(60, 1, 4, 128, 16, dtype="f16")
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, ctx, 16, 60)
    q = (rng.standard_normal((2, 28, 128)) * q_mag).astype(np.float32)
    scale = 1.0 / (q_mag * 30.0)  # scores of order one
    out = gpu_decode(pool, 0, tables, ctx, q, 28, scale)
    ref = O.decode_batch(K, V, geom_of(pool), 0, tables, np.array(ctx, np.int32), q, 28, scale)
    np.testing.assert_allclose(out, ref, atol=TOL["f16"], rtol=0)
    pool.close()


def test_one_upload_serves_decodes_with_other_head_counts(cuda):
    """A decode whose head count selects another kernel variant (and grid occupancy) than
    the one the upload planned for must reuse the uploaded step as is."""
    import torch

    rng = np.random.default_rng(15)
    pool = G.PagedBlockPool(700, 1, 8, 128, 16, dtype="bf16")
    K, V = random_arena(pool, rng)
    ctx = [3000, 40, 1500, 7]
    tables = random_tables(rng, ctx, 16, 700)
    pool.upload_step(tables, np.array(ctx, np.int32))  # planned without a head count
    for n_heads in (64, 8, 32, 56):  # tensor-core, group 1, group 4, tensor-core group 7
        q = rng.standard_normal((4, n_heads, 128)).astype(np.float32)
        out = torch.zeros((4, n_heads, 128), device=cuda)
        pool.paged_decode(0, torch.from_numpy(q).to(cuda), out, n_heads, 0.09)
        pool.sync()
        ref = O.decode_batch(K, V, geom_of(pool), 0, tables, np.array(ctx, np.int32), q, n_heads, 0.09)
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL["bf16"], rtol=0)
    pool.close()


def test_layer_addressing_multi_layer_pool(cuda):
    rng = np.random.default_rng(11)
    pool = G.PagedBlockPool(40, 3, 2, 64, 16, dtype="f32")
    K, V = random_arena(pool, rng)
    ctx = [100, 33, 250]
    tables = random_tables(rng, ctx, 16, 40)
    q = rng.standard_normal((3, 8, 64)).astype(np.float32)
    for layer in (0, 2):
        out = gpu_decode(pool, layer, tables, ctx, q, 8, 0.11)
        ref = O.decode_batch(K, V, geom_of(pool), layer, tables, np.array(ctx, np.int32), q, 8, 0.11)
        np.testing.assert_allclose(out, ref, atol=TOL["f32"], rtol=0)


def test_empty_sequences_leave_output_untouched(cuda):
    """n == 0 is a silent no-op in the reference (PagedAttentionKernel.cs:42)."""
    rng = np.random.default_rng(12)
    pool = G.PagedBlockPool(20, 1, 2, 128, 16)
    K, V = random_arena(pool, rng)
    ctx = [0, 40, 0]
    tables = random_tables(rng, ctx, 16, 20)
    q = rng.standard_normal((3, 4, 128)).astype(np.float32)
    out = gpu_decode(pool, 0, tables, ctx, q, 4, 0.1, out_init=7.0)
    assert np.all(out[0] == 7.0) and np.all(out[2] == 7.0)
    ref = O.decode_batch(K, V, geom_of(pool), 0, tables, np.array(ctx, np.int32), q, 4, 0.1)
    np.testing.assert_allclose(out[1], ref[1], atol=TOL["f32"], rtol=0)


@pytest.mark.parametrize("n_heads", [8, 28])
def test_sinks_per_head_and_scalar(cuda, n_heads):
    """Group 4 and group 14 (two head groups of eight heads)."""
    import torch

    rng = np.random.default_rng(13)
    pool = G.PagedBlockPool(64, 1, 2, 128, 16)
    K, V = random_arena(pool, rng)
    ctx = [200, 700]
    tables = random_tables(rng, ctx, 16, 64)
    q = rng.standard_normal((2, n_heads, 128)).astype(np.float32)
    sink = 0.75
    out = gpu_decode(pool, 0, tables, ctx, q, n_heads, 0.09, sinks=np.full(n_heads, sink, np.float32))
    ref = O.decode_batch(K, V, geom_of(pool), 0, tables, np.array(ctx, np.int32), q, n_heads, 0.09,
                         sink_logit=sink)
    np.testing.assert_allclose(out, ref, atol=TOL["f32"], rtol=0)
    # the scalar form through compute_attention (float? sinkLogit)
    t = G.BlockTable(pool)
    t.attach_prefix_blocks(tables[1][: (700 + 15) // 16].tolist(), 700)
    qd = torch.from_numpy(q[1].ravel()).to(cuda)
    od = torch.zeros(n_heads * 128, device=cuda)
    G.PagedAttentionKernel.compute_attention(0, 0, 699, qd, od, t, pool, n_heads, 2, 128, 128, 0.09, 4096,
                                             sink_logit=sink)
    pool.sync()
    np.testing.assert_allclose(od.view(n_heads, 128).cpu().numpy(), ref[1], atol=TOL["f32"], rtol=0)


def test_compute_attention_argument_errors(cuda):
    """PhaseCServeRemediationTests.cs:117-174 and PagedAttentionKernel.cs:34-39."""
    import torch

    pool = G.PagedBlockPool(4, 1, 1, 32, 16)
    t = G.BlockTable(pool)
    assert t.append_token()[0]
    q = torch.zeros(32, device=cuda)
    out = torch.zeros(32, device=cuda)
    for pos, msl in ((16, 16), (-1, 16), (0, 0)):
        with pytest.raises(G.ArgumentOutOfRangeError):
            G.PagedAttentionKernel.compute_attention(0, 0, pos, q, out, t, pool, 1, 1, 32, 32, 1 / math.sqrt(32), msl)
    with pytest.raises(G.ArgumentOutOfRangeError):  # stage layer outside the pool
        G.PagedAttentionKernel.compute_attention(1, 0, 0, q, out, t, pool, 1, 1, 32, 32, 1.0, 16)
    with pytest.raises(G.ArgumentOutOfRangeError):  # TokenCount > maxSeqLen
        for _ in range(20):
            t.append_token()
        G.PagedAttentionKernel.compute_attention(0, 0, 0, q, out, t, pool, 1, 1, 32, 32, 1.0, 16)


def test_upload_rejects_bad_tables_and_slots(cuda):
    pool = G.PagedBlockPool(8, 1, 1, 32, 16)
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.upload_step(np.array([[0, 9]], np.int32), np.array([20], np.int32))   # block 9 of 8
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.upload_step(np.array([[0]], np.int32), np.array([17], np.int32))      # ctx > table
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.upload_step(np.array([[0]], np.int32), np.array([3], np.int32), np.array([8 * 16], np.int64))
    pool.upload_step(np.array([[3, -1]], np.int32), np.array([16], np.int32), np.array([-1, 5], np.int64))


def test_decode_rejects_bad_head_counts_and_metadata_pools(cuda):
    import torch

    pool = G.PagedBlockPool(8, 1, 2, 32, 16)
    pool.upload_step(np.array([[0]], np.int32), np.array([4], np.int32))
    q = torch.zeros(1, 3, 32, device=cuda)
    out = torch.zeros(1, 3, 32, device=cuda)
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.paged_decode(0, q, out, 3, 1.0)
    meta = G.PagedBlockPool(8, 1, 2, 32, 16, allocate_device_arena=False)
    with pytest.raises(G.InvalidOperationError):
        meta.upload_step(np.array([[0]], np.int32), np.array([4], np.int32))
    odd = G.PagedBlockPool(8, 1, 1, 48, 16)
    odd.upload_step(np.array([[0]], np.int32), np.array([4], np.int32))
    with pytest.raises(G.UnsupportedError):
        odd.paged_decode(0, torch.zeros(1, 1, 48, device=cuda), torch.zeros(1, 1, 48, device=cuda), 1, 1.0)


def test_decode_launch_count(cuda):
    rng = np.random.default_rng(14)
    pool = G.PagedBlockPool(600, 1, 4, 128, 16)
    random_arena(pool, rng)
    ctx = [1000] * 8
    tables = random_tables(rng, ctx, 16, 600)
    q = rng.standard_normal((8, 28, 128)).astype(np.float32)
    gpu_decode(pool, 0, tables, ctx, q, 28, 0.1)
    assert pool.last_launch_count in (1, 2)


# ---- full-size configs: sampled oracle checks plus size-independent properties ----------

def test_cfg3_full_size_sampled_parity(cuda):
    from glacier_kv import workloads as W

    for dtype in ("f32", "bf16"):
        w = W.cfg3(dtype=dtype)
        pool = W.make_pool(w)
        W.fill_arena_randn(pool, seed=w.seed)
        rng = np.random.default_rng(w.seed)
        q = rng.standard_normal((w.batch, w.n_heads, w.head_dim)).astype(np.float32)
        out = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
        assert np.isfinite(out).all()
        rows = np.sort(rng.choice(w.batch, 12, replace=False))
        rows[0] = int(np.argmax(w.ctx_lens))  # include the longest sequence
        g, K, V, sub = compact(pool, w.tables, w.ctx_lens, rows)
        ref = O.decode_batch(K, V, g, 0, sub, w.ctx_lens[rows], q[rows], w.n_heads, w.scale)
        np.testing.assert_allclose(out[rows], ref, atol=TOL[dtype], rtol=0)
        pool.close()
