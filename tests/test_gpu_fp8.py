"""FP8 E4M3 KV storage with one K and one V scale per (layer, kv head), against the oracle.

Stores are e4m3(x * (1 / scale)), round to nearest even, saturated at +-448; both sides compute
the reciprocal with one IEEE division and the product with one fp32 multiply, so appended
bytes agree bit for bit.  The decode reads e4m3 * scale; it runs in fp32 on the same stored
values, so the bar is the fp32 one (the device folds the K scale into the score scale and the
V scale into the output, which changes only the rounding order)."""
import math
import zlib

import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, arena_to_host, geom_of, gpu_decode, random_arena, random_tables, scale_of
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _pool(nb, layers, nKv, d, bs=16, dv=None, seed=0, lo=0.02, hi=3.0):
    """An FP8 pool with random per-(layer, head) scales in [lo, hi)."""
    pool = G.PagedBlockPool(nb, layers, nKv, d, bs, dv or d, dtype="fp8")
    rng = np.random.default_rng(seed)
    pool.set_kv_scales(rng.uniform(lo, hi, (layers, nKv)), rng.uniform(lo, hi, (layers, nKv)))
    return pool


@pytest.mark.parametrize("d,dv", [(128, 128), (64, 64), (48, 16)])
def test_fp8_append_bit_exact_with_per_head_scales(cuda, d, dv):
    """Random slots with padding over two layers; values spread so that some saturate at
    +-448 * scale and some fall into the subnormals.  Nothing else in the arena changes."""
    import torch

    rng = np.random.default_rng(d)
    nb, bs, nKv, n = 700, 16, 4, 3001
    pool = _pool(nb, 2, nKv, d, bs, dv, seed=d + 1)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    slots = rng.choice(nb * bs, size=n, replace=False).astype(np.int64)
    slots[rng.choice(n, 29, replace=False)] = -1
    k = (rng.standard_normal((n, nKv, d)) * np.exp2(rng.uniform(-14, 10, (n, nKv, d)))).astype(np.float32)
    v = (rng.standard_normal((n, nKv, dv)) * np.exp2(rng.uniform(-14, 10, (n, nKv, dv)))).astype(np.float32)
    k[0, 0, :3] = [np.inf, -np.inf, -0.0]
    pool.reserve_step(1, 1, n, nKv)
    pool.upload_step(np.zeros((1, 1), np.int32), np.zeros(1, np.int32), slots)
    pool.kv_append(1, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    pool.sync()
    assert O.store_many(K, V, g, 1, slots, k, v) == 0
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    assert pool.last_launch_count == 1
    pool.close()


def test_fp8_block_copy_matches_oracle(cuda):
    rng = np.random.default_rng(31)
    pool = _pool(40, 3, 2, 64, 16, 32)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    src = rng.choice(20, 12, replace=False)
    dst = 20 + rng.choice(20, 12, replace=False)
    valid = np.array([1, 2, 7, 8, 9, 15, 16, 20, 0, -3, 5, 11])
    pool.block_copy(src, dst, valid)
    pool.sync()
    for s, d, n in zip(src, dst, valid):
        O.copy_block_data(K, V, g, int(s), int(d), int(n))
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    pool.close()


CASES = [
    # nH, nKv, d, bs, ctx
    (28, 4, 128, 16, [1, 7, 8, 9, 15, 16, 17, 31, 33, 127, 128, 129, 1000]),
    (32, 8, 128, 16, [2049, 2049, 5, 2049]),
    (40, 8, 128, 16, [3000, 7, 129]),               # group 5: idle heads of the pass
    (8, 8, 128, 16, [12000, 300, 5]),                # MHA; long and short splits
    (16, 1, 64, 16, [300, 45]),                      # group 16: two head groups
    (8, 2, 64, 12, [50, 12, 13]),                    # block size 12: chunks of 8 + 4
    (4, 4, 64, 16, [20000]),                         # one long sequence over many workers
    (28, 4, 128, 16, [12000, 700, 300, 90, 5]),
]


@pytest.mark.parametrize("case", CASES, ids=[f"h{c[0]}kv{c[1]}d{c[2]}bs{c[3]}" for c in CASES])
def test_fp8_decode_parity(cuda, case):
    nH, nKv, d, bs, ctx = case
    rng = np.random.default_rng(zlib.crc32(str(case).encode()))
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = _pool(need + 5, 2, nKv, d, bs, seed=nH, lo=0.25, hi=1.5)
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, ctx, bs, need + 5)
    q = rng.standard_normal((len(ctx), nH, d)).astype(np.float32)
    out = gpu_decode(pool, 1, tables, ctx, q, nH, scale_of(d))
    ref = O.decode_batch(K, V, geom_of(pool), 1, tables, np.array(ctx, np.int32), q, nH, scale_of(d))
    # the stored values are scaled up to 1.5x: the fp32 bar scales with the largest value
    vmax = float(np.abs(O.e4m3_bits_to_f32(V)).max() * pool.kv_scales[1].max())
    np.testing.assert_allclose(out, ref, atol=TOL["fp8"] * max(1.0, vmax), rtol=0)
    pool.close()


def test_fp8_append_then_decode_reads_the_scaled_values(cuda):
    """Append through the kernel, decode through the kernel: equal to the oracle's store +
    decode of the same inputs (the stored bytes are bit-exact, the decode within the bar)."""
    import torch

    rng = np.random.default_rng(41)
    nKv, nH, d, bs = 4, 28, 128, 16
    ctx = [333, 1, 64, 1500]
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = _pool(need, 1, nKv, d, bs, seed=3)
    g = geom_of(pool)
    K, V = O.new_arena(g)
    tables = random_tables(rng, ctx, bs, need)
    slots = np.concatenate([tables[b, np.arange(c) // bs].astype(np.int64) * bs + np.arange(c) % bs
                            for b, c in enumerate(ctx)])
    n = slots.size
    k = rng.standard_normal((n, nKv, d)).astype(np.float32)
    v = rng.standard_normal((n, nKv, d)).astype(np.float32)
    pool.reserve_step(len(ctx), tables.shape[1], n, nH)
    pool.upload_step(tables, np.asarray(ctx, np.int32), slots)
    pool.kv_append(0, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    q = rng.standard_normal((len(ctx), nH, d)).astype(np.float32)
    out = torch.zeros((len(ctx), nH, d), dtype=torch.float32, device=cuda)
    pool.paged_decode(0, torch.from_numpy(q).to(cuda), out, nH, scale_of(d))
    pool.sync()
    assert O.store_many(K, V, g, 0, slots, k, v) == 0
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    ref = O.decode_batch(K, V, g, 0, tables, np.asarray(ctx, np.int32), q, nH, scale_of(d))
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL["fp8"], rtol=0)
    pool.close()


@pytest.mark.parametrize("q_dtype", ["f32", "bf16"])
def test_fp8_prefill_parity(cuda, q_dtype):
    """FP8 pools run the chunked prefill on the decode kernel, one segment per query."""
    import torch

    rng = np.random.default_rng(51)
    prefixes, q_lens, nH, nKv, d = [0, 45, 300], [70, 1, 33], 28, 4, 128
    need = sum((p + n + 15) // 16 for p, n in zip(prefixes, q_lens)) + 2
    pool = _pool(need, 1, nKv, d, 16, seed=5, lo=0.25, hi=1.5)
    toks = [p + n for p, n in zip(prefixes, q_lens)]
    tables = random_tables(rng, toks, 16, need)
    K, V = random_arena(pool, rng)
    q = rng.standard_normal((sum(q_lens), nH, d)).astype(np.float32)
    if q_dtype == "bf16":
        q = O.bf16_bits_to_f32(O.f32_to_bf16_bits(q))
    qt = torch.from_numpy(q).to(cuda)
    if q_dtype == "bf16":
        qt = qt.to(torch.bfloat16)
    out = torch.zeros((sum(q_lens), nH, d), dtype=torch.float32, device=cuda)
    pool.upload_step(tables, np.asarray(toks, np.int32))
    pool.paged_prefill(0, qt, out, np.asarray(prefixes, np.int32), np.asarray(q_lens, np.int32), nH,
                       1 / math.sqrt(d))
    pool.sync()
    got, off, g = out.cpu().numpy(), 0, geom_of(pool)
    for b, n in enumerate(q_lens):
        ref = O.prefill_chunk(K, V, g, 0, tables[b], toks[b], prefixes[b], q[off:off + n], nH, 1 / math.sqrt(d))
        np.testing.assert_allclose(got[off:off + n], ref, atol=TOL["fp8"], rtol=0)
        off += n
    pool.close()


def test_fp8_rope_append_bit_exact(cuda):
    """The fused bias + QK RMSNorm + RoPE + append stores the rotated k with the K scale and the
    biased v with the V scale, bit for bit; q is rewritten exactly as for the other types."""
    import torch

    rng = np.random.default_rng(61)
    nb, bs, nKv, nH, d, n_tok = 64, 16, 4, 28, 128, 37
    pool = _pool(nb, 2, nKv, d, bs, seed=7)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    slots = rng.choice(nb * bs, size=n_tok, replace=False).astype(np.int64)
    slots[3] = -1
    pos = rng.integers(0, 131072, size=n_tok).astype(np.int32)
    q = rng.standard_normal((n_tok, nH, d)).astype(np.float32) * 3
    k = rng.standard_normal((n_tok, nKv, d)).astype(np.float32) * 3
    v = rng.standard_normal((n_tok, nKv, d)).astype(np.float32)
    terms = dict(q_bias=rng.standard_normal(nH * d).astype(np.float32),
                 k_bias=rng.standard_normal(nKv * d).astype(np.float32),
                 v_bias=rng.standard_normal(nKv * d).astype(np.float32),
                 q_norm=rng.uniform(0.5, 1.5, d).astype(np.float32),
                 k_norm=rng.uniform(0.5, 1.5, d).astype(np.float32))
    inv = G.rope_inv_freq(1_000_000.0, d)
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    qd = dev(q)
    pool.upload_step(np.zeros((1, 1), np.int32), np.zeros(1, np.int32), slots)
    pool.rope_append(1, qd, dev(k), dev(v), pos, nH, freq_base=1_000_000.0, eps=1e-6,
                     **{n: dev(a) for n, a in terms.items()})
    pool.sync()
    q_ref = O.rope_append(K, V, g, 1, q, k, v, pos, slots, inv, d, G.GKV_ROPE_NEOX, 1.0, eps=1e-6, **terms)
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(qd.cpu().numpy().view(np.uint32), q_ref.view(np.uint32))
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    pool.close()


def test_fp8_unsupported_shapes_and_noalloc_are_refused(cuda):
    """The FP8 decode is built for head dims 64 and 128; other dims are refused before any
    launch, and the raw-arena entry point (which has no scales to read) refuses FP8 arenas."""
    import torch

    pool = _pool(8, 1, 2, 32, 16)
    pool.upload_step(np.array([[0]], np.int32), np.array([5], np.int32))
    q = torch.zeros((1, 4, 32), device=cuda)
    out = torch.zeros((1, 4, 32), device=cuda)
    with pytest.raises(G.GkvError):
        pool.paged_decode(0, q, out, 4, 0.25)
    pool.close()
    pool = _pool(8, 1, 2, 64, 16)
    q = torch.zeros((1, 4, 64), device=cuda)
    out = torch.zeros((1, 4, 64), device=cuda)
    with pytest.raises(G.ArgumentOutOfRangeError):
        G.paged_decode_noalloc(pool, 0, np.array([[0]], np.int32), np.array([5], np.int32), q, out, 4, 0.125)
    pool.close()


def test_fp8_tensor_core_sinks_and_lse(cuda):
    """The tensor-core FP8 decode (group 7, d 128) with per-head sinks matches the oracle, and its
    lse output is ln of the softmax denominator over the scaled keys (long sequences split over
    warps, so the merged partials carry the scales too)."""
    import torch

    rng = np.random.default_rng(81)
    nH, nKv, d, bs = 28, 4, 128, 16
    ctx = [3000, 13, 700]
    need = sum((c + bs - 1) // bs for c in ctx)
    pool = _pool(need + 2, 1, nKv, d, bs, seed=9, lo=0.25, hi=1.5)
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, ctx, bs, need + 2)
    q = rng.standard_normal((len(ctx), nH, d)).astype(np.float32)
    g = geom_of(pool)
    sink = 0.6
    out = gpu_decode(pool, 0, tables, ctx, q, nH, scale_of(d), sinks=np.full(nH, sink, np.float32))
    ref = O.decode_batch(K, V, g, 0, tables, np.array(ctx, np.int32), q, nH, scale_of(d), sink_logit=sink)
    vmax = float(np.abs(O.e4m3_bits_to_f32(V)).max() * pool.kv_scales[1].max())
    np.testing.assert_allclose(out, ref, atol=TOL["fp8"] * max(1.0, vmax), rtol=0)
    # lse without sinks
    qd = torch.from_numpy(q).to(cuda)
    o2 = torch.zeros((len(ctx), nH, d), device=cuda)
    lse = torch.zeros((len(ctx), nH), device=cuda)
    pool.upload_step(tables, np.array(ctx, np.int32))
    pool.paged_decode_lse(0, qd, o2, lse, nH, scale_of(d))
    pool.sync()
    ks, _ = pool.kv_scales
    for b, c in enumerate(ctx):
        for h in (0, 13, 27):
            hk = h // (nH // nKv)
            kk = np.stack([O.e4m3_bits_to_f32(K[tables[b, t // bs], 0, hk, t % bs]) for t in range(c)]).astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) * float(ks[0, hk]) * scale_of(d)
            want = s.max() + math.log(np.exp(s - s.max()).sum())
            assert abs(float(lse[b, h]) - want) < 1e-3 * max(1.0, abs(want))
    pool.close()
