"""Pins the CPU oracle against the reference's own fixtures before it is trusted as checker.

The reference (C#) cannot run here; these are the values its tests fix (see
tests/golden/make_golden.py for provenance) plus the argument checks it throws on.
"""
import glob
import json
import math
import os

import numpy as np
import pytest

from conftest import ROOT
from oracle import pyoracle as O

GOLD = os.path.join(ROOT, "tests", "golden")


def kat_inputs(dtype=O.F32):
    kat = json.load(open(os.path.join(GOLD, "kat_compute_attention.json")))
    d, T, nH, nKv, bs = kat["head_dim"], kat["tokens"], kat["n_heads"], kat["n_heads_kv"], kat["block_size"]
    g = O.geom(8, 1, nKv, d, d, bs, dtype)
    K, V = O.new_arena(g)
    ids = []
    for t in range(T):  # BlockTable.AppendToken on a fresh pool -> blocks 0, 1
        blk, off = t // bs, t % bs
        if off == 0:
            ids.append(blk)
        k = np.zeros((nKv, d), np.float32)
        v = np.zeros((nKv, d), np.float32)
        for h in range(nKv):
            k[h] = kat["k_value_per_token"][t]
            v[h] = kat["v_scale_per_kv_head"][h] * (t + 1)
        assert O.store(K, V, g, blk, 0, off, k.ravel(), v.ravel()) == 0
    q = np.full((nH, d), kat["q_value"], np.float32)
    return kat, g, K, V, ids, q


def test_oracle_matches_closed_form_kat():
    kat, g, K, V, ids, q = kat_inputs()
    rc, out = O.compute_attention(K, V, g, 0, kat["tokens"] - 1, q, ids, kat["tokens"], kat["n_heads"],
                                  kat["n_heads_kv"], kat["head_dim"], kat["head_dim"], kat["attn_scale"],
                                  kat["tokens"])
    assert rc == 0
    for h, e in enumerate(kat["expected_per_head"]):
        assert out[h].min() > 0  # the reference test's assertion
        np.testing.assert_allclose(out[h], e, rtol=2e-6)  # fp32 arithmetic vs float64 closed form
        assert np.all(out[h] == out[h][0])  # per-head uniformity (:171-177)


def test_oracle_store_retrieve_exact():
    s = json.load(open(os.path.join(GOLD, "store_retrieve.json")))
    g = O.geom(s["total_blocks"], s["layers"], s["heads_kv"], s["head_dim"], s["head_dim"], s["block_size"])
    K, V = O.new_arena(g)
    assert O.store(K, V, g, 0, s["layer"], s["slot"], np.array(s["k"], np.float32), np.array(s["v"], np.float32)) == 0
    for h in range(2):
        assert list(K[0, s["layer"], h, s["slot"]]) == s["k"][4 * h: 4 * h + 4]
        assert list(V[0, s["layer"], h, s["slot"]]) == s["v"][4 * h: 4 * h + 4]
    assert K.sum() == sum(s["k"]) and V.sum() == sum(s["v"])


def test_oracle_copy_block_data_sentinels():
    """PrefixHashKvCacheTests.cs:134-181: the fork holds 42.0; mutating it leaves the source."""
    g = O.geom(16, 2, 2, 32, 32, 16)
    K, V = O.new_arena(g)
    K[0, 0, 0, 0, 0] = 42.0
    assert O.copy_block_data(K, V, g, 0, 1, 10) == 0
    assert K[1, 0, 0, 0, 0] == 42.0
    K[1, 0, 0, 0, 0] = 999.0
    assert K[0, 0, 0, 0, 0] == 42.0
    # only the first `valid` slots are copied (PagedBlockPool.cs:309-315)
    K[0, 1, 1, 12, :] = 7.0
    assert O.copy_block_data(K, V, g, 0, 2, 10) == 0
    assert np.all(K[2, 1, 1, 12] == 0)
    assert O.copy_block_data(K, V, g, 0, 3, 0) == 0 and np.all(K[3] == 0)


@pytest.mark.parametrize("dtype", [O.F32, O.BF16])
def test_oracle_batch_loops_equal_single_calls(dtype):
    """store_many / copy_many (the bench's CPU baseline loops) are one Store / CopyBlockData
    per entry; padding slots are skipped and a bad slot or block is rejected."""
    rng = np.random.default_rng(5)
    g = O.geom(20, 2, 3, 8, 4, 4, dtype)
    K1, V1 = O.new_arena(g)
    K2, V2 = O.new_arena(g)
    slots = np.array([5, -1, 79, 0, 33], np.int64)
    k = rng.standard_normal((5, 3, 8)).astype(np.float32)
    v = rng.standard_normal((5, 3, 4)).astype(np.float32)
    assert O.store_many(K1, V1, g, 1, slots, k, v) == 0
    for i, s in enumerate(slots):
        if s >= 0:
            assert O.store(K2, V2, g, int(s) // 4, 1, int(s) % 4, k[i], v[i]) == 0
    assert np.array_equal(K1, K2) and np.array_equal(V1, V2) and K1.any()
    assert O.copy_many(K1, V1, g, [1, 19, 8], [2, 3, 4], [4, 2, 0]) == 0
    for s, d, n in ((1, 2, 4), (19, 3, 2), (8, 4, 0)):
        assert O.copy_block_data(K2, V2, g, s, d, n) == 0
    assert np.array_equal(K1, K2) and np.array_equal(V1, V2)
    assert O.store_many(K1, V1, g, 0, np.array([80], np.int64), k[:1], v[:1]) != 0  # block 20 of 20
    assert O.copy_many(K1, V1, g, [0], [20], [4]) != 0


@pytest.mark.parametrize("pos", [16, -1])
def test_oracle_rejects_out_of_bounds_position(pos):
    """PhaseCServeRemediationTests.cs:117-174: pos outside [0, maxSeqLen) throws."""
    g = O.geom(4, 1, 1, 32, 32, 16)
    K, V = O.new_arena(g)
    rc, _ = O.compute_attention(K, V, g, 0, pos, np.zeros((1, 32), np.float32), [0], 1, 1, 1, 32, 32,
                                1 / math.sqrt(32), 16)
    assert rc == -1


def test_oracle_other_argument_checks_and_noop():
    g = O.geom(4, 1, 1, 32, 32, 16)
    K, V = O.new_arena(g)
    q = np.ones((1, 32), np.float32)
    assert O.compute_attention(K, V, g, 0, 0, q, [0], 1, 1, 1, 32, 32, 1.0, 0)[0] == -1   # maxSeqLen <= 0
    assert O.compute_attention(K, V, g, 0, 0, q, [0], 17, 1, 1, 32, 32, 1.0, 16)[0] == -1  # TokenCount > max
    rc, out = O.compute_attention(K, V, g, 0, 3, q, [], 0, 1, 1, 32, 32, 1.0, 16)          # n == 0: no-op
    assert rc == 0 and np.all(out == 0)


def test_oracle_causal_length_is_min_of_count_and_pos():
    """n = min(TokenCount, pos + 1) (PagedAttentionKernel.cs:41): pos < count attends a prefix."""
    rng = np.random.default_rng(3)
    g = O.geom(4, 1, 1, 32, 32, 16)
    K, V = O.new_arena(g)
    K[...] = rng.standard_normal(K.shape)
    V[...] = rng.standard_normal(V.shape)
    q = rng.standard_normal((2, 32)).astype(np.float32)
    _, a = O.compute_attention(K, V, g, 0, 9, q, [2, 0], 20, 2, 1, 32, 32, 0.2, 32)
    _, b = O.compute_attention(K, V, g, 0, 31, q, [2, 0], 10, 2, 1, 32, 32, 0.2, 32)
    np.testing.assert_array_equal(a, b)


def test_oracle_sink_only_enters_the_denominator():
    rng = np.random.default_rng(4)
    g = O.geom(2, 1, 1, 32, 32, 16)
    K, V = O.new_arena(g)
    K[...] = rng.standard_normal(K.shape)
    V[...] = rng.standard_normal(V.shape)
    q = rng.standard_normal((1, 32)).astype(np.float32)
    _, plain = O.compute_attention(K, V, g, 0, 11, q, [1], 12, 1, 1, 32, 32, 0.3, 16)
    _, sunk = O.compute_attention(K, V, g, 0, 11, q, [1], 12, 1, 1, 32, 32, 0.3, 16, sink_logit=0.5)
    # double-precision restatement of softmax with a sink
    s = np.array([float(np.dot(q[0].astype(np.float64), K[1, 0, 0, t])) * 0.3 for t in range(12)])
    m = max(s.max(), 0.5)
    w = np.exp(s - m)
    den = w.sum() + math.exp(0.5 - m)
    ref = (w[:, None] * V[1, 0, 0, :12].astype(np.float64)).sum(0) / den
    np.testing.assert_allclose(sunk[0], ref, atol=1e-5)
    np.testing.assert_allclose(plain[0] * (w.sum() / den), sunk[0], atol=1e-5)


def test_bf16_rounding_restatements_agree():
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 10 ** rng.uniform(-30, 30, 4096).astype(np.float32),
                        np.array([0.0, -0.0, 1.0, np.inf, -np.inf, 1.00390625, 1.01171875, 3.4e38], np.float32)])
    bits = O.f32_to_bf16_bits(x)
    for v, b in zip(x[::37], bits[::37]):
        assert O.lib.oracle_f32_to_bf16(float(v)) == b
    # ties go to even: 1 + 2^-8 is halfway between 1 and 1 + 2^-7
    assert O.lib.oracle_f32_to_bf16(1.00390625) == 0x3F80
    assert O.lib.oracle_f32_to_bf16(1.01171875) == 0x3F82


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "decode_small_*.npz"))))
def test_oracle_reproduces_committed_decode_fixtures(path):
    z = np.load(path)
    g = O.geom(*[int(x) for x in z["geom"]])
    out = O.decode_batch(z["K"], z["V"], g, 0, z["tables"], z["ctx"], z["q"], int(z["n_heads"]), float(z["scale"]))
    np.testing.assert_array_equal(out, z["out"])
    # the scheduling variant computes the same numbers
    par = O.decode_batch(z["K"], z["V"], g, 0, z["tables"], z["ctx"], z["q"], int(z["n_heads"]), float(z["scale"]),
                         parallel=True)
    np.testing.assert_array_equal(par, z["out"])


def test_oracle_decode_against_float64_numpy():
    """Independent float64 restatement of the math on one fixture (checks the C oracle)."""
    z = np.load(os.path.join(GOLD, "decode_small_gqa4_d32_bs16_f32.npz"))
    K, V, tables, ctx, q = z["K"], z["V"], z["tables"], z["ctx"], z["q"]
    nH, scale = int(z["n_heads"]), float(z["scale"])
    nKv = K.shape[2]
    for b, c in enumerate(ctx):
        rows = [(tables[b, t // 16], t % 16) for t in range(c)]
        for h in range(nH):
            kv = h // (nH // nKv)
            kk = np.stack([K[blk, 0, kv, o] for blk, o in rows]).astype(np.float64)
            vv = np.stack([V[blk, 0, kv, o] for blk, o in rows]).astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) * scale
            p = np.exp(s - s.max())
            p /= p.sum()
            np.testing.assert_allclose(z["out"][b, h], p @ vv, atol=2e-6)


def test_oracle_prefill_equals_per_token_compute():
    rng = np.random.default_rng(9)
    g = O.geom(6, 1, 2, 32, 32, 16)
    K, V = O.new_arena(g)
    K[...] = rng.standard_normal(K.shape)
    V[...] = rng.standard_normal(V.shape)
    ids = [4, 1, 3]
    q = rng.standard_normal((10, 4, 32)).astype(np.float32)
    out = O.prefill_chunk(K, V, g, 0, ids, 40, 30, q, 4, 0.25)
    for t in range(10):
        _, o = O.compute_attention(K, V, g, 0, 30 + t, q[t], ids, 40, 4, 2, 32, 32, 0.25, 48)
        np.testing.assert_array_equal(out[t], o)


def test_f16_storage_rounding_is_ieee_round_to_nearest_even():
    """The oracle's fp32 -> fp16 rounding (the storage rounding of fp16 arenas) agrees with
    IEEE 754 binary16 round-to-nearest-even as numpy implements it, over random bit patterns of
    the whole fp32 range and the edge cases (overflow, subnormals, ties), and fp16 -> fp32 is
    exact for all 65536 patterns."""
    import numpy as np

    from oracle import pyoracle as O

    rng = np.random.default_rng(16)
    x = rng.integers(0, 2**32, size=2_000_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    edge = np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e30, np.inf, -np.inf, 2.9802322e-08,
                     2.9802326e-08, 5.9604645e-08, 6.1035156e-05, 6.1033e-05, 1.0009766, 1.0004883, -2.5],
                    np.float32)
    x = np.concatenate([x, edge])
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    got = O.f32_to_f16_bits(x)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], ref[~nan])
    assert np.isnan(got[nan].view(np.float16)).all()
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    back = np.array([O.lib.oracle_f16_to_f32(int(v)) for v in h], np.float32)
    want = h.view(np.float16).astype(np.float32)
    assert ((back == want) | (np.isnan(back) & np.isnan(want))).all()


def test_f16_store_rounds_and_decodes_from_the_rounded_values():
    """Store into an fp16 arena keeps the rounded bits; the decode reads them back exactly."""
    import numpy as np

    from oracle import pyoracle as O

    rng = np.random.default_rng(17)
    g = O.geom(4, 1, 2, 16, 16, 4, O.F16)
    K, V = O.new_arena(g)
    k = rng.standard_normal(32).astype(np.float32)
    v = rng.standard_normal(32).astype(np.float32)
    assert O.store(K, V, g, 2, 0, 1, k, v) == 0
    assert np.array_equal(K[2, 0, :, 1].ravel(), O.f32_to_f16_bits(k))
    assert np.array_equal(V[2, 0, :, 1].ravel(), O.f32_to_f16_bits(v))
    # one token attended: the output is that token's (rounded) value row
    q = rng.standard_normal((1, 2, 16)).astype(np.float32)
    tables = np.array([[2]], np.int32)
    K2, V2 = O.new_arena(g)
    O.store(K2, V2, g, 2, 0, 0, k, v)
    out = O.decode_batch(K2, V2, g, 0, tables, np.array([1], np.int32), q, 2, 0.25)
    assert np.array_equal(out.reshape(-1), O.f16_bits_to_f32(O.f32_to_f16_bits(v)))


def test_e4m3_storage_rounding_matches_torch_float8_e4m3fn():
    """The oracle's fp32 -> FP8 E4M3 conversion (the storage rounding of FP8 arenas) is OCP
    E4M3 round-to-nearest-even saturated at +-448: over random values spanning the whole e4m3
    range, ties and the edges it agrees with torch's float8_e4m3fn cast of the value clamped to
    [-448, 448] (torch's cast itself does not saturate), and all 256 bytes decode as torch
    decodes them."""
    import numpy as np
    import torch

    from oracle import pyoracle as O

    rng = np.random.default_rng(8)
    mag = np.exp2(rng.uniform(-12.0, 9.5, 1_000_000)).astype(np.float32)
    x = mag * rng.choice(np.array([-1.0, 1.0], np.float32), mag.size)
    # exact ties between neighbouring e4m3 values, normals and subnormals
    grid = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    grid = np.unique(grid[np.isfinite(grid)])
    ties = ((grid[:-1].astype(np.float64) + grid[1:]) / 2).astype(np.float32)
    edge = np.array([0.0, -0.0, 448.0, 464.0, 480.0, 1e9, np.inf, -np.inf, 2.0**-9, 2.0**-10, 2.0**-11,
                     2.0**-6, 0.0009765625, 1e-30], np.float32)
    x = np.concatenate([x, ties, edge])
    got = O.f32_to_e4m3_bits(x)
    want = torch.from_numpy(np.clip(x, -448.0, 448.0)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(got, want)
    nan = O.f32_to_e4m3_bits(np.array([np.nan], np.float32))[0]
    assert (nan & 0x7F) == 0x7F
    b = np.arange(256, dtype=np.uint8)
    back = O.e4m3_bits_to_f32(b)
    ref = torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    assert ((back == ref) | (np.isnan(back) & np.isnan(ref))).all()


def test_fp8_store_applies_the_per_head_scales_and_decode_reads_them_back():
    """An FP8 arena stores e4m3(x * (1 / scale)) with the (layer, head) scale of the row and
    reads e4m3 * scale: one attended token returns its value row as stored and scaled back."""
    import numpy as np

    from oracle import pyoracle as O

    rng = np.random.default_rng(18)
    g = O.geom(4, 2, 2, 16, 16, 4, O.FP8)
    ks = np.array([[0.5, 2.0], [0.25, 4.0]], np.float32)
    vs = np.array([[3.0, 0.125], [1.5, 0.75]], np.float32)
    g.set_scales(ks, vs)
    K, V = O.new_arena(g)
    k = (rng.standard_normal(32) * 8).astype(np.float32)
    v = (rng.standard_normal(32) * 8).astype(np.float32)
    assert O.store(K, V, g, 2, 1, 0, k, v) == 0
    for h in range(2):
        inv_k = np.float32(1.0) / ks[1, h]
        inv_v = np.float32(1.0) / vs[1, h]
        assert np.array_equal(K[2, 1, h, 0], O.f32_to_e4m3_bits(k[h * 16:(h + 1) * 16] * inv_k))
        assert np.array_equal(V[2, 1, h, 0], O.f32_to_e4m3_bits(v[h * 16:(h + 1) * 16] * inv_v))
    q = rng.standard_normal((1, 2, 16)).astype(np.float32)
    out = O.decode_batch(K, V, g, 1, np.array([[2]], np.int32), np.array([1], np.int32), q, 2, 0.25)
    want = np.concatenate([O.e4m3_bits_to_f32(V[2, 1, h, 0]) * vs[1, h] for h in range(2)])
    assert np.array_equal(out.reshape(-1), want)
