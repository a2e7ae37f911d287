"""The restated q/k prologue (bias, per-head RMSNorm, RoPE) of the oracle, on the CPU: its sin and
cos against double-precision values, its rotation against a float64 restatement, and the
inverse-frequency table of the C ABI.  QuantKernels.RoPE / RMSNorm (NuGet Glacier.Inference 1.7.0)
are not in the reference tree, so this pins the stated formulas, not the reference's bits."""
import numpy as np
import pytest

from oracle import pyoracle as O


def test_sincos_within_two_ulp_of_double_precision():
    rng = np.random.default_rng(0)
    th = np.concatenate([rng.uniform(-7, 7, 4000), rng.uniform(0, 140_000, 4000),
                         np.arange(0, 64, 0.125), [0.0, np.pi / 4, np.pi / 2, 1e5]]).astype(np.float32)
    for t in th:
        s, c = O.sincos(float(t))
        assert abs(s - np.sin(np.float64(t))) <= 1.2e-7
        assert abs(c - np.cos(np.float64(t))) <= 1.2e-7
    assert O.sincos(0.0) == (0.0, 1.0)


def _rope_f64(x, pos, inv_freq, R, style, mscale):
    y = x.astype(np.float64).copy()
    for i in range(R // 2):
        a, b = (i, i + R // 2) if style == 0 else (2 * i, 2 * i + 1)
        th = np.float64(np.float32(pos) * np.float32(inv_freq[i]))
        c, s = np.cos(th), np.sin(th)
        y[..., a] = (x[..., a] * c - x[..., b] * s) * mscale
        y[..., b] = (x[..., b] * c + x[..., a] * s) * mscale
    return y


@pytest.mark.parametrize("style,R", [(0, 128), (1, 128), (0, 64), (1, 32)])
def test_rope_matches_a_float64_restatement(style, R):
    rng = np.random.default_rng(R + style)
    d, nH, nKv, n = 128, 4, 2, 5
    g = O.geom(4, 1, nKv, d, d, 16)
    K, V = O.new_arena(g)
    q = rng.standard_normal((n, nH, d)).astype(np.float32)
    k = rng.standard_normal((n, nKv, d)).astype(np.float32)
    v = rng.standard_normal((n, nKv, d)).astype(np.float32)
    pos = np.array([0, 1, 17, 4095, 131071], np.int32)
    slots = np.arange(n, dtype=np.int64) * 3
    inv = (10000.0 ** (-2.0 * np.arange(R // 2) / R)).astype(np.float32)
    qr = O.rope_append(K, V, g, 0, q, k, v, pos, slots, inv, R, style, mscale=1.25)
    for t in range(n):
        np.testing.assert_allclose(qr[t], _rope_f64(q[t], pos[t], inv, R, style, 1.25), atol=2e-5, rtol=0)
        blk, off = divmod(int(slots[t]), 16)
        np.testing.assert_allclose(K[blk, 0, :, off], _rope_f64(k[t], pos[t], inv, R, style, 1.25), atol=2e-5)
        assert np.array_equal(V[blk, 0, :, off], v[t])  # v is stored as is
    # position 0 rotates by nothing: q and k come back bit for bit (mscale 1)
    q0 = O.rope_append(K, V, g, 0, q[:1], k[:1], v[:1], pos[:1], slots[:1], inv, R, style)
    assert np.array_equal(q0, q[:1]) and np.array_equal(K[0, 0, :, 0], k[0])


def test_qk_norm_and_bias_restatement():
    rng = np.random.default_rng(3)
    d, nH, nKv = 64, 2, 1
    g = O.geom(2, 1, nKv, d, d, 16)
    K, V = O.new_arena(g)
    q = rng.standard_normal((1, nH, d)).astype(np.float32)
    k = rng.standard_normal((1, nKv, d)).astype(np.float32)
    v = rng.standard_normal((1, nKv, d)).astype(np.float32)
    qb, kb, vb = (rng.standard_normal(n).astype(np.float32) for n in (nH * d, nKv * d, nKv * d))
    qw, kw = (rng.uniform(0.5, 1.5, d).astype(np.float32) for _ in range(2))
    inv = np.ones(d // 2, np.float32)
    qr = O.rope_append(K, V, g, 0, q, k, v, [0], [0], inv, d, 0, 1.0, qb, kb, vb, qw, kw, 1e-6)
    x = (q.reshape(nH, d) + qb.reshape(nH, d)).astype(np.float64)
    want = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * qw
    np.testing.assert_allclose(qr.reshape(nH, d), want, atol=1e-5)
    x = (k.reshape(d) + kb).astype(np.float64)
    np.testing.assert_allclose(K[0, 0, 0, 0], x / np.sqrt((x * x).mean() + 1e-6) * kw, atol=1e-5)
    np.testing.assert_array_equal(V[0, 0, 0, 0], v.reshape(d) + vb)


def test_inverse_frequency_table_of_the_c_abi():
    import glacier_kv as G

    for base, R in ((10000.0, 128), (1_000_000.0, 64), (500000.0, 2)):
        want = (np.float64(base) ** (-2.0 * np.arange(R // 2) / R)).astype(np.float32)
        assert np.array_equal(G.rope_inv_freq(base, R), want)
    fac = np.linspace(1, 8, 64).astype(np.float32)
    want = (10000.0 ** (-2.0 * np.arange(64) / 128)).astype(np.float32) / fac
    assert np.array_equal(G.rope_inv_freq(10000.0, 128, fac), want)
    with pytest.raises(G.ArgumentOutOfRangeError):
        G.rope_inv_freq(10000.0, 7)
