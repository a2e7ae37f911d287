"""gkv_rope_append: bias + per-head RMSNorm + RoPE of q and k fused with the KV append, against the
oracle's restatement of PagedTransformerRunner.ForwardBatch's steps before Store
(PagedTransformerRunner.cs:612-634).  Every operation of both is an IEEE-rounded step in one stated
order, so the arena slots and the rewritten q agree bit for bit."""
import math

import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, arena_to_host, geom_of, gpu_decode, random_arena, random_tables
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _case(cuda, dtype, d, dv, nH, nKv, rope_dim, style, *, prologue, table, mscale, seed, n_tok=37,
          bs=16, layers=2, layer=1):
    import torch

    rng = np.random.default_rng(seed)
    nb = 64
    pool = G.PagedBlockPool(nb, layers, nKv, d, bs, dv, dtype=dtype)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    slots = rng.choice(nb * bs, size=n_tok, replace=False).astype(np.int64)
    slots[3] = -1  # a padding token: q is still rotated, nothing is stored
    pos = rng.integers(0, 131072, size=n_tok).astype(np.int32)
    pos[0] = 0
    q = rng.standard_normal((n_tok, nH, d)).astype(np.float32) * 3
    k = rng.standard_normal((n_tok, nKv, d)).astype(np.float32) * 3
    v = rng.standard_normal((n_tok, nKv, dv)).astype(np.float32)
    R = rope_dim or d
    inv = (rng.uniform(1e-6, 1.0, R // 2).astype(np.float32) if table
           else G.rope_inv_freq(1_000_000.0, R))
    terms = {}
    if prologue:
        terms = dict(q_bias=rng.standard_normal(nH * d).astype(np.float32),
                     k_bias=rng.standard_normal(nKv * d).astype(np.float32),
                     v_bias=rng.standard_normal(nKv * dv).astype(np.float32),
                     q_norm=rng.uniform(0.5, 1.5, d).astype(np.float32),
                     k_norm=rng.uniform(0.5, 1.5, d).astype(np.float32))
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    qd, kd, vd = dev(q), dev(k), dev(v)
    pool.upload_step(np.zeros((1, 1), np.int32), np.zeros(1, np.int32), slots)
    pool.rope_append(layer, qd, kd, vd, pos, nH, rope_dim=rope_dim, style=style,
                     inv_freq=inv if table else None, freq_base=1_000_000.0, mscale=mscale,
                     eps=1e-6, **{n: dev(a) for n, a in terms.items()})
    pool.sync()
    q_ref = O.rope_append(K, V, g, layer, q, k, v, pos, slots, inv, R, style, mscale, eps=1e-6, **terms)
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(qd.cpu().numpy().view(np.uint32), q_ref.view(np.uint32))
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    assert pool.last_launch_count == 1
    return pool, K, V, q_ref, slots, pos


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("style", [G.GKV_ROPE_NEOX, G.GKV_ROPE_INTERLEAVED])
def test_rope_append_bit_exact_qwen_shape(cuda, dtype, style):
    """28 q / 4 kv heads, d 128, biases and QK RMSNorm, the table built from freq_base."""
    pool, *_ = _case(cuda, dtype, 128, 128, 28, 4, 0, style, prologue=True, table=False, mscale=1.0,
                     seed=11 + style)
    pool.close()


@pytest.mark.parametrize("d,dv,nH,nKv,rope_dim,style", [
    (128, 128, 8, 8, 64, 0),    # partial rotary, MHA
    (64, 64, 16, 2, 0, 0),
    (64, 32, 4, 1, 32, 1),
    (32, 32, 6, 3, 0, 1),       # one element per lane: interleaved pairs across lanes
    (32, 64, 6, 3, 16, 0),
    (256, 256, 4, 1, 0, 0),
])
def test_rope_append_bit_exact_shapes(cuda, d, dv, nH, nKv, rope_dim, style):
    """Explicit inverse-frequency table (the YaRN case) and mscale, bf16 arena."""
    pool, *_ = _case(cuda, "bf16", d, dv, nH, nKv, rope_dim, style, prologue=d != 256, table=True,
                     mscale=1.0 + 0.1 * math.log(4.0), seed=d + nH + style, bs=8)
    pool.close()


def test_rope_append_then_decode(cuda):
    """The rotated q and the stored k feed the decode: its output matches the oracle's decode of
    the oracle's arena with the oracle's rotated q."""
    import torch

    rng = np.random.default_rng(5)
    ctx = [300, 17, 1000]
    pool = G.PagedBlockPool(120, 1, 4, 128, 16, dtype="f32")
    K, V = random_arena(pool, rng)
    tables = random_tables(rng, ctx, 16, 120)
    slots = np.array([tables[b, (c - 1) // 16] * 16 + (c - 1) % 16 for b, c in enumerate(ctx)], np.int64)
    pos = np.array(ctx, np.int32) - 1
    q = rng.standard_normal((3, 28, 128)).astype(np.float32)
    k = rng.standard_normal((3, 4, 128)).astype(np.float32)
    v = rng.standard_normal((3, 4, 128)).astype(np.float32)
    qd = torch.from_numpy(q).to(cuda)
    out = torch.zeros((3, 28, 128), device=cuda)
    pool.upload_step(tables, np.array(ctx, np.int32), slots)
    pool.rope_append(0, qd, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda), pos, 28)
    pool.paged_decode(0, qd, out, 28, 1 / math.sqrt(128))
    pool.sync()
    g = geom_of(pool)
    q_ref = O.rope_append(K, V, g, 0, q, k, v, pos, slots, G.rope_inv_freq(10000.0, 128), 128, 0)
    ref = O.decode_batch(K, V, g, 0, tables, np.array(ctx, np.int32), q_ref, 28, 1 / math.sqrt(128))
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL["f32"], rtol=0)
    pool.close()


def test_rope_append_argument_errors(cuda):
    import torch

    pool = G.PagedBlockPool(8, 1, 2, 128, 16)
    q = torch.zeros((2, 4, 128), device=cuda)
    k = torch.zeros((2, 2, 128), device=cuda)
    with pytest.raises(G.InvalidOperationError):
        pool.rope_append(0, q, k, k, [0, 1], 4)  # nothing uploaded
    pool.upload_step(np.zeros((1, 1), np.int32), np.zeros(1, np.int32), np.array([0, 1], np.int64))
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.rope_append(0, q, k, k, [0, -1], 4)  # negative position
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.rope_append(0, q, k, k, [0, 1], 4, rope_dim=7)
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.rope_append(0, q, k, k, [0, 1], 3)  # heads not a multiple of heads_kv
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.rope_append(1, q, k, k, [0, 1], 4)  # layer
    pool.close()
    odd = G.PagedBlockPool(8, 1, 1, 96, 16)
    q96 = torch.zeros((1, 1, 96), device=cuda)
    odd.upload_step(np.zeros((1, 1), np.int32), np.zeros(1, np.int32), np.array([0], np.int64))
    with pytest.raises(G.UnsupportedError):
        odd.rope_append(0, q96, q96, q96, [0], 1)
    odd.close()
