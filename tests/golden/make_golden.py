"""Generates the committed golden fixtures of tests/golden/.

    python tests/golden/make_golden.py

1. kat_compute_attention.json -- the closed-form case of the reference's own test
   PagedAttentionTests.ComputeAttention_HeadDim128_AccumulatesAccurately
   (tests/Glacier.Serve.Tests/PagedAttentionTests.cs:112-179): d=128, block 16, 32 tokens,
   4 query / 2 kv heads, K[t] = 0.01f*(t+1) (fp32 product, as in C#), V = (t+1) for kv head 0
   and 2(t+1) for kv head 1, Q = 1, scale = 1/sqrt(128).  The expected outputs are evaluated
   here in float64 from those fp32 inputs; the reference test itself only asserts positivity
   and per-head uniformity, so these numbers pin the closed form, not the C# bits.
2. store_retrieve.json -- PagedAttentionTests.cs:82-109 (Store at layer 1, slot 2).
3. decode_small_*.npz -- small seeded decode cases (inputs + CPU-oracle outputs) that pin the
   oracle against drift; the GPU parity tests recompute the oracle at run time.
"""
import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def kat():
    d, T, nH, nKv = 128, 32, 4, 2
    scale32 = np.float32(1.0) / np.float32(math.sqrt(d))
    kval = np.array([np.float32(0.01) * np.float32(t + 1) for t in range(T)], np.float32)
    out = np.zeros((nH,), np.float64)
    for h in range(nH):
        kv = h // (nH // nKv)
        c = 1.0 if kv == 0 else 2.0
        s = np.array([float(kval[t]) * d * float(scale32) for t in range(T)], np.float64)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = float(np.sum(p * c * np.arange(1, T + 1)))
    return {
        "source": "tests/Glacier.Serve.Tests/PagedAttentionTests.cs:112-179",
        "head_dim": d, "block_size": 16, "tokens": T, "n_heads": nH, "n_heads_kv": nKv,
        "k_value_per_token": [float(x) for x in kval], "v_scale_per_kv_head": [1.0, 2.0],
        "q_value": 1.0, "attn_scale": float(scale32),
        "expected_per_head": [float(x) for x in out],
        "note": "every output dim of head h equals expected_per_head[h]",
    }


def store_retrieve():
    return {
        "source": "tests/Glacier.Serve.Tests/PagedAttentionTests.cs:82-109",
        "total_blocks": 4, "layers": 2, "heads_kv": 2, "head_dim": 4, "block_size": 4,
        "layer": 1, "slot": 2,
        "k": [1, 2, 3, 4, 5, 6, 7, 8], "v": [10, 20, 30, 40, 50, 60, 70, 80],
    }


def decode_cases():
    from oracle import pyoracle as O

    cases = []
    rng = np.random.default_rng(20261201)
    for name, (nH, nKv, d, dv, bs, dtype, ctxs) in {
        "gqa4_d32_bs16_f32": (4, 2, 32, 32, 16, O.F32, [1, 15, 16, 17, 40]),
        "gqa7_d128_bs16_f32": (7, 1, 128, 128, 16, O.F32, [33, 100]),
        "mha_d64_bs4_bf16": (2, 2, 64, 64, 4, O.BF16, [5, 9, 0]),
        "asym_d32_dv64_bs8_f32": (2, 1, 32, 64, 8, O.F32, [20, 7]),
    }.items():
        mb = max(1, max((c + bs - 1) // bs for c in ctxs))
        total = len(ctxs) * mb + 3
        g = O.geom(total, 1, nKv, d, dv, bs, dtype)
        K, V = O.new_arena(g)
        kf = rng.standard_normal(K.shape).astype(np.float32)
        vf = rng.standard_normal(V.shape).astype(np.float32)
        if dtype == O.BF16:
            K[...] = O.f32_to_bf16_bits(kf)
            V[...] = O.f32_to_bf16_bits(vf)
        else:
            K[...] = kf
            V[...] = vf
        perm = rng.permutation(total).astype(np.int32)
        tables = np.full((len(ctxs), mb), -1, np.int32)
        for i, c in enumerate(ctxs):
            n = (c + bs - 1) // bs
            tables[i, :n] = perm[i * mb: i * mb + n]
        q = rng.standard_normal((len(ctxs), nH, d)).astype(np.float32)
        scale = 1.0 / math.sqrt(d)
        out = O.decode_batch(K, V, g, 0, tables, np.array(ctxs, np.int32), q, nH, scale)
        path = os.path.join(HERE, f"decode_small_{name}.npz")
        np.savez_compressed(path, K=K, V=V, tables=tables, ctx=np.array(ctxs, np.int32), q=q, out=out,
                            geom=np.array([total, 1, nKv, d, dv, bs, dtype], np.int32),
                            n_heads=nH, scale=np.float32(scale))
        cases.append(path)
    return cases


if __name__ == "__main__":
    with open(os.path.join(HERE, "kat_compute_attention.json"), "w") as f:
        json.dump(kat(), f, indent=1)
    with open(os.path.join(HERE, "store_retrieve.json"), "w") as f:
        json.dump(store_retrieve(), f, indent=1)
    for p in decode_cases():
        print("wrote", os.path.relpath(p, ROOT))
