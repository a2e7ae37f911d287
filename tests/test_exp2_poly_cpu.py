"""The FMA-pipe 2^x of the prefill softmax (exp2_fma2 in csrc/gkv_device.cuh) on the CPU: its steps
evaluated in fp32 with the constants read from the source, against double-precision 2^x.  The GPU
result is covered end to end by the prefill parity tests."""
import os
import re

import numpy as np

from conftest import ROOT


def _coeffs():
    src = open(os.path.join(ROOT, "glacier.serve_b200", "csrc", "gkv_device.cuh")).read()
    body = src[src.index("float2 exp2_fma2(float2 e)"):]
    body = body[: body.index("return __fmul2_rn")]
    return [float(x) for x in re.findall(r"make_float2\((0\.\d+)f, \1f\)", body)]


def _exp2_fma(e):
    f32 = np.float32
    c = [f32(x) for x in _coeffs()]  # highest degree first
    assert len(c) == 5
    e = np.maximum(e.astype(f32), f32(-127))
    t = (e + f32(12582912.0)).astype(f32)
    n = (t - f32(12582912.0)).astype(f32)
    fr = (e - n).astype(f32)
    p = np.full_like(fr, c[0])
    for k in c[1:]:  # fused multiply-add: exact product, one rounding (float64 holds the product)
        p = (p.astype(np.float64) * fr.astype(np.float64) + np.float64(k)).astype(f32)
    bits = ((t.view(np.int32) - 0x4B400000 + 127) << 23).astype(np.int32)
    return (p * bits.view(f32)).astype(f32)


def test_exp2_fma_relative_error_and_underflow():
    e = np.concatenate([np.linspace(-126, 8, 2_000_001), np.arange(-126, 9, 0.5)]).astype(np.float32)
    got = _exp2_fma(e).astype(np.float64)
    want = np.exp2(e.astype(np.float64))
    assert np.max(np.abs(got - want) / want) <= 4e-6
    low = np.array([-127, -127.5, -200, -np.inf], np.float32)
    assert (_exp2_fma(low) == 0).all()
