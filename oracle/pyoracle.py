"""ctypes wrapper of oracle/lib/libgkv_oracle.so (TEST INFRASTRUCTURE ONLY).

numpy in, numpy out.  Arena arrays are host copies in the device layout
[block][layer][head_kv][slot][dim], float32 or bf16 bit patterns (uint16).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_DIR, "lib", "libgkv_oracle.so")


def build() -> None:
    subprocess.run(["make", "-s", "-C", _DIR], check=True)


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        build()
    lib = C.CDLL(LIB_PATH)
    P, I, F = C.c_void_p, C.c_int32, C.c_float
    lib.oracle_f32_to_bf16.restype = C.c_uint16
    lib.oracle_f32_to_bf16.argtypes = [F]
    lib.oracle_bf16_to_f32.restype = F
    lib.oracle_bf16_to_f32.argtypes = [C.c_uint16]
    lib.oracle_f32_to_f16.restype = C.c_uint16
    lib.oracle_f32_to_f16.argtypes = [F]
    lib.oracle_f16_to_f32.restype = F
    lib.oracle_f16_to_f32.argtypes = [C.c_uint16]
    lib.oracle_f32_to_f16_many.restype = None
    lib.oracle_f32_to_f16_many.argtypes = [P, P, C.c_int64]
    lib.oracle_f32_to_e4m3.restype = C.c_uint8
    lib.oracle_f32_to_e4m3.argtypes = [F]
    lib.oracle_e4m3_to_f32.restype = F
    lib.oracle_e4m3_to_f32.argtypes = [C.c_uint8]
    lib.oracle_f32_to_e4m3_many.restype = None
    lib.oracle_f32_to_e4m3_many.argtypes = [P, P, C.c_int64]
    lib.oracle_store.argtypes = [P, P, P, I, I, I, P, P]
    lib.oracle_copy_block_data.argtypes = [P, P, P, I, I, I]
    lib.oracle_store_many.argtypes = [P, P, P, I, P, I, P, P]
    lib.oracle_copy_many.argtypes = [P, P, P, P, P, P, I]
    lib.oracle_compute_attention.argtypes = [P, P, P, I, I, P, P, P, I, I, I, I, I, I, F, P, I, I, F, I]
    lib.oracle_decode_batch.argtypes = [P, P, P, I, P, I, I, P, P, P, I, F, I, F, I]
    lib.oracle_decode_batch_parallel.argtypes = [P, P, P, I, P, I, I, P, P, P, I, F, I]
    lib.oracle_prefill_chunk.argtypes = [P, P, P, I, P, I, I, I, I, P, P, I, F, I]
    lib.oracle_max_threads.restype = C.c_int
    lib.oracle_sincos.restype = None
    lib.oracle_sincos.argtypes = [F, C.POINTER(F), C.POINTER(F)]
    lib.oracle_rope_append.restype = C.c_int
    lib.oracle_rope_append.argtypes = [P, P, P, I, P, P, P, I, I, P, P, P, I, I, F, P, P, P, P, P, F]
    for n in ("oracle_store", "oracle_copy_block_data", "oracle_store_many", "oracle_copy_many",
              "oracle_compute_attention",
              "oracle_decode_batch", "oracle_decode_batch_parallel", "oracle_prefill_chunk"):
        getattr(lib, n).restype = C.c_int
    return lib


lib = _load()

F32, BF16, F16, FP8 = 0, 1, 2, 3


class Geom(C.Structure):
    _fields_ = [(n, C.c_int32) for n in
                ("total_blocks", "layers", "heads_kv", "head_dim", "v_head_dim", "block_size", "dtype")] + [
        ("k_scale", C.c_void_p), ("v_scale", C.c_void_p)]

    def set_scales(self, k_scale, v_scale):
        """FP8 arenas: [layers][heads_kv] K and V scales (kept alive with the geometry)."""
        self._ks = np.ascontiguousarray(k_scale, np.float32)
        self._vs = np.ascontiguousarray(v_scale, np.float32)
        self.k_scale = self._ks.ctypes.data
        self.v_scale = self._vs.ctypes.data
        return self


def geom(total_blocks, layers, heads_kv, head_dim, v_head_dim=None, block_size=16, dtype=F32) -> Geom:
    return Geom(total_blocks, layers, heads_kv, head_dim, v_head_dim or head_dim, block_size, dtype)


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "arrays must be C-contiguous"
    return a.ctypes.data


def new_arena(g: Geom):
    kshape = (g.total_blocks, g.layers, g.heads_kv, g.block_size, g.head_dim)
    vshape = (g.total_blocks, g.layers, g.heads_kv, g.block_size, g.v_head_dim)
    dt = {F32: np.float32, BF16: np.uint16, F16: np.uint16, FP8: np.uint8}[g.dtype]
    return np.zeros(kshape, dt), np.zeros(vshape, dt)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (vectorised restatement of
    oracle_f32_to_bf16; tests check the two agree)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bit patterns through the oracle's own round-to-nearest-even conversion."""
    src = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(src.shape, np.uint16)
    lib.oracle_f32_to_f16_many(_p(src), _p(out), src.size)
    return out


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> FP8 E4M3 bytes through the oracle's round-to-nearest-even, saturating conversion."""
    src = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(src.shape, np.uint8)
    lib.oracle_f32_to_e4m3_many(_p(src), _p(out), src.size)
    return out


_E4M3 = None


def e4m3_bits_to_f32(b: np.ndarray) -> np.ndarray:
    global _E4M3
    if _E4M3 is None:
        _E4M3 = np.array([lib.oracle_e4m3_to_f32(i) for i in range(256)], np.float32)
    return _E4M3[np.asarray(b, dtype=np.uint8)]


def to_storage_bits(x: np.ndarray, dtype: int) -> np.ndarray:
    """fp32 values in an arena's storage representation (F32: unchanged; FP8 with scale 1)."""
    if dtype == BF16:
        return f32_to_bf16_bits(x)
    if dtype == F16:
        return f32_to_f16_bits(x)
    if dtype == FP8:
        return f32_to_e4m3_bits(x)
    return np.ascontiguousarray(x, dtype=np.float32)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def store(K, V, g: Geom, block, layer, slot, k: np.ndarray, v: np.ndarray) -> int:
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    return lib.oracle_store(_p(K), _p(V), C.byref(g), block, layer, slot, _p(k), _p(v))


def copy_block_data(K, V, g: Geom, src, dst, valid) -> int:
    return lib.oracle_copy_block_data(_p(K), _p(V), C.byref(g), src, dst, valid)


def store_many(K, V, g: Geom, layer, slots: np.ndarray, k: np.ndarray, v: np.ndarray) -> int:
    slots = np.ascontiguousarray(slots, np.int64)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    return lib.oracle_store_many(_p(K), _p(V), C.byref(g), layer, _p(slots), int(slots.size), _p(k), _p(v))


def copy_many(K, V, g: Geom, src, dst, valid) -> int:
    src = np.ascontiguousarray(src, np.int32)
    dst = np.ascontiguousarray(dst, np.int32)
    valid = np.ascontiguousarray(valid, np.int32)
    return lib.oracle_copy_many(_p(K), _p(V), C.byref(g), _p(src), _p(dst), _p(valid), int(src.size))


def compute_attention(K, V, g: Geom, stage_layer, pos, q, block_ids, token_count, n_heads, n_heads_kv,
                      head_dim, v_head_dim, attn_scale, max_seq_len, sink_logit=None, n_threads=0):
    """Returns (rc, out[n_heads, v_head_dim])."""
    q = np.ascontiguousarray(q, np.float32)
    ids = np.ascontiguousarray(np.asarray(block_ids, np.int32))
    out = np.zeros((n_heads, v_head_dim), np.float32)
    scratch = np.zeros(max(n_heads * max(max_seq_len, 1), 1), np.float32)
    rc = lib.oracle_compute_attention(
        _p(K), _p(V), C.byref(g), stage_layer, pos, _p(q), _p(out), _p(ids) if ids.size else None,
        ids.size, token_count, n_heads, n_heads_kv, head_dim, v_head_dim, attn_scale, _p(scratch),
        max_seq_len, 0 if sink_logit is None else 1, float(sink_logit or 0.0), n_threads)
    return rc, out


def decode_batch(K, V, g: Geom, layer, tables, ctx_lens, q, n_heads, scale, sink_logit=None,
                 n_threads=0, out=None, parallel=False):
    tables = np.ascontiguousarray(tables, np.int32)
    ctx = np.ascontiguousarray(ctx_lens, np.int32)
    q = np.ascontiguousarray(q, np.float32)
    B = tables.shape[0]
    if out is None:
        out = np.zeros((B, n_heads, g.v_head_dim), np.float32)
    if parallel:
        assert sink_logit is None
        rc = lib.oracle_decode_batch_parallel(_p(K), _p(V), C.byref(g), layer, _p(tables), B, tables.shape[1],
                                              _p(ctx), _p(q), _p(out), n_heads, scale, n_threads)
    else:
        rc = lib.oracle_decode_batch(_p(K), _p(V), C.byref(g), layer, _p(tables), B, tables.shape[1], _p(ctx),
                                     _p(q), _p(out), n_heads, scale, 0 if sink_logit is None else 1,
                                     float(sink_logit or 0.0), n_threads)
    if rc != 0:
        raise ValueError(f"oracle_decode_batch failed ({rc})")
    return out


def prefill_chunk(K, V, g: Geom, layer, block_ids, token_count, start_pos, q, n_heads, scale, n_threads=0):
    ids = np.ascontiguousarray(np.asarray(block_ids, np.int32))
    q = np.ascontiguousarray(q, np.float32)
    n_q = q.shape[0]
    out = np.zeros((n_q, n_heads, g.v_head_dim), np.float32)
    rc = lib.oracle_prefill_chunk(_p(K), _p(V), C.byref(g), layer, _p(ids), ids.size, token_count, start_pos,
                                  n_q, _p(q), _p(out), n_heads, scale, n_threads)
    if rc != 0:
        raise ValueError(f"oracle_prefill_chunk failed ({rc})")
    return out


def max_threads() -> int:
    """OpenMP's default team size (honours OMP_NUM_THREADS)."""
    return lib.oracle_max_threads()


def host_cores() -> int:
    """Host cores this process may run on, whatever OMP_NUM_THREADS says (a torchrun launch sets
    it to 1): the thread count the timed CPU baseline passes explicitly."""
    import os

    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def sincos(theta: float):
    s, c = C.c_float(), C.c_float()
    lib.oracle_sincos(float(theta), C.byref(s), C.byref(c))
    return s.value, c.value


def rope_append(K, V, g: Geom, layer, q, k, v, positions, slots, inv_freq, rope_dim, style=0, mscale=1.0,
                q_bias=None, k_bias=None, v_bias=None, q_norm=None, k_norm=None, eps=1e-6):
    """Restated prologue + Store (PagedTransformerRunner.cs:612-634); returns the rewritten q."""
    q = np.array(q, dtype=np.float32, copy=True, order="C")
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    positions = np.ascontiguousarray(positions, np.int32)
    slots = np.ascontiguousarray(slots, np.int64)
    inv_freq = np.ascontiguousarray(inv_freq, np.float32)
    terms = [None if a is None else np.ascontiguousarray(a, np.float32)
             for a in (q_bias, k_bias, v_bias, q_norm, k_norm)]  # kept alive across the call
    ptrs = [None if a is None else _p(a) for a in terms]
    rc = lib.oracle_rope_append(_p(K), _p(V), C.byref(g), layer, _p(q), _p(k), _p(v), int(positions.size),
                                int(q.shape[1]), _p(positions), _p(slots), _p(inv_freq), rope_dim, style,
                                float(mscale), *ptrs, float(eps))
    if rc != 0:
        raise ValueError(f"oracle_rope_append failed ({rc})")
    return q
