"""Python face of the B200 paged-KV shim (libglacier_kv.so).

Mirrors the reference's C# surface so callers and tests read like the reference's own:
``PagedBlockPool`` (src/Glacier.Serve/Inference/PagedAttention/PagedBlockPool.cs),
``BlockTable`` (BlockTable.cs) and ``PagedAttentionKernel.compute_attention``
(PagedAttentionKernel.cs:17), plus the batched step API that replaces the runners'
per-sequence loops.  ``ArgumentOutOfRangeError`` / ``InvalidOperationError`` are raised
where the reference throws ArgumentOutOfRangeException / InvalidOperationException.

Every call goes through the C ABI; device work runs in the sm_100a kernels of the shim.
Device tensors are torch CUDA tensors (plumbing only); host arrays may be numpy arrays.
"""
from __future__ import annotations

import ctypes as C
from typing import Iterable, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from ._lib import (DTYPES, GKV_DTYPE_BF16, GKV_DTYPE_F16, GKV_DTYPE_F32, GKV_DTYPE_FP8_E4M3, GKV_EDEVICE, GKV_EINVAL, GKV_ESTATE,
                   GKV_ETIMEDOUT, GKV_EUNSUPPORTED, GKV_OK, LIB_PATH, last_error, lib)

GKV_ROPE_NEOX, GKV_ROPE_INTERLEAVED = 0, 1

__all__ = [
    "PagedBlockPool", "BlockTable", "PagedAttentionKernel", "GkvError",
    "ArgumentOutOfRangeError", "InvalidOperationError", "DeviceError", "TimeoutError_",
    "UnsupportedError", "partition_lpt", "split_block_range", "plan_decode", "LIB_PATH", "version",
]


class GkvError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class ArgumentOutOfRangeError(GkvError, ValueError):
    """GKV_EINVAL: the reference throws ArgumentOutOfRangeException / ArgumentException."""


class InvalidOperationError(GkvError):
    """GKV_ESTATE: the reference throws InvalidOperationException."""


class DeviceError(GkvError):
    """GKV_EDEVICE: a kernel flagged a bad block id / slot or an expired bounded wait."""


class TimeoutError_(GkvError):
    """GKV_ETIMEDOUT: gkv_sync gave up waiting."""


class UnsupportedError(GkvError):
    """GKV_EUNSUPPORTED: shape not compiled into this build."""


_ERRORS = {
    GKV_EINVAL: ArgumentOutOfRangeError,
    GKV_ESTATE: InvalidOperationError,
    GKV_EDEVICE: DeviceError,
    GKV_ETIMEDOUT: TimeoutError_,
    GKV_EUNSUPPORTED: UnsupportedError,
}


def _check(rc: int) -> int:
    if rc < 0:
        raise _ERRORS.get(rc, GkvError)(rc, last_error())
    return rc


def version() -> str:
    return lib.gkv_version().decode()


def _ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("host array must be C-contiguous")
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return x.data_ptr()
    raise TypeError(f"cannot take a pointer of {type(x)!r}")


def _stream(stream, device: int) -> Optional[int]:
    if stream is None:
        import torch

        if torch.cuda.is_available():
            return torch.cuda.current_stream(device).cuda_stream
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _f32_dev(t, name: str):
    import torch

    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor")
    return t.data_ptr()


class _CudaArray:
    """__cuda_array_interface__ wrapper so torch can view the device arena in place."""

    def __init__(self, ptr: int, shape: Tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3,
            "strides": None,
        }


class PagedBlockPool:
    """Device block arena + host-mirrored free list (PagedBlockPool.cs:16).

    ``allocate_device_arena=False`` is the reference's metadata-only pool
    (``allocateHostBuffers: false``, PagedBlockPool.cs:61): allocator, prefix cache and CoW
    bookkeeping without touching CUDA.
    """

    DEFAULT_BLOCK_SIZE = 16

    def __init__(self, total_blocks: int, layers: int, heads_kv: int, head_dim: int,
                 block_size: int = DEFAULT_BLOCK_SIZE, v_head_dim: int = -1,
                 allocate_device_arena: bool = True, device: int = 0, dtype: str = "f32"):
        d = _lib.gkv_pool_desc()
        d.device = device
        d.total_blocks = total_blocks
        d.layers = layers
        d.heads_kv = heads_kv
        d.head_dim = head_dim
        d.v_head_dim = v_head_dim
        d.block_size = block_size
        d.dtype = DTYPES[dtype]
        d.allocate_device_arena = 1 if allocate_device_arena else 0
        h = C.c_void_p()
        _check(lib.gkv_pool_create(C.byref(d), C.byref(h)))
        self._h = h
        self.device = device
        self.dtype = dtype
        self._layers = layers
        self._heads_kv = heads_kv
        self._head_dim = head_dim
        self._v_head_dim = v_head_dim if v_head_dim > 0 else head_dim

    # ---- lifetime ----
    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.gkv_pool_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    # ---- counters, PagedBlockPool.cs:46-59 ----
    def stats(self) -> _lib.gkv_pool_stats:
        s = _lib.gkv_pool_stats()
        _check(lib.gkv_pool_stats_get(self._h, C.byref(s)))
        return s

    total_blocks = property(lambda self: self.stats().total_blocks)
    block_size = property(lambda self: self.stats().block_size)
    layers = property(lambda self: self._layers)
    heads_kv = property(lambda self: self._heads_kv)
    head_dim = property(lambda self: self._head_dim)
    value_head_dim = property(lambda self: self._v_head_dim)
    free_blocks_count = property(lambda self: self.stats().free_blocks)
    allocated_blocks_count = property(lambda self: self.stats().allocated_blocks)
    capacity_tokens = property(lambda self: self.stats().capacity_tokens)
    active_tokens = property(lambda self: self.stats().active_tokens)
    has_device_arena = property(lambda self: bool(self.stats().has_device_arena))
    total_memory_bytes = property(lambda self: self.stats().total_memory_bytes)
    pending_copies = property(lambda self: self.stats().pending_copies)

    def _kv_ptrs(self) -> Tuple[int, int]:
        k, v = C.c_void_p(), C.c_void_p()
        _check(lib.gkv_pool_kv_ptrs(self._h, C.byref(k), C.byref(v)))
        return k.value or 0, v.value or 0

    @property
    def key_buffer_address(self) -> int:
        return self._kv_ptrs()[0]

    @property
    def value_buffer_address(self) -> int:
        return self._kv_ptrs()[1]

    def element_offset(self, which: int, block: int, layer: int, head_kv: int, slot: int) -> int:
        """GetKeyPtr (which=0) / GetValuePtr (which=1) offsets, PagedBlockPool.cs:124-145."""
        out = C.c_int64()
        _check(lib.gkv_pool_element_offset(self._h, which, block, layer, head_kv, slot, C.byref(out)))
        return out.value

    def set_kv_scales(self, k_scales, v_scales) -> None:
        """FP8 pools: the [layers][heads_kv] K and V scales (an element reads back as
        e4m3 * scale and is stored as e4m3(x / scale)).  Set them before the first append."""
        n = self._layers * self._heads_kv
        ks = np.ascontiguousarray(np.asarray(k_scales, np.float32).reshape(-1))
        vs = np.ascontiguousarray(np.asarray(v_scales, np.float32).reshape(-1))
        if ks.size != n or vs.size != n:
            raise ArgumentOutOfRangeError(GKV_EINVAL, f"scales need {n} values each")
        pf = C.POINTER(C.c_float)
        _check(lib.gkv_pool_set_kv_scales(self._h, ks.ctypes.data_as(pf), vs.ctypes.data_as(pf)))
        self._kv_scales = (ks.reshape(self._layers, self._heads_kv).copy(), vs.reshape(self._layers, self._heads_kv).copy())

    @property
    def kv_scales(self):
        """The FP8 pool's ([layers][heads_kv] K, V) scales as last set (ones by default)."""
        ones = np.ones((self._layers, self._heads_kv), np.float32)
        return getattr(self, "_kv_scales", (ones, ones))

    def key_view(self):
        """torch view [blocks][layers][heads_kv][block_size][head_dim] of the K arena (uint8
        bytes for an FP8 pool, e4m3 bit patterns)."""
        return self._view(self._kv_ptrs()[0], self._head_dim)

    def value_view(self):
        return self._view(self._kv_ptrs()[1], self._v_head_dim)

    def _view(self, ptr: int, dim: int):
        import torch

        if not ptr:
            raise InvalidOperationError(GKV_ESTATE, "Host KV buffers were omitted.")
        shape = (self.total_blocks, self._layers, self._heads_kv, self.block_size, dim)
        if self.dtype == "fp8":
            return torch.as_tensor(_CudaArray(ptr, shape, "|u1"), device=f"cuda:{self.device}")
        if self.dtype in ("bf16", "f16"):
            t = torch.as_tensor(_CudaArray(ptr, shape, "<i2"), device=f"cuda:{self.device}")
            return t.view(torch.bfloat16 if self.dtype == "bf16" else torch.float16)
        return torch.as_tensor(_CudaArray(ptr, shape, "<f4"), device=f"cuda:{self.device}")

    # ---- allocator, PagedBlockPool.cs:178-353 ----
    def try_allocate_block(self) -> Tuple[bool, int]:
        out = C.c_int32()
        ok = _check(lib.gkv_pool_try_allocate_block(self._h, C.byref(out)))
        return bool(ok), out.value

    def release_block(self, block: int) -> int:
        return _check(lib.gkv_pool_release_block(self._h, block))

    def free_block(self, block: int) -> None:
        _check(lib.gkv_pool_free_block(self._h, block))

    def free_blocks(self, blocks: Iterable[int]) -> None:
        arr = np.ascontiguousarray(np.asarray(list(blocks), dtype=np.int32))
        _check(lib.gkv_pool_free_blocks(self._h, _ptr(arr), arr.size))

    def retain_block(self, block: int) -> int:
        return _check(lib.gkv_pool_retain_block(self._h, block))

    def get_ref_count(self, block: int) -> int:
        return _check(lib.gkv_pool_get_ref_count(self._h, block))

    def try_find_prefix_block(self, prefix_hash: int) -> Tuple[bool, int]:
        out = C.c_int32()
        ok = _check(lib.gkv_pool_try_find_prefix_block(self._h, prefix_hash & (2**64 - 1), C.byref(out)))
        return bool(ok), out.value

    def bind_prefix_block(self, prefix_hash: int, block: int) -> None:
        _check(lib.gkv_pool_bind_prefix_block(self._h, prefix_hash & (2**64 - 1), block))

    def try_fork_block(self, src_block: int, valid_tokens: int) -> Tuple[bool, int]:
        out = C.c_int32()
        ok = _check(lib.gkv_pool_try_fork_block(self._h, src_block, valid_tokens, C.byref(out)))
        return bool(ok), out.value

    def flush_copies(self, stream=None) -> None:
        _check(lib.gkv_pool_flush_copies(self._h, _stream(stream, self.device) if self.has_device_arena else None))

    def copy_block_data(self, src: int, dst: int, valid_tokens: int, stream=None) -> None:
        """CopyBlockData, PagedBlockPool.cs:304-327 (one op of the batched block copy)."""
        self.block_copy([src], [dst], [valid_tokens], stream)

    def block_copy(self, srcs: Sequence[int], dsts: Sequence[int], valids: Sequence[int], stream=None) -> None:
        s = np.ascontiguousarray(np.asarray(srcs, dtype=np.int32))
        d = np.ascontiguousarray(np.asarray(dsts, dtype=np.int32))
        v = np.ascontiguousarray(np.asarray(valids, dtype=np.int32))
        if not (s.size == d.size == v.size):
            raise ValueError("srcs/dsts/valids differ in length")
        _check(lib.gkv_block_copy(self._h, _ptr(s), _ptr(d), _ptr(v), s.size,
                                  _stream(stream, self.device) if self.has_device_arena else None))

    def store(self, block: int, layer: int, slot: int, k, v, stream=None) -> None:
        """Store, PagedBlockPool.cs:151-161: k [heads_kv*head_dim], v [heads_kv*v_head_dim]
        float32 CUDA tensors."""
        if not self.has_device_arena:
            _check(lib.gkv_pool_store(self._h, block, layer, slot, None, None, None))
        _check(lib.gkv_pool_store(self._h, block, layer, slot, _f32_dev(k, "k"), _f32_dev(v, "v"),
                                  _stream(stream, self.device)))

    def compact(self, tables: Sequence["BlockTable"], max_moves: int = 0, stream=None) -> Tuple[np.ndarray, np.ndarray]:
        """gkv_pool_compact: moves live blocks held only by `tables` into the lowest free ids
        (one batched block copy), rewrites the tables; returns the moves (src ids, dst ids)."""
        arr = (C.c_void_p * max(len(tables), 1))(*[t.handle.value for t in tables])
        cap = max_moves if max_moves > 0 else self.total_blocks
        src = np.zeros(max(cap, 1), np.int32)
        dst = np.zeros(max(cap, 1), np.int32)
        n = _check(lib.gkv_pool_compact(self._h, arr, len(tables), max_moves, _ptr(src), _ptr(dst), cap,
                                        _stream(stream, self.device) if self.has_device_arena else None))
        return src[:n], dst[:n]

    # ---- batched step ----
    def reserve_step(self, max_batch: int, max_blocks_per_seq: int, max_tokens: int, n_heads: int) -> None:
        _check(lib.gkv_step_reserve(self._h, max_batch, max_blocks_per_seq, max_tokens, n_heads))

    def set_static_step(self, enable: bool = True) -> None:
        """gkv_step_set_static: fixed-address step metadata read on the device, so that the
        per-layer kv_append + paged_decode launches can be captured once in a CUDA graph and
        replayed after every upload_step on the same stream (reserve_step first)."""
        _check(lib.gkv_step_set_static(self._h, 1 if enable else 0))

    def upload_step(self, block_tables: np.ndarray, ctx_lens: np.ndarray,
                    slot_mapping: Optional[np.ndarray] = None, stream=None) -> None:
        bt = np.ascontiguousarray(block_tables, dtype=np.int32)
        if bt.ndim != 2:
            raise ValueError("block_tables must be [batch, max_blocks]")
        cl = np.ascontiguousarray(ctx_lens, dtype=np.int32)
        sm = np.ascontiguousarray(slot_mapping if slot_mapping is not None else np.zeros(0), dtype=np.int64)
        if cl.shape != (bt.shape[0],):
            raise ValueError("ctx_lens must be [batch]")
        self._uploaded = (bt, cl, sm)  # keep host memory alive until the copy is enqueued
        _check(lib.gkv_upload_step(self._h, _ptr(bt), bt.shape[0], bt.shape[1], _ptr(cl), _ptr(sm),
                                   sm.size, _stream(stream, self.device)))

    def upload_step_tables(self, tables: Sequence["BlockTable"], ctx_lens=None, slot_mapping=None,
                           stream=None) -> None:
        arr = (C.c_void_p * len(tables))(*[t.handle.value for t in tables])
        cl = None if ctx_lens is None else np.ascontiguousarray(ctx_lens, dtype=np.int32)
        sm = np.ascontiguousarray(slot_mapping if slot_mapping is not None else np.zeros(0), dtype=np.int64)
        _check(lib.gkv_upload_step_tables(self._h, arr, len(tables), _ptr(cl), _ptr(sm), sm.size,
                                          _stream(stream, self.device)))

    def kv_append(self, layer: int, k, v, stream=None) -> None:
        """k [n_tok, heads_kv, head_dim], v [n_tok, heads_kv, v_head_dim] float32 CUDA."""
        n = k.shape[0]
        _check(lib.gkv_kv_append(self._h, layer, _f32_dev(k, "k"), _f32_dev(v, "v"), n,
                                 _stream(stream, self.device)))

    def rope_append(self, layer: int, q, k, v, positions, n_heads: int, rope_dim: int = 0, style: int = 0,
                    freq_base: float = 10000.0, inv_freq=None, freq_factors=None, mscale: float = 1.0,
                    q_bias=None, k_bias=None, v_bias=None, q_norm=None, k_norm=None, eps: float = 1e-6,
                    stream=None) -> None:
        """Bias + per-head RMSNorm + RoPE of q and k, then the append of k and v into the uploaded
        step's slots (gkv_rope_append).  q [n_tok, n_heads, head_dim] float32 CUDA is rewritten
        in place; k, v float32 CUDA; positions a host int array [n_tok]; inv_freq / freq_factors
        host float arrays [rope_dim/2] or None; biases and norm weights float32 CUDA or None."""
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        inv = None if inv_freq is None else np.ascontiguousarray(inv_freq, dtype=np.float32)
        fac = None if freq_factors is None else np.ascontiguousarray(freq_factors, dtype=np.float32)
        rd = _lib.gkv_rope_desc(rope_dim, style, float(freq_base), float(mscale), _ptr(inv), _ptr(fac))
        opt = lambda t, n: None if t is None else _f32_dev(t, n)  # noqa: E731
        pro = _lib.gkv_qkv_prologue(opt(q_bias, "q_bias"), opt(k_bias, "k_bias"), opt(v_bias, "v_bias"),
                                    opt(q_norm, "q_norm"), opt(k_norm, "k_norm"), float(eps))
        _check(lib.gkv_rope_append(self._h, layer, _f32_dev(q, "q"), _f32_dev(k, "k"), _f32_dev(v, "v"),
                                   int(pos.size), n_heads, _ptr(pos), C.byref(rd), C.byref(pro),
                                   _stream(stream, self.device)))

    def paged_decode(self, layer: int, q, out, n_heads: int, scale: float, sinks=None, stream=None) -> None:
        """q [batch, n_heads, head_dim] -> out [batch, n_heads, v_head_dim] float32 CUDA."""
        _check(lib.gkv_paged_decode(self._h, layer, _f32_dev(q, "q"), _f32_dev(out, "out"), n_heads,
                                    float(scale), None if sinks is None else _f32_dev(sinks, "sinks"),
                                    _stream(stream, self.device)))

    def paged_prefill(self, layer: int, q, out, q_start, q_len, n_heads: int, scale: float, stream=None) -> None:
        """Chunked causal prefill of the uploaded step: q [sum q_len, n_heads, head_dim] float32 or
        bfloat16 CUDA, packed by sequence; out [sum q_len, n_heads, v_head_dim] float32.  Query t
        of sequence b sits at position q_start[b] + t and attends keys
        [0, min(ctx_lens[b], q_start[b] + t + 1))."""
        import torch

        qdt = {torch.float32: GKV_DTYPE_F32, torch.bfloat16: GKV_DTYPE_BF16, torch.float16: GKV_DTYPE_F16}
        if not (isinstance(q, torch.Tensor) and q.is_cuda and q.is_contiguous() and q.dtype in qdt):
            raise ValueError("q must be a contiguous float32, bfloat16 or float16 CUDA tensor")
        qs = np.ascontiguousarray(q_start, dtype=np.int32)
        ql = np.ascontiguousarray(q_len, dtype=np.int32)
        qd = qdt[q.dtype]
        _check(lib.gkv_paged_prefill(self._h, layer, q.data_ptr(), qd, _f32_dev(out, "out"), _ptr(qs), _ptr(ql),
                                     n_heads, float(scale), _stream(stream, self.device)))

    def decode_step_host(self, layer: int, block_tables, ctx_lens, slot_mapping, k_new, v_new, q, out,
                         n_heads: int, scale: float, sinks=None, stream=None) -> None:
        """One append+decode iteration from host buffers (pinned torch tensors or numpy)."""
        bt = np.ascontiguousarray(block_tables, dtype=np.int32)
        cl = np.ascontiguousarray(ctx_lens, dtype=np.int32)
        sm = np.ascontiguousarray(slot_mapping, dtype=np.int64)
        self._uploaded = (bt, cl, sm)
        _check(lib.gkv_decode_step_host(
            self._h, layer, _ptr(bt), bt.shape[0], bt.shape[1], _ptr(cl), _ptr(sm), sm.size,
            _ptr(k_new), _ptr(v_new), _ptr(q), _ptr(out), n_heads, float(scale),
            None if sinks is None else _f32_dev(sinks, "sinks"), _stream(stream, self.device)))

    def wait_host_outputs(self, stream=None) -> None:
        """Orders `stream` after the output copies of every decode_step_host call so far."""
        _check(lib.gkv_wait_host_outputs(self._h, _stream(stream, self.device)))

    def paged_decode_lse(self, layer: int, q, out, lse, n_heads: int, scale: float, sinks=None, stream=None) -> None:
        """paged_decode plus lse [batch, n_heads] = ln(softmax denominator) of every row."""
        _check(lib.gkv_paged_decode_lse(self._h, layer, _f32_dev(q, "q"), _f32_dev(out, "out"),
                                        _f32_dev(lse, "lse"), n_heads, float(scale),
                                        None if sinks is None else _f32_dev(sinks, "sinks"),
                                        _stream(stream, self.device)))

    def paged_decode_splitkv_dist(self, comm: "Comm", layer: int, q, out, n_heads: int, scale: float,
                                  sinks=None, stream=None) -> None:
        """This rank's block ranges -> exchange of (out, lse) over the ranks (peer mailboxes over
        NVLink, or an NCCL all-gather) -> LSE merge into out on every rank."""
        _check(lib.gkv_paged_decode_splitkv_dist(self._h, comm.handle, layer, _f32_dev(q, "q"),
                                                 _f32_dev(out, "out"), n_heads, float(scale),
                                                 None if sinks is None else _f32_dev(sinks, "sinks"),
                                                 _stream(stream, self.device)))

    @property
    def last_launch_count(self) -> int:
        return _check(lib.gkv_pool_last_launch_count(self._h))

    def sync(self, stream=None, timeout_ms: int = 60_000) -> None:
        _check(lib.gkv_sync(self._h, _stream(stream, self.device), timeout_ms))


class BlockTable:
    """Per-sequence page table (BlockTable.cs:13)."""

    def __init__(self, pool: PagedBlockPool):
        if pool is None:
            raise ArgumentOutOfRangeError(GKV_EINVAL, "pool is None")
        h = C.c_void_p()
        _check(lib.gkv_table_create(pool.handle, C.byref(h)))
        self._h = h
        self._pool = pool

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib.gkv_table_destroy(self._h)
                self._h = None
        except Exception:
            pass

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @property
    def token_count(self) -> int:
        return _check(lib.gkv_table_token_count(self._h))

    @property
    def block_size(self) -> int:
        return self._pool.block_size

    @property
    def block_count(self) -> int:
        return _check(lib.gkv_table_block_count(self._h))

    @property
    def physical_block_ids(self) -> list:
        return list(self.as_span())

    def attach_prefix_blocks(self, prefix_block_ids: Sequence[int], token_count: int) -> None:
        arr = np.ascontiguousarray(np.asarray(prefix_block_ids, dtype=np.int32))
        _check(lib.gkv_table_attach_prefix_blocks(self._h, _ptr(arr), arr.size, token_count))

    def append_token(self) -> Tuple[bool, int, int]:
        b, o = C.c_int32(), C.c_int32()
        ok = _check(lib.gkv_table_append_token(self._h, C.byref(b), C.byref(o)))
        return bool(ok), b.value, o.value

    def get_token_location(self, token_index: int) -> Tuple[int, int]:
        b, o = C.c_int32(), C.c_int32()
        _check(lib.gkv_table_get_token_location(self._h, token_index, C.byref(b), C.byref(o)))
        return b.value, o.value

    def get_block_id(self, block_index: int) -> int:
        return _check(lib.gkv_table_get_block_id(self._h, block_index))

    def as_span(self) -> np.ndarray:
        n = self.block_count
        out = np.zeros(max(n, 1), dtype=np.int32)
        _check(lib.gkv_table_block_ids(self._h, _ptr(out), n))
        return out[:n]

    def release_all(self) -> None:
        _check(lib.gkv_table_release_all(self._h))


class PagedAttentionKernel:
    """PagedAttentionKernel.ComputeAttention (PagedAttentionKernel.cs:17-32) on the GPU."""

    @staticmethod
    def compute_attention(stage_layer: int, model_layer: int, pos: int, q, out, block_table: BlockTable,
                          pool: PagedBlockPool, n_heads: int, n_heads_kv: int, head_dim: int,
                          v_head_dim: int, attn_scale: float, max_seq_len: int,
                          sink_logit: Optional[float] = None, stream=None) -> None:
        has_sink = 0 if sink_logit is None else 1
        _check(lib.gkv_compute_attention(
            pool.handle, stage_layer, model_layer, pos, _f32_dev(q, "q"), _f32_dev(out, "out"),
            block_table.handle, n_heads, n_heads_kv, head_dim, v_head_dim, float(attn_scale),
            max_seq_len, has_sink, float(sink_logit or 0.0), _stream(stream, pool.device)))


def partition_lpt(ctx_lens: Sequence[int], n_ranks: int) -> np.ndarray:
    """Rank of every sequence under longest-first bin packing (one pool per GPU)."""
    cl = np.ascontiguousarray(np.asarray(ctx_lens, dtype=np.int32))
    out = np.zeros(max(cl.size, 1), dtype=np.int32)
    _check(lib.gkv_partition_lpt(_ptr(cl), cl.size, n_ranks, _ptr(out)))
    return out[: cl.size]


class Comm:
    """NCCL communicator of the ranks that split long sequences (gkv_comm_*)."""

    def __init__(self, unique_id: bytes, n_ranks: int, rank: int, device: int, timeout_ms: int = 60_000):
        if len(unique_id) != 128:
            raise ValueError("unique id must be 128 bytes")
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        h = C.c_void_p()
        _check(lib.gkv_comm_init(buf, n_ranks, rank, device, timeout_ms, C.byref(h)))
        self._h = h

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * 128)()
        _check(lib.gkv_comm_unique_id(buf))
        return bytes(buf)

    @property
    def handle(self):
        return self._h

    @property
    def exchange_kind(self) -> int:
        """0 = undecided (the first split-KV decode decides), 1 = NCCL all-gather, 2 = peer mailboxes."""
        return lib.gkv_comm_exchange_kind(self._h) if self._h else 0

    def abort(self) -> None:
        if self._h:
            lib.gkv_comm_abort(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.gkv_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def lse_merge(parts, n_parts: int, rows: int, dv: int, out, sinks=None, n_heads: int = 1, stream=None) -> None:
    """gkv_lse_merge: parts = n_parts blocks of ([rows, dv] outputs, [rows] lse), float32 CUDA."""
    import torch

    dev = parts.device.index or 0
    _check(lib.gkv_lse_merge(_f32_dev(parts, "parts"), n_parts, rows, dv,
                             None if sinks is None else _f32_dev(sinks, "sinks"), n_heads,
                             _f32_dev(out, "out"), _stream(stream, dev)))


def arena_desc(pool: PagedBlockPool) -> _lib.gkv_arena_desc:
    """The raw-pointer description of a pool's arena (for gkv_paged_decode_noalloc)."""
    k, v = pool._kv_ptrs()
    return _lib.gkv_arena_desc(k, v, pool.total_blocks, pool.layers, pool.heads_kv, pool.head_dim,
                               pool.value_head_dim, pool.block_size, DTYPES[pool.dtype])


def paged_decode_noalloc(pool: PagedBlockPool, layer: int, block_tables, ctx_lens, q, out, n_heads: int,
                         scale: float, sinks=None, stream=None) -> None:
    """gkv_paged_decode_noalloc on the pool's arena: the same decode as upload_step +
    paged_decode, with every scratch buffer in the library's fixed per-device array (the call
    allocates nothing).  Runs on the pool's device.  Copy-on-write copies the pool has queued
    are issued first on the same stream (the entry point sees only the raw arena)."""
    import torch

    desc = arena_desc(pool)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    cl = np.ascontiguousarray(ctx_lens, dtype=np.int32)
    if pool.pending_copies:
        pool.flush_copies(stream)
    with torch.cuda.device(pool.device):
        _check(lib.gkv_paged_decode_noalloc(
            C.byref(desc), layer, _ptr(bt), bt.shape[0], bt.shape[1], _ptr(cl), _f32_dev(q, "q"),
            _f32_dev(out, "out"), n_heads, float(scale), None if sinks is None else _f32_dev(sinks, "sinks"),
            _stream(stream, pool.device)))


def paged_decode_noalloc_status(device: int = 0, stream=None, timeout_ms: int = 60_000) -> None:
    """gkv_paged_decode_noalloc_status: raises DeviceError if an allocation-free decode on
    `device` since the last check met a bad block id or an expired bounded wait."""
    import torch

    with torch.cuda.device(device):
        _check(lib.gkv_paged_decode_noalloc_status(_stream(stream, device), timeout_ms))


def plan_decode(ctx_lens: Sequence[int], heads_kv: int, block_size: int, n_workers: int) -> dict:
    """The split-KV work list gkv_upload_step would build (host only, no GPU)."""
    cl = np.ascontiguousarray(np.asarray(ctx_lens, dtype=np.int32))
    info = _lib.gkv_plan_info()
    _check(lib.gkv_plan_decode(_ptr(cl) if cl.size else None, cl.size, heads_kv, block_size, n_workers,
                               C.byref(info), None, None, None, None, None, 0))
    n = max(info.n_pieces, 1)
    seg, c0, c1, slot = (np.zeros(n, np.int32) for _ in range(4))
    wb = np.zeros(n_workers + 1, np.int32)
    _check(lib.gkv_plan_decode(_ptr(cl) if cl.size else None, cl.size, heads_kv, block_size, n_workers,
                               C.byref(info), _ptr(seg), _ptr(c0), _ptr(c1), _ptr(slot), _ptr(wb), n))
    k = info.n_pieces
    return {"total_chunks": info.total_chunks, "n_pieces": k, "n_slots": info.n_slots,
            "n_merge": info.n_merge, "segment_cost": info.segment_cost, "piece_seg": seg[:k], "piece_c0": c0[:k], "piece_c1": c1[:k],
            "piece_slot": slot[:k], "worker_begin": wb}


def rope_inv_freq(freq_base: float, rope_dim: int, freq_factors=None) -> np.ndarray:
    """The inverse-frequency table gkv_rope_append builds when none is given."""
    fac = None if freq_factors is None else np.ascontiguousarray(freq_factors, dtype=np.float32)
    out = np.zeros(max(rope_dim // 2, 1), np.float32)
    _check(lib.gkv_rope_inv_freq(float(freq_base), rope_dim, _ptr(fac), _ptr(out)))
    return out[: rope_dim // 2]


def split_block_range(n_blocks: int, n_ranks: int, rank: int) -> Tuple[int, int]:
    b, e = C.c_int32(), C.c_int32()
    _check(lib.gkv_split_block_range(n_blocks, n_ranks, rank, C.byref(b), C.byref(e)))
    return b.value, e.value
