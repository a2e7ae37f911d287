"""ctypes binding of libglacier_kv.so (the C ABI declared in include/glacier_kv.h).

The shared library is built in-tree by ``make -C glacier.serve_b200/csrc`` (or
``__graft_entry__.build()``).  It is mapped on the first call through ``lib`` (so importing the
package, e.g. for its numpy-only workload generators, maps no native code); that first call
raises ImportError when the library is missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.normpath(os.path.join(_PKG_DIR, "..", "lib", "libglacier_kv.so"))

GKV_OK = 0
GKV_EINVAL = -1
GKV_ENOMEM = -2
GKV_ESTATE = -3
GKV_ECUDA = -4
GKV_ETIMEDOUT = -5
GKV_ENCCL = -6
GKV_EDEVICE = -7
GKV_EUNSUPPORTED = -8

GKV_DTYPE_F32 = 0
GKV_DTYPE_BF16 = 1
GKV_DTYPE_F16 = 2
GKV_DTYPE_FP8_E4M3 = 3
DTYPES = {"f32": GKV_DTYPE_F32, "bf16": GKV_DTYPE_BF16, "f16": GKV_DTYPE_F16, "fp8": GKV_DTYPE_FP8_E4M3}


class gkv_pool_desc(C.Structure):
    _fields_ = [
        ("device", C.c_int32),
        ("total_blocks", C.c_int32),
        ("layers", C.c_int32),
        ("heads_kv", C.c_int32),
        ("head_dim", C.c_int32),
        ("v_head_dim", C.c_int32),
        ("block_size", C.c_int32),
        ("dtype", C.c_int32),
        ("allocate_device_arena", C.c_int32),
    ]


class gkv_plan_info(C.Structure):
    _fields_ = [
        ("total_chunks", C.c_int64),
        ("n_pieces", C.c_int32),
        ("n_slots", C.c_int32),
        ("n_merge", C.c_int32),
        ("n_workers", C.c_int32),
        ("segment_cost", C.c_int32),
    ]


class gkv_arena_desc(C.Structure):
    _fields_ = [
        ("d_k", C.c_void_p),
        ("d_v", C.c_void_p),
        ("total_blocks", C.c_int32),
        ("layers", C.c_int32),
        ("heads_kv", C.c_int32),
        ("head_dim", C.c_int32),
        ("v_head_dim", C.c_int32),
        ("block_size", C.c_int32),
        ("dtype", C.c_int32),
    ]


class gkv_rope_desc(C.Structure):
    _fields_ = [
        ("rope_dim", C.c_int32),
        ("style", C.c_int32),
        ("freq_base", C.c_float),
        ("mscale", C.c_float),
        ("h_inv_freq", C.c_void_p),
        ("h_freq_factors", C.c_void_p),
    ]


class gkv_qkv_prologue(C.Structure):
    _fields_ = [
        ("d_q_bias", C.c_void_p),
        ("d_k_bias", C.c_void_p),
        ("d_v_bias", C.c_void_p),
        ("d_q_norm", C.c_void_p),
        ("d_k_norm", C.c_void_p),
        ("eps", C.c_float),
    ]


class gkv_pool_stats(C.Structure):
    _fields_ = [
        ("total_blocks", C.c_int32),
        ("free_blocks", C.c_int32),
        ("allocated_blocks", C.c_int32),
        ("capacity_tokens", C.c_int32),
        ("active_tokens", C.c_int32),
        ("block_size", C.c_int32),
        ("pending_copies", C.c_int32),
        ("has_device_arena", C.c_int32),
        ("total_memory_bytes", C.c_int64),
    ]


P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
U64 = C.c_uint64
F32 = C.c_float
PI32 = C.POINTER(C.c_int32)
PI64 = C.POINTER(C.c_int64)
PF32 = C.POINTER(C.c_float)

# name -> (restype, argtypes); every symbol of include/glacier_kv.h
SIGNATURES = {
    "gkv_pool_create": (C.c_int, [C.POINTER(gkv_pool_desc), C.POINTER(P)]),
    "gkv_pool_destroy": (C.c_int, [P]),
    "gkv_pool_stats_get": (C.c_int, [P, C.POINTER(gkv_pool_stats)]),
    "gkv_pool_set_kv_scales": (C.c_int, [P, PF32, PF32]),
    "gkv_pool_kv_ptrs": (C.c_int, [P, C.POINTER(P), C.POINTER(P)]),
    "gkv_pool_element_offset": (C.c_int, [P, I32, I32, I32, I32, I32, PI64]),
    "gkv_pool_try_allocate_block": (C.c_int, [P, PI32]),
    "gkv_pool_release_block": (C.c_int, [P, I32]),
    "gkv_pool_free_block": (C.c_int, [P, I32]),
    "gkv_pool_free_blocks": (C.c_int, [P, P, I32]),
    "gkv_pool_retain_block": (C.c_int, [P, I32]),
    "gkv_pool_get_ref_count": (C.c_int, [P, I32]),
    "gkv_pool_try_find_prefix_block": (C.c_int, [P, U64, PI32]),
    "gkv_pool_bind_prefix_block": (C.c_int, [P, U64, I32]),
    "gkv_pool_try_fork_block": (C.c_int, [P, I32, I32, PI32]),
    "gkv_pool_flush_copies": (C.c_int, [P, P]),
    "gkv_block_copy": (C.c_int, [P, P, P, P, I32, P]),
    "gkv_pool_store": (C.c_int, [P, I32, I32, I32, P, P, P]),
    "gkv_pool_compact": (C.c_int, [P, P, I32, I32, P, P, I32, P]),
    "gkv_table_create": (C.c_int, [P, C.POINTER(P)]),
    "gkv_table_destroy": (C.c_int, [P]),
    "gkv_table_attach_prefix_blocks": (C.c_int, [P, P, I32, I32]),
    "gkv_table_append_token": (C.c_int, [P, PI32, PI32]),
    "gkv_table_get_token_location": (C.c_int, [P, I32, PI32, PI32]),
    "gkv_table_get_block_id": (C.c_int, [P, I32]),
    "gkv_table_token_count": (C.c_int, [P]),
    "gkv_table_block_count": (C.c_int, [P]),
    "gkv_table_block_ids": (C.c_int, [P, P, I32]),
    "gkv_table_release_all": (C.c_int, [P]),
    "gkv_step_reserve": (C.c_int, [P, I32, I32, I32, I32]),
    "gkv_step_set_static": (C.c_int, [P, I32]),
    "gkv_upload_step": (C.c_int, [P, P, I32, I32, P, P, I32, P]),
    "gkv_upload_step_tables": (C.c_int, [P, P, I32, P, P, I32, P]),
    "gkv_kv_append": (C.c_int, [P, I32, P, P, I32, P]),
    "gkv_paged_decode": (C.c_int, [P, I32, P, P, I32, F32, P, P]),
    "gkv_rope_append": (C.c_int, [P, I32, P, P, P, I32, I32, P, C.POINTER(gkv_rope_desc),
                                  C.POINTER(gkv_qkv_prologue), P]),
    "gkv_rope_inv_freq": (C.c_int, [F32, I32, P, P]),
    "gkv_paged_prefill": (C.c_int, [P, I32, P, I32, P, P, P, I32, F32, P]),
    "gkv_compute_attention": (
        C.c_int,
        [P, I32, I32, I32, P, P, P, I32, I32, I32, I32, F32, I32, I32, F32, P],
    ),
    "gkv_decode_step_host": (
        C.c_int,
        [P, I32, P, I32, I32, P, P, I32, P, P, P, P, I32, F32, P, P],
    ),
    "gkv_paged_decode_noalloc": (
        C.c_int,
        [C.POINTER(gkv_arena_desc), I32, P, I32, I32, P, P, P, I32, F32, P, P],
    ),
    "gkv_paged_decode_noalloc_status": (C.c_int, [P, I32]),
    "gkv_wait_host_outputs": (C.c_int, [P, P]),
    "gkv_pool_last_launch_count": (C.c_int, [P]),
    "gkv_sync": (C.c_int, [P, P, I32]),
    "gkv_plan_decode": (C.c_int, [P, I32, I32, I32, I32, C.POINTER(gkv_plan_info), P, P, P, P, P, I32]),
    "gkv_paged_decode_lse": (C.c_int, [P, I32, P, P, P, I32, F32, P, P]),
    "gkv_lse_merge": (C.c_int, [P, I32, I32, I32, P, I32, P, P]),
    "gkv_comm_unique_id": (C.c_int, [P]),
    "gkv_comm_init": (C.c_int, [P, I32, I32, I32, I32, C.POINTER(P)]),
    "gkv_comm_abort": (C.c_int, [P]),
    "gkv_comm_destroy": (C.c_int, [P]),
    "gkv_comm_exchange_kind": (C.c_int, [P]),
    "gkv_paged_decode_splitkv_dist": (C.c_int, [P, P, I32, P, P, I32, F32, P, P]),
    "gkv_partition_lpt": (C.c_int, [P, I32, I32, P]),
    "gkv_split_block_range": (C.c_int, [I32, I32, I32, PI32, PI32]),
    "gkv_last_error": (C.c_char_p, []),
    "gkv_version": (C.c_char_p, []),
}


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C glacier.serve_b200/csrc` "
            "(or __graft_entry__.build()); glacier_kv has no CPU fallback"
        )
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class _LazyLib:
    """Loads libglacier_kv.so on first attribute access and forwards to the CDLL."""

    _cdll = None

    def __getattr__(self, name):
        if _LazyLib._cdll is None:
            _LazyLib._cdll = _load()
        return getattr(_LazyLib._cdll, name)

    @staticmethod
    def loaded() -> bool:
        return _LazyLib._cdll is not None


lib = _LazyLib()


def last_error() -> str:
    msg = lib.gkv_last_error()
    return msg.decode() if msg else ""
