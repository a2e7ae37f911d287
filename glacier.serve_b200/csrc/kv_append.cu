// KV append (reshape-and-cache scatter) for sm_100a.
//
// Replaces PagedBlockPool.Store (src/Glacier.Serve/Inference/PagedAttention/
// PagedBlockPool.cs:151-161), which the runners call once per sequence per layer
// (PagedTransformerRunner.cs:267,450,634).  One launch writes every token of the step:
// token i's row for kv head h is copied from the contiguous source [n_tok][heads_kv][dim]
// into arena element (block, layer, h, offset) with block = slot / block_size,
// offset = slot % block_size.  fp32 storage is a bit copy; bf16 and fp16 storage round to
// nearest even; fp8 e4m3 stores x * (1 / scale) of the row's (layer, head), rounded to nearest
// even and saturated.  HBM-bound: each (token, head) row is one warp moving 16-byte vectors, two rows per
// warp iteration.
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

// `inv` is the reciprocal of an FP8 arena's (layer, head) scale; the other types ignore it.
template <typename KV>
__device__ __forceinline__ void store4(KV* dst, float4 v, float inv);

template <>
__device__ __forceinline__ void store4<float>(float* dst, float4 v, float) {
    *reinterpret_cast<float4*>(dst) = v;
}

template <>
__device__ __forceinline__ void store4<__nv_fp8_e4m3>(__nv_fp8_e4m3* dst, float4 v, float inv) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v.x * inv, v.y * inv), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v.z * inv, v.w * inv), __NV_SATFINITE, __NV_E4M3);
    *reinterpret_cast<uint32_t*>(dst) = lo | (hi << 16);
}

template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float4 v, float) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(dst) = w;
}

template <>
__device__ __forceinline__ void store4<__half>(__half* dst, float4 v, float) {
    __half2 a = __floats2half2_rn(v.x, v.y);
    __half2 b = __floats2half2_rn(v.z, v.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(dst) = w;
}

template <typename KV>
__device__ __forceinline__ void store1(KV* dst, float v, float inv);
template <>
__device__ __forceinline__ void store1<float>(float* dst, float v, float) { *dst = v; }
template <>
__device__ __forceinline__ void store1<__nv_bfloat16>(__nv_bfloat16* dst, float v, float) {
    *dst = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void store1<__half>(__half* dst, float v, float) {
    *dst = __float2half_rn(v);
}
template <>
__device__ __forceinline__ void store1<__nv_fp8_e4m3>(__nv_fp8_e4m3* dst, float v, float inv) {
    dst->__x = __nv_cvt_float_to_fp8(v * inv, __NV_SATFINITE, __NV_E4M3);
}

// x / d and x % d for the non-negative row and slot indices; `shift` >= 0 when d is a power of
// two (the usual 16-token blocks and power-of-two head counts), which skips the division.
__device__ __forceinline__ int div_rows(int x, int d, int shift) {
    return shift >= 0 ? (x >> shift) : x / d;
}
__device__ __forceinline__ int64_t div_slot(int64_t x, int d, int shift) {
    return shift >= 0 ? (x >> shift) : x / d;
}

// Source and destination rows of one (token, kv head); ok == false past the end, for padding
// tokens and for bad slots (which set kErrBadSlot).
template <typename KV>
struct AppendRow {
    KV* dk;
    KV* dv;
    const float* sk;
    const float* sv;
    float kinv, vinv;  // FP8: reciprocal scales of the row's (layer, head)
    bool ok;
};

// Each warp moves kRows (token, head) rows per iteration.  All K and V loads of those rows are
// issued before the first store, so a lane keeps 2 x kRows 16-byte loads in flight, and the
// slots of the NEXT iteration's rows are read while this iteration's rows move, so the slot
// read is off the critical path.  Row indices are 32-bit (the host splits larger appends).
// The sources are read once (evict-first); the arena stores stay cacheable because the
// attention launch that follows reads them.
constexpr int kRows = 2;
constexpr int kMaxRowsPerLaunch = 1 << 30;

struct AppendArgs {
    int layer;
    const float* k;
    const float* v;
    int64_t k_tok_stride, v_tok_stride;
    const int64_t* slots;  // nullptr: every token goes to single_slot
    int64_t single_slot;
    int n_tok;
    int bs_shift, heads_shift;  // log2 of block_size / heads_kv, or -1
    int* err;
    const int32_t* dyn_tok;     // static step layout: the token count, read on the device
};

__device__ __forceinline__ void fetch_slots(int64_t (&s)[kRows], const AppendArgs& a,
                                            const ArenaGeom& g, int w0, int n_warps, int total) {
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
        const int row = w0 + u * n_warps;
        s[u] = -1;
        if (row < total)
            s[u] = a.slots ? __ldg(a.slots + div_rows(row, g.heads_kv, a.heads_shift)) : a.single_slot;
    }
}

template <typename KV>
__device__ __forceinline__ AppendRow<KV> resolve_row(const ArenaGeom& g, const AppendArgs& a,
                                                     int row, int64_t slot, int lane) {
    AppendRow<KV> r{nullptr, nullptr, nullptr, nullptr, 1.f, 1.f, false};
    if (slot < 0) return r;  // past the end, or a padding token
    const int64_t blk = div_slot(slot, g.block_size, a.bs_shift);
    const int off = static_cast<int>(slot - blk * g.block_size);
    if (blk >= g.total_blocks) {
        if (lane == 0 && a.err) atomicOr(a.err, kErrBadSlot);
        return r;
    }
    const int i = div_rows(row, g.heads_kv, a.heads_shift);
    const int h = row - i * g.heads_kv;
    r.dk = static_cast<KV*>(g.k) + blk * g.k_block_stride + a.layer * g.k_layer_stride +
           h * g.k_head_stride + static_cast<int64_t>(off) * g.head_dim;
    r.dv = static_cast<KV*>(g.v) + blk * g.v_block_stride + a.layer * g.v_layer_stride +
           h * g.v_head_stride + static_cast<int64_t>(off) * g.v_head_dim;
    r.sk = a.k + i * a.k_tok_stride + static_cast<int64_t>(h) * g.head_dim;
    r.sv = a.v + i * a.v_tok_stride + static_cast<int64_t>(h) * g.v_head_dim;
    if (g.k_inv) {
        r.kinv = __ldg(g.k_inv + a.layer * g.heads_kv + h);
        r.vinv = __ldg(g.v_inv + a.layer * g.heads_kv + h);
    }
    r.ok = true;
    return r;
}

template <typename KV, bool VEC>
__global__ void __launch_bounds__(256, 4) kv_append_kernel(ArenaGeom g, AppendArgs a) {
    // the decode that follows (a programmatic dependent launch) may be scheduled now; it waits
    // for this grid's completion before it reads the arena
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int n_warps = static_cast<int>((gridDim.x * blockDim.x) >> 5);
    const int n_tok = a.dyn_tok ? min(__ldg(a.dyn_tok), a.n_tok) : a.n_tok;
    const int total = n_tok * g.heads_kv;  // <= kMaxRowsPerLaunch
    const int step = kRows * n_warps;
    const int hd = g.head_dim, vhd = g.v_head_dim;
    int64_t next[kRows];
    fetch_slots(next, a, g, warp, n_warps, total);
    for (int w0 = warp; w0 < total; w0 += step) {
        int64_t cur[kRows];
#pragma unroll
        for (int u = 0; u < kRows; ++u) cur[u] = next[u];
        fetch_slots(next, a, g, w0 + step, n_warps, total);
        AppendRow<KV> r[kRows];
#pragma unroll
        for (int u = 0; u < kRows; ++u) r[u] = resolve_row<KV>(g, a, w0 + u * n_warps, cur[u], lane);
        if constexpr (VEC) {
            const int n = hd > vhd ? hd : vhd;
            for (int e = lane * 4; e < n; e += 128) {
                float4 x[kRows], y[kRows];
#pragma unroll
                for (int u = 0; u < kRows; ++u) {
                    if (r[u].ok && e < hd) x[u] = __ldcs(reinterpret_cast<const float4*>(r[u].sk + e));
                    if (r[u].ok && e < vhd) y[u] = __ldcs(reinterpret_cast<const float4*>(r[u].sv + e));
                }
#pragma unroll
                for (int u = 0; u < kRows; ++u) {
                    if (r[u].ok && e < hd) store4<KV>(r[u].dk + e, x[u], r[u].kinv);
                    if (r[u].ok && e < vhd) store4<KV>(r[u].dv + e, y[u], r[u].vinv);
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < kRows; ++u) {
                if (!r[u].ok) continue;
                for (int e = lane; e < hd; e += 32) store1<KV>(r[u].dk + e, __ldg(r[u].sk + e), r[u].kinv);
                for (int e = lane; e < vhd; e += 32) store1<KV>(r[u].dv + e, __ldg(r[u].sv + e), r[u].vinv);
            }
        }
    }
}

int log2_or_neg(int x) {
    if (x <= 0 || (x & (x - 1)) != 0) return -1;
    int s = 0;
    while ((1 << s) < x) ++s;
    return s;
}

template <typename KV>
cudaError_t launch_typed(const ArenaGeom& g, AppendArgs a, cudaStream_t stream) {
    const bool vec = (g.head_dim % 4 == 0) && (g.v_head_dim % 4 == 0) && (a.k_tok_stride % 4 == 0) &&
                     (a.v_tok_stride % 4 == 0) && (reinterpret_cast<uintptr_t>(a.k) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(a.v) % 16 == 0);
    a.bs_shift = log2_or_neg(g.block_size);
    a.heads_shift = log2_or_neg(g.heads_kv);
    const int max_tok = kMaxRowsPerLaunch / g.heads_kv;
    const int threads = 256;
    for (int t0 = 0; t0 < a.n_tok; t0 += max_tok) {  // one launch unless rows exceed 2^30
        AppendArgs c = a;
        c.n_tok = a.n_tok - t0 < max_tok ? a.n_tok - t0 : max_tok;
        c.k = a.k + static_cast<int64_t>(t0) * a.k_tok_stride;
        c.v = a.v + static_cast<int64_t>(t0) * a.v_tok_stride;
        if (a.slots) c.slots = a.slots + t0;
        const int64_t rows = static_cast<int64_t>(c.n_tok) * g.heads_kv;
        // one warp per kRows rows, at most one wave of 4 resident CTAs per SM (the launch
        // bound; grid-stride beyond)
        int64_t blocks = ((rows + kRows - 1) / kRows * 32 + threads - 1) / threads;
        if (blocks > 148 * 4) blocks = 148 * 4;
        if (blocks < 1) blocks = 1;
        if (vec)
            kv_append_kernel<KV, true><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(g, c);
        else
            kv_append_kernel<KV, false><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(g, c);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

cudaError_t launch_kv_append(const ArenaGeom& g, int layer, const float* k, const float* v,
                             int64_t k_tok_stride, int64_t v_tok_stride, const int64_t* slots,
                             int64_t single_slot, int n_tok, int* err, cudaStream_t stream,
                             const int32_t* dyn_tok) {
    if (n_tok <= 0) return cudaSuccess;
    // a device-side count must fit one launch (the host splits only counts it knows)
    if (dyn_tok && static_cast<int64_t>(n_tok) * g.heads_kv > kMaxRowsPerLaunch) return cudaErrorInvalidValue;
    AppendArgs a{layer, k, v, k_tok_stride, v_tok_stride, slots, single_slot, n_tok, -1, -1, err, dyn_tok};
    if (g.dtype == GKV_DTYPE_BF16) return launch_typed<__nv_bfloat16>(g, a, stream);
    if (g.dtype == GKV_DTYPE_F16) return launch_typed<__half>(g, a, stream);
    if (g.dtype == GKV_DTYPE_FP8_E4M3) return launch_typed<__nv_fp8_e4m3>(g, a, stream);
    return launch_typed<float>(g, a, stream);
}

}  // namespace gkv
