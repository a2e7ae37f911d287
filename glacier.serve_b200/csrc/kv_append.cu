// KV append (reshape-and-cache scatter) for sm_100a.
//
// Replaces PagedBlockPool.Store (src/Glacier.Serve/Inference/PagedAttention/
// PagedBlockPool.cs:151-161), which the runners call once per sequence per layer
// (PagedTransformerRunner.cs:267,450,634).  One launch writes every token of the step:
// token i's row for kv head h is copied from the contiguous source [n_tok][heads_kv][dim]
// into arena element (block, layer, h, offset) with block = slot / block_size,
// offset = slot % block_size.  fp32 storage is a bit copy; bf16 storage rounds to nearest
// even.  HBM-bound: each (token, head) row is one warp moving 16-byte vectors.
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

template <typename KV>
__device__ __forceinline__ void store4(KV* dst, float4 v);

template <>
__device__ __forceinline__ void store4<float>(float* dst, float4 v) {
    *reinterpret_cast<float4*>(dst) = v;
}

template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(dst) = w;
}

template <typename KV>
__device__ __forceinline__ void store1(KV* dst, float v);
template <>
__device__ __forceinline__ void store1<float>(float* dst, float v) { *dst = v; }
template <>
__device__ __forceinline__ void store1<__nv_bfloat16>(__nv_bfloat16* dst, float v) {
    *dst = __float2bfloat16_rn(v);
}

// Copies one row of `n` elements with the whole warp; VEC selects 16-byte source loads.
template <typename KV, bool VEC>
__device__ __forceinline__ void copy_row(KV* dst, const float* src, int n, int lane) {
    if constexpr (VEC) {
        for (int e = lane * 4; e < n; e += 128) {
            float4 v = __ldg(reinterpret_cast<const float4*>(src + e));
            store4<KV>(dst + e, v);
        }
    } else {
        for (int e = lane; e < n; e += 32) store1<KV>(dst + e, __ldg(src + e));
    }
}

template <typename KV, bool VEC>
__global__ void __launch_bounds__(256) kv_append_kernel(ArenaGeom g, int layer, const float* k,
                                                        const float* v, int64_t k_tok_stride,
                                                        int64_t v_tok_stride,
                                                        const int64_t* slots,
                                                        int64_t single_slot, int n_tok,
                                                        int* err) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t total = static_cast<int64_t>(n_tok) * g.heads_kv;
    KV* K = static_cast<KV*>(g.k);
    KV* V = static_cast<KV*>(g.v);
    for (int64_t w = warp; w < total; w += n_warps) {
        const int64_t i = w / g.heads_kv;
        const int h = static_cast<int>(w - i * g.heads_kv);
        const int64_t slot = slots ? slots[i] : single_slot;
        if (slot < 0) continue;  // padding token
        const int64_t blk = slot / g.block_size;
        const int off = static_cast<int>(slot - blk * g.block_size);
        if (blk >= g.total_blocks) {
            if (lane == 0 && err) atomicOr(err, kErrBadSlot);
            continue;
        }
        KV* dk = K + blk * g.k_block_stride + layer * g.k_layer_stride + h * g.k_head_stride +
                 static_cast<int64_t>(off) * g.head_dim;
        KV* dv = V + blk * g.v_block_stride + layer * g.v_layer_stride + h * g.v_head_stride +
                 static_cast<int64_t>(off) * g.v_head_dim;
        copy_row<KV, VEC>(dk, k + i * k_tok_stride + static_cast<int64_t>(h) * g.head_dim,
                          g.head_dim, lane);
        copy_row<KV, VEC>(dv, v + i * v_tok_stride + static_cast<int64_t>(h) * g.v_head_dim,
                          g.v_head_dim, lane);
    }
}

template <typename KV>
cudaError_t launch_typed(const ArenaGeom& g, int layer, const float* k, const float* v,
                         int64_t ks, int64_t vs, const int64_t* slots, int64_t single,
                         int n_tok, int* err, cudaStream_t stream) {
    const int64_t rows = static_cast<int64_t>(n_tok) * g.heads_kv;
    const int threads = 256;
    int64_t blocks = (rows * 32 + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;  // grid-stride beyond 16 CTAs per SM
    if (blocks < 1) blocks = 1;
    const bool vec = (g.head_dim % 4 == 0) && (g.v_head_dim % 4 == 0) && (ks % 4 == 0) &&
                     (vs % 4 == 0) && (reinterpret_cast<uintptr_t>(k) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(v) % 16 == 0);
    if (vec)
        kv_append_kernel<KV, true><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
            g, layer, k, v, ks, vs, slots, single, n_tok, err);
    else
        kv_append_kernel<KV, false><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
            g, layer, k, v, ks, vs, slots, single, n_tok, err);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_kv_append(const ArenaGeom& g, int layer, const float* k, const float* v,
                             int64_t k_tok_stride, int64_t v_tok_stride, const int64_t* slots,
                             int64_t single_slot, int n_tok, int* err, cudaStream_t stream) {
    if (n_tok <= 0) return cudaSuccess;
    if (g.dtype == GKV_DTYPE_BF16)
        return launch_typed<__nv_bfloat16>(g, layer, k, v, k_tok_stride, v_tok_stride, slots,
                                           single_slot, n_tok, err, stream);
    return launch_typed<float>(g, layer, k, v, k_tok_stride, v_tok_stride, slots, single_slot,
                               n_tok, err, stream);
}

}  // namespace gkv
