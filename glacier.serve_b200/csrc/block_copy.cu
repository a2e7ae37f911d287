// Batched block copy for copy-on-write forks, eviction and compaction (sm_100a).
//
// Replaces PagedBlockPool.CopyBlockData (src/Glacier.Serve/Inference/PagedAttention/
// PagedBlockPool.cs:304-327) as reached from TryForkBlock (:332-342) and
// BlockTable.AppendToken's CoW branch (BlockTable.cs:61-73).  The reference copies token
// rows one memcpy at a time; in the [block][layer][head][slot][dim] layout the first
// `valid` slots of one (block, layer, head) are ONE contiguous span, so each warp moves one
// span with 16-byte vectors.  One launch serves a whole batch of (src, dst, valid) ops.
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

__device__ __forceinline__ void copy_span(char* dst, const char* src, int64_t bytes, int lane,
                                          bool vec16) {
    int64_t done = 0;
    if (vec16) {
        const int64_t n16 = bytes >> 4;
        const uint4* s = reinterpret_cast<const uint4*>(src);
        uint4* d = reinterpret_cast<uint4*>(dst);
        for (int64_t i = lane; i < n16; i += 32) d[i] = s[i];
        done = n16 << 4;
    }
    // Tail (and the unaligned case) in 2-byte units: every storage type is >= 2 bytes.
    const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src + done);
    uint16_t* d2 = reinterpret_cast<uint16_t*>(dst + done);
    const int64_t n2 = (bytes - done) >> 1;
    for (int64_t i = lane; i < n2; i += 32) d2[i] = s2[i];
}

__global__ void __launch_bounds__(256) block_copy_kernel(ArenaGeom g, const int32_t* ops, int n,
                                                         int elem_bytes, bool vec16, int* err) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t per_op = static_cast<int64_t>(g.layers) * g.heads_kv;
    const int64_t total = per_op * n;
    char* K = static_cast<char*>(g.k);
    char* V = static_cast<char*>(g.v);
    for (int64_t w = warp; w < total; w += n_warps) {
        const int64_t op = w / per_op;
        const int64_t lh = w - op * per_op;
        const int l = static_cast<int>(lh / g.heads_kv);
        const int h = static_cast<int>(lh - static_cast<int64_t>(l) * g.heads_kv);
        const int src = ops[op * 3 + 0];
        const int dst = ops[op * 3 + 1];
        int valid = ops[op * 3 + 2];
        if (valid <= 0) continue;
        if (valid > g.block_size) valid = g.block_size;
        if (src < 0 || src >= g.total_blocks || dst < 0 || dst >= g.total_blocks) {
            if (lane == 0 && err) atomicOr(err, kErrBadBlock);
            continue;
        }
        const int64_t ko = static_cast<int64_t>(l) * g.k_layer_stride + h * g.k_head_stride;
        const int64_t vo = static_cast<int64_t>(l) * g.v_layer_stride + h * g.v_head_stride;
        copy_span(K + (dst * g.k_block_stride + ko) * elem_bytes,
                  K + (src * g.k_block_stride + ko) * elem_bytes,
                  static_cast<int64_t>(valid) * g.head_dim * elem_bytes, lane, vec16);
        copy_span(V + (dst * g.v_block_stride + vo) * elem_bytes,
                  V + (src * g.v_block_stride + vo) * elem_bytes,
                  static_cast<int64_t>(valid) * g.v_head_dim * elem_bytes, lane, vec16);
    }
}

}  // namespace

cudaError_t launch_block_copy(const ArenaGeom& g, const int32_t* ops, int n, int* err,
                              cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int eb = g.dtype == GKV_DTYPE_BF16 ? 2 : 4;
    // Every span starts at a multiple of the head stride; vectors need it 16-byte aligned.
    const bool vec16 = ((g.k_head_stride * eb) % 16 == 0) && ((g.v_head_stride * eb) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(g.k) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(g.v) % 16 == 0);
    const int64_t rows = static_cast<int64_t>(n) * g.layers * g.heads_kv;
    const int threads = 256;
    int64_t blocks = (rows * 32 + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    block_copy_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(g, ops, n, eb, vec16,
                                                                              err);
    return cudaGetLastError();
}

}  // namespace gkv
