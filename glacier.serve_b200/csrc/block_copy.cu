// Batched block copy for copy-on-write forks, eviction and compaction (sm_100a).
//
// Replaces PagedBlockPool.CopyBlockData (src/Glacier.Serve/Inference/PagedAttention/
// PagedBlockPool.cs:304-327) as reached from TryForkBlock (:332-342) and
// BlockTable.AppendToken's CoW branch (BlockTable.cs:61-73).  The reference copies token
// rows one memcpy at a time; in the [block][layer][head][slot][dim] layout the first
// `valid` slots of one (block, layer, head) are ONE contiguous span of K (and one of V),
// moved in 2 KB chunks of 16-byte vectors, one chunk per warp at a time.  One launch serves a
// whole batch of (src, dst, valid) ops.
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

// The work is cut into chunks of 32 lanes x kUnroll 16-byte vectors (2 KB) of one K or V span:
// each lane loads its kUnroll vectors before it stores them, and the chunks (not whole spans)
// are spread over the warps, so no warp is left with a whole extra span at the end.
constexpr int kUnroll = 4;
constexpr int kChunk16 = 32 * kUnroll;             // 16-byte vectors per chunk
constexpr int kMaxItemsPerLaunch = 1 << 30;

struct CopyArgs {
    const int32_t* ops;
    int n;            // ops in this launch
    int elem_bytes;
    int ck, cv;       // chunks of a full K / V span (16-byte path) or 1 (2-byte path)
    bool vec16;
    int* err;
};

// Copies bytes [from, to) of one span, 2 bytes per lane per step (unaligned geometries).
__device__ __forceinline__ void copy_bytes2(char* dst, const char* src, int64_t from, int64_t to,
                                            int lane) {
    const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
    uint16_t* d2 = reinterpret_cast<uint16_t*>(dst);
    for (int64_t i = (from >> 1) + lane; i < (to >> 1); i += 32) d2[i] = s2[i];
}

__global__ void __launch_bounds__(256, 4) block_copy_kernel(ArenaGeom g, CopyArgs a) {
    const int lane = threadIdx.x & 31;
    const int warp = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int n_warps = static_cast<int>((gridDim.x * blockDim.x) >> 5);
    const int per_unit = a.ck + a.cv;                  // chunks of one (op, layer, head)
    const int per_op = g.layers * g.heads_kv * per_unit;
    const int total = a.n * per_op;                    // <= kMaxItemsPerLaunch
    const int eb = a.elem_bytes;
    for (int w = warp; w < total; w += n_warps) {
        const int op = w / per_op;
        int r = w - op * per_op;
        const int lh = r / per_unit;
        const int c = r - lh * per_unit;
        const int l = lh / g.heads_kv;
        const int h = lh - l * g.heads_kv;
        const int src = __ldg(a.ops + op * 3 + 0);
        const int dst = __ldg(a.ops + op * 3 + 1);
        int valid = __ldg(a.ops + op * 3 + 2);
        if (valid <= 0) continue;
        if (valid > g.block_size) valid = g.block_size;
        if (src < 0 || src >= g.total_blocks || dst < 0 || dst >= g.total_blocks) {
            if (lane == 0 && c == 0 && a.err) atomicOr(a.err, kErrBadBlock);
            continue;
        }
        const bool is_k = c < a.ck;
        const int chunk = is_k ? c : c - a.ck;
        char* base = static_cast<char*>(is_k ? g.k : g.v);
        const int64_t bstride = is_k ? g.k_block_stride : g.v_block_stride;
        const int64_t off = static_cast<int64_t>(l) * (is_k ? g.k_layer_stride : g.v_layer_stride) +
                            static_cast<int64_t>(h) * (is_k ? g.k_head_stride : g.v_head_stride);
        const char* s = base + (src * bstride + off) * eb;
        char* d = base + (dst * bstride + off) * eb;
        const int64_t bytes = static_cast<int64_t>(valid) * (is_k ? g.head_dim : g.v_head_dim) * eb;
        if (!a.vec16) {  // one chunk per span
            copy_bytes2(d, s, 0, bytes, lane);
            continue;
        }
        const int64_t n16 = bytes >> 4;
        // the last chunk holding data (it also copies a tail shorter than 16 bytes)
        const int last = n16 > 0 ? static_cast<int>((n16 - 1) / kChunk16) : 0;
        if (chunk > last) continue;  // past the valid slots
        const int64_t v0 = static_cast<int64_t>(chunk) * kChunk16;
        const uint4* sv = reinterpret_cast<const uint4*>(s);
        uint4* dv = reinterpret_cast<uint4*>(d);
        uint4 t[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = v0 + 32 * u + lane;
            if (i < n16) t[u] = sv[i];
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = v0 + 32 * u + lane;
            if (i < n16) dv[i] = t[u];
        }
        if ((bytes & 15) != 0 && chunk == last) copy_bytes2(d, s, n16 << 4, bytes, lane);
    }
}

}  // namespace

cudaError_t launch_block_copy(const ArenaGeom& g, const int32_t* ops, int n, int* err,
                              cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int eb = elem_bytes_of(g.dtype);
    // Every span starts at a multiple of the head stride; vectors need it 16-byte aligned.
    const bool vec16 = ((g.k_head_stride * eb) % 16 == 0) && ((g.v_head_stride * eb) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(g.k) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(g.v) % 16 == 0);
    auto chunks = [&](int dim) {
        const int64_t full = static_cast<int64_t>(g.block_size) * dim * eb;
        return vec16 ? static_cast<int>((full + 16 * kChunk16 - 1) / (16 * kChunk16)) : 1;
    };
    CopyArgs a{ops, 0, eb, chunks(g.head_dim), chunks(g.v_head_dim), vec16, err};
    const int64_t per_op = static_cast<int64_t>(g.layers) * g.heads_kv * (a.ck + a.cv);
    const int max_ops = static_cast<int>(kMaxItemsPerLaunch / per_op) > 0
                            ? static_cast<int>(kMaxItemsPerLaunch / per_op) : 1;
    const int threads = 256;
    for (int o0 = 0; o0 < n; o0 += max_ops) {  // one launch unless the chunks exceed 2^30
        CopyArgs c = a;
        c.ops = ops + static_cast<int64_t>(o0) * 3;
        c.n = n - o0 < max_ops ? n - o0 : max_ops;
        int64_t blocks = (c.n * per_op * 32 + threads - 1) / threads;
        if (blocks > 148 * 4) blocks = 148 * 4;  // one wave of 4 resident CTAs per SM (launch bound)
        block_copy_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(g, c);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace gkv
