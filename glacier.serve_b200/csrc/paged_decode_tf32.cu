// Tensor-core variant of the split-KV paged decode for fp32 KV with wide GQA groups.
//
// The CUDA-core kernel (paged_decode.cu) runs a query group of 5..8 heads against fp32 KV at
// about 520 FP32-pipe instructions per 8-token chunk, and with two warps per scheduler it is
// bound by instruction issue, not by HBM.  This kernel moves both products onto the tensor
// cores with fp32-level accuracy: every operand x is split into a TF32 high part
// hi = rna_tf32(x) and a low part lo = x - hi, and a product is accumulated in fp32 as
// hi*hi + lo*hi + hi*lo (the lo*lo term, ~2^-22 relative, is dropped), the three-pass TF32
// scheme.  Same work decomposition, work list, partial layout and merge as the other decode
// kernels (warp-level stream-K over 8-token chunks of (sequence, kv head) segments).  Per chunk:
//
//  * Eight tiled TMA boxes (8 tokens x 32 fp32 dims = 1 KB each, 128-byte swizzle, no
//    multicast), four for K and four for V, from a 3-D view [block*layer*head][slot][dim] of
//    this GPU's own arena, issued by lanes 0-7 at once.
//  * S[8 heads x 8 tokens] = Q . K^T with mma.m16n8k8 (tf32 in, fp32 accumulate; rows 8..15
//    of the A operand are zero), 16 k-steps of 8 dims.  Inside a k-step the dims are taken in
//    the order 2t, 2t+1 (t = lane % 4) so that a lane's two K values are adjacent (one 8-byte
//    load); the query fragments use the same order.  The accumulator leaves lane L holding
//    head L/4 for tokens 2*(L%4) and 2*(L%4)+1, as in the bf16 tensor-core kernel.
//  * Online softmax on those fragments (base 2, max/sum over the 4 lanes of a head).
//  * O^T[128 dv x 8 heads] += V^T . P^T with mma.m16n8k8 over the chunk's tokens taken in the
//    order 0, 2, 4, 6, 1, 3, 5, 7, so that the B fragment is exactly the lane's own two
//    probabilities; the V^T fragments come from conflict-free 4-byte loads of the swizzled tile.
//
// About 300 instructions per chunk instead of ~520, 72 MMAs.  Roofline: HBM.
#include <cuda.h>

#include <atomic>

#include "decode_merge.cuh"
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

constexpr int kChunk = kDecodeChunk;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kGP = 8, kD = 128, kDV = 128;
constexpr int kBox = 1024;           // one box: 8 rows x 128 bytes (32 fp32)
constexpr int kStage = 8 * kBox;     // K dims [0,32) [32,64) [64,96) [96,128), then V the same
constexpr int kNW = 4;               // warp workers per CTA (as the other decode kernels)
constexpr int kS = 3;                // ring stages per warp (2 CTAs, 8 warps per SM)

// Byte offset of fp32 element (row, col) of a 128-byte-swizzled 8 x 32 box.
__device__ __forceinline__ uint32_t swz32(int row, int col) {
    return static_cast<uint32_t>(row * 128 + ((((col >> 2) ^ row) & 7) << 4) + (col & 3) * 4);
}

__device__ __forceinline__ uint32_t tf32_hi(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// hi = x rounded to TF32 (nearest, ties away), lo = x - hi (its low bits are truncated by the
// MMA, an error of ~2^-21 relative to x).
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = tf32_hi(x);
    lo = __float_as_uint(x - __uint_as_float(hi));
}

// D(16x8) += A(16x8, row) * B(8x8, col), tf32 in, fp32 accumulate.
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int NW, int S>
__global__ void __launch_bounds__(NW * 32) paged_decode_tf32_kernel(
    const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
    ArenaGeom g, DecodeWork w, DecodeArgs a, int group, int cpp) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms (1 KB slack is allocated)
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int hg = blockIdx.y;
    const int worker = blockIdx.x * NW + warp;
    const int gq = lane >> 2;   // query head of this lane's S rows / softmax
    const int tig = lane & 3;   // token pair 2*tig, 2*tig+1; accumulator heads 2*tig, 2*tig+1

    unsigned char* my_stages = smem + static_cast<size_t>(warp) * S * kStage;
    uint64_t* my_bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(NW) * S * kStage) + warp * S;
    if (lane < S) mbar_init(&my_bars[lane], 1);
    fence_mbar_init();
    __syncwarp();
    // the next kernel (the deferred merge) may be scheduled as soon as this grid is resident
    pdl_launch_dependents();

    // the work list comes from a host copy ordered before the previous kernel, so it is read
    // before pdl_wait; the arena (which a preceding append writes) only after it
    const int pb = __ldg(w.worker_piece_begin + worker);
    const int pe = __ldg(w.worker_piece_begin + worker + 1);
    if (pb >= pe) {
        pdl_wait();
        return;
    }

    const int bs = g.block_size;
    const bool cpp2 = (cpp == 2);
    auto chunk_geom = [&](int c, int ctx, int& page, int& tok0, int& ntok) {
        if (cpp2) {
            page = c >> 1;
            tok0 = (c & 1) * kChunk;
        } else {
            page = c / cpp;
            tok0 = (c - page * cpp) * kChunk;
        }
        int nt = bs - tok0;
        nt = nt < kChunk ? nt : kChunk;
        const int rem = ctx - page * bs - tok0;
        ntok = nt < rem ? nt : rem;
    };

    // ---- producer: lanes 0-7 issue the chunk's eight boxes, one each ----
    int p_piece = pb, p_j = 0, p_c0 = 0, p_cnt = 0, p_b = 0, p_h = 0, p_ctx = 0;
    auto p_load = [&]() {
        const int seg = __ldg(w.piece_seg + p_piece);
        p_b = seg / g.heads_kv;
        p_h = seg - p_b * g.heads_kv;
        p_c0 = __ldg(w.piece_c0 + p_piece);
        p_cnt = __ldg(w.piece_c1 + p_piece) - p_c0;
        p_ctx = __ldg(w.ctx_lens + p_b);
    };
    p_load();
    pdl_wait();
    auto issue = [&](int st) {
        int page, tok0, ntok;
        chunk_geom(p_c0 + p_j, p_ctx, page, tok0, ntok);
        int64_t blk = 0;
        if (lane == 0) blk = __ldg(w.tables + table_row(w, p_b) * w.max_blocks + page);
        blk = __shfl_sync(0xffffffffu, blk, 0);
        uint64_t* bar = &my_bars[st];
        const bool ok = blk >= 0 && blk < g.total_blocks && ntok > 0;
        if (lane == 0) {
            if (ok) {
                mbar_arrive_expect_tx(bar, kStage);
            } else {
                if (a.err) atomicOr(a.err, kErrBadBlock);
                mbar_arrive(bar);
            }
        }
        __syncwarp();  // the expected byte count precedes every box's completion
        if (ok && lane < 8) {
            const int z = static_cast<int>((blk * g.layers + a.layer) * g.heads_kv + p_h);
            unsigned char* dst = my_stages + static_cast<size_t>(st) * kStage + lane * kBox;
            fence_proxy_async_smem();
            tma_load_3d(dst, lane < 4 ? static_cast<const void*>(&tmk) : static_cast<const void*>(&tmv),
                        (lane & 3) * 32, tok0, z, bar);
        }
        if (++p_j >= p_cnt) {
            p_j = 0;
            if (++p_piece < pe) p_load();
        }
    };
#pragma unroll 1
    for (int s = 0; s < S && p_piece < pe; ++s) issue(s);

    bool dead = false;
    int ck = 0;
    const float scale_log2 = a.scale * kLog2e;

#pragma unroll 1
    for (int i = pb; i < pe; ++i) {
        const int seg = __ldg(w.piece_seg + i);
        const int c0 = __ldg(w.piece_c0 + i);
        const int cnt = __ldg(w.piece_c1 + i) - c0;
        const int b = seg / g.heads_kv;
        const int h = seg - b * g.heads_kv;
        const int ctx = __ldg(w.ctx_lens + b);
        const int q_head0 = h * group + hg * kGP;
        const int gcount = min(kGP, group - hg * kGP);

        // Q A-fragments of k-step s (rows = heads; rows 8..15 are zero): a0 = q[dim 8s + 2t],
        // a2 = q[dim 8s + 2t + 1], high and low TF32 parts
        uint32_t qh[16][2], ql[16][2];
        {
            const bool live = gq < gcount;
            const float* qp = a.q + (static_cast<int64_t>(b) * a.n_heads + q_head0 + gq) * kD + 2 * tig;
#pragma unroll
            for (int s = 0; s < 16; ++s) {
                const float2 v = live ? __ldg(reinterpret_cast<const float2*>(qp + 8 * s)) : make_float2(0.f, 0.f);
                split_tf32(v.x, qh[s][0], ql[s][0]);
                split_tf32(v.y, qh[s][1], ql[s][1]);
            }
        }
        float acc[8][4];
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
        float m_own = -INFINITY, l_own = 0.f;     // head gq
        float mc0 = -INFINITY, mc1 = -INFINITY;   // heads 2*tig, 2*tig+1 (accumulator columns)

#pragma unroll 1
        for (int j = 0; j < cnt; ++j) {
            const int st = ck % S;
            const uint32_t ph = static_cast<uint32_t>(ck / S) & 1u;
            int page, tok0, ntok;
            chunk_geom(c0 + j, ctx, page, tok0, ntok);
            // warp-uniform: the MMAs below and the refill are warp-collective
            if (!dead && !__all_sync(0xffffffffu, mbar_wait(&my_bars[st], ph))) {
                dead = true;
                if (lane == 0 && a.err) atomicOr(a.err, kErrWaitTimeout);
            }
            if (!dead && ntok > 0) {
                const unsigned char* stage = my_stages + static_cast<size_t>(st) * kStage;
                // ---- S = Q . K^T: six accumulator chains (three products x two k-step parities)
                float sa[6][4];
#pragma unroll
                for (int c = 0; c < 6; ++c) sa[c][0] = sa[c][1] = sa[c][2] = sa[c][3] = 0.f;
#pragma unroll
                for (int s = 0; s < 16; ++s) {
                    // K[token gq][dims 8s + 2t, 8s + 2t + 1] of box s/4
                    const float2 kv = *reinterpret_cast<const float2*>(
                        stage + (s >> 2) * kBox + swz32(gq, 8 * (s & 3) + 2 * tig));
                    uint32_t kh0, kl0, kh1, kl1;
                    split_tf32(kv.x, kh0, kl0);
                    split_tf32(kv.y, kh1, kl1);
                    float (&d0)[4] = sa[(s & 1) * 3 + 0];
                    float (&d1)[4] = sa[(s & 1) * 3 + 1];
                    float (&d2)[4] = sa[(s & 1) * 3 + 2];
                    mma_tf32(d0, qh[s][0], 0u, qh[s][1], 0u, kh0, kh1);
                    mma_tf32(d1, ql[s][0], 0u, ql[s][1], 0u, kh0, kh1);
                    mma_tf32(d2, qh[s][0], 0u, qh[s][1], 0u, kl0, kl1);
                }
                float sc[2];
#pragma unroll
                for (int e = 0; e < 2; ++e)
                    sc[e] = ((sa[0][e] + sa[3][e]) + (sa[1][e] + sa[4][e])) + (sa[2][e] + sa[5][e]);
                // ---- online softmax of head gq over tokens 2*tig, 2*tig+1 ----
                const bool v0 = 2 * tig < ntok, v1 = 2 * tig + 1 < ntok;
                const float s0 = v0 ? sc[0] * scale_log2 : -INFINITY;
                const float s1 = v1 ? sc[1] * scale_log2 : -INFINITY;
                float cmax = fmaxf(s0, s1);
                cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
                cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
                const float m_new = fmaxf(m_own, cmax);
                const float p0 = exp2f(s0 - m_new), p1 = exp2f(s1 - m_new);
                float psum = p0 + p1;
                psum += __shfl_xor_sync(0xffffffffu, psum, 1);
                psum += __shfl_xor_sync(0xffffffffu, psum, 2);
                const bool changed = m_new > m_own;
                l_own = l_own * exp2f(m_own - m_new) + psum;
                m_own = m_new;
                if (__any_sync(0xffffffffu, changed)) {
                    const float n0 = __shfl_sync(0xffffffffu, m_own, (2 * tig) * 4);
                    const float n1 = __shfl_sync(0xffffffffu, m_own, (2 * tig + 1) * 4);
                    const float a0 = exp2f(mc0 - n0), a1 = exp2f(mc1 - n1);
                    mc0 = n0;
                    mc1 = n1;
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        acc[t][0] *= a0;
                        acc[t][2] *= a0;
                        acc[t][1] *= a1;
                        acc[t][3] *= a1;
                    }
                }
                // ---- O^T += V^T . P^T over tokens (2t, 2t+1) = (k, k + 4) of the MMA ----
                uint32_t ph0, pl0, ph1, pl1;
                split_tf32(p0, ph0, pl0);
                split_tf32(p1, ph1, pl1);
                const unsigned char* vst = stage + 4 * kBox;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    // V[token][dv 16*mt + g (+8)]: box mt/2, column 16*(mt%2) + g (+8)
                    const unsigned char* vb = vst + (mt >> 1) * kBox;
                    const int col = 16 * (mt & 1) + gq;
                    // stale slots past the chunk's end are zeroed so that P = 0 never meets NaN
                    const float va0 = v0 ? *reinterpret_cast<const float*>(vb + swz32(2 * tig, col)) : 0.f;
                    const float va1 = v0 ? *reinterpret_cast<const float*>(vb + swz32(2 * tig, col + 8)) : 0.f;
                    const float va2 = v1 ? *reinterpret_cast<const float*>(vb + swz32(2 * tig + 1, col)) : 0.f;
                    const float va3 = v1 ? *reinterpret_cast<const float*>(vb + swz32(2 * tig + 1, col + 8)) : 0.f;
                    uint32_t ah0, al0, ah1, al1, ah2, al2, ah3, al3;
                    split_tf32(va0, ah0, al0);
                    split_tf32(va1, ah1, al1);
                    split_tf32(va2, ah2, al2);
                    split_tf32(va3, ah3, al3);
                    mma_tf32(acc[mt], ah0, ah1, ah2, ah3, ph0, ph1);
                    mma_tf32(acc[mt], al0, al1, al2, al3, ph0, ph1);
                    mma_tf32(acc[mt], ah0, ah1, ah2, ah3, pl0, pl1);
                }
            }
            __syncwarp();
            if (p_piece < pe && !dead) issue(st);
            ++ck;
        }
        if (dead) continue;

        // ---- end of piece ----
        const int hA = 2 * tig, hB = 2 * tig + 1;  // this lane's accumulator heads
        const float lA = __shfl_sync(0xffffffffu, l_own, hA * 4);
        const float lB = __shfl_sync(0xffffffffu, l_own, hB * 4);
        const float mA = __shfl_sync(0xffffffffu, m_own, hA * 4);
        const float mB = __shfl_sync(0xffffffffu, m_own, hB * 4);
        const int slot = __ldg(w.piece_slot + i);
        if (slot < 0) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int hh = cc ? hB : hA;
                if (hh >= gcount) continue;
                const float mm = cc ? mB : mA;
                float Ls = cc ? lB : lA, f = 1.f, Mref = mm;
                const int qh2 = q_head0 + hh;
                if (a.sinks || a.has_sink_all) {
                    const float sk = (a.sinks ? __ldg(a.sinks + qh2) : a.sink_all) * kLog2e;
                    const float M2 = fmaxf(mm, sk);
                    f = (mm == -INFINITY) ? 0.f : exp2f(mm - M2);
                    Ls = Ls * f + exp2f(sk - M2);
                    Mref = M2;
                }
                const float inv = Ls > 0.f ? f / Ls : 0.f;
                if (a.lse && gq == 0) a.lse[static_cast<int64_t>(b) * a.n_heads + qh2] = lse_ln(Mref, Ls);
                float* op = a.out + (static_cast<int64_t>(b) * a.n_heads + qh2) * kDV;
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    op[16 * t + gq] = acc[t][cc] * inv;
                    op[16 * t + gq + 8] = acc[t][cc + 2] * inv;
                }
            }
        } else {
            const int64_t base = (static_cast<int64_t>(hg) * w.n_slots + slot) * kGP;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                float* ap = a.part_acc + (base + (cc ? hB : hA)) * kDV;
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    ap[16 * t + gq] = acc[t][cc];
                    ap[16 * t + gq + 8] = acc[t][cc + 2];
                }
            }
            {
                const float mm = __shfl_sync(0xffffffffu, m_own, (lane & 7) * 4);
                const float ll = __shfl_sync(0xffffffffu, l_own, (lane & 7) * 4);
                if (lane < kGP) {
                    a.part_ml[(base + lane) * 2 + 0] = mm;
                    a.part_ml[(base + lane) * 2 + 1] = ll;
                }
            }
            const int mix = __ldg(w.piece_merge + i);
            if (mix >= 0) {  // merged here; otherwise the deferred-merge kernel does it
                const int ns = __ldg(w.merge_nslots + mix);
                __threadfence();
                __syncwarp();
                int prev = 0;
                int* counter = w.merge_count + static_cast<int64_t>(hg) * w.n_merge + mix;
                if (lane == 0) prev = atomicAdd(counter, 1);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == ns - 1) {
                    __threadfence();
                    merge_segment<kGP, kDV>(a, w, hg, __ldg(w.merge_slot0 + mix), ns, b, q_head0, gcount, lane);
                    if (lane == 0) atomicExch(counter, 0);
                }
            }
        }
    }
}

constexpr size_t kTf32Smem = static_cast<size_t>(kNW) * kS * kStage + kNW * kS * 8 + 1024;

cudaError_t tf32_prepare() {
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(paged_decode_tf32_kernel<kNW, kS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kTf32Smem));
    if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace

bool decode_tf32_eligible(const ArenaGeom& g, int n_heads) {
    if (g.dtype != GKV_DTYPE_F32 || g.head_dim != kD || g.v_head_dim != kDV) return false;
    if (g.block_size % kChunk != 0 || g.heads_kv <= 0 || n_heads % g.heads_kv != 0) return false;
    const int group = n_heads / g.heads_kv;
    if (group < 5) return false;  // gp 8 only; smaller groups are HBM-bound on the FP32 pipe
    if ((reinterpret_cast<uintptr_t>(g.k) | reinterpret_cast<uintptr_t>(g.v)) & 15) return false;
    const int64_t rows = static_cast<int64_t>(g.total_blocks) * g.layers * g.heads_kv;
    return rows < (int64_t{1} << 31) && tmap_encoder_available();
}

void decode_tf32_config(DecodeConfig& c) {
    c.warps = kNW;
    c.threads = kNW * 32;
    c.smem = kTf32Smem;
    int per_sm = 1;
    if (tf32_prepare() != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_tf32_kernel<kNW, kS>, c.threads,
                                                      kTf32Smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    c.ctas_per_sm = per_sm;
    c.supported = true;
}

cudaError_t launch_paged_decode_tf32(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                     int group, int head_groups, int* launches, cudaStream_t st) {
    // cached maps of the pool when present, else encoded here (host only, no allocation)
    alignas(64) CUtensorMap ek;
    alignas(64) CUtensorMap ev;
    const CUtensorMap* tk = static_cast<const CUtensorMap*>(g.tmap_k);
    const CUtensorMap* tv = static_cast<const CUtensorMap*>(g.tmap_v);
    if (!tk || !tv) {
        if (!encode_f32_arena_map(&ek, g.k, g, kD) || !encode_f32_arena_map(&ev, g.v, g, kDV))
            return cudaErrorInvalidValue;
        tk = &ek;
        tv = &ev;
    }
    cudaError_t e = tf32_prepare();
    if (e != cudaSuccess) return e;
    const int cpp = (g.block_size + kChunk - 1) / kChunk;
    dim3 grid(static_cast<unsigned>(w.n_ctas), static_cast<unsigned>(head_groups));
    e = launch_pdl(paged_decode_tf32_kernel<kNW, kS>, grid, dim3(kNW * 32), kTf32Smem, st, *tk, *tv, g, w, a,
                   group, cpp);
    if (e != cudaSuccess) return e;
    *launches = 1;
    if (w.n_deferred > 0) {
        e = launch_deferred_merge(g, w, a, group, kGP, head_groups, st);
        if (e == cudaSuccess) *launches = 2;
    }
    return e;
}

}  // namespace gkv
