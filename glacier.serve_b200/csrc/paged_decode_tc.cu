// Tensor-core variant of the split-KV paged decode for 16-bit KV (bf16 or fp16) with wide GQA
// groups.
//
// Same work decomposition, work list, partial layout and fused merge as paged_decode.cu
// (warp-level stream-K over 8-token chunks of (sequence, kv head) segments), for bf16 or fp16
// KV, d = dv = 128, block size a multiple of 8 and a query group of 5..8 heads (gp = 8): the
// configurations where the CUDA-core kernel is limited by the FP32 pipe, not by HBM
// (arithmetic intensity 2 * group / 2 bytes = 7-8 FLOP per KV byte).  Per chunk:
//
//  * Two tiled TMA loads (cp.async.bulk.tensor, 128-byte swizzle, no multicast) bring the
//    chunk's K rows and two bring its V rows: boxes of 8 tokens x 64 dims (1 KB each) from
//    a 3-D view [block*layer*head][slot][dim] of this GPU's own arena.  The swizzle makes the
//    ldmatrix reads below bank-conflict free.  (One 4-D box per operand -- both halves in one
//    2 KB copy -- measured the same on the full batch and 2 % slower on an 8th of it.)
//  * S^T[8 heads x 8 tokens] = Q . K^T with mma.m16n8k16 (16-bit in, fp32 accumulate; rows
//    8..15 of the A operand are zero).  Q is split into hi + lo parts of the arena's type (two
//    MMAs), so the scores carry ~16 (bf16) or ~22 (fp16) mantissa bits of q; K is exact.  For
//    fp16, q is first scaled by a power of two that brings the head group's largest |q| into
//    [2^13, 2^14) (exact; the scores are scaled back through the softmax scale), so any fp32 q
//    fits the fp16 range.  The accumulator fragment leaves
//    lane L holding head L/4 for tokens 2*(L%4) and 2*(L%4)+1.
//  * Online softmax on those fragments (base 2, max/sum over the 4 lanes of a head).
//  * O^T[128 dv x 8 heads] += V^T . P^T with mma.m16n8k8: the B fragment is exactly the
//    lane's own two probabilities (split hi + lo again), V^T comes from ldmatrix.trans.
//
// ~130 instructions per chunk instead of ~650 on the FP32 pipe.  Roofline: HBM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "decode_merge.cuh"
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

constexpr int kChunk = kDecodeChunk;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kGP = 8, kD = 128, kDV = 128;
constexpr int kBox = 1024;           // one box: 8 rows x 128 bytes
constexpr int kStage = 4 * kBox;     // K dims 0-63, K dims 64-127, V 0-63, V 64-127
constexpr int kNW = 4;               // warp workers per CTA (as the CUDA-core kernel)
constexpr int kS = 4;                // ring stages per warp (3 CTAs, 12 warps per SM)

__device__ __forceinline__ uint32_t swz(int row, int chunk16) {
    return static_cast<uint32_t>(row * 128 + ((chunk16 ^ row) << 4));
}

// DYN: the static step layout (the work list comes from the header at w.dyn); a separate
// instantiation, so the by-value work list of the normal launch stays in the parameter bank.
template <int NW, int S, bool F16, bool DYN>
__global__ void __launch_bounds__(NW * 32) paged_decode_tc_kernel(
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
    if constexpr (DYN) w = resolve_work(w);
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

    // ---- producer (lane 0): four box loads per chunk ----
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
    // Lanes 0-3 issue the chunk's four boxes, one each: a TMA instruction occupies its issuing
    // thread for on the order of a hundred cycles, so four from one lane would hold the warp
    // about as long as the chunk's math.
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
        if (ok && lane < 4) {
            const int z = static_cast<int>((blk * g.layers + a.layer) * g.heads_kv + p_h);
            unsigned char* dst = my_stages + static_cast<size_t>(st) * kStage + lane * kBox;
            fence_proxy_async_smem();
            tma_load_3d(dst, lane < 2 ? static_cast<const void*>(&tmk) : static_cast<const void*>(&tmv),
                        (lane & 1) * 64, tok0, z, bar);
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
    // per-lane ldmatrix offsets (bytes within a stage): matrix mi = lane/8, row = lane%8
    const int mi = lane >> 3, rr = lane & 7;

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

        // Q A-fragments (rows = heads; rows 8..15 are zero), hi and lo parts per k-step
        uint32_t qh[8][2], ql[8][2];
        float piece_scale_log2 = scale_log2;
        {
            const bool live = gq < gcount;
            const float* qp = a.q + (static_cast<int64_t>(b) * a.n_heads + q_head0 + gq) * kD;
            float qv[8][2][2];
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int d0 = ks * 16 + half * 8 + tig * 2;
                    qv[ks][half][0] = live ? __ldg(qp + d0) : 0.f;
                    qv[ks][half][1] = live ? __ldg(qp + d0 + 1) : 0.f;
                }
            }
            float qs = 1.f;
            if constexpr (F16) {
                // power-of-two scale 2^-e with max|q| * 2^-e in [2^13, 2^14)
                float mx = 0.f;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
#pragma unroll
                    for (int half = 0; half < 2; ++half)
                        mx = fmaxf(mx, fmaxf(fabsf(qv[ks][half][0]), fabsf(qv[ks][half][1])));
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                const int ef = static_cast<int>((__float_as_uint(mx) >> 23) & 0xffu);
                int e = (ef == 0 || ef == 0xff) ? 0 : ef - 126 - 14;  // mx < 2^(ef-126)
                e = e < -100 ? -100 : (e > 100 ? 100 : e);
                qs = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
                piece_scale_log2 = scale_log2 * __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
            }
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float h0, l0, h1, l1;
                    split_16<F16>(qv[ks][half][0] * qs, h0, l0);
                    split_16<F16>(qv[ks][half][1] * qs, h1, l1);
                    qh[ks][half] = pack_16x2<F16>(h0, h1);
                    ql[ks][half] = pack_16x2<F16>(l0, l1);
                }
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
            const int64_t blk = __ldg(w.tables + table_row(w, b) * w.max_blocks + page);
            // warp-uniform: the MMAs below and the refill are warp-collective
            if (!dead && !__all_sync(0xffffffffu, mbar_wait(&my_bars[st], ph))) {
                dead = true;
                if (lane == 0 && a.err) atomicOr(a.err, kErrWaitTimeout);
            }
            if (!dead && blk >= 0 && blk < g.total_blocks && ntok > 0) {
                const uint32_t sb = smem_u32(my_stages + static_cast<size_t>(st) * kStage);
                // ---- S^T = Q . K^T: four independent accumulator chains of 4 MMAs ----
                float sa[4][4];
#pragma unroll
                for (int c = 0; c < 4; ++c) sa[c][0] = sa[c][1] = sa[c][2] = sa[c][3] = 0.f;
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int dbase = 32 * jj + 8 * mi;
                    const uint32_t addr = sb + (dbase >> 6) * kBox + swz(rr, (dbase & 63) >> 3);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(addr, b0, b1, b2, b3);
                    mma_16816<F16>(sa[0], qh[2 * jj][0], 0u, qh[2 * jj][1], 0u, b0, b1);
                    mma_16816<F16>(sa[1], ql[2 * jj][0], 0u, ql[2 * jj][1], 0u, b0, b1);
                    mma_16816<F16>(sa[2], qh[2 * jj + 1][0], 0u, qh[2 * jj + 1][1], 0u, b2, b3);
                    mma_16816<F16>(sa[3], ql[2 * jj + 1][0], 0u, ql[2 * jj + 1][1], 0u, b2, b3);
                }
                float s[2];
                s[0] = (sa[0][0] + sa[2][0]) + (sa[1][0] + sa[3][0]);
                s[1] = (sa[0][1] + sa[2][1]) + (sa[1][1] + sa[3][1]);
                // ---- online softmax of head gq over tokens 2*tig, 2*tig+1 ----
                const bool v0 = 2 * tig < ntok, v1 = 2 * tig + 1 < ntok;
                const float s0 = v0 ? s[0] * piece_scale_log2 : -INFINITY;
                const float s1 = v1 ? s[1] * piece_scale_log2 : -INFINITY;
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
                // ---- O^T += V^T . P^T ----
                float ph0, pl0, ph1, pl1;
                split_16<F16>(p0, ph0, pl0);
                split_16<F16>(p1, ph1, pl1);
                const uint32_t bh = pack_16x2<F16>(ph0, ph1);
                const uint32_t bl = pack_16x2<F16>(pl0, pl1);
                // zero the V^T elements of tokens past the chunk's end (stale slots)
                const uint32_t vmask = (v0 ? 0x0000ffffu : 0u) | (v1 ? 0xffff0000u : 0u);
#pragma unroll
                for (int pp = 0; pp < 4; ++pp) {
                    const int vbase = 32 * pp + 8 * mi;
                    const uint32_t addr = sb + 2 * kBox + (vbase >> 6) * kBox + swz(rr, (vbase & 63) >> 3);
                    uint32_t r0, r1, r2, r3;
                    ldsm_x4_trans(addr, r0, r1, r2, r3);
                    r0 &= vmask;
                    r1 &= vmask;
                    r2 &= vmask;
                    r3 &= vmask;
                    mma_1688<F16>(acc[2 * pp], r0, r1, bh);
                    mma_1688<F16>(acc[2 * pp], r0, r1, bl);
                    mma_1688<F16>(acc[2 * pp + 1], r2, r3, bh);
                    mma_1688<F16>(acc[2 * pp + 1], r2, r3, bl);
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

constexpr size_t kTcSmem = static_cast<size_t>(kNW) * kS * kStage + kNW * kS * 8 + 1024;

cudaError_t tc_prepare() {
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
    for (auto k : {paged_decode_tc_kernel<kNW, kS, false, false>, paged_decode_tc_kernel<kNW, kS, true, false>,
                   paged_decode_tc_kernel<kNW, kS, false, true>, paged_decode_tc_kernel<kNW, kS, true, true>})
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTcSmem));
    if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

bool tmap_encoder_available() { return encode_fn() != nullptr; }

// Tiled map with 128-byte swizzle and no interleave; rank <= 5.
static bool encode_map(void* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
                       const uint64_t* strides, const uint32_t* box) {
    auto fn = encode_fn();
    if (!fn || rank < 1 || rank > 5) return false;
    cuuint64_t d[5], s[4];
    cuuint32_t b[5], estr[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        estr[i] = 1;
        if (i + 1 < rank) s[i] = strides[i];
    }
    return fn(static_cast<CUtensorMap*>(map), type, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The element type only sets the element size here (2 bytes): TMA copies bf16 and fp16 tiles
// alike, so one encoder serves both arenas.
bool encode_bf16_map3(void* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                      const uint32_t box[3]) {
    return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box);
}

// 3-D view [dim byte][slot][block * layer * head] of one FP8 arena (d = 128), 8-slot boxes.
static bool encode_fp8_map(void* map, void* base, const ArenaGeom& g, int dim) {
    if (dim != 128 || g.block_size % kChunk != 0) return false;
    const uint64_t dims[3] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(g.block_size),
                              static_cast<uint64_t>(g.total_blocks) * g.layers * g.heads_kv};
    const uint64_t strides[2] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(g.block_size) * dim};
    const uint32_t box[3] = {static_cast<uint32_t>(dim), static_cast<uint32_t>(kChunk), 1};
    return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box);
}

// 3-D view [block * layer * head][slot][dim] of one 16-bit arena, boxes of `rows` slots x 64 dims.
bool encode_arena_map(void* map, void* base, const ArenaGeom& g, int dim, int rows) {
    if (rows <= 0 || g.block_size % rows != 0) return false;
    const uint64_t dims[3] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(g.block_size),
                              static_cast<uint64_t>(g.total_blocks) * g.layers * g.heads_kv};
    const uint64_t strides[2] = {static_cast<uint64_t>(dim) * 2, static_cast<uint64_t>(g.block_size) * dim * 2};
    const uint32_t box[3] = {64, static_cast<uint32_t>(rows), 1};
    return encode_bf16_map3(map, base, dims, strides, box);
}

int encode_decode_tmaps(const ArenaGeom& g, void* tmap_k, void* tmap_v) {
    if (g.dtype == GKV_DTYPE_FP8_E4M3)
        return encode_fp8_map(tmap_k, g.k, g, g.head_dim) && encode_fp8_map(tmap_v, g.v, g, g.v_head_dim) ? 3 : 0;
    return encode_arena_map(static_cast<CUtensorMap*>(tmap_k), g.k, g, kD) &&
                   encode_arena_map(static_cast<CUtensorMap*>(tmap_v), g.v, g, kDV)
               ? 3
               : 0;
}

bool decode_tc_eligible(const ArenaGeom& g, int n_heads) {
    if ((g.dtype != GKV_DTYPE_BF16 && g.dtype != GKV_DTYPE_F16) || g.head_dim != kD || g.v_head_dim != kDV)
        return false;
    if (g.block_size % kChunk != 0 || g.heads_kv <= 0 || n_heads % g.heads_kv != 0) return false;
    const int group = n_heads / g.heads_kv;
    if (group < 5) return false;  // gp 8 only; smaller groups are HBM-bound on the FP32 pipe
    if ((reinterpret_cast<uintptr_t>(g.k) | reinterpret_cast<uintptr_t>(g.v)) & 15) return false;
    const int64_t rows = static_cast<int64_t>(g.total_blocks) * g.layers * g.heads_kv;
    return rows < (int64_t{1} << 31) && tmap_encoder_available();
}

void decode_tc_config(DecodeConfig& c) {
    c.warps = kNW;
    c.threads = kNW * 32;
    c.smem = kTcSmem;
    int per_sm = 1;
    if (tc_prepare() != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_tc_kernel<kNW, kS, false, false>, c.threads,
                                                      kTcSmem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    c.ctas_per_sm = per_sm;
    c.supported = true;
}

cudaError_t launch_paged_decode_tc(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                   int group, int head_groups, int* launches, cudaStream_t st) {
    // cached maps of the pool when present, else encoded here (host only, no allocation)
    CUtensorMap ek, ev;
    const CUtensorMap* tk = static_cast<const CUtensorMap*>(g.tmap_k);
    const CUtensorMap* tv = static_cast<const CUtensorMap*>(g.tmap_v);
    ArenaGeom gl = g;
    if (!tk || !tv) {
        gl.tmap_rank = encode_decode_tmaps(g, &ek, &ev);
        if (gl.tmap_rank == 0) return cudaErrorInvalidValue;
        tk = &ek;
        tv = &ev;
    }
    cudaError_t e = tc_prepare();
    if (e != cudaSuccess) return e;
    const int cpp = (g.block_size + kChunk - 1) / kChunk;
    dim3 grid(static_cast<unsigned>(w.n_ctas), static_cast<unsigned>(head_groups));
    auto go = [&](auto kern) {
        return launch_pdl(kern, grid, dim3(kNW * 32), kTcSmem, st, *tk, *tv, gl, w, a, group, cpp);
    };
    const bool f16 = g.dtype == GKV_DTYPE_F16;
    if (w.dyn)
        e = f16 ? go(paged_decode_tc_kernel<kNW, kS, true, true>) : go(paged_decode_tc_kernel<kNW, kS, false, true>);
    else
        e = f16 ? go(paged_decode_tc_kernel<kNW, kS, true, false>) : go(paged_decode_tc_kernel<kNW, kS, false, false>);
    if (e != cudaSuccess) return e;
    *launches = 1;
    if (w.n_deferred > 0 || w.merge_grid > 0) {
        e = launch_deferred_merge(gl, w, a, group, kGP, head_groups, st);
        if (e == cudaSuccess) *launches = 2;
    }
    return e;
}

}  // namespace gkv
