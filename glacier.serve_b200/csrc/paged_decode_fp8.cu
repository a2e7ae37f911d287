// Tensor-core split-KV paged decode for FP8 E4M3 KV (one K and one V scale per (layer, kv
// head)), wide GQA groups, d = dv = 128, block size a multiple of 8.
//
// Same work decomposition, work list, partial layout and merges as paged_decode.cu /
// paged_decode_tc.cu (warp-level stream-K over 8-token chunks of (sequence, kv head)
// segments).  An e4m3 value widens exactly to fp16, so the chunk's K and V feed fp16
// mma.sync with no loss; q and p are split into fp16 hi + lo as in the fp16 tensor-core
// kernel.  What differs is how the operands reach the registers:
//
//  * Fetch: two tiled TMA loads per chunk (cp.async.bulk.tensor, 128-byte swizzle, no
//    multicast), one box of 8 token rows x 128 bytes for K and one for V, into a per-warp ring.
//    (An earlier form with one K span and four padded V spans per chunk, plain bulk copies,
//    measured 0.319 ms on cfg3-fp8 against 0.288 ms for this one.)  The swizzle stores 16-byte
//    chunk c of row r at chunk c ^ r, which makes both read patterns below bank-conflict free.
//  * S^T[8 heads x 8 tokens] = Q . K^T with mma.m16n8k16.  The reduction over the 128 dims
//    may visit them in any order that A and B share: k-step ks of lane (g, t) = (lane / 4,
//    lane % 4) takes dims 32t + 4ks + {0,1} (fragment registers 0) and + {2,3} (registers 1).
//    So a lane's K operand for all eight k-steps is the 32 contiguous bytes [32t, 32t + 32) of
//    token row g: two 16-byte shared loads and sixteen e4m3x2 -> f16x2 conversions.
//  * O^T[128 dv x 8 heads] += V^T . P^T with mma.m16n8k8.  The B fragment is the lane's own
//    two probabilities (tokens 2t, 2t+1 of head g) as in the fp16 kernel; the A fragment pairs
//    tokens 2t and 2t+1 of one dv.  The dv rows may be assigned freely: tile m's row g is dv
//    16g + 2m and row g + 8 is dv 16g + 2m + 1, so lane (g, t) needs bytes [16g, 16g + 16)
//    of token rows 2t and 2t+1 -- two 16-byte loads, eight byte permutes (pairing the two
//    rows) and sixteen conversions -- and ends up holding sixteen CONTIGUOUS dv of heads 2t
//    and 2t+1, written with float4 stores.
//  * The K scale folds into the piece's score scale, the V scale into its output or partial.
//
// Roofline: HBM.  Algorithmic bytes per chunk = 8 x (128 + 128) x 1.
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
constexpr int kKBytes = kChunk * kD;  // 1 KB box of K rows per chunk (and one of V rows)
constexpr int kStage = 2 * kKBytes;   // 2 KB; stages are 1024-byte aligned for the swizzle
constexpr int kNW = 4;                // warp workers per CTA (as the other decodes)
constexpr int kS = 8;                 // ring stages per warp: 4 x 8 x 2 KB = 64 KB per CTA

// Byte offset of 16-byte chunk c of row r (< 8) in a box written with the 128-byte swizzle.
__device__ __forceinline__ int swz8(int r, int c) { return r * 128 + ((c ^ r) << 4); }

__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t pair16) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(pair16), __NV_E4M3);
    return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

template <int NW, int S, bool DYN>
__global__ void __launch_bounds__(NW * 32) paged_decode_fp8_kernel(const __grid_constant__ CUtensorMap tmk,
                                                                   const __grid_constant__ CUtensorMap tmv,
                                                                   ArenaGeom g, DecodeWork w, DecodeArgs a, int group,
                                                                   int cpp) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms (1 KB slack is allocated)
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int hg = blockIdx.y;
    const int worker = blockIdx.x * NW + warp;
    if constexpr (DYN) w = resolve_work(w);
    const int gq = lane >> 2;   // head of this lane's S rows / softmax; token row of its K reads
    const int tig = lane & 3;   // tokens 2*tig, 2*tig+1; accumulator heads 2*tig, 2*tig+1

    unsigned char* my_stages = smem + static_cast<size_t>(warp) * S * kStage;
    uint64_t* my_bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(NW) * S * kStage) + warp * S;
    if (lane < S) mbar_init(&my_bars[lane], 1);
    fence_mbar_init();
    __syncwarp();
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

    // ---- producer: lanes 0 and 1 issue the chunk's K and V boxes ----
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
                // whole 8-row boxes (the block size is a multiple of 8, so every row of the box is a
                // slot of this page); rows past ntok are masked below
                mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kStage));
            } else {
                if (a.err) atomicOr(a.err, kErrBadBlock);
                mbar_arrive(bar);
            }
        }
        __syncwarp();  // the expected byte count precedes every copy's completion
        if (ok && lane < 2) {
            const int z = static_cast<int>((blk * g.layers + a.layer) * g.heads_kv + p_h);
            unsigned char* dst = my_stages + static_cast<size_t>(st) * kStage + lane * kKBytes;
            fence_proxy_async_smem();
            tma_load_3d(dst, lane == 0 ? static_cast<const void*>(&tmk) : static_cast<const void*>(&tmv), 0, tok0, z,
                        bar);
        }
        if (++p_j >= p_cnt) {
            p_j = 0;
            if (++p_piece < pe) p_load();
        }
    };
    // Only the first stage goes out at launch: with every warp of the grid requesting at once,
    // each warp's first chunk lands sooner when it is alone in the queue; the other stages
    // follow as soon as it has landed.
    if (p_piece < pe) issue(0);
    bool primed = S == 1;

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
        const float ksc = __ldg(g.k_scale + a.layer * g.heads_kv + h);
        const float vsc = __ldg(g.v_scale + a.layer * g.heads_kv + h);

        // Q A-fragments of head gq (rows 8..15 zero): k-step ks, registers 0 / 1 = dims
        // 32*tig + 4*ks + {0,1} / {2,3}; hi and lo fp16 parts after a power-of-two scale that
        // brings the group's largest |q| into [2^13, 2^14)
        uint32_t qh[8][2], ql[8][2];
        float piece_scale_log2 = scale_log2 * ksc;
        {
            const bool live = gq < gcount;
            const float* qp = a.q + (static_cast<int64_t>(b) * a.n_heads + q_head0 + gq) * kD + 32 * tig;
            float qv[32];
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
                const float4 x = live ? __ldg(reinterpret_cast<const float4*>(qp + e)) : make_float4(0.f, 0.f, 0.f, 0.f);
                qv[e] = x.x;
                qv[e + 1] = x.y;
                qv[e + 2] = x.z;
                qv[e + 3] = x.w;
            }
            float mx = 0.f;
#pragma unroll
            for (int e = 0; e < 32; ++e) mx = fmaxf(mx, fabsf(qv[e]));
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const int ef = static_cast<int>((__float_as_uint(mx) >> 23) & 0xffu);
            int e = (ef == 0 || ef == 0xff) ? 0 : ef - 126 - 14;  // mx < 2^(ef-126)
            e = e < -100 ? -100 : (e > 100 ? 100 : e);
            const float qs = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
            piece_scale_log2 *= __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    float h0, l0, h1, l1;
                    split_16<true>(qv[4 * ks + 2 * r] * qs, h0, l0);
                    split_16<true>(qv[4 * ks + 2 * r + 1] * qs, h1, l1);
                    qh[ks][r] = pack_16x2<true>(h0, h1);
                    ql[ks][r] = pack_16x2<true>(l0, l1);
                }
            }
        }
        float acc[8][4];
#pragma unroll
        for (int m = 0; m < 8; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
        float m_own = -INFINITY, l_own = 0.f;     // head gq
        float mc0 = -INFINITY, mc1 = -INFINITY;   // heads 2*tig, 2*tig+1 (accumulator columns)

#pragma unroll 1
        for (int j = 0; j < cnt; ++j) {
            const int st = ck % S;
            const uint32_t ph = static_cast<uint32_t>(ck / S) & 1u;
            int page, tok0, ntok;
            chunk_geom(c0 + j, ctx, page, tok0, ntok);
            const int64_t blk = __ldg(w.tables + table_row(w, b) * w.max_blocks + page);
            if (!dead && !__all_sync(0xffffffffu, mbar_wait(&my_bars[st], ph))) {
                dead = true;
                if (lane == 0 && a.err) atomicOr(a.err, kErrWaitTimeout);
            }
            if (!primed) {
                primed = true;
#pragma unroll 1
                for (int s2 = 1; s2 < S && p_piece < pe && !dead; ++s2) issue(s2);
            }
            if (!dead && blk >= 0 && blk < g.total_blocks && ntok > 0) {
                const unsigned char* stage = my_stages + static_cast<size_t>(st) * kStage;
                // ---- K operand: 16-byte chunks 2*tig and 2*tig+1 of token row gq, widened ----
                const uint4 kw0 = *reinterpret_cast<const uint4*>(stage + swz8(gq, 2 * tig));
                const uint4 kw1 = *reinterpret_cast<const uint4*>(stage + swz8(gq, 2 * tig + 1));
                const uint32_t kwd[8] = {kw0.x, kw0.y, kw0.z, kw0.w, kw1.x, kw1.y, kw1.z, kw1.w};
                // ---- S^T = Q . K^T: four independent accumulator chains ----
                float sa[4][4];
#pragma unroll
                for (int c = 0; c < 4; ++c) sa[c][0] = sa[c][1] = sa[c][2] = sa[c][3] = 0.f;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint32_t b0 = cvt_e4m3x2_f16x2(kwd[ks] & 0xffffu);
                    const uint32_t b1 = cvt_e4m3x2_f16x2(kwd[ks] >> 16);
                    mma_16816<true>(sa[(ks & 1) * 2], qh[ks][0], 0u, qh[ks][1], 0u, b0, b1);
                    mma_16816<true>(sa[(ks & 1) * 2 + 1], ql[ks][0], 0u, ql[ks][1], 0u, b0, b1);
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
                    for (int m = 0; m < 8; ++m) {
                        acc[m][0] *= a0;
                        acc[m][2] *= a0;
                        acc[m][1] *= a1;
                        acc[m][3] *= a1;
                    }
                }
                // ---- O^T += V^T . P^T ----
                float ph0, pl0, ph1, pl1;
                split_16<true>(p0, ph0, pl0);
                split_16<true>(p1, ph1, pl1);
                const uint32_t bh = pack_16x2<true>(ph0, ph1);
                const uint32_t bl = pack_16x2<true>(pl0, pl1);
                // V^T elements of tokens past the chunk's end are zeroed (their slots are stale)
                const uint32_t vmask = (v0 ? 0x0000ffffu : 0u) | (v1 ? 0xffff0000u : 0u);
                const unsigned char* vs = stage + kKBytes;
                const uint4 r0 = *reinterpret_cast<const uint4*>(vs + swz8(2 * tig, gq));      // token 2*tig
                const uint4 r1 = *reinterpret_cast<const uint4*>(vs + swz8(2 * tig + 1, gq));  // token 2*tig + 1
                const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    // dv 16*gq + 4*q4 + {0,1}: tile 2*q4 rows gq / gq+8; + {2,3}: tile 2*q4+1
                    const uint32_t lo = __byte_perm(w0[q4], w1[q4], 0x5140);
                    const uint32_t hi = __byte_perm(w0[q4], w1[q4], 0x7362);
                    uint32_t a00 = cvt_e4m3x2_f16x2(lo & 0xffffu), a01 = cvt_e4m3x2_f16x2(lo >> 16);
                    uint32_t a10 = cvt_e4m3x2_f16x2(hi & 0xffffu), a11 = cvt_e4m3x2_f16x2(hi >> 16);
                    if (ntok < kChunk) {  // warp-uniform: only a sequence's last chunk
                        a00 &= vmask;
                        a01 &= vmask;
                        a10 &= vmask;
                        a11 &= vmask;
                    }
                    mma_1688<true>(acc[2 * q4], a00, a01, bh);
                    mma_1688<true>(acc[2 * q4], a00, a01, bl);
                    mma_1688<true>(acc[2 * q4 + 1], a10, a11, bh);
                    mma_1688<true>(acc[2 * q4 + 1], a10, a11, bl);
                }
            }
            __syncwarp();
            if (p_piece < pe && !dead) issue(st);
            ++ck;
        }
        if (dead) continue;

        // ---- end of piece: lane (gq, tig) holds dv 16*gq .. 16*gq + 15 of heads 2*tig, 2*tig+1:
        // tile m's (c0, c2) are dv 16*gq + 2m, + 2m + 1 of head 2*tig, (c1, c3) of head 2*tig+1 ----
        const int hA = 2 * tig, hB = 2 * tig + 1;
        const float lA = __shfl_sync(0xffffffffu, l_own, hA * 4);
        const float lB = __shfl_sync(0xffffffffu, l_own, hB * 4);
        const float mA = __shfl_sync(0xffffffffu, m_own, hA * 4);
        const float mB = __shfl_sync(0xffffffffu, m_own, hB * 4);
        const int slot = __ldg(w.piece_slot + i);
        auto store16 = [&](float* dst, int cc, float f) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
                *reinterpret_cast<float4*>(dst + 4 * q4) =
                    make_float4(acc[2 * q4][cc] * f, acc[2 * q4][cc + 2] * f, acc[2 * q4 + 1][cc] * f,
                                acc[2 * q4 + 1][cc + 2] * f);
        };
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
                store16(a.out + (static_cast<int64_t>(b) * a.n_heads + qh2) * kDV + 16 * gq, cc, inv * vsc);
            }
        } else {
            const int64_t base = (static_cast<int64_t>(hg) * w.n_slots + slot) * kGP;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) store16(a.part_acc + (base + (cc ? hB : hA)) * kDV + 16 * gq, cc, vsc);
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

constexpr size_t kFp8Smem = static_cast<size_t>(kNW) * kS * kStage + kNW * kS * 8 + 1024;

cudaError_t fp8_prepare() {
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
    for (auto k : {paged_decode_fp8_kernel<kNW, kS, false>, paged_decode_fp8_kernel<kNW, kS, true>})
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kFp8Smem));
    if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace

bool decode_fp8_tc_eligible(const ArenaGeom& g, int n_heads) {
    if (g.dtype != GKV_DTYPE_FP8_E4M3 || g.head_dim != kD || g.v_head_dim != kDV || !g.k_scale || !g.v_scale)
        return false;
    if (!g.tmap_k || !g.tmap_v || g.tmap_rank != 3) return false;  // the pool's FP8 boxes
    if (g.block_size % kChunk != 0 || g.heads_kv <= 0 || n_heads % g.heads_kv != 0) return false;
    const int group = n_heads / g.heads_kv;
    if (group < 5) return false;  // gp 8 only; smaller groups stay on the FP32 pipe
    return static_cast<int64_t>(g.total_blocks) * g.layers * g.heads_kv < (int64_t{1} << 31);  // box z index
}

void decode_fp8_tc_config(DecodeConfig& c) {
    c.warps = kNW;
    c.threads = kNW * 32;
    c.smem = kFp8Smem;
    int per_sm = 1, per_sm_dyn = 1;
    if (fp8_prepare() != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_fp8_kernel<kNW, kS, false>, c.threads,
                                                      kFp8Smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_dyn, paged_decode_fp8_kernel<kNW, kS, true>, c.threads,
                                                      kFp8Smem) != cudaSuccess ||
        per_sm < 1 || per_sm_dyn < 1) {
        cudaGetLastError();
        per_sm = per_sm_dyn = 1;
    }
    c.ctas_per_sm = per_sm_dyn < per_sm ? per_sm_dyn : per_sm;
    c.supported = true;
}

cudaError_t launch_paged_decode_fp8_tc(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a, int group,
                                       int head_groups, int* launches, cudaStream_t st) {
    cudaError_t e = fp8_prepare();
    if (e != cudaSuccess) return e;
    const int cpp = (g.block_size + kChunk - 1) / kChunk;
    const dim3 grid(static_cast<unsigned>(w.n_ctas), static_cast<unsigned>(head_groups));
    const CUtensorMap& tk = *static_cast<const CUtensorMap*>(g.tmap_k);
    const CUtensorMap& tv = *static_cast<const CUtensorMap*>(g.tmap_v);
    e = w.dyn ? launch_pdl(paged_decode_fp8_kernel<kNW, kS, true>, grid, dim3(kNW * 32), kFp8Smem, st, tk, tv, g, w,
                           a, group, cpp)
              : launch_pdl(paged_decode_fp8_kernel<kNW, kS, false>, grid, dim3(kNW * 32), kFp8Smem, st, tk, tv, g, w,
                           a, group, cpp);
    if (e != cudaSuccess) return e;
    *launches = 1;
    if (w.n_deferred > 0 || w.merge_grid > 0) {
        e = launch_deferred_merge(g, w, a, group, kGP, head_groups, st);
        if (e == cudaSuccess) *launches = 2;
    }
    return e;
}

}  // namespace gkv
