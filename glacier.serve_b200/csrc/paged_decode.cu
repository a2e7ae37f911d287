// Split-KV GQA paged-attention decode for sm_100a.
//
// Replaces PagedAttentionKernel.ComputeAttention (src/Glacier.Serve/Inference/
// PagedAttention/PagedAttentionKernel.cs:17-372), which the runners call once per sequence
// per layer (PagedTransformerRunner.cs:638) and which reads every K row and every V row
// once per QUERY head, in two passes (QK :55-67, PV :86-116).  Here:
//
//  * Work unit = "chunk": up to 8 consecutive tokens of one page of one (sequence, kv head)
//    segment.  In the [block][layer][head][slot][dim] arena a chunk's K rows and its V rows
//    are two contiguous spans, fetched by two bulk copies (cp.async.bulk on the TMA engine,
//    no multicast) into a ring of S shared-memory stages that completes on an mbarrier.
//  * Every warp is an independent worker.  The host splits the flattened chunk stream of
//    all segments into equal contiguous ranges, one per warp (warp-level stream-K); a
//    range intersects a few segments ("pieces").  Each warp prefetches S chunks ahead with
//    its own ring, across piece boundaries, and never waits for another warp (at launch only
//    its first chunk is requested; the rest of the ring follows once that chunk has landed).
//  * One pass serves all GP query heads that share the kv head, so each K/V byte is read
//    from HBM once.  Lane l owns dims [l*D/32, (l+1)*D/32) of q and of the accumulators.
//    The GP x 8 partial dot products of a chunk are reduced across the warp with a
//    transpose-reduce in which each shuffle level halves the values a lane holds.  Each
//    lane stores its partials at register positions XOR-permuted by its lane id, so at
//    every level the half a lane keeps is the lower half of its registers and the half it
//    sends is the upper half: one shuffle and one add per value, no selects.  fp32 pools with
//    d 128 and 8 head slots score with a half-warp split instead (HALF below): each half-warp
//    takes 4 of the chunk's tokens at 8 dims per lane, so the reduce runs over 16 lanes.
//  * Products use the packed two-wide fp32 FMA of sm_100 (fma.rn.f32x2).
//  * Softmax is online (running max and sum per head, base-2 exponent).  A piece that is a
//    whole segment writes the normalised output.  Otherwise it writes an unnormalised
//    partial (acc, max, sum) and bumps an arrival counter; the worker that completes a
//    segment merges its partials by log-sum-exp and resets the counter (no second launch).
//
// Roofline: HBM.  Algorithmic bytes per step = sum_b ctx_b * heads_kv * (D + DV) * elem
// (+ q and out).  FLOPs = 2 * sum_b ctx_b * n_heads * (D + DV) on the FP32 pipe.
#include <atomic>
#include <type_traits>

#include "decode_merge.cuh"
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

constexpr int kChunk = kDecodeChunk;
constexpr float kLog2e = 1.4426950408889634f;

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }

// fp32, d 128, a group of 7 in 8 head slots (the half-warp score split with the padding slot
// compiled out): three CTAs of 4 warps per SM, at most 168 registers and 2 ring stages each --
// 12 warps per SM hide the per-chunk shuffle and exp latencies better than 8 warps with 3
// stages.  (A full group of 8 spills more at 168 registers and keeps two CTAs.)
template <typename KV, int D, int GP, bool LD>
constexpr bool kThreeCtas = std::is_same<KV, float>::value && D == 128 && GP == 8 && LD;

// Selectless warp transpose-reduce of CUR values per lane (see file comment).  Positions
// must hold value j at position j ^ X(lane); afterwards lane L holds its R values at
// positions 0..R-1.
template <int CUR, int MASK>
__device__ __forceinline__ void transpose_reduce(float* x) {
    if constexpr (MASK >= 1) {
        if constexpr (CUR >= 2) {
            constexpr int H = CUR / 2;
#pragma unroll
            for (int i = 0; i < H; ++i) x[i] += __shfl_xor_sync(0xffffffffu, x[i + H], MASK);
            transpose_reduce<H, MASK / 2>(x);
        } else {
            x[0] += __shfl_xor_sync(0xffffffffu, x[0], MASK);
            transpose_reduce<1, MASK / 2>(x);
        }
    }
}

// Loads EPL consecutive KV elements from shared memory as EP2 = ceil(EPL/2) fp32 pairs
// (the odd tail, EPL == 1, gets a zero partner).
template <typename KV, int EPL>
__device__ __forceinline__ void load_pairs(const KV* p, float2 (&o)[(EPL + 1) / 2]) {
    if constexpr (std::is_same<KV, float>::value) {
        if constexpr (EPL == 1) {
            o[0] = make_float2(p[0], 0.f);
        } else if constexpr (EPL == 2) {
            o[0] = *reinterpret_cast<const float2*>(p);
        } else {
#pragma unroll
            for (int i = 0; i < EPL; i += 4) {
                const float4 v = *reinterpret_cast<const float4*>(p + i);
                o[i / 2] = make_float2(v.x, v.y);
                o[i / 2 + 1] = make_float2(v.z, v.w);
            }
        }
    } else if constexpr (std::is_same<KV, __half>::value) {
        if constexpr (EPL == 1) {
            o[0] = make_float2(__half2float(p[0]), 0.f);
        } else if constexpr (EPL == 2) {
            o[0] = __half22float2(*reinterpret_cast<const __half2*>(p));
        } else if constexpr (EPL == 4) {
            const uint2 w = *reinterpret_cast<const uint2*>(p);
            o[0] = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
            o[1] = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
        } else {
#pragma unroll
            for (int i = 0; i < EPL; i += 8) {
                const uint4 w = *reinterpret_cast<const uint4*>(p + i);
                o[i / 2 + 0] = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
                o[i / 2 + 1] = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
                o[i / 2 + 2] = __half22float2(*reinterpret_cast<const __half2*>(&w.z));
                o[i / 2 + 3] = __half22float2(*reinterpret_cast<const __half2*>(&w.w));
            }
        }
    } else if constexpr (std::is_same<KV, __nv_fp8_e4m3>::value) {
        // e4m3 -> fp16 -> fp32 is exact; the (layer, head) scale is applied by the caller
        const unsigned char* u = reinterpret_cast<const unsigned char*>(p);
        if constexpr (EPL == 1) {
            o[0] = make_float2(fp8x2_to_float2(u[0]).x, 0.f);
        } else if constexpr (EPL == 2) {
            o[0] = fp8x2_to_float2(*reinterpret_cast<const uint16_t*>(u));
        } else if constexpr (EPL == 4) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(u);
            o[0] = fp8x2_to_float2(w & 0xffffu);
            o[1] = fp8x2_to_float2(w >> 16);
        } else {
#pragma unroll
            for (int i = 0; i < EPL; i += 8) {
                const uint2 w = *reinterpret_cast<const uint2*>(u + i);
                o[i / 2 + 0] = fp8x2_to_float2(w.x & 0xffffu);
                o[i / 2 + 1] = fp8x2_to_float2(w.x >> 16);
                o[i / 2 + 2] = fp8x2_to_float2(w.y & 0xffffu);
                o[i / 2 + 3] = fp8x2_to_float2(w.y >> 16);
            }
        }
    } else {
        const uint16_t* u = reinterpret_cast<const uint16_t*>(p);
        if constexpr (EPL == 1) {
            o[0] = make_float2(__uint_as_float(static_cast<uint32_t>(u[0]) << 16), 0.f);
        } else if constexpr (EPL == 2) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(u);
            o[0] = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
        } else if constexpr (EPL == 4) {
            const uint2 w = *reinterpret_cast<const uint2*>(u);
            o[0] = make_float2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u));
            o[1] = make_float2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
        } else {
#pragma unroll
            for (int i = 0; i < EPL; i += 8) {
                const uint4 w = *reinterpret_cast<const uint4*>(u + i);
                o[i / 2 + 0] = make_float2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u));
                o[i / 2 + 1] = make_float2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
                o[i / 2 + 2] = make_float2(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xffff0000u));
                o[i / 2 + 3] = make_float2(__uint_as_float(w.w << 16), __uint_as_float(w.w & 0xffff0000u));
            }
        }
    }
}

template <int EP2>
__device__ __forceinline__ float dot_pairs(const float2 (&q)[EP2], const float2 (&k)[EP2]) {
    float2 p = __fmul2_rn(q[0], k[0]);
#pragma unroll
    for (int i = 1; i < EP2; ++i) p = __ffma2_rn(q[i], k[i], p);
    return p.x + p.y;
}

template <typename KV, int D, int DV, int GP, int NW, int S>
struct DecodeKernelTraits {
    static constexpr int EB = sizeof(KV);
    static constexpr int EPL = D / 32;
    static constexpr int EPLV = DV / 32;
    static constexpr int EP2 = (EPL + 1) / 2;
    static constexpr int EV2 = (EPLV + 1) / 2;
    static constexpr int KSTAGE = kChunk * D * EB;
    static constexpr int VSTAGE = kChunk * DV * EB;
    static constexpr int STAGE = ((KSTAGE + VSTAGE) + 127) / 128 * 128;
    static constexpr int NV = GP * kChunk;              // values per transpose-reduce
    static constexpr int NB = ilog2(NV);
    static constexpr int R = NV >= 32 ? NV / 32 : 1;    // reduced values per lane
    static constexpr int DUP = NV >= 32 ? 1 : 32 / NV;  // lanes holding the same value
    static constexpr int LG = 32 / GP;                  // lanes per query head after reduce
    // per-warp scratch: p duplicated into pairs [GP*8] float2, then the GP running maxima
    static constexpr int PBUF = (GP * kChunk * 2 + GP + 3) / 4 * 4;
    static constexpr size_t OFF_BAR = static_cast<size_t>(NW) * S * STAGE;
    static constexpr size_t OFF_PBUF = (OFF_BAR + static_cast<size_t>(NW) * S * 8 + 15) / 16 * 16;
    static constexpr size_t SMEM = OFF_PBUF + static_cast<size_t>(NW) * PBUF * 4;
    static_assert(D % 32 == 0 && DV % 32 == 0, "head dims must be multiples of 32");
    static_assert(GP == 1 || GP == 2 || GP == 4 || GP == 8, "GP");
};

// DYN: the static step layout (the work list comes from the header at w.dyn); a separate
// instantiation, so the by-value work list of the normal launch stays in the parameter bank.
// LD: the group is GP - 1 heads (7 of 8, 3 of 4), so head slot GP - 1 is padding in every
// piece; its P.V products and rescales are compiled out (its accumulator stays 0 and is never
// output).  Its scores still go through the transpose-reduce, whose lane permutation spreads
// every head over all slots.
template <typename KV, int D, int DV, int GP, int NW, int S, bool DYN, bool LD>
__global__ void __launch_bounds__(NW * 32, kThreeCtas<KV, D, GP, LD> ? 3 : 1) paged_decode_kernel(ArenaGeom g, DecodeWork w,
                                                               DecodeArgs a, int group, int cpp) {
    using Tr = DecodeKernelTraits<KV, D, DV, GP, NW, S>;
    constexpr int EPL = Tr::EPL, EPLV = Tr::EPLV, EP2 = Tr::EP2, EV2 = Tr::EV2;
    constexpr bool kFp8 = std::is_same<KV, __nv_fp8_e4m3>::value;
    constexpr int NV = Tr::NV, NB = Tr::NB, R = Tr::R, DUP = Tr::DUP, LG = Tr::LG;
    extern __shared__ __align__(128) unsigned char smem[];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int hg = blockIdx.y;
    const int worker = blockIdx.x * NW + warp;
    if constexpr (DYN) w = resolve_work(w);

    uint64_t* my_bars = reinterpret_cast<uint64_t*>(smem + Tr::OFF_BAR) + warp * S;
    float* pbuf = reinterpret_cast<float*>(smem + Tr::OFF_PBUF) + warp * Tr::PBUF;
    float2* pdup = reinterpret_cast<float2*>(pbuf);
    float* mbuf = pbuf + GP * kChunk * 2;
    unsigned char* my_stages = smem + static_cast<size_t>(warp) * S * Tr::STAGE;

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

    const char* Kb = static_cast<const char*>(g.k);
    const char* Vb = static_cast<const char*>(g.v);
    const int64_t k_l = static_cast<int64_t>(a.layer) * g.k_layer_stride;
    const int64_t v_l = static_cast<int64_t>(a.layer) * g.v_layer_stride;
    const int bs = g.block_size;
    const bool cpp2 = (cpp == 2);  // the 16-token block fast path: page = k >> 1

    // ---- producer: lane 0 issues the two bulk copies of chunk j of piece `piece` ----
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
    // Lane 0 issues the K span and lane 1 the V span: a bulk copy occupies its issuing thread
    // for on the order of a hundred cycles, so the two go in parallel.
    auto issue = [&](int st) {
        int page, tok0, ntok;
        chunk_geom(p_c0 + p_j, p_ctx, page, tok0, ntok);
        int64_t blk = 0;
        if (lane == 0) blk = __ldg(w.tables + table_row(w, p_b) * w.max_blocks + page);
        blk = __shfl_sync(0xffffffffu, blk, 0);
        uint64_t* bar = &my_bars[st];
        const bool ok = blk >= 0 && blk < g.total_blocks && ntok > 0;
        const uint32_t kb = static_cast<uint32_t>(ntok * D * Tr::EB);
        const uint32_t vb = static_cast<uint32_t>(ntok * DV * Tr::EB);
        if (lane == 0) {
            if (ok) {
                mbar_arrive_expect_tx(bar, kb + vb);
            } else {
                if (a.err) atomicOr(a.err, kErrBadBlock);
                mbar_arrive(bar);  // completes the phase without data; the consumer skips it
            }
        }
        __syncwarp();  // the expected byte count precedes both copies' completion
        if (ok && lane < 2) {
            unsigned char* dst = my_stages + static_cast<size_t>(st) * Tr::STAGE;
            fence_proxy_async_smem();
            if (lane == 0)
                bulk_g2s(dst, Kb + (blk * g.k_block_stride + k_l + p_h * g.k_head_stride +
                                    static_cast<int64_t>(tok0) * D) * Tr::EB, kb, bar);
            else
                bulk_g2s(dst + Tr::KSTAGE, Vb + (blk * g.v_block_stride + v_l + p_h * g.v_head_stride +
                                                 static_cast<int64_t>(tok0) * DV) * Tr::EB, vb, bar);
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

    bool dead = false;  // a bounded wait expired: stop consuming, skip remaining work
    int ck = 0;         // chunks consumed by this warp
    const float scale_log2 = a.scale * kLog2e;
    // this lane's register-position permutation and its first reduced value
    // HALF (fp32, d 128, GP 8): the two half-warps score different tokens of a chunk (lanes
    // [16 hf, 16 hf + 16) tokens 4 hf .. 4 hf + 3), each lane over 8 dims: [4 l, 4 l + 4) and
    // [64 + 4 l, 64 + 4 l + 4), l = lane % 16 (two 16-byte pieces 256 bytes apart, so the 8
    // lanes of a shared-memory phase hit 8 distinct bank groups).  The GP x 4 partials of a
    // lane reduce over its half-warp: 30 shuffles and adds instead of 62, and half the
    // pair-sums of the dot products.  Afterwards lane (hf, l) holds head l / 2, tokens
    // 4 hf + 2 (l % 2) + {0, 1}; a head's four lanes differ in lane bits 0 and 4.
    constexpr bool HALF = std::is_same<KV, float>::value && D == 128 && GP == 8;
    const int l16 = lane & 15, hf = lane >> 4;
    const int X = HALF ? (l16 << 1) : (NB >= 5) ? (lane << (NB - 5)) : (lane >> (5 - NB));
    const int Xg = HALF ? (X >> 2) : (X >> 3);
    const int Xt = HALF ? (X & 3) : (X & 7);
    const int g_own = HALF ? (l16 >> 1) : ((NV >= 32) ? lane * R : (lane / DUP)) / kChunk;
    const int t_own = HALF ? (4 * hf + 2 * (l16 & 1)) : ((NV >= 32) ? lane * R : (lane / DUP)) - g_own * kChunk;
    const int idx0 = g_own * kChunk + t_own;

#pragma unroll 1
    for (int i = pb; i < pe; ++i) {
        const int seg = __ldg(w.piece_seg + i);
        const int c0 = __ldg(w.piece_c0 + i);
        const int cnt = __ldg(w.piece_c1 + i) - c0;
        const int b = seg / g.heads_kv;
        const int h = seg - b * g.heads_kv;
        const int ctx = __ldg(w.ctx_lens + b);
        const int q_head0 = h * group + hg * GP;
        const int gcount = min(GP, group - hg * GP);
        // FP8: the K scale folds into the score scale, the V scale into the piece's output
        float sl2 = scale_log2, vsc = 1.f;
        if constexpr (kFp8) {
            sl2 = scale_log2 * __ldg(g.k_scale + a.layer * g.heads_kv + h);
            vsc = __ldg(g.v_scale + a.layer * g.heads_kv + h);
        }

        // q in permuted slots: slot gs holds head gs ^ Xg
        constexpr int QP2 = HALF ? 4 : EP2;
        float2 q[GP][QP2];
#pragma unroll
        for (int gs = 0; gs < GP; ++gs) {
            const int gh = gs ^ Xg;
            const bool live = gh < gcount;
            const float* qh = a.q + (static_cast<int64_t>(b) * a.n_heads + q_head0 + gh) * D;
            if constexpr (HALF) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float* qp = qh + (e >> 1) * 64 + 4 * l16 + 2 * (e & 1);
                    q[gs][e] = live ? make_float2(__ldg(qp), __ldg(qp + 1)) : make_float2(0.f, 0.f);
                }
            } else {
                const float* qp = qh + lane * EPL;
#pragma unroll
                for (int e = 0; e < EP2; ++e) {
                    q[gs][e].x = live ? __ldg(qp + 2 * e) : 0.f;
                    q[gs][e].y = (live && 2 * e + 1 < EPL) ? __ldg(qp + 2 * e + 1) : 0.f;
                }
            }
        }
        float m[GP];
        float2 acc[GP][EV2];
#pragma unroll
        for (int gg = 0; gg < GP; ++gg) {
            m[gg] = -INFINITY;
#pragma unroll
            for (int e = 0; e < EV2; ++e) acc[gg][e] = make_float2(0.f, 0.f);
        }
        float m_own = -INFINITY, l_own = 0.f;

#pragma unroll 1
        for (int j = 0; j < cnt; ++j) {
            const int st = ck % S;
            const uint32_t ph = static_cast<uint32_t>(ck / S) & 1u;
            int page, tok0, ntok;
            chunk_geom(c0 + j, ctx, page, tok0, ntok);
            const int64_t blk = __ldg(w.tables + table_row(w, b) * w.max_blocks + page);
            // warp-uniform: the transpose-reduce below is warp-collective
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
                const unsigned char* stage = my_stages + static_cast<size_t>(st) * Tr::STAGE;
                const KV* Ks = reinterpret_cast<const KV*>(stage);
                const KV* Vs = reinterpret_cast<const KV*>(stage + Tr::KSTAGE);
                // ---- scores at permuted positions, then the selectless transpose-reduce ----
                float sc[HALF ? NV / 2 : NV];
                if constexpr (HALF) {
#pragma unroll
                    for (int ts = 0; ts < 4; ++ts) {
                        const float* kr = reinterpret_cast<const float*>(Ks) + (4 * hf + (ts ^ Xt)) * D + 4 * l16;
                        const float4 k0 = *reinterpret_cast<const float4*>(kr);
                        const float4 k1 = *reinterpret_cast<const float4*>(kr + 64);
                        const float2 kv[4] = {make_float2(k0.x, k0.y), make_float2(k0.z, k0.w),
                                              make_float2(k1.x, k1.y), make_float2(k1.z, k1.w)};
#pragma unroll
                        for (int gs = 0; gs < GP; ++gs) sc[gs * 4 + ts] = dot_pairs<4>(q[gs], kv);
                    }
                    transpose_reduce<NV / 2, 8>(sc);
                } else {
#pragma unroll
                    for (int ts = 0; ts < kChunk; ++ts) {
                        float2 kv[EP2];
                        load_pairs<KV, EPL>(Ks + (ts ^ Xt) * D + lane * EPL, kv);
#pragma unroll
                        for (int gs = 0; gs < GP; ++gs) sc[gs * kChunk + ts] = dot_pairs<EP2>(q[gs], kv);
                    }
                    transpose_reduce<NV, 16>(sc);
                }
                // ---- online softmax of this lane's head ----
                float s2[R];
                float cmax = -INFINITY;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    s2[r] = (t_own + r < ntok) ? sc[r] * sl2 : -INFINITY;
                    cmax = fmaxf(cmax, s2[r]);
                }
                if constexpr (HALF) {
                    cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
                    cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 16));
                } else {
#pragma unroll
                    for (int mask = LG / 2; mask >= DUP; mask >>= 1)
                        cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, mask));
                }
                const float m_new = fmaxf(m_own, cmax);
                float p[R];
                float psum = 0.f;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    p[r] = exp2f(s2[r] - m_new);
                    psum += p[r];
                }
                if constexpr (HALF) {
                    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
                    psum += __shfl_xor_sync(0xffffffffu, psum, 16);
                } else {
#pragma unroll
                    for (int mask = LG / 2; mask >= DUP; mask >>= 1)
                        psum += __shfl_xor_sync(0xffffffffu, psum, mask);
                }
                const bool changed = m_new > m_own;
                l_own = l_own * exp2f(m_own - m_new) + psum;
                m_own = m_new;
                if ((lane % DUP) == 0) {
#pragma unroll
                    for (int r = 0; r < R; ++r) pdup[idx0 + r] = make_float2(p[r], p[r]);
                }
                if (HALF ? (lane & 17) == 0 : (lane % LG) == 0) mbuf[g_own] = m_new;
                __syncwarp();
                // ---- rescale the accumulators if any head's maximum moved ----
                if (__any_sync(0xffffffffu, changed)) {
#pragma unroll
                    for (int gg = 0; gg < GP; ++gg) {
                        if (LD && gg == GP - 1) continue;
                        const float mn = mbuf[gg];
                        const float alpha = exp2f(m[gg] - mn);
                        m[gg] = mn;
                        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
                        for (int e = 0; e < EV2; ++e) acc[gg][e] = __fmul2_rn(acc[gg][e], a2);
                    }
                }
                // ---- P.V ----
                if (ntok == kChunk) {
#pragma unroll
                    for (int t = 0; t < kChunk; t += 2) {
                        float2 v0[EV2], v1[EV2];
                        load_pairs<KV, EPLV>(Vs + t * DV + lane * EPLV, v0);
                        load_pairs<KV, EPLV>(Vs + (t + 1) * DV + lane * EPLV, v1);
#pragma unroll
                        for (int gg = 0; gg < GP; ++gg) {
                            if (LD && gg == GP - 1) continue;
                            const float4 pp = *reinterpret_cast<const float4*>(pdup + gg * kChunk + t);
                            const float2 pa = make_float2(pp.x, pp.y), pb2 = make_float2(pp.z, pp.w);
#pragma unroll
                            for (int e = 0; e < EV2; ++e) {
                                acc[gg][e] = __ffma2_rn(pa, v0[e], acc[gg][e]);
                                acc[gg][e] = __ffma2_rn(pb2, v1[e], acc[gg][e]);
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int t = 0; t < kChunk; ++t) {
                        if (t < ntok) {
                            float2 v0[EV2];
                            load_pairs<KV, EPLV>(Vs + t * DV + lane * EPLV, v0);
#pragma unroll
                            for (int gg = 0; gg < GP; ++gg) {
                                if (LD && gg == GP - 1) continue;
                                const float2 pa = pdup[gg * kChunk + t];
#pragma unroll
                                for (int e = 0; e < EV2; ++e) acc[gg][e] = __ffma2_rn(pa, v0[e], acc[gg][e]);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            // ---- refill the stage just consumed with the chunk S positions ahead ----
            if (p_piece < pe && !dead) issue(st);
            ++ck;
        }
        if (dead) continue;

        // ---- end of piece: final output, or partial + fused merge ----
        float lg[GP];
#pragma unroll
        for (int gg = 0; gg < GP; ++gg) lg[gg] = __shfl_sync(0xffffffffu, l_own, HALF ? 2 * gg : gg * LG);
        const int slot = __ldg(w.piece_slot + i);
        if (slot < 0) {
#pragma unroll
            for (int gg = 0; gg < GP; ++gg) {
                if (gg >= gcount) continue;
                const int qh = q_head0 + gg;
                float Ls = lg[gg], f = 1.f, Mref = m[gg];
                if (a.sinks || a.has_sink_all) {
                    const float sk = (a.sinks ? __ldg(a.sinks + qh) : a.sink_all) * kLog2e;
                    const float M2 = fmaxf(m[gg], sk);
                    f = (m[gg] == -INFINITY) ? 0.f : exp2f(m[gg] - M2);
                    Ls = Ls * f + exp2f(sk - M2);
                    Mref = M2;
                }
                float inv = Ls > 0.f ? f / Ls : 0.f;
                if constexpr (kFp8) inv *= vsc;
                if (a.lse && lane == 0) a.lse[static_cast<int64_t>(b) * a.n_heads + qh] = lse_ln(Mref, Ls);
                float* op = a.out + (static_cast<int64_t>(b) * a.n_heads + qh) * DV + lane * EPLV;
#pragma unroll
                for (int e = 0; e < EV2; ++e) {
                    op[2 * e] = acc[gg][e].x * inv;
                    if (2 * e + 1 < EPLV) op[2 * e + 1] = acc[gg][e].y * inv;
                }
            }
        } else {
            const int64_t base = (static_cast<int64_t>(hg) * w.n_slots + slot) * GP;
#pragma unroll
            for (int gg = 0; gg < GP; ++gg) {
                float* ap = a.part_acc + (base + gg) * DV + lane * EPLV;
#pragma unroll
                for (int e = 0; e < EV2; ++e) {
                    if constexpr (kFp8) acc[gg][e] = __fmul2_rn(acc[gg][e], make_float2(vsc, vsc));
                    ap[2 * e] = acc[gg][e].x;
                    if (2 * e + 1 < EPLV) ap[2 * e + 1] = acc[gg][e].y;
                }
            }
            if (lane < GP) {
                float mm = m[0], ll = lg[0];
#pragma unroll
                for (int gg = 1; gg < GP; ++gg)
                    if (lane == gg) {
                        mm = m[gg];
                        ll = lg[gg];
                    }
                a.part_ml[(base + lane) * 2 + 0] = mm;
                a.part_ml[(base + lane) * 2 + 1] = ll;
            }
            // arrival: the worker completing the segment merges every partial of it
            const int mi = __ldg(w.piece_merge + i);
            if (mi >= 0) {  // merged here; otherwise the deferred-merge kernel does it
                const int ns = __ldg(w.merge_nslots + mi);
                __threadfence();
                __syncwarp();
                int prev = 0;
                int* counter = w.merge_count + static_cast<int64_t>(hg) * w.n_merge + mi;
                if (lane == 0) prev = atomicAdd(counter, 1);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == ns - 1) {
                    __threadfence();
                    merge_segment<GP, DV>(a, w, hg, __ldg(w.merge_slot0 + mi), ns, b, q_head0, gcount, lane);
                    if (lane == 0) atomicExch(counter, 0);
                }
            }
        }
    }
}

// Warp workers per CTA and ring stages per warp.  Sized so that two CTAs fit on an SM
// (<= ~110 KB of shared memory each), three for kThreeCtas (<= ~74 KB), with 2-6 chunks of
// 8 tokens in flight per warp.
template <typename KV, int D, int DV, int GP, bool LD>
struct RingShape {
    static constexpr int NW = 4;
    static constexpr int STAGE = kChunk * (D + DV) * static_cast<int>(sizeof(KV));
    static constexpr int S_MAX = sizeof(KV) == 4 ? 3 : 6;
    static constexpr int S_FIT = ((kThreeCtas<KV, D, GP, LD> ? 72 : 108) * 1024) / (NW * STAGE);
    static constexpr int S = S_FIT < 2 ? 2 : (S_FIT < S_MAX ? S_FIT : S_MAX);
};

template <typename KV, int D, int DV, int GP, bool LD = false>
struct Inst {
    static constexpr int NW = RingShape<KV, D, DV, GP, LD>::NW;
    static constexpr int S = RingShape<KV, D, DV, GP, LD>::S;
    using Tr = DecodeKernelTraits<KV, D, DV, GP, NW, S>;

    static cudaError_t prepare() {
        // cudaFuncSetAttribute is per device: remember which devices are done.
        static std::atomic<uint64_t> done_mask{0};
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const uint64_t bit = 1ull << (dev & 63);
        if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
        e = cudaFuncSetAttribute(paged_decode_kernel<KV, D, DV, GP, NW, S, false, LD>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Tr::SMEM));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(paged_decode_kernel<KV, D, DV, GP, NW, S, true, LD>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Tr::SMEM));
        if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
        return e;
    }

    static void config(DecodeConfig& c) {
        c.warps = NW;
        c.threads = NW * 32;
        c.smem = Tr::SMEM;
        // the persistent grid must be resident in either instantiation
        int per_sm = 1, per_sm_dyn = 1;
        if (prepare() != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &per_sm, paged_decode_kernel<KV, D, DV, GP, NW, S, false, LD>, c.threads, Tr::SMEM) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &per_sm_dyn, paged_decode_kernel<KV, D, DV, GP, NW, S, true, LD>, c.threads, Tr::SMEM) != cudaSuccess ||
            per_sm < 1 || per_sm_dyn < 1) {
            cudaGetLastError();
            per_sm = per_sm_dyn = 1;
        }
        if (per_sm_dyn < per_sm) per_sm = per_sm_dyn;
        c.ctas_per_sm = per_sm;
        c.supported = true;
    }

    static cudaError_t launch(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                              int group, int head_groups, int* launches, cudaStream_t st) {
        const int cpp = (g.block_size + kChunk - 1) / kChunk;
        cudaError_t e = prepare();
        if (e != cudaSuccess) return e;
        dim3 grid(static_cast<unsigned>(w.n_ctas), static_cast<unsigned>(head_groups));
        e = w.dyn ? launch_pdl(paged_decode_kernel<KV, D, DV, GP, NW, S, true, LD>, grid, dim3(NW * 32), Tr::SMEM, st,
                               g, w, a, group, cpp)
                  : launch_pdl(paged_decode_kernel<KV, D, DV, GP, NW, S, false, LD>, grid, dim3(NW * 32), Tr::SMEM, st,
                               g, w, a, group, cpp);
        if (e != cudaSuccess) return e;
        *launches = 1;
        if (w.n_deferred > 0 || w.merge_grid > 0) {
            e = launch_deferred_merge(g, w, a, group, GP, head_groups, st);
            if (e == cudaSuccess) *launches = 2;
        }
        return e;
    }
};

// Dispatch over (storage type, head dims, GP); `f` receives a value of the Inst type.  fp32
// pools with a group of 7 or 3 get the LD instantiation (padding slot compiled out).
template <typename F>
bool dispatch(const ArenaGeom& g, int gp, int group, F&& f) {
    auto by_gp = [&](auto kv_tag, auto d_tag, auto dv_tag) -> bool {
        using KV = decltype(kv_tag);
        constexpr int D = decltype(d_tag)::value;
        constexpr int DV = decltype(dv_tag)::value;
        switch (gp) {
            case 1: f(Inst<KV, D, DV, 1>{}); return true;
            case 2: f(Inst<KV, D, DV, 2>{}); return true;
            case 4:
                if constexpr (std::is_same<KV, float>::value)
                    if (group == 3) return f(Inst<KV, D, DV, 4, true>{}), true;
                f(Inst<KV, D, DV, 4>{});
                return true;
            case 8:
                if constexpr (std::is_same<KV, float>::value)
                    if (group == 7) return f(Inst<KV, D, DV, 8, true>{}), true;
                f(Inst<KV, D, DV, 8>{});
                return true;
        }
        return false;
    };
    auto by_dims = [&](auto kv_tag) -> bool {
#define GKV_DIMS(DD, DDV)                                                                     \
    if (g.head_dim == DD && g.v_head_dim == DDV)                                              \
        return by_gp(kv_tag, std::integral_constant<int, DD>{}, std::integral_constant<int, DDV>{});
        GKV_DIMS(128, 128)
        GKV_DIMS(64, 64)
        GKV_DIMS(32, 32)
        GKV_DIMS(32, 64)
        GKV_DIMS(128, 64)
        GKV_DIMS(256, 256)
#undef GKV_DIMS
        return false;
    };
    if (g.dtype == GKV_DTYPE_BF16) return by_dims(__nv_bfloat16{});
    if (g.dtype == GKV_DTYPE_F16) return by_dims(__half{});
    if (g.dtype == GKV_DTYPE_FP8_E4M3) {  // the common head dims only
        if (g.head_dim == 128 && g.v_head_dim == 128)
            return by_gp(__nv_fp8_e4m3{}, std::integral_constant<int, 128>{}, std::integral_constant<int, 128>{});
        if (g.head_dim == 64 && g.v_head_dim == 64)
            return by_gp(__nv_fp8_e4m3{}, std::integral_constant<int, 64>{}, std::integral_constant<int, 64>{});
        return false;
    }
    return by_dims(float{});
}

int pick_gp(int group) {
    const int cap = group < 8 ? group : 8;
    int gp = 1;
    while (gp < cap) gp <<= 1;
    return gp;
}

}  // namespace

DecodeConfig decode_config(const ArenaGeom& g, int n_heads) {
    DecodeConfig c{};
    c.supported = false;
    if (n_heads <= 0 || g.heads_kv <= 0 || n_heads % g.heads_kv != 0) return c;
    const int group = n_heads / g.heads_kv;
    c.gp = pick_gp(group);
    c.head_groups = (group + c.gp - 1) / c.gp;
    if (decode_tc_eligible(g, n_heads)) {
        decode_tc_config(c);
        return c;
    }
    if (decode_fp8_tc_eligible(g, n_heads)) {
        decode_fp8_tc_config(c);
        return c;
    }
    dispatch(g, c.gp, group, [&](auto inst) { decltype(inst)::config(c); });
    return c;
}

namespace {
__global__ void fill_kernel(float* x, int64_t n, float value) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] = value;
}
}  // namespace

cudaError_t launch_fill(float* x, int64_t n, float value, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 1184) blocks = 1184;
    fill_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(x, n, value);
    return cudaGetLastError();
}

cudaError_t launch_lse_merge(const float* parts, int n_parts, int rows, int dv, const float* sinks,
                             int n_heads, float* out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    const int64_t threads = static_cast<int64_t>(rows) * 32;
    lse_merge_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(parts, n_parts, rows, dv,
                                                                                   sinks, n_heads, out);
    return cudaGetLastError();
}

cudaError_t launch_deferred_merge(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                  int group, int gp, int head_groups, cudaStream_t st) {
    if (w.n_deferred <= 0 && w.merge_grid <= 0) return cudaSuccess;
    // a CTA per (long segment, head), then a warp per (short segment, head), eight per CTA;
    // in the static step layout a fixed grid loops over them
    const int64_t per_entry = static_cast<int64_t>(head_groups) * gp;
    const int64_t short_items = static_cast<int64_t>(w.n_deferred - w.n_deferred_long) * per_entry;
    const dim3 grid(w.merge_grid > 0 ? static_cast<unsigned>(w.merge_grid)
                                     : static_cast<unsigned>(w.n_deferred_long * per_entry + (short_items + 7) / 8));
    auto go = [&](auto k_once, auto k_loop) {
        return w.merge_grid > 0 ? launch_pdl(k_loop, grid, dim3(256), 0, st, g, w, a, group, head_groups)
                                : launch_pdl(k_once, grid, dim3(256), 0, st, g, w, a, group, head_groups);
    };
#define GKV_MERGE_DV(GPV)                                                                             \
    switch (g.v_head_dim) {                                                                          \
        case 32: return go(deferred_merge_kernel<GPV, 32, false>, deferred_merge_kernel<GPV, 32, true>);    \
        case 64: return go(deferred_merge_kernel<GPV, 64, false>, deferred_merge_kernel<GPV, 64, true>);    \
        case 128: return go(deferred_merge_kernel<GPV, 128, false>, deferred_merge_kernel<GPV, 128, true>); \
        case 256: return go(deferred_merge_kernel<GPV, 256, false>, deferred_merge_kernel<GPV, 256, true>); \
        default: return cudaErrorInvalidValue;                                                       \
    }
    switch (gp) {
        case 1: GKV_MERGE_DV(1)
        case 2: GKV_MERGE_DV(2)
        case 4: GKV_MERGE_DV(4)
        case 8: GKV_MERGE_DV(8)
    }
#undef GKV_MERGE_DV
    return cudaErrorInvalidValue;
}

cudaError_t launch_paged_decode(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                int* launches, cudaStream_t stream) {
    *launches = 0;
    if (w.n_ctas <= 0) return cudaSuccess;
    const int group = a.n_heads / g.heads_kv;
    const int gp = pick_gp(group);
    const int head_groups = (group + gp - 1) / gp;
    const bool aligned = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.out) |
                           reinterpret_cast<uintptr_t>(a.part_acc)) & 15) == 0;
    if (aligned && decode_tc_eligible(g, a.n_heads))
        return launch_paged_decode_tc(g, w, a, group, head_groups, launches, stream);
    if (aligned && decode_fp8_tc_eligible(g, a.n_heads))
        return launch_paged_decode_fp8_tc(g, w, a, group, head_groups, launches, stream);
    cudaError_t err = cudaErrorInvalidValue;
    dispatch(g, gp, group, [&](auto inst) {
        err = decltype(inst)::launch(g, w, a, group, head_groups, launches, stream);
    });
    return err;
}

}  // namespace gkv
