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
//    its own ring, across piece boundaries, and never waits for another warp.
//  * One pass serves all GP query heads that share the kv head, so each K/V byte is read
//    from HBM once.  Lane l owns dims [l*D/32, (l+1)*D/32) of q and of the accumulators;
//    the GP x 8 partial dot products of a chunk are reduced across the warp with a
//    transpose-reduce (each shuffle step halves the values a lane holds), ~GP*8 shuffles per
//    chunk instead of 5*GP*8.
//  * Softmax is online (running max and sum per head, base-2 exponent).  A piece that is a
//    whole segment writes the normalised output; otherwise it writes an unnormalised
//    partial (acc, max, sum) and a second small kernel merges a segment's partials by
//    log-sum-exp.
//
// Roofline: HBM.  Algorithmic bytes per step = sum_b ctx_b * heads_kv * (D + DV) * elem
// (+ q and out).  FLOPs = 2 * sum_b ctx_b * n_heads * (D + DV) on the FP32 pipe.
#include <atomic>
#include <type_traits>

#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

constexpr int kChunk = kDecodeChunk;
constexpr float kLog2e = 1.4426950408889634f;

// Warp transpose-reduce of CUR values per lane.  After the call lane L holds
// R = max(CUR/32, 1) fully reduced values x[0..R-1] whose value index is L*R + r
// (CUR >= 32), or L >> log2(32/CUR) (CUR < 32; 32/CUR lanes hold the same value).
template <int CUR, int MASK>
__device__ __forceinline__ void transpose_reduce(float* x, int lane) {
    if constexpr (MASK >= 1) {
        if constexpr (CUR >= 2) {
            constexpr int H = CUR / 2;
            const bool upper = (lane & MASK) != 0;
#pragma unroll
            for (int i = 0; i < H; ++i) {
                const float send = upper ? x[i] : x[i + H];
                const float keep = upper ? x[i + H] : x[i];
                x[i] = keep + __shfl_xor_sync(0xffffffffu, send, MASK);
            }
            transpose_reduce<H, MASK / 2>(x, lane);
        } else {
            x[0] += __shfl_xor_sync(0xffffffffu, x[0], MASK);
            transpose_reduce<1, MASK / 2>(x, lane);
        }
    }
}

template <typename KV, int D, int DV, int GP, int NW, int S>
struct DecodeKernelTraits {
    static constexpr int EB = sizeof(KV);
    static constexpr int EPL = D / 32;
    static constexpr int EPLV = DV / 32;
    static constexpr int KSTAGE = kChunk * D * EB;
    static constexpr int VSTAGE = kChunk * DV * EB;
    static constexpr int STAGE = ((KSTAGE + VSTAGE) + 127) / 128 * 128;
    static constexpr int NV = GP * kChunk;              // values per transpose-reduce
    static constexpr int R = NV >= 32 ? NV / 32 : 1;    // reduced values per lane
    static constexpr int DUP = NV >= 32 ? 1 : 32 / NV;  // lanes holding the same value
    static constexpr int LG = 32 / GP;                  // lanes per query head after reduce
    static constexpr int PBUF = (GP * kChunk + GP + 3) / 4 * 4;  // per-warp p / max scratch
    static constexpr size_t OFF_BAR = static_cast<size_t>(NW) * S * STAGE;
    static constexpr size_t OFF_PBUF = (OFF_BAR + static_cast<size_t>(NW) * S * 8 + 15) / 16 * 16;
    static constexpr size_t SMEM = OFF_PBUF + static_cast<size_t>(NW) * PBUF * 4;
    static_assert(D % 32 == 0 && DV % 32 == 0, "head dims must be multiples of 32");
    static_assert(GP == 1 || GP == 2 || GP == 4 || GP == 8, "GP");
};

struct ChunkLoc {
    int b, h, ntok, tok0;
    int64_t blk;
};

__device__ __forceinline__ ChunkLoc locate(const ArenaGeom& g, const DecodeWork& w, int piece,
                                           int j, int cpp) {
    ChunkLoc L;
    const int seg = __ldg(w.piece_seg + piece);
    L.b = seg / g.heads_kv;
    L.h = seg - L.b * g.heads_kv;
    const int k = __ldg(w.piece_c0 + piece) + j;
    const int page = k / cpp;
    const int sub = k - page * cpp;
    L.tok0 = sub * kChunk;
    const int ctx = __ldg(w.ctx_lens + L.b);
    int nt = g.block_size - L.tok0;
    nt = nt < kChunk ? nt : kChunk;
    const int rem = ctx - page * g.block_size - L.tok0;
    L.ntok = nt < rem ? nt : rem;
    L.blk = __ldg(w.tables + static_cast<int64_t>(L.b) * w.max_blocks + page);
    return L;
}

template <typename KV, int D, int DV, int GP, int NW, int S>
__global__ void __launch_bounds__(NW * 32) paged_decode_kernel(ArenaGeom g, DecodeWork w,
                                                               DecodeArgs a, int group, int cpp) {
    using Tr = DecodeKernelTraits<KV, D, DV, GP, NW, S>;
    constexpr int EPL = Tr::EPL, EPLV = Tr::EPLV, R = Tr::R, DUP = Tr::DUP, LG = Tr::LG;
    extern __shared__ __align__(128) unsigned char smem[];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int hg = blockIdx.y;
    const int worker = blockIdx.x * NW + warp;

    uint64_t* my_bars = reinterpret_cast<uint64_t*>(smem + Tr::OFF_BAR) + warp * S;
    float* pbuf = reinterpret_cast<float*>(smem + Tr::OFF_PBUF) + warp * Tr::PBUF;
    unsigned char* my_stages = smem + static_cast<size_t>(warp) * S * Tr::STAGE;

    if (lane < S) mbar_init(&my_bars[lane], 1);
    fence_mbar_init();
    __syncwarp();

    const int pb = __ldg(w.worker_piece_begin + worker);
    const int pe = __ldg(w.worker_piece_begin + worker + 1);
    if (pb >= pe) return;

    const char* Kb = static_cast<const char*>(g.k);
    const char* Vb = static_cast<const char*>(g.v);
    const int64_t k_l = static_cast<int64_t>(a.layer) * g.k_layer_stride;
    const int64_t v_l = static_cast<int64_t>(a.layer) * g.v_layer_stride;

    // Producer: lane 0 issues the bulk copies of chunk (piece, j) into stage st.
    auto issue = [&](int piece, int j, int st) {
        const ChunkLoc L = locate(g, w, piece, j, cpp);
        if (lane == 0) {
            uint64_t* bar = &my_bars[st];
            if (L.blk >= 0 && L.blk < g.total_blocks && L.ntok > 0) {
                const uint32_t kb = static_cast<uint32_t>(L.ntok * D * Tr::EB);
                const uint32_t vb = static_cast<uint32_t>(L.ntok * DV * Tr::EB);
                const char* ks = Kb + (L.blk * g.k_block_stride + k_l + L.h * g.k_head_stride +
                                       static_cast<int64_t>(L.tok0) * D) * Tr::EB;
                const char* vs = Vb + (L.blk * g.v_block_stride + v_l + L.h * g.v_head_stride +
                                       static_cast<int64_t>(L.tok0) * DV) * Tr::EB;
                unsigned char* dst = my_stages + static_cast<size_t>(st) * Tr::STAGE;
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(bar, kb + vb);
                bulk_g2s(dst, ks, kb, bar);
                bulk_g2s(dst + Tr::KSTAGE, vs, vb, bar);
            } else {
                if (a.err) atomicOr(a.err, kErrBadBlock);
                mbar_arrive(bar);  // completes the phase without data; consumer skips it
            }
        }
    };

    // Producer cursor, S chunks ahead of the consumer.
    int p_piece = pb, p_j = 0;
    int p_cnt = __ldg(w.piece_c1 + pb) - __ldg(w.piece_c0 + pb);
    auto p_advance = [&]() {
        if (++p_j >= p_cnt) {
            p_j = 0;
            if (++p_piece < pe) p_cnt = __ldg(w.piece_c1 + p_piece) - __ldg(w.piece_c0 + p_piece);
        }
    };
#pragma unroll 1
    for (int s = 0; s < S && p_piece < pe; ++s) {
        issue(p_piece, p_j, s);
        p_advance();
    }

    bool dead = false;  // a bounded wait expired: stop consuming, skip remaining work
    int ck = 0;         // chunks consumed by this warp
    const float scale_log2 = a.scale * kLog2e;
    // value index of this lane's first reduced score, its head and token
    const int idx0 = (Tr::NV >= 32) ? lane * R : (lane / DUP);
    const int g_own = idx0 / kChunk;
    const int t_own = idx0 - g_own * kChunk;

#pragma unroll 1
    for (int i = pb; i < pe; ++i) {
        const int seg = __ldg(w.piece_seg + i);
        const int cnt = __ldg(w.piece_c1 + i) - __ldg(w.piece_c0 + i);
        const int b = seg / g.heads_kv;
        const int h = seg - b * g.heads_kv;
        const int q_head0 = h * group + hg * GP;
        const int gcount = min(GP, group - hg * GP);

        float q[GP][EPL];
#pragma unroll
        for (int gg = 0; gg < GP; ++gg) {
            const float* qp =
                a.q + (static_cast<int64_t>(b) * a.n_heads + q_head0 + gg) * D + lane * EPL;
#pragma unroll
            for (int e = 0; e < EPL; ++e) q[gg][e] = (gg < gcount) ? __ldg(qp + e) : 0.f;
        }
        float m[GP];
        float acc[GP][EPLV];
#pragma unroll
        for (int gg = 0; gg < GP; ++gg) {
            m[gg] = -INFINITY;
#pragma unroll
            for (int e = 0; e < EPLV; ++e) acc[gg][e] = 0.f;
        }
        float m_own = -INFINITY, l_own = 0.f;

#pragma unroll 1
        for (int j = 0; j < cnt; ++j) {
            const int st = ck % S;
            const uint32_t ph = static_cast<uint32_t>(ck / S) & 1u;
            const ChunkLoc L = locate(g, w, i, j, cpp);
            if (!dead && !mbar_wait(&my_bars[st], ph)) {
                dead = true;
                if (lane == 0 && a.err) atomicOr(a.err, kErrWaitTimeout);
            }
            if (!dead && L.blk >= 0 && L.blk < g.total_blocks && L.ntok > 0) {
                const unsigned char* stage = my_stages + static_cast<size_t>(st) * Tr::STAGE;
                const KV* Ks = reinterpret_cast<const KV*>(stage);
                const KV* Vs = reinterpret_cast<const KV*>(stage + Tr::KSTAGE);
                const int ntok = L.ntok;
                // ---- partial dots over this lane's dims, then transpose-reduce ----
                float sc[Tr::NV];
#pragma unroll
                for (int t = 0; t < kChunk; ++t) {
                    if (t < ntok) {
                        float kv[EPL];
                        SmemVec<KV, EPL>::load(Ks + t * D + lane * EPL, kv);
#pragma unroll
                        for (int gg = 0; gg < GP; ++gg) {
                            float s = q[gg][0] * kv[0];
#pragma unroll
                            for (int e = 1; e < EPL; ++e) s = fmaf(q[gg][e], kv[e], s);
                            sc[gg * kChunk + t] = s;
                        }
                    } else {
#pragma unroll
                        for (int gg = 0; gg < GP; ++gg) sc[gg * kChunk + t] = 0.f;
                    }
                }
                transpose_reduce<Tr::NV, 16>(sc, lane);
                // ---- online softmax of this lane's head ----
                float s2[R];
                float cmax = -INFINITY;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    s2[r] = (t_own + r < ntok) ? sc[r] * scale_log2 : -INFINITY;
                    cmax = fmaxf(cmax, s2[r]);
                }
#pragma unroll
                for (int mask = LG / 2; mask >= DUP; mask >>= 1)
                    cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, mask));
                const float m_new = fmaxf(m_own, cmax);
                float p[R];
                float psum = 0.f;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    p[r] = exp2f(s2[r] - m_new);
                    psum += p[r];
                }
#pragma unroll
                for (int mask = LG / 2; mask >= DUP; mask >>= 1)
                    psum += __shfl_xor_sync(0xffffffffu, psum, mask);
                l_own = l_own * exp2f(m_own - m_new) + psum;
                m_own = m_new;
                if ((lane % DUP) == 0) {
#pragma unroll
                    for (int r = 0; r < R; ++r) pbuf[idx0 + r] = p[r];
                }
                if ((lane % LG) == 0) pbuf[GP * kChunk + g_own] = m_new;
                __syncwarp();
                // ---- rescale the accumulators to the new maxima, then P.V ----
#pragma unroll
                for (int gg = 0; gg < GP; ++gg) {
                    const float mn = pbuf[GP * kChunk + gg];
                    const float alpha = exp2f(m[gg] - mn);
                    m[gg] = mn;
#pragma unroll
                    for (int e = 0; e < EPLV; ++e) acc[gg][e] *= alpha;
                }
                float pw[GP][kChunk];
#pragma unroll
                for (int gg = 0; gg < GP; ++gg) {
                    const float4 p0 = *reinterpret_cast<const float4*>(pbuf + gg * kChunk);
                    const float4 p1 = *reinterpret_cast<const float4*>(pbuf + gg * kChunk + 4);
                    pw[gg][0] = p0.x; pw[gg][1] = p0.y; pw[gg][2] = p0.z; pw[gg][3] = p0.w;
                    pw[gg][4] = p1.x; pw[gg][5] = p1.y; pw[gg][6] = p1.z; pw[gg][7] = p1.w;
                }
#pragma unroll
                for (int t = 0; t < kChunk; ++t) {
                    if (t < ntok) {
                        float vv[EPLV];
                        SmemVec<KV, EPLV>::load(Vs + t * DV + lane * EPLV, vv);
#pragma unroll
                        for (int gg = 0; gg < GP; ++gg) {
#pragma unroll
                            for (int e = 0; e < EPLV; ++e)
                                acc[gg][e] = fmaf(pw[gg][t], vv[e], acc[gg][e]);
                        }
                    }
                }
            }
            __syncwarp();
            // ---- refill the stage just consumed with the chunk S positions ahead ----
            if (p_piece < pe && !dead) {
                issue(p_piece, p_j, st);
                p_advance();
            }
            ++ck;
        }

        // ---- end of piece: final output or partial ----
        float lg[GP];
#pragma unroll
        for (int gg = 0; gg < GP; ++gg) lg[gg] = __shfl_sync(0xffffffffu, l_own, gg * LG);
        const int slot = __ldg(w.piece_slot + i);
        if (slot < 0) {
#pragma unroll
            for (int gg = 0; gg < GP; ++gg) {
                if (gg >= gcount) continue;
                const int qh = q_head0 + gg;
                float Ls = lg[gg], f = 1.f;
                if (a.sinks || a.has_sink_all) {
                    const float sk = (a.sinks ? __ldg(a.sinks + qh) : a.sink_all) * kLog2e;
                    const float M2 = fmaxf(m[gg], sk);
                    f = (m[gg] == -INFINITY) ? 0.f : exp2f(m[gg] - M2);
                    Ls = Ls * f + exp2f(sk - M2);
                }
                const float inv = Ls > 0.f ? f / Ls : 0.f;
                float* op = a.out + (static_cast<int64_t>(b) * a.n_heads + qh) * DV + lane * EPLV;
#pragma unroll
                for (int e = 0; e < EPLV; ++e) op[e] = acc[gg][e] * inv;
            }
        } else {
            const int64_t base = (static_cast<int64_t>(hg) * w.n_slots + slot) * GP;
#pragma unroll
            for (int gg = 0; gg < GP; ++gg) {
                float* ap = a.part_acc + (base + gg) * DV + lane * EPLV;
#pragma unroll
                for (int e = 0; e < EPLV; ++e) ap[e] = acc[gg][e];
            }
            if (lane < GP) {
                float mm = m[0], ll = lg[0];
#pragma unroll
                for (int gg = 1; gg < GP; ++gg)
                    if (lane == gg) { mm = m[gg]; ll = lg[gg]; }
                a.part_ml[(base + lane) * 2 + 0] = mm;
                a.part_ml[(base + lane) * 2 + 1] = ll;
            }
        }
    }
}

// Log-sum-exp merge of the partials of segments split over several workers.
template <int GP, int DV>
__global__ void __launch_bounds__(128) paged_decode_merge_kernel(ArenaGeom g, DecodeWork w,
                                                                 DecodeArgs a, int group) {
    const int i = blockIdx.x;
    const int hg = blockIdx.y;
    const int seg = w.merge_seg[i];
    const int s0 = w.merge_slot0[i];
    const int ns = w.merge_nslots[i];
    const int b = seg / g.heads_kv;
    const int h = seg - b * g.heads_kv;
    const int q_head0 = h * group + hg * GP;
    const int gcount = min(GP, group - hg * GP);
    for (int e = threadIdx.x; e < GP * DV; e += blockDim.x) {
        const int gg = e / DV;
        const int d = e - gg * DV;
        if (gg >= gcount) continue;
        float M = -INFINITY;
        for (int s = 0; s < ns; ++s) {
            const int64_t ps = (static_cast<int64_t>(hg) * w.n_slots + s0 + s) * GP + gg;
            M = fmaxf(M, a.part_ml[ps * 2]);
        }
        float Ls = 0.f, A = 0.f;
        if (M != -INFINITY) {
            for (int s = 0; s < ns; ++s) {
                const int64_t ps = (static_cast<int64_t>(hg) * w.n_slots + s0 + s) * GP + gg;
                const float f = exp2f(a.part_ml[ps * 2] - M);
                Ls += a.part_ml[ps * 2 + 1] * f;
                A += a.part_acc[ps * DV + d] * f;
            }
        }
        const int qh = q_head0 + gg;
        if (a.sinks || a.has_sink_all) {
            const float sk = (a.sinks ? a.sinks[qh] : a.sink_all) * kLog2e;
            const float M2 = fmaxf(M, sk);
            const float f = (M == -INFINITY) ? 0.f : exp2f(M - M2);
            Ls = Ls * f + exp2f(sk - M2);
            A *= f;
        }
        a.out[(static_cast<int64_t>(b) * a.n_heads + qh) * DV + d] = Ls > 0.f ? A / Ls : 0.f;
    }
}

// Warp workers per CTA and ring stages per warp.  Sized so that two CTAs fit on an SM
// (<= ~113 KB of shared memory each) with 2-3 chunks of 8 tokens in flight per warp.
template <typename KV, int D, int DV>
struct RingShape {
    static constexpr int NW = 4;
    static constexpr int STAGE = kChunk * (D + DV) * static_cast<int>(sizeof(KV));
    static constexpr int S_MAX = sizeof(KV) == 4 ? 3 : 6;
    static constexpr int S_FIT = (110 * 1024) / (NW * STAGE);
    static constexpr int S = S_FIT < 2 ? 2 : (S_FIT < S_MAX ? S_FIT : S_MAX);
};

template <typename KV, int D, int DV, int GP>
struct Inst {
    static constexpr int NW = RingShape<KV, D, DV>::NW;
    static constexpr int S = RingShape<KV, D, DV>::S;
    using Tr = DecodeKernelTraits<KV, D, DV, GP, NW, S>;

    static cudaError_t prepare() {
        // cudaFuncSetAttribute is per device: remember which devices are done.
        static std::atomic<uint64_t> done_mask{0};
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const uint64_t bit = 1ull << (dev & 63);
        if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
        e = cudaFuncSetAttribute(paged_decode_kernel<KV, D, DV, GP, NW, S>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(Tr::SMEM));
        if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
        return e;
    }

    static void config(DecodeConfig& c) {
        c.warps = NW;
        c.threads = NW * 32;
        c.smem = Tr::SMEM;
        int per_sm = 1;
        if (prepare() != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &per_sm, paged_decode_kernel<KV, D, DV, GP, NW, S>, c.threads, Tr::SMEM) !=
                cudaSuccess ||
            per_sm < 1) {
            cudaGetLastError();
            per_sm = 1;
        }
        c.ctas_per_sm = per_sm;
        c.supported = true;
    }

    static cudaError_t launch(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                              int group, int head_groups, int* launches, cudaStream_t st) {
        const int cpp = (g.block_size + kChunk - 1) / kChunk;
        cudaError_t e = prepare();
        if (e != cudaSuccess) return e;
        dim3 grid(static_cast<unsigned>(w.n_ctas), static_cast<unsigned>(head_groups));
        paged_decode_kernel<KV, D, DV, GP, NW, S><<<grid, NW * 32, Tr::SMEM, st>>>(g, w, a, group, cpp);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        *launches = 1;
        if (w.n_merge > 0) {
            dim3 mg(static_cast<unsigned>(w.n_merge), static_cast<unsigned>(head_groups));
            paged_decode_merge_kernel<GP, DV><<<mg, 128, 0, st>>>(g, w, a, group);
            e = cudaGetLastError();
            *launches = 2;
        }
        return e;
    }
};

// Dispatch over (storage type, head dims, GP); `f` receives a value of the Inst type.
template <typename F>
bool dispatch(const ArenaGeom& g, int gp, F&& f) {
    auto by_gp = [&](auto kv_tag, auto d_tag, auto dv_tag) -> bool {
        using KV = decltype(kv_tag);
        constexpr int D = decltype(d_tag)::value;
        constexpr int DV = decltype(dv_tag)::value;
        switch (gp) {
            case 1: f(Inst<KV, D, DV, 1>{}); return true;
            case 2: f(Inst<KV, D, DV, 2>{}); return true;
            case 4: f(Inst<KV, D, DV, 4>{}); return true;
            case 8: f(Inst<KV, D, DV, 8>{}); return true;
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
    dispatch(g, c.gp, [&](auto inst) { decltype(inst)::config(c); });
    return c;
}

cudaError_t launch_paged_decode(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                int* launches, cudaStream_t stream) {
    *launches = 0;
    if (w.n_ctas <= 0) return cudaSuccess;
    const int group = a.n_heads / g.heads_kv;
    const int gp = pick_gp(group);
    const int head_groups = (group + gp - 1) / gp;
    cudaError_t err = cudaErrorInvalidValue;
    dispatch(g, gp, [&](auto inst) {
        err = decltype(inst)::launch(g, w, a, group, head_groups, launches, stream);
    });
    return err;
}

}  // namespace gkv
