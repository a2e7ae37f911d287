// Log-sum-exp merge of one split segment's partials, run by the warp that completes the
// segment (fused into the decode kernels).
//
// Partials of a segment are contiguous slots s0 .. s0+ns-1; slot s holds, for each of the GP
// heads of the head group, an unnormalised accumulator acc[dv] and (max, sum) in the base-2
// domain.  The merge is three passes: per-head maxima and sums with the lanes striding over
// the slots (then warp reductions), and the accumulators with lane l owning dims
// [l*DV/32, (l+1)*DV/32) for every head at once, so each slot costs one round of independent
// loads instead of GP dependent ones.
#pragma once

#include "gkv_device.cuh"
#include "kernels.h"

namespace gkv {

// The work list a launch runs: `w` itself, or (static step layout, w.dyn set) the pointers
// and counts of the header the step's upload wrote at w.dyn.  The buffer comes from a host
// copy ordered before the launch, so it may be read before pdl_wait.
__device__ __forceinline__ DecodeWork resolve_work(DecodeWork w) {
    if (!w.dyn) return w;
    const int32_t* h = reinterpret_cast<const int32_t*>(w.dyn);
    auto at = [&](int k) { return reinterpret_cast<const int32_t*>(w.dyn + __ldg(h + k)); };
    w.max_blocks = __ldg(h + kHdrMaxBlocks);
    w.n_slots = __ldg(h + kHdrSlots);
    w.n_merge = __ldg(h + kHdrMerge);
    w.n_deferred = __ldg(h + kHdrDeferred);
    w.n_deferred_long = __ldg(h + kHdrDeferredLong);
    w.tables = at(kHdrTables);
    w.ctx_lens = at(kHdrCtx);
    w.piece_seg = at(kHdrPseg);
    w.piece_c0 = at(kHdrPc0);
    w.piece_c1 = at(kHdrPc1);
    w.piece_slot = at(kHdrPslot);
    w.piece_merge = at(kHdrPmerge);
    w.worker_piece_begin = at(kHdrWbeg);
    w.merge_seg = at(kHdrMseg);
    w.merge_slot0 = at(kHdrMs0);
    w.merge_nslots = at(kHdrMns);
    w.merge_deferred = at(kHdrMdef);
    return w;
}

// Block-table row of sequence b of a work list.
__device__ __forceinline__ int64_t table_row(const DecodeWork& w, int b) {
    return w.table_row ? static_cast<int64_t>(__ldg(w.table_row + b)) : static_cast<int64_t>(b);
}

// Natural-log softmax denominator from a base-2 running max and sum.
__device__ __forceinline__ float lse_ln(float m2, float l) {
    return (l > 0.f && m2 != -INFINITY) ? (m2 + log2f(l)) * 0.6931471805599453f : -INFINITY;
}

template <int GP, int DV>
__device__ __forceinline__ void merge_segment(const DecodeArgs& a, const DecodeWork& w, int hg,
                                              int s0, int ns, int b, int q_head0, int gcount,
                                              int lane) {
    constexpr int EPLV = DV / 32;
    constexpr float kL2e = 1.4426950408889634f;
    const int64_t b0 = (static_cast<int64_t>(hg) * w.n_slots + s0) * GP;
    const float* ml = a.part_ml;
    float M[GP], Ls[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g) {
        M[g] = -INFINITY;
        Ls[g] = 0.f;
    }
    for (int s = lane; s < ns; s += 32) {
#pragma unroll
        for (int g = 0; g < GP; ++g) M[g] = fmaxf(M[g], __ldcg(ml + (b0 + s * GP + g) * 2));
    }
#pragma unroll
    for (int g = 0; g < GP; ++g) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) M[g] = fmaxf(M[g], __shfl_xor_sync(0xffffffffu, M[g], o));
    }
    for (int s = lane; s < ns; s += 32) {
#pragma unroll
        for (int g = 0; g < GP; ++g) {
            const int64_t ps = b0 + s * GP + g;
            const float mm = __ldcg(ml + ps * 2);
            if (M[g] != -INFINITY) Ls[g] += __ldcg(ml + ps * 2 + 1) * exp2f(mm - M[g]);
        }
    }
#pragma unroll
    for (int g = 0; g < GP; ++g) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) Ls[g] += __shfl_xor_sync(0xffffffffu, Ls[g], o);
    }
    float A[GP][EPLV];
#pragma unroll
    for (int g = 0; g < GP; ++g) {
#pragma unroll
        for (int e = 0; e < EPLV; ++e) A[g][e] = 0.f;
    }
#pragma unroll 2
    for (int s = 0; s < ns; ++s) {
#pragma unroll
        for (int g = 0; g < GP; ++g) {
            const int64_t ps = b0 + s * GP + g;
            const float mm = __ldcg(ml + ps * 2);
            const float f = (M[g] == -INFINITY) ? 0.f : exp2f(mm - M[g]);
            const float* ap = a.part_acc + ps * DV + lane * EPLV;
            if constexpr (EPLV % 4 == 0) {
#pragma unroll
                for (int e = 0; e < EPLV; e += 4) {
                    const float4 v = __ldcg(reinterpret_cast<const float4*>(ap + e));
                    A[g][e] = fmaf(f, v.x, A[g][e]);
                    A[g][e + 1] = fmaf(f, v.y, A[g][e + 1]);
                    A[g][e + 2] = fmaf(f, v.z, A[g][e + 2]);
                    A[g][e + 3] = fmaf(f, v.w, A[g][e + 3]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < EPLV; ++e) A[g][e] = fmaf(f, __ldcg(ap + e), A[g][e]);
            }
        }
    }
#pragma unroll
    for (int g = 0; g < GP; ++g) {
        if (g >= gcount) continue;
        const int qh = q_head0 + g;
        float L = Ls[g], f = 1.f, Mref = M[g];
        if (a.sinks || a.has_sink_all) {
            const float sk = (a.sinks ? __ldg(a.sinks + qh) : a.sink_all) * kL2e;
            const float M2 = fmaxf(M[g], sk);
            f = (M[g] == -INFINITY) ? 0.f : exp2f(M[g] - M2);
            L = L * f + exp2f(sk - M2);
            Mref = M2;
        }
        const float inv = L > 0.f ? f / L : 0.f;
        if (a.lse && lane == 0) a.lse[static_cast<int64_t>(b) * a.n_heads + qh] = lse_ln(Mref, L);
        float* op = a.out + (static_cast<int64_t>(b) * a.n_heads + qh) * DV + lane * EPLV;
#pragma unroll
        for (int e = 0; e < EPLV; ++e) op[e] = A[g][e] * inv;
    }
}

// Unnormalised log-sum-exp merge of partial slots [s_lo, s_hi) of one (segment, head), by one
// warp; lane l owns dims [l*DV/32, (l+1)*DV/32).  Slot s's (max, sum) sits at part_ml[(base +
// s*GP)*2] (base 2), its accumulator at part_acc[(base + s*GP)*DV].  Two phases, so that nothing
// waits on a running state: lane j reads slot s_lo + j's (max, sum) while the first eight slots'
// accumulators are already in flight, one warp reduction gives the max M, each slot's weight
// 2^(m_s - M) stays in its own lane, and the accumulators are summed in batches of eight
// independent loads, each weight fetched from its lane with one shuffle.  On return every lane
// holds M (-inf when no slot has scores), the sum L and its accumulator dims, both relative to M.
template <int GP, int DV>
__device__ __forceinline__ void merge_slots(const DecodeArgs& a, int64_t base, int s_lo, int s_hi, int lane,
                                            float& M, float& L, float (&A)[DV / 32]) {
    constexpr int EPLV = DV / 32;
    constexpr int kBatch = 8;
    const int ns = s_hi - s_lo;
    auto ml_of = [&](int j) {
        return j < ns ? __ldcg(reinterpret_cast<const float2*>(a.part_ml + (base + static_cast<int64_t>(s_lo + j) * GP) * 2))
                      : make_float2(-INFINITY, 0.f);
    };
    auto acc_of = [&](int j, float (&v)[EPLV]) {
        const float* ap = a.part_acc + (base + static_cast<int64_t>(s_lo + j) * GP) * DV + lane * EPLV;
        if constexpr (EPLV % 4 == 0) {
#pragma unroll
            for (int e = 0; e < EPLV; e += 4) {
                const float4 x = __ldcg(reinterpret_cast<const float4*>(ap + e));
                v[e] = x.x;
                v[e + 1] = x.y;
                v[e + 2] = x.z;
                v[e + 3] = x.w;
            }
        } else if constexpr (EPLV == 2) {
            const float2 x = __ldcg(reinterpret_cast<const float2*>(ap));
            v[0] = x.x;
            v[1] = x.y;
        } else {
#pragma unroll
            for (int e = 0; e < EPLV; ++e) v[e] = __ldcg(ap + e);
        }
    };
    float v0[kBatch][EPLV];
#pragma unroll
    for (int k = 0; k < kBatch; ++k)
        if (k < ns) acc_of(k, v0[k]);
    float2 st = ml_of(lane);
    M = st.x;
    for (int c0 = 32; c0 < ns; c0 += 32) M = fmaxf(M, ml_of(c0 + lane).x);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    L = 0.f;
#pragma unroll
    for (int e = 0; e < EPLV; ++e) A[e] = 0.f;
    for (int c0 = 0; c0 < ns; c0 += 32) {
        if (c0 > 0) st = ml_of(c0 + lane);
        const float wgt = (st.x == -INFINITY || M == -INFINITY) ? 0.f : exp2f(st.x - M);
        L = fmaf(st.y, wgt, L);
        const int n = ns - c0 < 32 ? ns - c0 : 32;
        for (int k0 = 0; k0 < n; k0 += kBatch) {
            float v[kBatch][EPLV];
            if (c0 == 0 && k0 == 0) {
#pragma unroll
                for (int k = 0; k < kBatch; ++k)
#pragma unroll
                    for (int e = 0; e < EPLV; ++e) v[k][e] = v0[k][e];
            } else {
#pragma unroll
                for (int k = 0; k < kBatch; ++k)
                    if (k0 + k < n) acc_of(c0 + k0 + k, v[k]);
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const float wk = __shfl_sync(0xffffffffu, wgt, (k0 + k) & 31);
                if (k0 + k < n) {
#pragma unroll
                    for (int e = 0; e < EPLV; ++e) A[e] = fmaf(wk, v[k][e], A[e]);
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
}

// Normalises one merged row (plus the optional sink) and writes it, and its natural-log
// denominator when the caller asked for it.
template <int DV>
__device__ __forceinline__ void finish_row(const DecodeArgs& a, int b, int qh, float M, float L,
                                           const float (&A)[DV / 32], int lane) {
    constexpr int EPLV = DV / 32;
    constexpr float kL2e = 1.4426950408889634f;
    float f = 1.f, Mref = M;
    if (a.sinks || a.has_sink_all) {
        const float sk = (a.sinks ? __ldg(a.sinks + qh) : a.sink_all) * kL2e;
        const float M2 = fmaxf(M, sk);
        f = (M == -INFINITY) ? 0.f : exp2f(M - M2);
        L = L * f + exp2f(sk - M2);
        Mref = M2;
    }
    const float inv = L > 0.f ? f / L : 0.f;
    float* op = a.out + (static_cast<int64_t>(b) * a.n_heads + qh) * DV + lane * EPLV;
#pragma unroll
    for (int e = 0; e < EPLV; ++e) op[e] = A[e] * inv;
    if (a.lse && lane == 0) a.lse[static_cast<int64_t>(b) * a.n_heads + qh] = lse_ln(Mref, L);
}

// Merge of the segments split into more than kFusedMergeMaxSlots pieces, run as a second
// launch.  The deferred list starts with the w.n_deferred_long segments of more than
// kWarpMergeMaxSlots slots: each (long segment, head of a head group) gets a CTA of eight warps,
// warp k merging an eighth of the slots, the eight results combined through shared memory by warp
// 0.  The remaining (short segment, head) items get one warp each, eight per CTA, after the long
// ones.  These "CTA items" are numbered 0 .. n_items-1; CTA x takes item x (LOOP = false: one CTA
// per item) or items x, x + gridDim.x, ... (LOOP: the fixed grid of the static step layout).
// Every item has one role for the whole CTA, so the barriers are CTA-uniform.
template <int GP, int DV, bool LOOP>
__global__ void __launch_bounds__(256) deferred_merge_kernel(ArenaGeom g, DecodeWork w, DecodeArgs a, int group,
                                                         int head_groups) {
    static_assert(DV % 32 == 0, "DV must be a multiple of 32");
    constexpr int EPLV = DV / 32;
    constexpr int NW = 8;
    __shared__ float sm_m[NW], sm_l[NW];
    __shared__ __align__(16) float sm_a[NW][DV];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // the merge list comes from the step's host copy; the partials are the previous
    // (decode) kernel's output.  LOOP is only launched in the static step layout.
    if constexpr (LOOP) w = resolve_work(w);
    const int per_entry = head_groups * GP;
    const int long_ctas = w.n_deferred_long * per_entry;
    const int n_items = long_ctas + ((w.n_deferred - w.n_deferred_long) * per_entry + NW - 1) / NW;
    // One item's merge entry.  The first item's is read before pdl_wait: it comes from the
    // step's host copy, so its load latency overlaps the decode's tail.
    struct Item {
        bool cta_role, live;
        int hg, gg, seg, s0, ns;
    };
    auto prep = [&](int item) {
        Item r;
        r.cta_role = item < long_ctas;
        r.live = item < n_items;
        int di, y;
        if (r.cta_role) {
            di = item / per_entry;
            y = item - di * per_entry;
        } else {
            const int it = (item - long_ctas) * NW + warp;
            r.live = r.live && it < (w.n_deferred - w.n_deferred_long) * per_entry;
            const int k = r.live ? it / per_entry : 0;
            y = it - k * per_entry;
            di = w.n_deferred_long + k;
        }
        r.hg = y / GP;
        r.gg = y - r.hg * GP;
        const int mi = r.live ? __ldg(w.merge_deferred + di) : 0;
        r.seg = r.live ? __ldg(w.merge_seg + mi) : 0;
        r.s0 = r.live ? __ldg(w.merge_slot0 + mi) : 0;
        r.ns = r.live ? __ldg(w.merge_nslots + mi) : 0;
        return r;
    };
    Item cur = prep(static_cast<int>(blockIdx.x));
    pdl_launch_dependents();
    pdl_wait();
    // LOOP (the static layout's fixed grid): items x, x + gridDim.x, ...; otherwise item x alone
    const int step = LOOP ? static_cast<int>(gridDim.x) : n_items;
#pragma unroll 1
    for (int item = static_cast<int>(blockIdx.x); item < n_items; item += step) {
        if (item != static_cast<int>(blockIdx.x)) cur = prep(item);
        const bool cta_role = cur.cta_role;
        const int hg = cur.hg, gg = cur.gg, s0 = cur.s0, ns = cur.ns;
        const int b = cur.seg / g.heads_kv;
        const int h = cur.seg - b * g.heads_kv;
        const int q_head0 = h * group + hg * GP;
        const int gcount = min(GP, group - hg * GP);
        if (!cur.live || gg >= gcount) continue;  // CTA-uniform in the CTA role
        const int64_t base = (static_cast<int64_t>(hg) * w.n_slots + s0) * GP + gg;  // + s * GP
        float M, L, A[EPLV];
        if (!cta_role) {
            merge_slots<GP, DV>(a, base, 0, ns, lane, M, L, A);
            finish_row<DV>(a, b, q_head0 + gg, M, L, A, lane);
            continue;
        }
        const int per = (ns + NW - 1) / NW;
        const int lo = min(ns, warp * per), hi = min(ns, lo + per);
        merge_slots<GP, DV>(a, base, lo, hi, lane, M, L, A);
        if (lane == 0) {
            sm_m[warp] = M;
            sm_l[warp] = L;
        }
#pragma unroll
        for (int e = 0; e < EPLV; ++e) sm_a[warp][lane * EPLV + e] = A[e];
        __syncthreads();
        if (warp == 0) {
            float Mt = sm_m[0];
#pragma unroll
            for (int k = 1; k < NW; ++k) Mt = fmaxf(Mt, sm_m[k]);
            float Lt = 0.f, At[EPLV];
#pragma unroll
            for (int e = 0; e < EPLV; ++e) At[e] = 0.f;
#pragma unroll
            for (int k = 0; k < NW; ++k) {
                const float f = (sm_m[k] == -INFINITY || Mt == -INFINITY) ? 0.f : exp2f(sm_m[k] - Mt);
                Lt = fmaf(sm_l[k], f, Lt);
#pragma unroll
                for (int e = 0; e < EPLV; ++e) At[e] = fmaf(f, sm_a[k][lane * EPLV + e], At[e]);
            }
            finish_row<DV>(a, b, q_head0 + gg, Mt, Lt, At, lane);
        }
        __syncthreads();  // warp 0 has read the shared arrays before the next item writes them
    }
}

// Cross-part merge of normalised outputs with their log-sum-exps (multi-GPU split-KV: the
// parts are the ranks' block ranges).  One warp per row (= sequence x query head), lanes
// over dims.
static __global__ void __launch_bounds__(256) lse_merge_kernel(const float* __restrict__ parts, int n_parts,
                                                        int rows, int dv, const float* __restrict__ sinks,
                                                        int n_heads, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const int64_t part_stride = static_cast<int64_t>(rows) * (dv + 1);
    const float* lses = parts + static_cast<int64_t>(rows) * dv;  // lse block of part 0
    float M = -INFINITY;
    for (int p = 0; p < n_parts; ++p) M = fmaxf(M, __ldg(lses + p * part_stride + row));
    float sk = -INFINITY;
    if (sinks) {
        sk = __ldg(sinks + row % n_heads);
        M = fmaxf(M, sk);
    }
    float den = (M == -INFINITY) ? 0.f : ((sk == -INFINITY) ? 0.f : expf(sk - M));
    for (int p = 0; p < n_parts; ++p) {
        const float l = __ldg(lses + p * part_stride + row);
        if (l != -INFINITY) den += expf(l - M);
    }
    for (int d = lane; d < dv; d += 32) {
        float acc = 0.f;
        for (int p = 0; p < n_parts; ++p) {
            const float l = __ldg(lses + p * part_stride + row);
            if (l == -INFINITY) continue;
            acc = fmaf(expf(l - M), __ldg(parts + p * part_stride + row * dv + d), acc);
        }
        out[row * dv + d] = den > 0.f ? acc / den : 0.f;
    }
}

}  // namespace gkv
