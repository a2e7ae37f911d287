// Fused q/k/v prologue + KV append for sm_100a.
//
// Replaces the per-sequence steps that precede Store in the reference's batched runner
// (PagedTransformerRunner.ForwardBatch, src/Glacier.Serve/Inference/PagedAttention/
// PagedTransformerRunner.cs:612-634, and its prefill and single-token twins :431-450, :245-267):
// AddVector of the q/k/v biases (:612-614), ApplyQkNorm, a per-head RMSNorm of q and k
// (:616, :713-732), QuantKernels.RoPE with the YaRN inverse-frequency table and mscale
// (:619-631), and pool.Store of k and v (:634).  One launch does all of it for every token of
// the step: each warp takes one token; q rows are written back in place (ready for the decode
// or prefill that follows), k and v rows go straight into their arena slots, so the rotated k
// never makes a round trip through HBM.  The rotation angles depend on the position only, so a
// lane computes its few (sin, cos) pairs once and applies them to every q and k head of the
// token.
//
// The formulas of QuantKernels.RMSNorm and QuantKernels.RoPE are not in the reference tree
// (NuGet Glacier.Inference 1.7.0); the ones computed here are stated next to each step, and
// every step is an IEEE-rounded operation in a fixed order (no contraction by the compiler),
// so a CPU restatement of the same steps gives the same bits.
//
// Roofline: HBM.  Bytes per token = (n_heads * d) * 8 (q read + written) + heads_kv * (d + dv)
// * (4 + elem) (k, v read, arena written).
#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

// sin and cos of a float angle: Cody-Waite reduction by pi/2 in double precision (pi/2 split
// into two doubles, fused multiply-adds), then Taylor polynomials of sin and cos on |x| <= pi/4
// in float (Horner with fused multiply-adds; truncation error below 2^-28).
__device__ __forceinline__ void rope_sincos(float theta, float& s_out, float& c_out) {
    const double t = static_cast<double>(theta);
    const double k = rint(__dmul_rn(t, 0.63661977236758134308));  // 2/pi
    double r = __fma_rn(-k, 1.5707963267948966192, t);              // pi/2, high part
    r = __fma_rn(-k, 6.1232339957367660359e-17, r);                 // pi/2, low part
    const float x = __double2float_rn(r);
    const float x2 = __fmul_rn(x, x);
    // sin x = x + x^3 (-1/3! + x^2 (1/5! + x^2 (-1/7! + x^2 (1/9! - x^2/11!))))
    float ps = __fmaf_rn(x2, -2.5052108385441720e-8f, 2.7557319223985893e-6f);
    ps = __fmaf_rn(x2, ps, -1.9841269841269841e-4f);
    ps = __fmaf_rn(x2, ps, 8.3333333333333333e-3f);
    ps = __fmaf_rn(x2, ps, -1.6666666666666667e-1f);
    const float sn = __fmaf_rn(__fmul_rn(x, x2), ps, x);
    // cos x = 1 + x^2 (-1/2! + x^2 (1/4! + x^2 (-1/6! + x^2 (1/8! - x^2/10!))))
    float pc = __fmaf_rn(x2, -2.7557319223985891e-7f, 2.4801587301587302e-5f);
    pc = __fmaf_rn(x2, pc, -1.3888888888888889e-3f);
    pc = __fmaf_rn(x2, pc, 4.1666666666666667e-2f);
    pc = __fmaf_rn(x2, pc, -0.5f);
    const float cs = __fmaf_rn(x2, pc, 1.0f);
    switch (static_cast<long long>(k) & 3) {
        case 0: s_out = sn; c_out = cs; break;
        case 1: s_out = cs; c_out = -sn; break;
        case 2: s_out = -sn; c_out = -cs; break;
        default: s_out = -cs; c_out = sn; break;
    }
}

struct RopeArgs {
    int layer;
    float* q;                  // [n_tok][n_heads][d], rewritten in place
    const float* k;            // [n_tok][heads_kv][d]
    const float* v;            // [n_tok][heads_kv][dv]
    int n_tok, n_heads;
    const int32_t* positions;  // [n_tok]
    const float* inv_freq;     // [rope_dim / 2]
    int rope_dim, style;       // style 0: pairs (i, i + R/2); 1: pairs (2i, 2i + 1)
    float mscale;
    const float *q_bias, *k_bias, *v_bias, *q_norm, *k_norm;
    float eps;
    const int64_t* slots;      // [n_tok], -1 = padding (k/v not stored)
    int* err;
};

// `inv` is the reciprocal of an FP8 arena's (layer, head) scale; the other types ignore it.
template <typename KV>
__device__ __forceinline__ void store_elem(KV* p, float x, float inv);
template <>
__device__ __forceinline__ void store_elem<float>(float* p, float x, float) { *p = x; }
template <>
__device__ __forceinline__ void store_elem<__nv_bfloat16>(__nv_bfloat16* p, float x, float) {
    *p = __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ void store_elem<__half>(__half* p, float x, float) { *p = __float2half_rn(x); }
template <>
__device__ __forceinline__ void store_elem<__nv_fp8_e4m3>(__nv_fp8_e4m3* p, float x, float inv) {
    p->__x = __nv_cvt_float_to_fp8(x * inv, __NV_SATFINITE, __NV_E4M3);
}

// Angles of the pairs this lane's E elements belong to, for position pos: (sin, cos) per element
// (elements from rope_dim on get none).  NEOX pairs (i, i + R/2): element j < R/2 is pair j, and
// j >= R/2 pair j - R/2; interleaved pairs (2i, 2i+1): element j is pair j/2.  The angle is
// pos * inv_freq[i], one fp32 multiply.
template <int E>
__device__ __forceinline__ void lane_angles(const RopeArgs& a, int pos, int lane, float (&sn)[E], float (&cs)[E]) {
    const int R = a.rope_dim;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int j = lane * E + e;
        sn[e] = 0.f;
        cs[e] = 1.f;
        if (j < R) {
            const int i = a.style == 0 ? (j < R / 2 ? j : j - R / 2) : j / 2;
            rope_sincos(__fmul_rn(static_cast<float>(pos), __ldg(a.inv_freq + i)), sn[e], cs[e]);
        }
    }
}

// One q or k head row of D = 32 * E elements, lane l holding elements [l*E, (l+1)*E): bias,
// RMSNorm, rotation with the lane's precomputed angles.  RMSNorm: lane l sums the squares of its
// elements in order (x*x, then fused multiply-adds), a butterfly over lanes 16, 8, 4, 2, 1 adds
// the partial sums (every lane ends with the same value), r = sqrt(sum * (1/D) + eps) (1/D is
// exact: D is a power of two), inv = 1 / r, y = (x * inv) * w.  Rotation of pair (a, b):
// y_a = fma(x_a, c, -(x_b * s)), y_b = fma(x_b, c, x_a * s), each times mscale.  `nw` holds the
// lane's elements of the norm weight (read once per token).
template <int E>
__device__ __forceinline__ void prologue_row(float (&x)[E], const float* bias, bool norm, const float (&nw)[E],
                                             const RopeArgs& a, const float (&sn)[E], const float (&cs)[E],
                                             int lane) {
    constexpr int D = 32 * E;
    if (bias) {
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = __fadd_rn(x[e], __ldg(bias + lane * E + e));
    }
    if (norm) {
        float p = __fmul_rn(x[0], x[0]);
#pragma unroll
        for (int e = 1; e < E; ++e) p = __fmaf_rn(x[e], x[e], p);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, off));
        const float r = __fsqrt_rn(__fadd_rn(__fmul_rn(p, 1.f / static_cast<float>(D)), a.eps));
        const float inv = __fdiv_rn(1.f, r);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], inv), nw[e]);
    }
    const int R = a.rope_dim;
    if (R <= 0) return;
    if (a.style == 0) {
        // pairs (i, i + R/2): the partner of element j < R/2 sits (R/2)/E lanes up
        const int half = R / 2;
        const int dl = half / E;  // lanes between partners (the host checks half % E == 0)
        const bool low = lane * E < half;
        const int src = low ? lane + dl : lane - dl;
        float y[E];
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const float other = __shfl_sync(0xffffffffu, x[e], src & 31);
            y[e] = x[e];
            if (lane * E + e < R) {
                // low element: y = x*c - other*s; high element: y = x*c + other*s
                y[e] = low ? __fmaf_rn(x[e], cs[e], -__fmul_rn(other, sn[e]))
                           : __fmaf_rn(x[e], cs[e], __fmul_rn(other, sn[e]));
                y[e] = __fmul_rn(y[e], a.mscale);
            }
        }
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = y[e];
    } else {
        // pairs (2i, 2i+1): within a lane for even E, across lanes l and l^1 for E == 1
        if constexpr (E % 2 == 0) {
#pragma unroll
            for (int e = 0; e < E; e += 2) {
                if (lane * E + e < R) {
                    const float x0 = x[e], x1 = x[e + 1];
                    x[e] = __fmul_rn(__fmaf_rn(x0, cs[e], -__fmul_rn(x1, sn[e])), a.mscale);
                    x[e + 1] = __fmul_rn(__fmaf_rn(x1, cs[e], __fmul_rn(x0, sn[e])), a.mscale);
                }
            }
        } else {
            const float other = __shfl_xor_sync(0xffffffffu, x[0], 1);
            if (lane < R) {
                const bool even = (lane & 1) == 0;
                x[0] = even ? __fmaf_rn(x[0], cs[0], -__fmul_rn(other, sn[0]))
                            : __fmaf_rn(x[0], cs[0], __fmul_rn(other, sn[0]));
                x[0] = __fmul_rn(x[0], a.mscale);
            }
        }
    }
}

template <int E>
__device__ __forceinline__ void load_row(const float* p, float (&x)[E]) {
    if constexpr (E % 4 == 0) {
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            const float4 v = *reinterpret_cast<const float4*>(p + e);
            x[e] = v.x;
            x[e + 1] = v.y;
            x[e + 2] = v.z;
            x[e + 3] = v.w;
        }
    } else if constexpr (E == 2) {
        const float2 v = *reinterpret_cast<const float2*>(p);
        x[0] = v.x;
        x[1] = v.y;
    } else {
        x[0] = *p;
    }
}

template <int E>
__device__ __forceinline__ void store_row(float* p, const float (&x)[E]) {
    if constexpr (E % 4 == 0) {
#pragma unroll
        for (int e = 0; e < E; e += 4) *reinterpret_cast<float4*>(p + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
    } else if constexpr (E == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
    } else {
        *p = x[0];
    }
}

// One warp per token: the lane's angles are computed once and serve every q and k head of the
// token; q heads go U at a time (their loads issued together), then the k heads into the arena,
// then the v heads.
template <typename KV, int E>
__global__ void __launch_bounds__(256) rope_append_kernel(ArenaGeom g, RopeArgs a) {
    pdl_launch_dependents();  // the decode that follows waits for this grid before reading the arena
    constexpr int D = 32 * E;
    constexpr int U = 4;
    const int lane = threadIdx.x & 31;
    const int n_warps = static_cast<int>((static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5);
    for (int t = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5); t < a.n_tok;
         t += n_warps) {
        const int pos = __ldg(a.positions + t);
        float sn[E], cs[E], qw[E], kw[E];
        lane_angles<E>(a, pos, lane, sn, cs);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            qw[e] = a.q_norm ? __ldg(a.q_norm + lane * E + e) : 1.f;
            kw[e] = a.k_norm ? __ldg(a.k_norm + lane * E + e) : 1.f;
        }
        float* qt = a.q + static_cast<int64_t>(t) * a.n_heads * D + lane * E;
        for (int h0 = 0; h0 < a.n_heads; h0 += U) {
            float x[U][E];
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (h0 + u < a.n_heads) load_row<E>(qt + (h0 + u) * D, x[u]);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (h0 + u < a.n_heads) {  // warp-uniform
                    prologue_row<E>(x[u], a.q_bias ? a.q_bias + (h0 + u) * D : nullptr, a.q_norm != nullptr, qw, a, sn, cs,
                                    lane);
                    store_row<E>(qt + (h0 + u) * D, x[u]);
                }
            }
        }
        const int64_t slot = __ldg(a.slots + t);
        if (slot < 0) continue;  // padding token: nothing to store
        const int64_t blk = slot / g.block_size;
        const int off = static_cast<int>(slot - blk * g.block_size);
        if (blk >= g.total_blocks) {
            if (lane == 0 && a.err) atomicOr(a.err, kErrBadSlot);
            continue;
        }
        const float* kt = a.k + static_cast<int64_t>(t) * g.heads_kv * D + lane * E;
        for (int h0 = 0; h0 < g.heads_kv; h0 += U) {
            float x[U][E];
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (h0 + u < g.heads_kv) load_row<E>(kt + (h0 + u) * D, x[u]);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (h0 + u < g.heads_kv) {
                    prologue_row<E>(x[u], a.k_bias ? a.k_bias + (h0 + u) * D : nullptr, a.k_norm != nullptr, kw, a, sn, cs,
                                    lane);
                    KV* dst = static_cast<KV*>(g.k) + blk * g.k_block_stride + a.layer * g.k_layer_stride +
                              (h0 + u) * g.k_head_stride + static_cast<int64_t>(off) * D + lane * E;
                    const float inv = g.k_inv ? __ldg(g.k_inv + a.layer * g.heads_kv + h0 + u) : 1.f;
#pragma unroll
                    for (int e = 0; e < E; ++e) store_elem<KV>(dst + e, x[u][e], inv);
                }
            }
        }
        const int dv = g.v_head_dim;
        for (int h = 0; h < g.heads_kv; ++h) {
            const float* vp = a.v + (static_cast<int64_t>(t) * g.heads_kv + h) * dv;
            KV* dst = static_cast<KV*>(g.v) + blk * g.v_block_stride + a.layer * g.v_layer_stride +
                      h * g.v_head_stride + static_cast<int64_t>(off) * dv;
            const float inv = g.v_inv ? __ldg(g.v_inv + a.layer * g.heads_kv + h) : 1.f;
            for (int e = lane; e < dv; e += 32) {
                float x = __ldg(vp + e);
                if (a.v_bias) x = __fadd_rn(x, __ldg(a.v_bias + h * dv + e));
                store_elem<KV>(dst + e, x, inv);
            }
        }
    }
}

template <typename KV>
cudaError_t launch_typed(const ArenaGeom& g, const RopeArgs& a, cudaStream_t st) {
    int64_t blocks = (static_cast<int64_t>(a.n_tok) * 32 + 255) / 256;  // a warp per token
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    const dim3 grid(static_cast<unsigned>(blocks));
    switch (g.head_dim) {
        case 32: rope_append_kernel<KV, 1><<<grid, 256, 0, st>>>(g, a); break;
        case 64: rope_append_kernel<KV, 2><<<grid, 256, 0, st>>>(g, a); break;
        case 128: rope_append_kernel<KV, 4><<<grid, 256, 0, st>>>(g, a); break;
        case 256: rope_append_kernel<KV, 8><<<grid, 256, 0, st>>>(g, a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace

bool rope_append_supported(const ArenaGeom& g, int rope_dim) {
    if (g.head_dim != 32 && g.head_dim != 64 && g.head_dim != 128 && g.head_dim != 256) return false;
    if (rope_dim < 0 || rope_dim > g.head_dim || (rope_dim & 1)) return false;
    const int E = g.head_dim / 32;
    return (rope_dim / 2) % E == 0;  // NEOX partners a whole number of lanes apart
}

cudaError_t launch_rope_append(const ArenaGeom& g, const RopeAppendParams& p, cudaStream_t st) {
    if (p.n_tok <= 0) return cudaSuccess;
    RopeArgs a{p.layer, p.q, p.k, p.v, p.n_tok, p.n_heads, p.positions, p.inv_freq, p.rope_dim, p.style,
               p.mscale, p.q_bias, p.k_bias, p.v_bias, p.q_norm, p.k_norm, p.eps, p.slots, p.err};
    if (g.dtype == GKV_DTYPE_BF16) return launch_typed<__nv_bfloat16>(g, a, st);
    if (g.dtype == GKV_DTYPE_F16) return launch_typed<__half>(g, a, st);
    if (g.dtype == GKV_DTYPE_FP8_E4M3) return launch_typed<__nv_fp8_e4m3>(g, a, st);
    return launch_typed<float>(g, a, st);
}

}  // namespace gkv
