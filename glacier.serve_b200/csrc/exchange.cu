// Peer-memory exchange of split-KV partials over NVLink, fused with the merge that needs it.
//
// Each rank owns a mailbox in its own HBM, [2 parities][n_ranks][slot] floats followed by
// [2][n_ranks] epoch flags, mapped into every other rank's address space once (CUDA IPC).
// Per split-KV decode (epoch e, parity e & 1) a rank's decode kernels write its (out, lse)
// block straight into its OWN mailbox, slot [parity][me] -- no send buffer, no push kernel.
// Then ONE kernel (pull_merge_kernel, launched as a programmatic dependent of the decode):
//  * after griddepcontrol.wait (the decode and its merge have completed), threads 0..n-1 of
//    CTA 0 publish e in flag [parity][me] of every rank (fence.sc.sys, then st.release.sys);
//  * every CTA waits until all n_ranks flags of its own mailbox read e (ld.acquire.sys,
//    bounded: on expiry it raises kErrWaitTimeout and writes nothing);
//  * one warp per output row merges the n_ranks blocks by log-sum-exp, reading rank r's block
//    from rank r's mailbox with plain loads over NVLink (no TMA, no multicast).
// Two parities suffice: rank r rewrites its slot of parity p at epoch e+2 only after its own
// merge of e+1, which waited for every peer's flag of e+1, which each peer published only
// after its merge of e -- the last read of r's slot of epoch e -- had completed.
#include <cmath>

#include "gkv_device.cuh"
#include "kernels.h"

namespace gkv {

namespace {

constexpr uint32_t kFlagWaitLimit = 1u << 24;  // polls (with a short sleep) before giving up

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Loads from another GPU's memory that a later epoch rewrites: never served from L1.
__device__ __forceinline__ float ld_peer(const float* p) {
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float4 ld_peer4(const float4* p) {
    float4 v;
    asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// A slot holds out [rows][dv] fp32 (dv a multiple of 4), then lse [rows].
__global__ void __launch_bounds__(256) pull_merge_kernel(ExchangePeers p, int me, int parity, unsigned epoch,
                                                         int rows, int dv, const float* __restrict__ sinks,
                                                         int n_heads, float* __restrict__ out, int* err) {
    __shared__ int ready;
    pdl_wait();  // this rank's block is complete in its own mailbox
    const int n = p.n_ranks;
    if (blockIdx.x == 0 && threadIdx.x < n) {
        __threadfence_system();
        st_release_sys(p.flags[threadIdx.x] + parity * n + me, epoch);
    }
    if (threadIdx.x == 0) {
        const unsigned* fl = p.flags[me] + parity * n;
        int good = 1;
        for (int r = 0; r < n && good; ++r) {
            uint32_t it = 0;
            while (ld_acquire_sys(fl + r) != epoch) {
                if (++it > kFlagWaitLimit) {
                    good = 0;
                    atomicOr(err, kErrWaitTimeout);
                    break;
                }
                __nanosleep(64);
            }
        }
        ready = good;
    }
    __syncthreads();
    if (!ready) return;
    const int lane = threadIdx.x & 31;
    const int row = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    if (row >= rows) return;
    const int64_t slot_off = static_cast<int64_t>(parity) * n * p.slot;
    // Peer loads take on the order of a microsecond: each group of kGroup ranks' float4s is
    // issued back to back before any of them is used, so a row waits about one round trip
    // per group instead of one per rank.  The first group of the first dims is issued with the
    // lse loads, before the weights are known (a rank with no tokens is loaded and ignored: its
    // slot is mapped memory of any content), so the common dv <= 128, n <= 8 row takes one trip.
    constexpr int kGroup = 8;
    auto out_of = [&](int r, int d) {
        return reinterpret_cast<const float4*>(p.mbox[r] + slot_off + r * p.slot + static_cast<int64_t>(row) * dv + d);
    };
    // lane r < n holds rank r's lse of this row
    float l = -INFINITY;
    if (lane < n) l = ld_peer(p.mbox[lane] + slot_off + lane * p.slot + static_cast<int64_t>(rows) * dv + row);
    float4 v0[kGroup];
    const int d0 = lane * 4;
#pragma unroll
    for (int i = 0; i < kGroup; ++i)
        v0[i] = (i < n && d0 < dv) ? ld_peer4(out_of(i, d0)) : make_float4(0.f, 0.f, 0.f, 0.f);
    float M = l;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float sk = -INFINITY;
    if (sinks) {
        sk = __ldg(sinks + row % n_heads);
        M = fmaxf(M, sk);
    }
    const float w = (l == -INFINITY) ? 0.f : expf(l - M);
    float den = w;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (sk != -INFINITY) den += expf(sk - M);
    const float inv = den > 0.f ? 1.f / den : 0.f;
    for (int d = d0; d < dv; d += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r0 = 0; r0 < n; r0 += kGroup) {
            float4 v[kGroup];
            float wr[kGroup];
#pragma unroll
            for (int i = 0; i < kGroup; ++i) {
                const int r = r0 + i;
                wr[i] = __shfl_sync(0xffffffffu, w, r & 31);
                if (d == d0 && r0 == 0)
                    v[i] = v0[i];
                else  // no tokens there (its block may hold anything): weight 0, nothing loaded
                    v[i] = (r < n && wr[i] != 0.f) ? ld_peer4(out_of(r, d)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < kGroup; ++i) {
                if (r0 + i >= n || wr[i] == 0.f) continue;
                acc.x = fmaf(wr[i], v[i].x, acc.x);
                acc.y = fmaf(wr[i], v[i].y, acc.y);
                acc.z = fmaf(wr[i], v[i].z, acc.z);
                acc.w = fmaf(wr[i], v[i].w, acc.w);
            }
        }
        *reinterpret_cast<float4*>(out + static_cast<int64_t>(row) * dv + d) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
}

}  // namespace

float* exchange_slot(const ExchangePeers& p, int me, int parity) {
    return p.mbox[me] + (static_cast<int64_t>(parity) * p.n_ranks + me) * p.slot;
}

cudaError_t launch_exchange_pull_merge(const ExchangePeers& p, int me, int parity, unsigned epoch, int rows, int dv,
                                       const float* sinks, int n_heads, float* out, int* err, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    if (dv % 4 != 0) return cudaErrorInvalidValue;
    const int64_t threads = static_cast<int64_t>(rows) * 32;
    return launch_pdl(pull_merge_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, st, p,
                      me, parity, epoch, rows, dv, sinks, n_heads, out, err);
}

}  // namespace gkv
