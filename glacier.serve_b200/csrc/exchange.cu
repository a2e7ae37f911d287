// Peer-memory exchange of split-KV partials over NVLink, and the merge that waits for it.
//
// Each rank owns a mailbox in its own HBM, [2 parities][n_ranks][slot] floats followed by
// [2][n_ranks] epoch flags, mapped into every other rank's address space once (CUDA IPC).
// Per split-KV decode (epoch e, parity e & 1):
//  * push_kernel: CTA r stores this rank's (out, lse) block into rank r's mailbox slot
//    [parity][me] with plain 16-byte stores to peer memory (no TMA, no multicast), fences at
//    system scope and publishes e in rank r's flag [parity][me] (st.release.sys).
//  * wait_merge_kernel: every CTA waits until all n_ranks flags of its own mailbox read e
//    (ld.acquire.sys, bounded: on expiry it raises kErrWaitTimeout and writes nothing), then
//    merges the blocks by log-sum-exp exactly as lse_merge_kernel.
// Two parities suffice: a rank pushes epoch e+2 only after its merge of e+1, which waited for
// every peer's push of e+1, which each peer issued after its own merge of e.
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

__global__ void __launch_bounds__(1024) push_kernel(const float4* __restrict__ src, int64_t n4, ExchangePeers p,
                                                    int me, unsigned epoch, int parity) {
    const int r = blockIdx.x;
    float4* dst = reinterpret_cast<float4*>(p.mbox[r] + (static_cast<int64_t>(parity) * p.n_ranks + me) * p.slot);
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = src[i];
    __threadfence_system();  // this thread's stores reach rank r before the flag below
    __syncthreads();
    if (threadIdx.x == 0) st_release_sys(p.flags[r] + parity * p.n_ranks + me, epoch);
}

__global__ void __launch_bounds__(256) wait_merge_kernel(const float* __restrict__ mbox, const unsigned* flags,
                                                         int n_parts, int64_t slot, int rows, int dv,
                                                         const float* __restrict__ sinks, int n_heads,
                                                         float* __restrict__ out, unsigned epoch, int* err) {
    __shared__ int ready;
    if (threadIdx.x == 0) {
        int good = 1;
        for (int r = 0; r < n_parts && good; ++r) {
            uint32_t it = 0;
            while (ld_acquire_sys(flags + r) != epoch) {
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
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    // the blocks were written by other GPUs: read through L2 (never a stale L1 line)
    const float* lses = mbox + static_cast<int64_t>(rows) * dv;  // lse block of part 0
    float M = -INFINITY;
    for (int p = 0; p < n_parts; ++p) M = fmaxf(M, __ldcg(lses + p * slot + row));
    float sk = -INFINITY;
    if (sinks) {
        sk = __ldg(sinks + row % n_heads);
        M = fmaxf(M, sk);
    }
    float den = (M == -INFINITY) ? 0.f : ((sk == -INFINITY) ? 0.f : expf(sk - M));
    for (int p = 0; p < n_parts; ++p) {
        const float l = __ldcg(lses + p * slot + row);
        if (l != -INFINITY) den += expf(l - M);
    }
    for (int d = lane; d < dv; d += 32) {
        float acc = 0.f;
        for (int p = 0; p < n_parts; ++p) {
            const float l = __ldcg(lses + p * slot + row);
            if (l == -INFINITY) continue;
            acc = fmaf(expf(l - M), __ldcg(mbox + p * slot + row * dv + d), acc);
        }
        out[row * dv + d] = den > 0.f ? acc / den : 0.f;
    }
}

}  // namespace

cudaError_t launch_exchange_push(const float* src, int64_t n_floats, const ExchangePeers& p, int me, unsigned epoch,
                                 int parity, cudaStream_t st) {
    if (n_floats <= 0) return cudaSuccess;
    const int64_t n4 = (n_floats + 3) / 4;  // src and the slots hold whole float4s
    push_kernel<<<static_cast<unsigned>(p.n_ranks), 1024, 0, st>>>(reinterpret_cast<const float4*>(src), n4, p, me,
                                                                   epoch, parity);
    return cudaGetLastError();
}

cudaError_t launch_exchange_merge(const float* mbox_parity, const unsigned* flags_parity, int n_parts, int64_t slot,
                                  int rows, int dv, const float* sinks, int n_heads, float* out, unsigned epoch,
                                  int* err, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    const int64_t threads = static_cast<int64_t>(rows) * 32;
    wait_merge_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(
        mbox_parity, flags_parity, n_parts, slot, rows, dv, sinks, n_heads, out, epoch, err);
    return cudaGetLastError();
}

}  // namespace gkv
