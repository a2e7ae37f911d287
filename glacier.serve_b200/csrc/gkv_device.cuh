// Device-side helpers shared by the sm_100a kernels: bf16 unpacking, mbarrier / bulk-copy
// (TMA, non-multicast) wrappers with bounded waits, and the error-flag bits kernels raise.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace gkv {

// Bits OR-ed into the step workspace's device error word.
enum : int {
    kErrBadBlock = 1,      // a block id outside [0, total_blocks) reached a kernel
    kErrWaitTimeout = 2,   // a bounded mbarrier wait expired
    kErrBadSlot = 4        // an append slot outside the arena
};

// Upper bound of try_wait polls before a wait is declared stuck.  Each try_wait blocks for
// a hardware-defined slice, so this bounds a wait to well under a minute while being
// unreachable in correct operation.
constexpr uint32_t kWaitLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Makes the mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

// Bounded parity wait; returns false if the barrier did not complete within kWaitLimit
// polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Bulk (non-tensor) global -> shared copy completing on an mbarrier.  No multicast: the
// source is always this GPU's own arena.  dst, src and bytes must be 16-byte aligned.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Tiled 3-D TMA load (no multicast) of one box into shared memory, completing on `bar`.
// `tmap` is the address of a __grid_constant__ CUtensorMap kernel parameter.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A(16x8 bf16, row) * B(8x8 bf16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// Two fp32 values as one bf16x2 word (lo in bits 0-15), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Splits x into bf16 hi + lo with x ~= hi + lo to about 16 mantissa bits.
__device__ __forceinline__ void split_bf16(float x, float& hi, float& lo) {
    hi = __bfloat162float(__float2bfloat16_rn(x));
    lo = x - hi;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t lo16) {
    return __uint_as_float(lo16 << 16);
}

// Loads EPL consecutive KV elements from shared memory as fp32.
template <typename KV, int EPL>
struct SmemVec;

template <int EPL>
struct SmemVec<float, EPL> {
    static __device__ __forceinline__ void load(const float* p, float (&x)[EPL]) {
        if constexpr (EPL == 1) {
            x[0] = p[0];
        } else if constexpr (EPL == 2) {
            float2 v = *reinterpret_cast<const float2*>(p);
            x[0] = v.x; x[1] = v.y;
        } else {
            static_assert(EPL % 4 == 0, "EPL");
#pragma unroll
            for (int i = 0; i < EPL; i += 4) {
                float4 v = *reinterpret_cast<const float4*>(p + i);
                x[i] = v.x; x[i + 1] = v.y; x[i + 2] = v.z; x[i + 3] = v.w;
            }
        }
    }
};

template <int EPL>
struct SmemVec<__nv_bfloat16, EPL> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&x)[EPL]) {
        const uint16_t* u = reinterpret_cast<const uint16_t*>(p);
        if constexpr (EPL == 1) {
            x[0] = bf16_bits_to_f32(u[0]);
        } else if constexpr (EPL == 2) {
            uint32_t w = *reinterpret_cast<const uint32_t*>(u);
            x[0] = __uint_as_float(w << 16);
            x[1] = __uint_as_float(w & 0xffff0000u);
        } else if constexpr (EPL == 4) {
            uint2 w = *reinterpret_cast<const uint2*>(u);
            x[0] = __uint_as_float(w.x << 16); x[1] = __uint_as_float(w.x & 0xffff0000u);
            x[2] = __uint_as_float(w.y << 16); x[3] = __uint_as_float(w.y & 0xffff0000u);
        } else {
            static_assert(EPL % 8 == 0, "EPL");
#pragma unroll
            for (int i = 0; i < EPL; i += 8) {
                uint4 w = *reinterpret_cast<const uint4*>(u + i);
                x[i + 0] = __uint_as_float(w.x << 16); x[i + 1] = __uint_as_float(w.x & 0xffff0000u);
                x[i + 2] = __uint_as_float(w.y << 16); x[i + 3] = __uint_as_float(w.y & 0xffff0000u);
                x[i + 4] = __uint_as_float(w.z << 16); x[i + 5] = __uint_as_float(w.z & 0xffff0000u);
                x[i + 6] = __uint_as_float(w.w << 16); x[i + 7] = __uint_as_float(w.w & 0xffff0000u);
            }
        }
    }
};

}  // namespace gkv
