// Chunked causal prefill over the paged arena on the 5th-generation tensor cores (tcgen05,
// accumulators in tensor memory).
//
// The reference's CPU runner attends a prefill chunk one query at a time
// (PagedTransformerRunner.ForwardPrefillSubBatch, PagedTransformerRunner.cs:424-471): the
// chunk's K/V are stored first, then query t runs ComputeAttention with pos = start + t,
// whose causal length is min(TokenCount, pos + 1) (PagedAttentionKernel.cs:41).  Here one
// CTA takes 128 consecutive queries of one (sequence, query head) and streams the
// sequence's pages in tiles of 64 keys:
//
//  * warps 8 and 9 (TMA producers, K and V): the Q tile once (two boxes of 128 rows x 64
//    dims), then per key tile one box per page (16 slots; 8 when the block size is not a
//    multiple of 16) and dim half, gathered from the arena through the block table with tiled
//    cp.async.bulk.tensor (128-byte swizzle, no multicast) into 2-stage K and V rings.  Each
//    lane issues one box: a TMA instruction occupies its issuing thread for on the order of
//    a hundred cycles, so one thread alone starves the tensor cores.  K and V have their own
//    warps so that V (which waits for P V two tiles back) never holds back K.
//  * warp 10 (one thread issues): S = Q K^T (M=128, N=64, K=128: 8 tcgen05.mma kind::f16,
//    both operands K-major in shared memory) into one of two TMEM S buffers, then
//    O += P V (M=128, N=128, K=64: 4 MMAs, P read from TMEM, V MN-major in shared memory).
//    S of tile j+1 is issued before P V of tile j, so the tensor pipe works while the
//    softmax runs; the issuer never waits for its own MMAs (they execute in issue order).
//  * warps 0-7 (two threads per query row through the 16x32bx2 TMEM shape): load S, causal
//    mask, base-2 online softmax with lazy rescaling (O in TMEM is rescaled only when the
//    running max grows by more than 8, so P stays <= 2^8), P in the arena's 16-bit type
//    (bf16 or fp16; A and B of one MMA share it) written back over its own S columns.  Epilogue: O / l through shared memory as coalesced fp32 rows.
//
// Two CTAs share an SM (96 KB shared memory and 256 TMEM columns each), so one CTA's softmax
// overlaps the other's MMAs; one CTA with two Q tiles sharing K/V measured slower (its
// single issuer waits on whichever tile's softmax is late), and so did a third K stage.
// Every mbarrier wait is bounded: on expiry the CTA raises kErrWaitTimeout, lets its copies
// and MMAs finish and frees its TMEM.
#include <cuda.h>

#include <atomic>
#include <cmath>
#include <type_traits>

#include "gkv_device.cuh"
#include "kernels.h"
#include "../../include/glacier_kv.h"

namespace gkv {

namespace {

constexpr int kBM = 128;                           // query rows per CTA
constexpr int kBN = 64;                            // keys per tile
constexpr int kD = 128;                            // head_dim = v_head_dim
constexpr int kSoftmaxWarps = 8;                   // two threads per query row
constexpr int kKWarp = 8, kVWarp = 9, kMmaWarp = 10;  // K producer, V producer, MMA issuer
constexpr int kThreads = 352;
constexpr uint32_t kQBytes = kBM * kD * 2;         // 32 KB
constexpr uint32_t kQHalf = kQBytes / 2;           // 128 rows x 128 B (64 dims)
constexpr uint32_t kTile = kBN * kD * 2;           // 16 KB: one K or V tile
constexpr uint32_t kHalf = kTile / 2;              // 64 rows x 128 B
constexpr uint32_t kTmemCols = 256;                // S0 [0,64) S1 [64,128) O [128,256)
constexpr uint32_t kColO = 128;
constexpr size_t kSmemData = kQBytes + 4 * kTile;  // Q + 2 K stages + 2 V stages = 96 KB
constexpr size_t kSmem = kSmemData + 256 + 1024;   // + barriers + 1024-byte alignment slack
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;

// Instruction descriptor of tcgen05.mma kind::f16 with fp32 D, A K-major, and A and B both
// bf16 (format 1) or both fp16 (format 0).
constexpr uint32_t idesc_16(int m, int n, bool b_mn_major, bool f16) {
    const uint32_t fmt = f16 ? 0u : 1u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// One lane of a producer warp per TMA box.  A key tile of K (or of V) is 64 / R boxes of R
// keys (R = 16: a whole 16-slot page; R = 8 otherwise) for each dim half: lane l < 2*64/R
// loads rows [chunk*R, chunk*R + R) of dims [half*64, half*64 + 64), chunk = l/2, half = l%2.
// A TMA instruction costs its issuing thread on the order of a hundred cycles, so one thread
// cannot feed the tensor cores; 8 or 16 lanes in parallel can.
template <int R>
struct BoxLane {
    static constexpr int kBoxes = kBN / R;  // boxes per dim half per tile
    int chunk, half;
    bool active;
    __device__ __forceinline__ explicit BoxLane(int lane) {
        chunk = (lane >> 1) % kBoxes;
        half = lane & 1;
        active = lane < 2 * kBoxes;
    }
    // Block-table entry of this lane's box in tile j (raw: checked where it is used, so the
    // load can be issued a tile ahead without stalling), or -1 past the item's keys.
    __device__ __forceinline__ int block_of(int j, int n_keys, const int32_t* trow, int block_size) const {
        const int key = j * kBN + chunk * R;
        return (active && key < n_keys) ? __ldg(trow + key / block_size) : -1;
    }
    // Bytes a tile with keys [key0, n_keys) delivers to its operand's barrier.
    static __device__ __forceinline__ uint32_t tile_bytes(int key0, int n_keys) {
        int n = (n_keys - key0 + R - 1) / R;
        if (n > kBoxes) n = kBoxes;
        return static_cast<uint32_t>(n) * 2u * R * 128u;
    }
};

template <int R, bool F16>
__global__ void __launch_bounds__(kThreads, 2)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv, const ArenaGeom g, const PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
    uint8_t* sQ = smem;
    uint8_t* sK = smem + kQBytes;
    uint8_t* sV = sK + 2 * kTile;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sV + 2 * kTile);
    uint64_t* q_full = bar;
    uint64_t* k_full = bar + 1;   // [2] per stage
    uint64_t* k_empty = bar + 3;  // [2]
    uint64_t* v_full = bar + 5;   // [2]
    uint64_t* v_empty = bar + 7;  // [2]
    uint64_t* s_full = bar + 9;   // [2] per S buffer
    uint64_t* p_full = bar + 11;  // [2]
    uint64_t* pv_done = bar + 13; // [2]
    uint64_t* drained = bar + 15;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 16);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 17);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x / a.n_heads;
    const int h = blockIdx.x - item * a.n_heads;
    const int32_t* it = a.items + static_cast<int64_t>(item) * kPrefillItemInts;
    const int seq = __ldg(it + 0), qpos0 = __ldg(it + 1), qrow0 = __ldg(it + 2);
    const int n_q = __ldg(it + 3), n_keys = __ldg(it + 4), tok = __ldg(it + 5);
    const int n_tiles = (n_keys + kBN - 1) / kBN;
    const int hkv = h / (a.n_heads / g.heads_kv);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(k_full + s, 1);
            mbar_init(k_empty + s, 1);
            mbar_init(v_full + s, 1);
            mbar_init(v_empty + s, 1);
            mbar_init(s_full + s, 1);
            mbar_init(p_full + s, kSoftmaxWarps * 32);
            mbar_init(pv_done + s, 1);
        }
        mbar_init(drained, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;

    if (warp == kKWarp || warp == kVWarp) {
        // ------------- TMA producers: one warp for K, one for V, one box per lane -------------
        // Separate warps: V of tile j waits for P V of tile j-2, which must not hold back K.
        using BL = BoxLane<R>;
        const BL bl(lane);
        const bool is_k = warp == kKWarp;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        uint8_t* ring = is_k ? sK : sV;
        const CUtensorMap* tm = is_k ? &tmk : &tmv;
        const int32_t* trow = a.tables + static_cast<int64_t>(seq) * a.max_blocks;
        uint32_t armed0 = 0, armed1 = 0;  // lane 0's expect_tx count per stage
        if (is_k && lane == 0) {
            mbar_arrive_expect_tx(q_full, kQBytes);
            tma_load_3d(sQ, &tmq, 0, h, qrow0, q_full);
            tma_load_3d(sQ + kQHalf, &tmq, 64, h, qrow0, q_full);
        }
        int blk = bl.block_of(0, n_keys, trow, g.block_size);
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            const int s = j & 1;
            // the next tile's table read is in flight while this tile waits for its stage
            const int blk_next = j + 1 < n_tiles ? bl.block_of(j + 1, n_keys, trow, g.block_size) : -1;
            if (j >= 2 && !__all_sync(~0u, mbar_wait(empty + s, ((j >> 1) & 1) ^ 1))) {
                ok = false;
                break;
            }
            if (__any_sync(~0u, *abort_flag != 0)) break;
            if (lane == 0) {
                mbar_arrive_expect_tx(full + s, BL::tile_bytes(j * kBN, n_keys));
                if (s) ++armed1; else ++armed0;
            }
            __syncwarp();  // expect_tx precedes every complete_tx of this stage
            if (blk >= 0 || (bl.active && j * kBN + bl.chunk * R < n_keys)) {
                int b = blk;
                if (b < 0 || b >= g.total_blocks) {  // validated on the host; never dereference it
                    atomicOr(a.err, kErrBadBlock);
                    b = 0;
                }
                const int z = static_cast<int>((static_cast<int64_t>(b) * g.layers + a.layer) * g.heads_kv + hkv);
                const int slot = (j * kBN + bl.chunk * R) % g.block_size;
                tma_load_3d(ring + s * kTile + bl.half * kHalf + bl.chunk * R * 128, tm, bl.half * 64, slot, z,
                            full + s);
            }
            blk = blk_next;
        }
        if (lane == 0) {
            if (!ok) {
                atomicOr(a.err, kErrWaitTimeout);
                *abort_flag = 1;
            }
            if (*abort_flag) {
                // every armed copy must land before the CTA's shared memory goes away
                if (is_k) mbar_wait(q_full, 0);
                if (armed0) mbar_wait(full, (armed0 - 1) & 1);
                if (armed1) mbar_wait(full + 1, (armed1 - 1) & 1);
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_16(kBM, kBN, false, F16);
            constexpr uint32_t kIdO = idesc_16(kBM, kD, true, F16);
            const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
            bool ok = mbar_wait(q_full, 0);
            tc_fence_after();
            for (int j = 0; ok && j <= n_tiles; ++j) {
                if (*abort_flag) break;
                if (j < n_tiles) {
                    const int b = j & 1;
                    // S buffer b last held P of tile j-2, read by the P V issued before this
                    // point: tcgen05.mma from one thread execute in issue order, so the write of
                    // S_j cannot overtake that read and the issuer never waits for its own MMAs.
                    if (!(ok = mbar_wait(k_full + b, (j >> 1) & 1))) break;
                    tc_fence_after();
                    const uint32_t kb = k_addr + b * kTile;
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk) {
                        const uint64_t da = umma_desc_sw128(q_addr + (kk >> 2) * kQHalf + (kk & 3) * 32, 16, 1024);
                        const uint64_t db = umma_desc_sw128(kb + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
                        umma_f16(tbase + b * kBN, da, db, kIdS, kk > 0 ? 1u : 0u);
                    }
                    umma_commit(s_full + b);
                    umma_commit(k_empty + b);
                }
                if (j >= 1) {
                    const int jj = j - 1, b = jj & 1;
                    if (!(ok = mbar_wait(p_full + b, (jj >> 1) & 1))) break;
                    if (!(ok = mbar_wait(v_full + b, (jj >> 1) & 1))) break;
                    tc_fence_after();
                    const uint32_t vb = v_addr + b * kTile;
#pragma unroll
                    for (int kk = 0; kk < kBN / 16; ++kk) {
                        // V tile [key][dv]: MN-major, 8-key groups 1 KB apart (SBO), dv 64-127
                        // in the second half (LBO)
                        const uint64_t dv = umma_desc_sw128(vb + kk * 2048, kHalf, 1024);
                        umma_f16_ts(tbase + kColO, tbase + b * kBN + kk * 8, dv, kIdO,
                                    (jj > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(pv_done + b);
                    umma_commit(v_empty + b);
                }
            }
            if (!ok) {
                atomicOr(a.err, kErrWaitTimeout);
                *abort_flag = 1;
            }
            umma_commit(drained);  // all MMAs of this CTA complete before TMEM is freed
            if (!mbar_wait(drained, 0)) atomicOr(a.err, kErrWaitTimeout);
        }
        __syncwarp();
    } else {
        // ---------------- softmax + epilogue: two threads per query row ----------------
        // Warp w owns TMEM lanes [row0, row0 + 16), row0 = 32*(w%4) + 16*(w/4) (its own lane
        // quarter); lane l takes row row0 + l%16 and key columns [32*(l/16), +32) of each tile
        // (the 16x32bx2 TMEM shape), so the two halves of a row meet in one warp (shfl 16).
        const int hc = lane >> 4;
        const int r16 = lane & 15;
        const int row0 = 32 * (warp & 3) + 16 * (warp >> 2);
        const int r = row0 + r16;
        const uint32_t t_w = tbase + (static_cast<uint32_t>(row0) << 16);
        const int qpos = qpos0 + r;
        const int limit = min(tok, qpos + 1);  // keys [0, limit) are visible to this row
        const float sl = a.scale * kLog2e;
        const int tail = n_keys - (n_tiles - 1) * kBN;  // valid keys of the last tile
        float m_run = -INFINITY, l_run = 0.f;           // l_run: this thread's half of the row sum
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            if (__any_sync(~0u, *abort_flag != 0)) {
                ok = false;
                break;
            }
            const int b = j & 1;
            if (!__all_sync(~0u, mbar_wait(s_full + b, (j >> 1) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sv[32];
            tmem_ld16x2_32<32>(t_w + b * kBN, sv);
            tmem_wait_ld();
            // raw scores; masked keys become -inf (sl > 0, so the max commutes with the scale)
            float x[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) x[c] = __uint_as_float(sv[c]);
            const int kb = j * kBN + hc * 32;
            if (kb + 32 > limit) {
#pragma unroll
                for (int c = 0; c < 32; ++c) x[c] = (kb + c < limit) ? x[c] : -INFINITY;
            }
            // three-input maxima (sm_100): 18 instructions instead of 31, four chains deep 4
            float mq[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                mq[k] = fmax3(x[k], x[k + 4], x[k + 8]);
                mq[k] = fmax3(mq[k], x[k + 12], x[k + 16]);
                mq[k] = fmax3(mq[k], x[k + 20], x[k + 24]);
                mq[k] = fmaxf(mq[k], x[k + 28]);
            }
            float mx = fmaxf(fmax3(mq[0], mq[1], mq[2]), mq[3]);
            mx = fmaxf(mx, __shfl_xor_sync(~0u, mx, 16));  // the row's other half
            const float mt = mx * sl;
            const bool need = mt > m_run + kRescaleLog2;
            float alpha = 1.f;
            if (need) {
                alpha = fast_exp2(m_run - mt);  // 0 on the first tile (m_run = -inf)
                m_run = mt;
                l_run *= alpha;
            }
            // p = 2^(s * sl - m): one packed FMA per key pair, then the SFU
            uint32_t pk[16];
            float2 sum2 = make_float2(0.f, 0.f);
            const float2 sl2 = make_float2(sl, sl), nm2 = make_float2(-m_run, -m_run);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float2 e = __ffma2_rn(make_float2(x[2 * c], x[2 * c + 1]), sl2, nm2);
                const float2 p = make_float2(fast_exp2(e.x), fast_exp2(e.y));
                sum2 = __fadd2_rn(sum2, p);
                pk[c] = pack_16x2<F16>(p.x, p.y);
            }
            l_run += sum2.x + sum2.y;
            if (j == n_tiles - 1 && tail < kBN) {
                // keys past n_keys were never loaded (or are unwritten slots): zero their V
                // rows so that P = 0 never meets a non-finite value in the MMA
                if (!__all_sync(~0u, mbar_wait(v_full + b, (j >> 1) & 1))) {
                    ok = false;
                    break;
                }
                const int t = threadIdx.x;  // 0..255: (dim half, key) = (t / 64, t % 64) for t < 128
                const int row = t & (kBN - 1);
                if (t < 2 * kBN && row >= tail) {
                    uint4* dst = reinterpret_cast<uint4*>(sV + b * kTile + (t >> 6) * kHalf + (row >> 3) * 1024 +
                                                          (row & 7) * 128);
#pragma unroll
                    for (int i = 0; i < 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
                }
                fence_proxy_async_smem();
            }
            // P over the first 32 columns of its S buffer: keys 0-31 -> cols 0-15, 32-63 -> 16-31
            tmem_st16x2_16<16>(t_w + b * kBN, pk);
            if (j > 0 && __any_sync(~0u, need)) {
                // O holds P V up to tile j-1: wait for it, then rescale the rows that need it
                if (!__all_sync(~0u, mbar_wait(pv_done + ((j - 1) & 1), ((j - 1) >> 1) & 1))) {
                    tmem_wait_st();
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c2 = 0; c2 < 2; ++c2) {  // this thread's 64 of the 128 O columns
                    uint32_t o[32];
                    tmem_ld16x2_32<64>(t_w + kColO + c2 * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st16x2_32<64>(t_w + kColO + c2 * 32, o);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_full + b);
        }
        if (!ok) {
            atomicOr(a.err, kErrWaitTimeout);
            *abort_flag = 1;
        } else if (!__all_sync(~0u, mbar_wait(pv_done + ((n_tiles - 1) & 1), ((n_tiles - 1) >> 1) & 1))) {
            atomicOr(a.err, kErrWaitTimeout);
            *abort_flag = 1;
        } else {
            tc_fence_after();
            // all MMAs and copies are complete: the K/V rings (64 KB) become the staging area,
            // 8 KB = 16 rows x 512 B per warp, 16-byte chunks XOR-swizzled by row
            const float inv = 1.f / (l_run + __shfl_xor_sync(~0u, l_run, 16));
            uint8_t* stage = sK + warp * (16 * 512);
#pragma unroll 1
            for (int c2 = 0; c2 < 2; ++c2) {
                uint32_t o[32];
                tmem_ld16x2_32<64>(t_w + kColO + c2 * 32, o);
                tmem_wait_ld();
                const int ch0 = (hc * 64 + c2 * 32) / 4;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 v = make_float4(__uint_as_float(o[4 * q]) * inv, __uint_as_float(o[4 * q + 1]) * inv,
                                                 __uint_as_float(o[4 * q + 2]) * inv,
                                                 __uint_as_float(o[4 * q + 3]) * inv);
                    *reinterpret_cast<float4*>(stage + r16 * 512 + (((ch0 + q) ^ (r16 & 7)) << 4)) = v;
                }
            }
            __syncwarp();
#pragma unroll 4
            for (int rr = 0; rr < 16; ++rr) {
                const int t = row0 + rr;
                if (t < n_q) {
                    const float4 v = *reinterpret_cast<const float4*>(stage + rr * 512 + ((lane ^ (rr & 7)) << 4));
                    float* dst = a.out + (static_cast<int64_t>(qrow0 + t) * a.n_heads + h) * kD + lane * 4;
                    __stcs(reinterpret_cast<float4*>(dst), v);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tbase, kTmemCols);
    }
}

// Element conversion of q between the three GKV_DTYPE_* types (round to nearest even; fp16
// results saturate at +-65504 instead of rounding to infinity).
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) {
    return __float2half_rn(fminf(fmaxf(x, -65504.f), 65504.f));
}

template <typename S, typename D>
__global__ void convert_kernel(const S* __restrict__ src, D* __restrict__ dst, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = from_f32<D>(to_f32<S>(src[i]));
}

cudaError_t prefill_prepare() {
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
    for (auto k : {paged_prefill_tc_kernel<8, false>, paged_prefill_tc_kernel<16, false>,
                   paged_prefill_tc_kernel<8, true>, paged_prefill_tc_kernel<16, true>})
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem));
    if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace

bool prefill_tc_eligible(const ArenaGeom& g, int n_heads) {
    if ((g.dtype != GKV_DTYPE_BF16 && g.dtype != GKV_DTYPE_F16) || g.head_dim != kD || g.v_head_dim != kD)
        return false;
    if (g.block_size % 8 != 0 || g.heads_kv <= 0 || n_heads <= 0 || n_heads % g.heads_kv != 0) return false;
    if ((reinterpret_cast<uintptr_t>(g.k) | reinterpret_cast<uintptr_t>(g.v)) & 15) return false;
    const int64_t rows = static_cast<int64_t>(g.total_blocks) * g.layers * g.heads_kv;
    return rows < (int64_t{1} << 31) && tmap_encoder_available();
}

cudaError_t launch_convert(const void* src, int32_t src_dtype, void* dst, int32_t dst_dtype, int64_t n,
                           cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (!valid_q_dtype(src_dtype) || !valid_q_dtype(dst_dtype) || src_dtype == dst_dtype)
        return cudaErrorInvalidValue;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    const dim3 grid(static_cast<unsigned>(blocks));
    auto go = [&](auto s_tag, auto d_tag) {
        using S = decltype(s_tag);
        using D = decltype(d_tag);
        convert_kernel<S, D><<<grid, 256, 0, st>>>(static_cast<const S*>(src), static_cast<D*>(dst), n);
    };
    auto by_dst = [&](auto s_tag) {
        if (dst_dtype == GKV_DTYPE_F32) go(s_tag, float{});
        else if (dst_dtype == GKV_DTYPE_BF16) go(s_tag, __nv_bfloat16{});
        else go(s_tag, __half{});
    };
    if (src_dtype == GKV_DTYPE_F32) by_dst(float{});
    else if (src_dtype == GKV_DTYPE_BF16) by_dst(__nv_bfloat16{});
    else by_dst(__half{});
    return cudaGetLastError();
}

cudaError_t launch_paged_prefill_tc(const ArenaGeom& g, const PrefillArgs& a, const void* q16,
                                    int64_t total_q, cudaStream_t st) {
    if (a.n_items <= 0) return cudaSuccess;
    alignas(64) CUtensorMap mq;
    alignas(64) CUtensorMap ek;
    alignas(64) CUtensorMap ev;
    const uint64_t dims[3] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(a.n_heads),
                              static_cast<uint64_t>(total_q)};
    const uint64_t strides[2] = {static_cast<uint64_t>(kD) * 2, static_cast<uint64_t>(a.n_heads) * kD * 2};
    const uint32_t box[3] = {64, 1, static_cast<uint32_t>(kBM)};
    if (!encode_bf16_map3(&mq, q16, dims, strides, box)) return cudaErrorInvalidValue;
    // whole 16-slot pages per box when the block size allows, else 8-slot boxes.  The pool
    // caches the 16-slot pair; the decode's 8-slot pair is reused only when it is the 3-D view
    // this kernel's loads address (a 4-D decode map must never reach a 3-D load)
    const int rows = g.block_size % 16 == 0 ? 16 : 8;
    const void* ck = rows == 16 ? g.tmap_pk : (g.tmap_rank == 3 ? g.tmap_k : nullptr);
    const void* cv = rows == 16 ? g.tmap_pv : (g.tmap_rank == 3 ? g.tmap_v : nullptr);
    const CUtensorMap* tk = static_cast<const CUtensorMap*>(ck);
    const CUtensorMap* tv = static_cast<const CUtensorMap*>(cv);
    if (!tk || !tv) {
        if (!encode_arena_map(&ek, g.k, g, kD, rows) || !encode_arena_map(&ev, g.v, g, kD, rows))
            return cudaErrorInvalidValue;
        tk = &ek;
        tv = &ev;
    }
    cudaError_t e = prefill_prepare();
    if (e != cudaSuccess) return e;
    const int64_t grid = static_cast<int64_t>(a.n_items) * a.n_heads;
    if (grid > 0x7fffffff) return cudaErrorInvalidValue;
    const bool f16 = g.dtype == GKV_DTYPE_F16;
    auto kern = rows == 16 ? (f16 ? paged_prefill_tc_kernel<16, true> : paged_prefill_tc_kernel<16, false>)
                           : (f16 ? paged_prefill_tc_kernel<8, true> : paged_prefill_tc_kernel<8, false>);
    kern<<<static_cast<unsigned>(grid), kThreads, kSmem, st>>>(mq, *tk, *tv, g, a);
    return cudaGetLastError();
}

}  // namespace gkv
