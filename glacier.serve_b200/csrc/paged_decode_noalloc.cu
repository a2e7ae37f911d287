// Paged decode that allocates nothing.
//
// Some callers cannot call cudaMalloc on the decode path: hosts whose device memory belongs
// to another allocator (a framework's caching allocator, or a fixed region reserved at start
// -up under a hard memory budget) must not take memory behind its back, and serving loops
// cannot afford cudaMalloc/cudaFree there, which may synchronize the device.  They already
// own the KV arena, the queries and the output; what the decode additionally needs -- the
// step's packed block tables and context lengths, the split-KV work list and the partial
// (max, sum, acc) results of sequences split over several warps -- lives here in one
// file-scope __device__ array of fixed size instead of a per-pool workspace.
//
// Limits and sharing:
//  * kScratchBytes (16 MiB) per device holds everything; a call whose tables, work list or
//    partials do not fit is rejected with GKV_EINVAL before anything is enqueued.  Every GPU
//    that loads this library keeps the array until the process exits.
//  * Host-side staging uses a file-scope host array under a mutex (no heap allocation); the
//    upload is a cudaMemcpyAsync from that pageable buffer, which returns once the bytes are
//    staged, so the buffer is free for the next call.
//  * All calls on a device share the one array, which keeps the last call's contents.  Calls
//    whose kernels overlap on the GPU (different streams, no ordering between them) race on
//    it; order them on one stream or with events.
//  * The first call on each device resolves the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it.  No call may be captured
//    in a CUDA graph (its table upload would not be replayed): a capturing stream gets
//    GKV_ESTATE.
//  * A kernel that meets a bad block id or gives up a bounded wait ORs a bit into an error word
//    at the end of the array.  Calls never clear it; gkv_paged_decode_noalloc_status waits for
//    the caller's stream, reads the word and clears it, so bits of every call since the last
//    check are reported.
#include <chrono>
#include <mutex>
#include <thread>

#include "gkv_device.cuh"
#include "gkv_internal.h"

namespace gkv {

namespace {

constexpr size_t kScratchBytes = 16u << 20;   // per device
constexpr size_t kMetaBytes = 4u << 20;       // tables, context lengths, work list
constexpr size_t kErrOffset = kScratchBytes - 256;
constexpr size_t kPartBytes = kErrOffset - kMetaBytes;
constexpr int kMaxDevices = 64;

}  // namespace

// The scratch itself.  Host code must not use this name as an address (it is a host-side
// stand-in); the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

namespace {

std::mutex g_mu;
void* g_scratch_dev[kMaxDevices];
alignas(64) unsigned char g_stage[kMetaBytes];

size_t up16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

struct Layout {
    size_t tables, ctx, pseg, pc0, pc1, pslot, pmerge, wbeg, mseg, ms0, mns, mdef, counters, total;
};

Layout layout_for(int64_t batch, int64_t max_blocks, int64_t max_pieces, int64_t n_workers,
                  int64_t max_merge, int64_t head_groups) {
    Layout L{};
    size_t o = 0;
    auto take = [&](int64_t bytes) {
        const size_t at = o;
        o = up16(o + static_cast<size_t>(bytes));
        return at;
    };
    L.tables = take(batch * max_blocks * 4);
    L.ctx = take(batch * 4);
    L.pseg = take(max_pieces * 4);
    L.pc0 = take(max_pieces * 4);
    L.pc1 = take(max_pieces * 4);
    L.pslot = take(max_pieces * 4);
    L.pmerge = take(max_pieces * 4);
    L.wbeg = take((n_workers + 1) * 4);
    L.mseg = take(max_merge * 4);
    L.ms0 = take(max_merge * 4);
    L.mns = take(max_merge * 4);
    L.mdef = take(max_merge * 4);
    L.counters = take(max_merge * head_groups * 4);  // merge arrival counters, staged as zeros
    L.total = o;
    return L;
}

}  // namespace

}  // namespace gkv

using gkv::set_error;

extern "C" int gkv_paged_decode_noalloc(const gkv_arena_desc* arena, int32_t layer,
                                        const int32_t* h_block_tables, int32_t batch,
                                        int32_t max_blocks, const int32_t* h_ctx_lens,
                                        const float* d_q, float* d_out, int32_t n_heads,
                                        float scale, const float* d_sinks, void* stream) {
    using namespace gkv;
    if (!arena || !arena->d_k || !arena->d_v) return set_error(GKV_EINVAL, "arena / arena pointers are NULL");
    const gkv_arena_desc& A = *arena;
    const int32_t bs = A.block_size > 0 ? A.block_size : 16;
    const int32_t dv = A.v_head_dim > 0 ? A.v_head_dim : A.head_dim;
    if (A.total_blocks < 1 || A.layers < 1 || A.heads_kv < 1 || A.head_dim < 1 ||
        !valid_kv_dtype(A.dtype))
        return set_error(GKV_EINVAL, "invalid arena description");
    if (A.dtype == GKV_DTYPE_FP8_E4M3)  // the description carries no per-head scales
        return set_error(GKV_EINVAL, "an FP8 arena needs its pool's scales: use gkv_paged_decode");
    if (layer < 0 || layer >= A.layers) return set_error(GKV_EINVAL, "layer %d outside [0, %d)", layer, A.layers);
    if (n_heads <= 0 || n_heads % A.heads_kv != 0)
        return set_error(GKV_EINVAL, "n_heads %d is not a positive multiple of heads_kv %d", n_heads, A.heads_kv);
    if (batch < 0 || max_blocks < 0 || (batch > 0 && (!h_ctx_lens || !d_q || !d_out || (max_blocks > 0 && !h_block_tables))))
        return set_error(GKV_EINVAL, "bad batch / NULL tables, ctx_lens, q or out");
    // host validation of everything a kernel will dereference
    int64_t total = 0;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t c = h_ctx_lens[b];
        if (c < 0 || static_cast<int64_t>(c) > static_cast<int64_t>(max_blocks) * bs)
            return set_error(GKV_EINVAL, "sequence %d: ctx_len %d outside [0, %lld]", b, c,
                             static_cast<long long>(max_blocks) * bs);
        for (int32_t pg = 0; pg < (c + bs - 1) / bs; ++pg) {
            const int32_t id = h_block_tables[static_cast<int64_t>(b) * max_blocks + pg];
            if (id < 0 || id >= A.total_blocks)
                return set_error(GKV_EINVAL, "sequence %d: block table entry %d = %d outside [0, %d)", b, pg, id,
                                 A.total_blocks);
        }
        total += chunks_of(c, bs);
    }
    total *= A.heads_kv;

    ArenaGeom g{};
    g.k = A.d_k;
    g.v = A.d_v;
    g.k_head_stride = static_cast<int64_t>(bs) * A.head_dim;
    g.k_layer_stride = static_cast<int64_t>(A.heads_kv) * g.k_head_stride;
    g.k_block_stride = static_cast<int64_t>(A.layers) * g.k_layer_stride;
    g.v_head_stride = static_cast<int64_t>(bs) * dv;
    g.v_layer_stride = static_cast<int64_t>(A.heads_kv) * g.v_head_stride;
    g.v_block_stride = static_cast<int64_t>(A.layers) * g.v_layer_stride;
    g.total_blocks = A.total_blocks;
    g.layers = A.layers;
    g.heads_kv = A.heads_kv;
    g.head_dim = A.head_dim;
    g.v_head_dim = dv;
    g.block_size = bs;
    g.dtype = A.dtype;

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return set_error(GKV_EINVAL, "device %d beyond %d", dev, kMaxDevices);
    const DecodeConfig cfg = decode_config(g, n_heads);
    if (!cfg.supported)
        return set_error(GKV_EUNSUPPORTED, "decode not built for head_dim %d / v_head_dim %d", A.head_dim, dv);

    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_dev[dev]) {
        // once per device, with that device current
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_decode_scratch)");
        g_scratch_dev[dev] = p;
    }
    char* dbase = static_cast<char*>(g_scratch_dev[dev]);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    {
        // the host-to-device copy of this call's tables is not something a graph can replay
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
            return set_error(GKV_ESTATE, "gkv_paged_decode_noalloc must not be captured (its table upload would not be "
                                         "replayed); capture pool decodes in the static step layout instead");
        cudaGetLastError();
    }
    if (batch == 0 || total == 0) return GKV_OK;

    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    // the same grid and work list as the pool's decode (gkv_upload_step + gkv_paged_decode)
    const int64_t ctas = decode_grid_ctas(total, cfg.warps, static_cast<int64_t>(sms) * cfg.ctas_per_sm);
    const int32_t n_workers = static_cast<int32_t>(ctas * cfg.warps);
    const int64_t n_seg = static_cast<int64_t>(batch) * A.heads_kv;
    const int64_t max_pieces = n_workers + n_seg;
    const Layout L = layout_for(batch, max_blocks, max_pieces, n_workers, n_seg, cfg.head_groups);
    if (L.total > kMetaBytes)
        return set_error(GKV_EINVAL, "step metadata needs %zu bytes, more than the %zu-byte static scratch allows",
                         L.total, kMetaBytes);
    unsigned char* h = g_stage;
    if (batch && max_blocks) memcpy(h + L.tables, h_block_tables, static_cast<size_t>(batch) * max_blocks * 4);
    memcpy(h + L.ctx, h_ctx_lens, static_cast<size_t>(batch) * 4);
    auto at = [&](size_t off) { return reinterpret_cast<int32_t*>(h + off); };
    PlanArrays P{at(L.pseg), at(L.pc0), at(L.pc1), at(L.pslot), at(L.pmerge), at(L.wbeg),
                 at(L.mseg), at(L.ms0), at(L.mns), at(L.mdef), 0, 0, 0, 0, 0, 0};
    plan_work_into(h_ctx_lens, batch, A.heads_kv, bs, n_workers, &P);
    const int32_t nslots = P.n_slots, nmerge = P.n_merge, ndef = P.n_deferred;
    // the fused merge's arrival counters must start at zero on every call
    memset(h + L.counters, 0, static_cast<size_t>(n_seg) * cfg.head_groups * 4);
    // partials: (max, sum) pairs, then the accumulators at a 256-byte boundary (the
    // tensor-core decode reads them with 16-byte vectors)
    const size_t ml_bytes = static_cast<size_t>(nslots) * cfg.head_groups * cfg.gp * 2 * sizeof(float);
    const size_t acc_off = (ml_bytes + 255) & ~static_cast<size_t>(255);
    const size_t part_bytes =
        acc_off + static_cast<size_t>(nslots) * cfg.head_groups * cfg.gp * static_cast<size_t>(dv) * sizeof(float);
    if (part_bytes > kPartBytes)
        return set_error(GKV_EINVAL, "decode partials need %zu bytes, more than the %zu-byte static scratch allows",
                         part_bytes, kPartBytes);

    e = cudaMemcpyAsync(dbase, h, L.total, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(static scratch)");
    // the error word starts at zero (static storage) and is read and cleared by
    // gkv_paged_decode_noalloc_status; kernels only OR bits into it
    int* d_err = reinterpret_cast<int*>(dbase + kErrOffset);

    DecodeWork w{};
    auto dp = [&](size_t off) { return reinterpret_cast<const int32_t*>(dbase + off); };
    w.tables = dp(L.tables);
    w.ctx_lens = dp(L.ctx);
    w.max_blocks = max_blocks;
    w.piece_seg = dp(L.pseg);
    w.piece_c0 = dp(L.pc0);
    w.piece_c1 = dp(L.pc1);
    w.piece_slot = dp(L.pslot);
    w.worker_piece_begin = dp(L.wbeg);
    w.n_ctas = static_cast<int32_t>(ctas);
    w.n_slots = nslots;
    w.merge_seg = dp(L.mseg);
    w.merge_slot0 = dp(L.ms0);
    w.merge_nslots = dp(L.mns);
    w.piece_merge = dp(L.pmerge);
    w.n_merge = nmerge;
    w.merge_count = reinterpret_cast<int32_t*>(dbase + L.counters);
    w.merge_deferred = dp(L.mdef);
    w.n_deferred = ndef;
    w.n_deferred_long = P.n_deferred_long;

    DecodeArgs a{};
    a.layer = layer;
    a.q = d_q;
    a.out = d_out;
    a.n_heads = n_heads;
    a.scale = scale;
    a.sinks = d_sinks;
    a.part_ml = reinterpret_cast<float*>(dbase + kMetaBytes);
    a.part_acc = reinterpret_cast<float*>(dbase + kMetaBytes + acc_off);
    a.err = d_err;
    int launches = 0;
    e = launch_paged_decode(g, w, a, &launches, st);
    if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
    return GKV_OK;
}

extern "C" int gkv_paged_decode_noalloc_status(void* stream, int32_t timeout_ms) {
    using namespace gkv;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return set_error(GKV_EINVAL, "device %d beyond %d", dev, kMaxDevices);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // bounded wait for the caller's stream (no call here may hang)
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        e = cudaStreamQuery(st);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (timeout_ms >= 0 && ms >= timeout_ms)
            return set_error(GKV_ETIMEDOUT, "stream still busy after %d ms", timeout_ms);
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    char* dbase = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        dbase = static_cast<char*>(g_scratch_dev[dev]);
    }
    if (!dbase) return GKV_OK;  // no allocation-free decode ran on this device yet
    int* d_err = reinterpret_cast<int*>(dbase + kErrOffset);
    int flag = 0;
    e = cudaMemcpy(&flag, d_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(error word)");
    if (flag == 0) return GKV_OK;
    const int zero = 0;
    e = cudaMemcpy(d_err, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(error word)");
    return set_error(GKV_EDEVICE,
                     "an allocation-free decode reported error bits 0x%x (1 = bad block id, 2 = wait timeout)", flag);
}
