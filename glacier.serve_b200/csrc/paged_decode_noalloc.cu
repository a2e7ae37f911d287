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
//    cudaGetSymbolAddress (with that device current) and caches it; make that first call
//    before any stream capture.
#include <mutex>

#include "gkv_device.cuh"
#include "gkv_internal.h"

namespace gkv {

namespace {

constexpr size_t kScratchBytes = 16u << 20;   // per device
constexpr size_t kMetaBytes = 4u << 20;       // tables, context lengths, work list
constexpr size_t kErrOffset = kScratchBytes - 256;
constexpr size_t kPartBytes = kErrOffset - kMetaBytes;
constexpr int kMaxDevices = 64;
constexpr int kMinChunks = 16;

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

// The work list of step.cpp's build_work_list, written into fixed arrays (no heap).
void plan_fixed(const int32_t* ctx, int32_t batch, int32_t heads_kv, int32_t bs, int32_t n_workers,
                int64_t total, int32_t* pseg, int32_t* pc0, int32_t* pc1, int32_t* pslot,
                int32_t* pmerge, int32_t* wbeg, int32_t* mseg, int32_t* ms0, int32_t* mns, int32_t* mdef,
                int32_t* n_pieces, int32_t* n_slots, int32_t* n_merge, int32_t* n_deferred) {
    // the charged stream: every non-empty segment spans kSegmentCost units, then its chunks
    const int64_t n_seg = static_cast<int64_t>(batch) * heads_kv;
    auto span = [&](int64_t seg) {
        const int64_t c = chunks_of(ctx[seg / heads_kv], bs);
        return c > 0 ? c + kSegmentCost : 0;
    };
    int64_t vtotal = 0;
    for (int64_t seg = 0; seg < n_seg; ++seg) vtotal += span(seg);
    (void)total;
    int64_t s = 0, s0 = 0, s1 = n_seg > 0 ? span(0) : 0;
    int32_t np = 0;
    for (int32_t w = 0; w < n_workers; ++w) {
        wbeg[w] = np;
        int64_t lo = vtotal * w / n_workers;
        const int64_t hi = vtotal * (w + 1) / n_workers;
        while (lo < hi) {
            while (s1 <= lo) {
                ++s;
                s0 = s1;
                s1 = s0 + span(s);
            }
            const int64_t end = hi < s1 ? hi : s1;
            const int64_t c0 = lo - s0 - kSegmentCost, c1 = end - s0 - kSegmentCost;
            if (c1 > 0) {  // a range inside the overhead units holds no chunk
                pseg[np] = static_cast<int32_t>(s);
                pc0[np] = static_cast<int32_t>(c0 > 0 ? c0 : 0);
                pc1[np] = static_cast<int32_t>(c1);
                ++np;
            }
            lo = end;
        }
    }
    wbeg[n_workers] = np;
    int32_t slots = 0, merges = 0, deferred = 0, i = 0;
    while (i < np) {
        int32_t j = i + 1;
        while (j < np && pseg[j] == pseg[i]) ++j;
        if (j - i > 1) {
            const bool defer = (j - i) > kFusedMergeMaxSlots;
            mseg[merges] = pseg[i];
            ms0[merges] = slots;
            mns[merges] = j - i;
            if (defer) mdef[deferred++] = merges;
            for (int32_t k = i; k < j; ++k) {
                pslot[k] = slots++;
                pmerge[k] = defer ? -2 : merges;
            }
            ++merges;
        } else {
            pslot[i] = -1;
            pmerge[i] = -1;
        }
        i = j;
    }
    *n_pieces = np;
    *n_slots = slots;
    *n_merge = merges;
    *n_deferred = deferred;
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
        (A.dtype != GKV_DTYPE_F32 && A.dtype != GKV_DTYPE_BF16))
        return set_error(GKV_EINVAL, "invalid arena description");
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
    if (batch == 0 || total == 0) return GKV_OK;

    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    const int64_t max_ctas = static_cast<int64_t>(sms) * cfg.ctas_per_sm;
    int64_t ctas = ((total + kMinChunks - 1) / kMinChunks + cfg.warps - 1) / cfg.warps;
    if (ctas > max_ctas) ctas = max_ctas;
    if (ctas < 1) ctas = 1;
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
    int32_t np = 0, nslots = 0, nmerge = 0, ndef = 0;
    auto at = [&](size_t off) { return reinterpret_cast<int32_t*>(h + off); };
    plan_fixed(h_ctx_lens, batch, A.heads_kv, bs, n_workers, total, at(L.pseg), at(L.pc0), at(L.pc1),
               at(L.pslot), at(L.pmerge), at(L.wbeg), at(L.mseg), at(L.ms0), at(L.mns), at(L.mdef), &np,
               &nslots, &nmerge, &ndef);
    // the fused merge's arrival counters must start at zero on every call
    memset(h + L.counters, 0, static_cast<size_t>(n_seg) * cfg.head_groups * 4);
    const size_t part_floats =
        static_cast<size_t>(nslots) * cfg.head_groups * cfg.gp * (static_cast<size_t>(dv) + 2);
    if (part_floats * sizeof(float) > kPartBytes)
        return set_error(GKV_EINVAL, "decode partials need %zu bytes, more than the %zu-byte static scratch allows",
                         part_floats * sizeof(float), kPartBytes);

    e = cudaMemcpyAsync(dbase, h, L.total, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(static scratch)");
    int* d_err = reinterpret_cast<int*>(dbase + kErrOffset);
    e = cudaMemsetAsync(d_err, 0, sizeof(int), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(error word)");

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
    int64_t def_slots = 0;  // mean slots of the deferred entries (selects the merge form)
    for (int32_t k = 0; k < ndef; ++k) def_slots += at(L.mns)[at(L.mdef)[k]];
    w.deferred_avg_slots = ndef > 0 ? static_cast<int32_t>((def_slots + ndef - 1) / ndef) : 0;

    DecodeArgs a{};
    a.layer = layer;
    a.q = d_q;
    a.out = d_out;
    a.n_heads = n_heads;
    a.scale = scale;
    a.sinks = d_sinks;
    float* part = reinterpret_cast<float*>(dbase + kMetaBytes);
    a.part_ml = part;
    a.part_acc = part + static_cast<size_t>(nslots) * cfg.head_groups * cfg.gp * 2;
    a.err = d_err;
    int launches = 0;
    e = launch_paged_decode(g, w, a, &launches, st);
    if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
    return GKV_OK;
}
