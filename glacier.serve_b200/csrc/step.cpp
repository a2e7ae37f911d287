// One decode/append step: packed metadata upload, split-KV work list, kernel dispatch.
//
// Replaces the per-sequence UploadBlockTable + ForwardPagedToken loop of
// CudaPagedTransformerRunner.ForwardBatch (src/Glacier.Serve/Inference/PagedAttention/
// CudaPagedTransformerRunner.cs:307-379) and the serial per-sequence Store +
// ComputeAttention loop of PagedTransformerRunner.ForwardBatch (PagedTransformerRunner.cs:
// 605-656): every table, context length and slot of the step travels in ONE host-to-device
// copy, then one append launch and one decode launch (+ one merge launch) serve the batch.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>

#include "gkv_internal.h"

namespace gkv {

namespace {

// Fewest chunks a warp worker is given: small batches spread over more warps (the grid is
// capped at one wave, so large batches are unaffected).  Measured on cfg1 (20 sequences):
// 16 -> 52 us, 4 -> 43 us; cfg2 / cfg3 unchanged.
constexpr int kMinChunksPerWorker = 4;


size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int stage_copy(StageBuf& sb, const void* host, size_t bytes, cudaStream_t st, const char* what);
void stage_free(StageBuf& sb);

int sm_count(int device) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 148;
    }
    return n;
}

// Byte layout of the packed step metadata (identical on host and device).
struct MetaLayout {
    size_t hdr, slots, tables, ctx, pseg, pc0, pc1, pslot, pmerge, wbeg, mseg, ms0, mns, mdef, total;
};

MetaLayout meta_layout(int64_t n_tok, int64_t batch, int64_t max_blocks, int64_t n_pieces,
                       int64_t n_workers, int64_t n_merge) {
    MetaLayout L{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes, 16);
        return at;
    };
    L.hdr = take(kHdrBytes);  // counts + offsets (kHdr*), then the slots at kHdrBytes
    L.slots = take(static_cast<size_t>(n_tok) * 8);
    L.tables = take(static_cast<size_t>(batch * max_blocks) * 4);
    L.ctx = take(static_cast<size_t>(batch) * 4);
    L.pseg = take(static_cast<size_t>(n_pieces) * 4);
    L.pc0 = take(static_cast<size_t>(n_pieces) * 4);
    L.pc1 = take(static_cast<size_t>(n_pieces) * 4);
    L.pslot = take(static_cast<size_t>(n_pieces) * 4);
    L.pmerge = take(static_cast<size_t>(n_pieces) * 4);
    L.wbeg = take(static_cast<size_t>(n_workers + 1) * 4);
    L.mseg = take(static_cast<size_t>(n_merge) * 4);
    L.ms0 = take(static_cast<size_t>(n_merge) * 4);
    L.mns = take(static_cast<size_t>(n_merge) * 4);
    L.mdef = take(static_cast<size_t>(n_merge) * 4);
    L.total = o;
    return L;
}

int grow_device(void** p, size_t* cap, size_t need, const char* what) {
    if (need <= *cap) return GKV_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    const size_t sz = align_up(need + need / 4, 256);
    cudaError_t e = cudaMalloc(p, sz);
    if (e != cudaSuccess) return cuda_fail(e, what);
    *cap = sz;
    return GKV_OK;
}

}  // namespace

int32_t chunks_of(int32_t ctx, int32_t block_size) {
    if (ctx <= 0) return 0;
    const int32_t cpp = (block_size + kDecodeChunk - 1) / kDecodeChunk;
    const int32_t full = ctx / block_size;
    const int32_t rem = ctx - full * block_size;
    return full * cpp + (rem + kDecodeChunk - 1) / kDecodeChunk;
}

void plan_work_into(const int32_t* ctx_lens, int32_t batch, int32_t heads_kv, int32_t block_size,
                    int32_t n_workers, PlanArrays* out) {
    PlanArrays& A = *out;
    // The charged stream: every non-empty (sequence, kv head) segment spans kSegmentCost units
    // of per-piece overhead, then its chunks.  All heads of a sequence have the same span, so
    // the walk below keeps a (sequence, head) cursor and needs no per-segment table.
    int64_t total = 0, real_total = 0;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t c = chunks_of(ctx_lens[b], block_size);
        total += (c > 0 ? c + kSegmentCost : 0) * static_cast<int64_t>(heads_kv);
        real_total += static_cast<int64_t>(c) * heads_kv;
    }
    A.total_chunks = real_total;
    // Worker w covers [total*w/n, total*(w+1)/n), stepped without divisions; every worker
    // range is cut at segment ends, so there are at most n_workers + n_seg pieces.
    const int64_t q = n_workers > 0 ? total / n_workers : 0;  // no workers: an empty step
    const int64_t r = n_workers > 0 ? total % n_workers : 0;
    int64_t hi = 0, frac = 0;
    // cursor: segment (b, h) = b * heads_kv + h spans [s0, s1) of the charged stream
    int32_t cb = 0, ch = 0;
    int64_t span = batch > 0 ? (chunks_of(ctx_lens[0], block_size) > 0
                                    ? chunks_of(ctx_lens[0], block_size) + kSegmentCost : 0) : 0;
    int64_t s0 = 0, s1 = span;
    int32_t np = 0;
    for (int32_t w = 0; w < n_workers; ++w) {
        A.worker_begin[w] = np;
        int64_t lo = hi;
        hi += q;
        frac += r;
        if (frac >= n_workers) {
            frac -= n_workers;
            ++hi;
        }
        while (lo < hi) {
            while (s1 <= lo) {  // advance to the segment holding unit `lo`
                if (++ch == heads_kv) {
                    ch = 0;
                    ++cb;
                    const int32_t c = chunks_of(ctx_lens[cb], block_size);
                    span = c > 0 ? c + kSegmentCost : 0;
                }
                s0 = s1;
                s1 = s0 + span;
            }
            const int64_t end = hi < s1 ? hi : s1;
            const int64_t c0 = lo - s0 - kSegmentCost, c1 = end - s0 - kSegmentCost;
            if (c1 > 0) {  // a range inside the overhead units holds no chunk
                A.piece_seg[np] = cb * heads_kv + ch;
                A.piece_c0[np] = static_cast<int32_t>(c0 > 0 ? c0 : 0);
                A.piece_c1[np] = static_cast<int32_t>(c1);
                ++np;
            }
            lo = end;
        }
    }
    A.worker_begin[n_workers > 0 ? n_workers : 0] = np;
    A.n_pieces = np;
    // Pieces of one segment are adjacent; a segment cut into several pieces gets contiguous
    // partial slots and one merge entry.  A segment of more than kFusedMergeMaxSlots pieces is
    // merged by the second launch; once that launch is needed, it takes every split segment,
    // so that no warp of the decode merges at its tail (on a 20-sequence GQA-7 batch those
    // fused merges made the slowest warps 10 us late).
    bool defer_all = false;
    for (int32_t i = 0; i < np && !defer_all;) {
        int32_t j = i + 1;
        while (j < np && A.piece_seg[j] == A.piece_seg[i]) ++j;
        defer_all = (j - i) > kFusedMergeMaxSlots;
        i = j;
    }
    int32_t slots = 0, merges = 0, deferred = 0;
    for (int32_t i = 0; i < np;) {
        int32_t j = i + 1;
        while (j < np && A.piece_seg[j] == A.piece_seg[i]) ++j;
        if (j - i > 1) {
            A.merge_seg[merges] = A.piece_seg[i];
            A.merge_slot0[merges] = slots;
            A.merge_nslots[merges] = j - i;
            if (defer_all) A.merge_deferred[deferred++] = merges;
            for (int32_t k = i; k < j; ++k) {
                A.piece_slot[k] = slots++;
                A.piece_merge[k] = defer_all ? -2 : merges;
            }
            ++merges;
        } else {
            A.piece_slot[i] = -1;
            A.piece_merge[i] = -1;
        }
        i = j;
    }
    // the merge kernel gives a segment of more than kWarpMergeMaxSlots slots a CTA of its own and
    // the others a warp each: the long ones go first in the deferred list
    std::stable_partition(A.merge_deferred, A.merge_deferred + deferred,
                          [&](int32_t m) { return A.merge_nslots[m] > kWarpMergeMaxSlots; });
    int32_t n_long = 0;
    while (n_long < deferred && A.merge_nslots[A.merge_deferred[n_long]] > kWarpMergeMaxSlots) ++n_long;
    A.n_slots = slots;
    A.n_merge = merges;
    A.n_deferred = deferred;
    A.n_deferred_long = n_long;
}

void build_work_list(const int32_t* ctx_lens, int32_t batch, int32_t heads_kv, int32_t block_size,
                     int32_t n_workers, WorkList* out) {
    WorkList& W = *out;
    const size_t n_seg = static_cast<size_t>(batch) * static_cast<size_t>(heads_kv > 0 ? heads_kv : 0);
    const size_t cap = static_cast<size_t>(n_workers > 0 ? n_workers : 0) + n_seg;
    // resized, not reassigned: a work list kept across steps keeps its capacity
    for (auto* v : {&W.piece_seg, &W.piece_c0, &W.piece_c1, &W.piece_slot, &W.piece_merge}) v->resize(cap);
    for (auto* v : {&W.merge_seg, &W.merge_slot0, &W.merge_nslots, &W.merge_deferred}) v->resize(n_seg);
    W.worker_begin.resize(static_cast<size_t>(n_workers > 0 ? n_workers : 0) + 1);
    PlanArrays A{W.piece_seg.data(), W.piece_c0.data(), W.piece_c1.data(), W.piece_slot.data(),
                 W.piece_merge.data(), W.worker_begin.data(), W.merge_seg.data(), W.merge_slot0.data(),
                 W.merge_nslots.data(), W.merge_deferred.data(), 0, 0, 0, 0, 0, 0};
    plan_work_into(ctx_lens, batch, heads_kv, block_size, n_workers, &A);
    for (auto* v : {&W.piece_seg, &W.piece_c0, &W.piece_c1, &W.piece_slot, &W.piece_merge})
        v->resize(static_cast<size_t>(A.n_pieces));
    for (auto* v : {&W.merge_seg, &W.merge_slot0, &W.merge_nslots}) v->resize(static_cast<size_t>(A.n_merge));
    W.merge_deferred.resize(static_cast<size_t>(A.n_deferred));
    W.n_slots = A.n_slots;
    W.n_deferred_long = A.n_deferred_long;
    W.total_chunks = A.total_chunks;
}


int64_t decode_grid_ctas(int64_t total_chunks, int warps, int64_t max_ctas) {
    if (total_chunks <= 0) return 0;
    const int64_t want_workers = (total_chunks + kMinChunksPerWorker - 1) / kMinChunksPerWorker;
    int64_t ctas = (want_workers + warps - 1) / warps;
    if (ctas > max_ctas) ctas = max_ctas;
    return ctas < 1 ? 1 : ctas;
}


// Sizes the pinned + device metadata buffers for `bytes`.  Only called while no step of
// this pool is in use by a kernel that has not been ordered before the next upload
// (cudaFree synchronises the device).
static int ensure_meta(Pool* p, size_t bytes) {
    StepWorkspace& ws = p->ws;
    for (int i = 0; i < 2; ++i) {
        for (cudaEvent_t* ev : {&ws.meta_copied[i], &ws.meta_mark[i]})
            if (!*ev) {
                cudaError_t e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
                if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
            }
    }
    if (!ws.meta_stream) {
        cudaError_t e = cudaStreamCreateWithFlags(&ws.meta_stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate(step metadata)");
    }
    if (bytes <= ws.meta_cap) return GKV_OK;
    for (int i = 0; i < 2; ++i) {
        if (ws.meta_pending[i]) cudaEventSynchronize(ws.meta_copied[i]);
        ws.meta_pending[i] = false;
        ws.meta_marked[i] = false;
        if (ws.h_meta[i]) cudaFreeHost(ws.h_meta[i]);
        ws.h_meta[i] = nullptr;
        if (ws.d_meta[i]) cudaFree(ws.d_meta[i]);
        ws.d_meta[i] = nullptr;
    }
    ws.meta_cap = 0;
    ws.uploaded = false;  // the previous step's metadata is gone
    const size_t cap = align_up(bytes, 4096);
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaMallocHost(&ws.h_meta[i], cap);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocHost(step metadata)");
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaMalloc(&ws.d_meta[i], cap);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(step metadata)");
    ws.meta_cap = cap;
    return GKV_OK;
}

// Decode configuration for n_heads plus partial / counter buffers for `slots` partial slots
// and `merges` split segments.  Never touches the uploaded step metadata, so it is safe
// between gkv_upload_step and gkv_paged_decode.
static int decode_buffers(Pool* p, int32_t n_heads, int64_t slots, int64_t merges) {
    StepWorkspace& ws = p->ws;
    if (n_heads % p->desc.heads_kv != 0)
        return set_error(GKV_EINVAL, "n_heads %d is not a multiple of heads_kv %d", n_heads, p->desc.heads_kv);
    if (n_heads != ws.n_heads || !ws.cfg.supported) {
        ws.n_heads = n_heads;
        ws.cfg = decode_config(p->geom, n_heads);
        const int ctas_per_sm = ws.cfg.supported ? ws.cfg.ctas_per_sm : 1;
        ws.n_ctas_max = sm_count(p->desc.device) * ctas_per_sm;  // grid of the next upload
    }
    if (!ws.cfg.supported) return GKV_OK;
    const size_t need = static_cast<size_t>(slots > 0 ? slots : 1) * ws.cfg.head_groups * ws.cfg.gp;
    if (need > ws.part_slots_cap) {
        if (ws.d_part_acc) cudaFree(ws.d_part_acc);
        if (ws.d_part_ml) cudaFree(ws.d_part_ml);
        ws.d_part_acc = nullptr;
        ws.d_part_ml = nullptr;
        ws.part_slots_cap = 0;
        cudaError_t e = cudaMalloc(&ws.d_part_acc, need * p->desc.v_head_dim * sizeof(float));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(decode partials)");
        e = cudaMalloc(&ws.d_part_ml, need * 2 * sizeof(float));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(decode partials)");
        ws.part_slots_cap = need;
    }
    // one arrival counter per (head group, split segment), zeroed when allocated; kernels
    // leave them at zero
    const size_t counters = static_cast<size_t>(merges > 0 ? merges : 1) * ws.cfg.head_groups;
    if (counters > ws.merge_count_cap) {
        if (ws.d_merge_count) cudaFree(ws.d_merge_count);
        ws.d_merge_count = nullptr;
        ws.merge_count_cap = 0;
        cudaError_t e = cudaMalloc(&ws.d_merge_count, counters * sizeof(int32_t));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(merge counters)");
        e = cudaMemset(ws.d_merge_count, 0, counters * sizeof(int32_t));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(merge counters)");
        ws.merge_count_cap = counters;
    }
    return GKV_OK;
}

int step_reserve(Pool* p, int32_t max_batch, int32_t max_blocks, int32_t max_tokens,
                 int32_t n_heads) {
    StepWorkspace& ws = p->ws;
    if (max_batch < 0 || max_blocks < 0 || max_tokens < 0)
        return set_error(GKV_EINVAL, "negative reservation");
    if (n_heads <= 0) n_heads = ws.n_heads > 0 ? ws.n_heads : p->desc.heads_kv;
    if (max_batch > ws.max_batch) ws.max_batch = max_batch;
    if (max_blocks > ws.max_blocks) ws.max_blocks = max_blocks;
    if (max_tokens > ws.max_tokens) ws.max_tokens = max_tokens;
    // the worker count depends on the decode configuration: settle it first
    int rc = decode_buffers(p, n_heads, 0, 0);
    if (rc != GKV_OK) return rc;
    const int warps = ws.cfg.supported ? ws.cfg.warps : 4;
    const int64_t workers = static_cast<int64_t>(ws.n_ctas_max) * warps;
    const int64_t n_seg = static_cast<int64_t>(ws.max_batch) * p->desc.heads_kv;
    const MetaLayout L = meta_layout(ws.max_tokens, ws.max_batch, ws.max_blocks, workers + n_seg,
                                     workers, n_seg);
    rc = ensure_meta(p, L.total);
    if (rc != GKV_OK) return rc;
    // every piece of the largest work list could be a partial, every segment a merge
    return decode_buffers(p, n_heads, workers + n_seg, n_seg);
}

int step_set_static(Pool* p, bool enable) {
    StepWorkspace& ws = p->ws;
    if (!p->has_arena) return set_error(GKV_ESTATE, "pool has no device arena (metadata-only pool)");
    if (enable) {
        if (ws.meta_cap == 0 || ws.max_batch <= 0 || ws.n_heads <= 0)
            return set_error(GKV_ESTATE, "reserve the step first (gkv_step_reserve with the batch, blocks, tokens "
                                         "and query heads of the largest step)");
        if (!ws.cfg.supported)
            return set_error(GKV_EUNSUPPORTED, "decode not built for head_dim %d / v_head_dim %d", p->desc.head_dim,
                             p->desc.v_head_dim);
        if (static_cast<int64_t>(ws.max_tokens) * p->desc.heads_kv > (int64_t{1} << 30))
            return set_error(GKV_EINVAL, "max_tokens %d too large for one append launch", ws.max_tokens);
        // pinned staging buffers may still feed copies into d_meta[1]: settle them
        for (int i = 0; i < 2; ++i)
            if (ws.meta_pending[i]) {
                cudaError_t e = cudaEventSynchronize(ws.meta_copied[i]);
                if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize(step metadata)");
                ws.meta_pending[i] = false;
            }
        ws.static_merge_grid = sm_count(p->desc.device);  // the looping merge kernel: one CTA per SM
    }
    ws.static_mode = enable;
    ws.uploaded = false;  // the next upload writes the layout the launches will read
    return GKV_OK;
}

void step_free(Pool* p) {
    StepWorkspace& ws = p->ws;
    if (ws.meta_stream) cudaStreamSynchronize(ws.meta_stream);
    for (int i = 0; i < 2; ++i) {
        if (ws.meta_copied[i]) cudaEventDestroy(ws.meta_copied[i]);
        if (ws.meta_mark[i]) cudaEventDestroy(ws.meta_mark[i]);
        if (ws.h_meta[i]) cudaFreeHost(ws.h_meta[i]);
        if (ws.d_meta[i]) cudaFree(ws.d_meta[i]);
        ws.meta_copied[i] = ws.meta_mark[i] = nullptr;
        ws.h_meta[i] = nullptr;
        ws.d_meta[i] = nullptr;
        ws.meta_marked[i] = false;
    }
    if (ws.meta_stream) cudaStreamDestroy(ws.meta_stream);
    ws.meta_stream = nullptr;
    if (ws.d_part_acc) cudaFree(ws.d_part_acc);
    if (ws.d_part_ml) cudaFree(ws.d_part_ml);
    if (ws.d_merge_count) cudaFree(ws.d_merge_count);
    ws.d_merge_count = nullptr;
    if (ws.io_in) cudaStreamSynchronize(ws.io_in);
    if (ws.io_out) cudaStreamSynchronize(ws.io_out);
    for (auto& io : ws.io) {
        if (io.d_q) cudaFree(io.d_q);
        if (io.d_out) cudaFree(io.d_out);
        if (io.d_knew) cudaFree(io.d_knew);
        if (io.d_vnew) cudaFree(io.d_vnew);
        if (io.in_done) cudaEventDestroy(io.in_done);
        if (io.used) cudaEventDestroy(io.used);
        if (io.out_done) cudaEventDestroy(io.out_done);
        io = StepWorkspace::IoSlot{};
    }
    if (ws.io_in) cudaStreamDestroy(ws.io_in);
    if (ws.io_out) cudaStreamDestroy(ws.io_out);
    ws.io_in = ws.io_out = nullptr;
    stage_free(ws.pre);
    stage_free(ws.rope);
    if (ws.d_qconv) cudaFree(ws.d_qconv);
    ws.d_qconv = nullptr;
    ws.d_part_acc = ws.d_part_ml = nullptr;
}

int step_upload(Pool* p, const int32_t* tables, int32_t batch, int32_t max_blocks,
                const int32_t* ctx_lens, const int64_t* slots, int32_t n_tok, cudaStream_t st) {
    StepWorkspace& ws = p->ws;
    const int32_t bs = p->desc.block_size;
    if (batch < 0 || n_tok < 0 || max_blocks < 0)
        return set_error(GKV_EINVAL, "negative batch/n_tok/max_blocks");
    if (batch > 0 && (!ctx_lens || (max_blocks > 0 && !tables)))
        return set_error(GKV_EINVAL, "tables/ctx_lens is NULL");
    if (n_tok > 0 && !slots) return set_error(GKV_EINVAL, "slot_mapping is NULL");
    // Host validation of everything a kernel will dereference.
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t c = ctx_lens[b];
        if (c < 0 || static_cast<int64_t>(c) > static_cast<int64_t>(max_blocks) * bs)
            return set_error(GKV_EINVAL, "sequence %d: ctx_len %d outside [0, %lld]", b, c,
                             static_cast<long long>(max_blocks) * bs);
        const int32_t pages = (c + bs - 1) / bs;
        for (int32_t pg = 0; pg < pages; ++pg) {
            const int32_t id = tables[static_cast<int64_t>(b) * max_blocks + pg];
            if (!p->in_range(id))
                return set_error(GKV_EINVAL, "sequence %d: block table entry %d = %d outside [0, %d)",
                                 b, pg, id, p->desc.total_blocks);
        }
    }
    const int64_t n_slots_total = static_cast<int64_t>(p->desc.total_blocks) * bs;
    for (int32_t i = 0; i < n_tok; ++i)
        if (slots[i] < -1 || slots[i] >= n_slots_total)
            return set_error(GKV_EINVAL, "slot_mapping[%d] = %lld outside [-1, %lld)", i,
                             static_cast<long long>(slots[i]), static_cast<long long>(n_slots_total));

    if (ws.static_mode) {  // the captured launches were sized for the reservation
        if (batch > ws.max_batch || max_blocks > ws.max_blocks || n_tok > ws.max_tokens)
            return set_error(GKV_EINVAL, "batch %d / max_blocks %d / n_tok %d exceed the static step reservation "
                             "(%d / %d / %d)", batch, max_blocks, n_tok, ws.max_batch, ws.max_blocks, ws.max_tokens);
    } else if (batch > ws.max_batch || max_blocks > ws.max_blocks || n_tok > ws.max_tokens || ws.meta_cap == 0) {
        const int rc = step_reserve(p, batch, max_blocks, n_tok, ws.n_heads);
        if (rc != GKV_OK) return rc;
    }
    // Work list over a persistent grid: enough workers for the chunks, at most one wave (the
    // whole wave in the static layout, whose grid is fixed).
    int64_t total = 0;
    for (int32_t b = 0; b < batch; ++b) total += chunks_of(ctx_lens[b], bs);
    total *= p->desc.heads_kv;
    const int warps = ws.cfg.supported ? ws.cfg.warps : 4;
    const int64_t ctas = ws.static_mode ? ws.n_ctas_max : decode_grid_ctas(total, warps, ws.n_ctas_max);
    WorkList& W = ws.wl;
    build_work_list(ctx_lens, batch, p->desc.heads_kv, bs, static_cast<int32_t>(ctas * warps), &W);
    const int64_t n_pieces = static_cast<int64_t>(W.piece_seg.size());
    const int64_t n_workers = static_cast<int64_t>(ctas) * warps;
    const int64_t n_merge = static_cast<int64_t>(W.merge_seg.size());
    const MetaLayout L = meta_layout(n_tok, batch, max_blocks, n_pieces, n_workers, n_merge);
    if (ws.static_mode) {
        if (L.total > ws.meta_cap) return set_error(GKV_ESTATE, "static step buffer too small");
    } else {
        int mrc = ensure_meta(p, L.total);
        if (mrc != GKV_OK) return mrc;
    }

    // This staging buffer fed the copy two uploads ago, normally long finished.
    const int mi = ws.meta_flip;
    if (ws.meta_pending[mi]) {
        cudaError_t e = cudaEventSynchronize(ws.meta_copied[mi]);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize(step metadata)");
        ws.meta_pending[mi] = false;
    }
    char* h = ws.h_meta[mi];
    if (n_tok) memcpy(h + L.slots, slots, static_cast<size_t>(n_tok) * 8);
    if (batch && max_blocks) memcpy(h + L.tables, tables, static_cast<size_t>(batch) * max_blocks * 4);
    if (batch) memcpy(h + L.ctx, ctx_lens, static_cast<size_t>(batch) * 4);
    auto put = [&](size_t off, const std::vector<int32_t>& v) {
        if (!v.empty()) memcpy(h + off, v.data(), v.size() * 4);
    };
    put(L.pseg, W.piece_seg);
    put(L.pc0, W.piece_c0);
    put(L.pc1, W.piece_c1);
    put(L.pslot, W.piece_slot);
    put(L.pmerge, W.piece_merge);
    put(L.wbeg, W.worker_begin);
    put(L.mseg, W.merge_seg);
    put(L.ms0, W.merge_slot0);
    put(L.mns, W.merge_nslots);
    put(L.mdef, W.merge_deferred);
    {
        int32_t hd[kHdrInts];
        hd[kHdrTok] = n_tok;
        hd[kHdrBatch] = batch;
        hd[kHdrMaxBlocks] = max_blocks;
        hd[kHdrSlots] = W.n_slots;
        hd[kHdrMerge] = static_cast<int32_t>(n_merge);
        hd[kHdrDeferred] = static_cast<int32_t>(W.merge_deferred.size());
        hd[kHdrDeferredLong] = W.n_deferred_long;
        hd[kHdrWorkers] = static_cast<int32_t>(n_workers);
        const size_t offs[] = {L.tables, L.ctx, L.pseg, L.pc0, L.pc1, L.pslot, L.pmerge,
                               L.wbeg, L.mseg, L.ms0, L.mns, L.mdef};
        for (int k = 0; k < kHdrInts - kHdrTables; ++k) hd[kHdrTables + k] = static_cast<int32_t>(offs[k]);
        memcpy(h + L.hdr, hd, sizeof(hd));
    }
    cudaError_t e = cudaSuccess;
    if (ws.static_mode) {
        // one device buffer at a fixed address, rewritten in stream order: the previous step's
        // launches (queued before on `st`) have read it by the time the copy runs
        e = cudaMemcpyAsync(ws.d_meta[0], h, L.total, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(step metadata)");
        e = cudaEventRecord(ws.meta_copied[mi], st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord(step metadata)");
        ws.meta_pending[mi] = true;
        ws.meta_flip ^= 1;
    }
    // Device buffer mi last served the step uploaded two calls ago, whose kernels were queued
    // before the previous upload: the copy waits for the mark that upload recorded, then the
    // caller's stream waits for the copy.
    else {
        if (ws.meta_marked[mi ^ 1]) e = cudaStreamWaitEvent(ws.meta_stream, ws.meta_mark[mi ^ 1], 0);
        if (e == cudaSuccess) e = cudaEventRecord(ws.meta_mark[mi], st);
        if (e != cudaSuccess) return cuda_fail(e, "step metadata ordering");
        ws.meta_marked[mi] = true;
        e = cudaMemcpyAsync(ws.d_meta[mi], h, L.total, cudaMemcpyHostToDevice, ws.meta_stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(step metadata)");
        e = cudaEventRecord(ws.meta_copied[mi], ws.meta_stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, ws.meta_copied[mi], 0);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord(step metadata)");
        ws.meta_pending[mi] = true;
        ws.meta_flip ^= 1;
    }

    char* d = ws.static_mode ? ws.d_meta[0] : ws.d_meta[mi];
    DecodeWork& w = ws.work;
    w.tables = reinterpret_cast<const int32_t*>(d + L.tables);
    w.ctx_lens = reinterpret_cast<const int32_t*>(d + L.ctx);
    w.max_blocks = max_blocks;
    w.piece_seg = reinterpret_cast<const int32_t*>(d + L.pseg);
    w.piece_c0 = reinterpret_cast<const int32_t*>(d + L.pc0);
    w.piece_c1 = reinterpret_cast<const int32_t*>(d + L.pc1);
    w.piece_slot = reinterpret_cast<const int32_t*>(d + L.pslot);
    w.worker_piece_begin = reinterpret_cast<const int32_t*>(d + L.wbeg);
    w.n_ctas = (total > 0 || ws.static_mode) ? static_cast<int32_t>(ctas) : 0;
    w.n_slots = W.n_slots;
    w.merge_seg = reinterpret_cast<const int32_t*>(d + L.mseg);
    w.merge_slot0 = reinterpret_cast<const int32_t*>(d + L.ms0);
    w.merge_nslots = reinterpret_cast<const int32_t*>(d + L.mns);
    w.piece_merge = reinterpret_cast<const int32_t*>(d + L.pmerge);
    w.n_merge = static_cast<int32_t>(n_merge);
    w.merge_deferred = reinterpret_cast<const int32_t*>(d + L.mdef);
    w.n_deferred = static_cast<int32_t>(W.merge_deferred.size());
    w.n_deferred_long = W.n_deferred_long;
    w.merge_count = ws.d_merge_count;
    w.table_row = nullptr;
    w.dyn = ws.static_mode ? reinterpret_cast<const unsigned char*>(d) : nullptr;
    w.merge_grid = ws.static_mode ? ws.static_merge_grid : 0;
    ws.d_slots = reinterpret_cast<const int64_t*>(d + L.slots);
    ws.h_ctx.assign(ctx_lens, ctx_lens + batch);
    ws.batch = batch;
    ws.n_tok = n_tok;
    ws.up_max_blocks = max_blocks;
    ws.uploaded = true;
    return GKV_OK;
}

// In the static step layout a launch must not depend on host state that changes between steps:
// copy-on-write copies queued since the last flush would be captured into the graph.
static int static_guard(Pool* p) {
    if (p->ws.static_mode && p->stats_pending_copies() > 0)
        return set_error(GKV_ESTATE, "static step layout: flush the queued block copies (gkv_pool_flush_copies) "
                                     "before the captured launches");
    return GKV_OK;
}

int step_append(Pool* p, int32_t layer, const float* d_k, const float* d_v, int32_t n_tok,
                cudaStream_t st) {
    StepWorkspace& ws = p->ws;
    if (!ws.uploaded) return set_error(GKV_ESTATE, "no step uploaded (call gkv_upload_step first)");
    if (layer < 0 || layer >= p->desc.layers)
        return set_error(GKV_EINVAL, "layer %d outside [0, %d)", layer, p->desc.layers);
    if (!ws.static_mode && (n_tok < 0 || n_tok > ws.n_tok))  // static: the uploaded count is used
        return set_error(GKV_EINVAL, "n_tok %d exceeds the uploaded slot mapping (%d)", n_tok, ws.n_tok);
    if (n_tok > 0 && (!d_k || !d_v)) return set_error(GKV_EINVAL, "k/v source is NULL");
    int rc = static_guard(p);
    if (rc != GKV_OK) return rc;
    rc = p->flush_copies(st);
    if (rc != GKV_OK) return rc;
    // static layout: the kernel appends the uploaded step's token count, read on the device,
    // with a grid for the reserved maximum (d_k / d_v must hold that many rows)
    if (ws.static_mode) {
        if (ws.max_tokens == 0) return GKV_OK;
        if (!d_k || !d_v) return set_error(GKV_EINVAL, "k/v source is NULL");
    } else if (n_tok == 0) {
        return GKV_OK;
    }
    const int32_t* dyn_tok =
        ws.static_mode ? reinterpret_cast<const int32_t*>(ws.d_meta[0]) + kHdrTok : nullptr;
    cudaError_t e = launch_kv_append(p->geom, layer, d_k, d_v,
                                     static_cast<int64_t>(p->desc.heads_kv) * p->desc.head_dim,
                                     static_cast<int64_t>(p->desc.heads_kv) * p->desc.v_head_dim,
                                     ws.d_slots, 0, ws.static_mode ? ws.max_tokens : n_tok, ws.d_err, st, dyn_tok);
    if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
    p->last_launches += 1;
    return GKV_OK;
}

static int decode_common(Pool* p, int32_t layer, const float* d_q, float* d_out, int32_t n_heads,
                         float scale, const float* d_sinks, bool has_sink_all, float sink_all,
                         cudaStream_t st, float* d_lse = nullptr) {
    StepWorkspace& ws = p->ws;
    if (!ws.uploaded) return set_error(GKV_ESTATE, "no step uploaded (call gkv_upload_step first)");
    if (layer < 0 || layer >= p->desc.layers)
        return set_error(GKV_EINVAL, "layer %d outside [0, %d)", layer, p->desc.layers);
    if (n_heads <= 0 || n_heads % p->desc.heads_kv != 0)
        return set_error(GKV_EINVAL, "n_heads %d is not a positive multiple of heads_kv %d", n_heads,
                         p->desc.heads_kv);
    if (ws.batch > 0 && (!d_q || !d_out)) return set_error(GKV_EINVAL, "q/out is NULL");
    if (ws.static_mode) {  // the reservation fixed the configuration and every buffer
        if (n_heads != ws.n_heads)
            return set_error(GKV_EINVAL, "static step layout reserved for %d query heads, not %d", ws.n_heads,
                             n_heads);
        if (d_lse && ws.max_batch > 0 && !d_out) return set_error(GKV_EINVAL, "out is NULL");
        const int rc = static_guard(p);
        if (rc != GKV_OK) return rc;
    } else {
        // decode config + partial/counter capacity for the uploaded work list; the uploaded
        // metadata itself is left alone (the work list works with any kernel variant: every
        // variant runs the same number of warps per CTA)
        const int rc = decode_buffers(p, n_heads, ws.work.n_slots, ws.work.n_merge);
        if (rc != GKV_OK) return rc;
    }
    if (!ws.cfg.supported)
        return set_error(GKV_EUNSUPPORTED, "decode not built for head_dim %d / v_head_dim %d",
                         p->desc.head_dim, p->desc.v_head_dim);
    int rc = p->flush_copies(st);
    if (rc != GKV_OK) return rc;
    const size_t need = static_cast<size_t>(ws.work.n_slots) * ws.cfg.head_groups * ws.cfg.gp;
    if (need > ws.part_slots_cap) return set_error(GKV_ESTATE, "decode partial buffer too small");
    if (static_cast<size_t>(ws.work.n_merge) * ws.cfg.head_groups > ws.merge_count_cap)
        return set_error(GKV_ESTATE, "decode merge counters too small");
    ws.work.merge_count = ws.d_merge_count;  // may have been reallocated by a re-reserve
    DecodeArgs a{};
    a.layer = layer;
    a.q = d_q;
    a.out = d_out;
    a.n_heads = n_heads;
    a.scale = scale;
    a.sinks = d_sinks;
    a.has_sink_all = has_sink_all ? 1 : 0;
    a.sink_all = sink_all;
    a.part_acc = ws.d_part_acc;
    a.part_ml = ws.d_part_ml;
    a.err = ws.d_err;
    a.lse = d_lse;
    int launches = 0;
    cudaError_t e = launch_paged_decode(p->geom, ws.work, a, &launches, st);
    if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
    p->last_launches += launches;
    return GKV_OK;
}

int step_decode(Pool* p, int32_t layer, const float* d_q, float* d_out, int32_t n_heads,
                float scale, const float* d_sinks, cudaStream_t st) {
    return decode_common(p, layer, d_q, d_out, n_heads, scale, d_sinks, false, 0.f, st);
}

int step_decode_lse(Pool* p, int32_t layer, const float* d_q, float* d_out, float* d_lse,
                    int32_t n_heads, float scale, const float* d_sinks, cudaStream_t st) {
    return decode_common(p, layer, d_q, d_out, n_heads, scale, d_sinks, false, 0.f, st, d_lse);
}

// ---- chunked causal prefill ------------------------------------------------------------

namespace {

constexpr int kPrefillRows = 128;  // queries per tensor-core work item

// Copies `bytes` of host data into a staging buffer's device side (one pinned staging copy on
// `st`).  The pinned side is reused once its previous copy has landed.
int stage_copy(StageBuf& sb, const void* host, size_t bytes, cudaStream_t st, const char* what) {
    if (!sb.copied) {
        cudaError_t e = cudaEventCreateWithFlags(&sb.copied, cudaEventDisableTiming);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
    }
    if (sb.pending) {
        cudaError_t e = cudaEventSynchronize(sb.copied);
        if (e != cudaSuccess) return cuda_fail(e, what);
        sb.pending = false;
    }
    if (bytes > sb.cap) {
        if (sb.h) cudaFreeHost(sb.h);
        if (sb.d) cudaFree(sb.d);
        sb.h = sb.d = nullptr;
        sb.cap = 0;
        const size_t cap = align_up(bytes, 4096);
        cudaError_t e = cudaMallocHost(&sb.h, cap);
        if (e != cudaSuccess) return cuda_fail(e, what);
        e = cudaMalloc(&sb.d, cap);
        if (e != cudaSuccess) return cuda_fail(e, what);
        sb.cap = cap;
    }
    if (bytes == 0) return GKV_OK;
    memcpy(sb.h, host, bytes);
    cudaError_t e = cudaMemcpyAsync(sb.d, sb.h, bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, what);
    e = cudaEventRecord(sb.copied, st);
    if (e != cudaSuccess) return cuda_fail(e, what);
    sb.pending = true;
    return GKV_OK;
}

void stage_free(StageBuf& sb) {
    if (sb.pending && sb.copied) cudaEventSynchronize(sb.copied);
    if (sb.copied) cudaEventDestroy(sb.copied);
    if (sb.h) cudaFreeHost(sb.h);
    if (sb.d) cudaFree(sb.d);
    sb = StageBuf{};
}

int stage_prefill(Pool* p, const std::vector<char>& host, cudaStream_t st) {
    return stage_copy(p->ws.pre, host.data(), host.size(), st, "prefill metadata upload");
}

int ensure_qconv(Pool* p, size_t bytes) {
    StepWorkspace& ws = p->ws;
    if (bytes <= ws.qconv_cap) return GKV_OK;
    if (ws.d_qconv) cudaFree(ws.d_qconv);
    ws.d_qconv = nullptr;
    ws.qconv_cap = 0;
    cudaError_t e = cudaMalloc(&ws.d_qconv, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(prefill q conversion)");
    ws.qconv_cap = bytes;
    return GKV_OK;
}

template <class T>
void put_vec(std::vector<char>& buf, size_t off, const std::vector<T>& v) {
    if (!v.empty()) memcpy(buf.data() + off, v.data(), v.size() * sizeof(T));
}

}  // namespace

int step_prefill(Pool* p, int32_t layer, const void* d_q, int32_t q_dtype, float* d_out,
                 const int32_t* q_start, const int32_t* q_len, int32_t n_heads, float scale,
                 cudaStream_t st) {
    StepWorkspace& ws = p->ws;
    if (ws.static_mode)
        return set_error(GKV_ESTATE, "the chunked prefill is not available in the static step layout");
    if (!ws.uploaded) return set_error(GKV_ESTATE, "no step uploaded (call gkv_upload_step first)");
    if (layer < 0 || layer >= p->desc.layers)
        return set_error(GKV_EINVAL, "layer %d outside [0, %d)", layer, p->desc.layers);
    if (n_heads <= 0 || n_heads % p->desc.heads_kv != 0)
        return set_error(GKV_EINVAL, "n_heads %d is not a positive multiple of heads_kv %d", n_heads,
                         p->desc.heads_kv);
    if (!valid_q_dtype(q_dtype))
        return set_error(GKV_EINVAL, "q_dtype %d is not GKV_DTYPE_F32, GKV_DTYPE_BF16 or GKV_DTYPE_F16", q_dtype);
    const int32_t batch = ws.batch;
    if (batch > 0 && (!q_start || !q_len)) return set_error(GKV_EINVAL, "q_start/q_len is NULL");
    const int64_t max_seq = static_cast<int64_t>(ws.up_max_blocks) * p->desc.block_size;
    int64_t total_q = 0;
    for (int32_t b = 0; b < batch; ++b) {
        if (q_len[b] < 0 || q_start[b] < 0)
            return set_error(GKV_EINVAL, "sequence %d: negative q_start %d / q_len %d", b, q_start[b], q_len[b]);
        // ComputeAttention throws for pos >= maxSeqLen (PagedAttentionKernel.cs:34-39)
        if (q_len[b] > 0 && static_cast<int64_t>(q_start[b]) + q_len[b] > max_seq)
            return set_error(GKV_EINVAL, "sequence %d: positions up to %lld reach the table capacity %lld", b,
                             static_cast<long long>(q_start[b]) + q_len[b] - 1, static_cast<long long>(max_seq));
        total_q += q_len[b];
    }
    if (total_q > 0 && (!d_q || !d_out)) return set_error(GKV_EINVAL, "q/out is NULL");
    if (total_q * n_heads >= (int64_t{1} << 31))
        return set_error(GKV_EINVAL, "%lld query rows exceed the supported size", static_cast<long long>(total_q));
    int rc = p->flush_copies(st);
    if (rc != GKV_OK) return rc;
    if (total_q == 0) return GKV_OK;
    const int64_t q_elems = total_q * n_heads * p->desc.head_dim;

    // the tensor-core kernel takes the row max on unscaled scores: it needs scale > 0
    if (prefill_tc_eligible(p->geom, n_heads) && scale > 0.f) {
        // work items of up to 128 queries, heaviest first (longest key range)
        std::vector<int32_t> items;
        std::vector<std::pair<int32_t, int32_t>> order;  // (-n_keys, item)
        int64_t q_off = 0;
        for (int32_t b = 0; b < batch; ++b) {
            const int32_t tok = ws.h_ctx[static_cast<size_t>(b)];
            for (int32_t t0 = 0; t0 < q_len[b]; t0 += kPrefillRows) {
                const int32_t nq = std::min(kPrefillRows, q_len[b] - t0);
                const int64_t last = static_cast<int64_t>(q_start[b]) + t0 + nq - 1;
                const int32_t n_keys = static_cast<int32_t>(std::min<int64_t>(tok, last + 1));
                if (n_keys <= 0) continue;  // no keys: the reference leaves these rows alone
                const int32_t id = static_cast<int32_t>(order.size());
                order.emplace_back(-n_keys, id);
                const int32_t rec[kPrefillItemInts] = {b, q_start[b] + t0, static_cast<int32_t>(q_off + t0), nq,
                                                       n_keys, tok, 0, 0};
                items.insert(items.end(), rec, rec + kPrefillItemInts);
            }
            q_off += q_len[b];
        }
        std::stable_sort(order.begin(), order.end());
        std::vector<char> host(order.size() * kPrefillItemInts * 4);
        for (size_t i = 0; i < order.size(); ++i)
            memcpy(host.data() + i * kPrefillItemInts * 4,
                   items.data() + static_cast<size_t>(order[i].second) * kPrefillItemInts, kPrefillItemInts * 4);
        rc = stage_prefill(p, host, st);
        if (rc != GKV_OK) return rc;
        // the MMAs take q in the arena's 16-bit type
        const void* qb = d_q;
        int launches = 0;
        if (q_dtype != p->desc.dtype) {
            rc = ensure_qconv(p, static_cast<size_t>(q_elems) * 2);
            if (rc != GKV_OK) return rc;
            cudaError_t e = launch_convert(d_q, q_dtype, ws.d_qconv, p->desc.dtype, q_elems, st);
            if (e != cudaSuccess) return cuda_fail(e, "prefill q conversion");
            qb = ws.d_qconv;
            ++launches;
        } else if (reinterpret_cast<uintptr_t>(d_q) & 15) {
            return set_error(GKV_EINVAL, "16-bit q must be 16-byte aligned");
        }
        PrefillArgs a{};
        a.items = reinterpret_cast<const int32_t*>(ws.pre.d);
        a.n_items = static_cast<int32_t>(order.size());
        a.tables = ws.work.tables;
        a.max_blocks = ws.up_max_blocks;
        a.layer = layer;
        a.n_heads = n_heads;
        a.scale = scale;
        a.out = d_out;
        a.err = ws.d_err;
        if (a.n_items > 0) {
            cudaError_t e = launch_paged_prefill_tc(p->geom, a, qb, total_q, st);
            if (e != cudaSuccess) return cuda_fail(e, "paged_prefill launch");
            ++launches;
        }
        p->last_launches += launches;
        return GKV_OK;
    }

    // Any other pool: the split-KV decode kernel with one segment per query, all on the
    // sequence's table row, each with its causal length.
    std::vector<int32_t> ctx_e, row_e;
    ctx_e.reserve(static_cast<size_t>(total_q));
    row_e.reserve(static_cast<size_t>(total_q));
    for (int32_t b = 0; b < batch; ++b)
        for (int32_t t = 0; t < q_len[b]; ++t) {
            ctx_e.push_back(static_cast<int32_t>(
                std::min<int64_t>(ws.h_ctx[static_cast<size_t>(b)], static_cast<int64_t>(q_start[b]) + t + 1)));
            row_e.push_back(b);
        }
    const int32_t n_e = static_cast<int32_t>(total_q);
    rc = decode_buffers(p, n_heads, 0, 0);
    if (rc != GKV_OK) return rc;
    if (!ws.cfg.supported)
        return set_error(GKV_EUNSUPPORTED, "prefill not built for head_dim %d / v_head_dim %d", p->desc.head_dim,
                         p->desc.v_head_dim);
    const int32_t bs = p->desc.block_size;
    int64_t chunks = 0;
    for (int32_t c : ctx_e) chunks += chunks_of(c, bs);
    chunks *= p->desc.heads_kv;
    const int warps = ws.cfg.warps;
    int64_t ctas = decode_grid_ctas(chunks, warps, ws.n_ctas_max);
    if (ctas < 1) ctas = 1;
    WorkList W;
    build_work_list(ctx_e.data(), n_e, p->desc.heads_kv, bs, static_cast<int32_t>(ctas * warps), &W);
    const int64_t n_pieces = static_cast<int64_t>(W.piece_seg.size());
    const int64_t n_merge = static_cast<int64_t>(W.merge_seg.size());
    rc = decode_buffers(p, n_heads, W.n_slots, n_merge);
    if (rc != GKV_OK) return rc;
    const MetaLayout L = meta_layout(0, n_e, 0, n_pieces, ctas * warps, n_merge);
    const size_t rows_off = L.total;
    std::vector<char> host(rows_off + align_up(static_cast<size_t>(n_e) * 4, 16));
    put_vec(host, L.ctx, ctx_e);
    put_vec(host, L.pseg, W.piece_seg);
    put_vec(host, L.pc0, W.piece_c0);
    put_vec(host, L.pc1, W.piece_c1);
    put_vec(host, L.pslot, W.piece_slot);
    put_vec(host, L.pmerge, W.piece_merge);
    put_vec(host, L.wbeg, W.worker_begin);
    put_vec(host, L.mseg, W.merge_seg);
    put_vec(host, L.ms0, W.merge_slot0);
    put_vec(host, L.mns, W.merge_nslots);
    put_vec(host, L.mdef, W.merge_deferred);
    put_vec(host, rows_off, row_e);
    rc = stage_prefill(p, host, st);
    if (rc != GKV_OK) return rc;
    const char* d = ws.pre.d;
    auto at = [&](size_t off) { return reinterpret_cast<const int32_t*>(d + off); };
    DecodeWork w{};
    w.tables = ws.work.tables;
    w.ctx_lens = at(L.ctx);
    w.max_blocks = ws.up_max_blocks;
    w.piece_seg = at(L.pseg);
    w.piece_c0 = at(L.pc0);
    w.piece_c1 = at(L.pc1);
    w.piece_slot = at(L.pslot);
    w.worker_piece_begin = at(L.wbeg);
    w.n_ctas = chunks > 0 ? static_cast<int32_t>(ctas) : 0;
    w.n_slots = W.n_slots;
    w.merge_seg = at(L.mseg);
    w.merge_slot0 = at(L.ms0);
    w.merge_nslots = at(L.mns);
    w.piece_merge = at(L.pmerge);
    w.n_merge = static_cast<int32_t>(n_merge);
    w.merge_deferred = at(L.mdef);
    w.n_deferred = static_cast<int32_t>(W.merge_deferred.size());
    w.n_deferred_long = W.n_deferred_long;
    w.merge_count = ws.d_merge_count;
    w.table_row = at(rows_off);
    const float* qf = static_cast<const float*>(d_q);
    int launches = 0;
    if (q_dtype != GKV_DTYPE_F32) {
        rc = ensure_qconv(p, static_cast<size_t>(q_elems) * 4);
        if (rc != GKV_OK) return rc;
        cudaError_t e = launch_convert(d_q, q_dtype, ws.d_qconv, GKV_DTYPE_F32, q_elems, st);
        if (e != cudaSuccess) return cuda_fail(e, "prefill q conversion");
        qf = static_cast<const float*>(ws.d_qconv);
        ++launches;
    }
    DecodeArgs a{};
    a.layer = layer;
    a.q = qf;
    a.out = d_out;
    a.n_heads = n_heads;
    a.scale = scale;
    a.part_acc = ws.d_part_acc;
    a.part_ml = ws.d_part_ml;
    a.err = ws.d_err;
    int dl = 0;
    if (w.n_ctas > 0) {
        cudaError_t e = launch_paged_decode(p->geom, w, a, &dl, st);
        if (e != cudaSuccess) return cuda_fail(e, "prefill (decode kernel) launch");
    }
    p->last_launches += launches + dl;
    return GKV_OK;
}

void rope_inv_freq(float freq_base, int32_t rope_dim, const float* factors, float* out) {
    for (int32_t i = 0; i < rope_dim / 2; ++i) {
        float f = static_cast<float>(std::pow(static_cast<double>(freq_base), -2.0 * i / rope_dim));
        if (factors) f = f / factors[i];
        out[i] = f;
    }
}

int step_rope_append(Pool* p, int32_t layer, float* d_q, const float* d_k, const float* d_v, int32_t n_tok,
                     int32_t n_heads, const int32_t* positions, const gkv_rope_desc* rope,
                     const gkv_qkv_prologue* pro, cudaStream_t st) {
    StepWorkspace& ws = p->ws;
    if (!ws.uploaded) return set_error(GKV_ESTATE, "no step uploaded (call gkv_upload_step first)");
    if (!rope) return set_error(GKV_EINVAL, "rope description is NULL");
    if (layer < 0 || layer >= p->desc.layers)
        return set_error(GKV_EINVAL, "layer %d outside [0, %d)", layer, p->desc.layers);
    if (n_tok < 0 || n_tok > ws.n_tok)
        return set_error(GKV_EINVAL, "n_tok %d exceeds the uploaded slot mapping (%d)", n_tok, ws.n_tok);
    if (n_heads <= 0 || n_heads % p->desc.heads_kv != 0)
        return set_error(GKV_EINVAL, "n_heads %d is not a positive multiple of heads_kv %d", n_heads,
                         p->desc.heads_kv);
    const int32_t R = rope->rope_dim == 0 ? p->desc.head_dim : rope->rope_dim;
    if (rope->style != GKV_ROPE_NEOX && rope->style != GKV_ROPE_INTERLEAVED)
        return set_error(GKV_EINVAL, "rope style %d is neither GKV_ROPE_NEOX nor GKV_ROPE_INTERLEAVED", rope->style);
    if (R < 0 || R > p->desc.head_dim || (R & 1))
        return set_error(GKV_EINVAL, "rope_dim %d must be even and within [0, head_dim %d]", R, p->desc.head_dim);
    if (!rope_append_supported(p->geom, R))
        return set_error(GKV_EUNSUPPORTED, "fused rope append not built for head_dim %d / rope_dim %d",
                         p->desc.head_dim, R);
    if (!rope->h_inv_freq && !(rope->freq_base > 0.f))
        return set_error(GKV_EINVAL, "freq_base must be positive when no inverse-frequency table is given");
    if (n_tok > 0 && (!d_q || !d_k || !d_v || !positions)) return set_error(GKV_EINVAL, "q/k/v/positions is NULL");
    for (int32_t i = 0; i < n_tok; ++i)
        if (positions[i] < 0) return set_error(GKV_EINVAL, "positions[%d] = %d is negative", i, positions[i]);
    int rc = p->flush_copies(st);
    if (rc != GKV_OK) return rc;
    if (n_tok == 0) return GKV_OK;
    // one staged upload: positions, then the inverse-frequency table at a 16-byte boundary
    const size_t pos_bytes = align_up(static_cast<size_t>(n_tok) * 4, 16);
    std::vector<char> host(pos_bytes + static_cast<size_t>(R / 2 > 0 ? R / 2 : 1) * 4);
    memcpy(host.data(), positions, static_cast<size_t>(n_tok) * 4);
    float* tab = reinterpret_cast<float*>(host.data() + pos_bytes);
    if (rope->h_inv_freq) {
        for (int32_t i = 0; i < R / 2; ++i)
            tab[i] = rope->h_freq_factors ? rope->h_inv_freq[i] / rope->h_freq_factors[i] : rope->h_inv_freq[i];
    } else {
        rope_inv_freq(rope->freq_base, R, rope->h_freq_factors, tab);
    }
    rc = stage_copy(ws.rope, host.data(), host.size(), st, "rope metadata upload");
    if (rc != GKV_OK) return rc;
    RopeAppendParams a{};
    a.layer = layer;
    a.q = d_q;
    a.k = d_k;
    a.v = d_v;
    a.n_tok = n_tok;
    a.n_heads = n_heads;
    a.positions = reinterpret_cast<const int32_t*>(ws.rope.d);
    a.inv_freq = reinterpret_cast<const float*>(ws.rope.d + pos_bytes);
    a.rope_dim = R;
    a.style = rope->style;
    a.mscale = rope->mscale == 0.f ? 1.f : rope->mscale;
    if (pro) {
        a.q_bias = pro->d_q_bias;
        a.k_bias = pro->d_k_bias;
        a.v_bias = pro->d_v_bias;
        a.q_norm = pro->d_q_norm;
        a.k_norm = pro->d_k_norm;
        a.eps = pro->eps;
    }
    a.slots = ws.d_slots;
    a.err = ws.d_err;
    cudaError_t e = launch_rope_append(p->geom, a, st);
    if (e != cudaSuccess) return cuda_fail(e, "rope_append launch");
    p->last_launches += 1;
    return GKV_OK;
}

}  // namespace gkv

using gkv::Pool;
using gkv::set_error;

#define GKV_DEVICE_POOL(pool)                                                              \
    do {                                                                                   \
        if (!(pool)) return set_error(GKV_EINVAL, "pool handle is NULL");                  \
        if (!(pool)->impl.has_arena)                                                       \
            return set_error(GKV_ESTATE, "pool has no device arena (metadata-only pool)"); \
    } while (0)

extern "C" {

int gkv_step_reserve(gkv_pool* pool, int32_t max_batch, int32_t max_blocks_per_seq,
                     int32_t max_tokens, int32_t n_heads) {
    GKV_DEVICE_POOL(pool);
    gkv::DeviceGuard guard(pool->impl.desc.device);
    if (pool->impl.ws.static_mode)
        return set_error(GKV_ESTATE, "the static step layout is fixed: disable it before reserving again");
    return gkv::step_reserve(&pool->impl, max_batch, max_blocks_per_seq, max_tokens, n_heads);
}

int gkv_step_set_static(gkv_pool* pool, int32_t enable) {
    if (!pool) return set_error(GKV_EINVAL, "pool handle is NULL");
    if (!pool->impl.has_arena) return set_error(GKV_ESTATE, "pool has no device arena (metadata-only pool)");
    gkv::DeviceGuard guard(pool->impl.desc.device);
    return gkv::step_set_static(&pool->impl, enable != 0);
}

int gkv_upload_step(gkv_pool* pool, const int32_t* h_block_tables, int32_t batch,
                    int32_t max_blocks, const int32_t* h_ctx_lens, const int64_t* h_slot_mapping,
                    int32_t n_tok, void* stream) {
    GKV_DEVICE_POOL(pool);
    gkv::DeviceGuard guard(pool->impl.desc.device);
    return gkv::step_upload(&pool->impl, h_block_tables, batch, max_blocks, h_ctx_lens,
                            h_slot_mapping, n_tok, static_cast<cudaStream_t>(stream));
}

int gkv_upload_step_tables(gkv_pool* pool, gkv_table* const* tables, int32_t batch,
                           const int32_t* h_ctx_lens, const int64_t* h_slot_mapping, int32_t n_tok,
                           void* stream) {
    GKV_DEVICE_POOL(pool);
    if (batch < 0 || (batch > 0 && !tables)) return set_error(GKV_EINVAL, "tables is NULL");
    int32_t max_blocks = 1;
    for (int32_t b = 0; b < batch; ++b) {
        if (!tables[b] || tables[b]->impl.pool != &pool->impl)
            return set_error(GKV_EINVAL, "table %d is NULL or belongs to another pool", b);
        const int32_t n = static_cast<int32_t>(tables[b]->impl.ids.size());
        if (n > max_blocks) max_blocks = n;
    }
    std::vector<int32_t> packed(static_cast<size_t>(batch) * max_blocks, -1);
    std::vector<int32_t> ctx(static_cast<size_t>(batch));
    for (int32_t b = 0; b < batch; ++b) {
        const auto& ids = tables[b]->impl.ids;
        std::copy(ids.begin(), ids.end(), packed.begin() + static_cast<int64_t>(b) * max_blocks);
        ctx[static_cast<size_t>(b)] = h_ctx_lens ? h_ctx_lens[b] : tables[b]->impl.token_count;
    }
    gkv::DeviceGuard guard(pool->impl.desc.device);
    return gkv::step_upload(&pool->impl, packed.data(), batch, max_blocks, ctx.data(),
                            h_slot_mapping, n_tok, static_cast<cudaStream_t>(stream));
}

int gkv_kv_append(gkv_pool* pool, int32_t layer, const float* d_k, const float* d_v,
                  int32_t n_tok, void* stream) {
    GKV_DEVICE_POOL(pool);
    gkv::DeviceGuard guard(pool->impl.desc.device);
    pool->impl.last_launches = 0;
    return gkv::step_append(&pool->impl, layer, d_k, d_v, n_tok, static_cast<cudaStream_t>(stream));
}

int gkv_paged_decode(gkv_pool* pool, int32_t layer, const float* d_q, float* d_out,
                     int32_t n_heads, float scale, const float* d_sinks, void* stream) {
    GKV_DEVICE_POOL(pool);
    gkv::DeviceGuard guard(pool->impl.desc.device);
    pool->impl.last_launches = 0;
    return gkv::step_decode(&pool->impl, layer, d_q, d_out, n_heads, scale, d_sinks,
                            static_cast<cudaStream_t>(stream));
}

int gkv_paged_prefill(gkv_pool* pool, int32_t layer, const void* d_q, int32_t q_dtype, float* d_out,
                      const int32_t* h_q_start, const int32_t* h_q_len, int32_t n_heads, float scale,
                      void* stream) {
    GKV_DEVICE_POOL(pool);
    gkv::DeviceGuard guard(pool->impl.desc.device);
    pool->impl.last_launches = 0;
    return gkv::step_prefill(&pool->impl, layer, d_q, q_dtype, d_out, h_q_start, h_q_len, n_heads, scale,
                             static_cast<cudaStream_t>(stream));
}

int gkv_compute_attention(gkv_pool* pool, int32_t stage_layer, int32_t model_layer, int32_t pos,
                          const float* d_q, float* d_out, const gkv_table* table, int32_t n_heads,
                          int32_t n_heads_kv, int32_t head_dim, int32_t v_head_dim,
                          float attn_scale, int32_t max_seq_len, int32_t has_sink,
                          float sink_logit, void* stream) {
    (void)model_layer;  // unused, as in PagedAttentionKernel.cs:19
    GKV_DEVICE_POOL(pool);
    if (!table) return set_error(GKV_EINVAL, "blockTable is NULL");
    Pool& P = pool->impl;
    // PagedAttentionKernel.cs:34-39
    if (max_seq_len <= 0) return set_error(GKV_EINVAL, "maxSeqLen must be positive (got %d).", max_seq_len);
    if (pos < 0 || pos >= max_seq_len)
        return set_error(GKV_EINVAL, "Token position %d exceeds valid sequence range [0, %d].", pos, max_seq_len - 1);
    const gkv::Table& T = table->impl;
    if (T.token_count > max_seq_len)
        return set_error(GKV_EINVAL, "BlockTable token count %d exceeds maxSeqLen %d.", T.token_count, max_seq_len);
    if (T.pool != &P) return set_error(GKV_EINVAL, "blockTable belongs to another pool");
    if (n_heads_kv != P.desc.heads_kv || head_dim != P.desc.head_dim || v_head_dim != P.desc.v_head_dim)
        return set_error(GKV_EINVAL, "nHeadsKv/headDim/vHeadDim (%d/%d/%d) differ from the pool's (%d/%d/%d)",
                         n_heads_kv, head_dim, v_head_dim, P.desc.heads_kv, P.desc.head_dim, P.desc.v_head_dim);
    if (stage_layer < 0 || stage_layer >= P.desc.layers)
        return set_error(GKV_EINVAL, "stageLayer %d outside [0, %d)", stage_layer, P.desc.layers);
    // PagedAttentionKernel.cs:41-42
    const int32_t n = T.token_count < pos + 1 ? T.token_count : pos + 1;
    gkv::DeviceGuard guard(P.desc.device);
    P.last_launches = 0;
    if (n == 0) return GKV_OK;
    const int32_t nb = static_cast<int32_t>(T.ids.size());
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = gkv::step_upload(&P, T.ids.data(), 1, nb, &n, nullptr, 0, st);
    if (rc != GKV_OK) return rc;
    return gkv::decode_common(&P, stage_layer, d_q, d_out, n_heads, attn_scale, nullptr,
                              has_sink != 0, sink_logit, st);
}

int gkv_decode_step_host(gkv_pool* pool, int32_t layer, const int32_t* h_block_tables,
                         int32_t batch, int32_t max_blocks, const int32_t* h_ctx_lens,
                         const int64_t* h_slot_mapping, int32_t n_tok, const float* h_k_new,
                         const float* h_v_new, const float* h_q, float* h_out, int32_t n_heads,
                         float scale, const float* d_sinks, void* stream) {
    GKV_DEVICE_POOL(pool);
    Pool& P = pool->impl;
    if (batch > 0 && (!h_q || !h_out)) return set_error(GKV_EINVAL, "h_q/h_out is NULL");
    if (n_tok > 0 && (!h_k_new || !h_v_new)) return set_error(GKV_EINVAL, "h_k_new/h_v_new is NULL");
    if (n_heads <= 0 || n_heads % P.desc.heads_kv != 0)
        return set_error(GKV_EINVAL, "n_heads %d is not a positive multiple of heads_kv %d", n_heads, P.desc.heads_kv);
    gkv::DeviceGuard guard(P.desc.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    gkv::StepWorkspace& ws = P.ws;
    P.last_launches = 0;
    const size_t qb = static_cast<size_t>(batch) * n_heads * P.desc.head_dim * sizeof(float);
    const size_t ob = static_cast<size_t>(batch) * n_heads * P.desc.v_head_dim * sizeof(float);
    const size_t kb = static_cast<size_t>(n_tok) * P.desc.heads_kv * P.desc.head_dim * sizeof(float);
    const size_t vb = static_cast<size_t>(n_tok) * P.desc.heads_kv * P.desc.v_head_dim * sizeof(float);
    cudaError_t e = cudaSuccess;
    if (!ws.io_in) e = cudaStreamCreateWithFlags(&ws.io_in, cudaStreamNonBlocking);
    if (e == cudaSuccess && !ws.io_out) e = cudaStreamCreateWithFlags(&ws.io_out, cudaStreamNonBlocking);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaStreamCreate(step copies)");
    // Slot of this call; the call two back used it last.
    auto& io = ws.io[ws.io_next];
    auto& prev = ws.io[ws.io_next ^ 1];
    for (cudaEvent_t* ev : {&io.in_done, &io.used, &io.out_done})
        if (!*ev && (e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming)) != cudaSuccess)
            return gkv::cuda_fail(e, "cudaEventCreate(step copies)");
    if (qb > io.cap_q || ob > io.cap_out || kb > io.cap_k || vb > io.cap_v) {
        // growing frees buffers the earlier calls' copies may still use
        cudaStreamSynchronize(ws.io_in);
        cudaStreamSynchronize(ws.io_out);
        cudaStreamSynchronize(st);
    }
    int rc = gkv::grow_device(reinterpret_cast<void**>(&io.d_q), &io.cap_q, qb, "cudaMalloc(q)");
    if (rc == GKV_OK) rc = gkv::grow_device(reinterpret_cast<void**>(&io.d_out), &io.cap_out, ob, "cudaMalloc(out)");
    if (rc == GKV_OK) rc = gkv::grow_device(reinterpret_cast<void**>(&io.d_knew), &io.cap_k, kb, "cudaMalloc(k_new)");
    if (rc == GKV_OK) rc = gkv::grow_device(reinterpret_cast<void**>(&io.d_vnew), &io.cap_v, vb, "cudaMalloc(v_new)");
    if (rc != GKV_OK) return rc;
    // inputs: on the copy stream, once the call two back has finished reading this slot
    if (io.used_pending) e = cudaStreamWaitEvent(ws.io_in, io.used, 0);
    if (e == cudaSuccess && qb) e = cudaMemcpyAsync(io.d_q, h_q, qb, cudaMemcpyHostToDevice, ws.io_in);
    if (e == cudaSuccess && kb) e = cudaMemcpyAsync(io.d_knew, h_k_new, kb, cudaMemcpyHostToDevice, ws.io_in);
    if (e == cudaSuccess && vb) e = cudaMemcpyAsync(io.d_vnew, h_v_new, vb, cudaMemcpyHostToDevice, ws.io_in);
    if (e == cudaSuccess) e = cudaEventRecord(io.in_done, ws.io_in);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaMemcpyAsync(step inputs)");
    rc = gkv::step_upload(&P, h_block_tables, batch, max_blocks, h_ctx_lens, h_slot_mapping, n_tok, st);
    if (rc != GKV_OK) return rc;
    // compute on the caller's stream once the inputs are in and this slot's previous output
    // has been copied out
    e = cudaStreamWaitEvent(st, io.in_done, 0);
    if (e == cudaSuccess && io.out_pending) e = cudaStreamWaitEvent(st, io.out_done, 0);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaStreamWaitEvent(step inputs)");
    rc = gkv::step_append(&P, layer, io.d_knew, io.d_vnew, n_tok, st);
    if (rc != GKV_OK) return rc;
    rc = gkv::step_decode(&P, layer, io.d_q, io.d_out, n_heads, scale, d_sinks, st);
    if (rc != GKV_OK) return rc;
    e = cudaEventRecord(io.used, st);
    io.used_pending = e == cudaSuccess;
    // output: on the other copy stream, overlapping the next call's compute
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ws.io_out, io.used, 0);
    if (e == cudaSuccess && ob) e = cudaMemcpyAsync(h_out, io.d_out, ob, cudaMemcpyDeviceToHost, ws.io_out);
    if (e == cudaSuccess) e = cudaEventRecord(io.out_done, ws.io_out);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaMemcpyAsync(step output)");
    io.out_pending = true;
    // the caller's stream passes this point only after the previous call's output arrived, so
    // completing call k on `stream` means h_out of call k-1 is there; gkv_sync covers call k
    if (prev.out_pending) {
        e = cudaStreamWaitEvent(st, prev.out_done, 0);
        if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaStreamWaitEvent(previous output)");
    }
    ws.io_next ^= 1;
    return GKV_OK;
}

int gkv_rope_append(gkv_pool* pool, int32_t layer, float* d_q, const float* d_k, const float* d_v,
                    int32_t n_tok, int32_t n_heads, const int32_t* h_positions, const gkv_rope_desc* rope,
                    const gkv_qkv_prologue* prologue, void* stream) {
    GKV_DEVICE_POOL(pool);
    gkv::DeviceGuard guard(pool->impl.desc.device);
    pool->impl.last_launches = 0;
    return gkv::step_rope_append(&pool->impl, layer, d_q, d_k, d_v, n_tok, n_heads, h_positions, rope, prologue,
                                 static_cast<cudaStream_t>(stream));
}

int gkv_rope_inv_freq(float freq_base, int32_t rope_dim, const float* h_freq_factors, float* out) {
    if (rope_dim < 0 || (rope_dim & 1) || !(freq_base > 0.f) || (rope_dim > 0 && !out))
        return set_error(GKV_EINVAL, "freq_base %g / rope_dim %d / out", static_cast<double>(freq_base), rope_dim);
    gkv::rope_inv_freq(freq_base, rope_dim, h_freq_factors, out);
    return GKV_OK;
}

int gkv_wait_host_outputs(gkv_pool* pool, void* stream) {
    GKV_DEVICE_POOL(pool);
    Pool& P = pool->impl;
    gkv::DeviceGuard guard(P.desc.device);
    // the last call's slot; the output copies run in order on io_out, so its event covers all
    auto& last = P.ws.io[P.ws.io_next ^ 1];
    if (!last.out_pending) return GKV_OK;
    cudaError_t e = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), last.out_done, 0);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaStreamWaitEvent(host outputs)");
    return GKV_OK;
}

int gkv_plan_decode(const int32_t* ctx_lens, int32_t batch, int32_t heads_kv, int32_t block_size,
                    int32_t n_workers, gkv_plan_info* info, int32_t* piece_seg, int32_t* piece_c0,
                    int32_t* piece_c1, int32_t* piece_slot, int32_t* worker_begin,
                    int32_t cap_pieces) {
    if (batch < 0 || heads_kv < 1 || block_size < 1 || n_workers < 1 || (batch > 0 && !ctx_lens))
        return set_error(GKV_EINVAL, "batch=%d heads_kv=%d block_size=%d n_workers=%d", batch,
                         heads_kv, block_size, n_workers);
    gkv::WorkList W;
    gkv::build_work_list(ctx_lens, batch, heads_kv, block_size, n_workers, &W);
    const int32_t np = static_cast<int32_t>(W.piece_seg.size());
    if (info) {
        info->total_chunks = W.total_chunks;
        info->n_pieces = np;
        info->n_slots = W.n_slots;
        info->n_merge = static_cast<int32_t>(W.merge_seg.size());
        info->n_workers = n_workers;
        info->segment_cost = static_cast<int32_t>(gkv::kSegmentCost);
    }
    if (piece_seg || piece_c0 || piece_c1 || piece_slot) {
        if (cap_pieces < np) return set_error(GKV_EINVAL, "cap_pieces %d < %d pieces", cap_pieces, np);
        for (int32_t i = 0; i < np; ++i) {
            if (piece_seg) piece_seg[i] = W.piece_seg[static_cast<size_t>(i)];
            if (piece_c0) piece_c0[i] = W.piece_c0[static_cast<size_t>(i)];
            if (piece_c1) piece_c1[i] = W.piece_c1[static_cast<size_t>(i)];
            if (piece_slot) piece_slot[i] = W.piece_slot[static_cast<size_t>(i)];
        }
    }
    if (worker_begin)
        for (int32_t w = 0; w <= n_workers; ++w) worker_begin[w] = W.worker_begin[static_cast<size_t>(w)];
    return GKV_OK;
}

int gkv_sync(gkv_pool* pool, void* stream, int32_t timeout_ms) {
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::unique_ptr<gkv::DeviceGuard> guard;
    if (pool && pool->impl.has_arena) guard.reset(new gkv::DeviceGuard(pool->impl.desc.device));
    const auto t0 = std::chrono::steady_clock::now();
    // the host-buffer step copies its output back on an internal stream
    const cudaStream_t io_out = (pool && pool->impl.has_arena) ? pool->impl.ws.io_out : nullptr;
    for (;;) {
        cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess && io_out) e = cudaStreamQuery(io_out);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return gkv::cuda_fail(e, "cudaStreamQuery");
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (timeout_ms >= 0 && ms >= timeout_ms)
            return set_error(GKV_ETIMEDOUT, "stream still busy after %d ms", timeout_ms);
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    if (pool && pool->impl.has_arena && pool->impl.ws.d_err) {
        int flag = 0;
        cudaError_t e = cudaMemcpy(&flag, pool->impl.ws.d_err, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaMemcpy(error word)");
        if (flag != 0) {
            cudaMemset(pool->impl.ws.d_err, 0, sizeof(int));
            // a decode that stopped early may leave merge counters raised: start clean
            if (pool->impl.ws.d_merge_count)
                cudaMemset(pool->impl.ws.d_merge_count, 0, pool->impl.ws.merge_count_cap * sizeof(int32_t));
            return set_error(GKV_EDEVICE, "a kernel reported error bits 0x%x (1 = bad block id, 2 = wait timeout, 4 = bad slot)", flag);
        }
    }
    return GKV_OK;
}

}  // extern "C"
