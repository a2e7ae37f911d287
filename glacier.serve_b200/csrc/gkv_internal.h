// Internal C++ state behind the C ABI of include/glacier_kv.h.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/glacier_kv.h"
#include "kernels.h"

namespace gkv {

// ---- error reporting -------------------------------------------------------------------
int set_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int cuda_fail(cudaError_t e, const char* what);

// Restores the calling thread's current device on scope exit.
class DeviceGuard {
   public:
    explicit DeviceGuard(int device);
    ~DeviceGuard();
    bool ok() const { return ok_; }

   private:
    int prev_ = -1;
    bool ok_ = false;
};

// ---- host mirror of the free list (PagedBlockPool.cs:39,112-120,178-189,251-279) --------
// Treiber stack over block indices.  The head packs (ABA tag << 32 | (index + 1)); a tagged
// compare-exchange makes pop safe against a concurrent pop/push of the same index.
class FreeStack {
   public:
    void init(int32_t n);  // pushes n-1 .. 0 so that 0 pops first
    // Replaces the contents with pop_order (first element pops first).  Not safe against
    // concurrent push/pop: the caller excludes every other allocator call.
    void rebuild(const std::vector<int32_t>& pop_order);
    void push(int32_t idx);
    int32_t pop();         // -1 when empty
    int32_t count() const { return count_.load(std::memory_order_acquire); }

   private:
    std::unique_ptr<std::atomic<int32_t>[]> next_;
    std::atomic<uint64_t> head_{0};
    std::atomic<int32_t> count_{0};
};

// ConcurrentDictionary<ulong,int> analogue for the prefix map (PagedBlockPool.cs:43):
// sharded, each shard under its own mutex.
class PrefixMap {
   public:
    bool find(uint64_t h, int32_t* out) const;
    void set(uint64_t h, int32_t id);
    void remove_if(uint64_t h, int32_t id);  // TryRemove(KeyValuePair(h, id))

   private:
    static constexpr int kShards = 64;
    struct Shard {
        mutable std::mutex mu;
        std::unordered_map<uint64_t, int32_t> map;
    };
    Shard shards_[kShards];
    static int shard_of(uint64_t h) { return static_cast<int>((h ^ (h >> 29) ^ (h >> 47)) & (kShards - 1)); }
};

// Work-list construction (host only; unit-tested through the C ABI helpers).
//
// plan_work_into is the one planner of the decode work list.  It writes into caller-owned
// arrays (no heap), sized for n_workers + batch * heads_kv pieces and batch * heads_kv merge
// entries; build_work_list wraps it with vectors, and the allocation-free decode calls it on its
// static staging buffer.
struct PlanArrays {
    int32_t *piece_seg, *piece_c0, *piece_c1, *piece_slot, *piece_merge;
    int32_t* worker_begin;  // n_workers + 1
    int32_t *merge_seg, *merge_slot0, *merge_nslots, *merge_deferred;
    // results
    int32_t n_pieces, n_slots, n_merge, n_deferred;
    int64_t total_chunks;
    int32_t n_deferred_long;  // leading deferred entries with more than kWarpMergeMaxSlots slots
};
void plan_work_into(const int32_t* ctx_lens, int32_t batch, int32_t heads_kv, int32_t block_size,
                    int32_t n_workers, PlanArrays* out);
// Persistent-grid size of a decode over `total_chunks` chunks: enough warp workers for
// kMinChunksPerWorker chunks each, at most max_ctas CTAs of `warps` workers, >= 1 CTA when
// there is work.
int64_t decode_grid_ctas(int64_t total_chunks, int warps, int64_t max_ctas);

struct WorkList {
    std::vector<int32_t> piece_seg, piece_c0, piece_c1, piece_slot, piece_merge, merge_deferred;
    std::vector<int32_t> worker_begin;  // n_workers + 1
    std::vector<int32_t> merge_seg, merge_slot0, merge_nslots;
    int32_t n_slots = 0;
    int32_t n_deferred_long = 0;
    int64_t total_chunks = 0;
};

// A pinned staging buffer and its device twin for small per-call uploads: the host copy is
// reused once the previous upload from it has landed; the device copy is ordered on the stream.
struct StageBuf {
    char* h = nullptr;
    char* d = nullptr;
    size_t cap = 0;
    cudaEvent_t copied = nullptr;
    bool pending = false;
};

// Device + pinned buffers of one step (block tables, ctx lens, slot mapping, work list).
struct StepWorkspace {
    int32_t max_batch = 0, max_blocks = 0, max_tokens = 0, n_heads = 0;
    DecodeConfig cfg{};
    int32_t n_ctas_max = 0;   // persistent grid size for this geometry
    // Packed metadata: one copy per step, from two pinned staging buffers into two device
    // buffers used in turn.  The copy runs on meta_stream as soon as the step that last used
    // its buffer (two uploads ago) has finished, so it overlaps the previous step's kernels;
    // the caller's stream then waits for it.
    char* h_meta[2] = {nullptr, nullptr};
    char* d_meta[2] = {nullptr, nullptr};
    size_t meta_cap = 0;
    cudaEvent_t meta_copied[2] = {nullptr, nullptr};  // staging + device buffer i filled
    bool meta_pending[2] = {false, false};
    // recorded on the caller's stream at upload time: everything queued before that upload
    cudaEvent_t meta_mark[2] = {nullptr, nullptr};
    bool meta_marked[2] = {false, false};
    cudaStream_t meta_stream = nullptr;
    int meta_flip = 0;
    // Static step layout (gkv_step_set_static): every upload goes to d_meta[0] on the caller's
    // stream and the launches read the header there, so that they can be captured once in a
    // CUDA graph and replayed every step; grids are the reserved maxima.
    bool static_mode = false;
    int32_t static_merge_grid = 0;
    // partial results of split segments
    float* d_part_acc = nullptr;
    float* d_part_ml = nullptr;
    size_t part_slots_cap = 0;  // slots (x head_groups x gp) the buffers hold
    // arrival counters of the fused merge; zero between launches (kernels reset them)
    int32_t* d_merge_count = nullptr;
    size_t merge_count_cap = 0;
    // device error word shared by every kernel of this pool
    int* d_err = nullptr;
    // e2e staging for gkv_decode_step_host
    // Two slots, used by consecutive calls in turn: the inputs of call k+1 travel on io_in and
    // the output of call k on io_out while the caller's stream computes.
    struct IoSlot {
        float* d_q = nullptr;
        float* d_out = nullptr;
        float* d_knew = nullptr;
        float* d_vnew = nullptr;
        size_t cap_q = 0, cap_out = 0, cap_k = 0, cap_v = 0;
        cudaEvent_t in_done = nullptr;    // inputs copied
        cudaEvent_t used = nullptr;       // append + decode finished reading inputs, writing out
        cudaEvent_t out_done = nullptr;   // output copied back
        bool used_pending = false, out_pending = false;
    } io[2];
    cudaStream_t io_in = nullptr, io_out = nullptr;
    int io_next = 0;
    // the uploaded step
    int32_t batch = 0, n_tok = 0, up_max_blocks = 0;
    DecodeWork work{};
    const int64_t* d_slots = nullptr;
    bool uploaded = false;
    std::vector<int32_t> h_ctx;  // ctx_lens of the uploaded step
    WorkList wl;                 // the uploaded step's work list (kept for its capacity)
    // chunked prefill: pinned + device buffer of its work items / work list, and q in the
    // dtype its kernel reads
    StageBuf pre;
    // fused rope + append: positions and the inverse-frequency table
    StageBuf rope;
    void* d_qconv = nullptr;
    size_t qconv_cap = 0;
};

struct Pool {
    gkv_pool_desc desc{};
    ArenaGeom geom{};
    size_t elem_bytes = 4;
    int64_t k_bytes = 0, v_bytes = 0;
    bool has_arena = false;

    FreeStack free_stack;
    std::unique_ptr<std::atomic<int32_t>[]> allocated;
    std::unique_ptr<std::atomic<int32_t>[]> refcount;
    std::unique_ptr<std::atomic<uint64_t>[]> prefix_hash;
    PrefixMap prefix_map;

    std::mutex pending_mu;
    std::vector<int32_t> pending;  // queued CoW copies, (src, dst, valid) triples
    int32_t* d_copy_ops = nullptr;
    size_t copy_ops_cap = 0;
    int32_t* h_copy_ops = nullptr;  // pinned staging for the op list
    cudaEvent_t copy_ops_copied = nullptr;

    StepWorkspace ws;
    int last_launches = 0;
    // FP8 pools: [4][layers][heads_kv] device floats (K scale, V scale, their reciprocals)
    float* d_scales = nullptr;
    // TMA maps of the arena for the tensor-core decode, encoded once at creation
    alignas(64) unsigned char tmap_k[128];
    alignas(64) unsigned char tmap_v[128];
    // the same views with 16-slot boxes, for the prefill kernel
    alignas(64) unsigned char tmap_pk[128];
    alignas(64) unsigned char tmap_pv[128];

    bool in_range(int32_t b) const {
        return static_cast<uint32_t>(b) < static_cast<uint32_t>(desc.total_blocks);
    }
    // allocator primitives (reference semantics)
    int32_t try_allocate();
    int release(int32_t b);
    int retain(int32_t b);
    int refs(int32_t b) const;
    bool try_find_prefix(uint64_t h, int32_t* out);
    bool try_fork(int32_t src, int32_t valid, int32_t* out);
    size_t stats_pending_copies() {
        std::lock_guard<std::mutex> lk(pending_mu);
        return pending.size() / 3;
    }
    // device helpers (caller holds a DeviceGuard)
    int flush_copies(cudaStream_t st);
    // Moves movable live blocks into the lowest free ids (compact.cpp); returns the number of
    // moves (src[i] -> dst[i]) or a negative code.  Excludes concurrent allocator calls.
    int compact(struct Table* const* tables, int32_t n_tables, int32_t max_moves, std::vector<int32_t>* src,
                std::vector<int32_t>* dst, cudaStream_t st);
    int launch_copies(const int32_t* h_ops, int n, cudaStream_t st);
};

struct Table {
    Pool* pool = nullptr;
    std::vector<int32_t> ids;
    int32_t token_count = 0;
};

// step.cpp
int step_upload(Pool* p, const int32_t* tables, int32_t batch, int32_t max_blocks,
                const int32_t* ctx_lens, const int64_t* slots, int32_t n_tok, cudaStream_t st);
int step_decode(Pool* p, int32_t layer, const float* d_q, float* d_out, int32_t n_heads,
                float scale, const float* d_sinks, cudaStream_t st);
int step_append(Pool* p, int32_t layer, const float* d_k, const float* d_v, int32_t n_tok,
                cudaStream_t st);
int step_decode_lse(Pool* p, int32_t layer, const float* d_q, float* d_out, float* d_lse,
                    int32_t n_heads, float scale, const float* d_sinks, cudaStream_t st);
int step_set_static(Pool* p, bool enable);
int step_reserve(Pool* p, int32_t max_batch, int32_t max_blocks, int32_t max_tokens,
                 int32_t n_heads);
int step_prefill(Pool* p, int32_t layer, const void* d_q, int32_t q_dtype, float* d_out,
                 const int32_t* q_start, const int32_t* q_len, int32_t n_heads, float scale,
                 cudaStream_t st);
int step_rope_append(Pool* p, int32_t layer, float* d_q, const float* d_k, const float* d_v, int32_t n_tok,
                     int32_t n_heads, const int32_t* positions, const gkv_rope_desc* rope,
                     const gkv_qkv_prologue* pro, cudaStream_t st);
void rope_inv_freq(float freq_base, int32_t rope_dim, const float* factors, float* out);
void step_free(Pool* p);

int32_t chunks_of(int32_t ctx, int32_t block_size);
void build_work_list(const int32_t* ctx_lens, int32_t batch, int32_t heads_kv, int32_t block_size,
                     int32_t n_workers, WorkList* out);

}  // namespace gkv

struct gkv_pool {
    gkv::Pool impl;
};
struct gkv_table {
    gkv::Table impl;
};
