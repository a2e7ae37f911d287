// Host-side launch interface of the sm_100a kernels (C++ linkage, internal to the shim).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gkv {

// Bytes per stored KV element of a GKV_DTYPE_* (fp32: 4; bf16 and fp16: 2; fp8 e4m3: 1).
inline int elem_bytes_of(int dtype) { return dtype == 0 ? 4 : (dtype == 3 ? 1 : 2); }
inline bool valid_kv_dtype(int dtype) { return dtype >= 0 && dtype <= 3; }
// Query / conversion types: fp32, bf16 and fp16 (fp8 is a storage format only).
inline bool valid_q_dtype(int dtype) { return dtype >= 0 && dtype <= 2; }

// Geometry of one pool's arenas, in ELEMENTS of the storage type.
struct ArenaGeom {
    void* k;                 // K arena base
    void* v;                 // V arena base
    int64_t k_block_stride, k_layer_stride, k_head_stride;
    int64_t v_block_stride, v_layer_stride, v_head_stride;
    int32_t total_blocks, layers, heads_kv, head_dim, v_head_dim, block_size;
    int32_t dtype;           // GKV_DTYPE_*
    // Host-side cache of the TMA tensor maps of K and V (CUtensorMap, 64-byte aligned) for
    // the tensor-core decodes; nullptr means "encode at launch".  Never read on the device.
    // tmap_rank is the maps' rank (3) once encoded, 0 when there are none.
    const void* tmap_k = nullptr;
    const void* tmap_v = nullptr;
    int32_t tmap_rank = 0;
    // The same with boxes of 16 slots (block sizes that are multiples of 16), for the prefill.
    const void* tmap_pk = nullptr;
    const void* tmap_pv = nullptr;
    // FP8 arenas: device [layers][heads_kv] K and V scales and their reciprocals (an element
    // stores e4m3(x * inv) and reads back as e4m3 * scale); nullptr for every other type.
    const float* k_scale = nullptr;
    const float* v_scale = nullptr;
    const float* k_inv = nullptr;
    const float* v_inv = nullptr;
};

// ---- packed step metadata ----
// The step's metadata is one buffer: a header of counts and byte offsets, then the slot
// mapping (at a fixed offset), then the tables, context lengths and work list.  A launch
// normally receives the pointers and counts by value; in the static step layout (the launches
// of a step captured once in a CUDA graph and replayed every step) it receives the buffer's
// base (DecodeWork::dyn) and reads them from the header, which every upload rewrites.
enum : int {
    kHdrTok, kHdrBatch, kHdrMaxBlocks, kHdrSlots, kHdrMerge, kHdrDeferred, kHdrDeferredLong, kHdrWorkers,
    kHdrTables, kHdrCtx, kHdrPseg, kHdrPc0, kHdrPc1, kHdrPslot, kHdrPmerge, kHdrWbeg, kHdrMseg, kHdrMs0,
    kHdrMns, kHdrMdef, kHdrInts
};
constexpr size_t kHdrBytes = 128;  // the slot mapping starts here
static_assert(kHdrInts * 4 <= static_cast<int>(kHdrBytes), "step header");

// ---- kv append ----
// Writes token i's K/V rows into slot slots[i] (or `single_slot` when slots == nullptr and
// n_tok == 1).  Source row stride in elements per token: k_tok_stride / v_tok_stride.  With
// dyn_tok set (the static step layout), the token count is read from *dyn_tok on the device
// (at most n_tok, which then sizes the grid).
cudaError_t launch_kv_append(const ArenaGeom& g, int layer, const float* k, const float* v,
                             int64_t k_tok_stride, int64_t v_tok_stride, const int64_t* slots,
                             int64_t single_slot, int n_tok, int* err, cudaStream_t stream,
                             const int32_t* dyn_tok = nullptr);

// ---- fused q/k/v prologue + KV append (rope_append.cu) ----
struct RopeAppendParams {
    int layer;
    float* q;                  // [n_tok][n_heads][head_dim], rewritten in place
    const float* k;            // [n_tok][heads_kv][head_dim]
    const float* v;            // [n_tok][heads_kv][v_head_dim]
    int n_tok, n_heads;
    const int32_t* positions;  // device [n_tok]
    const float* inv_freq;     // device [rope_dim / 2]
    int rope_dim, style;       // style 0: pairs (i, i + rope_dim/2); 1: pairs (2i, 2i+1)
    float mscale;
    const float *q_bias, *k_bias, *v_bias, *q_norm, *k_norm;  // device or nullptr
    float eps;
    const int64_t* slots;      // device [n_tok]
    int* err;
};
// head_dim in {32, 64, 128, 256}, rope_dim even, <= head_dim, (rope_dim/2) % (head_dim/32) == 0.
bool rope_append_supported(const ArenaGeom& g, int rope_dim);
cudaError_t launch_rope_append(const ArenaGeom& g, const RopeAppendParams& p, cudaStream_t st);

// ---- block copy ----
// ops: [n][3] int32 (src, dst, valid_tokens) in device memory.
cudaError_t launch_block_copy(const ArenaGeom& g, const int32_t* ops, int n, int* err,
                              cudaStream_t stream);

// ---- paged decode ----
constexpr int kDecodeChunk = 8;  // tokens per decode work chunk
// Segments split into more pieces than this are merged by the merge kernel, the others by the
// decode warp that completes them.  0: the merge kernel takes every split segment.  In-kernel
// merging costs each arriving warp a fence + atomic round trip (~4 us under full HBM load)
// and puts merges on the decode's tail; with the merge launch overlapped (programmatic
// dependent launch) the merge kernel measured 2 % faster on cfg2 and equal elsewhere.
constexpr int kFusedMergeMaxSlots = 0;
// Chunks' worth of time charged to every segment when the chunk stream is cut into equal
// worker ranges, so a warp that starts more segments (a q load, a new table row, a partial
// per piece) gets fewer chunks.  Measured on the lognormal 256-sequence batch: 0 -> 4 took the
// fp32 decode from 0.782 to 0.807 of HBM and bf16 from 0.727 to 0.774; 8 was worse than 4;
// the uniform 64 x 2049 batch was unchanged.
constexpr int64_t kSegmentCost = 4;
// A deferred merge of a segment with more than this many slots gets a CTA of eight warps per
// (segment, head), the others one warp each (eight per CTA), in the same launch.  On a lognormal
// 32-sequence batch one 21k-token sequence split into 240 slots took a lone warp 18 us while the
// other 1000 merges took 3 us; a CTA for every merge took 9 us (3.5 waves of mostly idle warps).
constexpr int kWarpMergeMaxSlots = 32;

// Work list of one step, built on the host (all pointers are device pointers).
//  segment s = b * heads_kv + h; its chunks are k = 0 .. n_chunks(ctx_b) - 1, chunk k
//  covering tokens [page*bs + sub*8, ...) with page = k / cpp, sub = k % cpp,
//  cpp = ceil(block_size / 8).
//  piece  = contiguous chunk range [c0, c1) of one segment handled by one warp worker.
struct DecodeWork {
    const int32_t* tables;             // [batch][max_blocks]
    const int32_t* ctx_lens;           // [batch]
    int32_t max_blocks;
    const int32_t* piece_seg;          // [n_pieces]
    const int32_t* piece_c0;           // [n_pieces]
    const int32_t* piece_c1;           // [n_pieces]
    const int32_t* piece_slot;         // partial slot, or -1 when the piece is a whole segment
    const int32_t* worker_piece_begin; // [n_workers + 1]
    int32_t n_ctas;                    // grid.x; n_workers = n_ctas * warps per CTA
    int32_t n_slots;                   // partial slots in this step
    const int32_t* merge_seg;          // [n_merge] segments split over several workers
    const int32_t* merge_slot0;        // their first partial slot (slots are contiguous)
    const int32_t* merge_nslots;
    // [n_pieces] merge entry of a split piece whose segment is merged inside the decode
    // kernel (at most kFusedMergeMaxSlots pieces); -1 for an unsplit piece; -2 when the
    // segment is merged afterwards by the deferred-merge kernel.
    const int32_t* piece_merge;
    int32_t n_merge;
    const int32_t* merge_deferred;     // [n_deferred] merge entries left to the merge kernel
    int32_t n_deferred;
    int32_t n_deferred_long;           // the first entries of merge_deferred with > kWarpMergeMaxSlots slots
    // Arrival counters of the fused merge, [head_groups][n_merge] ints.  They must be zero
    // when a launch starts; the worker that completes a segment resets its counter, so they
    // are zero again after every launch that ran to completion.
    int32_t* merge_count;
    // [batch] table row of each sequence, or nullptr for row = sequence.  The prefill over
    // the decode kernel makes every query of a sequence a sequence of its own on one row.
    const int32_t* table_row;
    // Static step layout: the packed step buffer, whose header supplies every pointer and
    // count above except merge_count and table_row (nullptr: use the fields as given).
    const unsigned char* dyn;
    // Static step layout: the deferred-merge kernel is launched on every call with this fixed
    // grid and loops over the entries the header counts (0: launched only when n_deferred > 0,
    // with one CTA per item group).
    int32_t merge_grid;
};

struct DecodeArgs {
    int layer;
    const float* q;      // [batch][n_heads][head_dim]
    float* out;          // [batch][n_heads][v_head_dim]
    int n_heads;
    float scale;
    const float* sinks;  // [n_heads] or nullptr
    int has_sink_all;    // when sinks == nullptr: 1 = every head uses sink_all
    float sink_all;
    float* part_acc;     // [head_groups][n_slots][gp][v_head_dim]
    float* part_ml;      // [head_groups][n_slots][gp][2]
    int* err;
    // Optional [batch][n_heads]: natural-log softmax denominator of every written output row,
    // ln(sum_t exp(s_t) [+ exp(sink)]), for merging outputs computed over disjoint token ranges.
    float* lse = nullptr;
};

// out[r][d] = sum_p exp(lse_p[r] - LSE[r]) * part_p[r][d] with LSE[r] = ln(sum_p exp(lse_p[r])
// [+ exp(sink[r % n_heads])]).  parts: n_parts blocks of (rows * dv outputs, then rows lses).
cudaError_t launch_lse_merge(const float* parts, int n_parts, int rows, int dv, const float* sinks,
                             int n_heads, float* out, cudaStream_t st);
// x[0..n) = value
cudaError_t launch_fill(float* x, int64_t n, float value, cudaStream_t st);

// ---- peer-memory exchange of split-KV partials (exchange.cu) ----
// Mailbox of rank r, as this rank addresses it: mbox[r] = [2][n_ranks][slot] floats,
// flags[r] = [2][n_ranks] epoch words (own rank: local pointers; peers: CUDA IPC mappings).
constexpr int kMaxExchangeRanks = 16;
struct ExchangePeers {
    float* mbox[kMaxExchangeRanks];
    unsigned* flags[kMaxExchangeRanks];
    int n_ranks;
    int64_t slot;  // floats per slot, a multiple of 4
};
// Slot [parity][me] of this rank's own mailbox: where its decode writes (out [rows][dv], then
// lse [rows]) for an epoch of that parity.
float* exchange_slot(const ExchangePeers& p, int me, int parity);
// After the decode that filled this rank's slot (a programmatic dependent launch): publishes
// `epoch` in flag [parity][me] of every rank, waits (bounded) until all of this rank's flags
// of the parity read `epoch`, then merges every rank's block of the parity by log-sum-exp into
// out [rows][dv] (dv a multiple of 4), as launch_lse_merge.
cudaError_t launch_exchange_pull_merge(const ExchangePeers& p, int me, int parity, unsigned epoch, int rows, int dv,
                                       const float* sinks, int n_heads, float* out, int* err, cudaStream_t st);

// Launch configuration the decode kernel uses for this geometry and query-head count.
struct DecodeConfig {
    bool supported;
    int gp;            // query heads per pass (power of two <= 8)
    int head_groups;   // ceil(group / gp)
    int warps;         // warp workers per CTA
    int threads;
    size_t smem;
    int ctas_per_sm;
};
DecodeConfig decode_config(const ArenaGeom& g, int n_heads);

// Second launch of a decode whose work list defers merges (w.n_deferred > 0, or w.merge_grid
// > 0 in the static step layout).
cudaError_t launch_deferred_merge(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                  int group, int gp, int head_groups, cudaStream_t st);

// Tensor-core variant (paged_decode_tc.cu): bf16 KV, d = dv = 128, block size a multiple of
// 8, query group 5..8 per head group.  Same work list and partial layout; 4 warps per CTA.
bool decode_tc_eligible(const ArenaGeom& g, int n_heads);
// Encodes the K and V TMA maps of the arena into two 128-byte, 64-byte aligned buffers.
// Encodes the decode maps of an arena with d = dv = 128 (8-token boxes, 128-byte swizzle) and
// returns their rank (3), 0 on failure: bf16 / fp16 views [dim][slot][block*layer*head] with
// boxes of 8 slots x 64 dims; FP8 views with boxes of 8 slots x 128 one-byte dims.
int encode_decode_tmaps(const ArenaGeom& g, void* tmap_k, void* tmap_v);
// Tiled TMA maps (bf16, 128-byte swizzle, no interleave; `map` is a 64-byte aligned
// 128-byte CUtensorMap).  encode_arena_map: the 3-D view [block*layer*head][slot][dim] of
// one arena with boxes of `rows` slots x 64 dims.
bool tmap_encoder_available();
bool encode_bf16_map3(void* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                      const uint32_t box[3]);
bool encode_arena_map(void* map, void* base, const ArenaGeom& g, int dim, int rows = kDecodeChunk);
void decode_tc_config(DecodeConfig& c);
// Tensor-core variant for FP8 E4M3 KV (paged_decode_fp8.cu): d = dv = 128, block size a
// multiple of 8, query group 5..8 per head group, scales present.  Same work list and partials.
bool decode_fp8_tc_eligible(const ArenaGeom& g, int n_heads);
void decode_fp8_tc_config(DecodeConfig& c);
cudaError_t launch_paged_decode_fp8_tc(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a, int group,
                                       int head_groups, int* launches, cudaStream_t st);
cudaError_t launch_paged_decode_tc(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                   int group, int head_groups, int* launches, cudaStream_t st);

// ---- chunked causal prefill (paged_prefill_tc.cu) ----
// One work item = up to 128 consecutive queries of one sequence; the kernel runs one CTA per
// (item, query head).  Item ints: sequence (table row), position of the first query, its
// row in the packed q / out, query count, keys attended by the item (min(token_count,
// last position + 1)), token_count, 2 unused.
constexpr int kPrefillItemInts = 8;
struct PrefillArgs {
    const int32_t* items;    // device [n_items][kPrefillItemInts], heaviest first
    int32_t n_items;
    const int32_t* tables;   // uploaded block tables [batch][max_blocks]
    int32_t max_blocks;
    int32_t layer;
    int32_t n_heads;
    float scale;
    float* out;              // [total_q][n_heads][v_head_dim] fp32
    int* err;
};
// bf16 or fp16 KV, d = dv = 128, block size a multiple of 8.
bool prefill_tc_eligible(const ArenaGeom& g, int n_heads);
// q16: [total_q][n_heads][128] in the arena's 16-bit type, 16-byte aligned.
cudaError_t launch_paged_prefill_tc(const ArenaGeom& g, const PrefillArgs& a, const void* q16,
                                    int64_t total_q, cudaStream_t st);
// n elements of GKV_DTYPE_* src_dtype -> dst_dtype (different types), round to nearest even;
// fp16 results saturate at +-65504.
cudaError_t launch_convert(const void* src, int32_t src_dtype, void* dst, int32_t dst_dtype, int64_t n,
                           cudaStream_t st);

// Enqueues the split-KV decode (the cross-worker merge is fused into it).  *launches
// receives the number of kernels enqueued.
cudaError_t launch_paged_decode(const ArenaGeom& g, const DecodeWork& w, const DecodeArgs& a,
                                int* launches, cudaStream_t stream);

}  // namespace gkv
