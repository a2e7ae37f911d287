/*
 * glacier_kv.h -- C ABI of the B200 (sm_100a) paged-KV hot path for Glacier.Serve.
 *
 * The C# engine (ContinuousBatchEngine / CudaPagedTransformerRunner) P/Invokes these
 * entry points in place of its host-side PagedBlockPool arena, its per-sequence
 * BlockTable uploads and its CPU PagedAttentionKernel.  Every declaration below cites the
 * reference member it replaces as `path:line` inside the Glacier.Serve repository
 * (src/Glacier.Serve/Inference/PagedAttention/...).
 *
 * Conventions
 *   - Every call returns an int status: GKV_OK (0) or a negative GKV_E* code.  Nothing
 *     throws or aborts across the ABI; gkv_last_error() returns a thread-local message
 *     for the last failing call on the calling thread.  The reference's
 *     ArgumentOutOfRangeException maps to GKV_EINVAL, InvalidOperationException to
 *     GKV_ESTATE.
 *   - Calls named try_* return 1 (success) / 0 (pool exhausted or not found) like the
 *     reference's bool TryXxx(out ...) methods, and a negative code on a bad argument.
 *   - Pointers named d_* are device pointers on the pool's device, h_* are host pointers
 *     (pinned memory recommended).  Streams are cudaStream_t passed as void*; NULL is the
 *     legacy default stream.  All device work is enqueued asynchronously on the stream.
 *   - Pool, table and step objects are not thread-safe for concurrent device calls, but the
 *     allocator calls (allocate / retain / release / find / bind / fork) are lock-free or
 *     internally locked and may be called from any thread, as in the reference
 *     (PagedBlockPool.cs:16 "thread-safe O(1) lock-free block allocation").
 */
#ifndef GLACIER_KV_H
#define GLACIER_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GKV_API __attribute__((visibility("default")))
#else
#define GKV_API
#endif

/* ---- status codes -------------------------------------------------------------------- */
enum {
    GKV_OK = 0,
    GKV_EINVAL = -1,        /* argument out of range (reference: ArgumentOutOfRangeException)  */
    GKV_ENOMEM = -2,        /* device/pinned allocation failed                                */
    GKV_ESTATE = -3,        /* invalid object state (reference: InvalidOperationException)    */
    GKV_ECUDA = -4,         /* a CUDA runtime call failed                                     */
    GKV_ETIMEDOUT = -5,     /* gkv_sync gave up waiting                                       */
    GKV_ENCCL = -6,         /* an NCCL call failed or was aborted                              */
    GKV_EDEVICE = -7,       /* a kernel reported a bad block id / bounded wait expiry          */
    GKV_EUNSUPPORTED = -8   /* shape not compiled into this build (e.g. head_dim % 32 != 0)   */
};

/* KV storage types of the device arena.  Sources handed to append/store are always fp32
 * (the reference stores fp32, PagedBlockPool.cs:151-161); bf16 and fp16 storage round to
 * nearest even on append.  GKV_DTYPE_F16 is the precision of the reference's GPU pools
 * (CudaPagedTransformerRunner.cs:118-119, KvCachePrecision.Fp16 at :139).  GKV_DTYPE_FP8_E4M3 (no
 * reference counterpart) keeps e4m3(x * (1 / scale)), rounded to nearest even and saturated at
 * +-448, with one K scale and one V scale per (layer, kv head) (gkv_pool_set_kv_scales, default
 * 1); it reads back as e4m3 * scale.  FP8 pools run the CUDA-core decode (head dims 64 and 128)
 * and the decode-kernel prefill. */
enum { GKV_DTYPE_F32 = 0, GKV_DTYPE_BF16 = 1, GKV_DTYPE_F16 = 2, GKV_DTYPE_FP8_E4M3 = 3 };

typedef struct gkv_pool gkv_pool;
typedef struct gkv_table gkv_table;
typedef struct gkv_comm gkv_comm;

/* ---- 1. the device block arena (PagedBlockPool) ------------------------------------- */

typedef struct gkv_pool_desc {
    int32_t device;                /* CUDA device ordinal that holds the arena            */
    int32_t total_blocks;          /* PagedBlockPool(totalBlocks ...)                     */
    int32_t layers;
    int32_t heads_kv;
    int32_t head_dim;
    int32_t v_head_dim;            /* <= 0 means head_dim (PagedBlockPool.cs:73)          */
    int32_t block_size;            /* tokens per block; 0 means 16 (PagedBlockPool.cs:18) */
    int32_t dtype;                 /* GKV_DTYPE_F32, _BF16, _F16 or _FP8_E4M3             */
    int32_t allocate_device_arena; /* 0 = metadata-only pool: allocator, tables and CoW
                                      bookkeeping without any CUDA call (the reference's
                                      allocateHostBuffers:false, PagedBlockPool.cs:61,106) */
} gkv_pool_desc;

typedef struct gkv_pool_stats {
    int32_t total_blocks;          /* TotalBlocks          PagedBlockPool.cs:46 */
    int32_t free_blocks;           /* FreeBlocksCount      PagedBlockPool.cs:52 */
    int32_t allocated_blocks;      /* AllocatedBlocksCount PagedBlockPool.cs:53 */
    int32_t capacity_tokens;       /* CapacityTokens       PagedBlockPool.cs:54 */
    int32_t active_tokens;         /* ActiveTokens         PagedBlockPool.cs:55 */
    int32_t block_size;            /* BlockSize            PagedBlockPool.cs:47 */
    int32_t pending_copies;        /* CoW forks queued for the next device call          */
    int32_t has_device_arena;      /* HasHostBuffers analogue, PagedBlockPool.cs:56      */
    int64_t total_memory_bytes;    /* TotalMemoryBytes     PagedBlockPool.cs:57 */
} gkv_pool_stats;

/* PagedBlockPool ctor, PagedBlockPool.cs:61-121: validates every size >= 1 (:63-67),
 * allocates the zeroed K and V arenas in the layout [block][layer][head_kv][slot][dim]
 * (strides :77-83) and fills the free list so that block 0 is popped first (:116-120). */
GKV_API int gkv_pool_create(const gkv_pool_desc* desc, gkv_pool** out_pool);
/* PagedBlockPool.Dispose, PagedBlockPool.cs:355-364. */
GKV_API int gkv_pool_destroy(gkv_pool* pool);
/* Counters of PagedBlockPool.cs:46-57. */
GKV_API int gkv_pool_stats_get(const gkv_pool* pool, gkv_pool_stats* out_stats);
/* The K and V scales of an FP8 pool, h_k_scales / h_v_scales [layers][heads_kv], positive and
 * finite (GKV_EINVAL otherwise; GKV_ESTATE for a pool of another type).  Set them before the
 * first append: elements already stored keep the scale they were stored with.  A synchronous
 * host-to-device copy.  No reference counterpart (the reference stores fp32). */
GKV_API int gkv_pool_set_kv_scales(gkv_pool* pool, const float* h_k_scales, const float* h_v_scales);
/* KeyBufferAddress / ValueBufferAddress, PagedBlockPool.cs:58-59 (device pointers; NULL
 * for a metadata-only pool). */
GKV_API int gkv_pool_kv_ptrs(const gkv_pool* pool, void** d_k, void** d_v);
/* Element offset of (block, layer, head_kv, slot) in the K or V arena:
 * GetKeyPtr / GetValuePtr, PagedBlockPool.cs:124-145.  which: 0 = K, 1 = V. */
GKV_API int gkv_pool_element_offset(const gkv_pool* pool, int32_t which, int32_t block,
                                    int32_t layer, int32_t head_kv, int32_t slot,
                                    int64_t* out_offset);

/* TryAllocateBlock, PagedBlockPool.cs:178-189: returns 1 and the block id, or 0 and -1. */
GKV_API int gkv_pool_try_allocate_block(gkv_pool* pool, int32_t* out_block);
/* ReleaseBlock, PagedBlockPool.cs:251-279: returns the remaining reference count (>= 0);
 * out-of-range ids and double releases return 0 and change nothing. */
GKV_API int gkv_pool_release_block(gkv_pool* pool, int32_t block);
/* FreeBlock / FreeBlocks, PagedBlockPool.cs:296-299,347-353 (idempotent). */
GKV_API int gkv_pool_free_block(gkv_pool* pool, int32_t block);
GKV_API int gkv_pool_free_blocks(gkv_pool* pool, const int32_t* blocks, int32_t n);
/* RetainBlock, PagedBlockPool.cs:240-245: GKV_EINVAL for an out-of-range id, otherwise the
 * new reference count. */
GKV_API int gkv_pool_retain_block(gkv_pool* pool, int32_t block);
/* GetRefCount, PagedBlockPool.cs:285-289 (0 for out-of-range ids). */
GKV_API int gkv_pool_get_ref_count(const gkv_pool* pool, int32_t block);
/* TryFindPrefixBlock, PagedBlockPool.cs:194-220 (hash computed by the caller, as in
 * ContinuousBatchEngine.cs:232): 1 with the block id and one more reference, or 0 and -1. */
GKV_API int gkv_pool_try_find_prefix_block(gkv_pool* pool, uint64_t prefix_hash,
                                           int32_t* out_block);
/* BindPrefixBlock, PagedBlockPool.cs:225-234: GKV_EINVAL for hash 0 or an out-of-range id. */
GKV_API int gkv_pool_bind_prefix_block(gkv_pool* pool, uint64_t prefix_hash, int32_t block);
/* TryForkBlock, PagedBlockPool.cs:332-342: allocates a block and queues a device copy of
 * the first valid_tokens slots of every (layer, head) from src.  Queued copies are issued
 * as ONE batched block-copy launch by the next device call on this pool (or by
 * gkv_pool_flush_copies), always before that call's own kernels. */
GKV_API int gkv_pool_try_fork_block(gkv_pool* pool, int32_t src_block, int32_t valid_tokens,
                                    int32_t* out_block);
/* Issues the queued CoW copies now (one launch). */
GKV_API int gkv_pool_flush_copies(gkv_pool* pool, void* stream);
/* CopyBlockData, PagedBlockPool.cs:304-327, batched: for i < n copies the first
 * valid_tokens[i] slots (clamped to block_size; <= 0 skips) of every layer and head from
 * src_blocks[i] to dst_blocks[i].  Host arrays; one kernel launch.  GKV_ESTATE on a
 * metadata-only pool (PagedBlockPool.cs:306-307). */
GKV_API int gkv_block_copy(gkv_pool* pool, const int32_t* h_src_blocks,
                           const int32_t* h_dst_blocks, const int32_t* h_valid_tokens,
                           int32_t n, void* stream);
/* Store, PagedBlockPool.cs:151-161: writes one token's K [heads_kv][head_dim] and
 * V [heads_kv][v_head_dim] (device fp32) into (block, layer, slot).  Bit-exact for fp32
 * storage.  GKV_ESTATE on a metadata-only pool (PagedBlockPool.cs:126-127). */
GKV_API int gkv_pool_store(gkv_pool* pool, int32_t block, int32_t layer, int32_t slot,
                           const float* d_k, const float* d_v, void* stream);

/* ---- 2. the per-sequence page table (BlockTable) ------------------------------------ */

/* new BlockTable(pool), BlockTable.cs:23-26. */
GKV_API int gkv_table_create(gkv_pool* pool, gkv_table** out_table);
GKV_API int gkv_table_destroy(gkv_table* table);
/* AttachPrefixBlocks, BlockTable.cs:31-39 (GKV_EINVAL for token_count < 0). */
GKV_API int gkv_table_attach_prefix_blocks(gkv_table* table, const int32_t* blocks, int32_t n,
                                           int32_t token_count);
/* AppendToken, BlockTable.cs:46-80: allocates at block boundaries and CoW-forks a shared
 * partial last block; returns 1 with (block, offset) or 0 with (-1, -1) when the pool is
 * exhausted, leaving the table unchanged. */
GKV_API int gkv_table_append_token(gkv_table* table, int32_t* out_block, int32_t* out_offset);
/* GetTokenLocation, BlockTable.cs:86-91. */
GKV_API int gkv_table_get_token_location(const gkv_table* table, int32_t token_index,
                                         int32_t* out_block, int32_t* out_offset);
/* GetBlockId, BlockTable.cs:94-97: the id, or GKV_EINVAL. */
GKV_API int gkv_table_get_block_id(const gkv_table* table, int32_t block_index);
/* TokenCount / BlockCount, BlockTable.cs:18-20. */
GKV_API int gkv_table_token_count(const gkv_table* table);
GKV_API int gkv_table_block_count(const gkv_table* table);
/* AsSpan, BlockTable.cs:103: copies up to cap ids into out, returns BlockCount. */
GKV_API int gkv_table_block_ids(const gkv_table* table, int32_t* out, int32_t cap);
/* ReleaseAll, BlockTable.cs:108-116. */
GKV_API int gkv_table_release_all(gkv_table* table);

/* Compaction after evictions (the engine's evict loop, ContinuousBatchEngine.cs:498-512, frees
 * blocks wherever they sit; the reference never moves a live block).  Moves live blocks into
 * the lowest free ids: a block moves only if its reference count equals its number of
 * occurrences in the n_tables tables passed (blocks also held elsewhere stay put).  Free ids
 * are filled from the bottom with movable blocks taken from the top until the two meet, at most
 * max_moves (<= 0: no limit; the capacity cap of out_src/out_dst when those are given).  ONE
 * batched block copy (CopyBlockData of whole blocks, every layer and head, PagedBlockPool.cs:
 * 304-327) runs on `stream` after the pool's queued copy-on-write copies; reference counts and
 * prefix-cache bindings move with the blocks, the passed tables are rewritten, and the free list
 * is rebuilt so that the lowest free id pops first.  out_src/out_dst (optional) receive the
 * moves, for hosts that keep table copies of their own.  Returns the number of moves.  The
 * caller excludes every other call on this pool while it runs, and orders the kernels that read
 * the old ids before it on `stream`.  A metadata-only pool moves bookkeeping only. */
GKV_API int gkv_pool_compact(gkv_pool* pool, gkv_table* const* tables, int32_t n_tables,
                             int32_t max_moves, int32_t* out_src, int32_t* out_dst, int32_t cap,
                             void* stream);

/* ---- 3. one decode / append step ------------------------------------------------------ */

/* Sizes the pool's step workspace (device + pinned staging) once, outside the hot loop:
 * up to max_batch sequences, max_blocks_per_seq table entries each, max_tokens appended
 * tokens per step, and n_heads query heads for the decode launches.  Reference analogue:
 * the device block-table buffer of CudaPagedTransformerRunner.cs:115-120,143. */
GKV_API int gkv_step_reserve(gkv_pool* pool, int32_t max_batch, int32_t max_blocks_per_seq,
                             int32_t max_tokens, int32_t n_heads);
/* Static step layout (enable != 0), for a decode iteration captured ONCE in a CUDA graph
 * (stream capture of the caller's per-layer gkv_kv_append + gkv_paged_decode calls, across
 * all layers) and replayed every step after gkv_upload_step on the same stream -- the
 * reference's per-sequence launches and uploads of CudaPagedTransformerRunner.ForwardBatch
 * (CudaPagedTransformerRunner.cs:307-364) become one graph launch per step.  While enabled:
 *  - every upload writes one device buffer at a fixed address with a copy on the caller's
 *    stream, and the launches read the step's counts and work list from its header, so the
 *    captured launch parameters stay valid; grids are the reservation's maxima;
 *  - uploads must fit the reservation (GKV_EINVAL otherwise) and decodes use its n_heads;
 *  - gkv_kv_append appends the UPLOADED step's token count (its n_tok argument is ignored;
 *    the sources must hold max_tokens rows);
 *  - queued copy-on-write copies must be flushed (gkv_pool_flush_copies) before the captured
 *    launches run: a capturable call refuses to run with copies pending (GKV_ESTATE);
 *  - gkv_paged_prefill is refused (GKV_ESTATE); gkv_rope_append works but copies its host
 *    positions per call, so it is not capturable.
 * Requires a prior gkv_step_reserve (GKV_ESTATE otherwise).  Enabling or disabling drops the
 * uploaded step.  No reference counterpart (the reference has no CUDA graphs). */
GKV_API int gkv_step_set_static(gkv_pool* pool, int32_t enable);
/* Uploads one step's packed metadata with ONE host-to-device copy, ordered before the rest
 * of `stream`:
 *   h_block_tables [batch][max_blocks] int32 (unused entries may hold -1),
 *   h_ctx_lens     [batch] tokens each sequence attends (0 = skip, output untouched,
 *                  PagedAttentionKernel.cs:42),
 *   h_slot_mapping [n_tok] int64 slot = block * block_size + offset of each appended
 *                  token (-1 = skip).
 * Validates every referenced block id and every ctx_len <= max_blocks * block_size on the
 * host (GKV_EINVAL), then builds the split-KV work list.  Replaces the per-sequence
 * UploadBlockTable, CudaPagedTransformerRunner.cs:344,367-379.
 * The copy runs on a stream of the pool's own, into one of two device buffers used in turn,
 * once the work queued on `stream` before the PREVIOUS upload has finished; `stream` then
 * waits for it.  So the launches of a step (append, decode, prefill) belong on the stream of
 * its upload, or must be ordered before the next-but-one upload by the caller. */
GKV_API int gkv_upload_step(gkv_pool* pool, const int32_t* h_block_tables, int32_t batch,
                            int32_t max_blocks, const int32_t* h_ctx_lens,
                            const int64_t* h_slot_mapping, int32_t n_tok, void* stream);
/* Packs `batch` host tables (BlockTable.AsSpan) plus ctx_lens / slot mapping and calls
 * gkv_upload_step.  h_ctx_lens may be NULL (each table's TokenCount is used). */
GKV_API int gkv_upload_step_tables(gkv_pool* pool, gkv_table* const* tables, int32_t batch,
                                   const int32_t* h_ctx_lens, const int64_t* h_slot_mapping,
                                   int32_t n_tok, void* stream);
/* KV append (reshape-and-cache scatter) of the uploaded step's n_tok tokens:
 * d_k [n_tok][heads_kv][head_dim], d_v [n_tok][heads_kv][v_head_dim] fp32, into `layer`.
 * Replaces the per-sequence Store calls, PagedTransformerRunner.cs:634 /
 * PagedBlockPool.cs:151-161.  Bit-exact for fp32 storage, RNE for bf16. */
GKV_API int gkv_kv_append(gkv_pool* pool, int32_t layer, const float* d_k, const float* d_v,
                          int32_t n_tok, void* stream);
/* Rotary position embedding of gkv_rope_append.  Pairs (i, i + rope_dim/2) for
 * GKV_ROPE_NEOX (the half-split layout of Qwen2 / GPT-NeoX) or (2i, 2i+1) for
 * GKV_ROPE_INTERLEAVED, i < rope_dim/2; elements from rope_dim on are not rotated. */
enum { GKV_ROPE_NEOX = 0, GKV_ROPE_INTERLEAVED = 1 };
typedef struct gkv_rope_desc {
    int32_t rope_dim;              /* rotated dims per head: even, <= head_dim; 0 = head_dim      */
    int32_t style;                 /* GKV_ROPE_NEOX or GKV_ROPE_INTERLEAVED                       */
    float freq_base;               /* inv_freq[i] = freq_base^(-2i/rope_dim) when h_inv_freq = NULL */
    float mscale;                  /* multiplies the rotated q and k (YaRN mscale); 0 means 1     */
    const float* h_inv_freq;       /* [rope_dim/2] host table (the YaRN table) or NULL            */
    const float* h_freq_factors;   /* [rope_dim/2] host divisors of the frequencies, or NULL      */
} gkv_rope_desc;
/* Optional per-layer terms applied before the rotation (device pointers, NULL = absent). */
typedef struct gkv_qkv_prologue {
    const float* d_q_bias;         /* [n_heads * head_dim]     AddVector(q, QBias)                */
    const float* d_k_bias;         /* [heads_kv * head_dim]    AddVector(k, KBias)                */
    const float* d_v_bias;         /* [heads_kv * v_head_dim]  AddVector(v, VBias)                */
    const float* d_q_norm;         /* [head_dim] per-head RMSNorm weight of q (AttnQNormWeight)   */
    const float* d_k_norm;         /* [head_dim] per-head RMSNorm weight of k (AttnKNormWeight)   */
    float eps;                     /* RmsNormEps                                                  */
} gkv_qkv_prologue;
/* The steps between the q/k/v projections and Store, fused with the append, for the
 * uploaded step's n_tok tokens at h_positions[n_tok]: bias add (PagedTransformerRunner.cs:
 * 612-614), per-head RMSNorm of q and k (ApplyQkNorm, :616,713-732), rotary position embedding
 * of q and k with the inverse-frequency table and mscale (QuantKernels.RoPE, :619-631), then
 * Store of the rotated k and of v into each token's slot (:634), all in one launch.
 * d_q [n_tok][n_heads][head_dim] fp32 is rewritten in place (ready for gkv_paged_decode /
 * gkv_paged_prefill); d_k [n_tok][heads_kv][head_dim] and d_v [n_tok][heads_kv][v_head_dim]
 * fp32 are read only.  Formulas (QuantKernels' own are not in the reference tree):
 * RMSNorm y = (x * (1 / sqrt(sum(x^2) / head_dim + eps))) * w; rotation by angle pos * inv_freq[i]
 * (one fp32 multiply): (a, b) -> (a cos - b sin, b cos + a sin), times mscale.  head_dim must
 * be 32, 64, 128 or 256 (GKV_EUNSUPPORTED otherwise). */
GKV_API int gkv_rope_append(gkv_pool* pool, int32_t layer, float* d_q, const float* d_k,
                            const float* d_v, int32_t n_tok, int32_t n_heads,
                            const int32_t* h_positions, const gkv_rope_desc* rope,
                            const gkv_qkv_prologue* prologue, void* stream);
/* The inverse-frequency table gkv_rope_append uses when rope->h_inv_freq is NULL:
 * out[i] = (float)(freq_base^(-2i/rope_dim)) / h_freq_factors[i] (the divisor only when given),
 * i < rope_dim/2.  Host only. */
GKV_API int gkv_rope_inv_freq(float freq_base, int32_t rope_dim, const float* h_freq_factors,
                              float* out);
/* Split-KV GQA paged decode of the uploaded step for `layer`:
 * d_q [batch][n_heads][head_dim] fp32 -> d_out [batch][n_heads][v_head_dim] fp32.
 * out = softmax(scale * q.K^T [, sink]) . V over each sequence's ctx_len tokens, query
 * head h reading kv head h / (n_heads / heads_kv).  d_sinks: NULL or [n_heads] sink
 * logits (the reference's single sinkLogit is the all-equal case).  Replaces
 * PagedAttentionKernel.ComputeAttention, PagedAttentionKernel.cs:17-372, for a batch. */
GKV_API int gkv_paged_decode(gkv_pool* pool, int32_t layer, const float* d_q, float* d_out,
                             int32_t n_heads, float scale, const float* d_sinks, void* stream);
/* Chunked causal prefill of the uploaded step for `layer`.  Sequence b (row b of the
 * uploaded tables, ctx_lens[b] = its TokenCount with the chunk's K/V already appended) has
 * h_q_len[b] queries at positions h_q_start[b] .. h_q_start[b] + h_q_len[b] - 1; query t
 * attends keys [0, min(ctx_lens[b], h_q_start[b] + t + 1)) and a sequence with no keys
 * leaves its rows of d_out untouched.  Queries are packed by sequence in batch order:
 * d_q [sum q_len][n_heads][head_dim], q_dtype GKV_DTYPE_F32, GKV_DTYPE_BF16 or GKV_DTYPE_F16;
 * d_out [sum q_len][n_heads][v_head_dim] fp32.  Same result as one
 * PagedAttentionKernel.ComputeAttention per chunk token with pos = start + t
 * (PagedTransformerRunner.ForwardPrefillSubBatch, PagedTransformerRunner.cs:424-471).
 * bf16 and fp16 pools with head_dim = v_head_dim = 128 run on the tensor cores (tcgen05,
 * operands in the arena's type: a q of another type is rounded to it first, fp16 saturating
 * at +-65504); every other pool runs the split-KV decode kernel over one segment per query.  GKV_EINVAL when a position reaches
 * max_blocks * block_size of the upload (ComputeAttention's pos < maxSeqLen check). */
GKV_API int gkv_paged_prefill(gkv_pool* pool, int32_t layer, const void* d_q, int32_t q_dtype,
                              float* d_out, const int32_t* h_q_start, const int32_t* h_q_len,
                              int32_t n_heads, float scale, void* stream);
/* ComputeAttention for ONE sequence with the reference's argument checks
 * (PagedAttentionKernel.cs:17-42): GKV_EINVAL when max_seq_len <= 0, pos outside
 * [0, max_seq_len) or TokenCount > max_seq_len; a no-op when min(TokenCount, pos+1) == 0.
 * head_dim / v_head_dim must equal the pool's.  has_sink / sink_logit mirror
 * `float? sinkLogit`.  model_layer is accepted and unused, as in the reference. */
GKV_API int gkv_compute_attention(gkv_pool* pool, int32_t stage_layer, int32_t model_layer,
                                  int32_t pos, const float* d_q, float* d_out,
                                  const gkv_table* table, int32_t n_heads, int32_t n_heads_kv,
                                  int32_t head_dim, int32_t v_head_dim, float attn_scale,
                                  int32_t max_seq_len, int32_t has_sink, float sink_logit,
                                  void* stream);
/* One whole continuous-batching attention iteration from HOST buffers, the shape of
 * CudaPagedTransformerRunner.ForwardBatch (CudaPagedTransformerRunner.cs:307-364) for the
 * attention part: copies h_q, h_k_new, h_v_new and the packed metadata to the device,
 * appends the new tokens, decodes every sequence and copies the output back to h_out.
 * Consecutive calls overlap: the host-to-device copies of a call and the device-to-host
 * copy of the previous one run on the pool's own copy streams while `stream` computes.  The
 * compute is enqueued on `stream`, which also waits for the previous call's output copy;
 * call gkv_sync(pool, stream, ...) before reading h_out or reusing the host inputs. */
GKV_API int gkv_decode_step_host(gkv_pool* pool, int32_t layer, const int32_t* h_block_tables,
                                 int32_t batch, int32_t max_blocks, const int32_t* h_ctx_lens,
                                 const int64_t* h_slot_mapping, int32_t n_tok,
                                 const float* h_k_new, const float* h_v_new, const float* h_q,
                                 float* h_out, int32_t n_heads, float scale,
                                 const float* d_sinks, void* stream);
/* Makes `stream` wait (on the device, without blocking the host) for the device-to-host output
 * copies of every gkv_decode_step_host call made on this pool so far, so that an event recorded
 * on `stream` afterwards marks every h_out as written.  The reference's ForwardBatch returns
 * with its logits on the host (CudaPagedTransformerRunner.cs:307-364); this is the
 * asynchronous form of that guarantee. */
GKV_API int gkv_wait_host_outputs(gkv_pool* pool, void* stream);
/* A KV arena described by raw device pointers, in the same layout and meaning as a pool's
 * (gkv_pool_kv_ptrs returns a pool's pointers). */
typedef struct gkv_arena_desc {
    void* d_k;
    void* d_v;
    int32_t total_blocks, layers, heads_kv, head_dim, v_head_dim, block_size, dtype;
} gkv_arena_desc;
/* Decode that allocates nothing.  No counterpart in the reference: it exists for callers
 * that cannot call cudaMalloc on the decode path -- hosts whose device memory belongs to
 * another allocator or to a region reserved at start-up under a hard budget, and serving
 * loops that cannot afford a call that may synchronize the device.  The caller passes the
 * arena, host block tables and context lengths (as gkv_upload_step), q and out (as
 * gkv_paged_decode); the packed tables, the work list and the split-KV partials live in one
 * fixed 16 MiB device array per GPU inside the library, held until the process exits.
 * Calls that would need more (about 4 MiB of tables and work list, 12 MiB of partials)
 * return GKV_EINVAL.  Runs on the calling thread's current device and on `stream`.  Not
 * capturable in a CUDA graph (its table upload would not be replayed): a capturing stream
 * gets GKV_ESTATE -- gkv_step_set_static is the capturable decode.  All calls on a device
 * share the array and leave their contents in it; calls whose kernels overlap on the GPU race
 * on it, so order them on one stream. */
GKV_API int gkv_paged_decode_noalloc(const gkv_arena_desc* arena, int32_t layer,
                                     const int32_t* h_block_tables, int32_t batch,
                                     int32_t max_blocks, const int32_t* h_ctx_lens,
                                     const float* d_q, float* d_out, int32_t n_heads, float scale,
                                     const float* d_sinks, void* stream);
/* Error check of gkv_paged_decode_noalloc on the calling thread's current device (no
 * counterpart in the reference; the status half of the allocation-free decode).  Waits for
 * `stream` with a bound (GKV_ETIMEDOUT after timeout_ms, < 0: no bound), then reads and clears
 * the device's error word: GKV_EDEVICE if a decode since the last check met a bad block id or
 * gave up a bounded wait (its output is then wrong), GKV_OK otherwise.  It allocates nothing.
 * The arena is read as it is: copy-on-write copies queued on a pool (gkv_pool_try_fork_block)
 * must have been issued (gkv_pool_flush_copies) on `stream` before the decode. */
GKV_API int gkv_paged_decode_noalloc_status(void* stream, int32_t timeout_ms);
/* Number of kernel launches the last gkv_kv_append / gkv_paged_decode /
 * gkv_decode_step_host / gkv_compute_attention call on this pool enqueued. */
GKV_API int gkv_pool_last_launch_count(const gkv_pool* pool);
/* Waits for `stream` with a bound: GKV_ETIMEDOUT after timeout_ms instead of hanging.  Also
 * reports GKV_EDEVICE if a kernel of this pool flagged a bad block id or an expired wait
 * since the last check (pool may be NULL to skip that check). */
GKV_API int gkv_sync(gkv_pool* pool, void* stream, int32_t timeout_ms);

/* Shape of the split-KV work list gkv_upload_step builds (diagnostics and tests). */
typedef struct gkv_plan_info {
    int64_t total_chunks;  /* chunks of <= 8 tokens over all (sequence, kv head) segments */
    int32_t n_pieces;      /* contiguous chunk ranges, one segment each                 */
    int32_t n_slots;       /* pieces that write a partial (segment split over workers)  */
    int32_t n_merge;       /* segments merged by the log-sum-exp kernel                 */
    int32_t n_workers;
    int32_t segment_cost;  /* chunks' worth of time charged to each segment in the split */
} gkv_plan_info;
/* Builds the decode work list for n_workers warp workers without touching a GPU: the
 * flattened stream of all segments, each charged segment_cost chunks for its per-piece
 * overhead ahead of its chunks, is split into n_workers equal contiguous ranges.
 * The piece arrays (cap_pieces entries each) and worker_begin (n_workers + 1) are optional;
 * pass NULL to query sizes only.  (No reference counterpart: the reference runs one
 * sequence per call, PagedTransformerRunner.cs:605-656.) */
GKV_API int gkv_plan_decode(const int32_t* ctx_lens, int32_t batch, int32_t heads_kv,
                            int32_t block_size, int32_t n_workers, gkv_plan_info* info,
                            int32_t* piece_seg, int32_t* piece_c0, int32_t* piece_c1,
                            int32_t* piece_slot, int32_t* worker_begin, int32_t cap_pieces);

/* ---- 4. multi-GPU host logic ---------------------------------------------------------- */

/* Sequence partitioning for the per-GPU pools: longest-processing-time-first bin packing
 * of ctx_lens onto n_ranks (each rank owns its pool, no collective).  out_rank[i] = rank of
 * sequence i.  Ties broken by lower index, then lower rank, so every rank computes the same
 * answer.  (No reference counterpart: the reference is single-GPU,
 * CudaPagedTransformerRunner.cs:108.) */
GKV_API int gkv_partition_lpt(const int32_t* ctx_lens, int32_t n, int32_t n_ranks,
                              int32_t* out_rank);
/* Contiguous block range [begin, end) of rank r when n_blocks table entries are split over
 * n_ranks for long-context split-KV (remainder to the lowest ranks). */
GKV_API int gkv_split_block_range(int32_t n_blocks, int32_t n_ranks, int32_t rank,
                                  int32_t* out_begin, int32_t* out_end);

/* Long-context split-KV across GPUs (no reference counterpart: the reference runs one
 * sequence on one GPU, CudaPagedTransformerRunner.cs:108).  A sequence's block table is
 * split into contiguous ranges (gkv_split_block_range); each rank uploads its range as the
 * step (ctx_len = tokens in its range) and calls gkv_paged_decode_splitkv_dist. */

/* gkv_paged_decode plus, per (sequence, query head), the natural-log softmax denominator
 * lse = ln(sum_t exp(s_t) [+ exp(sink)]) into d_lse [batch][n_heads].  Rows of sequences
 * with ctx_len 0 are left untouched in both outputs. */
GKV_API int gkv_paged_decode_lse(gkv_pool* pool, int32_t layer, const float* d_q, float* d_out,
                                 float* d_lse, int32_t n_heads, float scale, const float* d_sinks,
                                 void* stream);
/* Merges n_parts partial decodes of the same rows over disjoint token ranges:
 * d_parts = n_parts blocks of [rows][dv] outputs followed by [rows] lse (a row of lse
 * -inf contributes nothing); out[r] = sum_p exp(lse_p - LSE) out_p with
 * LSE = ln(sum_p exp(lse_p) [+ exp(sink[r % n_heads])]). */
GKV_API int gkv_lse_merge(const float* d_parts, int32_t n_parts, int32_t rows, int32_t dv,
                          const float* d_sinks, int32_t n_heads, float* d_out, void* stream);
/* NCCL communicator of the ranks that split sequences.  The 128-byte id comes from
 * gkv_comm_unique_id on one rank and reaches the others through the host's own channel.
 * Initialisation and every later NCCL wait give up after timeout_ms (< 0: never), abort the
 * communicator and return GKV_ETIMEDOUT instead of hanging. */
GKV_API int gkv_comm_unique_id(uint8_t* out_id_128);
GKV_API int gkv_comm_init(const uint8_t* unique_id_128, int32_t n_ranks, int32_t rank,
                          int32_t device, int32_t timeout_ms, gkv_comm** out_comm);
GKV_API int gkv_comm_abort(gkv_comm* comm);
GKV_API int gkv_comm_destroy(gkv_comm* comm);
/* How the communicator's split-KV decodes exchange their partials: 0 = not decided yet (the
 * first gkv_paged_decode_splitkv_dist decides, collectively), 1 = NCCL all-gather, 2 = peer
 * mailboxes over NVLink (CUDA IPC peer mappings): each rank's decode writes its block into its
 * own mailbox and every rank's merge reads all blocks with plain peer loads. */
GKV_API int gkv_comm_exchange_kind(const gkv_comm* comm);
/* This rank's share of a split-KV decode: decode of the uploaded step (this rank's block
 * ranges) with lse, exchange of (out, lse) over the ranks -- through the peer mailboxes when
 * the ranks map each other (gkv_comm_exchange_kind 2: the decode writes into this rank's own
 * mailbox, one kernel publishes an epoch flag, waits for every rank's and merges), else an NCCL
 * all-gather -- and the log-sum-exp merge (plus the optional sinks, applied once) into d_out
 * [batch][n_heads][v_head_dim] on every rank.  All ranks must call it with the same batch and
 * n_heads.  Merged rows of sequences with no tokens on any rank are 0. */
GKV_API int gkv_paged_decode_splitkv_dist(gkv_pool* pool, gkv_comm* comm, int32_t layer,
                                          const float* d_q, float* d_out, int32_t n_heads,
                                          float scale, const float* d_sinks, void* stream);

/* ---- misc ----------------------------------------------------------------------------- */
GKV_API const char* gkv_last_error(void);
/* Build identification, e.g. "glacier_kv 0.1 sm_100a". */
GKV_API const char* gkv_version(void);

#ifdef __cplusplus
}
#endif
#endif /* GLACIER_KV_H */
