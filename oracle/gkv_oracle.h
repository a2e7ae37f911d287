/*
 * gkv_oracle.h -- CPU restatement of Glacier.Serve's paged-KV path.  TEST INFRASTRUCTURE
 * ONLY: it is the checker of the CUDA path (tests/, __graft_entry__.smoke()) and the timed
 * CPU baseline of bench.py.  The product library (libglacier_kv.so) never links or calls it.
 *
 * Every function follows a reference member, cited as path:line inside the Glacier.Serve
 * repository (src/Glacier.Serve/Inference/PagedAttention/...).
 *
 * Parity pinning: the reference is C# on .NET 10 and its arithmetic helpers
 * (QuantKernels.VecDotF32, QuantKernels.Softmax) live in the NuGet package
 * Glacier.Inference 1.7.0, which is not vendored; nothing here can run the reference.  The
 * oracle is pinned against every value the reference's own tests fix (the closed-form
 * ComputeAttention case of PagedAttentionTests.cs:112-179, the Store/retrieve values of
 * PagedAttentionTests.cs:82-109, the CoW sentinel values of PrefixHashKvCacheTests.cs:
 * 135-182 and PrefixHashKvCacheAdversarialTests.cs:43-107, the bounds errors of
 * PhaseCServeRemediationTests.cs:117-174).  The summation order inside VecDotF32 and the
 * exact Softmax formula are NOT pinned (no test fixes them); the choices are stated below.
 */
#ifndef GKV_ORACLE_H
#define GKV_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_F32 = 0, ORACLE_BF16 = 1, ORACLE_F16 = 2, ORACLE_FP8 = 3 };
enum { ORACLE_OK = 0, ORACLE_EINVAL = -1 };

/* Geometry of a host copy of the arena, layout [block][layer][head_kv][slot][dim]
 * (PagedBlockPool.cs:77-83,124-145). */
typedef struct oracle_geom {
    int32_t total_blocks, layers, heads_kv, head_dim, v_head_dim, block_size, dtype;
    /* FP8 arenas: the K and V scales per (layer, kv head), [layers][heads_kv]; NULL means 1.
     * An element stores e4m3(x * (1 / scale)) and reads back as e4m3 * scale. */
    const float* k_scale;
    const float* v_scale;
} oracle_geom;

/* fp32 -> bf16 round to nearest even (storage rounding of the bf16 arena). */
uint16_t oracle_f32_to_bf16(float f);
float oracle_bf16_to_f32(uint16_t h);
/* fp32 -> IEEE binary16 round to nearest even, overflow to infinity, subnormal results kept,
 * NaN -> 0x7e00 (storage rounding of the fp16 arena, the reference GPU pools' precision,
 * CudaPagedTransformerRunner.cs:118-119,139), and back (exact). */
uint16_t oracle_f32_to_f16(float f);
float oracle_f16_to_f32(uint16_t h);
void oracle_f32_to_f16_many(const float* src, uint16_t* dst, int64_t n);
/* fp32 -> OCP FP8 E4M3 (1 sign, 4 exponent bits with bias 7, 3 fraction bits, no infinities,
 * S.1111.111 = NaN), round to nearest even, saturating at +-448 (satfinite); and back (exact). */
uint8_t oracle_f32_to_e4m3(float f);
float oracle_e4m3_to_f32(uint8_t b);
void oracle_f32_to_e4m3_many(const float* src, uint8_t* dst, int64_t n);

/* PagedBlockPool.Store, PagedBlockPool.cs:151-161. */
int oracle_store(void* kpool, void* vpool, const oracle_geom* g, int32_t block, int32_t layer,
                 int32_t slot, const float* k, const float* v);

/* PagedBlockPool.CopyBlockData, PagedBlockPool.cs:304-327. */
int oracle_copy_block_data(void* kpool, void* vpool, const oracle_geom* g, int32_t src,
                           int32_t dst, int32_t valid_tokens);

/* The runners' per-token Store loop (PagedTransformerRunner.cs:450) over flat slot indices
 * (slot = block * block_size + offset; negative = padding); k, v are [n_tok][heads][dim]. */
int oracle_store_many(void* kpool, void* vpool, const oracle_geom* g, int32_t layer,
                      const int64_t* slots, int32_t n_tok, const float* k, const float* v);

/* CopyBlockData for each of n (src, dst, valid) forks. */
int oracle_copy_many(void* kpool, void* vpool, const oracle_geom* g, const int32_t* src,
                     const int32_t* dst, const int32_t* valid, int32_t n);

/* PagedAttentionKernel.ComputeAttention, PagedAttentionKernel.cs:17-372, for one sequence
 * whose table holds n_block_ids ids and token_count tokens.  head_scores: scratch of
 * n_heads * max_seq_len floats (the reference's headScores).  n_threads <= 0 uses OpenMP's
 * default.  Returns ORACLE_EINVAL where the reference throws ArgumentOutOfRangeException. */
int oracle_compute_attention(const void* kpool, const void* vpool, const oracle_geom* g,
                             int32_t stage_layer, int32_t pos, const float* q, float* out,
                             const int32_t* block_ids, int32_t n_block_ids, int32_t token_count,
                             int32_t n_heads, int32_t n_heads_kv, int32_t head_dim,
                             int32_t v_head_dim, float attn_scale, float* head_scores,
                             int32_t max_seq_len, int32_t has_sink, float sink_logit,
                             int32_t n_threads);

/* The batched decode the runners perform (PagedTransformerRunner.cs:605-656): sequences in
 * order, ComputeAttention per sequence with pos = ctx_lens[b] - 1 over tables[b][...]
 * (max_blocks entries per row) and token_count = ctx_lens[b].  q [batch][n_heads][d],
 * out [batch][n_heads][dv].  Sequences with ctx 0 leave out untouched. */
int oracle_decode_batch(const void* kpool, const void* vpool, const oracle_geom* g,
                        int32_t layer, const int32_t* tables, int32_t batch, int32_t max_blocks,
                        const int32_t* ctx_lens, const float* q, float* out, int32_t n_heads,
                        float scale, int32_t has_sink, float sink_logit, int32_t n_threads);

/* Same work spread over (sequence x head) with all threads: the "best-effort" CPU variant. */
int oracle_decode_batch_parallel(const void* kpool, const void* vpool, const oracle_geom* g,
                                 int32_t layer, const int32_t* tables, int32_t batch,
                                 int32_t max_blocks, const int32_t* ctx_lens, const float* q,
                                 float* out, int32_t n_heads, float scale, int32_t n_threads);

/* Causal chunked prefill as the CPU runner does it (PagedTransformerRunner.cs:424-471):
 * for t in [0, n_q): ComputeAttention(pos = start_pos + t) over a table holding
 * token_count tokens (prefix + chunk, all stored first).  q [n_q][n_heads][d],
 * out [n_q][n_heads][dv]. */
int oracle_prefill_chunk(const void* kpool, const void* vpool, const oracle_geom* g,
                         int32_t layer, const int32_t* block_ids, int32_t n_block_ids,
                         int32_t token_count, int32_t start_pos, int32_t n_q, const float* q,
                         float* out, int32_t n_heads, float scale, int32_t n_threads);

int oracle_max_threads(void);

/* sin and cos of a float angle (Cody-Waite reduction in double, Taylor polynomials in float). */
void oracle_sincos(float theta, float* s_out, float* c_out);
/* Bias add, per-head RMSNorm of q and k, RoPE of q and k, then Store of the rotated k and v at
 * slots[t] (< 0: skipped); q is rewritten in place.  PagedTransformerRunner.cs:612-634. */
int oracle_rope_append(void* kpool, void* vpool, const oracle_geom* g, int32_t layer, float* q,
                       const float* k, const float* v, int32_t n_tok, int32_t n_heads,
                       const int32_t* positions, const int64_t* slots, const float* inv_freq,
                       int32_t rope_dim, int32_t style, float mscale, const float* q_bias,
                       const float* k_bias, const float* v_bias, const float* q_norm,
                       const float* k_norm, float eps);

#ifdef __cplusplus
}
#endif
#endif
