/*
 * gkv_oracle.c -- CPU restatement of Glacier.Serve's paged-KV path (TEST INFRASTRUCTURE:
 * the checker of the CUDA path and the timed CPU baseline; never part of the product).
 *
 * Follows src/Glacier.Serve/Inference/PagedAttention/PagedAttentionKernel.cs and
 * PagedBlockPool.cs of the reference; see gkv_oracle.h for what is and is not pinned.
 * Build: oracle/Makefile (gcc -O3 -march=native -fopenmp), output oracle/lib/.
 */
#include "gkv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)0x7fff; /* canonical NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                                /* round half to even */
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE 754 binary16: 1 sign bit, 5 exponent bits (bias 15), 10 fraction bits.  Rounding to
 * nearest even is done on the integer significand: the bits shifted out are compared with
 * half of the last kept unit, ties going to the even result; a carry out of the fraction
 * moves into the exponent, which turns the largest finite value into infinity exactly when
 * the input rounds past it. */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const int32_t e32 = (int32_t)((u >> 23) & 0xffu);
    const uint32_t frac = u & 0x7fffffu;
    if (e32 == 0xff) return (uint16_t)(sign | (frac ? 0x7e00u : 0x7c00u)); /* NaN / inf */
    if (e32 == 0) return sign;              /* fp32 zero or subnormal: below half the fp16 minimum */
    const int32_t e16 = e32 - 127 + 15;     /* biased binary16 exponent */
    if (e16 >= 31) return (uint16_t)(sign | 0x7c00u);
    const uint32_t sig = frac | 0x800000u;  /* 24-bit significand */
    uint32_t shift, base;
    if (e16 >= 1) {                         /* normal result: keep 11 significant bits */
        shift = 13;
        base = (uint32_t)e16 << 10;
    } else {                                /* subnormal result: units of 2^-24 */
        shift = (uint32_t)(14 - e16);
        if (shift > 24) return sign;        /* below a quarter unit: rounds to zero */
        base = 0;
    }
    const uint32_t kept = (e16 >= 1) ? (frac >> shift) : (sig >> shift);
    const uint32_t rem = (e16 >= 1 ? frac : sig) & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    uint32_t r = base + kept;
    if (rem > half || (rem == half && (kept & 1u))) ++r; /* may carry into the exponent */
    return (uint16_t)(sign | r);
}

float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t frac = h & 0x3ffu;
    uint32_t u;
    if (e == 0x1f) {
        u = sign | 0x7f800000u | (frac << 13);
    } else if (e == 0) {
        /* subnormal: frac * 2^-24, exact in fp32 */
        const float v = (float)frac * 5.9604644775390625e-8f;
        memcpy(&u, &v, 4);
        u |= sign;
    } else {
        u = sign | ((e - 15 + 127) << 23) | (frac << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

void oracle_f32_to_f16_many(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_f16(src[i]);
}

/* E4M3 from its definition, like the binary16 conversion above: rounding to nearest even on the
 * integer significand, a carry moving into the exponent; results past 448 (the largest finite
 * value, S.1111.110) saturate to it, and NaN stays NaN. */
uint8_t oracle_f32_to_e4m3(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    const int32_t e32 = (int32_t)((u >> 23) & 0xffu);
    const uint32_t frac = u & 0x7fffffu;
    if (e32 == 0xff && frac) return (uint8_t)(sign | 0x7fu); /* NaN */
    if (e32 == 0xff) return (uint8_t)(sign | 0x7eu);         /* infinity saturates */
    if (e32 == 0) return sign;                               /* far below the smallest subnormal */
    const int32_t e8 = e32 - 127 + 7;                        /* biased e4m3 exponent */
    if (e8 >= 16) return (uint8_t)(sign | 0x7eu);
    const uint32_t sig = frac | 0x800000u;
    uint32_t shift, base, kept, rem;
    if (e8 >= 1) {                                           /* normal: keep 3 fraction bits */
        shift = 20;
        base = (uint32_t)e8 << 3;
        kept = frac >> shift;
        rem = frac & ((1u << shift) - 1u);
    } else {                                                 /* subnormal: units of 2^-9 */
        shift = (uint32_t)(21 - e8);
        if (shift > 24) return sign;                         /* below a quarter unit */
        base = 0;
        kept = sig >> shift;
        rem = sig & ((1u << shift) - 1u);
    }
    const uint32_t half = 1u << (shift - 1);
    uint32_t r = base + kept;
    if (rem > half || (rem == half && (kept & 1u))) ++r;     /* may carry into the exponent */
    if (r > 0x7eu) r = 0x7eu;                                /* satfinite */
    return (uint8_t)(sign | r);
}

float oracle_e4m3_to_f32(uint8_t b) {
    const float sign = (b & 0x80u) ? -1.0f : 1.0f;
    const uint32_t e = (b >> 3) & 0xfu, m = b & 7u;
    if (e == 0xf && m == 7) return NAN;
    if (e == 0) return sign * (float)m * 0.001953125f;       /* m * 2^-9 */
    return sign * ldexpf(1.0f + (float)m * 0.125f, (int)e - 7);
}

void oracle_f32_to_e4m3_many(const float* src, uint8_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_e4m3(src[i]);
}

static size_t elem_size(const oracle_geom* g) { return g->dtype == ORACLE_F32 ? 4 : (g->dtype == ORACLE_FP8 ? 1 : 2); }

/* Scale of (layer, head) of an FP8 arena (1 for every other type). */
static float kv_scale(const float* scales, const oracle_geom* g, int32_t layer, int32_t h) {
    return (g->dtype == ORACLE_FP8 && scales) ? scales[(int64_t)layer * g->heads_kv + h] : 1.0f;
}

/* Element offsets of GetKeyPtr / GetValuePtr, PagedBlockPool.cs:124-145. */
static int64_t k_off(const oracle_geom* g, int64_t blk, int64_t layer, int64_t h, int64_t slot) {
    const int64_t hs = (int64_t)g->block_size * g->head_dim;
    const int64_t ls = (int64_t)g->heads_kv * hs;
    const int64_t bs = (int64_t)g->layers * ls;
    return blk * bs + layer * ls + h * hs + slot * g->head_dim;
}

static int64_t v_off(const oracle_geom* g, int64_t blk, int64_t layer, int64_t h, int64_t slot) {
    const int64_t hs = (int64_t)g->block_size * g->v_head_dim;
    const int64_t ls = (int64_t)g->heads_kv * hs;
    const int64_t bs = (int64_t)g->layers * ls;
    return blk * bs + layer * ls + h * hs + slot * g->v_head_dim;
}

/* An element as fp32: FP8 elements are multiplied by their (layer, head) scale `sc`, every other
 * type is read exactly (sc is 1). */
static inline float load_elem(const void* base, int dtype, int64_t i, float sc) {
    if (dtype == ORACLE_BF16) return oracle_bf16_to_f32(((const uint16_t*)base)[i]);
    if (dtype == ORACLE_F16) return oracle_f16_to_f32(((const uint16_t*)base)[i]);
    if (dtype == ORACLE_FP8) return oracle_e4m3_to_f32(((const uint8_t*)base)[i]) * sc;
    return ((const float*)base)[i];
}

/* Stores v in the arena's type; FP8 stores e4m3(v * inv_sc) with inv_sc = 1 / scale. */
static inline void store_elem(void* base, int dtype, int64_t i, float v, float inv_sc) {
    if (dtype == ORACLE_BF16)
        ((uint16_t*)base)[i] = oracle_f32_to_bf16(v);
    else if (dtype == ORACLE_F16)
        ((uint16_t*)base)[i] = oracle_f32_to_f16(v);
    else if (dtype == ORACLE_FP8)
        ((uint8_t*)base)[i] = oracle_f32_to_e4m3(v * inv_sc);
    else
        ((float*)base)[i] = v;
}

int oracle_store(void* kpool, void* vpool, const oracle_geom* g, int32_t block, int32_t layer,
                 int32_t slot, const float* k, const float* v) {
    /* Store, PagedBlockPool.cs:151-161: per kv head, copy head_dim floats of K and
     * v_head_dim floats of V from the contiguous [heads_kv][dim] sources. */
    if (block < 0 || block >= g->total_blocks || layer < 0 || layer >= g->layers || slot < 0 ||
        slot >= g->block_size)
        return ORACLE_EINVAL;
    for (int32_t h = 0; h < g->heads_kv; ++h) {
        const int64_t ko = k_off(g, block, layer, h, slot);
        const int64_t vo = v_off(g, block, layer, h, slot);
        const float kinv = 1.0f / kv_scale(g->k_scale, g, layer, h);
        const float vinv = 1.0f / kv_scale(g->v_scale, g, layer, h);
        for (int32_t d = 0; d < g->head_dim; ++d)
            store_elem(kpool, g->dtype, ko + d, k[(int64_t)h * g->head_dim + d], kinv);
        for (int32_t d = 0; d < g->v_head_dim; ++d)
            store_elem(vpool, g->dtype, vo + d, v[(int64_t)h * g->v_head_dim + d], vinv);
    }
    return ORACLE_OK;
}

int oracle_copy_block_data(void* kpool, void* vpool, const oracle_geom* g, int32_t src,
                           int32_t dst, int32_t valid_tokens) {
    /* CopyBlockData, PagedBlockPool.cs:304-327: the first min(valid, block_size) slots of
     * every (layer, head), K and V. */
    if (valid_tokens <= 0) return ORACLE_OK;
    if (src < 0 || src >= g->total_blocks || dst < 0 || dst >= g->total_blocks) return ORACLE_EINVAL;
    const int32_t count = valid_tokens < g->block_size ? valid_tokens : g->block_size;
    const size_t es = elem_size(g);
    for (int32_t l = 0; l < g->layers; ++l)
        for (int32_t h = 0; h < g->heads_kv; ++h)
            for (int32_t t = 0; t < count; ++t) {
                memcpy((char*)kpool + k_off(g, dst, l, h, t) * es,
                       (const char*)kpool + k_off(g, src, l, h, t) * es, (size_t)g->head_dim * es);
                memcpy((char*)vpool + v_off(g, dst, l, h, t) * es,
                       (const char*)vpool + v_off(g, src, l, h, t) * es, (size_t)g->v_head_dim * es);
            }
    return ORACLE_OK;
}

int oracle_store_many(void* kpool, void* vpool, const oracle_geom* g, int32_t layer,
                      const int64_t* slots, int32_t n_tok, const float* k, const float* v) {
    /* The runners' per-token Store loop (PagedTransformerRunner.cs:450: pool.Store(blockId,
     * layer, offset, k, v) for each token of the chunk), with (block, offset) taken from the
     * flat slot index; negative slots are padding and skipped. */
    const int64_t kstride = (int64_t)g->heads_kv * g->head_dim;
    const int64_t vstride = (int64_t)g->heads_kv * g->v_head_dim;
    for (int32_t i = 0; i < n_tok; ++i) {
        if (slots[i] < 0) continue;
        const int rc = oracle_store(kpool, vpool, g, (int32_t)(slots[i] / g->block_size), layer,
                                    (int32_t)(slots[i] % g->block_size), k + i * kstride,
                                    v + i * vstride);
        if (rc != ORACLE_OK) return rc;
    }
    return ORACLE_OK;
}

int oracle_copy_many(void* kpool, void* vpool, const oracle_geom* g, const int32_t* src,
                     const int32_t* dst, const int32_t* valid, int32_t n) {
    /* One CopyBlockData per queued fork (TryForkBlock, PagedBlockPool.cs:332-342). */
    for (int32_t i = 0; i < n; ++i) {
        const int rc = oracle_copy_block_data(kpool, vpool, g, src[i], dst[i], valid[i]);
        if (rc != ORACLE_OK) return rc;
    }
    return ORACLE_OK;
}

/* QuantKernels.VecDotF32 (NuGet Glacier.Inference 1.7.0, called at
 * PagedAttentionKernel.cs:64): source absent.  Restated as an in-order fp32 fused
 * multiply-add chain; the reference's lane order is unpinned. */
static float vec_dot(const float* q, const void* kbase, int dtype, int64_t ko, int32_t n, float ksc) {
    float s = 0.f;
    for (int32_t i = 0; i < n; ++i) s = fmaf(q[i], load_elem(kbase, dtype, ko + i, ksc), s);
    return s;
}

/* QuantKernels.Softmax(scores, n, sinkLogit) (called at PagedAttentionKernel.cs:70): source
 * absent.  Restated as the conventional max-subtracted softmax; an attention sink takes
 * part in the max and adds exp(sink - max) to the denominator only.  Unpinned. */
static void softmax(float* s, int32_t n, int32_t has_sink, float sink) {
    float mx = -INFINITY;
    for (int32_t i = 0; i < n; ++i) mx = s[i] > mx ? s[i] : mx;
    if (has_sink && sink > mx) mx = sink;
    float sum = 0.f;
    for (int32_t i = 0; i < n; ++i) {
        s[i] = expf(s[i] - mx);
        sum += s[i];
    }
    if (has_sink) sum += expf(sink - mx);
    const float inv = 1.f / sum;
    for (int32_t i = 0; i < n; ++i) s[i] *= inv;
}

int oracle_compute_attention(const void* kpool, const void* vpool, const oracle_geom* g,
                             int32_t stage_layer, int32_t pos, const float* q, float* out,
                             const int32_t* block_ids, int32_t n_block_ids, int32_t token_count,
                             int32_t n_heads, int32_t n_heads_kv, int32_t head_dim,
                             int32_t v_head_dim, float attn_scale, float* head_scores,
                             int32_t max_seq_len, int32_t has_sink, float sink_logit,
                             int32_t n_threads) {
    /* argument checks, PagedAttentionKernel.cs:34-39 */
    if (max_seq_len <= 0) return ORACLE_EINVAL;
    if (pos < 0 || pos >= max_seq_len) return ORACLE_EINVAL;
    if (token_count > max_seq_len) return ORACLE_EINVAL;
    /* causal length, :41-42 */
    const int32_t total = token_count < pos + 1 ? token_count : pos + 1;
    if (total == 0) return ORACLE_OK;
    if (n_heads_kv <= 0 || n_heads % n_heads_kv != 0) return ORACLE_EINVAL;
    const int32_t group = n_heads / n_heads_kv; /* :44 */
    const int32_t bsz = g->block_size;          /* :45 */
    const int32_t block_count = (total + bsz - 1) / bsz; /* :46 */
    if (block_count > n_block_ids) return ORACLE_EINVAL; /* GetBlockId would throw */
    for (int32_t b = 0; b < block_count; ++b)
        if (block_ids[b] < 0 || block_ids[b] >= g->total_blocks) return ORACLE_EINVAL;

#ifdef _OPENMP
    const int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(static)
#endif
    for (int32_t h = 0; h < n_heads; ++h) { /* Parallel.For over heads, :48 */
        const int32_t hkv = h / group;      /* :50 */
        const float* qh = q + (int64_t)h * head_dim;
        float* scores = head_scores + (int64_t)h * max_seq_len;
        /* 1. Q.K^T per token through the block table, :55-67 */
        for (int32_t b = 0; b < block_count; ++b) {
            const int32_t pid = block_ids[b];
            const int32_t base = b * bsz;
            const int32_t tib = bsz < total - base ? bsz : total - base;
            for (int32_t t = 0; t < tib; ++t) {
                const float dot = vec_dot(qh, kpool, g->dtype, k_off(g, pid, stage_layer, hkv, t), head_dim,
                                          kv_scale(g->k_scale, g, stage_layer, hkv));
                scores[base + t] = dot * attn_scale;
            }
        }
        /* 2. softmax over all valid tokens, :70 */
        softmax(scores, total, has_sink, sink_logit);
        /* 3. P.V: each output lane is an independent in-order FMA chain over tokens, exactly
         * the reference's AVX-512 / AVX2 / generic accumulators, :75-117,:290-306,:326-370 */
        float* oh = out + (int64_t)h * v_head_dim;
        for (int32_t d = 0; d < v_head_dim; ++d) oh[d] = 0.f;
        for (int32_t b = 0; b < block_count; ++b) {
            const int32_t pid = block_ids[b];
            const int32_t base = b * bsz;
            const int32_t tib = bsz < total - base ? bsz : total - base;
            for (int32_t t = 0; t < tib; ++t) {
                const float w = scores[base + t];
                const int64_t vo = v_off(g, pid, stage_layer, hkv, t);
                for (int32_t d = 0; d < v_head_dim; ++d)
                    oh[d] = fmaf(w, load_elem(vpool, g->dtype, vo + d, kv_scale(g->v_scale, g, stage_layer, hkv)), oh[d]);
            }
        }
    }
    return ORACLE_OK;
}

int oracle_decode_batch(const void* kpool, const void* vpool, const oracle_geom* g,
                        int32_t layer, const int32_t* tables, int32_t batch, int32_t max_blocks,
                        const int32_t* ctx_lens, const float* q, float* out, int32_t n_heads,
                        float scale, int32_t has_sink, float sink_logit, int32_t n_threads) {
    const int32_t max_seq = max_blocks * g->block_size;
    if (max_seq <= 0) return batch > 0 ? ORACLE_EINVAL : ORACLE_OK;
    float* scratch = (float*)malloc(sizeof(float) * (size_t)n_heads * (size_t)max_seq);
    if (!scratch) return ORACLE_EINVAL;
    int rc = ORACLE_OK;
    for (int32_t b = 0; b < batch && rc == ORACLE_OK; ++b) { /* sequences serial */
        const int32_t ctx = ctx_lens[b];
        if (ctx <= 0) continue;
        rc = oracle_compute_attention(kpool, vpool, g, layer, ctx - 1,
                                      q + (int64_t)b * n_heads * g->head_dim,
                                      out + (int64_t)b * n_heads * g->v_head_dim,
                                      tables + (int64_t)b * max_blocks, max_blocks, ctx, n_heads,
                                      g->heads_kv, g->head_dim, g->v_head_dim, scale, scratch,
                                      max_seq, has_sink, sink_logit, n_threads);
    }
    free(scratch);
    return rc;
}

int oracle_decode_batch_parallel(const void* kpool, const void* vpool, const oracle_geom* g,
                                 int32_t layer, const int32_t* tables, int32_t batch,
                                 int32_t max_blocks, const int32_t* ctx_lens, const float* q,
                                 float* out, int32_t n_heads, float scale, int32_t n_threads) {
    /* Same arithmetic as oracle_compute_attention, scheduled over (sequence, head) pairs. */
    const int32_t max_seq = max_blocks * g->block_size;
    const int32_t group = n_heads / g->heads_kv;
    const int32_t bsz = g->block_size;
    int bad = 0;
#ifdef _OPENMP
    const int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
#pragma omp parallel num_threads(nt) reduction(| : bad)
#endif
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)(max_seq > 0 ? max_seq : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t bh = 0; bh < (int64_t)batch * n_heads; ++bh) {
            const int32_t b = (int32_t)(bh / n_heads);
            const int32_t h = (int32_t)(bh % n_heads);
            const int32_t total = ctx_lens[b];
            if (total <= 0 || !scores) continue;
            const int32_t* ids = tables + (int64_t)b * max_blocks;
            const int32_t hkv = h / group;
            const float* qh = q + ((int64_t)b * n_heads + h) * g->head_dim;
            const int32_t block_count = (total + bsz - 1) / bsz;
            if (block_count > max_blocks) { bad = 1; continue; }
            for (int32_t bb = 0; bb < block_count; ++bb) {
                const int32_t base = bb * bsz;
                const int32_t tib = bsz < total - base ? bsz : total - base;
                for (int32_t t = 0; t < tib; ++t)
                    scores[base + t] = vec_dot(qh, kpool, g->dtype, k_off(g, ids[bb], layer, hkv, t), g->head_dim,
                                               kv_scale(g->k_scale, g, layer, hkv)) * scale;
            }
            softmax(scores, total, 0, 0.f);
            float* oh = out + ((int64_t)b * n_heads + h) * g->v_head_dim;
            for (int32_t d = 0; d < g->v_head_dim; ++d) oh[d] = 0.f;
            for (int32_t bb = 0; bb < block_count; ++bb) {
                const int32_t base = bb * bsz;
                const int32_t tib = bsz < total - base ? bsz : total - base;
                for (int32_t t = 0; t < tib; ++t) {
                    const float w = scores[base + t];
                    const int64_t vo = v_off(g, ids[bb], layer, hkv, t);
                    for (int32_t d = 0; d < g->v_head_dim; ++d)
                        oh[d] = fmaf(w, load_elem(vpool, g->dtype, vo + d, kv_scale(g->v_scale, g, layer, hkv)), oh[d]);
                }
            }
        }
        free(scores);
    }
    return bad ? ORACLE_EINVAL : ORACLE_OK;
}

int oracle_prefill_chunk(const void* kpool, const void* vpool, const oracle_geom* g,
                         int32_t layer, const int32_t* block_ids, int32_t n_block_ids,
                         int32_t token_count, int32_t start_pos, int32_t n_q, const float* q,
                         float* out, int32_t n_heads, float scale, int32_t n_threads) {
    /* ForwardPrefillSubBatch, PagedTransformerRunner.cs:454-471: one ComputeAttention per
     * chunk token with pos = chunkStart + t; the causal mask is min(TokenCount, pos + 1). */
    const int32_t max_seq = n_block_ids * g->block_size;
    float* scratch = (float*)malloc(sizeof(float) * (size_t)n_heads * (size_t)(max_seq > 0 ? max_seq : 1));
    if (!scratch) return ORACLE_EINVAL;
    int rc = ORACLE_OK;
    for (int32_t t = 0; t < n_q && rc == ORACLE_OK; ++t)
        rc = oracle_compute_attention(kpool, vpool, g, layer, start_pos + t,
                                      q + (int64_t)t * n_heads * g->head_dim,
                                      out + (int64_t)t * n_heads * g->v_head_dim, block_ids,
                                      n_block_ids, token_count, n_heads, g->heads_kv, g->head_dim,
                                      g->v_head_dim, scale, scratch, max_seq, 0, 0.f, n_threads);
    free(scratch);
    return rc;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- the per-token prologue before Store: bias, QK RMSNorm, RoPE ---------------------------
 * PagedTransformerRunner.ForwardBatch (PagedTransformerRunner.cs:612-634) runs, per sequence:
 * AddVector of the q/k/v biases (:612-614, AddVector :735-752), ApplyQkNorm (per-head RMSNorm of
 * q and k, :616 / :713-732), QuantKernels.RoPE with the YaRN inverse-frequency table and mscale
 * (:619-631), then pool.Store of k and v (:634).  QuantKernels.RMSNorm and QuantKernels.RoPE
 * live in the un-vendored NuGet Glacier.Inference 1.7.0: their exact formulas are UNPINNED and
 * restated here as stated below; the CUDA kernel computes the same operations in the same order,
 * so slot contents agree bit for bit. */

/* sin and cos of a float angle: Cody-Waite reduction by pi/2 in double precision (pi/2 split
 * into two doubles, fused multiply-adds), then Taylor polynomials of sin and cos on
 * |x| <= pi/4 in float (Horner, fused multiply-adds; truncation error below 2^-28). */
void oracle_sincos(float theta, float* s_out, float* c_out) {
    const double t = (double)theta;
    const double k = rint(t * 0.63661977236758134308);            /* 2/pi */
    double r = fma(-k, 1.5707963267948966192, t);                  /* pi/2, high part */
    r = fma(-k, 6.1232339957367660359e-17, r);                     /* pi/2, low part */
    const float x = (float)r;
    const float x2 = x * x;
    /* sin x = x + x^3 (-1/3! + x^2 (1/5! + x^2 (-1/7! + x^2 (1/9! - x^2/11!)))) */
    float ps = fmaf(x2, -2.5052108385441720e-8f, 2.7557319223985893e-6f);
    ps = fmaf(x2, ps, -1.9841269841269841e-4f);
    ps = fmaf(x2, ps, 8.3333333333333333e-3f);
    ps = fmaf(x2, ps, -1.6666666666666667e-1f);
    const float sn = fmaf(x * x2, ps, x);
    /* cos x = 1 + x^2 (-1/2! + x^2 (1/4! + x^2 (-1/6! + x^2 (1/8! - x^2/10!)))) */
    float pc = fmaf(x2, -2.7557319223985891e-7f, 2.4801587301587302e-5f);
    pc = fmaf(x2, pc, -1.3888888888888889e-3f);
    pc = fmaf(x2, pc, 4.1666666666666667e-2f);
    pc = fmaf(x2, pc, -0.5f);
    const float cs = fmaf(x2, pc, 1.0f);
    switch (((long long)k) & 3) {
        case 0: *s_out = sn; *c_out = cs; break;
        case 1: *s_out = cs; *c_out = -sn; break;
        case 2: *s_out = -sn; *c_out = -cs; break;
        default: *s_out = -cs; *c_out = sn; break;
    }
}

/* RMSNorm of one head row of length n = 32*E (E elements per lane of a 32-lane group): lane l
 * sums the squares of its elements [l*E, (l+1)*E) in order (first x*x, then fused multiply-adds),
 * the 32 partial sums are combined by a butterfly (lane l adds lane l^16's sum, then l^8, l^4,
 * l^2, l^1); then r = sqrt(sum * (1/n) + eps) (n a power of two: 1/n is exact), inv = 1 / r and
 * y_i = (x_i * inv) * w_i, each step rounded. */
static void rmsnorm_row(float* x, const float* w, int32_t n, float eps) {
    const int32_t E = n / 32;
    float part[32];
    for (int l = 0; l < 32; ++l) {
        float p = x[l * E] * x[l * E];
        for (int32_t e = 1; e < E; ++e) p = fmaf(x[l * E + e], x[l * E + e], p);
        part[l] = p;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ off];
        memcpy(part, nxt, sizeof(part));
    }
    const float r = sqrtf(part[0] * (1.0f / (float)n) + eps);
    const float inv = 1.0f / r;
    for (int32_t i = 0; i < n; ++i) x[i] = (x[i] * inv) * w[i];
}

/* Rotation of one head row by position pos: pairs (i, i + R/2) (style 0, NEOX) or (2i, 2i+1)
 * (style 1, interleaved) for i < R/2, angle pos * inv_freq[i] (one float multiply), then every
 * rotated element times mscale; elements from R on pass through. */
static void rope_row(float* x, int32_t pos, const float* inv_freq, int32_t R, int32_t style, float mscale) {
    for (int32_t i = 0; i < R / 2; ++i) {
        const int32_t a = style == 0 ? i : 2 * i;
        const int32_t b = style == 0 ? i + R / 2 : 2 * i + 1;
        float s, c;
        oracle_sincos((float)pos * inv_freq[i], &s, &c);
        const float x0 = x[a], x1 = x[b];
        const float y0 = fmaf(x0, c, -(x1 * s));
        const float y1 = fmaf(x1, c, x0 * s);
        x[a] = y0 * mscale;
        x[b] = y1 * mscale;
    }
}

int oracle_rope_append(void* kpool, void* vpool, const oracle_geom* g, int32_t layer, float* q,
                       const float* k, const float* v, int32_t n_tok, int32_t n_heads,
                       const int32_t* positions, const int64_t* slots, const float* inv_freq,
                       int32_t rope_dim, int32_t style, float mscale, const float* q_bias,
                       const float* k_bias, const float* v_bias, const float* q_norm,
                       const float* k_norm, float eps) {
    const int32_t d = g->head_dim, dv = g->v_head_dim, hkv = g->heads_kv;
    if (d % 32 != 0 || rope_dim < 0 || rope_dim > d || rope_dim % 2 != 0) return ORACLE_EINVAL;
    float* kr = (float*)malloc(sizeof(float) * (size_t)hkv * (size_t)d);
    float* vr = (float*)malloc(sizeof(float) * (size_t)hkv * (size_t)dv);
    if (!kr || !vr) {
        free(kr);
        free(vr);
        return ORACLE_EINVAL;
    }
    int rc = ORACLE_OK;
    for (int32_t t = 0; t < n_tok && rc == ORACLE_OK; ++t) {
        float* qt = q + (int64_t)t * n_heads * d;
        memcpy(kr, k + (int64_t)t * hkv * d, sizeof(float) * (size_t)hkv * (size_t)d);
        memcpy(vr, v + (int64_t)t * hkv * dv, sizeof(float) * (size_t)hkv * (size_t)dv);
        /* AddVector, :612-614 */
        if (q_bias) for (int32_t i = 0; i < n_heads * d; ++i) qt[i] = qt[i] + q_bias[i];
        if (k_bias) for (int32_t i = 0; i < hkv * d; ++i) kr[i] = kr[i] + k_bias[i];
        if (v_bias) for (int32_t i = 0; i < hkv * dv; ++i) vr[i] = vr[i] + v_bias[i];
        /* ApplyQkNorm, :713-732 */
        if (q_norm) for (int32_t h = 0; h < n_heads; ++h) rmsnorm_row(qt + (int64_t)h * d, q_norm, d, eps);
        if (k_norm) for (int32_t h = 0; h < hkv; ++h) rmsnorm_row(kr + (int64_t)h * d, k_norm, d, eps);
        /* QuantKernels.RoPE, :619-631 */
        for (int32_t h = 0; h < n_heads; ++h) rope_row(qt + (int64_t)h * d, positions[t], inv_freq, rope_dim, style, mscale);
        for (int32_t h = 0; h < hkv; ++h) rope_row(kr + (int64_t)h * d, positions[t], inv_freq, rope_dim, style, mscale);
        /* pool.Store, :634 */
        if (slots[t] >= 0)
            rc = oracle_store(kpool, vpool, g, (int32_t)(slots[t] / g->block_size), layer,
                              (int32_t)(slots[t] % g->block_size), kr, vr);
    }
    free(kr);
    free(vr);
    return rc;
}
