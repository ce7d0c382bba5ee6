/*
 * CPU oracle for the cottus-runtime decode hot path (restatement in C99).
 *
 * TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py as the checker.  Never linked into, loaded by
 * or called from the product library.  See oracle.h for the contract and the
 * reference citations.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

float oracle_fp16_to_fp32(uint16_t h) {
    /* paged_attention_cpu.cpp:10-22 */
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h & 0x7C00u) >> 10;
    uint32_t m = (uint32_t)h & 0x03FFu;
    if (e == 0) return 0.0f;
    uint32_t bits = sign | ((e - 15u + 127u) << 23) | (m << 13);
    float r;
    memcpy(&r, &bits, sizeof r);
    return r;
}

uint16_t oracle_fp32_to_fp16_trunc(float f) {
    /* generic_transformer.cpp:255-262 */
    uint32_t bits;
    memcpy(&bits, &f, sizeof bits);
    uint32_t sign = (bits & 0x80000000u) >> 16;
    int32_t e = (int32_t)((bits & 0x7F800000u) >> 23) - 127 + 15;
    uint32_t m = (bits & 0x007FFFFFu) >> 13;
    if (e <= 0) return (uint16_t)sign;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | m);
}

int64_t oracle_kv_offset(int64_t block, int32_t layer, int32_t kv, int32_t token, int32_t kv_head,
                         int32_t d, int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                         int32_t num_layers) {
    /* paged_attention_cpu.cpp:45-46,63-67,88-92 with int64 arithmetic */
    int64_t per_layer_kv = (int64_t)block_size * num_kv_heads * head_dim;
    int64_t per_block = 2 * per_layer_kv * num_layers;
    return block * per_block + (int64_t)layer * 2 * per_layer_kv + (int64_t)kv * per_layer_kv +
           (int64_t)token * num_kv_heads * head_dim + (int64_t)kv_head * head_dim + d;
}

int oracle_paged_attention(float *out, const float *query, const uint16_t *kv,
                           const int32_t *block_table, int32_t num_table_blocks, int32_t seq_len,
                           int32_t layer, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, int32_t num_layers) {
    /* argument checks in the order of paged_attention_cpu.cpp:37-41 */
    if (seq_len <= 0) return ORACLE_INVALID_ARGUMENT;
    if (layer < 0) return ORACLE_INVALID_ARGUMENT;
    if (num_heads <= 0 || num_kv_heads <= 0) return ORACLE_INVALID_ARGUMENT;
    if (head_dim <= 0) return ORACLE_INVALID_ARGUMENT;
    if (block_size <= 0) return ORACLE_INVALID_ARGUMENT;

    const int64_t per_layer_kv = (int64_t)block_size * num_kv_heads * head_dim;
    const int64_t per_block = 2 * per_layer_kv * num_layers;
    const int64_t layer_off = (int64_t)layer * 2 * per_layer_kv;

    float *acc = (float *)malloc(sizeof(float) * (size_t)head_dim);
    float *scores = (float *)malloc(sizeof(float) * (size_t)seq_len);
    if (!acc || !scores) {
        free(acc);
        free(scores);
        return ORACLE_RUNTIME_ERROR;
    }
    for (int32_t qh = 0; qh < num_heads; ++qh) {
        /* GQA map: paged_attention_cpu.cpp:48 */
        int32_t kvh = (qh * num_kv_heads) / num_heads;
        for (int32_t d = 0; d < head_dim; ++d) acc[d] = 0.0f;
        float sum_exp = 0.0f;
        float max_score = -INFINITY;
        /* pass 1: scores and running max (paged_attention_cpu.cpp:53-80) */
        for (int32_t t = 0; t < seq_len; ++t) {
            int32_t lb = t / block_size;
            int32_t tib = t % block_size;
            if (lb >= num_table_blocks) {
                free(acc);
                free(scores);
                return ORACLE_OUT_OF_RANGE;
            }
            int64_t blk = block_table[lb];
            int64_t koff = blk * per_block + layer_off + (int64_t)tib * num_kv_heads * head_dim +
                           (int64_t)kvh * head_dim;
            float qk = 0.0f;
            for (int32_t d = 0; d < head_dim; ++d) {
                float qv = query[(int64_t)qh * head_dim + d];
                float kval = oracle_fp16_to_fp32(kv[koff + d]);
                qk += qv * kval;
            }
            float scale = 1.0f / sqrtf((float)head_dim);
            qk *= scale;
            scores[t] = qk;
            if (qk > max_score) max_score = qk;
        }
        /* pass 2: exp, sum and value accumulation (paged_attention_cpu.cpp:81-98) */
        for (int32_t t = 0; t < seq_len; ++t) {
            float qk = scores[t];
            float e = expf(qk - max_score);
            sum_exp += e;
            int32_t lb = t / block_size;
            int32_t tib = t % block_size;
            int64_t blk = block_table[lb];
            int64_t voff = blk * per_block + layer_off + per_layer_kv +
                           (int64_t)tib * num_kv_heads * head_dim + (int64_t)kvh * head_dim;
            for (int32_t d = 0; d < head_dim; ++d) {
                float vv = oracle_fp16_to_fp32(kv[voff + d]);
                acc[d] += e * vv;
            }
        }
        /* normalisation (paged_attention_cpu.cpp:99-101) */
        for (int32_t d = 0; d < head_dim; ++d) out[(int64_t)qh * head_dim + d] = acc[d] / sum_exp;
    }
    free(acc);
    free(scores);
    return ORACLE_OK;
}

int oracle_paged_attention_batch(float *out, const float *query, const uint16_t *kv,
                                 const int32_t *block_table, int32_t max_blocks,
                                 const int32_t *context_lens, int32_t batch, int32_t layer,
                                 int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t block_size, int32_t num_layers) {
    const int64_t stride = (int64_t)num_heads * head_dim;
    for (int32_t b = 0; b < batch; ++b) {
        float *o = out + b * stride;
        if (context_lens[b] == 0) {
            for (int64_t i = 0; i < stride; ++i) o[i] = 0.0f;
            continue;
        }
        int rc = oracle_paged_attention(o, query + b * stride, kv, block_table + (int64_t)b * max_blocks,
                                        max_blocks, context_lens[b], layer, num_heads, num_kv_heads,
                                        head_dim, block_size, num_layers);
        if (rc != ORACLE_OK) return rc;
    }
    return ORACLE_OK;
}

/* compute_primitives_cpu.cpp:6-23 (gemmCPU): C[m][n] = sum over k, in
 * increasing k, of A[m][k] * B[k][n], each product rounded to float and
 * added in float (the file is compiled without contraction). */
void oracle_gemm(float *c, const float *a, const float *b, int32_t m, int32_t n, int32_t k) {
    for (int32_t i = 0; i < m; ++i)
        for (int32_t j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int32_t t = 0; t < k; ++t) sum += a[(size_t)i * k + t] * b[(size_t)t * n + j];
            c[(size_t)i * n + j] = sum;
        }
}

void oracle_rope_cos_sin(int32_t pos, int32_t pair, int32_t head_dim, float theta, float *cos_out,
                         float *sin_out) {
    /* compute_primitives_cpu.cpp:54-57: float pow/cos/sin of float arguments */
    float freq = 1.0f / powf(theta, (2.0f * (float)pair) / (float)head_dim);
    float angle = (float)pos * freq;
    *cos_out = cosf(angle);
    *sin_out = sinf(angle);
}

void oracle_rope(float *out, const float *in, int32_t pos, int32_t num_heads, int32_t head_dim,
                 float theta) {
    /* compute_primitives_cpu.cpp:46-73 */
    for (int32_t h = 0; h < num_heads; ++h) {
        for (int32_t d = 0; d < head_dim / 2; ++d) {
            float c, s;
            oracle_rope_cos_sin(pos, d, head_dim, theta, &c, &s);
            int64_t i0 = (int64_t)h * head_dim + 2 * d;
            int64_t i1 = i0 + 1;
            float x0 = in[i0];
            float x1 = in[i1];
            out[i0] = x0 * c - x1 * s;
            out[i1] = x0 * s + x1 * c;
        }
    }
}

int oracle_kv_append(uint16_t *kv, const float *k, const float *v, const int32_t *block_table,
                     int32_t num_table_blocks, int32_t pos, int32_t layer, int32_t num_kv_heads,
                     int32_t head_dim, int32_t block_size, int32_t num_layers) {
    /* generic_transformer.cpp:221-233 (slot) and :248-284 (encode + scatter) */
    if (pos < 0) return ORACLE_OUT_OF_RANGE;
    int32_t lb = pos / block_size;
    int32_t tib = pos % block_size;
    if (lb >= num_table_blocks) return ORACLE_OUT_OF_RANGE;
    int64_t blk = block_table[lb];
    for (int32_t h = 0; h < num_kv_heads; ++h) {
        for (int32_t d = 0; d < head_dim; ++d) {
            int64_t ko = oracle_kv_offset(blk, layer, 0, tib, h, d, block_size, num_kv_heads,
                                          head_dim, num_layers);
            kv[ko] = oracle_fp32_to_fp16_trunc(k[(int64_t)h * head_dim + d]);
        }
    }
    for (int32_t h = 0; h < num_kv_heads; ++h) {
        for (int32_t d = 0; d < head_dim; ++d) {
            int64_t vo = oracle_kv_offset(blk, layer, 1, tib, h, d, block_size, num_kv_heads,
                                          head_dim, num_layers);
            kv[vo] = oracle_fp32_to_fp16_trunc(v[(int64_t)h * head_dim + d]);
        }
    }
    return ORACLE_OK;
}

int oracle_gather_kv(uint16_t *k_out, uint16_t *v_out, const uint16_t *kv, const int32_t *block_table,
                     int32_t num_table_blocks, int32_t seq_len, int32_t layer, int32_t num_kv_heads,
                     int32_t head_dim, int32_t block_size, int32_t num_layers) {
    if (seq_len < 0) return ORACLE_INVALID_ARGUMENT;
    const int64_t row = (int64_t)num_kv_heads * head_dim;
    for (int32_t t = 0; t < seq_len; ++t) {
        int32_t lb = t / block_size;
        if (lb >= num_table_blocks) return ORACLE_OUT_OF_RANGE;
        int64_t blk = block_table[lb];
        int64_t ko = oracle_kv_offset(blk, layer, 0, t % block_size, 0, 0, block_size, num_kv_heads,
                                      head_dim, num_layers);
        int64_t vo = oracle_kv_offset(blk, layer, 1, t % block_size, 0, 0, block_size, num_kv_heads,
                                      head_dim, num_layers);
        memcpy(k_out + t * row, kv + ko, sizeof(uint16_t) * (size_t)row);
        memcpy(v_out + t * row, kv + vo, sizeof(uint16_t) * (size_t)row);
    }
    return ORACLE_OK;
}

struct oracle_allocator {
    int32_t total;
    int32_t block_size;
    int32_t n_free;
    int32_t *free_list; /* stack; top = free_list[n_free-1] */
    unsigned char *allocated;
};

oracle_allocator *oracle_allocator_create(int32_t total_blocks, int32_t block_size) {
    /* block_allocator.cpp:7-19 */
    if (total_blocks <= 0 || block_size <= 0) return NULL;
    oracle_allocator *a = (oracle_allocator *)calloc(1, sizeof *a);
    if (!a) return NULL;
    a->total = total_blocks;
    a->block_size = block_size;
    a->free_list = (int32_t *)malloc(sizeof(int32_t) * (size_t)total_blocks);
    a->allocated = (unsigned char *)calloc((size_t)total_blocks, 1);
    if (!a->free_list || !a->allocated) {
        oracle_allocator_destroy(a);
        return NULL;
    }
    /* pushed in descending order so that the first pop returns 0 */
    for (int32_t i = 0; i < total_blocks; ++i) a->free_list[i] = total_blocks - 1 - i;
    a->n_free = total_blocks;
    return a;
}

void oracle_allocator_destroy(oracle_allocator *a) {
    if (!a) return;
    free(a->free_list);
    free(a->allocated);
    free(a);
}

int32_t oracle_allocator_alloc(oracle_allocator *a) {
    /* block_allocator.cpp:21-31 */
    if (a->n_free == 0) return ORACLE_RUNTIME_ERROR;
    int32_t id = a->free_list[--a->n_free];
    a->allocated[id] = 1;
    return id;
}

int oracle_allocator_free(oracle_allocator *a, int32_t block_id) {
    /* block_allocator.cpp:33-45 */
    if (block_id < 0 || block_id >= a->total) return ORACLE_INVALID_ARGUMENT;
    if (!a->allocated[block_id]) return ORACLE_RUNTIME_ERROR;
    a->allocated[block_id] = 0;
    a->free_list[a->n_free++] = block_id;
    return ORACLE_OK;
}

int32_t oracle_allocator_num_free(const oracle_allocator *a) { return a->n_free; }
