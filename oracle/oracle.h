/*
 * CPU oracle for the cottus-runtime decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker.
 *
 * Every function restates one piece of the reference's CPU behaviour in plain
 * C99 (file:line citations are relative to the cottus-runtime project root).
 * Build flags mirror the reference's Release build (-O3 -DNDEBUG, no -march,
 * -ffp-contract=off), so the fp32 arithmetic order and rounding are the same
 * as the reference's compiled code; the tests check this bit-for-bit against
 * the reference sources compiled into oracle/_ref/.
 *
 * Deliberate difference: element offsets are int64 (the reference uses
 * int32, paged_attention_cpu.cpp:45-46,63-67, which overflows for pools of
 * more than 2^31 fp16 elements).  Results are identical wherever the
 * reference does not overflow.
 */
#ifndef COTTUS_ORACLE_H
#define COTTUS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes mirror the reference's exception classes. */
#define ORACLE_OK 0
#define ORACLE_INVALID_ARGUMENT (-1) /* std::invalid_argument */
#define ORACLE_OUT_OF_RANGE (-2)     /* std::out_of_range */
#define ORACLE_RUNTIME_ERROR (-3)    /* std::runtime_error (OOM, double free) */

/* fp16 bits -> fp32: paged_attention_cpu.cpp:10-22.  exp==0 (zero and
 * subnormals) decodes to +0.0f regardless of sign; exp==31 is decoded as a
 * finite number (no inf/NaN special case). */
float oracle_fp16_to_fp32(uint16_t h);

/* fp32 -> fp16 bits by truncation: generic_transformer.cpp:255-262 (also
 * tests/test_paged_attention_cpu.cpp:11-23).  Mantissa truncated, biased
 * exponent <= 0 -> signed zero, >= 31 (incl. inf/NaN) -> signed inf. */
uint16_t oracle_fp32_to_fp16_trunc(float f);

/* Element offset of (block, layer, kv, token, kvHead, d) inside the pool:
 * layout [block][layer][K|V][blockSize][numKvHeads][headDim]
 * (paged_attention_cpu.cpp:45-46,63-67,88-92; tests/test_kv_layout_hardening.cpp:21-35). */
int64_t oracle_kv_offset(int64_t block, int32_t layer, int32_t kv, int32_t token, int32_t kv_head,
                         int32_t d, int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                         int32_t num_layers);

/* Single-sequence, single-query paged attention: paged_attention_cpu.cpp:24-103.
 * block_table[0..num_table_blocks) plays the role of PageTable.
 * query/out: fp32 [num_heads][head_dim]; kv: fp16 bits pool. */
int oracle_paged_attention(float *out, const float *query, const uint16_t *kv,
                           const int32_t *block_table, int32_t num_table_blocks, int32_t seq_len,
                           int32_t layer, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, int32_t num_layers);

/* Batched convenience: sequence b uses block_table + b*max_blocks and
 * context_lens[b].  A sequence with context length 0 gets zeros (the
 * batched product API defines that case; the reference has no batch). */
int oracle_paged_attention_batch(float *out, const float *query, const uint16_t *kv,
                                 const int32_t *block_table, int32_t max_blocks,
                                 const int32_t *context_lens, int32_t batch, int32_t layer,
                                 int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t block_size, int32_t num_layers);

/* Interleaved-pair RoPE, in place allowed: compute_primitives_cpu.cpp:46-73. */
void oracle_rope(float *out, const float *in, int32_t pos, int32_t num_heads, int32_t head_dim,
                 float theta);

/* cos/sin of the RoPE angle for one (pos, pair), evaluated with the same
 * float expressions as compute_primitives_cpu.cpp:54-57. */
void oracle_gemm(float *c, const float *a, const float *b, int32_t m, int32_t n, int32_t k);
void oracle_rope_cos_sin(int32_t pos, int32_t pair, int32_t head_dim, float theta, float *cos_out,
                         float *sin_out);

/* KV append for one token of one layer: generic_transformer.cpp:221-284.
 * k, v: fp32 [num_kv_heads][head_dim] (k already rotated). */
int oracle_kv_append(uint16_t *kv, const float *k, const float *v, const int32_t *block_table,
                     int32_t num_table_blocks, int32_t pos, int32_t layer, int32_t num_kv_heads,
                     int32_t head_dim, int32_t block_size, int32_t num_layers);

/* Dense gather of one sequence's K and V rows for one layer, in logical
 * order (the block-table walk of paged_attention_cpu.cpp:53-67,86-92):
 * k_out, v_out: fp16 bits [seq_len][num_kv_heads][head_dim]. */
int oracle_gather_kv(uint16_t *k_out, uint16_t *v_out, const uint16_t *kv, const int32_t *block_table,
                     int32_t num_table_blocks, int32_t seq_len, int32_t layer, int32_t num_kv_heads,
                     int32_t head_dim, int32_t block_size, int32_t num_layers);

/* LIFO block pool: block_allocator.cpp:7-55.  The first allocation returns
 * block 0; freed blocks are reused last-in first-out. */
typedef struct oracle_allocator oracle_allocator;
oracle_allocator *oracle_allocator_create(int32_t total_blocks, int32_t block_size);
void oracle_allocator_destroy(oracle_allocator *a);
/* Returns the block id, or ORACLE_RUNTIME_ERROR when the pool is empty. */
int32_t oracle_allocator_alloc(oracle_allocator *a);
/* Returns ORACLE_OK, ORACLE_INVALID_ARGUMENT (bad id) or ORACLE_RUNTIME_ERROR (double free). */
int oracle_allocator_free(oracle_allocator *a, int32_t block_id);
int32_t oracle_allocator_num_free(const oracle_allocator *a);

#ifdef __cplusplus
}
#endif

#endif
