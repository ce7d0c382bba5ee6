/*
 * cottus_b200 — B200 (sm_100a) decode hot path of cottus-runtime behind a C ABI.
 *
 * Paged decode attention over the BlockAllocator / PageTable fp16 KV cache,
 * the fused RoPE + KV-cache append that feeds it, the split-KV
 * log-sum-exp merge, and the host-side block pool.  Plain pointers and
 * sizes only; every device pointer is caller-owned; nothing here allocates
 * device memory per call (split-KV scratch is a caller-provided workspace).
 * Calls are stream-ordered and never synchronise the device, except the
 * host-side helpers marked "host".
 *
 * Citations are to the cottus-runtime sources (path:line from the project
 * root).
 *
 * KV pool layout (identical to the reference, paged_attention_cpu.cpp:45-46,
 * 63-67, 88-92; tests/test_kv_layout_hardening.cpp:6-35):
 *   uint16 fp16 bit patterns
 *   [num_physical_blocks][num_layers][K|V][block_size][num_kv_heads][head_dim]
 * GQA map (paged_attention_cpu.cpp:48): kv_head(h) = h * num_kv_heads / num_heads.
 */
#ifndef COTTUS_B200_H
#define COTTUS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st *cottus_stream_t;

/* Return codes.  The reference throws; the ABI never does. */
enum cottus_status {
    COTTUS_OK = 0,
    COTTUS_ERR_INVALID_ARGUMENT = -1, /* std::invalid_argument (paged_attention_cuda.cu:109-113) */
    COTTUS_ERR_OUT_OF_RANGE = -2,     /* std::out_of_range (page_table.cpp:18-26, generic_transformer.cpp:224-226) */
    COTTUS_ERR_CUDA = -3,             /* std::runtime_error("CUDA error: ...") (paged_attention_cuda.cu:8-14) */
    COTTUS_ERR_UNSUPPORTED = -4,      /* shape outside what the kernels implement */
    COTTUS_ERR_WORKSPACE = -5,        /* split-KV workspace missing or too small */
    COTTUS_ERR_OUT_OF_MEMORY = -6,    /* BlockAllocator "Out of memory" (block_allocator.cpp:23-25) */
    COTTUS_ERR_DOUBLE_FREE = -7       /* BlockAllocator "Double free detected" (block_allocator.cpp:38-40) */
};

/* Bits OR-ed into the optional device status word by the kernels.  Device
 * checks cannot throw; they zero the affected output rows and set a bit. */
#define COTTUS_STATUS_BAD_BLOCK_ID 0x1u /* block id outside [0, num_physical_blocks) */
#define COTTUS_STATUS_BAD_CONTEXT 0x2u  /* context < 0 or > max_blocks_per_seq * block_size */
#define COTTUS_STATUS_BAD_POSITION 0x4u /* position outside the table / RoPE cache */
#define COTTUS_STATUS_TIMEOUT 0x8u      /* a bounded wait inside a kernel gave up */

enum cottus_dtype { COTTUS_F32 = 0, COTTUS_F16 = 1 };

/* Message of the last error returned on this host thread (mirrors the
 * reference's exception text where one exists). */
const char *cottus_last_error(void);
const char *cottus_status_string(int status);
int cottus_version(void);

/* ------------------------------------------------------------------------
 * Batched paged decode attention.
 * Replaces cottus::pagedAttentionCUDA (paged_attention_cuda.h:9-21,
 * paged_attention_cuda.cu:96-149) and its CPU twin cottus::pagedAttentionCPU
 * (paged_attention_cpu.h:8-20): one query token per sequence, a whole batch
 * per call, device-resident pool and block table, caller's stream.
 * For each sequence b and query head h:
 *   out[b][h] = softmax(scale * q[b][h] . K_b^T) V_b over the first
 *   context_lens[b] tokens of sequence b, K_b/V_b gathered through
 *   block_table[b][:] from layer `layer` of the pool.
 * context_lens[b] == 0 writes zeros (an idle batch slot); the reference has
 * no batch and rejects seqLen <= 0.
 * ---------------------------------------------------------------------- */
typedef struct {
    void *out;                  /* [batch][num_heads][head_dim], out_dtype */
    const void *query;          /* [batch][num_heads][head_dim], q_dtype */
    const uint16_t *kv_pool;    /* fp16 bit patterns, layout above */
    const int32_t *block_table; /* [batch][max_blocks_per_seq] physical block ids */
    const int32_t *context_lens;/* [batch] tokens per sequence */
    int64_t num_physical_blocks;
    int32_t batch;
    int32_t num_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t block_size;
    int32_t num_layers;
    int32_t layer;
    int32_t max_blocks_per_seq;
    int32_t q_dtype;            /* enum cottus_dtype */
    int32_t out_dtype;          /* enum cottus_dtype */
    float scale;                /* <= 0 selects 1/sqrt(head_dim) (paged_attention_cpu.cpp:75) */
    /* Optional split-KV partial mode: when non-NULL, `out` receives the
     * normalised partial output and lse_out[b][h] its natural-log
     * log-sum-exp, for cottus_lse_combine across context shards. */
    float *lse_out;
    void *workspace;            /* >= cottus_paged_decode_workspace_size() bytes, 16-B aligned, zero-filled
                                   once after allocation (the kernels leave the words that must be zero at
                                   zero; after a call that reported COTTUS_STATUS_TIMEOUT, zero it again) */
    size_t workspace_bytes;
    uint32_t *status;           /* optional device word, COTTUS_STATUS_* bits */
} cottus_paged_decode_params;

/* Scratch bytes that cottus_paged_decode needs for these parameters on the
 * current device (independent of the context lengths).  0 means none. */
size_t cottus_paged_decode_workspace_size(const cottus_paged_decode_params *p);
int cottus_paged_decode(const cottus_paged_decode_params *p, cottus_stream_t stream);

/* Allocation-free variant of cottus_paged_decode.  No counterpart in the
 * reference.  For callers that cannot allocate device memory when attention
 * runs (code inside an allocator or memory-pool callback, engines that
 * reserve all device memory up front, plugin hosts that pass only a stream
 * and the call's tensors): instead of a caller workspace it uses a 32 MiB
 * scratch array compiled into the library, which every GPU that loads the
 * library keeps until the process exits.  p->workspace and
 * p->workspace_bytes are ignored.  Calls needing more scratch than 32 MiB
 * (see cottus_paged_decode_workspace_size) fail with COTTUS_ERR_WORKSPACE.
 * The first call on a device (and the first after a device reset) looks up
 * the array's device address; make that first call before any stream
 * capture.  Arguments are checked as cottus_paged_decode checks them before
 * anything is queued.  All calls on a device share the
 * array: calls whose executions overlap on the GPU race and must be ordered
 * by the caller.  Nothing is allocated or freed. */
int cottus_paged_decode_static_scratch(const cottus_paged_decode_params *p, cottus_stream_t stream);

/* ------------------------------------------------------------------------
 * Split-KV merge of partial (normalised output, log-sum-exp) pairs produced
 * over disjoint context shards (e.g. one per GPU):
 *   lse = log(sum_i exp(lse_i));  out = sum_i exp(lse_i - lse) * out_i.
 * No reference counterpart (the reference never splits a context); its
 * result equals the un-split cottus::pagedAttentionCPU output.
 * ---------------------------------------------------------------------- */
typedef struct {
    void *out;                /* [batch][num_heads][head_dim], out_dtype */
    float *lse_out;           /* optional [batch][num_heads] */
    const float *partial_out; /* [num_parts][batch][num_heads][head_dim] */
    const float *partial_lse; /* [num_parts][batch][num_heads]; -inf marks an empty shard */
    int32_t num_parts;
    int32_t batch;
    int32_t num_heads;
    int32_t head_dim;
    int32_t out_dtype;
} cottus_lse_combine_params;

int cottus_lse_combine(const cottus_lse_combine_params *p, cottus_stream_t stream);

/* ------------------------------------------------------------------------
 * RoPE.  Replaces cottus::ropeCUDA / ropeCPU (compute_primitives_cuda.h:22-29,
 * compute_primitives_cpu.cpp:46-73): interleaved pairs (2d, 2d+1),
 *   out0 = x0*cos - x1*sin,  out1 = x0*sin + x1*cos,
 * angle = pos / theta^(2d/head_dim).  The (cos, sin) values come from a
 * table filled on the host with the reference's float formula, and the
 * rotation is evaluated without fused multiply-adds, so results are
 * bit-identical to ropeCPU.
 * ---------------------------------------------------------------------- */

/* host: table[max_position][head_dim/2][2] = (cos, sin), reference formula. */
int cottus_rope_cos_sin_fill(float *host_table, int32_t max_position, int32_t head_dim, float theta);

/* x[num_tokens][num_heads][head_dim] fp32, in place allowed; positions[t]
 * is token t's position; cos_sin: device table from cottus_rope_cos_sin_fill. */
int cottus_rope(float *out, const float *in, const int32_t *positions, int32_t num_tokens, int32_t num_heads,
                int32_t head_dim, const float *cos_sin, int32_t max_position, cottus_stream_t stream);

/* ------------------------------------------------------------------------
 * One decode step of one layer: RoPE on the new token's q and k, KV append
 * (fp32 -> fp16 by truncation, subnormal results flushed to signed zero,
 * overflow/NaN -> signed inf; written to slot positions[b] % block_size of
 * block block_table[b][positions[b] / block_size]), optionally followed by
 * paged attention over positions[b] + 1 tokens, in one kernel.
 * Replaces generic_transformer.cpp:196-291 (ropeCUDA x2, the host-side
 * encode/scatter loop and pagedAttentionCUDA).
 * ---------------------------------------------------------------------- */
typedef struct {
    const void *query;          /* [batch][num_heads][head_dim], qkv_dtype (not yet rotated) */
    const void *key;            /* [batch][num_kv_heads][head_dim], qkv_dtype (not yet rotated) */
    const void *value;          /* [batch][num_kv_heads][head_dim], qkv_dtype */
    int32_t qkv_dtype;          /* enum cottus_dtype */
    const int32_t *positions;   /* [batch] position of the new token */
    const float *cos_sin;       /* device [max_position][head_dim/2][2]; NULL = no rotation */
    int32_t max_position;
    uint16_t *kv_pool;
    const int32_t *block_table; /* [batch][max_blocks_per_seq] */
    int64_t num_physical_blocks;
    int32_t batch;
    int32_t num_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t block_size;
    int32_t num_layers;
    int32_t layer;
    int32_t max_blocks_per_seq;
    void *query_out;            /* optional rotated query, qkv_dtype, [batch][num_heads][head_dim] */
    /* attention part (cottus_rope_append_decode only) */
    void *out;                  /* [batch][num_heads][head_dim], out_dtype */
    int32_t out_dtype;
    float scale;                /* <= 0: 1/sqrt(head_dim) */
    void *workspace;            /* as cottus_paged_decode_params.workspace */
    size_t workspace_bytes;
    uint32_t *status;           /* optional device word */
} cottus_decode_step_params;

/* RoPE + append only (no attention; `out`, `workspace` ignored). */
int cottus_rope_append(const cottus_decode_step_params *p, cottus_stream_t stream);
/* RoPE + append + paged attention over positions[b] + 1 tokens. */
size_t cottus_rope_append_decode_workspace_size(const cottus_decode_step_params *p);
int cottus_rope_append_decode(const cottus_decode_step_params *p, cottus_stream_t stream);

/* ------------------------------------------------------------------------
 * The step before attention, fused: QKV projection of each sequence's new
 * token, RoPE on q and k, and the KV append, in one call (a tensor-core
 * projection kernel writing split partials to the workspace, then an
 * epilogue kernel; stream-ordered, no host synchronisation).  Replaces
 * generic_transformer.cpp:169-284 per layer and token (gemmCUDA x3 =
 * cuBLAS SGEMM, compute_primitives_cuda.cu:30-55; ropeCUDA x2; the host
 * truncating encode and scatter).  Weights and activations are fp16 with
 * fp32 accumulation:  qkv[b][n] = sum_k x[b][k] * weight[n][k], rows n of
 * `weight` = Wq rows (num_heads*head_dim), then Wk, then Wv rows (the
 * reference's [hidden][out] matrices transposed and stacked).  Then, as
 * cottus_rope_append: q and k rotated at positions[b] with the (cos, sin)
 * table, the rotated query written to query_out, k and v encoded by
 * truncation into slot positions[b] % block_size of block
 * block_table[b][positions[b] / block_size], layer `layer`.  hidden must be
 * a multiple of 64 and the stacked row count of 128; batches above 64 run as
 * several launches.  Feed query_out to cottus_paged_decode with
 * context_lens = positions + 1 for the attention.
 * ---------------------------------------------------------------------- */
typedef struct {
    const void *x;              /* [batch][hidden] fp16, 16-B aligned */
    const void *weight;         /* [(num_heads + 2*num_kv_heads)*head_dim][hidden] fp16, 16-B aligned */
    int32_t hidden;
    const int32_t *positions;   /* [batch] */
    const float *cos_sin;       /* device [max_position][head_dim/2][2] (cottus_rope_cos_sin_fill) */
    int32_t max_position;
    uint16_t *kv_pool;
    const int32_t *block_table; /* [batch][max_blocks_per_seq] */
    int64_t num_physical_blocks;
    int32_t batch;
    int32_t num_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t block_size;
    int32_t num_layers;
    int32_t layer;
    int32_t max_blocks_per_seq;
    void *query_out;            /* [batch][num_heads][head_dim] rotated query */
    int32_t query_out_dtype;    /* enum cottus_dtype */
    float *qkv_out;             /* optional [batch][rows] fp32 projections before rotation */
    void *workspace;            /* cottus_qkv_rope_append_workspace_size() bytes, 16-B aligned, any contents
                                   (not a buffer that cottus_paged_decode relies on: it is overwritten) */
    size_t workspace_bytes;
    uint32_t *status;           /* optional device word */
} cottus_qkv_params;

size_t cottus_qkv_rope_append_workspace_size(const cottus_qkv_params *p);
int cottus_qkv_rope_append(const cottus_qkv_params *p, cottus_stream_t stream);

/* ------------------------------------------------------------------------
 * The step after attention: output projection and residual add, on the
 * same tensor-core kernel as cottus_qkv_rope_append.  Replaces
 * generic_transformer.cpp:305-325 per layer and token (gemmCUDA with wo,
 * then residualAddCUDA):  out[b][n] = (sum_k x[b][k] * weight[n][k]) +
 * residual[b][n], fp16 x and weight, fp32 accumulation and residual.
 * in_features a multiple of 64, out_features of 128.  x is typically the
 * attention output [batch][num_heads*head_dim] (fp16, cottus_paged_decode).
 * ---------------------------------------------------------------------- */
typedef struct {
    const void *x;          /* [batch][in_features] fp16, 16-B aligned */
    const void *weight;     /* [out_features][in_features] fp16 (the reference's wo [in][out] transposed) */
    int32_t in_features;
    int32_t out_features;
    int32_t batch;
    const float *residual;  /* [batch][out_features] fp32 (may equal out when out_dtype is fp32) */
    void *out;              /* [batch][out_features], out_dtype */
    int32_t out_dtype;      /* enum cottus_dtype */
    void *workspace;        /* cottus_o_proj_residual_workspace_size() bytes, 16-B aligned, any contents
                               (overwritten; not a decode workspace) */
    size_t workspace_bytes;
    uint32_t *status;       /* optional device word */
} cottus_o_proj_params;

size_t cottus_o_proj_residual_workspace_size(const cottus_o_proj_params *p);
int cottus_o_proj_residual(const cottus_o_proj_params *p, cottus_stream_t stream);

/* ------------------------------------------------------------------------
 * Block-table gather: copies, bit for bit, the K and V rows of layer
 * `layer` for the first context_lens[b] tokens of each sequence into dense
 * k_out/v_out [batch][max_context][num_kv_heads][head_dim] (fp16 bits);
 * rows past a sequence's context are left untouched.  This is the gather of
 * paged_attention_cpu.cpp:53-67,86-92 (and paged_attention_cuda.cu:131-135)
 * exposed on its own.
 * ---------------------------------------------------------------------- */
int cottus_paged_gather(uint16_t *k_out, uint16_t *v_out, const uint16_t *kv_pool, const int32_t *block_table,
                        const int32_t *context_lens, int64_t num_physical_blocks, int32_t batch,
                        int32_t max_context, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                        int32_t num_layers, int32_t layer, int32_t max_blocks_per_seq, uint32_t *status,
                        cottus_stream_t stream);

/* ------------------------------------------------------------------------
 * host: LIFO block pool, cottus::BlockAllocator (block_allocator.h:9-14,
 * block_allocator.cpp:7-55).  The first allocation returns block 0.
 * ---------------------------------------------------------------------- */
typedef struct cottus_block_allocator cottus_block_allocator;
int cottus_block_allocator_create(int32_t total_blocks, int32_t block_size, cottus_block_allocator **out);
void cottus_block_allocator_destroy(cottus_block_allocator *a);
int cottus_block_allocator_allocate(cottus_block_allocator *a, int32_t *block_id);
int cottus_block_allocator_free(cottus_block_allocator *a, int32_t block_id);
int32_t cottus_block_allocator_num_free(const cottus_block_allocator *a);
int32_t cottus_block_allocator_total_blocks(const cottus_block_allocator *a);

/* ------------------------------------------------------------------------
 * host (+ one small kernel per step): batched decode-step driver.  The block
 * bookkeeping of Engine::generate (engine.cpp:52-95: a block allocated
 * whenever a sequence's next position starts one, engine.cpp:73-77; blocks
 * returned in allocation order when the sequence ends, engine.cpp:88-90)
 * for many sequences at once, with the block table resident in device
 * memory instead of a host PageTable copied to the device on every call
 * (paged_attention_cuda.cu:125-135).
 *
 * The active sequences occupy rows 0..size-1 of a caller-owned device table
 * device_block_table[max_batch][max_blocks_per_seq] and of
 * device_positions[max_batch] (the position of each row's next token).
 * Adding a sequence appends a row at position 0; releasing one moves the
 * last row into its place (cottus_decode_batch_rows gives the order).
 * A step: cottus_decode_batch_begin_step allocates the blocks the step
 * needs and sends the changed table entries and the positions to the device
 * (one small kernel on `stream`, parameters passed by value: no device
 * scratch and no copy call); run cottus_rope_append_decode (or
 * cottus_rope_append / cottus_qkv_rope_append, then cottus_paged_decode with
 * context_lens = device_context_lens) once per layer with
 * batch = cottus_decode_batch_size(), block_table = device_block_table,
 * positions = device_positions, max_blocks_per_seq as given here; then
 * cottus_decode_batch_end_step advances every position by one.  With both
 * device pointers NULL the object keeps the host bookkeeping only.
 * Errors: COTTUS_ERR_OUT_OF_MEMORY when the pool is exhausted (the step's
 * allocations are undone; "Out of memory: no free blocks",
 * block_allocator.cpp:23-25), COTTUS_ERR_OUT_OF_RANGE when a row would pass
 * max_blocks_per_seq * block_size tokens (the reference's maxSeqLen
 * length_error, engine.cpp:43-45) or the batch is full.  Not thread-safe.
 * ---------------------------------------------------------------------- */
typedef struct cottus_decode_batch cottus_decode_batch;
typedef struct {
    int32_t num_blocks;          /* pool capacity in blocks (BlockAllocator totalBlocks) */
    int32_t block_size;
    int32_t max_batch;           /* rows of the device table */
    int32_t max_blocks_per_seq;  /* columns of the device table */
    int32_t *device_block_table; /* [max_batch][max_blocks_per_seq], or NULL (host bookkeeping only) */
    int32_t *device_positions;   /* [max_batch], or NULL */
    int32_t *device_context_lens; /* optional [max_batch]: position + 1 of each row's step token (the
                                     context_lens of a cottus_paged_decode after cottus_qkv_rope_append), or NULL */
} cottus_decode_batch_desc;

int cottus_decode_batch_create(const cottus_decode_batch_desc *desc, cottus_decode_batch **out);
void cottus_decode_batch_destroy(cottus_decode_batch *b);
/* new sequence at position 0 in the next free row (*row may be NULL) */
int cottus_decode_batch_add(cottus_decode_batch *b, int64_t seq_id, int32_t *row);
/* frees the sequence's blocks; the last row moves into its row */
int cottus_decode_batch_release(cottus_decode_batch *b, int64_t seq_id);
int cottus_decode_batch_begin_step(cottus_decode_batch *b, cottus_stream_t stream);
int cottus_decode_batch_end_step(cottus_decode_batch *b);
int32_t cottus_decode_batch_size(const cottus_decode_batch *b);
int32_t cottus_decode_batch_free_blocks(const cottus_decode_batch *b);
/* sequence ids in row order; returns the number of rows */
int cottus_decode_batch_rows(const cottus_decode_batch *b, int64_t *seq_ids, int32_t cap);
/* host mirror of one sequence: its row, next position and blocks (up to cap) */
int cottus_decode_batch_sequence(const cottus_decode_batch *b, int64_t seq_id, int32_t *row, int32_t *position,
                                 int32_t *blocks, int32_t cap, int32_t *num_blocks);

/* ------------------------------------------------------------------------
 * Split-context decode across the GPUs of one node, exchange through peer
 * memory (no collective library call).  No reference counterpart (the
 * reference never splits a context); the merged result equals the
 * un-split cottus::pagedAttentionCUDA output.
 *
 * Every rank (one process per GPU) creates an exchange for its
 * (batch, num_heads, head_dim) — one cudaMalloc at set-up, nothing per
 * call — gives its 64-byte IPC handle to every other rank (any host
 * transport), opens all handles, and then calls cottus_split_decode in
 * lockstep with the other ranks: p describes this rank's page range of
 * every sequence (its pool shard, block table and token counts); p->out
 * receives the merged output [batch][num_heads][head_dim] and p->lse_out
 * (optional) the merged natural-log LSE.  One decode kernel writes this
 * rank's partials into its exchange buffer and, once all its CTAs have
 * stored them, flags completion to every rank; then (bounded) waits until
 * every rank has flagged this step or a later one, and merges the ranks'
 * partials with peer loads over NVLink (the arithmetic of
 * cottus_lse_combine).  On the tensor-core decode path (grouped queries,
 * head_dim 64/128, block size 16) the wait and merge run in the decode
 * kernel itself; other shapes use a separate combine kernel.  At most 8
 * ranks.
 *
 * Failure detection: a rank that does not take part in a step makes the
 * others' combine give up after the wait limit (default 2e9 GPU clock
 * cycles, about a second; cottus_peer_exchange_set_wait_cycles) with
 * COTTUS_STATUS_TIMEOUT in p->status and the output untouched.  A timeout
 * marks the exchange broken on every rank: each later combine of any rank
 * reports COTTUS_STATUS_TIMEOUT at once and writes nothing.  To recover,
 * every rank synchronises its stream, the ranks agree (host side) that all
 * of them are done with the exchange, destroy it and create a new one.
 * ---------------------------------------------------------------------- */
#define COTTUS_IPC_HANDLE_BYTES 64
typedef struct cottus_peer_exchange cottus_peer_exchange;
int cottus_peer_exchange_create(int32_t world, int32_t rank, int32_t batch, int32_t num_heads, int32_t head_dim,
                                cottus_peer_exchange **out, void *ipc_handle /* COTTUS_IPC_HANDLE_BYTES, out */);
/* handles: world x COTTUS_IPC_HANDLE_BYTES, in rank order (this rank's own is
 * skipped).  A handle of all zero bytes stands for a rank that takes no part
 * (a process that never joined): it gets a stand-in buffer on this GPU whose
 * flag nothing raises, so every combine of this exchange waits out its limit
 * and reports COTTUS_STATUS_TIMEOUT.  This lets failure handling be
 * exercised on one GPU. */
int cottus_peer_exchange_open(cottus_peer_exchange *ex, const void *handles);
/* Wait limit of the combine kernel in GPU clock cycles, in [1e3, 1e12]
 * (default 2e9); applies to the calls made after it. */
int cottus_peer_exchange_set_wait_cycles(cottus_peer_exchange *ex, int64_t cycles);
/* call on every rank only after all ranks stopped using the exchange */
void cottus_peer_exchange_destroy(cottus_peer_exchange *ex);
/* p->workspace must hold cottus_split_decode_workspace_size(p) bytes (the
 * decode runs in partial mode), under the rules of cottus_paged_decode. */
size_t cottus_split_decode_workspace_size(const cottus_paged_decode_params *p);
int cottus_split_decode(const cottus_paged_decode_params *p, cottus_peer_exchange *ex, cottus_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* COTTUS_B200_H */
