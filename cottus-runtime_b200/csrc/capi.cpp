// C-ABI entry points (include/cottus_b200.h): argument validation that
// mirrors the reference's checks and messages, path selection (TMA fast
// path or generic kernel) and launch.  Never throws across the ABI.
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "cottus_b200.h"
#include "internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e) {
    // message prefix of the reference's CUDA_CHECK (paged_attention_cuda.cu:8-14)
    return fail(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e));
}

bool valid_dtype(int32_t t) { return t == COTTUS_F32 || t == COTTUS_F16; }

// Checks shared by every attention entry point, in the order of
// paged_attention_cuda.cu:109-113 / paged_attention_cpu.cpp:37-41.
int check_common(int32_t batch, int32_t layer, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                 int32_t block_size, int32_t num_layers, int32_t max_blocks, int64_t num_blocks) {
    if (batch < 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "batch must be non-negative");
    if (layer < 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "layerIdx must be non-negative");
    if (num_heads <= 0 || num_kv_heads <= 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "numHeads must be positive");
    if (head_dim <= 0 || head_dim > 512) return fail(COTTUS_ERR_INVALID_ARGUMENT, "headDim must be in (0, 512]");
    if (block_size <= 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "blockSize must be positive");
    if (num_layers <= 0 || layer >= num_layers)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "layerIdx must be less than numLayers");
    if (max_blocks < 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "max_blocks_per_seq must be non-negative");
    if (num_blocks < 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "num_physical_blocks must be non-negative");
    return COTTUS_OK;
}

float resolve_scale(float scale, int32_t head_dim) {
    // paged_attention_cpu.cpp:75: 1.0f / std::sqrt(static_cast<float>(headDim))
    return scale > 0.f ? scale : 1.0f / std::sqrt(static_cast<float>(head_dim));
}

int run_decode(const cb200::DecodeDesc& d, cudaStream_t st) {
    if (d.batch == 0) return COTTUS_OK;
    cudaError_t e;
    if (cb200::tma_supported(d)) {
        const size_t need = cb200::tma_workspace_bytes(d);
        if (!d.workspace || d.workspace_bytes < need)
            return fail(COTTUS_ERR_WORKSPACE, "workspace missing or smaller than the required " + std::to_string(need) +
                                                  " bytes");
        if (reinterpret_cast<uintptr_t>(d.workspace) & 15)
            return fail(COTTUS_ERR_WORKSPACE, "workspace must be 16-byte aligned");
        e = cb200::launch_decode_tma(d, st);
    } else {
        if (d.rope) {
            e = cb200::launch_rope_append(d, st);
            if (e != cudaSuccess) return cuda_fail(e);
        }
        e = cb200::launch_decode_generic(d, st);
    }
    if (e != cudaSuccess) return cuda_fail(e);
    return COTTUS_OK;
}

cb200::DecodeDesc desc_from(const cottus_paged_decode_params* p) {
    cb200::DecodeDesc d;
    d.out = p->out;
    d.q = p->query;
    d.kv = p->kv_pool;
    d.block_table = p->block_table;
    d.context_lens = p->context_lens;
    d.num_blocks = p->num_physical_blocks;
    d.batch = p->batch;
    d.num_heads = p->num_heads;
    d.num_kv_heads = p->num_kv_heads;
    d.head_dim = p->head_dim;
    d.block_size = p->block_size;
    d.num_layers = p->num_layers;
    d.layer = p->layer;
    d.max_blocks = p->max_blocks_per_seq;
    d.q_f16 = p->q_dtype == COTTUS_F16;
    d.out_f16 = p->out_dtype == COTTUS_F16;
    d.scale = resolve_scale(p->scale, p->head_dim);
    d.lse = p->lse_out;
    d.workspace = p->workspace;
    d.workspace_bytes = p->workspace_bytes;
    d.status = p->status;
    return d;
}

cb200::DecodeDesc desc_from(const cottus_decode_step_params* p) {
    cb200::DecodeDesc d;
    d.out = p->out;
    d.q = p->query;
    d.kv = p->kv_pool;
    d.kv_mut = p->kv_pool;
    d.block_table = p->block_table;
    d.num_blocks = p->num_physical_blocks;
    d.batch = p->batch;
    d.num_heads = p->num_heads;
    d.num_kv_heads = p->num_kv_heads;
    d.head_dim = p->head_dim;
    d.block_size = p->block_size;
    d.num_layers = p->num_layers;
    d.layer = p->layer;
    d.max_blocks = p->max_blocks_per_seq;
    d.q_f16 = p->qkv_dtype == COTTUS_F16;
    d.out_f16 = p->out_dtype == COTTUS_F16;
    d.scale = resolve_scale(p->scale, p->head_dim);
    d.workspace = p->workspace;
    d.workspace_bytes = p->workspace_bytes;
    d.status = p->status;
    d.rope = true;
    d.positions = p->positions;
    d.k_new = p->key;
    d.v_new = p->value;
    d.cos_sin = p->cos_sin;
    d.max_position = p->max_position;
    d.q_out = p->query_out;
    return d;
}

int check_step(const cottus_decode_step_params* p, bool with_attention) {
    if (!p) return fail(COTTUS_ERR_INVALID_ARGUMENT, "params must not be NULL");
    int rc = check_common(p->batch, p->layer, p->num_heads, p->num_kv_heads, p->head_dim, p->block_size,
                          p->num_layers, p->max_blocks_per_seq, p->num_physical_blocks);
    if (rc) return rc;
    if (!valid_dtype(p->qkv_dtype) || (with_attention && !valid_dtype(p->out_dtype)))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (p->cos_sin && (p->max_position <= 0 || (p->head_dim % 2) != 0))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "RoPE needs max_position > 0 and an even headDim");
    if (p->batch > 0 && (!p->query || !p->key || !p->value || !p->positions || !p->kv_pool || !p->block_table))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL input pointer");
    if (with_attention && p->batch > 0 && !p->out) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL output pointer");
    return COTTUS_OK;
}

}  // namespace

extern "C" {

const char* cottus_last_error(void) { return g_last_error.c_str(); }

const char* cottus_status_string(int s) {
    switch (s) {
        case COTTUS_OK: return "ok";
        case COTTUS_ERR_INVALID_ARGUMENT: return "invalid argument";
        case COTTUS_ERR_OUT_OF_RANGE: return "out of range";
        case COTTUS_ERR_CUDA: return "CUDA error";
        case COTTUS_ERR_UNSUPPORTED: return "unsupported";
        case COTTUS_ERR_WORKSPACE: return "workspace";
        case COTTUS_ERR_OUT_OF_MEMORY: return "out of memory";
        case COTTUS_ERR_DOUBLE_FREE: return "double free";
    }
    return "unknown";
}

int cottus_version(void) { return 10000; }

size_t cottus_paged_decode_workspace_size(const cottus_paged_decode_params* p) {
    if (!p) return 0;
    cb200::DecodeDesc d = desc_from(p);
    return cb200::tma_supported(d) ? cb200::tma_workspace_bytes(d) : 0;
}

int cottus_paged_decode(const cottus_paged_decode_params* p, cottus_stream_t stream) {
    const int rc = cb200::validate_decode_params(p);
    if (rc) return rc;
    return run_decode(desc_from(p), reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace cb200 {
// Argument checks of cottus_paged_decode, shared with the entry points that
// wrap it (they run before anything is sized, allocated or queued).
int validate_decode_params(const cottus_paged_decode_params* p) {
    if (!p) return fail(COTTUS_ERR_INVALID_ARGUMENT, "params must not be NULL");
    int rc = check_common(p->batch, p->layer, p->num_heads, p->num_kv_heads, p->head_dim, p->block_size,
                          p->num_layers, p->max_blocks_per_seq, p->num_physical_blocks);
    if (rc) return rc;
    if (!valid_dtype(p->q_dtype) || !valid_dtype(p->out_dtype)) return fail(COTTUS_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (p->batch > 0 && (!p->out || !p->query || !p->kv_pool || !p->block_table || !p->context_lens))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL pointer argument");
    return COTTUS_OK;
}

// cottus_paged_decode whose completion is signalled to the ranks of a split
// context (peer_exchange.cu): by the fast-path kernel itself, or by a
// signal kernel after the generic one.
int paged_decode_signalled(const cottus_paged_decode_params* p, const PeerSignal& sig, cudaStream_t st) {
    int rc = validate_decode_params(p);
    if (rc) return rc;
    if (p->batch <= 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "empty batch");
    DecodeDesc d = desc_from(p);
    if (tma_supported(d)) {
        d.signal = sig;
        return run_decode(d, st);
    }
    rc = run_decode(d, st);
    if (rc) return rc;
    const cudaError_t e = launch_peer_signal(sig, st);
    return e == cudaSuccess ? COTTUS_OK : cuda_fail(e);
}

int paged_decode_exchanged(const cottus_paged_decode_params* p, const PeerSignal& sig, const PeerMerge& pm,
                           cudaStream_t st) {
    int rc = validate_decode_params(p);
    if (rc) return rc;
    if (p->batch <= 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "empty batch");
    DecodeDesc d = desc_from(p);
    if (!tma_supported(d) || !mma_supported(d))
        return fail(COTTUS_ERR_UNSUPPORTED, "the merge runs in the decode kernel only on the tensor-core path");
    d.signal = sig;
    d.merge = pm;
    return run_decode(d, st);
}
}  // namespace cb200

extern "C" {

int cottus_lse_combine(const cottus_lse_combine_params* p, cottus_stream_t stream) {
    if (!p) return fail(COTTUS_ERR_INVALID_ARGUMENT, "params must not be NULL");
    if (p->num_parts <= 0 || p->batch < 0 || p->num_heads <= 0 || p->head_dim <= 0)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "num_parts, num_heads and head_dim must be positive");
    if (!valid_dtype(p->out_dtype)) return fail(COTTUS_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (p->batch > 0 && (!p->out || !p->partial_out || !p->partial_lse))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL pointer argument");
    cudaError_t e = cb200::launch_lse_combine(p->out, p->out_dtype == COTTUS_F16, p->lse_out, p->partial_out,
                                              p->partial_lse, p->num_parts, p->batch, p->num_heads, p->head_dim,
                                              reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? COTTUS_OK : cuda_fail(e);
}

int cottus_rope_cos_sin_fill(float* host_table, int32_t max_position, int32_t head_dim, float theta) {
    if (!host_table || max_position <= 0 || head_dim <= 0 || (head_dim % 2) != 0)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "need a table, max_position > 0 and an even headDim");
    const int pairs = head_dim / 2;
    for (int32_t p = 0; p < max_position; ++p)
        for (int d = 0; d < pairs; ++d)
            cb200::rope_cos_sin_host(p, d, head_dim, theta, &host_table[((size_t)p * pairs + d) * 2],
                                     &host_table[((size_t)p * pairs + d) * 2 + 1]);
    return COTTUS_OK;
}

int cottus_rope(float* out, const float* in, const int32_t* positions, int32_t num_tokens, int32_t num_heads,
                int32_t head_dim, const float* cos_sin, int32_t max_position, cottus_stream_t stream) {
    if (num_tokens < 0 || num_heads <= 0 || head_dim <= 0 || (head_dim % 2) != 0 || max_position <= 0)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "invalid RoPE shape");
    if (num_tokens > 0 && (!out || !in || !positions || !cos_sin))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL pointer argument");
    cudaError_t e = cb200::launch_rope(out, in, positions, num_tokens, num_heads, head_dim, cos_sin, max_position,
                                       reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? COTTUS_OK : cuda_fail(e);
}

int cottus_rope_append(const cottus_decode_step_params* p, cottus_stream_t stream) {
    int rc = check_step(p, false);
    if (rc) return rc;
    if (p->batch == 0) return COTTUS_OK;
    cudaError_t e = cb200::launch_rope_append(desc_from(p), reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? COTTUS_OK : cuda_fail(e);
}

size_t cottus_rope_append_decode_workspace_size(const cottus_decode_step_params* p) {
    if (!p) return 0;
    cb200::DecodeDesc d = desc_from(p);
    return cb200::tma_supported(d) ? cb200::tma_workspace_bytes(d) : 0;
}

int cottus_rope_append_decode(const cottus_decode_step_params* p, cottus_stream_t stream) {
    int rc = check_step(p, true);
    if (rc) return rc;
    return run_decode(desc_from(p), reinterpret_cast<cudaStream_t>(stream));
}

int cottus_paged_gather(uint16_t* k_out, uint16_t* v_out, const uint16_t* kv_pool, const int32_t* block_table,
                        const int32_t* context_lens, int64_t num_physical_blocks, int32_t batch, int32_t max_context,
                        int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_layers, int32_t layer,
                        int32_t max_blocks_per_seq, uint32_t* status, cottus_stream_t stream) {
    int rc = check_common(batch, layer, num_kv_heads, num_kv_heads, head_dim, block_size, num_layers,
                          max_blocks_per_seq, num_physical_blocks);
    if (rc) return rc;
    if (max_context < 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "max_context must be non-negative");
    if (batch > 0 && (!k_out || !v_out || !kv_pool || !block_table || !context_lens))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL pointer argument");
    cudaError_t e = cb200::launch_gather(k_out, v_out, kv_pool, block_table, context_lens, num_physical_blocks, batch,
                                         max_context, num_kv_heads, head_dim, block_size, num_layers, layer,
                                         max_blocks_per_seq, status, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? COTTUS_OK : cuda_fail(e);
}

}  // extern "C"

// Internal error hook for the C++ shims in the same library.
namespace cb200 {
int set_error(int code, const std::string& msg) { return fail(code, msg); }
}  // namespace cb200
