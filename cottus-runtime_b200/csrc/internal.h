// Internal launch interface between the C-ABI layer (capi.cpp) and the
// kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "cottus_b200.h"

namespace cb200 {

// Completion signal of a split-context decode (one rank of `world`): when
// the launch has stored all its outputs, its last CTA writes `epoch` to
// flags[r][rank] for every rank r (device pointers valid on this GPU: its
// own array, and the peers' mapped over NVLink).  world == 0: none.
constexpr int kMaxPeers = 8;
struct PeerSignal {
    uint32_t* flags[kMaxPeers] = {};
    uint32_t* done = nullptr;  // CTA completion counter of this launch, zero between launches
    int32_t rank = 0, world = 0;
    uint32_t epoch = 0;
};

// The merge of a split-context step done by the decode kernel itself, after
// its completion signal (fast-path kernels; see peer_exchange.cu): every CTA
// waits (bounded) until every rank's flag in `flags` has reached the signal's
// epoch, then merges a share of the (sequence, head) rows from every rank's
// partial slot (part / lse, peer pointers) into `out`.  A wait that runs out
// reports COTTUS_STATUS_TIMEOUT, writes nothing and stores 1 into every
// rank's broken word; a set broken word of this rank makes the merge refuse
// at once.  enabled == 0: none.
struct PeerMerge {
    const float* part[kMaxPeers] = {};
    const float* lse[kMaxPeers] = {};
    uint32_t* broken[kMaxPeers] = {};
    const uint32_t* flags = nullptr;  // this rank's flag words, one per rank
    uint32_t* broken_own = nullptr;
    void* out = nullptr;
    float* lse_out = nullptr;
    long long wait_cycles = 0;
    int32_t out_f16 = 0, enabled = 0;
};

// One resolved decode launch.  In rope mode the context length of sequence
// b is positions[b] + 1 and the kernel first rotates q/k and appends k/v.
struct DecodeDesc {
    void* out = nullptr;
    const void* q = nullptr;
    const uint16_t* kv = nullptr;
    const int32_t* block_table = nullptr;
    const int32_t* context_lens = nullptr;
    int64_t num_blocks = 0;
    int32_t batch = 0, num_heads = 0, num_kv_heads = 0, head_dim = 0, block_size = 0, num_layers = 0, layer = 0,
            max_blocks = 0;
    int32_t q_f16 = 0, out_f16 = 0;
    float scale = 0.f;
    float* lse = nullptr;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    uint32_t* status = nullptr;
    // rope / append (rope mode)
    bool rope = false;
    const int32_t* positions = nullptr;
    const void* k_new = nullptr;
    const void* v_new = nullptr;
    const float* cos_sin = nullptr;
    int32_t max_position = 0;
    void* q_out = nullptr;
    uint16_t* kv_mut = nullptr;
    PeerSignal signal;  // split-context decode across GPUs (fast path kernels)
    PeerMerge merge;    // with signal: the merge done in the same kernel (tensor-core kernel only)
};

// Fast path: persistent stream-K TMA kernel (block_size 16, head_dim in
// {64,128,256}, group size in {1,2,4,8}, 16-B aligned pool).
bool tma_supported(const DecodeDesc& d);
size_t tma_workspace_bytes(const DecodeDesc& d);
cudaError_t launch_decode_tma(const DecodeDesc& d, cudaStream_t st);

// Instantiation entry points, one per head_dim translation unit.
cudaError_t launch_decode_tma_d64(const DecodeDesc& d, cudaStream_t st);
cudaError_t launch_decode_tma_d128(const DecodeDesc& d, cudaStream_t st);
cudaError_t launch_decode_tma_d256(const DecodeDesc& d, cudaStream_t st);
size_t tma_workers_d64(const DecodeDesc& d);
size_t tma_workers_d128(const DecodeDesc& d);
size_t tma_workers_d256(const DecodeDesc& d);

// Tensor-core variant of the fast path (head_dim 64/128, fp16 output or
// LSE partials).
bool mma_supported(const DecodeDesc& d);
cudaError_t launch_decode_mma_d64(const DecodeDesc& d, cudaStream_t st);
cudaError_t launch_decode_mma_d128(const DecodeDesc& d, cudaStream_t st);
size_t mma_workers_d64(const DecodeDesc& d);
size_t mma_workers_d128(const DecodeDesc& d);

// Bytes at the start of a decode workspace that hold a reserved word and
// the pair arrival counters (zero before a launch that has never used the
// workspace).
size_t workspace_zero_prefix_bytes(int32_t batch, int32_t num_kv_heads);

// Generic path: any head_dim <= 512, any block size; one CTA per (seq, head).
cudaError_t launch_decode_generic(const DecodeDesc& d, cudaStream_t st);

// RoPE + append (no attention).
cudaError_t launch_rope_append(const DecodeDesc& d, cudaStream_t st);
cudaError_t launch_rope(float* out, const float* in, const int32_t* positions, int32_t num_tokens,
                        int32_t num_heads, int32_t head_dim, const float* cos_sin, int32_t max_position,
                        cudaStream_t st);
// Single-position rotation with (cos, sin) pairs passed by value (ropeCUDA shim).
cudaError_t launch_rope_single(float* out, const float* in, const float* host_cos_sin, int32_t num_heads,
                               int32_t head_dim, cudaStream_t st);

cudaError_t launch_lse_combine(void* out, int out_f16, float* lse_out, const float* part_out,
                               const float* part_lse, int32_t num_parts, int32_t batch, int32_t num_heads,
                               int32_t head_dim, cudaStream_t st);

cudaError_t launch_gather(uint16_t* k_out, uint16_t* v_out, const uint16_t* kv, const int32_t* block_table,
                          const int32_t* context_lens, int64_t num_blocks, int32_t batch, int32_t max_context,
                          int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_layers,
                          int32_t layer, int32_t max_blocks, uint32_t* status, cudaStream_t st);

// Argument checks of cottus_paged_decode (capi.cpp); COTTUS_OK or the
// error code, with the message set.
int validate_decode_params(const cottus_paged_decode_params* p);

// Split-context decode (peer_exchange.cu): the decode whose completion is
// signalled to every rank, and the stand-alone signal used after the
// generic kernel.
int paged_decode_signalled(const cottus_paged_decode_params* p, const PeerSignal& sig, cudaStream_t st);
// The same step with the merge in the decode kernel itself; returns
// COTTUS_ERR_UNSUPPORTED (nothing launched) where the shape takes another kernel.
int paged_decode_exchanged(const cottus_paged_decode_params* p, const PeerSignal& sig, const PeerMerge& pm,
                           cudaStream_t st);
cudaError_t launch_peer_signal(const PeerSignal& sig, cudaStream_t st);

// Host-side (cos, sin) of the reference formula (compute_primitives_cpu.cpp:54-57).
void rope_cos_sin_host(int32_t pos, int32_t pair, int32_t head_dim, float theta, float* c, float* s);

}  // namespace cb200
