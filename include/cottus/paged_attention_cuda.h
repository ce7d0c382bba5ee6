// Same-signature drop-in for the reference's cottus::pagedAttentionCUDA
// (paged_attention_cuda.h:9-21): host output/query pointers, host KV cache,
// one sequence, synchronous.  Internally stages only the pages the
// PageTable names (for layer `layerIdx`) through cached device buffers and
// runs the batched sm_100a decode kernel with batch 1.  Errors throw the
// reference's exception types and messages (paged_attention_cuda.cu:8-14,
// 109-113; paged_attention_cpu.cpp:58-60).
#pragma once

#include <cstdint>

#include "page_table.h"

namespace cottus {

void pagedAttentionCUDA(float* output, const float* query, const void* kvCacheBase, const PageTable& pageTable,
                        int32_t seqLen, int32_t layerIdx, int32_t numHeads, int32_t numKvHeads, int32_t headDim,
                        int32_t blockSize, int32_t numLayers);

}  // namespace cottus
