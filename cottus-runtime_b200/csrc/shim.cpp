// Host-side C++ surface with the reference's names and behaviour:
// cottus::PageTable, cottus::BlockAllocator, cottus::pagedAttentionCUDA and
// cottus::ropeCUDA, plus the C-ABI wrappers of the block pool and the
// host (cos, sin) formula.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "cottus/block_allocator.h"
#include "cottus/compute_primitives_cuda.h"
#include "cottus/page_table.h"
#include "cottus/paged_attention_cuda.h"
#include "cottus_b200.h"
#include "internal.h"

namespace cb200 {
int set_error(int code, const std::string& msg);

void rope_cos_sin_host(int32_t pos, int32_t pair, int32_t head_dim, float theta, float* c, float* s) {
    // compute_primitives_cpu.cpp:54-57 (float overloads of pow/cos/sin)
    float freq = 1.0f / std::pow(theta, (2.0f * static_cast<float>(pair)) / static_cast<float>(head_dim));
    float angle = static_cast<float>(pos) * freq;
    *c = std::cos(angle);
    *s = std::sin(angle);
}
}  // namespace cb200

namespace cottus {

// ---- PageTable (page_table.cpp:7-38) ----------------------------------------
PageTable::PageTable(int32_t blockSize) : blockSize_(blockSize) {
    if (blockSize <= 0) throw std::invalid_argument("blockSize must be positive");
}
void PageTable::appendBlock(int32_t blockId) { blocks_.push_back(blockId); }
int32_t PageTable::getBlock(int32_t logicalIndex) const {
    if (logicalIndex < 0 || logicalIndex >= static_cast<int32_t>(blocks_.size()))
        throw std::out_of_range("Logical index " + std::to_string(logicalIndex) + " out of range [0, " +
                                std::to_string(blocks_.size()) + ")");
    return blocks_[logicalIndex];
}
int32_t PageTable::operator[](int32_t logicalIndex) const { return getBlock(logicalIndex); }
int32_t PageTable::numBlocks() const { return static_cast<int32_t>(blocks_.size()); }
int32_t PageTable::blockSize() const { return blockSize_; }

// ---- BlockAllocator (block_allocator.cpp:7-55) --------------------------------
BlockAllocator::BlockAllocator(int32_t totalBlocks, int32_t blockSize) : total_(totalBlocks), blockSize_(blockSize) {
    if (totalBlocks <= 0) throw std::invalid_argument("totalBlocks must be positive");
    if (blockSize <= 0) throw std::invalid_argument("blockSize must be positive");
    // stack top is the end of the vector; push the highest id first so that
    // the first allocation returns block 0
    freeStack_.resize(totalBlocks);
    for (int32_t i = 0; i < totalBlocks; ++i) freeStack_[i] = totalBlocks - 1 - i;
    inUse_.assign(totalBlocks, 0);
}
int32_t BlockAllocator::allocateBlock() {
    if (freeStack_.empty()) throw std::runtime_error("Out of memory: no free blocks");
    int32_t id = freeStack_.back();
    freeStack_.pop_back();
    inUse_[id] = 1;
    return id;
}
void BlockAllocator::freeBlock(int32_t blockId) {
    if (blockId < 0 || blockId >= total_) throw std::invalid_argument("Invalid block ID: " + std::to_string(blockId));
    if (!inUse_[blockId]) throw std::runtime_error("Double free detected for block " + std::to_string(blockId));
    inUse_[blockId] = 0;
    freeStack_.push_back(blockId);
}
int32_t BlockAllocator::numFreeBlocks() const { return static_cast<int32_t>(freeStack_.size()); }
int32_t BlockAllocator::totalBlocks() const { return total_; }
int32_t BlockAllocator::blockSize() const { return blockSize_; }

namespace {

void throw_cuda(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e));
}

// Staging used only by the host-pointer shim: pinned host + device buffers
// grown on demand and kept per host thread and device.
struct Staging {
    int device = -1;
    cudaStream_t stream = nullptr;
    void* host = nullptr;
    size_t host_bytes = 0;
    void* dev = nullptr;
    size_t dev_bytes = 0;
    ~Staging() { release(); }
    void release() {
        if (host) cudaFreeHost(host);
        if (dev) cudaFree(dev);
        if (stream) cudaStreamDestroy(stream);
        host = dev = nullptr;
        stream = nullptr;
        host_bytes = dev_bytes = 0;
    }
    void ensure(size_t hbytes, size_t dbytes) {
        int cur = 0;
        throw_cuda(cudaGetDevice(&cur));
        if (cur != device) {
            release();
            device = cur;
        }
        if (!stream) throw_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        if (hbytes > host_bytes) {
            if (host) cudaFreeHost(host);
            host = nullptr;
            throw_cuda(cudaMallocHost(&host, hbytes));
            host_bytes = hbytes;
        }
        if (dbytes > dev_bytes) {
            if (dev) cudaFree(dev);
            dev = nullptr;
            throw_cuda(cudaMalloc(&dev, dbytes));
            dev_bytes = dbytes;
        }
    }
};
thread_local Staging g_staging;

size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

void pagedAttentionCUDA(float* output, const float* query, const void* kvCacheBase, const PageTable& pageTable,
                        int32_t seqLen, int32_t layerIdx, int32_t numHeads, int32_t numKvHeads, int32_t headDim,
                        int32_t blockSize, int32_t numLayers) {
    // paged_attention_cuda.cu:109-113
    if (seqLen <= 0) throw std::invalid_argument("seqLen must be positive");
    if (layerIdx < 0) throw std::invalid_argument("layerIdx must be non-negative");
    if (numHeads <= 0 || numKvHeads <= 0) throw std::invalid_argument("numHeads must be positive");
    if (headDim <= 0 || headDim > 256) throw std::invalid_argument("headDim must be in (0, 256]");
    if (blockSize <= 0) throw std::invalid_argument("blockSize must be positive");
    if (numLayers <= layerIdx) throw std::invalid_argument("layerIdx must be less than numLayers");
    const int32_t nblk = (seqLen + blockSize - 1) / blockSize;
    // paged_attention_cpu.cpp:58-60
    if (nblk > pageTable.numBlocks()) throw std::out_of_range("Token position exceeds page table");

    // Stage only this layer's K|V slice of each referenced block, in logical
    // order, so the device pool is dense and the device table is 0..nblk-1.
    const size_t slice = (size_t)2 * blockSize * numKvHeads * headDim;  // fp16 elements
    const size_t per_block = slice * numLayers;
    const size_t qo_bytes = (size_t)numHeads * headDim * sizeof(float);
    const size_t pool_bytes = slice * nblk * sizeof(uint16_t);
    const size_t table_bytes = (size_t)nblk * sizeof(int32_t) + sizeof(int32_t);

    cottus_paged_decode_params p;
    std::memset(&p, 0, sizeof p);
    p.batch = 1;
    p.num_heads = numHeads;
    p.num_kv_heads = numKvHeads;
    p.head_dim = headDim;
    p.block_size = blockSize;
    p.num_layers = 1;
    p.layer = 0;
    p.max_blocks_per_seq = nblk;
    p.num_physical_blocks = nblk;
    p.q_dtype = COTTUS_F32;
    p.out_dtype = COTTUS_F32;
    p.query = reinterpret_cast<const void*>(16);  // placeholders for the size query (aligned, non-null)
    p.out = reinterpret_cast<void*>(16);
    p.kv_pool = reinterpret_cast<const uint16_t*>(16);
    const size_t ws = cottus_paged_decode_workspace_size(&p);

    const size_t off_pool = 0;
    const size_t off_q = align_up(off_pool + pool_bytes);
    const size_t off_table = align_up(off_q + qo_bytes);
    const size_t host_bytes = align_up(off_table + table_bytes);
    const size_t off_out = host_bytes;
    const size_t off_ws = align_up(off_out + qo_bytes);
    const size_t dev_bytes = align_up(off_ws + ws);

    Staging& st = g_staging;
    st.ensure(host_bytes, dev_bytes);
    auto* h = static_cast<uint8_t*>(st.host);
    auto* d = static_cast<uint8_t*>(st.dev);
    const auto* src = static_cast<const uint16_t*>(kvCacheBase);
    for (int32_t i = 0; i < nblk; ++i) {
        const int64_t blk = pageTable[i];
        std::memcpy(h + off_pool + (size_t)i * slice * 2, src + blk * per_block + (size_t)layerIdx * slice, slice * 2);
    }
    auto* table = reinterpret_cast<int32_t*>(h + off_table);
    for (int32_t i = 0; i < nblk; ++i) table[i] = i;
    table[nblk] = seqLen;

    throw_cuda(cudaMemcpyAsync(d, h, host_bytes, cudaMemcpyHostToDevice, st.stream));
    throw_cuda(cudaMemcpyAsync(d + off_q, query, qo_bytes, cudaMemcpyDefault, st.stream));
    p.query = d + off_q;
    p.out = d + off_out;
    p.kv_pool = reinterpret_cast<const uint16_t*>(d + off_pool);
    p.block_table = reinterpret_cast<const int32_t*>(d + off_table);
    p.context_lens = reinterpret_cast<const int32_t*>(d + off_table) + nblk;
    p.workspace = ws ? d + off_ws : nullptr;
    p.workspace_bytes = ws;
    const int rc = cottus_paged_decode(&p, reinterpret_cast<cottus_stream_t>(st.stream));
    if (rc != COTTUS_OK) {
        if (rc == COTTUS_ERR_CUDA) throw std::runtime_error(cottus_last_error());
        throw std::invalid_argument(cottus_last_error());
    }
    throw_cuda(cudaMemcpyAsync(output, d + off_out, qo_bytes, cudaMemcpyDefault, st.stream));
    throw_cuda(cudaStreamSynchronize(st.stream));
}

void ropeCUDA(float* d_output, const float* d_input, int32_t pos, int32_t numHeads, int32_t headDim, float theta) {
    if (numHeads <= 0 || headDim < 2) return;  // the reference launches no work in this case
    const int pairs = headDim / 2;
    std::vector<float> cs(2 * pairs);
    for (int d = 0; d < pairs; ++d) cb200::rope_cos_sin_host(pos, d, headDim, theta, &cs[2 * d], &cs[2 * d + 1]);
    if (headDim <= 256) {
        throw_cuda(cb200::launch_rope_single(d_output, d_input, cs.data(), numHeads, headDim, nullptr));
        return;
    }
    // wide heads: pass the table through a small device buffer on the default stream
    float* dcs = nullptr;
    throw_cuda(cudaMalloc(&dcs, cs.size() * sizeof(float)));
    int32_t* dpos = nullptr;
    cudaError_t e = cudaMalloc(&dpos, sizeof(int32_t));
    const int32_t zero = 0;
    if (e == cudaSuccess) e = cudaMemcpy(dcs, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dpos, &zero, sizeof zero, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cb200::launch_rope(d_output, d_input, dpos, 1, numHeads, headDim, dcs, 1, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(dcs);
    cudaFree(dpos);
    throw_cuda(e);
}

}  // namespace cottus

// ---- C-ABI block pool ---------------------------------------------------------
struct cottus_block_allocator {
    cottus::BlockAllocator impl;
    cottus_block_allocator(int32_t t, int32_t b) : impl(t, b) {}
};

extern "C" {

int cottus_block_allocator_create(int32_t total_blocks, int32_t block_size, cottus_block_allocator** out) {
    if (!out) return cb200::set_error(COTTUS_ERR_INVALID_ARGUMENT, "out must not be NULL");
    *out = nullptr;
    try {
        *out = new cottus_block_allocator(total_blocks, block_size);
        return COTTUS_OK;
    } catch (const std::invalid_argument& e) {
        return cb200::set_error(COTTUS_ERR_INVALID_ARGUMENT, e.what());
    } catch (const std::exception& e) {
        return cb200::set_error(COTTUS_ERR_OUT_OF_MEMORY, e.what());
    }
}

void cottus_block_allocator_destroy(cottus_block_allocator* a) { delete a; }

int cottus_block_allocator_allocate(cottus_block_allocator* a, int32_t* block_id) {
    if (!a || !block_id) return cb200::set_error(COTTUS_ERR_INVALID_ARGUMENT, "NULL argument");
    try {
        *block_id = a->impl.allocateBlock();
        return COTTUS_OK;
    } catch (const std::exception& e) {
        *block_id = -1;
        return cb200::set_error(COTTUS_ERR_OUT_OF_MEMORY, e.what());
    }
}

int cottus_block_allocator_free(cottus_block_allocator* a, int32_t block_id) {
    if (!a) return cb200::set_error(COTTUS_ERR_INVALID_ARGUMENT, "NULL allocator");
    try {
        a->impl.freeBlock(block_id);
        return COTTUS_OK;
    } catch (const std::invalid_argument& e) {
        return cb200::set_error(COTTUS_ERR_INVALID_ARGUMENT, e.what());
    } catch (const std::exception& e) {
        return cb200::set_error(COTTUS_ERR_DOUBLE_FREE, e.what());
    }
}

int32_t cottus_block_allocator_num_free(const cottus_block_allocator* a) { return a ? a->impl.numFreeBlocks() : 0; }
int32_t cottus_block_allocator_total_blocks(const cottus_block_allocator* a) { return a ? a->impl.totalBlocks() : 0; }

}  // extern "C"
