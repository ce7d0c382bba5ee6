// Batched decode-step driver: the block bookkeeping of Engine::generate
// (engine.cpp:52-95) for many sequences at once, with the block table kept
// in device memory and updated incrementally.
//
// The reference keeps one host PageTable per generate() call, a host KV
// cache, and copies the table (and the KV region) to the device on every
// attention call (paged_attention_cuda.cu:125-135).  Here the active
// sequences are the rows of a caller-owned device table
// [max_batch][max_blocks_per_seq] plus a device position per row; the host
// keeps a mirror, and each step sends only what changed (the block appended
// to a row whose next token starts a block, rows moved by a release, and
// the positions) as the parameters of one small kernel: no device scratch,
// no host-to-device copy call, stream-ordered before the step's kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "common.cuh"
#include "cottus/block_allocator.h"
#include "cottus_b200.h"
#include "internal.h"

namespace cb200 {
int set_error(int code, const std::string& msg);

namespace {

// Entries per update launch: 2 x 4 bytes each, 16 KB of kernel parameters
// (within the 32 KB that sm_70 and later accept).
constexpr int kMaxTableUpdates = 2048;

struct TableUpdates {
    int32_t n;
    int32_t idx[kMaxTableUpdates];  // < table_elems: block table entry; else position of row idx - table_elems
    int32_t val[kMaxTableUpdates];
};

__global__ void table_update_kernel(const __grid_constant__ TableUpdates u, int32_t* table, int32_t table_elems,
                                    int32_t* positions, int32_t* context_lens) {
    for (int i = threadIdx.x; i < u.n; i += blockDim.x) {
        const int32_t idx = u.idx[i];
        if (idx < table_elems) {
            table[idx] = u.val[i];
        } else {
            positions[idx - table_elems] = u.val[i];
            if (context_lens) context_lens[idx - table_elems] = u.val[i] + 1;  // the prefix and the step's token
        }
    }
}

}  // namespace
}  // namespace cb200

struct cottus_decode_batch {
    struct Seq {
        int64_t id;
        int32_t pos;                  // position of the sequence's next token
        std::vector<int32_t> blocks;  // physical ids in allocation (logical) order
    };

    cottus_decode_batch_desc d;
    cottus::BlockAllocator alloc;
    std::vector<Seq> rows;
    std::unordered_map<int64_t, int32_t> row_of;
    std::vector<std::pair<int32_t, int32_t>> pending;  // device updates not yet sent
    bool in_step = false;

    explicit cottus_decode_batch(const cottus_decode_batch_desc& desc)
        : d(desc), alloc(desc.num_blocks, desc.block_size) {}

    int32_t table_elems() const { return d.max_batch * d.max_blocks_per_seq; }

    // every entry of row r (blocks and position) as pending updates
    void queue_row(int32_t r) {
        const Seq& s = rows[r];
        for (size_t j = 0; j < s.blocks.size(); ++j)
            pending.emplace_back(r * d.max_blocks_per_seq + (int32_t)j, s.blocks[j]);
        pending.emplace_back(table_elems() + r, s.pos);
    }
};

namespace {

int fail(int code, const std::string& msg) { return cb200::set_error(code, msg); }

bool has_device(const cottus_decode_batch* b) { return b->d.device_block_table && b->d.device_positions; }

}  // namespace

extern "C" {

int cottus_decode_batch_create(const cottus_decode_batch_desc* desc, cottus_decode_batch** out) {
    if (!desc || !out) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (desc->block_size <= 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "blockSize must be positive");
    if (desc->num_blocks <= 0) return fail(COTTUS_ERR_INVALID_ARGUMENT, "totalBlocks must be positive");
    if (desc->max_batch <= 0 || desc->max_blocks_per_seq <= 0)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "max_batch and max_blocks_per_seq must be positive");
    if ((int64_t)desc->max_batch * desc->max_blocks_per_seq + desc->max_batch >= (int64_t(1) << 31))
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "block table too large for 32-bit entry indices");
    if (!desc->device_block_table != !desc->device_positions)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "give both device arrays or neither");
    if (desc->device_context_lens && !desc->device_positions)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "device_context_lens needs the device table and positions");
    try {
        *out = new cottus_decode_batch(*desc);
    } catch (const std::exception& e) {
        return fail(COTTUS_ERR_INVALID_ARGUMENT, e.what());
    }
    return COTTUS_OK;
}

void cottus_decode_batch_destroy(cottus_decode_batch* b) { delete b; }

int cottus_decode_batch_add(cottus_decode_batch* b, int64_t seq_id, int32_t* row) {
    if (!b) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL batch");
    if (b->in_step) return fail(COTTUS_ERR_INVALID_ARGUMENT, "cannot add a sequence inside a step");
    if (b->row_of.count(seq_id)) return fail(COTTUS_ERR_INVALID_ARGUMENT, "sequence " + std::to_string(seq_id) +
                                                                             " is already in the batch");
    if ((int32_t)b->rows.size() >= b->d.max_batch)
        return fail(COTTUS_ERR_OUT_OF_RANGE, "batch is full (" + std::to_string(b->d.max_batch) + " rows)");
    const int32_t r = (int32_t)b->rows.size();
    b->rows.push_back({seq_id, 0, {}});
    b->row_of[seq_id] = r;
    b->pending.emplace_back(b->table_elems() + r, 0);
    if (row) *row = r;
    return COTTUS_OK;
}

int cottus_decode_batch_release(cottus_decode_batch* b, int64_t seq_id) {
    if (!b) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL batch");
    if (b->in_step) return fail(COTTUS_ERR_INVALID_ARGUMENT, "cannot release a sequence inside a step");
    auto it = b->row_of.find(seq_id);
    if (it == b->row_of.end())
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "sequence " + std::to_string(seq_id) + " is not in the batch");
    const int32_t r = it->second;
    // blocks go back in allocation order (engine.cpp:88-90)
    for (int32_t blk : b->rows[r].blocks) {
        try {
            b->alloc.freeBlock(blk);
        } catch (const std::exception& e) {
            return fail(COTTUS_ERR_DOUBLE_FREE, e.what());
        }
    }
    b->row_of.erase(it);
    const int32_t last = (int32_t)b->rows.size() - 1;
    if (r != last) {  // the last row takes the freed one
        b->rows[r] = std::move(b->rows[last]);
        b->row_of[b->rows[r].id] = r;
        b->rows.pop_back();
        b->queue_row(r);
    } else {
        b->rows.pop_back();
    }
    return COTTUS_OK;
}

int cottus_decode_batch_begin_step(cottus_decode_batch* b, cottus_stream_t stream) {
    if (!b) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL batch");
    if (b->in_step) return fail(COTTUS_ERR_INVALID_ARGUMENT, "step already begun");
    const int32_t cap_tokens = b->d.max_blocks_per_seq * b->d.block_size;
    for (const auto& s : b->rows)
        if (s.pos >= cap_tokens)
            return fail(COTTUS_ERR_OUT_OF_RANGE, "sequence " + std::to_string(s.id) + " would exceed " +
                                                     std::to_string(cap_tokens) + " tokens (max_blocks_per_seq * block_size)");
    // a block for every row whose next token starts one (engine.cpp:73-77);
    // on exhaustion the step's allocations are undone in reverse order,
    // which restores the LIFO free list exactly
    std::vector<int32_t> grown;
    for (int32_t r = 0; r < (int32_t)b->rows.size(); ++r) {
        auto& s = b->rows[r];
        if (s.pos % b->d.block_size != 0) continue;
        int32_t blk;
        try {
            blk = b->alloc.allocateBlock();
        } catch (const std::exception& e) {
            for (auto it = grown.rbegin(); it != grown.rend(); ++it) {
                auto& g = b->rows[*it];
                b->alloc.freeBlock(g.blocks.back());
                g.blocks.pop_back();
            }
            return fail(COTTUS_ERR_OUT_OF_MEMORY, e.what());
        }
        s.blocks.push_back(blk);
        grown.push_back(r);
    }
    for (int32_t r : grown)
        b->pending.emplace_back(r * b->d.max_blocks_per_seq + (int32_t)b->rows[r].blocks.size() - 1,
                                b->rows[r].blocks.back());
    for (int32_t r = 0; r < (int32_t)b->rows.size(); ++r) b->pending.emplace_back(b->table_elems() + r, b->rows[r].pos);
    if (has_device(b)) {
        // one entry per index, the latest one (the kernel writes its entries in parallel)
        std::vector<std::pair<int32_t, int32_t>> send;
        send.reserve(b->pending.size());
        std::unordered_map<int32_t, bool> seen;
        for (auto it = b->pending.rbegin(); it != b->pending.rend(); ++it)
            if (seen.emplace(it->first, true).second) send.push_back(*it);
        cb200::TableUpdates u;
        size_t i = 0;
        while (i < send.size()) {
            u.n = 0;
            for (; i < send.size() && u.n < cb200::kMaxTableUpdates; ++i) {
                u.idx[u.n] = send[i].first;
                u.val[u.n] = send[i].second;
                ++u.n;
            }
            const cudaError_t e = cb200::launch_kernel(cb200::table_update_kernel, dim3(1), dim3(256), 0,
                                                       reinterpret_cast<cudaStream_t>(stream), u,
                                                       b->d.device_block_table, b->table_elems(),
                                                       b->d.device_positions, b->d.device_context_lens);
            if (e != cudaSuccess) return fail(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e));
        }
    }
    b->pending.clear();
    b->in_step = true;
    return COTTUS_OK;
}

int cottus_decode_batch_end_step(cottus_decode_batch* b) {
    if (!b) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL batch");
    if (!b->in_step) return fail(COTTUS_ERR_INVALID_ARGUMENT, "no step to end");
    for (auto& s : b->rows) ++s.pos;
    b->in_step = false;
    return COTTUS_OK;
}

int32_t cottus_decode_batch_size(const cottus_decode_batch* b) { return b ? (int32_t)b->rows.size() : 0; }

int32_t cottus_decode_batch_free_blocks(const cottus_decode_batch* b) { return b ? b->alloc.numFreeBlocks() : 0; }

int cottus_decode_batch_rows(const cottus_decode_batch* b, int64_t* seq_ids, int32_t cap) {
    if (!b || (!seq_ids && cap > 0)) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL argument");
    const int32_t n = std::min(cap, (int32_t)b->rows.size());
    for (int32_t r = 0; r < n; ++r) seq_ids[r] = b->rows[r].id;
    return (int32_t)b->rows.size();
}

int cottus_decode_batch_sequence(const cottus_decode_batch* b, int64_t seq_id, int32_t* row, int32_t* position,
                                 int32_t* blocks, int32_t cap, int32_t* num_blocks) {
    if (!b) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL batch");
    auto it = b->row_of.find(seq_id);
    if (it == b->row_of.end())
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "sequence " + std::to_string(seq_id) + " is not in the batch");
    const auto& s = b->rows[it->second];
    if (row) *row = it->second;
    if (position) *position = s.pos;
    if (num_blocks) *num_blocks = (int32_t)s.blocks.size();
    if (blocks)
        for (int32_t j = 0; j < std::min(cap, (int32_t)s.blocks.size()); ++j) blocks[j] = s.blocks[j];
    return COTTUS_OK;
}

}  // extern "C"
