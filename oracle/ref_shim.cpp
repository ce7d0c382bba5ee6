// C-linkage wrappers over the reference's own CPU code (cottus-runtime,
// cottus/csrc/{paged_attention_cpu,page_table,block_allocator,
// compute_primitives_cpu}.cpp), compiled from the reference tree by
// oracle/Makefile into oracle/_ref/libcottus_ref.so.
//
// TEST INFRASTRUCTURE ONLY: lets tests pin the C restatement (oracle.c)
// against the reference itself and lets bench.py time the reference CPU path.
// Exceptions are mapped to the oracle's status codes:
//   std::invalid_argument -> -1, std::out_of_range -> -2, other -> -3.
#include <cstdint>
#include <stdexcept>
#include <thread>
#include <vector>

#include "block_allocator.h"
#include "compute_primitives_cpu.h"
#include "page_table.h"
#include "paged_attention_cpu.h"

namespace {
template <class F>
int guarded(F &&f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument &) {
        return -1;
    } catch (const std::out_of_range &) {
        return -2;
    } catch (...) {
        return -3;
    }
}
}  // namespace

extern "C" {

// cottus::pagedAttentionCPU (paged_attention_cpu.cpp:24-103) for one sequence;
// block_table[0..n) is appended to a reference PageTable first.
int ref_paged_attention_cpu(float *out, const float *query, const void *kv, const int32_t *block_table,
                            int32_t num_table_blocks, int32_t seq_len, int32_t layer, int32_t num_heads,
                            int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                            int32_t num_layers) {
    return guarded([&] {
        cottus::PageTable pt(block_size);
        for (int32_t i = 0; i < num_table_blocks; ++i) pt.appendBlock(block_table[i]);
        cottus::pagedAttentionCPU(out, query, kv, pt, seq_len, layer, num_heads, num_kv_heads, head_dim,
                                  block_size, num_layers);
    });
}

// Batch of sequences spread over `threads` host threads (the reference itself
// is single-threaded; the thread split is the harness's, by sequence).
// kv_bases[b] lets the caller rebase each sequence's pool so the reference's
// int32 offsets stay in range (block ids in block_table are relative to it).
int ref_paged_attention_cpu_batch(float *out, const float *query, const void *const *kv_bases,
                                  const int32_t *block_table, int32_t max_blocks,
                                  const int32_t *context_lens, int32_t batch, int32_t layer,
                                  int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                  int32_t block_size, int32_t num_layers, int32_t threads) {
    if (threads < 1) threads = 1;
    std::vector<int> rcs(batch, 0);
    const int64_t stride = static_cast<int64_t>(num_heads) * head_dim;
    auto work = [&](int tid) {
        for (int32_t b = tid; b < batch; b += threads) {
            int32_t nblk = (context_lens[b] + block_size - 1) / block_size;
            rcs[b] = ref_paged_attention_cpu(out + b * stride, query + b * stride, kv_bases[b],
                                             block_table + static_cast<int64_t>(b) * max_blocks, nblk,
                                             context_lens[b], layer, num_heads, num_kv_heads, head_dim,
                                             block_size, num_layers);
        }
    };
    if (threads == 1) {
        work(0);
    } else {
        std::vector<std::thread> pool;
        for (int t = 0; t < threads; ++t) pool.emplace_back(work, t);
        for (auto &th : pool) th.join();
    }
    for (int rc : rcs)
        if (rc != 0) return rc;
    return 0;
}

// cottus::ropeCPU (compute_primitives_cpu.cpp:46-73).
// cottus::gemmCPU (compute_primitives_cpu.cpp:6-23): C[M][N] = A[M][K] B[K][N].
void ref_gemm_cpu(float *c, const float *a, const float *b, int32_t m, int32_t n, int32_t k) {
    cottus::gemmCPU(c, a, b, m, n, k);
}

void ref_rope_cpu(float *out, const float *in, int32_t pos, int32_t num_heads, int32_t head_dim,
                  float theta) {
    cottus::ropeCPU(out, in, pos, num_heads, head_dim, theta);
}

// cottus::BlockAllocator (block_allocator.cpp:7-55).
void *ref_allocator_create(int32_t total_blocks, int32_t block_size) {
    try {
        return new cottus::BlockAllocator(total_blocks, block_size);
    } catch (...) {
        return nullptr;
    }
}
void ref_allocator_destroy(void *a) { delete static_cast<cottus::BlockAllocator *>(a); }
// Returns the block id, or -3 on "Out of memory".
int32_t ref_allocator_alloc(void *a) {
    try {
        return static_cast<cottus::BlockAllocator *>(a)->allocateBlock();
    } catch (...) {
        return -3;
    }
}
int ref_allocator_free(void *a, int32_t id) {
    return guarded([&] { static_cast<cottus::BlockAllocator *>(a)->freeBlock(id); });
}
int32_t ref_allocator_num_free(void *a) { return static_cast<cottus::BlockAllocator *>(a)->numFreeBlocks(); }

// cottus::PageTable bounds behaviour (page_table.cpp:18-26): returns the
// block id or -2 when getBlock throws std::out_of_range.
int32_t ref_page_table_get(const int32_t *blocks, int32_t n, int32_t block_size, int32_t idx) {
    try {
        cottus::PageTable pt(block_size);
        for (int32_t i = 0; i < n; ++i) pt.appendBlock(blocks[i]);
        return pt[idx];
    } catch (const std::out_of_range &) {
        return -2;
    } catch (...) {
        return -3;
    }
}

}  // extern "C"
