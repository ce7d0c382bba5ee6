// Drop-in check of the same-signature C++ surface (cottus::PageTable,
// cottus::BlockAllocator, cottus::pagedAttentionCUDA, cottus::ropeCUDA),
// written the way the reference's own CTest programs are
// (tests/test_paged_attention_parity.cpp, tests/test_compute_primitives_parity.cpp):
// plain main(), checks, "PASS" lines.  The CPU side of every comparison is
// the oracle (oracle/oracle.c).  Needs a GPU; run by tests/test_shim_gpu.py.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <stdexcept>
#include <vector>

#include "cottus/block_allocator.h"
#include "cottus/compute_primitives_cuda.h"
#include "cottus/page_table.h"
#include "cottus/paged_attention_cuda.h"
#include "oracle.h"

#define CHECK(c)                                                              \
    do {                                                                      \
        if (!(c)) {                                                           \
            std::fprintf(stderr, "FAILED %s at %s:%d\n", #c, __FILE__, __LINE__); \
            std::exit(1);                                                     \
        }                                                                     \
    } while (0)

using namespace cottus;

static uint16_t enc(float f) { return oracle_fp32_to_fp16_trunc(f); }

static float max_diff(const std::vector<float>& a, const std::vector<float>& b) {
    float m = 0.f;
    for (size_t i = 0; i < a.size(); ++i) m = std::fmax(m, std::fabs(a[i] - b[i]));
    return m;
}

static void test_single_head() {
    // tests/test_paged_attention_parity.cpp:28-78
    const int H = 1, Hkv = 1, D = 4, bs = 2, n = 2;
    std::vector<float> q = {1, 0, 0, 0};
    std::vector<uint16_t> kv(16, enc(0.f));
    kv[0] = enc(1.f);
    kv[5] = enc(1.f);
    for (int i = 0; i < 4; ++i) kv[8 + i] = enc(1.f), kv[12 + i] = enc(2.f);
    PageTable pt(bs);
    pt.appendBlock(0);
    std::vector<float> gpu(H * D), cpu(H * D);
    pagedAttentionCUDA(gpu.data(), q.data(), kv.data(), pt, n, 0, H, Hkv, D, bs, 1);
    int32_t table[] = {0};
    CHECK(oracle_paged_attention(cpu.data(), q.data(), kv.data(), table, 1, n, 0, H, Hkv, D, bs, 1) == 0);
    CHECK(max_diff(gpu, cpu) < 1e-5f);
    CHECK(std::fabs(gpu[0] - 1.378f) < 0.01f);
    std::puts("PASS: single head, single block");
}

static void test_gqa_shuffled_multilayer() {
    // GQA (group 4), shuffled table, 3 layers, context not a multiple of the block
    const int H = 16, Hkv = 4, D = 128, bs = 16, L = 3, layer = 2, n = 150;
    const int nblk = (n + bs - 1) / bs, pool_blocks = nblk + 5;
    std::mt19937 rng(7);
    std::normal_distribution<float> nd;
    std::vector<uint16_t> kv((size_t)pool_blocks * 2 * L * bs * Hkv * D);
    for (auto& x : kv) x = enc(nd(rng));
    std::vector<float> q(H * D);
    for (auto& x : q) x = nd(rng);
    std::vector<int32_t> perm(pool_blocks);
    for (int i = 0; i < pool_blocks; ++i) perm[i] = i;
    std::shuffle(perm.begin(), perm.end(), rng);
    PageTable pt(bs);
    for (int i = 0; i < nblk; ++i) pt.appendBlock(perm[i]);
    std::vector<float> gpu(H * D), cpu(H * D);
    pagedAttentionCUDA(gpu.data(), q.data(), kv.data(), pt, n, layer, H, Hkv, D, bs, L);
    CHECK(oracle_paged_attention(cpu.data(), q.data(), kv.data(), perm.data(), nblk, n, layer, H, Hkv, D, bs, L) == 0);
    CHECK(max_diff(gpu, cpu) < 1e-5f);
    std::puts("PASS: GQA, shuffled table, layer 2 of 3");
}

static void test_errors() {
    PageTable pt(16);
    pt.appendBlock(0);
    std::vector<float> q(4), o(4);
    std::vector<uint16_t> kv(2 * 16 * 4);
    bool threw = false;
    try {
        pagedAttentionCUDA(o.data(), q.data(), kv.data(), pt, 0, 0, 1, 1, 4, 16, 1);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    CHECK(threw);
    threw = false;
    try {
        pagedAttentionCUDA(o.data(), q.data(), kv.data(), pt, 17, 0, 1, 1, 4, 16, 1);  // past the table
    } catch (const std::out_of_range&) {
        threw = true;
    }
    CHECK(threw);
    threw = false;
    try {
        pt.getBlock(3);
    } catch (const std::out_of_range&) {
        threw = true;
    }
    CHECK(threw);
    BlockAllocator a(2, 16);
    CHECK(a.allocateBlock() == 0);
    CHECK(a.allocateBlock() == 1);
    threw = false;
    try {
        a.allocateBlock();
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw);
    std::puts("PASS: exceptions");
}

static void test_determinism() {
    // tests/test_paged_attention_parity.cpp:178-215
    const int H = 2, Hkv = 2, D = 4, bs = 2, n = 3;
    std::vector<float> q(H * D, 1.f);
    std::vector<uint16_t> kv(2 * 2 * bs * Hkv * D, enc(1.f));
    PageTable pt(bs);
    pt.appendBlock(0);
    pt.appendBlock(1);
    std::vector<float> ref(H * D), o(H * D);
    pagedAttentionCUDA(ref.data(), q.data(), kv.data(), pt, n, 0, H, Hkv, D, bs, 1);
    for (int r = 0; r < 9; ++r) {
        pagedAttentionCUDA(o.data(), q.data(), kv.data(), pt, n, 0, H, Hkv, D, bs, 1);
        for (int i = 0; i < H * D; ++i) CHECK(o[i] == ref[i]);
    }
    std::puts("PASS: 10 runs bitwise identical");
}

static void test_rope() {
    // tests/test_compute_primitives_parity.cpp:118-160, compared bit for bit
    for (int trial = 0; trial < 3; ++trial) {
        const int H = trial == 0 ? 2 : 8, D = trial == 0 ? 8 : (trial == 1 ? 64 : 300), pos = trial == 0 ? 5 : 1234;
        const int N = H * D;
        std::vector<float> in(N), cpu(N), gpu(N);
        for (int i = 0; i < N; ++i) in[i] = (i % 10) * 0.1f - (trial ? 0.37f : 0.f);
        oracle_rope(cpu.data(), in.data(), pos, H, D, 10000.0f);
        float *d_in = nullptr, *d_out = nullptr;
        CHECK(cudaMalloc(&d_in, N * sizeof(float)) == cudaSuccess);
        CHECK(cudaMalloc(&d_out, N * sizeof(float)) == cudaSuccess);
        CHECK(cudaMemcpy(d_in, in.data(), N * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess);
        ropeCUDA(d_out, d_in, pos, H, D);
        ropeCUDA(d_in, d_in, pos, H, D);  // in place, as generic_transformer.cpp:197 calls it
        CHECK(cudaMemcpy(gpu.data(), d_out, N * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess);
        for (int i = 0; i < N; ++i) CHECK(gpu[i] == cpu[i]);
        CHECK(cudaMemcpy(gpu.data(), d_in, N * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess);
        for (int i = 0; i < N; ++i) CHECK(gpu[i] == cpu[i]);
        cudaFree(d_in);
        cudaFree(d_out);
    }
    std::puts("PASS: ropeCUDA == ropeCPU bit for bit");
}

int main() {
    test_single_head();
    test_gqa_shuffled_multilayer();
    test_errors();
    test_determinism();
    test_rope();
    std::puts("ALL PASS");
    return 0;
}
