// The steps either side of the attention path on the tensor cores: the QKV
// projection of each sequence's new token fused with RoPE on q and k and
// the KV-cache append (before), and the output projection fused with the
// residual add (after, generic_transformer.cpp:305-325).
//
// Replaces, per layer and token, generic_transformer.cpp:169-284: three
// gemmCUDA calls (cuBLAS SGEMM, compute_primitives_cuda.cu:30-55), two
// ropeCUDA calls, two device-to-host copies and the host-side truncating
// encode and scatter of k and v into the page of position `pos`.
//
// out[t][n] = sum_k x[t][k] * W[n][k] for the batch's tokens t (at most 64
// per launch, more are chunked by the host) and the stacked rows n of Wq,
// Wk, Wv.  The op streams the weights once, so HBM bandwidth bounds it:
//   * CTA tile: 128 weight rows x all tokens (padded to 16, 32 or 64), every
//     splits-th 64-wide k-step; grid = (rows/128) x splits, splits (at most
//     16) chosen so the grid fills one wave of two CTAs per SM;
//   * weights and activations staged by TMA in 64-element (128-byte) rows
//     with 128B swizzle through a 4-stage mbarrier ring (warp 0 produces;
//     two CTAs per SM);
//   * 5th-generation tensor cores: one thread of warp 1 issues
//     tcgen05.mma (kind::f16, M = 128 weight rows, N = tokens, K = 16, fp32
//     accumulator in tensor memory) straight from the swizzled tiles
//     through shared-memory matrix descriptors, and tcgen05.commit frees
//     each stage when its multiplies are done; the four warps then read the
//     accumulator rows of their 32 TMEM lanes with tcgen05.ld;
//   * each split writes its partial sums to the workspace; a second kernel
//     (programmatic dependent launch, one thread per (token, row pair))
//     adds the splits in order (deterministic), rotates q and k with the
//     (cos, sin) table of the reference formula (FMA-free, bit-identical to
//     ropeCPU on the same sums), writes the rotated query, and encodes k and
//     v by truncation into the pool.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "cottus_b200.h"
#include "decode_mma.cuh"
#include "internal.h"

namespace cb200 {
int set_error(int code, const std::string& msg);
CUtensorMap make_tensor_map_2d_f16(const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_bytes,
                                   uint32_t box_inner, uint32_t box_outer, bool swizzle128, cudaError_t* err);

namespace {

constexpr int kQRows = 128;  // weight rows per CTA tile (the MMA's M)
constexpr int kQK = 64;      // k elements per stage (one 128-byte swizzled row)
constexpr int kQStages = 4;  // ring depth (two CTAs per SM)
constexpr int kQThreads = 128;
constexpr int kQMaxTokens = 64;
constexpr int kQMaxSplits = 16;

struct QkvArgs {
    const uint16_t* w;
    int N, K, B, H, Hkv, D, bs, L, layer, maxb, max_pos;
    long long num_blocks;
    const int32_t* pos;
    const float* cos_sin;
    uint16_t* kv;
    const int32_t* bt;
    void* q_out;
    int q_out_f16;
    float* qkv_out;
    float* part;  // [splits][B][N]
    int splits, ksteps;
    uint32_t* status;
    const float* residual;  // O-projection: [B][N] added to the product
    void* out;              // O-projection: [B][N]
    int out_f16;
};

template <int BP>
constexpr size_t qkv_smem_bytes() {
    return (size_t)kQStages * (kQRows * kQK * 2 + BP * kQK * 2) + (2 * kQStages + 1) * 8 + 1024;
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with
// 128B swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart; the tile
// base 1024-byte aligned): start address >> 4, leading offset 1 (unused
// when swizzled), stride offset 1024 >> 4, descriptor version 1, layout
// SWIZZLE_128B (2).  A k-slice of 16 elements starts 32 bytes further.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_byte_addr) {
    return (uint64_t)((smem_byte_addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor of kind::f16: fp16 A and B, fp32 accumulator,
// both K-major, N = tokens, M = 128.
template <int N>
constexpr uint32_t f16_idesc() {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kQRows >> 4) << 24);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
template <int BP>
__global__ void __launch_bounds__(kQThreads) qkv_proj_kernel(const __grid_constant__ CUtensorMap wmap,
                                                              const __grid_constant__ CUtensorMap xmap,
                                                              const QkvArgs a) {
    constexpr int W_BYTES = kQRows * kQK * 2, X_BYTES = BP * kQK * 2, STAGE = W_BYTES + X_BYTES;
    constexpr uint32_t TMEM_COLS = BP < 32 ? 32 : BP;
    static_assert(STAGE % 1024 == 0, "stages must keep 1024-byte alignment for the 128B swizzle");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kQStages * STAGE);
    uint64_t* empty = full + kQStages;
    uint64_t* done = empty + kQStages;
    __shared__ uint32_t tmem_base;
    __shared__ int failed, issued, consumed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, split = blockIdx.y;
    const int row0 = tile * kQRows;
    // k-steps split, split + splits, ...: at any moment the splits of a row
    // tile read neighbouring 128-byte pieces of the same weight rows
    const int nsteps = split < a.ksteps ? (a.ksteps - split + a.splits - 1) / a.splits : 0;
    const int npre = nsteps < kQStages ? nsteps : kQStages;
    // (the finish kernel is released once this CTA's multiplies are done;
    // released at the start, with the finish kernels also releasing early, a
    // chained decode step measured up to 28 us slower; released at exit,
    // the O-projection took 12.6 us instead of 12.0 and the QKV step 17.9
    // instead of 17.2)

    if (threadIdx.x == 0) {
        prefetch_tensormap(&wmap);
        prefetch_tensormap(&xmap);
        for (int s = 0; s < kQStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        failed = 0;
        issued = consumed = 0;
        // the weights do not depend on the preceding kernel: the first stages'
        // tiles are requested before waiting for it
        for (int i = 0; i < npre; ++i) {
            mbar_arrive_expect_tx(&full[i], STAGE);
            tma_load_2d(smem + (size_t)i * STAGE, &wmap, &full[i], (split + i * a.splits) * kQK, row0);
        }
    }
    if (warp == 0) {  // accumulator: TMEM_COLS columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    grid_dependency_wait();  // the preceding kernel is complete: activations ready, workspace free

    if (threadIdx.x == 0) {
        // ---- producer: weights and activations of stage i ----------------
        for (int i = 0; i < nsteps; ++i) {
            const int slot = i % kQStages;
            if (i >= kQStages && !mbar_wait_bounded(&empty[slot], ((i / kQStages) - 1) & 1)) {
                failed = 1;
                break;
            }
            uint8_t* st = smem + (size_t)slot * STAGE;
            const int kx = (split + i * a.splits) * kQK;
            if (i >= npre) {
                mbar_arrive_expect_tx(&full[slot], STAGE);
                tma_load_2d(st, &wmap, &full[slot], kx, row0);
            }
            tma_load_2d(st + W_BYTES, &xmap, &full[slot], kx, 0);
            issued = i + 1;
        }
    } else if (threadIdx.x == 32) {
        // ---- MMA issue: D[128 rows][BP tokens] += W[rows][k] . X[tokens][k]^T
        constexpr uint32_t idesc = f16_idesc<BP>();
        for (int i = 0; i < nsteps; ++i) {
            const int slot = i % kQStages;
            if (!mbar_wait_bounded(&full[slot], (i / kQStages) & 1)) {
                failed = 1;
                break;
            }
            tc_fence_after();
            const uint32_t wa = smem_addr(smem + (size_t)slot * STAGE), xa = wa + W_BYTES;
#pragma unroll
            for (int kk = 0; kk < kQK / 16; ++kk) {
                const uint64_t ad = sw128_desc(wa + kk * 32), bd = sw128_desc(xa + kk * 32);
                const uint32_t accumulate = (i | kk) != 0;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem),
                    "l"(ad), "l"(bd), "r"(idesc), "r"(accumulate), "r"(0u)
                    : "memory");
            }
            // the stage is free once these multiplies have read it
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_addr(&empty[slot]))
                         : "memory");
            consumed = i + 1;
        }
        // every multiply issued so far is complete when `done` fires
        if (consumed > 0)
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_addr(done))
                         : "memory");
        else
            mbar_arrive(done);
    }
    __syncwarp();
    const bool got = mbar_wait_bounded(done, 0);
    tc_fence_after();
    const bool ok = __syncthreads_and(got) && !failed;
    // the finish kernel may become resident now; it waits for this grid
    // (grid_dependency_wait) before it reads a partial
    grid_dependents_launch();
    if (!ok && threadIdx.x == 0) {
        // report, let the copies still in flight land (bounded), and go on
        // with zero partials
        report(a.status, COTTUS_STATUS_TIMEOUT);
        // (the producer waits for nothing before it has requested the
        // activations of the prefetched stages, so issued >= npre)
        for (int i = consumed; i < issued; ++i) (void)mbar_wait_bounded(&full[i % kQStages], (i / kQStages) & 1);
    }
    __syncthreads();

    // ---- this split's partials: TMEM lane = weight row, column = token -------
    {
        const int r = row0 + warp * 32 + lane;
        float* p = a.part + (size_t)split * a.B * a.N;
#pragma unroll
        for (int c0 = 0; c0 < BP; c0 += 16) {
            uint32_t v[16];
            if (nsteps > 0 && ok) {
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15])
                    : "r"(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0u;  // an empty (or failed) split contributes zeros
            }
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (c0 + j < a.B) p[(size_t)(c0 + j) * a.N + r] = __uint_as_float(v[j]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// One thread per (token, row pair): the splits added in order, then RoPE,
// the rotated query and the append.
__global__ void __launch_bounds__(256) qkv_finish_kernel(const QkvArgs a) {
    // the next kernel may become resident now and run its prologue (a
    // projection prefetches its weights, a decode warms its first pages);
    // it waits for this grid before it reads anything this one writes
    grid_dependents_launch();
    grid_dependency_wait();  // the partials of the projection kernel are complete
    const int pairs_all = a.N / 2;
    const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (idx >= (long long)a.B * pairs_all) return;
    const int t = (int)(idx / pairs_all), n = 2 * (int)(idx % pairs_all);
    const int HD = a.H * a.D, KD = a.Hkv * a.D;
    const int p = a.pos[t];
    float2 pv[kQMaxSplits];
#pragma unroll
    for (int s = 0; s < kQMaxSplits; ++s)
        pv[s] = s < a.splits ? __ldcg(reinterpret_cast<const float2*>(a.part + ((size_t)s * a.B + t) * a.N + n))
                             : make_float2(0.f, 0.f);
    float v0 = 0.f, v1 = 0.f;
#pragma unroll
    for (int s = 0; s < kQMaxSplits; ++s)
        if (s < a.splits) {  // splits added in order
            v0 = __fadd_rn(v0, pv[s].x);
            v1 = __fadd_rn(v1, pv[s].y);
        }
    if (a.qkv_out) *reinterpret_cast<float2*>(a.qkv_out + (size_t)t * a.N + n) = make_float2(v0, v1);
    if (p < 0 || p >= a.max_pos || p >= a.maxb * a.bs) {
        if (n == 0) report(a.status, COTTUS_STATUS_BAD_POSITION);
        return;
    }
    const int d = n % a.D;
    if (n < HD + KD) {  // q or k: rotate the interleaved pair (d, d + 1)
        const float2 cs = *reinterpret_cast<const float2*>(a.cos_sin + ((size_t)p * (a.D / 2) + d / 2) * 2);
        rope_pair(v0, v1, cs.x, cs.y, v0, v1);
    }
    if (n < HD) {
        const size_t e = (size_t)t * HD + n;
        if (a.q_out_f16) {
            reinterpret_cast<__half*>(a.q_out)[e] = __float2half_rn(v0);
            reinterpret_cast<__half*>(a.q_out)[e + 1] = __float2half_rn(v1);
        } else {
            reinterpret_cast<float*>(a.q_out)[e] = v0;
            reinterpret_cast<float*>(a.q_out)[e + 1] = v1;
        }
        return;
    }
    const bool is_v = n >= HD + KD;
    const int kvh = (n - HD - (is_v ? KD : 0)) / a.D;
    const int blk = a.bt[(size_t)t * a.maxb + p / a.bs];
    if (blk < 0 || (long long)blk >= a.num_blocks) {
        if (n == HD) report(a.status, COTTUS_STATUS_BAD_BLOCK_ID);
        return;
    }
    // [block][layer][K|V][slot][kv head][dim] (generic_transformer.cpp:234-281)
    const size_t o = ((((size_t)blk * a.L + a.layer) * 2 + (is_v ? 1 : 0)) * a.bs + (p % a.bs)) * KD +
                     (size_t)kvh * a.D + d;
    a.kv[o] = f32_to_f16_trunc(v0);
    a.kv[o + 1] = f32_to_f16_trunc(v1);
}

// One thread per (token, column pair) of the O-projection: the splits added
// in order, then the residual (generic_transformer.cpp:305-325: x = att . Wo,
// then x = x + xb).
__global__ void __launch_bounds__(256) oproj_finish_kernel(const QkvArgs a) {
    grid_dependents_launch();  // (as in qkv_finish_kernel)
    grid_dependency_wait();
    const int pairs_all = a.N / 2;
    const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (idx >= (long long)a.B * pairs_all) return;
    const int t = (int)(idx / pairs_all), n = 2 * (int)(idx % pairs_all);
    float2 pv[kQMaxSplits];
#pragma unroll
    for (int s = 0; s < kQMaxSplits; ++s)
        pv[s] = s < a.splits ? __ldcg(reinterpret_cast<const float2*>(a.part + ((size_t)s * a.B + t) * a.N + n))
                             : make_float2(0.f, 0.f);
    const float2 r = *reinterpret_cast<const float2*>(a.residual + (size_t)t * a.N + n);
    float v0 = 0.f, v1 = 0.f;
#pragma unroll
    for (int s = 0; s < kQMaxSplits; ++s)
        if (s < a.splits) {
            v0 = __fadd_rn(v0, pv[s].x);
            v1 = __fadd_rn(v1, pv[s].y);
        }
    v0 = __fadd_rn(v0, r.x);
    v1 = __fadd_rn(v1, r.y);
    const size_t e = (size_t)t * a.N + n;
    if (a.out_f16) {
        reinterpret_cast<__half*>(a.out)[e] = __float2half_rn(v0);
        reinterpret_cast<__half*>(a.out)[e + 1] = __float2half_rn(v1);
    } else {
        *reinterpret_cast<float2*>(reinterpret_cast<float*>(a.out) + e) = make_float2(v0, v1);
    }
}

template <int BP, bool QKV>
cudaError_t launch_proj(const CUtensorMap& wmap, const CUtensorMap& xmap, const QkvArgs& a, int row_tiles,
                        cudaStream_t st) {
    auto kern = qkv_proj_kernel<BP>;
    const size_t smem = qkv_smem_bytes<BP>();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(row_tiles, a.splits);
    cfg.blockDim = dim3(kQThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, wmap, xmap, a);
    if (e != cudaSuccess) return e;
    const long long items = (long long)a.B * (a.N / 2);
    cudaLaunchConfig_t fc = cfg;
    fc.gridDim = dim3((unsigned)((items + 255) / 256));
    fc.blockDim = dim3(256);
    fc.dynamicSmemBytes = 0;
    if constexpr (QKV) return cudaLaunchKernelEx(&fc, qkv_finish_kernel, a);
    else return cudaLaunchKernelEx(&fc, oproj_finish_kernel, a);
}

// Resident CTAs per SM: the SM's shared memory (the kernel asks for the
// largest carveout) over what one CTA takes, dynamic + static + the block
// reserve; 128 threads and a few dozen registers never bind first.
template <int BP>
int ctas_per_sm(int dev) {
    static int cache[64] = {};
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    auto kern = qkv_proj_kernel<BP>;
    const size_t smem = qkv_smem_bytes<BP>();
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    cudaFuncAttributes fa = {};
    int sm_smem = 0, reserve = 0;
    int n = 1;
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess &&
        cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&reserve, cudaDevAttrReservedSharedMemoryPerBlock, dev) == cudaSuccess)
        n = (int)((size_t)sm_smem / (smem + fa.sharedSizeBytes + (size_t)reserve));
    if (n < 1) n = 1;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}

// Splits of K so that the grid fills one wave, at most kQMaxSplits.
template <int BP>
int splits_for(int row_tiles, int ksteps) {
    int dev = 0;
    cudaGetDevice(&dev);
    int s = device_sm_count(dev) * ctas_per_sm<BP>(dev) / row_tiles;
    if (s > kQMaxSplits) s = kQMaxSplits;
    if (s > ksteps) s = ksteps;
    return s < 1 ? 1 : s;
}

int splits_for_tokens(int BP, int row_tiles, int ksteps) {
    return BP == 16 ? splits_for<16>(row_tiles, ksteps)
                    : (BP == 32 ? splits_for<32>(row_tiles, ksteps) : splits_for<64>(row_tiles, ksteps));
}

int fail(int code, const std::string& msg) { return set_error(code, msg); }

}  // namespace

}  // namespace cb200

extern "C" {

size_t cottus_qkv_rope_append_workspace_size(const cottus_qkv_params* p) {
    using namespace cb200;
    if (!p || p->batch <= 0 || p->hidden <= 0 || p->head_dim <= 0) return 0;
    const long long N = (long long)(p->num_heads + 2 * p->num_kv_heads) * p->head_dim;
    const int row_tiles = (int)(N / kQRows), ksteps = p->hidden / kQK;
    if (row_tiles <= 0 || ksteps <= 0) return 0;
    const int B = p->batch < kQMaxTokens ? p->batch : kQMaxTokens;
    const int BP = B <= 16 ? 16 : (B <= 32 ? 32 : 64);
    const int S = splits_for_tokens(BP, row_tiles, ksteps);
    return (size_t)S * B * N * sizeof(float);  // split partials of one launch of at most 64 tokens
}

int cottus_qkv_rope_append(const cottus_qkv_params* p, cottus_stream_t stream) {
    using namespace cb200;
    if (!p) return fail(COTTUS_ERR_INVALID_ARGUMENT, "params must not be NULL");
    if (p->batch < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0 || p->head_dim <= 0 || p->block_size <= 0 ||
        p->num_layers <= 0 || p->layer < 0 || p->layer >= p->num_layers || p->max_blocks_per_seq <= 0 ||
        p->hidden <= 0 || p->max_position <= 0)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "invalid dimensions");
    if (p->batch == 0) return COTTUS_OK;
    const long long N = (long long)(p->num_heads + 2 * p->num_kv_heads) * p->head_dim;
    if (p->hidden % kQK != 0 || N % kQRows != 0 || (p->head_dim % 2) != 0)
        return fail(COTTUS_ERR_UNSUPPORTED, "hidden must be a multiple of 64, the stacked q/k/v rows a multiple of 128, "
                                            "and head_dim even");
    if (N >= (1LL << 31) / 2) return fail(COTTUS_ERR_UNSUPPORTED, "projection too large");
    if (!p->x || !p->weight || !p->positions || !p->cos_sin || !p->kv_pool || !p->block_table || !p->query_out)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL pointer argument");
    if ((reinterpret_cast<uintptr_t>(p->x) | reinterpret_cast<uintptr_t>(p->weight)) & 15)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "x and weight must be 16-byte aligned");
    if (p->query_out_dtype != COTTUS_F16 && p->query_out_dtype != COTTUS_F32)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "unknown dtype");
    const size_t need = cottus_qkv_rope_append_workspace_size(p);
    if (!p->workspace || p->workspace_bytes < need || (reinterpret_cast<uintptr_t>(p->workspace) & 15))
        return fail(COTTUS_ERR_WORKSPACE, "workspace missing, unaligned or smaller than the required " +
                                              std::to_string(need) + " bytes");
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int row_tiles = (int)(N / kQRows), ksteps = p->hidden / kQK;
    cudaError_t err = cudaSuccess;
    const CUtensorMap wmap = make_tensor_map_2d_f16(p->weight, p->hidden, N, (uint64_t)p->hidden * 2, kQK, kQRows,
                                                    true, &err);
    if (err != cudaSuccess) return fail(COTTUS_ERR_CUDA, "weight tensor map rejected");
    for (int b0 = 0; b0 < p->batch; b0 += kQMaxTokens) {
        const int B = p->batch - b0 < kQMaxTokens ? p->batch - b0 : kQMaxTokens;
        const int BP = B <= 16 ? 16 : (B <= 32 ? 32 : 64);
        const CUtensorMap xmap = make_tensor_map_2d_f16(static_cast<const __half*>(p->x) + (size_t)b0 * p->hidden,
                                                        p->hidden, B, (uint64_t)p->hidden * 2, kQK, BP, true, &err);
        if (err != cudaSuccess) return fail(COTTUS_ERR_CUDA, "activation tensor map rejected");
        QkvArgs a;
        a.w = static_cast<const uint16_t*>(p->weight);
        a.N = (int)N;
        a.K = p->hidden;
        a.B = B;
        a.H = p->num_heads;
        a.Hkv = p->num_kv_heads;
        a.D = p->head_dim;
        a.bs = p->block_size;
        a.L = p->num_layers;
        a.layer = p->layer;
        a.maxb = p->max_blocks_per_seq;
        a.max_pos = p->max_position;
        a.num_blocks = p->num_physical_blocks;
        a.pos = p->positions + b0;
        a.cos_sin = p->cos_sin;
        a.kv = p->kv_pool;
        a.bt = p->block_table + (size_t)b0 * p->max_blocks_per_seq;
        const size_t qe = p->query_out_dtype == COTTUS_F16 ? 2 : 4;
        a.q_out = static_cast<uint8_t*>(p->query_out) + (size_t)b0 * p->num_heads * p->head_dim * qe;
        a.q_out_f16 = p->query_out_dtype == COTTUS_F16;
        a.qkv_out = p->qkv_out ? p->qkv_out + (size_t)b0 * N : nullptr;
        const int S = splits_for_tokens(BP, row_tiles, ksteps);
        a.part = static_cast<float*>(p->workspace);
        a.splits = S;
        a.ksteps = ksteps;
        a.status = p->status;
        a.residual = nullptr;
        a.out = nullptr;
        a.out_f16 = 0;
        if (BP == 16) err = launch_proj<16, true>(wmap, xmap, a, row_tiles, st);
        else if (BP == 32) err = launch_proj<32, true>(wmap, xmap, a, row_tiles, st);
        else err = launch_proj<64, true>(wmap, xmap, a, row_tiles, st);
        if (err != cudaSuccess) return fail(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    }
    return COTTUS_OK;
}

size_t cottus_o_proj_residual_workspace_size(const cottus_o_proj_params* p) {
    using namespace cb200;
    if (!p || p->batch <= 0 || p->in_features <= 0 || p->out_features <= 0) return 0;
    const int row_tiles = p->out_features / kQRows, ksteps = p->in_features / kQK;
    if (row_tiles <= 0 || ksteps <= 0) return 0;
    const int B = p->batch < kQMaxTokens ? p->batch : kQMaxTokens;
    const int BP = B <= 16 ? 16 : (B <= 32 ? 32 : 64);
    const int S = splits_for_tokens(BP, row_tiles, ksteps);
    return (size_t)S * B * p->out_features * sizeof(float);
}

int cottus_o_proj_residual(const cottus_o_proj_params* p, cottus_stream_t stream) {
    using namespace cb200;
    if (!p) return fail(COTTUS_ERR_INVALID_ARGUMENT, "params must not be NULL");
    if (p->batch < 0 || p->in_features <= 0 || p->out_features <= 0)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "invalid dimensions");
    if (p->batch == 0) return COTTUS_OK;
    if (p->in_features % kQK != 0 || p->out_features % kQRows != 0)
        return fail(COTTUS_ERR_UNSUPPORTED, "in_features must be a multiple of 64 and out_features of 128");
    if (!p->x || !p->weight || !p->residual || !p->out) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL pointer argument");
    if ((reinterpret_cast<uintptr_t>(p->x) | reinterpret_cast<uintptr_t>(p->weight) |
         reinterpret_cast<uintptr_t>(p->residual) | reinterpret_cast<uintptr_t>(p->out)) & 15)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "x, weight, residual and out must be 16-byte aligned");
    if (p->out_dtype != COTTUS_F16 && p->out_dtype != COTTUS_F32)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "unknown dtype");
    const size_t need = cottus_o_proj_residual_workspace_size(p);
    if (!p->workspace || p->workspace_bytes < need || (reinterpret_cast<uintptr_t>(p->workspace) & 15))
        return fail(COTTUS_ERR_WORKSPACE, "workspace missing, unaligned or smaller than the required " +
                                              std::to_string(need) + " bytes");
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int N = p->out_features, K = p->in_features, row_tiles = N / kQRows, ksteps = K / kQK;
    cudaError_t err = cudaSuccess;
    const CUtensorMap wmap = make_tensor_map_2d_f16(p->weight, K, N, (uint64_t)K * 2, kQK, kQRows, true, &err);
    if (err != cudaSuccess) return fail(COTTUS_ERR_CUDA, "weight tensor map rejected");
    const size_t oe = p->out_dtype == COTTUS_F16 ? 2 : 4;
    for (int b0 = 0; b0 < p->batch; b0 += kQMaxTokens) {
        const int B = p->batch - b0 < kQMaxTokens ? p->batch - b0 : kQMaxTokens;
        const int BP = B <= 16 ? 16 : (B <= 32 ? 32 : 64);
        const CUtensorMap xmap = make_tensor_map_2d_f16(static_cast<const __half*>(p->x) + (size_t)b0 * K, K, B,
                                                        (uint64_t)K * 2, kQK, BP, true, &err);
        if (err != cudaSuccess) return fail(COTTUS_ERR_CUDA, "activation tensor map rejected");
        QkvArgs a = {};
        a.w = static_cast<const uint16_t*>(p->weight);
        a.N = N;
        a.K = K;
        a.B = B;
        a.part = static_cast<float*>(p->workspace);
        const int S = splits_for_tokens(BP, row_tiles, ksteps);
        a.splits = S;
        a.ksteps = ksteps;
        a.status = p->status;
        a.residual = p->residual + (size_t)b0 * N;
        a.out = static_cast<uint8_t*>(p->out) + (size_t)b0 * N * oe;
        a.out_f16 = p->out_dtype == COTTUS_F16;
        if (BP == 16) err = launch_proj<16, false>(wmap, xmap, a, row_tiles, st);
        else if (BP == 32) err = launch_proj<32, false>(wmap, xmap, a, row_tiles, st);
        else err = launch_proj<64, false>(wmap, xmap, a, row_tiles, st);
        if (err != cudaSuccess) return fail(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    }
    return COTTUS_OK;
}

}  // extern "C"
