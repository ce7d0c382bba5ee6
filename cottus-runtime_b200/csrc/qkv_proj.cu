// The step before the attention path, fused: QKV projection of each
// sequence's new token, RoPE on q and k, and the KV-cache append.
//
// Replaces, per layer and token, generic_transformer.cpp:169-284: three
// gemmCUDA calls (cuBLAS SGEMM, compute_primitives_cuda.cu:30-55), two
// ropeCUDA calls, two device-to-host copies and the host-side truncating
// encode and scatter of k and v into the page of position `pos`.
//
// out[t][n] = sum_k x[t][k] * W[n][k] for the batch's tokens t (at most 64
// per launch, more are chunked by the host) and the stacked rows n of Wq,
// Wk, Wv.  The op streams the weights once, so HBM bandwidth bounds it:
//   * CTA tile: 64 weight rows x all tokens, a split of the K range; grid =
//     (rows/64) x splits, splits chosen so the grid covers the SMs twice;
//   * weights and activations staged by TMA in 64-element (128-byte) rows
//     with 128B swizzle through a 6-stage mbarrier ring (one producer
//     thread, per-stage full/empty barriers);
//   * each warp multiplies 16 weight rows by all tokens on the tensor cores
//     (mma.sync m16n8k16, fp16 in, fp32 accumulate; A = weights by ldmatrix,
//     B = activations by ldmatrix, both from the swizzled tiles);
//   * split partial sums go to the workspace; the last CTA of a row tile to
//     finish (epoch-tagged counter) adds them in split order (deterministic),
//     rotates q and k with the (cos, sin) table of the reference formula
//     (FMA-free, bit-identical to ropeCPU on the same sums), writes the
//     rotated query, and encodes k and v by truncation into the pool.
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

constexpr int kQRows = 64;   // weight rows per CTA tile
constexpr int kQK = 64;      // k elements per stage (one 128-byte swizzled row)
constexpr int kQStages = 6;  // ring depth
constexpr int kQThreads = 128;
constexpr int kQMaxTokens = 64;

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
    float* part;                    // [splits][B][N]
    unsigned long long* counters;   // [row tiles]
    unsigned epoch;
    int splits, ksteps, ks_per_split;
    uint32_t* status;
};

template <int BP>
constexpr size_t qkv_smem_bytes() {
    return (size_t)kQStages * (kQRows * kQK * 2 + BP * kQK * 2) + 2 * kQStages * 8 + 1024;
}

template <int BP>
__global__ void __launch_bounds__(kQThreads) qkv_proj_kernel(const __grid_constant__ CUtensorMap wmap,
                                                              const __grid_constant__ CUtensorMap xmap,
                                                              const QkvArgs a) {
    constexpr unsigned FULL = 0xffffffffu;
    constexpr int W_BYTES = kQRows * kQK * 2, X_BYTES = BP * kQK * 2, STAGE = W_BYTES + X_BYTES;
    constexpr int NT = BP / 8;  // token tiles of 8
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kQStages * STAGE);
    uint64_t* empty = full + kQStages;
    __shared__ int last_tile;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, split = blockIdx.y;
    const int row0 = tile * kQRows;
    const int k0 = split * a.ks_per_split;
    const int k1 = min(k0 + a.ks_per_split, a.ksteps);
    const int nsteps = k1 > k0 ? k1 - k0 : 0;

    if (threadIdx.x == 0) {
        prefetch_tensormap(&wmap);
        prefetch_tensormap(&xmap);
        for (int s = 0; s < kQStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kQThreads / 32);
        }
        fence_barrier_init();
    }
    __syncthreads();
    grid_dependency_wait();
    grid_dependents_launch();

    auto issue = [&](int i) {  // thread 0: stage i of this split
        const int slot = i % kQStages;
        uint8_t* st = smem + (size_t)slot * STAGE;
        mbar_arrive_expect_tx(&full[slot], STAGE);
        const int kx = (k0 + i) * kQK;
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                smem_addr(st)),
            "l"(reinterpret_cast<uint64_t>(&wmap)), "r"(kx), "r"(row0), "r"(smem_addr(&full[slot]))
            : "memory");
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                smem_addr(st + W_BYTES)),
            "l"(reinterpret_cast<uint64_t>(&xmap)), "r"(kx), "r"(0), "r"(smem_addr(&full[slot]))
            : "memory");
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < nsteps && i < kQStages; ++i) issue(i);

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

    bool ok = true;
    int consumed = 0;
    for (int i = 0; i < nsteps; ++i) {
        const int slot = i % kQStages;
        ok = __all_sync(FULL, mbar_wait_bounded(&full[slot], (i / kQStages) & 1));
        if (!ok) break;
        const uint32_t ws = smem_addr(smem + (size_t)slot * STAGE), xs = ws + W_BYTES;
#pragma unroll
        for (int kk = 0; kk < kQK / 16; ++kk) {
            uint32_t af[4];
            {
                const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                ldsm_x4(ws + swz(0, row, kk * 2 + (lane >> 4)), af);
            }
#pragma unroll
            for (int jp = 0; jp < NT / 2; ++jp) {
                uint32_t bf[4];
                const int tok = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
                ldsm_x4(xs + swz(0, tok, kk * 2 + ((lane >> 3) & 1)), bf);
                mma16816(acc[2 * jp], af, bf[0], bf[1]);
                mma16816(acc[2 * jp + 1], af, bf[2], bf[3]);
            }
        }
        __syncwarp();
        consumed = i + 1;
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (threadIdx.x == 0 && i + kQStages < nsteps) {
            // the slot is free once every warp has read it
            ok = mbar_wait_bounded(&empty[slot], (i / kQStages) & 1);
            if (ok) {
                fence_proxy_async_smem();
                issue(i + kQStages);
            }
        }
        ok = __all_sync(FULL, ok);
        if (!ok) break;
    }
    if (!__syncthreads_and(ok)) {
        if (threadIdx.x == 0) {
            report(a.status, COTTUS_STATUS_TIMEOUT);
            // let the copies still in flight land (bounded) before the CTA leaves
            const int issued = min(nsteps, consumed + kQStages);
            for (int i = consumed; i < issued; ++i) (void)mbar_wait_bounded(&full[i % kQStages], (i / kQStages) & 1);
        }
        return;
    }

    // ---- split partials: C fragment rows are weight rows, columns tokens ----
    {
        const int r = row0 + warp * 16 + (lane >> 2);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int t = j * 8 + (lane & 3) * 2;
            float* p = a.part + (size_t)split * a.B * a.N;
            if (t < a.B) {
                p[(size_t)t * a.N + r] = acc[j][0];
                p[(size_t)t * a.N + r + 8] = acc[j][2];
            }
            if (t + 1 < a.B) {
                p[(size_t)(t + 1) * a.N + r] = acc[j][1];
                p[(size_t)(t + 1) * a.N + r + 8] = acc[j][3];
            }
        }
    }
    // ---- the last split of this row tile finishes it ------------------------
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int last = 1;
        if (a.splits > 1) {
            unsigned long long* ctr = a.counters + tile;
            unsigned long long old = 0;
            while (true) {  // each failure means another split arrived: at most `splits` rounds
                const unsigned long long nv =
                    (unsigned)(old >> 32) == a.epoch ? old + 1 : (((unsigned long long)a.epoch << 32) | 1ull);
                const unsigned long long prev = atomicCAS(ctr, old, nv);
                if (prev == old) {
                    last = (int)(nv & 0xffffffffull) == a.splits;
                    break;
                }
                old = prev;
            }
            if (last) __threadfence();
        }
        last_tile = last;
    }
    __syncthreads();
    if (!last_tile) return;

    const int pairs = kQRows / 2;
    const int HD = a.H * a.D, KD = a.Hkv * a.D;
    for (int idx = threadIdx.x; idx < a.B * pairs; idx += kQThreads) {
        const int t = idx / pairs, n = row0 + 2 * (idx % pairs);
        float v0 = 0.f, v1 = 0.f;
        for (int s = 0; s < a.splits; ++s) {
            const float2 pv = __ldcg(reinterpret_cast<const float2*>(a.part + ((size_t)s * a.B + t) * a.N + n));
            v0 = __fadd_rn(v0, pv.x);
            v1 = __fadd_rn(v1, pv.y);
        }
        if (a.qkv_out) *reinterpret_cast<float2*>(a.qkv_out + (size_t)t * a.N + n) = make_float2(v0, v1);
        const int p = a.pos[t];
        if (p < 0 || p >= a.max_pos || p >= a.maxb * a.bs) {
            if ((idx % pairs) == 0) report(a.status, COTTUS_STATUS_BAD_POSITION);
            continue;
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
            continue;
        }
        const bool is_v = n >= HD + KD;
        const int kvh = (n - HD - (is_v ? KD : 0)) / a.D;
        const int blk = a.bt[(size_t)t * a.maxb + p / a.bs];
        if (blk < 0 || (long long)blk >= a.num_blocks) {
            if ((idx % pairs) == 0) report(a.status, COTTUS_STATUS_BAD_BLOCK_ID);
            continue;
        }
        // [block][layer][K|V][slot][kv head][dim] (generic_transformer.cpp:234-281)
        const size_t off = ((((size_t)blk * a.L + a.layer) * 2 + (is_v ? 1 : 0)) * a.bs + (p % a.bs)) * KD +
                           (size_t)kvh * a.D + d;
        a.kv[off] = f32_to_f16_trunc(v0);
        a.kv[off + 1] = f32_to_f16_trunc(v1);
    }
}

template <int BP>
cudaError_t launch_qkv(const CUtensorMap& wmap, const CUtensorMap& xmap, const QkvArgs& a, int row_tiles,
                       cudaStream_t st) {
    auto kern = qkv_proj_kernel<BP>;
    const size_t smem = qkv_smem_bytes<BP>();
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr_set[dev] = true;
    }
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
    return cudaLaunchKernelEx(&cfg, kern, wmap, xmap, a);
}

int splits_for(int row_tiles, int ksteps, int sms) {
    int s = (2 * sms + row_tiles - 1) / row_tiles;
    if (s < 1) s = 1;
    if (s > ksteps) s = ksteps;
    return s;
}

int fail(int code, const std::string& msg) { return set_error(code, msg); }

}  // namespace

int device_sm_count(int device);
unsigned next_epoch();

}  // namespace cb200

extern "C" {

size_t cottus_qkv_rope_append_workspace_size(const cottus_qkv_params* p) {
    if (!p || p->batch <= 0 || p->hidden <= 0 || p->head_dim <= 0) return 0;
    const long long N = (long long)(p->num_heads + 2 * p->num_kv_heads) * p->head_dim;
    const int row_tiles = (int)(N / cb200::kQRows), ksteps = p->hidden / cb200::kQK;
    int dev = 0;
    cudaGetDevice(&dev);
    const int S = cb200::splits_for(row_tiles > 0 ? row_tiles : 1, ksteps > 0 ? ksteps : 1, cb200::device_sm_count(dev));
    const long long B = p->batch < cb200::kQMaxTokens ? p->batch : cb200::kQMaxTokens;
    return (((size_t)row_tiles * 8 + 255) & ~size_t(255)) + (size_t)S * B * N * sizeof(float);
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
        return fail(COTTUS_ERR_UNSUPPORTED, "hidden must be a multiple of 64, the stacked q/k/v rows a multiple of 64, "
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
    int dev = 0;
    cudaGetDevice(&dev);
    const int S = splits_for(row_tiles, ksteps, device_sm_count(dev));
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
        a.counters = static_cast<unsigned long long*>(p->workspace);
        a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(p->workspace) + (((size_t)row_tiles * 8 + 255) & ~size_t(255)));
        a.epoch = next_epoch();
        a.splits = S;
        a.ksteps = ksteps;
        a.ks_per_split = (ksteps + S - 1) / S;
        a.status = p->status;
        if (BP == 16) err = launch_qkv<16>(wmap, xmap, a, row_tiles, st);
        else if (BP == 32) err = launch_qkv<32>(wmap, xmap, a, row_tiles, st);
        else err = launch_qkv<64>(wmap, xmap, a, row_tiles, st);
        if (err != cudaSuccess) return fail(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    }
    return COTTUS_OK;
}

}  // extern "C"
