// Device-side building blocks shared by the cottus_b200 kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "cottus_b200.h"

namespace cb200 {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Cycles a kernel waits on one barrier before it gives up and reports
// COTTUS_STATUS_TIMEOUT (about 1 s at the B200 boost clock).
constexpr long long kWaitLimitCycles = 2000000000LL;

// ---------------------------------------------------------------------------
// fp16 <-> fp32
// ---------------------------------------------------------------------------

// fp32 -> fp16 bits by truncation, the KV-cache encoder of the reference
// (generic_transformer.cpp:255-262): mantissa truncated, biased exponent
// <= 0 -> signed zero, >= 31 (including inf and NaN) -> signed inf.
__device__ __forceinline__ uint16_t f32_to_f16_trunc(float f) {
    uint32_t bits = __float_as_uint(f);
    uint32_t sign = (bits & 0x80000000u) >> 16;
    int32_t e = (int32_t)((bits >> 23) & 0xFFu) - 112;
    uint32_t m = (bits & 0x007FFFFFu) >> 13;
    uint32_t r = e <= 0 ? sign : (e >= 31 ? (sign | 0x7C00u) : (sign | ((uint32_t)e << 10) | m));
    return (uint16_t)r;
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t x) {
    __half2 h = *reinterpret_cast<__half2*>(&x);
    return __half22float2(h);
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Loads 8 consecutive elements (16 B of fp16 or 32 B of fp32) as fp32.
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
    uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    float2 f;
    f = h2_to_f2(r.x); v[0] = f.x; v[1] = f.y;
    f = h2_to_f2(r.y); v[2] = f.x; v[3] = f.y;
    f = h2_to_f2(r.z); v[4] = f.x; v[5] = f.y;
    f = h2_to_f2(r.w); v[6] = f.x; v[7] = f.y;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void store8(__half* p, const float (&v)[8]) {
    uint4 r;
    r.x = pack_h2(v[0], v[1]);
    r.y = pack_h2(v[2], v[3]);
    r.z = pack_h2(v[4], v[5]);
    r.w = pack_h2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = r;
}

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100 FFMA2 / FMUL2)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long ra = *reinterpret_cast<unsigned long long*>(&a);
    unsigned long long rb = *reinterpret_cast<unsigned long long*>(&b);
    unsigned long long rc = *reinterpret_cast<unsigned long long*>(&c);
    unsigned long long rd;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
    return *reinterpret_cast<float2*>(&rd);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long ra = *reinterpret_cast<unsigned long long*>(&a);
    unsigned long long rb = *reinterpret_cast<unsigned long long*>(&b);
    unsigned long long rd;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
    return *reinterpret_cast<float2*>(&rd);
}

// ---------------------------------------------------------------------------
// RoPE rotation of one interleaved pair without FMA contraction
// (compute_primitives_cpu.cpp:69-71 evaluated in plain fp32, as the
// reference's -O3 x86-64 build does).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void rope_pair(float x0, float x1, float c, float s, float& o0, float& o1) {
    o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    o1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

// ---------------------------------------------------------------------------
// mbarrier + TMA (cp.async.bulk.tensor) wrappers.  No multicast anywhere.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for phase `parity` of `bar` to complete; gives up after
// kWaitLimitCycles and returns false (the caller reports a timeout).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
    return true;
}
// 3-D tiled TMA load into this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                           int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
        : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}
// 3-D tiled TMA prefetch into L2 (no shared memory, no barrier; the tensor
// map bounds-checks the box).
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
// L1 prefetch of the line holding a global address (a hint: nothing is
// written, so no later instruction waits on it).
__device__ __forceinline__ void prefetch_l1(const void* p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Programmatic dependent launch: wait until the preceding kernel of the
// stream has completed (and its writes are visible) before touching global
// memory; let the next kernel of the stream start its own prologue early.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Device-scope acquire-release fence: orders this thread's earlier memory
// operations before its later ones as seen by other SMs.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// A plain global load issued where it stands (volatile asm: the compiler does
// not sink it into a later branch that uses it), so that it is in flight
// together with the loads issued next to it.
__device__ __forceinline__ int ld_now_i32(const int32_t* p) {
    int v;
    asm volatile("ld.global.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
// Relaxed device-scope load (reads the current value at the coherence point).
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// System-scope acquire load (a word another GPU writes over NVLink).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void report(uint32_t* status, uint32_t bits) {
    if (status) atomicOr(status, bits);
}

__device__ __forceinline__ int32_t div_up(int32_t a, int32_t b) { return (a + b - 1) / b; }

// Split-KV merge of one (sequence, head) by one warp: P <= kMergeParts parts,
// part p with natural-log LSE lse[p][hw] and normalised output row
// row[p][hw * D .. + D).  lse = log(sum_p exp(lse_p)), out = sum_p
// exp(lse_p - lse) * row_p, parts in increasing order (the same bits
// whichever kernel calls it).  All parts' loads are issued together (one
// round trip even when the parts live in other GPUs' memory); a lane covers
// 4 consecutive dims.
constexpr int kMergeParts = 8;
// Dims d .. d+3 (fewer at the end of the row) of every part's row.
__device__ __forceinline__ void load_part_rows(float4 (&x)[kMergeParts], const float* const (&row)[kMergeParts], int P,
                                               long long hw, int D, int d) {
    const int n = D - d < 4 ? D - d : 4;
#pragma unroll
    for (int p = 0; p < kMergeParts; ++p) {
        x[p] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p < P) {
            const float* src = row[p] + hw * D + d;
            if (n == 4 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                x[p] = __ldcg(reinterpret_cast<const float4*>(src));
            } else {
                x[p].x = __ldcg(src);
                if (n > 1) x[p].y = __ldcg(src + 1);
                if (n > 2) x[p].z = __ldcg(src + 2);
                if (n > 3) x[p].w = __ldcg(src + 3);
            }
        }
    }
}
__device__ __forceinline__ void merge_head_parts(const float* const (&lse)[kMergeParts],
                                                 const float* const (&row)[kMergeParts], int P, long long hw, int D,
                                                 int lane, void* out, int out_f16, float* lse_out) {
    float lp[kMergeParts];
#pragma unroll
    for (int p = 0; p < kMergeParts; ++p) lp[p] = p < P ? __ldcg(lse[p] + hw) : -INFINITY;
    // the lane's first dims of every part are requested together with the
    // LSEs (their addresses do not depend on them): one round trip, not two;
    // a part without valid tokens (LSE -inf) is loaded but never added
    const int d0 = lane * 4;
    float4 x0[kMergeParts];
    if (d0 < D) load_part_rows(x0, row, P, hw, D, d0);
    float M = -INFINITY;
#pragma unroll
    for (int p = 0; p < kMergeParts; ++p) M = fmaxf(M, lp[p]);
    float S = 0.f;
    if (M != -INFINITY) {
#pragma unroll
        for (int p = 0; p < kMergeParts; ++p)
            if (p < P) S += expf(lp[p] - M);
    }
    const float L = M == -INFINITY ? -INFINITY : M + logf(S);
    float wt[kMergeParts];
#pragma unroll
    for (int p = 0; p < kMergeParts; ++p) wt[p] = (p < P && lp[p] != -INFINITY) ? expf(lp[p] - L) : 0.f;
    for (int d = d0; d < D; d += 128) {
        float4 x[kMergeParts];
        if (d == d0) {
#pragma unroll
            for (int p = 0; p < kMergeParts; ++p) x[p] = x0[p];
        } else {
            load_part_rows(x, row, P, hw, D, d);
        }
        const int n = D - d < 4 ? D - d : 4;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < kMergeParts; ++p) {
            if (p < P && lp[p] != -INFINITY) {
                acc[0] += wt[p] * x[p].x;
                acc[1] += wt[p] * x[p].y;
                acc[2] += wt[p] * x[p].z;
                acc[3] += wt[p] * x[p].w;
            }
        }
        for (int e = 0; e < n; ++e) {
            if (out_f16) reinterpret_cast<__half*>(out)[hw * D + d + e] = __float2half_rn(acc[e]);
            else reinterpret_cast<float*>(out)[hw * D + d + e] = acc[e];
        }
    }
    if (lse_out && lane == 0) lse_out[hw] = L;
}

// Plain launch whose return value is this launch's own error (a sticky
// error left by an earlier, unrelated launch is not picked up and reported
// as this one's, as cudaGetLastError after <<<>>> would).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace cb200
