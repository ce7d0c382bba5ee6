// Generic paged decode (any head_dim <= 512, any block size), RoPE, KV
// append, block-table gather and split-KV log-sum-exp merge.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace cb200 {

// ---------------------------------------------------------------------------
// Generic paged decode: one CTA per (query head, sequence), 128 threads.
// Tokens are processed 128 at a time: thread j scores token t0+j (full dot
// product over head_dim, as paged_attention_cpu.cpp:69-76 does), the chunk
// max/sum go through shared memory, then each thread accumulates P.V for
// its own dims.  Online softmax across chunks.  Used for shapes outside the
// TMA fast path (small known-answer cases, odd head_dim / block sizes).
// ---------------------------------------------------------------------------
struct GenericArgs {
    void* out;
    const void* q;
    const uint16_t* kv;
    const int32_t* bt;
    const int32_t* ctx;
    const int32_t* positions;
    const float* cos_sin;
    float* lse;
    uint32_t* status;
    long long num_blocks;
    int B, H, Hkv, D, bs, L, layer, maxb, max_pos;
    int q_f16, out_f16;
    float scale;
};

constexpr int kGenThreads = 128;
constexpr int kGenMaxDimsPerThread = 4;  // head_dim <= 512

template <bool ROPE>
__global__ void __launch_bounds__(kGenThreads) decode_generic_kernel(const GenericArgs a) {
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    extern __shared__ float gsm[];
    float* q_s = gsm;                              // [D] (padded to an even count)
    float* p_s = q_s + ((a.D + 1) & ~1);           // [128]
    long long* off_s = reinterpret_cast<long long*>(p_s + kGenThreads);  // [128] K offsets (-1 = masked), 8-B aligned
    __shared__ float red[kGenThreads / 32];

    const long long head = (long long)b * a.H + h;
    int n;
    bool valid;
    if (ROPE) {
        const int pos = a.positions[b];
        n = pos + 1;
        valid = pos >= 0 && (a.cos_sin == nullptr || pos < a.max_pos) && n <= a.maxb * a.bs;
    } else {
        n = a.ctx[b];
        valid = n >= 0 && n <= a.maxb * a.bs;
    }
    if (!valid || n == 0) {
        if (!valid && tid == 0 && h == 0)
            report(a.status, ROPE ? COTTUS_STATUS_BAD_POSITION : COTTUS_STATUS_BAD_CONTEXT);
        for (int d = tid; d < a.D; d += kGenThreads) {
            if (a.out_f16) reinterpret_cast<__half*>(a.out)[head * a.D + d] = __float2half_rn(0.f);
            else reinterpret_cast<float*>(a.out)[head * a.D + d] = 0.f;
        }
        if (a.lse && tid == 0) a.lse[head] = -INFINITY;
        return;
    }
    const int kvh = (int)(((long long)h * a.Hkv) / a.H);
    for (int d = tid; d < a.D; d += kGenThreads) {
        const long long qi = head * a.D + d;
        q_s[d] = a.q_f16 ? __half2float(reinterpret_cast<const __half*>(a.q)[qi])
                         : reinterpret_cast<const float*>(a.q)[qi];
    }
    __syncthreads();
    if (ROPE && a.cos_sin) {
        for (int pr = tid; pr < a.D / 2; pr += kGenThreads) {
            const float c = a.cos_sin[((long long)(n - 1) * (a.D / 2) + pr) * 2];
            const float s = a.cos_sin[((long long)(n - 1) * (a.D / 2) + pr) * 2 + 1];
            float o0, o1;
            rope_pair(q_s[2 * pr], q_s[2 * pr + 1], c, s, o0, o1);
            q_s[2 * pr] = o0;
            q_s[2 * pr + 1] = o1;
        }
        __syncthreads();
    }
    const long long per_layer_kv = (long long)a.bs * a.Hkv * a.D;
    float acc[kGenMaxDimsPerThread] = {0.f, 0.f, 0.f, 0.f};
    float m = -INFINITY, l = 0.f;
    for (int t0 = 0; t0 < n; t0 += kGenThreads) {
        const int t = t0 + tid;
        float s = -INFINITY;
        long long koff = -1;
        if (t < n) {
            const int blk = a.bt[(long long)b * a.maxb + t / a.bs];
            if (blk >= 0 && blk < a.num_blocks) {
                koff = ((long long)blk * a.L + a.layer) * 2 * per_layer_kv + (long long)(t % a.bs) * a.Hkv * a.D +
                       (long long)kvh * a.D;
                float dot = 0.f;
                for (int d = 0; d < a.D; ++d)
                    dot = __fadd_rn(dot, __fmul_rn(q_s[d], __half2float(__ushort_as_half(a.kv[koff + d]))));
                s = dot * a.scale;
            } else {
                report(a.status, COTTUS_STATUS_BAD_BLOCK_ID);
            }
        }
        off_s[tid] = koff;
        // chunk max
        float v = s;
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if ((tid & 31) == 0) red[tid >> 5] = v;
        __syncthreads();
        float cm = red[0];
        for (int i = 1; i < kGenThreads / 32; ++i) cm = fmaxf(cm, red[i]);
        __syncthreads();
        const float m_new = fmaxf(m, cm);
        const float alpha = m_new == -INFINITY ? 1.f : expf(m - m_new);
        const float p = koff >= 0 ? expf(s - m_new) : 0.f;
        p_s[tid] = p;
        float ps = p;
        for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        if ((tid & 31) == 0) red[tid >> 5] = ps;
        __syncthreads();
        float csum = 0.f;
        for (int i = 0; i < kGenThreads / 32; ++i) csum += red[i];
        l = l * alpha + csum;
        m = m_new;
        const int cnt = min(kGenThreads, n - t0);
#pragma unroll
        for (int k = 0; k < kGenMaxDimsPerThread; ++k) {
            const int d = tid + k * kGenThreads;
            if (d < a.D) {
                float x = acc[k] * alpha;
                for (int j = 0; j < cnt; ++j) {
                    const long long ko = off_s[j];
                    if (ko >= 0) x = __fmaf_rn(p_s[j], __half2float(__ushort_as_half(a.kv[ko + per_layer_kv + d])), x);
                }
                acc[k] = x;
            }
        }
        __syncthreads();
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int k = 0; k < kGenMaxDimsPerThread; ++k) {
        const int d = tid + k * kGenThreads;
        if (d < a.D) {
            if (a.out_f16) reinterpret_cast<__half*>(a.out)[head * a.D + d] = __float2half_rn(acc[k] * inv);
            else reinterpret_cast<float*>(a.out)[head * a.D + d] = acc[k] * inv;
        }
    }
    if (a.lse && tid == 0) a.lse[head] = l > 0.f ? m + logf(l) : -INFINITY;
}

cudaError_t launch_decode_generic(const DecodeDesc& d, cudaStream_t st) {
    GenericArgs a;
    a.out = d.out;
    a.q = d.q;
    a.kv = d.rope ? d.kv_mut : d.kv;
    a.bt = d.block_table;
    a.ctx = d.context_lens;
    a.positions = d.positions;
    a.cos_sin = d.cos_sin;
    a.lse = d.lse;
    a.status = d.status;
    a.num_blocks = d.num_blocks;
    a.B = d.batch;
    a.H = d.num_heads;
    a.Hkv = d.num_kv_heads;
    a.D = d.head_dim;
    a.bs = d.block_size;
    a.L = d.num_layers;
    a.layer = d.layer;
    a.maxb = d.max_blocks;
    a.max_pos = d.max_position;
    a.q_f16 = d.q_f16;
    a.out_f16 = d.out_f16;
    a.scale = d.scale;
    const size_t smem = (size_t)((d.head_dim + 1) & ~1) * 4 + kGenThreads * 4 + kGenThreads * 8;
    dim3 grid(d.num_heads, d.batch);
    // In rope mode the query is rotated in fp32 inside the kernel (the
    // append kernel launched before has already written k/v and q_out).
    if (d.rope) return launch_kernel(decode_generic_kernel<true>, grid, dim3(kGenThreads), smem, st, a);
    return launch_kernel(decode_generic_kernel<false>, grid, dim3(kGenThreads), smem, st, a);
}

// ---------------------------------------------------------------------------
// RoPE + KV append for one new token per sequence.  One CTA per sequence;
// one thread per 8-element chunk of each query / key / value row.
// k is rotated then, like v, encoded by truncation and scattered into slot
// pos % block_size of block block_table[b][pos / block_size]
// (generic_transformer.cpp:196-284).
// ---------------------------------------------------------------------------
struct AppendArgs {
    const void* q;
    const void* k;
    const void* v;
    void* q_out;
    uint16_t* kv;
    const int32_t* bt;
    const int32_t* positions;
    const float* cos_sin;
    uint32_t* status;
    long long num_blocks;
    int H, Hkv, D, bs, L, layer, maxb, max_pos, f16;
};

__device__ __forceinline__ float ld_elem(const void* p, long long i, int f16) {
    return f16 ? __half2float(reinterpret_cast<const __half*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_elem(void* p, long long i, float x, int f16) {
    if (f16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
    else reinterpret_cast<float*>(p)[i] = x;
}

__global__ void rope_append_kernel(const AppendArgs a) {
    const int b = blockIdx.x;
    const int pos = a.positions[b];
    const bool pos_ok = pos >= 0 && (pos / a.bs) < a.maxb && (a.cos_sin == nullptr || pos < a.max_pos);
    if (!pos_ok) {
        if (threadIdx.x == 0) report(a.status, COTTUS_STATUS_BAD_POSITION);
        return;
    }
    const int blk = a.bt[(long long)b * a.maxb + pos / a.bs];
    const bool blk_ok = blk >= 0 && blk < a.num_blocks;
    if (!blk_ok && threadIdx.x == 0) report(a.status, COTTUS_STATUS_BAD_BLOCK_ID);
    const int pairs = a.D / 2;
    const int rows = a.H + 2 * a.Hkv;
    const long long per_layer_kv = (long long)a.bs * a.Hkv * a.D;
    const long long base = ((long long)blk * a.L + a.layer) * 2 * per_layer_kv + (long long)(pos % a.bs) * a.Hkv * a.D;
    // One thread per element; an element of a rotated pair reads its partner.
    // With an odd head_dim the last element is not rotated (as ropeCPU).
    for (int i = threadIdx.x; i < rows * a.D; i += blockDim.x) {
        const int r = i / a.D, d = i % a.D;
        const int pr = d / 2;
        const bool rot = a.cos_sin != nullptr && pr < pairs;
        float c = 1.f, s = 0.f;
        if (rot) {
            c = a.cos_sin[((long long)pos * pairs + pr) * 2];
            s = a.cos_sin[((long long)pos * pairs + pr) * 2 + 1];
        }
        if (r < a.H + a.Hkv) {  // query or key row: rotate
            const void* src = r < a.H ? a.q : a.k;
            const long long row = r < a.H ? ((long long)b * a.H + r) : ((long long)b * a.Hkv + (r - a.H));
            float y = ld_elem(src, row * a.D + d, a.f16);
            if (rot) {
                const float x0 = ld_elem(src, row * a.D + 2 * pr, a.f16);
                const float x1 = ld_elem(src, row * a.D + 2 * pr + 1, a.f16);
                float o0, o1;
                rope_pair(x0, x1, c, s, o0, o1);
                y = (d & 1) ? o1 : o0;
            }
            if (r < a.H) {
                if (a.q_out) st_elem(a.q_out, row * a.D + d, y, a.f16);
            } else if (blk_ok) {
                a.kv[base + (long long)(r - a.H) * a.D + d] = f32_to_f16_trunc(y);
            }
        } else if (blk_ok) {  // value row: encode only
            const int h = r - a.H - a.Hkv;
            const float y = ld_elem(a.v, ((long long)b * a.Hkv + h) * a.D + d, a.f16);
            a.kv[base + per_layer_kv + (long long)h * a.D + d] = f32_to_f16_trunc(y);
        }
    }
}

cudaError_t launch_rope_append(const DecodeDesc& d, cudaStream_t st) {
    AppendArgs a;
    a.q = d.q;
    a.k = d.k_new;
    a.v = d.v_new;
    a.q_out = d.q_out;
    a.kv = d.kv_mut;
    a.bt = d.block_table;
    a.positions = d.positions;
    a.cos_sin = d.cos_sin;
    a.status = d.status;
    a.num_blocks = d.num_blocks;
    a.H = d.num_heads;
    a.Hkv = d.num_kv_heads;
    a.D = d.head_dim;
    a.bs = d.block_size;
    a.L = d.num_layers;
    a.layer = d.layer;
    a.maxb = d.max_blocks;
    a.max_pos = d.max_position;
    a.f16 = d.q_f16;
    return launch_kernel(rope_append_kernel, dim3(d.batch), dim3(256), 0, st, a);
}

// ---------------------------------------------------------------------------
// Batched RoPE of fp32 rows with a device (cos, sin) table.
// ---------------------------------------------------------------------------
__global__ void rope_kernel(float* out, const float* in, const int32_t* positions, int num_tokens, int H, int D,
                            const float* cos_sin, int max_pos) {
    const int pairs = D / 2;
    const long long total = (long long)num_tokens * H * pairs;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int pr = (int)(i % pairs);
        const long long th = i / pairs;  // token * H + head
        const int t = (int)(th / H);
        int pos = positions[t];
        pos = pos < 0 ? 0 : (pos >= max_pos ? max_pos - 1 : pos);
        const float c = cos_sin[((long long)pos * pairs + pr) * 2];
        const float s = cos_sin[((long long)pos * pairs + pr) * 2 + 1];
        const long long e = th * D + 2 * pr;
        float o0, o1;
        rope_pair(in[e], in[e + 1], c, s, o0, o1);
        out[e] = o0;
        out[e + 1] = o1;
    }
}

cudaError_t launch_rope(float* out, const float* in, const int32_t* positions, int32_t num_tokens, int32_t H,
                        int32_t D, const float* cos_sin, int32_t max_pos, cudaStream_t st) {
    const long long total = (long long)num_tokens * H * (D / 2);
    if (total == 0) return cudaSuccess;
    const int blocks = (int)((total + 255) / 256 < 65535 ? (total + 255) / 256 : 65535);
    return launch_kernel(rope_kernel, dim3(blocks), dim3(256), 0, st, out, in, positions, num_tokens, H, D, cos_sin,
                         max_pos);
}

// (cos, sin) pairs for one position passed by value (<= 128 pairs).
struct CosSinPairs {
    float v[256];
};
__global__ void rope_single_kernel(float* out, const float* in, const CosSinPairs cs, int H, int D) {
    const int pairs = D / 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H * pairs) return;
    const int pr = i % pairs, h = i / pairs;
    const int e = h * D + 2 * pr;
    float o0, o1;
    rope_pair(in[e], in[e + 1], cs.v[2 * pr], cs.v[2 * pr + 1], o0, o1);
    out[e] = o0;
    out[e + 1] = o1;
}

cudaError_t launch_rope_single(float* out, const float* in, const float* host_cos_sin, int32_t H, int32_t D,
                               cudaStream_t st) {
    CosSinPairs cs;
    for (int i = 0; i < D && i < 256; ++i) cs.v[i] = host_cos_sin[i];
    const int total = H * (D / 2);
    if (total == 0) return cudaSuccess;
    return launch_kernel(rope_single_kernel, dim3((total + 255) / 256), dim3(256), 0, st, out, in, cs, H, D);
}

// ---------------------------------------------------------------------------
// Split-KV merge of (normalised partial, lse) pairs.  One warp per head;
// up to kMergeParts parts with merge_head_parts (all loads in flight at
// once), more with the same arithmetic in a loop over the parts.
// ---------------------------------------------------------------------------
__global__ void lse_combine_kernel(void* out, int out_f16, float* lse_out, const float* part_out,
                                   const float* part_lse, int P, long long heads, int D) {
    const long long hw = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (hw >= heads) return;
    if (P <= kMergeParts) {
        const float* lse[kMergeParts];
        const float* row[kMergeParts];
#pragma unroll
        for (int p = 0; p < kMergeParts; ++p) {
            lse[p] = part_lse + (long long)(p < P ? p : 0) * heads;
            row[p] = part_out + (long long)(p < P ? p : 0) * heads * D;
        }
        merge_head_parts(lse, row, P, hw, D, lane, out, out_f16, lse_out);
        return;
    }
    float M = -INFINITY;
    for (int p = 0; p < P; ++p) M = fmaxf(M, part_lse[p * heads + hw]);
    float S = 0.f;
    if (M != -INFINITY)
        for (int p = 0; p < P; ++p) S += expf(part_lse[p * heads + hw] - M);
    const float lse = M == -INFINITY ? -INFINITY : M + logf(S);
    for (int d = lane; d < D; d += 32) {
        float acc = 0.f;
        if (M != -INFINITY)
            for (int p = 0; p < P; ++p) {
                const float lp = part_lse[p * heads + hw];
                if (lp != -INFINITY) acc += expf(lp - lse) * part_out[(p * heads + hw) * D + d];
            }
        if (out_f16) reinterpret_cast<__half*>(out)[hw * D + d] = __float2half_rn(acc);
        else reinterpret_cast<float*>(out)[hw * D + d] = acc;
    }
    if (lse_out && lane == 0) lse_out[hw] = lse;
}

cudaError_t launch_lse_combine(void* out, int out_f16, float* lse_out, const float* part_out, const float* part_lse,
                               int32_t P, int32_t B, int32_t H, int32_t D, cudaStream_t st) {
    const long long heads = (long long)B * H;
    if (heads == 0) return cudaSuccess;
    const long long threads = heads * 32;
    return launch_kernel(lse_combine_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, out, out_f16,
                         lse_out, part_out, part_lse, P, heads, D);
}

// ---------------------------------------------------------------------------
// Block-table gather: one CTA per (page, sequence); a page's valid K (then
// V) rows for all kv heads are contiguous in both pool and output.
// ---------------------------------------------------------------------------
__global__ void gather_kernel(uint16_t* k_out, uint16_t* v_out, const uint16_t* kv, const int32_t* bt,
                              const int32_t* ctx, long long num_blocks, int max_ctx, int Hkv, int D, int bs, int L,
                              int layer, int maxb, uint32_t* status) {
    const int p = blockIdx.x, b = blockIdx.y;
    const int n = ctx[b];
    if (n < 0 || n > max_ctx || n > maxb * bs) {
        if (threadIdx.x == 0 && p == 0) report(status, COTTUS_STATUS_BAD_CONTEXT);
        return;
    }
    const int t0 = p * bs;
    if (t0 >= n) return;
    const int rows = min(bs, n - t0);
    const int blk = bt[(long long)b * maxb + p];
    if (blk < 0 || blk >= num_blocks) {
        if (threadIdx.x == 0) report(status, COTTUS_STATUS_BAD_BLOCK_ID);
        return;
    }
    const long long row = (long long)Hkv * D;
    const long long per_layer_kv = (long long)bs * row;
    const uint16_t* ks = kv + ((long long)blk * L + layer) * 2 * per_layer_kv;
    const uint16_t* vs = ks + per_layer_kv;
    uint16_t* kd = k_out + ((long long)b * max_ctx + t0) * row;
    uint16_t* vd = v_out + ((long long)b * max_ctx + t0) * row;
    const long long nel = rows * row;
    const bool vec = ((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(kd) |
                       reinterpret_cast<uintptr_t>(vd)) & 15) == 0 && (nel % 8) == 0;
    if (vec) {
        for (long long i = threadIdx.x; i < nel / 8; i += blockDim.x) {
            reinterpret_cast<uint4*>(kd)[i] = __ldg(reinterpret_cast<const uint4*>(ks) + i);
            reinterpret_cast<uint4*>(vd)[i] = __ldg(reinterpret_cast<const uint4*>(vs) + i);
        }
    } else {
        for (long long i = threadIdx.x; i < nel; i += blockDim.x) {
            kd[i] = ks[i];
            vd[i] = vs[i];
        }
    }
}

cudaError_t launch_gather(uint16_t* k_out, uint16_t* v_out, const uint16_t* kv, const int32_t* bt, const int32_t* ctx,
                          int64_t num_blocks, int32_t B, int32_t max_ctx, int32_t Hkv, int32_t D, int32_t bs, int32_t L,
                          int32_t layer, int32_t maxb, uint32_t* status, cudaStream_t st) {
    const int pages = (max_ctx + bs - 1) / bs;
    if (pages == 0 || B == 0) return cudaSuccess;
    dim3 grid(pages, B);
    return launch_kernel(gather_kernel, grid, dim3(256), 0, st, k_out, v_out, kv, bt, ctx, num_blocks, max_ctx, Hkv, D,
                         bs, L, layer, maxb, status);
}

}  // namespace cb200
