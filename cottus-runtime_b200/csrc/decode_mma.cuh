// Paged decode attention with the QK and PV tile products on the tensor
// cores (warp-level mma.sync m16n8k16, fp16 inputs, fp32 accumulation),
// one CTA per stream-K worker.
//
// Schedule.  Units are (sequence, kv head, page) in sequence-major order,
// as in decode_tma_kernel, but the worker is a whole CTA: CTA c owns one
// contiguous chunk of ceil(units / CTAs) units.  A chunk is a list of
// segments, its intersection with each (sequence, kv head) pair.  The 4
// warps split every segment's pages (unit k of the chunk goes to warp
// k mod 4), each warp with its own TMA ring and its own online-softmax
// state; at the end of a segment the warps' (m, l, o) states are merged in
// shared memory and the whole CTA writes the pair's output (or, for a pair
// cut by chunk boundaries, one partial per chunk; the last CTA to finish
// such a pair merges the partials).  Against one warp per chunk, a pair is
// cut into 4x fewer parts, so the merges that end a launch are 4x shorter
// and their arrival counters see little contention, and a warp's block-table
// entries for the first pages are loaded in parallel, not one after another.
//
// Math per page and warp:
//   S^T[16 tokens x 8 cols] = K[16 x D] . Q^T[D x 8]      (D/16 MMAs)
//       A = the page's K rows (ldmatrix from a 128B-swizzled TMA tile),
//       B = the GQA group's query rows (columns >= G are zero), kept in
//       registers for the whole segment.  fp32 queries (and rotated ones)
//       are split into fp16 hi + lo parts, two MMAs per k-step, so scores
//       keep fp32 accuracy.
//   online softmax in the log2 domain on the C fragment: a lane holds two
//       heads x two tokens, so the max needs 3 shuffles and the rescale of
//       its own accumulator columns needs no broadcast.
//   O^T[D x 8 cols] += V^T[D x 16] . P^T[16 x 8]          (D/16 MMAs)
//       A = V rows through ldmatrix.trans, B = the probabilities in fp16,
//       transposed in registers with movmatrix.  fp16 probabilities bound
//       the relative error of each weight by 2^-11: enough where the output
//       is fp16, or fp32 LSE partials of a split context (whose merged
//       result is fp16).  For fp32 outputs (PSPLIT) each probability is
//       also split into fp16 hi + lo parts (hi = its fp16 rounding, lo = the
//       fp16 rounding of the remainder), two MMAs per dim tile, so weights
//       keep about 2^-22 relative accuracy, as with fp32 queries above.
#pragma once

#include "decode_tma.cuh"

namespace cb200 {

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ float2 unpack_h2(uint32_t x) { return h2_to_f2(x); }

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` (0..31) in
// column region `region` of a slot written by {64, 1, 32} TMA boxes with
// 128B swizzle: chunk index XOR (row mod 8).
__device__ __forceinline__ uint32_t swz(int region, int row, int chunk) {
    return (uint32_t)(region * (32 * 128) + row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int D, int G>
struct MmaCfg {
    static constexpr int KSTEPS = D / 16;   // QK k-steps = PV dim tiles
    static constexpr int REGIONS = D / 64;  // 128-byte column regions per slot
    static constexpr int SLOT_BYTES = 2 * kBS * D * 2;
    static constexpr int OST = D + 4;       // head stride of the merge area in floats (padded: no bank conflicts)
    static constexpr int MERGE_FLOATS = kNW * G * OST + kNW * G * 2;
};

template <int RING, int D, int G>
constexpr size_t mma_smem_bytes() {
    using C = MmaCfg<D, G>;
    return (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 8 + (size_t)kNW * RING * 4 +
           (size_t)C::MERGE_FLOATS * 4 + 1024 + 16;
}

// CTAs per SM the register budget is fitted to (8 or 12 warps per SM).
#ifndef CB200_MMA_MIN_CTAS_D64
#define CB200_MMA_MIN_CTAS_D64 3
#endif
#ifndef CB200_MMA_MIN_CTAS_D128
#define CB200_MMA_MIN_CTAS_D128 2
#endif
template <int D>
constexpr int mma_min_ctas() { return D == 64 ? CB200_MMA_MIN_CTAS_D64 : CB200_MMA_MIN_CTAS_D128; }

// Virtual units after each pair's pages in the partition into chunks: a
// pair's fixed cost (staging and rotating its query, the warps' merge at
// its end, the arrival of a cut pair) counted in units, so that a chunk
// full of short pairs gets fewer pages.  Cursors skip them.
#ifndef CB200_PAIR_PAD_D64
#define CB200_PAIR_PAD_D64 24
#endif
#ifndef CB200_PAIR_PAD_D128
#define CB200_PAIR_PAD_D128 8
#endif
template <int D>
constexpr int pair_pad() { return D == 64 ? CB200_PAIR_PAD_D64 : CB200_PAIR_PAD_D128; }
// Fewest units in a CTA's chunk (4 per warp).
constexpr long long kMinChunkCta = 4 * kNW;
// Own units per warp warmed in L2 before the wait for the preceding kernel.
#ifndef CB200_MMA_WARM_PAGES
#define CB200_MMA_WARM_PAGES 3
#endif
// Whether a vote on the lanes' own scores gates the reduction of a page's max
// (measured: faster at head_dim 64 and at head_dim 128 with groups of 4; at
// head_dim 128 with groups of 8 the long-context shape ran 0.7 % slower).
#ifndef CB200_MMA_VOTE_D128_G8
#define CB200_MMA_VOTE_D128_G8 0
#endif
template <int D, int G>
constexpr bool vote_max() { return D == 128 && G == 8 ? CB200_MMA_VOTE_D128_G8 : true; }

// One segment of a chunk [u0, u1): the chunk's real units inside one
// (sequence, kv head) pair.  c is at the segment's first page, r0 counts
// the chunk's real units before it, len is its number of pages (0: the
// chunk has no further segment).
struct Segment {
    Cursor c;
    int r0, len;
};

// Real pages of the pair at c (from page c.p) that lie before unit u1.
__device__ __forceinline__ int pages_before(const Cursor& c, const TmaArgs& a, long long u1) {
    if (c.b >= a.B || c.ps + c.p >= u1) return 0;
    return (int)min((long long)c.np, u1 - c.ps) - c.p;
}

template <bool ROPE, int PAD>
__device__ __forceinline__ void next_segment(Segment& s, const TmaArgs& a, long long u1) {
    s.r0 += s.len;
    s.c.p = s.c.np - 1;
    cursor_next<ROPE>(s.c, a, PAD);  // page 0 of the next pair
    s.len = pages_before(s.c, a, u1);
}

// Moves c forward by n real units (n small).
template <bool ROPE, int PAD>
__device__ __forceinline__ void cursor_advance(Cursor& c, const TmaArgs& a, int n) {
    if (c.p + n < c.np) {  // within the pair: the common case
        c.p += n;
        return;
    }
    for (int i = 0; i < n; ++i) cursor_next<ROPE>(c, a, PAD);
}

// A warp's first own units (units warp, warp + kNW, ... of its chunk): lane
// j <= RING gets own unit j's block-table index and kv head (idx -1: no such
// unit); count is the number of own units among the first RING.  With REGS
// the walk reads nothing but the snapshot r, so that the result computed
// before the wait for the preceding kernel is the one computed after it
// whenever the lengths read again match the snapshot; without, it reads the
// lengths (batches above kPlanRegs * 32 sequences, after the wait).
struct PrimeIdx {
    long long idx;
    int h, count;
};
template <int RING, bool REGS, bool ROPE, int PAD>
__device__ __forceinline__ PrimeIdx prime_index(const WorkerPlan& pl, const PlanRegs& r, const TmaArgs& a, int warp,
                                                int lane) {
    PrimeIdx x = {-1, 0, 0};
    if (pl.u0 >= pl.u1) return x;
    Cursor c = pl.cur;
    int step = warp;
    for (int j = 0; j <= RING; ++j) {
        if (c.p + step < c.np) {
            c.p += step;
        } else {
            for (int i = 0; i < step; ++i) {
                if constexpr (REGS) cursor_next_regs(c, r, a, lane, PAD);
                else cursor_next<ROPE>(c, a, PAD);
            }
        }
        if (c.b >= a.B || c.ps + c.p >= pl.u1) break;
        if (lane == j) {
            x.idx = (long long)c.b * a.maxb + c.p;
            x.h = c.h;
        }
        if (j < RING) ++x.count;
        step = kNW;
    }
    return x;
}

// The new token of a pair (fused step), lane < D/8 of the warp that owns the
// pair's last page: rotates k, encodes k and v by truncation, writes them to
// slot t_new of the page in the pool and in the page's shared-memory tile
// `sl` (so the token attends to itself).  Out of line: it runs once per pair,
// and keeping it out of the page loop keeps that loop's code compact.
template <int D>
__device__ __noinline__ void append_new_token(uint8_t* sl, uint16_t* kv, const void* k_new, const void* v_new,
                                            const float* cos_sin, int qkv_f16, long long blk, int L, int layer,
                                            int Hkv, int b, int h, int ctx, int lane) {
    const int t_new = (ctx - 1) % kBS;
    const long long src = ((long long)b * Hkv + h) * D + lane * 8;
    float kx[8], vx[8];
    if (qkv_f16) {
        load8(reinterpret_cast<const __half*>(k_new) + src, kx);
        load8(reinterpret_cast<const __half*>(v_new) + src, vx);
    } else {
        load8(reinterpret_cast<const float*>(k_new) + src, kx);
        load8(reinterpret_cast<const float*>(v_new) + src, vx);
    }
    const float4* cs = reinterpret_cast<const float4*>(cos_sin + ((long long)(ctx - 1) * (D / 2) + lane * 4) * 2);
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
        const float4 c4 = __ldg(cs + pr);
        rope_pair(kx[4 * pr], kx[4 * pr + 1], c4.x, c4.y, kx[4 * pr], kx[4 * pr + 1]);
        rope_pair(kx[4 * pr + 2], kx[4 * pr + 3], c4.z, c4.w, kx[4 * pr + 2], kx[4 * pr + 3]);
    }
    uint32_t kw[4], vw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        kw[j] = (uint32_t)f32_to_f16_trunc(kx[2 * j]) | ((uint32_t)f32_to_f16_trunc(kx[2 * j + 1]) << 16);
        vw[j] = (uint32_t)f32_to_f16_trunc(vx[2 * j]) | ((uint32_t)f32_to_f16_trunc(vx[2 * j + 1]) << 16);
    }
    const uint4 k4 = make_uint4(kw[0], kw[1], kw[2], kw[3]);
    const uint4 v4 = make_uint4(vw[0], vw[1], vw[2], vw[3]);
    *reinterpret_cast<uint4*>(sl + swz(lane / 8, t_new, lane % 8)) = k4;
    *reinterpret_cast<uint4*>(sl + swz(lane / 8, kBS + t_new, lane % 8)) = v4;
    const long long row0 = (blk * L + layer) * (2 * kBS);
    *reinterpret_cast<uint4*>(kv + ((row0 + t_new) * Hkv + h) * D + lane * 8) = k4;
    *reinterpret_cast<uint4*>(kv + ((row0 + kBS + t_new) * Hkv + h) * D + lane * 8) = v4;
}

// Arrival of a cut pair (every thread of the CTA has stored its part of the
// pair's partial) on the pair's counter, tagged with the launch epoch so that
// a count left by an aborted launch, or bytes of another layout that used the
// same workspace, read as zero (a completed pair leaves its counter at zero,
// which a CUDA-graph replay with the same tag needs); the CTA that completes
// the pair merges all its parts.  Chunk c owns units [c*chunk, (c+1)*chunk),
// so the parts of a pair whose pages are units [ps, ps + np) belong to chunks
// ps/chunk .. (ps+np-1)/chunk; a chunk's part is in slot 2c when the pair
// starts at or before the chunk, else in slot 2c+1.  Called by every thread of
// the CTA; out of line (see append_new_token).
// The launch's fields that the arrival and merge read (passed by value: a
// reference to the kernel's argument block would copy it to local memory).
struct MergeArgs {
    unsigned long long* counters;
    const float* ws_o;
    const float* ws_ml;
    void* out;
    float* lse;
    int H, Hkv, out_f16;
    unsigned epoch;
};

template <int D, int G>
__device__ __noinline__ void arrive_cut_pair(const MergeArgs a, long long chunk, int pb, int ph, int pnp, long long pps,
                                           unsigned long long hint, int* s_last) {
    const long long w0 = pps / chunk, w1 = (pps + pnp - 1) / chunk;
    const int nparts = (int)(w1 - w0 + 1);
    __syncthreads();  // every thread's partial stores, then one release fence for the CTA
    if (threadIdx.x == 0) {
        fence_acq_rel_gpu();
        unsigned long long* ctr = a.counters + 1 + (long long)pb * a.Hkv + ph;
        unsigned long long old = hint;
        int last = 0;
        // Once a part of this launch has arrived, the counter carries this
        // launch's tag until the pair completes (which needs this part): an
        // add.  Before that, the first arrival replaces whatever the word holds
        // by (tag, 1) with a compare-and-swap; one that fails because another
        // part arrived in between falls back to the add.
        bool added = false;
        while ((unsigned)(old >> 32) != a.epoch) {
            const unsigned long long first = ((unsigned long long)a.epoch << 32) | 1ull;
            const unsigned long long prev = atomicCAS(ctr, old, first);
            if (prev == old) {
                added = true;
                break;
            }
            old = prev;
        }
        if (!added) {
            old = atomicAdd(ctr, 1ull);
            last = (int)(old & 0xffffffffull) + 1 == nparts;
            if (last) *reinterpret_cast<volatile unsigned long long*>(ctr) = 0ull;  // every part is in: no other writer
        }
        *s_last = last;
    }
    __syncthreads();
    if (!*s_last) return;
    fence_acq_rel_gpu();
    const long long slot0 = w0 * chunk >= pps ? 2 * w0 : 2 * w0 + 1;  // later parts start inside the pair
    constexpr int PB = 4;  // parts loaded together
    constexpr int ITEMS = G * D / 4;
    for (int it = threadIdx.x; it < ITEMS; it += kNW * 32) {
        const int g = it / (D / 4), c4 = it % (D / 4);
        float M = -INFINITY, L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
        for (int j0 = 0; j0 < nparts; j0 += PB) {
            float2 ml[PB];
            float4 x[PB];
#pragma unroll
            for (int q = 0; q < PB; ++q) {
                ml[q] = make_float2(-INFINITY, 0.f);
                x[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (j0 + q < nparts) {
                    const long long sl = j0 + q == 0 ? slot0 : 2 * (w0 + j0 + q);
                    ml[q] = __ldcg(reinterpret_cast<const float2*>(a.ws_ml + (sl * G + g) * 2));
                    x[q] = __ldcg(reinterpret_cast<const float4*>(a.ws_o + (sl * G + g) * D + c4 * 4));
                }
            }
#pragma unroll
            for (int q = 0; q < PB; ++q) {
                const float m = ml[q].x;
                if (m == -INFINITY) continue;  // a part without valid tokens (or past the last part)
                const float Mn = fmaxf(M, m);
                const float sa = exp2f(M - Mn), sb = exp2f(m - Mn);
                M = Mn;
                L = L * sa + ml[q].y * sb;
                acc.x = acc.x * sa + x[q].x * sb;
                acc.y = acc.y * sa + x[q].y * sb;
                acc.z = acc.z * sa + x[q].z * sb;
                acc.w = acc.w * sa + x[q].w * sb;
            }
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        const long long head = (long long)pb * a.H + (long long)ph * G + g;
        if (a.out_f16) {
            *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(a.out) + head * D + c4 * 4) =
                make_uint2(pack_h2(acc.x * inv, acc.y * inv), pack_h2(acc.z * inv, acc.w * inv));
        } else {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + head * D + c4 * 4) =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
        if (a.lse && c4 == 0) a.lse[head] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
    }
}

template <int D, int G, int RING, bool ROPE, bool QSPLIT, bool PSPLIT>
__global__ void __launch_bounds__(kNW * 32, mma_min_ctas<D>())
    decode_mma_kernel(const __grid_constant__ CUtensorMap kv_map, const TmaArgs a) {
    using C = MmaCfg<D, G>;
    constexpr int KS = C::KSTEPS, REG = C::REGIONS, LW = D / 8, OST = C::OST, PAD = pair_pad<D>();
    constexpr unsigned FULL = 0xffffffffu;
    static_assert(G <= 8, "group larger than the MMA n dimension");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* slots = smem + (size_t)warp * RING * C::SLOT_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kNW * RING * C::SLOT_BYTES) + warp * RING;
    int* slot_blk =
        reinterpret_cast<int*>(smem + (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 8) + warp * RING;
    float* merge_o = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(smem + (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 12) + 15) &
        ~uintptr_t(15));                    // [kNW][G][OST]
    float* merge_ml = merge_o + kNW * G * OST;  // [kNW][G][2]

    __shared__ int s_abort;  // a warp of this CTA gave up on a wait
    __shared__ int s_last;   // this CTA is the last to finish a cut pair
    if (lane == 0) {
        if (warp == 0) {
            prefetch_tensormap(&kv_map);
            s_abort = 0;
        }
#pragma unroll
        for (int r = 0; r < RING; ++r) mbar_init(&bars[r], 1);
        fence_barrier_init();
    }
    __syncthreads();

    const long long W = gridDim.x, cid = blockIdx.x;
    // fragment coordinates of this lane
    const int qc = lane & 3;   // column pair: heads 2qc, 2qc+1 of C fragments
    const int qr = lane >> 2;  // row: token qr / qr+8 of C fragments; head qr of B fragments
    const int h0 = 2 * qc, h1 = 2 * qc + 1;
    const uint32_t slots_s = smem_addr(slots);

    uint32_t qb[KS][2];
    uint32_t ql[QSPLIT ? KS : 1][2];
    float o[KS][4];
    // query of the next segment, loaded a segment early and kept as loaded (so
    // that nothing waits for the loads before the segment starts): fp32 values,
    // or fp16 pairs as stored (in qs as bit patterns where they get split,
    // in qn where they are used as they are); with RoPE also the (cos, sin)
    // pairs of the two dims pairs this lane rotates per k-step
    float qs[QSPLIT ? KS : 1][4];
    uint32_t qn[QSPLIT ? 1 : KS][2];
    float2 csn[ROPE ? KS : 1][2];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    // this lane's query elements of pair (b, h): head qr, dims kk*16 + 2qc + {0, 1, 8, 9}
    auto load_q = [&](int b, int h, int n) {
        const bool live = qr < G;
        const long long qrow = ((long long)b * a.H + (long long)h * G + (live ? qr : 0)) * D;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            const int d0 = kk * 16 + 2 * qc, d1 = d0 + 8;
            if constexpr (!QSPLIT) {  // fp16 queries, kept packed
                const unsigned* qh = reinterpret_cast<const unsigned*>(reinterpret_cast<const __half*>(a.q) + qrow);
                qn[kk][0] = live ? __ldg(qh + d0 / 2) : 0u;
                qn[kk][1] = live ? __ldg(qh + d1 / 2) : 0u;
            } else {
                if (!live) {
                    qs[kk][0] = qs[kk][1] = qs[kk][2] = qs[kk][3] = 0.f;
                } else if (a.q_f16) {
                    const unsigned* qh = reinterpret_cast<const unsigned*>(reinterpret_cast<const __half*>(a.q) + qrow);
                    qs[kk][0] = __uint_as_float(__ldg(qh + d0 / 2));
                    qs[kk][1] = __uint_as_float(__ldg(qh + d1 / 2));
                } else {
                    const float2 u = __ldg(reinterpret_cast<const float2*>(reinterpret_cast<const float*>(a.q) + qrow + d0));
                    const float2 v = __ldg(reinterpret_cast<const float2*>(reinterpret_cast<const float*>(a.q) + qrow + d1));
                    qs[kk][0] = u.x; qs[kk][1] = u.y; qs[kk][2] = v.x; qs[kk][3] = v.y;
                }
                if constexpr (ROPE) {
                    const float* cs = a.cos_sin + (long long)(n - 1) * D;  // row of D/2 (cos, sin) pairs
                    csn[kk][0] = live ? __ldg(reinterpret_cast<const float2*>(cs + d0)) : make_float2(1.f, 0.f);
                    csn[kk][1] = live ? __ldg(reinterpret_cast<const float2*>(cs + d1)) : make_float2(1.f, 0.f);
                }
            }
        }
    };

    // The plan is made before the wait for the preceding kernel, from a
    // snapshot of the lengths that kernel may still be writing, with the
    // block-table entries of the warp's first units, and those pages are
    // warmed in L2 (TMA prefetch: nothing written; block ids range-checked,
    // the tensor map bounds the box; L2 is the point of coherence, so a stale
    // snapshot only warms the wrong lines).  These early reads go to L2
    // (ld.global.cg) and leave nothing in L1.  After the wait the lengths and
    // the table entries are read again in one round: plan and entries are
    // kept if the lengths match the snapshot (both were computed from it
    // alone), else made again.  Batches above kPlanRegs * 32 sequences plan
    // after the wait only.
    const bool small = a.B <= 32 * kPlanRegs;
    PlanRegs snap;
    WorkerPlan pl;
    PrimeIdx pi;
    int prime_blk = 0;  // lane j <= RING: block id of own unit j
    if (small) {
        snap = load_plan_regs<ROPE, true>(a, lane);
        pl = plan_from_regs<ROPE>(a, snap, cid, W, lane, kMinChunkCta, PAD);
        pi = prime_index<RING, true, ROPE, PAD>(pl, snap, a, warp, lane);
        if (lane < CB200_MMA_WARM_PAGES && lane < pi.count) {
            const int blk = __ldcg(a.bt + pi.idx);
            if (blk >= 0 && (long long)blk < a.num_blocks)
                for (int q = 0; q < REG; ++q)
                    tma_prefetch_l2_3d(&kv_map, q * 64, pi.h, (blk * a.L + a.layer) * (2 * kBS));
        }
    }
    grid_dependency_wait();
    grid_dependents_launch();
    // (the first segment's query is loaded in the same round, from the same plan)
    if (small) {
        const PlanRegs now = load_plan_regs<ROPE>(a, lane);
        prime_blk = pi.idx >= 0 ? ld_now_i32(a.bt + pi.idx) : 0;
        if (pl.u0 < pl.u1 && pages_before(pl.cur, a, pl.u1) > 0) load_q(pl.cur.b, pl.cur.h, pl.cur.n);
        if (!same_plan_regs<ROPE>(snap, now)) {
            pl = plan_from_regs<ROPE>(a, now, cid, W, lane, kMinChunkCta, PAD);
            pi = prime_index<RING, true, ROPE, PAD>(pl, now, a, warp, lane);
            prime_blk = pi.idx >= 0 ? a.bt[pi.idx] : 0;
            if (pl.u0 < pl.u1 && pages_before(pl.cur, a, pl.u1) > 0) load_q(pl.cur.b, pl.cur.h, pl.cur.n);
        }
        if (warp == 0) zero_fill_from_regs<D, ROPE>(a, now, cid, lane);
    } else {
        pl = plan_worker<D, ROPE>(a, cid, W, lane, kMinChunkCta, warp == 0, PAD);
        pi = prime_index<RING, false, ROPE, PAD>(pl, snap, a, warp, lane);
        prime_blk = pi.idx >= 0 ? a.bt[pi.idx] : 0;
        if (pl.u0 < pl.u1 && pages_before(pl.cur, a, pl.u1) > 0) load_q(pl.cur.b, pl.cur.h, pl.cur.n);
    }
    const long long chunk = pl.chunk, u0 = pl.u0, u1 = pl.u1;
    const bool has_work = u0 < u1 && pages_before(pl.cur, a, u1) > 0;

    // ---- this warp's units: the chunk's real units warp, warp + 4, ... -------
    auto valid = [&](const Cursor& c) { return c.b < a.B && c.ps + c.p < u1; };
    int issued = 0, mine = 0;
    Cursor ic = pl.cur;  // issue cursor: at this warp's next unit to load
    bool ic_ok = false;  // ic is inside the chunk
    int blk_next = 0;    // (lane 0) block id of the unit at ic
    auto issue_one = [&](bool load_next) {
        if (lane == 0) {
            const int slot = issued % RING;
            const int blk = blk_next;
            slot_blk[slot] = blk;
            if (blk < 0 || (long long)blk >= a.num_blocks) {
                mbar_arrive(&bars[slot]);  // nothing to load; the consumer masks the page
            } else {
                mbar_arrive_expect_tx(&bars[slot], C::SLOT_BYTES);
                const int row0 = (blk * a.L + a.layer) * (2 * kBS);
#pragma unroll
                for (int r = 0; r < REG; ++r)
                    tma_load_3d(slots + (size_t)slot * C::SLOT_BYTES + r * (32 * 128), &kv_map, &bars[slot], 64 * r,
                                ic.h, row0);
            }
        }
        ++issued;
        cursor_advance<ROPE, PAD>(ic, a, kNW);
        ic_ok = valid(ic);
        if (ic_ok) {
            if (load_next && lane == 0) {
                const int32_t* row = a.bt + (long long)ic.b * a.maxb;
                blk_next = row[ic.p];
                // the table line 8 own units ahead (own pages are kNW apart), so that
                // the load above hits L1 when it gets there
                if (ic.p + 8 * kNW < ic.np) prefetch_l1(row + ic.p + 8 * kNW);
            }
        }
    };
    // drains this warp's loads still in flight (bounded) before it leaves
    auto drain = [&]() {
        for (int j = mine; j < issued; ++j) (void)mbar_wait_bounded(&bars[j % RING], (j / RING) & 1);
        mine = issued;
    };

    if (has_work) {
        // prime the ring: lane 0 issues the loads of the first own units back to
        // back, with the block ids read with the plan
        cursor_advance<ROPE, PAD>(ic, a, warp);
        ic_ok = valid(ic);
        for (int j = 0; j < pi.count; ++j) {
            blk_next = __shfl_sync(FULL, prime_blk, j);
            issue_one(false);
        }
        if (ic_ok) blk_next = __shfl_sync(FULL, prime_blk, pi.count);
    }

    Segment seg;
    seg.c = pl.cur;
    seg.r0 = 0;
    seg.len = has_work ? pages_before(pl.cur, a, u1) : 0;

    bool ok = true;  // this warp's waits all completed
    while (seg.len > 0) {
        const int ctx_b = seg.c.n;
        const bool whole = seg.c.p == 0 && seg.len == seg.c.np;
        // ---- segment start: (rotate,) split and pack the staged query ----------
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
        {
            const bool live = qr < G;
            const long long qrow = ((long long)seg.c.b * a.H + (long long)seg.c.h * G + (live ? qr : 0)) * D;
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
                if constexpr (!QSPLIT) {
                    qb[kk][0] = qn[kk][0];
                    qb[kk][1] = qn[kk][1];
                } else {
                    const int d0 = kk * 16 + 2 * qc, d1 = d0 + 8;
                    float x[4] = {qs[kk][0], qs[kk][1], qs[kk][2], qs[kk][3]};
                    if (a.q_f16) {  // staged as fp16 pairs
                        const float2 u = unpack_h2(__float_as_uint(qs[kk][0])), v = unpack_h2(__float_as_uint(qs[kk][1]));
                        x[0] = u.x; x[1] = u.y; x[2] = v.x; x[3] = v.y;
                    }
                    if (ROPE && live) {
                        const float2 c0 = csn[kk][0], c1 = csn[kk][1];
                        rope_pair(x[0], x[1], c0.x, c0.y, x[0], x[1]);
                        rope_pair(x[2], x[3], c1.x, c1.y, x[2], x[3]);
                        if (a.q_out && seg.c.p == 0 && warp == 0) {
                            if (a.q_f16) {
                                *reinterpret_cast<uint32_t*>(reinterpret_cast<__half*>(a.q_out) + qrow + d0) = pack_h2(x[0], x[1]);
                                *reinterpret_cast<uint32_t*>(reinterpret_cast<__half*>(a.q_out) + qrow + d1) = pack_h2(x[2], x[3]);
                            } else {
                                *reinterpret_cast<float2*>(reinterpret_cast<float*>(a.q_out) + qrow + d0) = make_float2(x[0], x[1]);
                                *reinterpret_cast<float2*>(reinterpret_cast<float*>(a.q_out) + qrow + d1) = make_float2(x[2], x[3]);
                            }
                        }
                    }
                    qb[kk][0] = pack_h2(x[0], x[1]);
                    qb[kk][1] = pack_h2(x[2], x[3]);
                    if constexpr (QSPLIT) {
                        const float2 hA = unpack_h2(qb[kk][0]), hB = unpack_h2(qb[kk][1]);
                        ql[kk][0] = pack_h2(x[0] - hA.x, x[1] - hA.y);
                        ql[kk][1] = pack_h2(x[2] - hB.x, x[3] - hB.y);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) o[kk][i] = 0.f;
            }
        }
        // stage the next segment's query now: its loads overlap this segment's pages
        unsigned long long ctr_hint = 0;  // the pair's arrival counter, read a segment early
        {
            Segment nx = seg;
            next_segment<ROPE, PAD>(nx, a, u1);
            if (nx.len > 0) load_q(nx.c.b, nx.c.h, nx.c.n);
            if (!whole && threadIdx.x == 0)
                ctr_hint = ld_relaxed_u64(a.counters + 1 + (long long)seg.c.b * a.Hkv + seg.c.h);
        }

        // ---- this warp's pages of the segment ----------------------------------
        const int o0 = ((warp - seg.r0) % kNW + kNW) % kNW;
        for (int off = o0; off < seg.len && ok; off += kNW) {
            const int p = seg.c.p + off;
            const int slot = mine % RING;
            ok = __all_sync(FULL, mbar_wait_bounded(&bars[slot], (mine / RING) & 1));
            if (!ok) {
                if (lane == 0) {
                    report(a.status, COTTUS_STATUS_TIMEOUT);
                    s_abort = 1;
                }
                ++mine;
                drain();
                break;
            }
            const int blk = slot_blk[slot];
            const bool blk_ok = blk >= 0 && (long long)blk < a.num_blocks;
            if (!blk_ok && lane == 0) report(a.status, COTTUS_STATUS_BAD_BLOCK_ID);
            int n_valid = blk_ok ? ctx_b - p * kBS : 0;
            n_valid = n_valid > kBS ? kBS : n_valid;
            uint8_t* sl = slots + (size_t)slot * C::SLOT_BYTES;
            const uint32_t sl_s = slots_s + (uint32_t)(slot * C::SLOT_BYTES);

            if (ROPE && blk_ok && p == seg.c.np - 1 && lane < LW)
                append_new_token<D>(sl, a.kv, a.k_new, a.v_new, a.cos_sin, a.q_f16, blk, a.L, a.layer, a.Hkv,
                                    seg.c.b, seg.c.h, ctx_b, lane);
            if (n_valid < kBS) {
                // V rows past the context may hold any bits (NaN, inf); zero them
                // so that 0-probability tokens contribute exactly 0
                const int nz = (kBS - n_valid) * REG * 8;  // 16-byte chunks
                for (int i = lane; i < nz; i += 32) {
                    const int row = n_valid + i / (REG * 8), rc = i % (REG * 8);
                    *reinterpret_cast<uint4*>(sl + swz(rc / 8, kBS + row, rc % 8)) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            if (ROPE || n_valid < kBS) __syncwarp();

            // ---- S^T = K . Q^T ----------------------------------------------------
            // two independent accumulator chains (hi and lo query parts, or even and
            // odd k-steps), added at the end: half the dependent MMA latency
            float s[4] = {0.f, 0.f, 0.f, 0.f};
            {
                float s2[4] = {0.f, 0.f, 0.f, 0.f};
                const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
                const int csel = lane >> 4;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    uint32_t af[4];
                    ldsm_x4(sl_s + swz(kk / 4, row, (kk % 4) * 2 + csel), af);
                    if constexpr (QSPLIT) {
                        mma16816(s, af, qb[kk][0], qb[kk][1]);
                        mma16816(s2, af, ql[kk][0], ql[kk][1]);
                    } else if (kk & 1) {
                        mma16816(s2, af, qb[kk][0], qb[kk][1]);
                    } else {
                        mma16816(s, af, qb[kk][0], qb[kk][1]);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) s[i] += s2[i];
            }
            // ---- online softmax on the fragment -----------------------------------
            const bool ok0 = qr < n_valid, ok1 = qr + 8 < n_valid;
            const float s00 = ok0 ? s[0] * a.qscale : -INFINITY, s01 = ok0 ? s[1] * a.qscale : -INFINITY;
            const float s10 = ok1 ? s[2] * a.qscale : -INFINITY, s11 = ok1 ? s[3] * a.qscale : -INFINITY;
            // The running max is raised only when the page's max exceeds it by
            // more than 8; one vote on the lanes' own scores decides whether the
            // page's max is needed at all (the same decisions as reducing it on
            // every page, without the 3 dependent shuffles on most pages).
            float c0 = fmaxf(s00, s10), c1 = fmaxf(s01, s11);
            if (!vote_max<D, G>() || __any_sync(FULL, c0 > m0 + 8.0f || c1 > m1 + 8.0f)) {
#pragma unroll
                for (int sh = 4; sh < 32; sh <<= 1) {
                    c0 = fmaxf(c0, __shfl_xor_sync(FULL, c0, sh));
                    c1 = fmaxf(c1, __shfl_xor_sync(FULL, c1, sh));
                }
                if (c0 > m0 + 8.0f) {
                    const float al = exp2f(m0 - c0);
                    m0 = c0;
                    l0 *= al;
#pragma unroll
                    for (int j = 0; j < KS; ++j) {
                        o[j][0] *= al;
                        o[j][2] *= al;
                    }
                }
                if (c1 > m1 + 8.0f) {
                    const float al = exp2f(m1 - c1);
                    m1 = c1;
                    l1 *= al;
#pragma unroll
                    for (int j = 0; j < KS; ++j) {
                        o[j][1] *= al;
                        o[j][3] *= al;
                    }
                }
            }
            const float p00 = ok0 ? exp2f(s00 - m0) : 0.f, p01 = ok0 ? exp2f(s01 - m1) : 0.f;
            const float p10 = ok1 ? exp2f(s10 - m0) : 0.f, p11 = ok1 ? exp2f(s11 - m1) : 0.f;
            l0 += p00 + p10;
            l1 += p01 + p11;
            const uint32_t pb0 = movmatrix_trans(pack_h2(p00, p01));  // tokens 0-7
            const uint32_t pb1 = movmatrix_trans(pack_h2(p10, p11));  // tokens 8-15
            uint32_t pl0 = 0u, pl1 = 0u;  // fp32 outputs: the remainders of the fp16 roundings
            if constexpr (PSPLIT) {
                const float2 e0 = unpack_h2(pack_h2(p00, p01)), e1 = unpack_h2(pack_h2(p10, p11));
                pl0 = movmatrix_trans(pack_h2(p00 - e0.x, p01 - e0.y));
                pl1 = movmatrix_trans(pack_h2(p10 - e1.x, p11 - e1.y));
            }

            // ---- O^T += V^T . P^T --------------------------------------------------
            {
                const int tok = (lane & 7) + ((lane >> 4) & 1) * 8;
                const int csel = (lane >> 3) & 1;
#pragma unroll
                for (int j = 0; j < KS; ++j) {
                    uint32_t af[4];
                    ldsm_x4_t(sl_s + swz(j / 4, kBS + tok, (j % 4) * 2 + csel), af);
                    mma16816(o[j], af, pb0, pb1);
                    if constexpr (PSPLIT) mma16816(o[j], af, pl0, pl1);
                }
            }
            __syncwarp();
            ++mine;
            if (ic_ok) {
                fence_proxy_async_smem();
                issue_one(true);
            }
        }

        // ---- segment end: merge the warps' states in shared memory --------------
        {
            float lt0 = l0, lt1 = l1;
#pragma unroll
            for (int sh = 4; sh < 32; sh <<= 1) {
                lt0 += __shfl_xor_sync(FULL, lt0, sh);
                lt1 += __shfl_xor_sync(FULL, lt1, sh);
            }
            float* mo = merge_o + warp * G * OST;
            float* mml = merge_ml + warp * G * 2;
            if (h0 < G) {
#pragma unroll
                for (int j = 0; j < KS; ++j) {
                    mo[h0 * OST + j * 16 + qr] = o[j][0];
                    mo[h0 * OST + j * 16 + qr + 8] = o[j][2];
                }
                if (qr == 0) {
                    mml[h0 * 2] = m0;
                    mml[h0 * 2 + 1] = lt0;
                }
            }
            if (h1 < G) {
#pragma unroll
                for (int j = 0; j < KS; ++j) {
                    mo[h1 * OST + j * 16 + qr] = o[j][1];
                    mo[h1 * OST + j * 16 + qr + 8] = o[j][3];
                }
                if (qr == 0) {
                    mml[h1 * 2] = m1;
                    mml[h1 * 2 + 1] = lt1;
                }
            }
        }
        __syncthreads();
        if (s_abort) {  // every warp sees the same flag after the barrier
            drain();
            return;
        }
        const long long slot_id = seg.c.ps <= u0 ? 2 * cid : 2 * cid + 1;
        constexpr int ITEMS = G * D / 4;  // (head, 4 dims)
        for (int it = threadIdx.x; it < ITEMS; it += kNW * 32) {
            const int g = it / (D / 4), c4 = it % (D / 4);
            float M = -INFINITY;
            float mw[kNW];
#pragma unroll
            for (int w = 0; w < kNW; ++w) {
                mw[w] = merge_ml[(w * G + g) * 2];
                M = fmaxf(M, mw[w]);
            }
            float L = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < kNW; ++w) {
                    if (mw[w] == -INFINITY) continue;
                    const float sc = exp2f(mw[w] - M);
                    L += merge_ml[(w * G + g) * 2 + 1] * sc;
                    const float4 x = *reinterpret_cast<const float4*>(merge_o + (w * G + g) * OST + c4 * 4);
                    acc.x += x.x * sc;
                    acc.y += x.y * sc;
                    acc.z += x.z * sc;
                    acc.w += x.w * sc;
                }
            }
            const long long head = (long long)seg.c.b * a.H + (long long)seg.c.h * G + g;
            if (whole) {
                const float inv = L > 0.f ? 1.0f / L : 0.f;
                const float v4[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
                if (a.out_f16) {
                    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(a.out) + head * D + c4 * 4) =
                        make_uint2(pack_h2(v4[0], v4[1]), pack_h2(v4[2], v4[3]));
                } else {
                    *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + head * D + c4 * 4) =
                        make_float4(v4[0], v4[1], v4[2], v4[3]);
                }
                if (a.lse && c4 == 0) a.lse[head] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
            } else {
                *reinterpret_cast<float4*>(a.ws_o + (slot_id * G + g) * D + c4 * 4) = acc;
                if (c4 == 0) *reinterpret_cast<float2*>(a.ws_ml + (slot_id * G + g) * 2) = make_float2(M, L);
            }
        }
        if (!whole) {
            const MergeArgs ma = {a.counters, a.ws_o, a.ws_ml, a.out, a.lse, a.H, a.Hkv, a.out_f16, a.epoch};
            arrive_cut_pair<D, G>(ma, chunk, seg.c.b, seg.c.h, seg.c.np, seg.c.ps, ctr_hint, &s_last);
        }
        __syncthreads();  // the merge area is free for the next segment
        next_segment<ROPE, PAD>(seg, a, u1);
    }

    // ---- split-context completion signal: once every CTA has stored its outputs ----
    if (a.sig.world != 0) {
        __threadfence();  // this thread's outputs, before the CTA counts itself
        __syncthreads();
    }
    if (a.sig.world != 0 && threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.sig.done, 1u) == gridDim.x - 1) {
            *reinterpret_cast<volatile unsigned*>(a.sig.done) = 0u;  // for the next launch
            __threadfence_system();
            for (int r = 0; r < a.sig.world; ++r)
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.sig.flags[r] + a.sig.rank), "r"(a.sig.epoch)
                             : "memory");
        }
    }

    // ---- split-context merge in the same launch --------------------------------
    // Every CTA waits (bounded) until every rank's flag has reached this step
    // (its own flag included: then every CTA of this launch has stored its
    // partials), then merges rows CTA-strided, one warp per (sequence, head),
    // all ranks' loads in flight together (merge_head_parts: the arithmetic of
    // cottus_lse_combine, so the NCCL path gives the same bits).  The grid is
    // one CTA per resident slot, so the CTAs that wait do not keep the others
    // from running.  A serial-number comparison accepts a peer one step ahead.
    // Only the CTAs that have rows to merge (one row per warp) wait; the
    // others leave at once, so that the next launch's CTAs can take their
    // slots and run their prologue during the exchange.
    if (a.pm.enabled) {
        const long long rows = (long long)a.B * a.H;
        const long long mctas = min((long long)gridDim.x, (rows + kNW - 1) / kNW);
        if (cid >= mctas) return;
        if (threadIdx.x == 0) {
            bool ready = ld_acquire_sys(a.pm.broken_own) == 0u;
            const long long t0 = clock64();
            for (int r = 0; r < a.sig.world && ready; ++r)
                while ((int32_t)(ld_acquire_sys(a.pm.flags + r) - a.sig.epoch) < 0)
                    if (clock64() - t0 > a.pm.wait_cycles) {
                        ready = false;
                        break;
                    }
            s_last = ready;
            if (!ready) {
                report(a.status, COTTUS_STATUS_TIMEOUT);
                // every later step of every rank refuses at once
                for (int r = 0; r < a.sig.world; ++r)
                    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.pm.broken[r]), "r"(1u) : "memory");
            }
        }
        __syncthreads();
        if (s_last) {
            for (long long hw = cid * kNW + warp; hw < rows; hw += mctas * kNW)
                merge_head_parts(a.pm.lse, a.pm.part, a.sig.world, hw, D, lane, a.pm.out, a.pm.out_f16,
                                 a.pm.lse_out);
        }
    }
}

template <int D, int G, int RING, bool ROPE, bool QSPLIT, bool PSPLIT>
struct MmaLauncher {
    static int blocks_per_sm(int device) {
        static int cache[64] = {0};
        if (device < 0 || device >= 64) return 1;
        if (cache[device] == 0) {
            auto kern = decode_mma_kernel<D, G, RING, ROPE, QSPLIT, PSPLIT>;
            const size_t smem = mma_smem_bytes<RING, D, G>();
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            int n = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kNW * 32, smem);
            cache[device] = n > 0 ? n : 1;
        }
        return cache[device];
    }
    // workers: one per CTA
    static long long workers(int device) { return (long long)device_sm_count(device) * blocks_per_sm(device); }
    static cudaError_t launch(const DecodeDesc& d, cudaStream_t st) {
        int dev = 0;
        cudaGetDevice(&dev);
        const long long W = workers(dev);
        cudaError_t err = cudaSuccess;
        const CUtensorMap map = make_kv_tensor_map(d, true, &err);
        if (err != cudaSuccess) return err;
        TmaArgs a = make_tma_args(d, W, G, D);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)W);
        cfg.blockDim = dim3(kNW * 32);
        cfg.dynamicSmemBytes = mma_smem_bytes<RING, D, G>();
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, decode_mma_kernel<D, G, RING, ROPE, QSPLIT, PSPLIT>, map, a);
    }
};

template <int D, int RING, bool ROPE, bool QSPLIT, bool PSPLIT>
cudaError_t dispatch_mma_g(const DecodeDesc& d, cudaStream_t st, bool workers_only, long long* W) {
    int dev = 0;
    cudaGetDevice(&dev);
    switch (d.num_heads / d.num_kv_heads) {  // grouped queries only: MHA takes the SIMT kernel
#define CB200_CASE(GG)                                                           \
    case GG:                                                                     \
        if (workers_only) {                                                      \
            *W = MmaLauncher<D, GG, RING, ROPE, QSPLIT, PSPLIT>::workers(dev);   \
            return cudaSuccess;                                                  \
        }                                                                        \
        return MmaLauncher<D, GG, RING, ROPE, QSPLIT, PSPLIT>::launch(d, st);
        CB200_CASE(2)
        CB200_CASE(4)
        CB200_CASE(8)
#undef CB200_CASE
    }
    return cudaErrorInvalidValue;
}

// fp32 outputs (not LSE partials) split the probabilities too.
template <int D, int RING, bool PSPLIT>
cudaError_t dispatch_mma_p(const DecodeDesc& d, cudaStream_t st, bool workers_only, long long* W) {
    if (d.rope) return dispatch_mma_g<D, RING, true, true, PSPLIT>(d, st, workers_only, W);
    if (d.q_f16) return dispatch_mma_g<D, RING, false, false, PSPLIT>(d, st, workers_only, W);
    return dispatch_mma_g<D, RING, false, true, PSPLIT>(d, st, workers_only, W);
}

template <int D, int RING>
cudaError_t dispatch_mma(const DecodeDesc& d, cudaStream_t st, bool workers_only, long long* W) {
    if (!d.out_f16 && d.lse == nullptr) return dispatch_mma_p<D, RING, true>(d, st, workers_only, W);
    return dispatch_mma_p<D, RING, false>(d, st, workers_only, W);
}

}  // namespace cb200
