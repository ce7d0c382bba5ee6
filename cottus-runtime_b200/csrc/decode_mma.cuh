// Paged decode attention with the QK and PV tile products on the tensor
// cores (warp-level mma.sync m16n8k16, fp16 inputs, fp32 accumulation).
//
// Same stream-K schedule, per-warp TMA ring, merge and epilogue contract as
// decode_tma_kernel; only the math per page differs:
//
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

template <int D>
struct MmaCfg {
    static constexpr int KSTEPS = D / 16;   // QK k-steps = PV dim tiles
    static constexpr int REGIONS = D / 64;  // 128-byte column regions per slot
    static constexpr int SLOT_BYTES = 2 * kBS * D * 2;
};

template <int RING, int D>
constexpr size_t mma_smem_bytes() {
    return (size_t)kNW * RING * MmaCfg<D>::SLOT_BYTES + (size_t)kNW * RING * 8 + (size_t)kNW * RING * 4 + 1024;
}

// CTAs per SM the register budget is fitted to: two.  Three (168
// registers) keep more pages in flight, but the launch then has 1.5x the
// workers, so more (sequence, kv head) pairs are cut between workers and
// merged at the end: measured on the Llama-3-8B shape (batch 64, context
// 2048), 94.8 us per step with three against 90.5 us with two.
constexpr int kMmaMinCtas = 2;

template <int D, int G, int RING, bool ROPE, bool QSPLIT, bool PSPLIT>
__global__ void __launch_bounds__(kNW * 32, kMmaMinCtas)
    decode_mma_kernel(const __grid_constant__ CUtensorMap kv_map, const TmaArgs a) {
    using C = MmaCfg<D>;
    constexpr int KS = C::KSTEPS, REG = C::REGIONS, LW = D / 8;
    constexpr unsigned FULL = 0xffffffffu;
    static_assert(G <= 8, "group larger than the MMA n dimension");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* slots = smem + (size_t)warp * RING * C::SLOT_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kNW * RING * C::SLOT_BYTES) + warp * RING;
    int* slot_blk =
        reinterpret_cast<int*>(smem + (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 8) + warp * RING;

    __shared__ unsigned cta_done;  // warps of this CTA that finished (split-context signal)
    if (lane == 0) {
        if (warp == 0) {
            prefetch_tensormap(&kv_map);
            cta_done = 0;
        }
#pragma unroll
        for (int r = 0; r < RING; ++r) mbar_init(&bars[r], 1);
        fence_barrier_init();
    }
    __syncthreads();

    const long long W = (long long)gridDim.x * kNW;
    const long long w = (long long)blockIdx.x * kNW + warp;
    warm_first_pages<ROPE>(a, &kv_map, w, W, lane, REG, 64);
    grid_dependency_wait();
    grid_dependents_launch();
    const WorkerPlan pl = plan_worker<D, ROPE>(a, w, W, lane);
    const long long U = pl.U, chunk = pl.chunk;
    const long long NC = (U + chunk - 1) / chunk;

    // fragment coordinates of this lane
    const int qc = lane & 3;   // column pair: heads 2qc, 2qc+1 of C fragments
    const int qr = lane >> 2;  // row: token qr / qr+8 of C fragments; head qr of B fragments
    const int h0 = 2 * qc, h1 = 2 * qc + 1;
    const uint32_t slots_s = smem_addr(slots);

    uint32_t qb[KS][2];
    uint32_t ql[QSPLIT ? KS : 1][2];
    float o[KS][4];
    // query of the next segment, loaded a page early: raw fp32 values where
    // they get split (fp32 or rotated queries), else the fp16 pairs as stored
    float qs[QSPLIT ? KS : 1][4];
    uint32_t qn[QSPLIT ? 1 : KS][2];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    // this lane's query elements of pair (b, h): head qr, dims kk*16 + 2qc + {0, 1, 8, 9}
    auto load_q = [&](int b, int h) {
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
                float2 u = make_float2(0.f, 0.f), v = make_float2(0.f, 0.f);
                if (live) {
                    if (a.q_f16) {
                        u = unpack_h2(__ldg(reinterpret_cast<const unsigned*>(reinterpret_cast<const __half*>(a.q) + qrow + d0)));
                        v = unpack_h2(__ldg(reinterpret_cast<const unsigned*>(reinterpret_cast<const __half*>(a.q) + qrow + d1)));
                    } else {
                        u = __ldg(reinterpret_cast<const float2*>(reinterpret_cast<const float*>(a.q) + qrow + d0));
                        v = __ldg(reinterpret_cast<const float2*>(reinterpret_cast<const float*>(a.q) + qrow + d1));
                    }
                }
                qs[kk][0] = u.x; qs[kk][1] = u.y; qs[kk][2] = v.x; qs[kk][3] = v.y;
            }
        }
    };

    // ---- work: static chunk w, then chunks from the queue ------------------
    long long cid = w < NC ? w : (NC > W ? grab_chunk(a, W, NC, lane) : NC);
    Cursor cur = pl.cur;
    bool have_cur = w < NC;  // the plan located chunk w's first unit
    int kg = 0;              // units consumed by this warp so far (ring slot / phase counter)

    while (cid < NC) {
        const long long u0 = cid * chunk, u1 = min(u0 + chunk, U);
        const int nu = (int)(u1 - u0);
        if (!have_cur) cur = locate_unit<ROPE>(a, u0, lane);
        have_cur = false;

        // ---- TMA issue (lane 0), block id prefetched one page ahead ----------
        Cursor ic = cur;
        int blk_next = lane == 0 ? a.bt[(long long)ic.b * a.maxb + ic.p] : 0;
        auto issue = [&](int k) {
            if (lane == 0) {
                const int slot = (kg + k) % RING;
                const int blk = blk_next;
                slot_blk[slot] = blk;
                if (blk < 0 || (long long)blk >= a.num_blocks) {
                    mbar_arrive(&bars[slot]);
                } else {
                    mbar_arrive_expect_tx(&bars[slot], C::SLOT_BYTES);
                    const int row0 = (blk * a.L + a.layer) * (2 * kBS);
#pragma unroll
                    for (int r = 0; r < REG; ++r)
                        tma_load_3d(slots + (size_t)slot * C::SLOT_BYTES + r * (32 * 128), &kv_map, &bars[slot], 64 * r,
                                    ic.h, row0);
                }
                cursor_next<ROPE>(ic, a);
                if (k + 1 < nu) blk_next = a.bt[(long long)ic.b * a.maxb + ic.p];
            }
        };
        const int prime = nu < RING ? nu : RING;
        for (int k = 0; k < prime; ++k) issue(k);
        load_q(cur.b, cur.h);

        bool seg_open = false, seg_first = true;
        int seg_start_p = 0;
        unsigned long long ctr_hint = 0;  // arrival counter of the open segment's pair, read a page early
        for (int k = 0; k < nu; ++k) {
            const int slot = (kg + k) % RING;
            const int ctx_b = cur.n;
            if (!seg_open) {
                // ---- segment start: (rotate,) split and pack the staged query ----
                seg_open = true;
                seg_first = (k == 0);
                seg_start_p = cur.p;
                ctr_hint = 0;
                m0 = m1 = -INFINITY;
                l0 = l1 = 0.f;
                const bool live = qr < G;
                const long long qrow = ((long long)cur.b * a.H + (long long)cur.h * G + (live ? qr : 0)) * D;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    if constexpr (!QSPLIT) {
                        qb[kk][0] = qn[kk][0];
                        qb[kk][1] = qn[kk][1];
                    } else {
                        const int d0 = kk * 16 + 2 * qc, d1 = d0 + 8;
                        float x[4] = {qs[kk][0], qs[kk][1], qs[kk][2], qs[kk][3]};
                        if (ROPE && live) {
                            const float* cs = a.cos_sin + (long long)(ctx_b - 1) * D;  // row of D/2 (cos, sin) pairs
                            const float2 c0 = *reinterpret_cast<const float2*>(cs + d0);
                            const float2 c1 = *reinterpret_cast<const float2*>(cs + d1);
                            rope_pair(x[0], x[1], c0.x, c0.y, x[0], x[1]);
                            rope_pair(x[2], x[3], c1.x, c1.y, x[2], x[3]);
                            if (a.q_out && cur.p == 0) {
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
            if (cur.p == cur.np - 1 && k + 1 < nu) {
                // this page ends the segment: stage the next pair's query now so
                // the load latency hides behind this page's math
                Cursor nx = cur;
                cursor_next<ROPE>(nx, a);
                load_q(nx.b, nx.h);
            }

            const bool landed = __all_sync(FULL, mbar_wait_bounded(&bars[slot], ((kg + k) / RING) & 1));
            if (!landed) {
                if (lane == 0) report(a.status, COTTUS_STATUS_TIMEOUT);
                for (int kk = k + 1; kk < k + RING && kk < nu; ++kk)
                    (void)__all_sync(FULL, mbar_wait_bounded(&bars[(kg + kk) % RING], ((kg + kk) / RING) & 1));
                return;
            }
            const int blk = slot_blk[slot];
            const bool blk_ok = blk >= 0 && (long long)blk < a.num_blocks;
            if (!blk_ok && lane == 0) report(a.status, COTTUS_STATUS_BAD_BLOCK_ID);
            int n_valid = blk_ok ? ctx_b - cur.p * kBS : 0;
            n_valid = n_valid > kBS ? kBS : n_valid;
            uint8_t* sl = slots + (size_t)slot * C::SLOT_BYTES;
            const uint32_t sl_s = slots_s + (uint32_t)(slot * C::SLOT_BYTES);

            if (ROPE && blk_ok && cur.p == cur.np - 1 && lane < LW) {
                // the new token: rotate k, encode k and v (truncation), append
                const int t_new = (ctx_b - 1) % kBS;
                const long long src = ((long long)cur.b * a.Hkv + cur.h) * D + lane * 8;
                float kx[8], vx[8];
                if (a.q_f16) {
                    load8(reinterpret_cast<const __half*>(a.k_new) + src, kx);
                    load8(reinterpret_cast<const __half*>(a.v_new) + src, vx);
                } else {
                    load8(reinterpret_cast<const float*>(a.k_new) + src, kx);
                    load8(reinterpret_cast<const float*>(a.v_new) + src, vx);
                }
                const float4* cs =
                    reinterpret_cast<const float4*>(a.cos_sin + ((long long)(ctx_b - 1) * (D / 2) + lane * 4) * 2);
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
                const long long row0 = ((long long)blk * a.L + a.layer) * (2 * kBS);
                *reinterpret_cast<uint4*>(a.kv + ((row0 + t_new) * a.Hkv + cur.h) * D + lane * 8) = k4;
                *reinterpret_cast<uint4*>(a.kv + ((row0 + kBS + t_new) * a.Hkv + cur.h) * D + lane * 8) = v4;
            }
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
            float s[4] = {0.f, 0.f, 0.f, 0.f};
            {
                const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
                const int csel = lane >> 4;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    uint32_t af[4];
                    ldsm_x4(sl_s + swz(kk / 4, row, (kk % 4) * 2 + csel), af);
                    mma16816(s, af, qb[kk][0], qb[kk][1]);
                    if constexpr (QSPLIT) mma16816(s, af, ql[kk][0], ql[kk][1]);
                }
            }
            // ---- online softmax on the fragment -----------------------------------
            const bool ok0 = qr < n_valid, ok1 = qr + 8 < n_valid;
            const float s00 = ok0 ? s[0] * a.qscale : -INFINITY, s01 = ok0 ? s[1] * a.qscale : -INFINITY;
            const float s10 = ok1 ? s[2] * a.qscale : -INFINITY, s11 = ok1 ? s[3] * a.qscale : -INFINITY;
            float c0 = fmaxf(s00, s10), c1 = fmaxf(s01, s11);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                c0 = fmaxf(c0, __shfl_xor_sync(FULL, c0, off));
                c1 = fmaxf(c1, __shfl_xor_sync(FULL, c1, off));
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
            const float p00 = ok0 ? exp2f(s00 - m0) : 0.f, p01 = ok0 ? exp2f(s01 - m1) : 0.f;
            const float p10 = ok1 ? exp2f(s10 - m0) : 0.f, p11 = ok1 ? exp2f(s11 - m1) : 0.f;
            l0 += p00 + p10;
            l1 += p01 + p11;
            const uint32_t pb0 = movmatrix_trans(pack_h2(p00, p01));  // tokens 0-7
            const uint32_t pb1 = movmatrix_trans(pack_h2(p10, p11));  // tokens 8-15
            uint32_t pl0 = 0u, pl1 = 0u;  // fp32 outputs: the remainders of the fp16 roundings
            if constexpr (PSPLIT) {
                const float2 h0 = unpack_h2(pack_h2(p00, p01)), h1 = unpack_h2(pack_h2(p10, p11));
                pl0 = movmatrix_trans(pack_h2(p00 - h0.x, p01 - h0.y));
                pl1 = movmatrix_trans(pack_h2(p10 - h1.x, p11 - h1.y));
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

            if (k + RING < nu) {
                fence_proxy_async_smem();
                issue(k + RING);
            }

            // the next page ends a cut segment of this pair: read the pair's
            // arrival counter now, so the arrival's compare-and-swap finds it
            if (lane == 0 && k + 1 < nu && cur.p + 1 < cur.np && (cur.p + 2 == cur.np || k + 2 == nu) &&
                !(seg_start_p == 0 && cur.p + 2 == cur.np))
                ctr_hint = ld_relaxed_u64(a.counters + 1 + (long long)cur.b * a.Hkv + cur.h);

            const bool seg_end = (cur.p == cur.np - 1) || (k == nu - 1);
            if (seg_end) {
                float lt0 = l0, lt1 = l1;
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    lt0 += __shfl_xor_sync(FULL, lt0, off);
                    lt1 += __shfl_xor_sync(FULL, lt1, off);
                }
                const bool whole = seg_start_p == 0 && cur.p == cur.np - 1;
                const long long slot_id = seg_first ? 2 * cid : 2 * cid + 1;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int g = hh ? h1 : h0;
                    if (g >= G) continue;
                    const float mg = hh ? m1 : m0, lg = hh ? lt1 : lt0;
                    const long long head = (long long)cur.b * a.H + (long long)cur.h * G + g;
                    if (whole) {
                        const float inv = lg > 0.f ? 1.0f / lg : 0.f;
#pragma unroll
                        for (int j = 0; j < KS; ++j) {
                            const float x0 = o[j][hh] * inv, x1 = o[j][2 + hh] * inv;
                            const long long e0 = head * D + j * 16 + qr;
                            if (a.out_f16) {
                                reinterpret_cast<__half*>(a.out)[e0] = __float2half_rn(x0);
                                reinterpret_cast<__half*>(a.out)[e0 + 8] = __float2half_rn(x1);
                            } else {
                                reinterpret_cast<float*>(a.out)[e0] = x0;
                                reinterpret_cast<float*>(a.out)[e0 + 8] = x1;
                            }
                        }
                        if (a.lse && qr == 0) a.lse[head] = lg > 0.f ? (mg + log2f(lg)) * kLn2 : -INFINITY;
                    } else {
                        float* dst = a.ws_o + (slot_id * G + g) * D;
#pragma unroll
                        for (int j = 0; j < KS; ++j) {
                            dst[j * 16 + qr] = o[j][hh];
                            dst[j * 16 + qr + 8] = o[j][2 + hh];
                        }
                        if (qr == 0) {
                            a.ws_ml[(slot_id * G + g) * 2] = mg;
                            a.ws_ml[(slot_id * G + g) * 2 + 1] = lg;
                        }
                    }
                }
                if (!whole)
                    merge_if_last<D, G>(a, cur.b, cur.h, u0 + k - cur.p, cur.np, chunk, lane, ctr_hint);
                __syncwarp();
                seg_open = false;
            }
            if (k + 1 < nu) cursor_next<ROPE>(cur, a);
        }
        kg += nu;
        cid = NC > W ? grab_chunk(a, W, NC, lane) : NC;
    }
    signal_done(a, lane, &cta_done);
}

template <int D, int G, int RING, bool ROPE, bool QSPLIT, bool PSPLIT>
struct MmaLauncher {
    static int blocks_per_sm(int device) {
        static int cache[64] = {0};
        if (device < 0 || device >= 64) return 1;
        if (cache[device] == 0) {
            auto kern = decode_mma_kernel<D, G, RING, ROPE, QSPLIT, PSPLIT>;
            const size_t smem = mma_smem_bytes<RING, D>();
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            int n = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kNW * 32, smem);
            cache[device] = n > 0 ? n : 1;
        }
        return cache[device];
    }
    static long long workers(int device) {
        return (long long)device_sm_count(device) * blocks_per_sm(device) * kNW;
    }
    static cudaError_t launch(const DecodeDesc& d, cudaStream_t st) {
        int dev = 0;
        cudaGetDevice(&dev);
        const long long W = workers(dev);
        cudaError_t err = cudaSuccess;
        const CUtensorMap map = make_kv_tensor_map(d, true, &err);
        if (err != cudaSuccess) return err;
        TmaArgs a = make_tma_args(d, W, G, D);
        return launch_pdl(decode_mma_kernel<D, G, RING, ROPE, QSPLIT, PSPLIT>, (int)(W / kNW), mma_smem_bytes<RING, D>(), st,
                          map, a);
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
