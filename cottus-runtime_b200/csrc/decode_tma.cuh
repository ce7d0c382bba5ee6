// Paged decode attention, sm_100a fast path.
//
// Work decomposition (stream-K over pages): a unit is one 16-token page of
// one (sequence, kv head) pair; units are ordered sequence-major, then kv
// head, then page.  Every warp of the persistent grid is a worker that owns
// one contiguous chunk of ceil(units / workers) units (at least kMinChunk),
// so skewed (ragged) batches and long contexts balance across the 148 SMs.
//
// Per warp: a ring of RING shared-memory slots, each holding the K and V
// tiles (2 x 16 rows x head_dim fp16) of one page for one kv head, filled
// by a single 3-D TMA load (the K and V rows of a page/layer are adjacent
// in the pool) with completion on an mbarrier; lane 0 refills a slot as
// soon as the warp has consumed it, so RING-1 pages are always in flight.
//
// Math per page: each lane owns 8 consecutive dims of a K/V row (16-byte
// shared loads, conflict-free), keeps the G query rows of the GQA group in
// registers (so each KV byte is read from HBM once per group), computes
// partial dot products with packed fp32x2 FMAs, and reduces them across the
// D/8 lanes of a row with a transpose-reduce (each shuffle level halves the
// values a lane holds).  After the reduction every lane holds the scores of
// ONE head, so the online-softmax max needs only log2(32/G) shuffles.
// Softmax runs in the log2 domain; the running max is only raised when a
// new score exceeds it by more than 8 (so exp2 arguments stay <= 8 and the
// accumulator rescale is rare).  Probabilities go through a per-warp
// shared scratch to the P.V product, again with packed FMAs.
//
// A worker writes a finished (sequence, kv head) pair straight to `out`;
// a pair cut by a worker boundary leaves (m, l, o) partials in the
// workspace; the last worker to finish such a pair (an arrival counter per
// pair) merges its partials, so one launch does the whole decode.
//
// The reference computes the same function per sequence and head with two
// passes over K (paged_attention_cpu.cpp:53-103); results agree to fp32
// rounding (summation order and exp2-vs-exp differ).
#pragma once

#include "common.cuh"
#include "internal.h"

namespace cb200 {

constexpr int kBS = 16;   // tokens per page on the fast path
constexpr int kNW = 4;    // worker warps per CTA
constexpr int kMinChunk = 8;  // fewest pages in a warp's chunk (limits partials on tiny batches)

struct TmaArgs {
    void* out;
    const void* q;
    const int32_t* bt;
    const int32_t* ctx;
    const int32_t* positions;
    float* lse;
    float* ws_o;
    float* ws_ml;
    unsigned long long* counters;  // a reserved word, then [B * Hkv] arrival counters tagged with `epoch`
    uint32_t* status;
    const void* k_new;
    const void* v_new;
    const float* cos_sin;
    void* q_out;
    uint16_t* kv;
    long long num_blocks;
    int B, H, Hkv, L, layer, maxb, max_pos;
    int q_f16, out_f16;
    unsigned epoch;  // per-launch tag of the arrival counters
    float qscale;    // softmax scale * log2(e)
    PeerSignal sig;  // completion signal to the other ranks of a split context
    PeerMerge pm;    // the split context's merge in the same launch (decode_mma_kernel)
};

// End of a warp's work.  In a split-context launch, once every warp of every
// CTA has stored its outputs, the last one tells every rank that this
// rank's partials are complete: a system-scope fence, then flag[rank] =
// epoch in each rank's flag array (peer stores over NVLink).  Each warp's
// outputs are fenced before it counts itself, so the chain of counts carries
// all of them before the fence.  A warp that gave up on a wait never counts,
// and the other ranks' bounded waits report the timeout.
__device__ __forceinline__ void signal_done(const TmaArgs& a, int lane, unsigned* cta_done) {
    if (a.sig.world == 0) return;
    __syncwarp();
    if (lane == 0) {
        __threadfence();
        if (atomicAdd(cta_done, 1u) == kNW - 1) {
            __threadfence();
            if (atomicAdd(a.sig.done, 1u) == gridDim.x - 1) {
                *reinterpret_cast<volatile unsigned*>(a.sig.done) = 0u;  // for the next launch
                __threadfence_system();
                for (int r = 0; r < a.sig.world; ++r)
                    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.sig.flags[r] + a.sig.rank),
                                 "r"(a.sig.epoch)
                                 : "memory");
            }
        }
    }
}

// Pages of sequence b, or 0 when its context is empty or invalid; *ctx_out
// receives the context length.  CG: read at L2 (ld.global.cg), for reads made
// before the wait for the preceding kernel, so that no line of lengths that
// kernel may still write is left in L1.
template <bool ROPE, bool CG = false>
__device__ __forceinline__ int seq_pages(const TmaArgs& a, int b, int* ctx_out = nullptr) {
    int n;
    if (ROPE) {
        const int pos = CG ? __ldcg(a.positions + b) : a.positions[b];
        if (pos < 0 || pos >= a.max_pos) return 0;
        n = pos + 1;
    } else {
        n = CG ? __ldcg(a.ctx + b) : a.ctx[b];
    }
    if (ctx_out) *ctx_out = n;
    if (n <= 0 || n > a.maxb * kBS) return 0;
    return (n + kBS - 1) / kBS;
}
template <bool ROPE>
__device__ __forceinline__ int seq_ctx(const TmaArgs& a, int b) {
    return ROPE ? a.positions[b] + 1 : a.ctx[b];
}

template <int D, int G>
struct TmaCfg {
    static constexpr int LW = D / 8;          // lanes covering one row
    static constexpr int RPS = 32 / LW;       // rows per warp step
    static constexpr int STEPS_MAX = 16 / RPS;
    static constexpr int STEPS = (32 / G) < STEPS_MAX ? (32 / G) : STEPS_MAX;  // steps per chunk
    static constexpr int CH = RPS * STEPS;    // tokens per chunk
    static constexpr int NCH = kBS / CH;      // chunks per page
    static constexpr int N = G * STEPS;       // partial dot products per lane per chunk
    static constexpr int NV = N >= LW ? N / LW : 1;  // values per lane after the reduction
    static constexpr int CL = LW / G;         // lanes per head inside a row group
    static constexpr int DUP = N >= LW ? 1 : LW / N;
    static constexpr int SLOT_BYTES = 2 * kBS * D * 2;
    static_assert(G <= LW, "group larger than lanes per row");
    static_assert(kBS % CH == 0, "chunk must divide the page");
};

template <int RING, int D, int G>
constexpr size_t tma_smem_bytes() {
    using C = TmaCfg<D, G>;
    return (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 8 + (size_t)kNW * C::CH * G * 4 +
           (size_t)kNW * 2 * G * 4 + (size_t)kNW * RING * 4 + 128;
}

// Transpose-reduce: CNT values per lane are summed over the lanes that
// differ in the bits O, O/2, ..., 1; each level keeps half the values.
template <int CNT, int O>
struct TransposeReduce {
    __device__ __forceinline__ static void run(float* v, int lq) {
        if constexpr (O > 0) {
            if constexpr (CNT > 1) {
                constexpr int H = CNT / 2;
                const bool upper = (lq & O) != 0;
#pragma unroll
                for (int i = 0; i < H; ++i) {
                    float send = upper ? v[i] : v[i + H];
                    float keep = upper ? v[i + H] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
                }
                TransposeReduce<H, O / 2>::run(v, lq);
            } else {
                v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
                TransposeReduce<1, O / 2>::run(v, lq);
            }
        }
    }
};

// A position in the unit order.  Units of a pair may be followed by `pad`
// virtual units (no page: they only weigh a pair's fixed cost in the
// partition into chunks); cursors visit real pages only, and ps is the unit
// index of the current pair's first unit.
struct Cursor {
    int b, h, p, np, n;  // sequence, kv head, page, pages of b, context of b
    long long ps;
};

template <bool ROPE>
__device__ __forceinline__ void cursor_next(Cursor& c, const TmaArgs& a, int pad = 0) {
    if (++c.p == c.np) {
        c.ps += c.np + pad;
        c.p = 0;
        if (++c.h == a.Hkv) {
            c.h = 0;
            do {
                ++c.b;
                c.np = c.b < a.B ? seq_pages<ROPE>(a, c.b, &c.n) : 1;
            } while (c.np == 0);
        }
    }
}

// Sequences with no pages (empty or invalid context) get zero output rows;
// worker w covers sequences w, w + W, ...
template <int D, bool ROPE>
__device__ __forceinline__ void zero_empty_sequences(const TmaArgs& a, long long w, long long W, int lane) {
    for (long long b = w; b < a.B; b += W) {
        int n = 0;
        if (seq_pages<ROPE>(a, (int)b, &n) != 0) continue;
        if (lane == 0 && (ROPE || n != 0))
            report(a.status, ROPE ? COTTUS_STATUS_BAD_POSITION : COTTUS_STATUS_BAD_CONTEXT);
        const long long nel = (long long)a.H * D;
        for (long long i = lane * 8; i < nel; i += 32 * 8) {
            const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (a.out_f16) store8(reinterpret_cast<__half*>(a.out) + b * nel + i, z);
            else store8(reinterpret_cast<float*>(a.out) + b * nel + i, z);
        }
        if (a.lse)
            for (int i = lane; i < a.H; i += 32) a.lse[b * a.H + i] = -INFINITY;
    }
}

// (sequence, kv head, page) of unit u (< total units): a warp-wide prefix
// scan over the sequences' page counts, then division by the page count.
template <bool ROPE>
__device__ __forceinline__ Cursor locate_unit(const TmaArgs& a, long long u, int lane, int pad = 0) {
    constexpr unsigned FULL = 0xffffffffu;
    long long base = 0;
    int found_b = -1;
    long long found_excl = 0;
    for (int bb = 0; bb < a.B && found_b < 0; bb += 32) {
        const int b = bb + lane;
        const int pg = b < a.B ? seq_pages<ROPE>(a, b) : 0;
        const long long units = pg > 0 ? (long long)(pg + pad) * a.Hkv : 0;
        long long incl = units;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            long long t = __shfl_up_sync(FULL, incl, o);
            if (lane >= o) incl += t;
        }
        incl += base;
        const long long excl = incl - units;
        const unsigned hit = __ballot_sync(FULL, units > 0 && excl <= u && u < incl);
        if (hit) {
            const int src = __ffs(hit) - 1;
            found_b = bb + src;
            found_excl = __shfl_sync(FULL, excl, src);
        }
        base = __shfl_sync(FULL, incl, 31);
    }
    Cursor c;
    int n_b = 0;
    const int np = seq_pages<ROPE>(a, found_b, &n_b);
    const long long r = u - found_excl;
    c.b = found_b;
    c.np = np;
    c.n = n_b;
    c.h = (int)(r / (np + pad));
    c.p = (int)(r % (np + pad));
    c.ps = found_excl + (long long)c.h * (np + pad);
    if (c.p >= np) {  // a virtual unit: the next real one is page 0 of the next pair
        c.p = np - 1;
        cursor_next<ROPE>(c, a, pad);
    }
    return c;
}

// This worker's static share of the launch: total units U, chunk size, the
// unit range [u0, u1) of chunk w and the cursor at u0.  For batches up to kPlanRegs*32
// sequences the page counts are loaded once into registers and both the
// total and the start position come from them; larger batches fall back to
// repeated scans.  Also zero-fills the outputs of sequences without pages.
constexpr int kPlanRegs = 8;
struct WorkerPlan {
    long long U, chunk, u0, u1;
    Cursor cur;
};

// The sequence that holds unit u, from per-lane page counts: pg[i] of lane
// l is the page count of sequence 32 i + l.  Returns the sequence (-1 if no
// sequence holds u), the units before it, and the register slot and lane
// it came from (for reading other per-sequence values of the same snapshot).
struct CachedHit {
    int b, i, src;
    long long excl;
};
__device__ __forceinline__ CachedHit locate_cached(const int (&pg)[kPlanRegs], long long u, int Hkv, int lane,
                                                  int pad = 0) {
    constexpr unsigned FULL = 0xffffffffu;
    CachedHit h = {-1, 0, 0, 0};
    long long base = 0;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) {
        if (h.b >= 0) break;
        const long long units = pg[i] > 0 ? (long long)(pg[i] + pad) * Hkv : 0;
        long long incl = units;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long t = __shfl_up_sync(FULL, incl, o);
            if (lane >= o) incl += t;
        }
        incl += base;
        const long long excl = incl - units;
        const unsigned hit = __ballot_sync(FULL, units > 0 && excl <= u && u < incl);
        if (hit) {
            h.src = __ffs(hit) - 1;
            h.i = i;
            h.b = 32 * i + h.src;
            h.excl = __shfl_sync(FULL, excl, h.src);
        }
        base = __shfl_sync(FULL, incl, 31);
    }
    return h;
}

// Worker w of W (a warp, or a whole CTA whose warps share the chunk): its
// chunk is at least min_chunk units; zero_fill selects the one warp of the
// worker that writes the zero rows of empty sequences.
// Per-lane snapshot of the page counts and context lengths of sequences
// lane, lane + 32, ... (batches up to kPlanRegs * 32).
struct PlanRegs {
    int pg[kPlanRegs], cx[kPlanRegs];
};
template <bool ROPE, bool CG = false>
__device__ __forceinline__ PlanRegs load_plan_regs(const TmaArgs& a, int lane) {
    PlanRegs r;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) {
        const int b = lane + 32 * i;
        r.cx[i] = 0;
        r.pg[i] = b < a.B ? seq_pages<ROPE, CG>(a, b, &r.cx[i]) : 0;
    }
    return r;
}
// cursor_next over a snapshot (no memory reads): the same steps, with the
// page counts and lengths of later sequences taken from the lanes that hold
// them.  A plan made before the wait for the preceding kernel from one
// snapshot is then exactly the plan made after it when the lengths read
// again match the snapshot.
__device__ __forceinline__ void cursor_next_regs(Cursor& c, const PlanRegs& r, const TmaArgs& a, int lane, int pad) {
    constexpr unsigned FULL = 0xffffffffu;
    if (++c.p < c.np) return;
    c.ps += c.np + pad;
    c.p = 0;
    if (++c.h < a.Hkv) return;
    c.h = 0;
    int reg = -1, src = 0;  // the first sequence after c.b with pages: register slot and lane
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) {
        const unsigned hit = __ballot_sync(FULL, 32 * i + lane > c.b && r.pg[i] > 0);
        if (reg < 0 && hit) {
            reg = i;
            src = __ffs(hit) - 1;
        }
    }
    int np = 1, n = 0;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) {  // register arrays are indexed with constants only
        const int np_i = __shfl_sync(FULL, r.pg[i], src), n_i = __shfl_sync(FULL, r.cx[i], src);
        if (i == reg) {
            np = np_i;
            n = n_i;
        }
    }
    c.b = reg < 0 ? a.B : 32 * reg + src;
    c.np = np;
    c.n = n;
}

template <bool ROPE>
__device__ __forceinline__ bool same_plan_regs(const PlanRegs& x, const PlanRegs& y) {
    bool same = true;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) same = same && x.pg[i] == y.pg[i] && x.cx[i] == y.cx[i];
    return __all_sync(0xffffffffu, same);
}

// Worker w < kPlanRegs writes the zero rows of the empty sequences among
// 32w .. 32w + 31 (and reports the invalid lengths among them).
template <int D, bool ROPE>
__device__ __forceinline__ void zero_fill_from_regs(const TmaArgs& a, const PlanRegs& r, long long w, int lane) {
    constexpr unsigned FULL = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) {
        if (w != i) continue;
        const int b = lane + 32 * i;
        unsigned empty = __ballot_sync(FULL, b < a.B && r.pg[i] == 0);
        if (b < a.B && r.pg[i] == 0 && (ROPE || r.cx[i] != 0))
            report(a.status, ROPE ? COTTUS_STATUS_BAD_POSITION : COTTUS_STATUS_BAD_CONTEXT);
        const long long nel = (long long)a.H * D;
        while (empty) {
            const int src = __ffs(empty) - 1;
            empty &= empty - 1;
            const long long bb = 32 * i + src;
            const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (long long e = lane * 8; e < nel; e += 32 * 8) {
                if (a.out_f16) store8(reinterpret_cast<__half*>(a.out) + bb * nel + e, z);
                else store8(reinterpret_cast<float*>(a.out) + bb * nel + e, z);
            }
            if (a.lse)
                for (int e = lane; e < a.H; e += 32) a.lse[bb * a.H + e] = -INFINITY;
        }
    }
}

// The plan of worker w from a snapshot (no memory reads).
template <bool ROPE>
__device__ __forceinline__ WorkerPlan plan_from_regs(const TmaArgs& a, const PlanRegs& r, long long w,
                                                     long long W, int lane, long long min_chunk, int pad) {
    constexpr unsigned FULL = 0xffffffffu;
    WorkerPlan pl;
    long long total = 0;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) total += r.pg[i] > 0 ? r.pg[i] + pad : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(FULL, total, o);
    pl.U = total * a.Hkv;
    pl.chunk = max((pl.U + W - 1) / W, min_chunk);
    pl.u0 = min(w * pl.chunk, pl.U);
    pl.u1 = min(pl.u0 + pl.chunk, pl.U);
    if (pl.u0 >= pl.u1) return pl;
    // locate u0 from the cached page counts
    const CachedHit hit = locate_cached(r.pg, pl.u0, a.Hkv, lane, pad);
    int fnp = 0, fn = 0;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) {  // register arrays are indexed with constants only
        const int np_i = __shfl_sync(FULL, r.pg[i], hit.src), n_i = __shfl_sync(FULL, r.cx[i], hit.src);
        if (i == hit.i) {
            fnp = np_i;
            fn = n_i;
        }
    }
    const long long rr = pl.u0 - hit.excl;
    pl.cur.b = hit.b;
    pl.cur.np = fnp;
    pl.cur.n = fn;
    pl.cur.h = (int)(rr / (fnp + pad));
    pl.cur.p = (int)(rr % (fnp + pad));
    pl.cur.ps = hit.excl + (long long)pl.cur.h * (fnp + pad);
    if (pl.cur.p >= fnp) {  // a virtual unit: the next real one is page 0 of the next pair
        pl.cur.p = fnp - 1;
        cursor_next_regs(pl.cur, r, a, lane, pad);
    }
    return pl;
}

// With pad > 0 every pair is followed by pad virtual units (see Cursor);
// the cursor returned is at the first real unit at or after u0 (which may
// lie at or past u1 when the chunk holds only virtual units).
template <int D, bool ROPE>
__device__ __forceinline__ WorkerPlan plan_worker(const TmaArgs& a, long long w, long long W, int lane,
                                                  long long min_chunk = kMinChunk, bool zero_fill = true,
                                                  int pad = 0) {
    constexpr unsigned FULL = 0xffffffffu;
    WorkerPlan pl;
    if (a.B > 32 * kPlanRegs) {
        long long total_pages = 0;
        for (int b = lane; b < a.B; b += 32) {
            const int pg = seq_pages<ROPE>(a, b);
            total_pages += pg > 0 ? pg + pad : 0;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) total_pages += __shfl_xor_sync(FULL, total_pages, o);
        pl.U = total_pages * a.Hkv;
        pl.chunk = max((pl.U + W - 1) / W, min_chunk);
        pl.u0 = min(w * pl.chunk, pl.U);
        pl.u1 = min(pl.u0 + pl.chunk, pl.U);
        if (zero_fill) zero_empty_sequences<D, ROPE>(a, w, W, lane);
        if (pl.u0 < pl.u1) pl.cur = locate_unit<ROPE>(a, pl.u0, lane, pad);
        return pl;
    }
    const PlanRegs r = load_plan_regs<ROPE>(a, lane);
    if (zero_fill) zero_fill_from_regs<D, ROPE>(a, r, w, lane);
    return plan_from_regs<ROPE>(a, r, w, W, lane, min_chunk, pad);
}

// Pages of a worker's static chunk warmed in L2 before the wait for the
// preceding kernel.
constexpr int kWarmPages = 2;

// L2 prefetch (TMA, nothing written) of units u0 + first and
// u0 + first + stride of this worker's chunk (the first pages the warp will
// load), issued before griddepcontrol.wait so that a launch made resident
// during the preceding kernel's tail streams its first pages meanwhile.  The
// chunk is located as plan_worker locates it, from one snapshot of the
// lengths that the preceding kernel may still be writing: a stale snapshot
// only warms the wrong lines (every index is checked against the snapshot
// and the table's bounds, block ids against the pool, the tensor map bounds
// the box, and the real loads come after the wait; L2 is the point of
// coherence, so nothing stale can be read from it).  Batches beyond
// kPlanRegs * 32 sequences are not warmed.
template <bool ROPE>
__device__ __forceinline__ void warm_first_pages(const TmaArgs& a, const CUtensorMap* map, long long w,
                                                 long long W, int lane, int boxes, int box_elems,
                                                 long long min_chunk = kMinChunk, int first = 0, int stride = 1,
                                                 int pad = 0) {
    constexpr unsigned FULL = 0xffffffffu;
    if (kWarmPages == 0 || a.B > 32 * kPlanRegs) return;
    int pg[kPlanRegs];
    long long total = 0;
#pragma unroll
    for (int i = 0; i < kPlanRegs; ++i) {
        const int b = lane + 32 * i;
        pg[i] = b < a.B ? seq_pages<ROPE, true>(a, b) : 0;
        total += pg[i] > 0 ? pg[i] + pad : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(FULL, total, o);
    const long long U = total * a.Hkv;
    const long long chunk = max((U + W - 1) / W, min_chunk);
    const long long u0 = w * chunk, u1 = min(u0 + chunk, U);
#pragma unroll 1
    for (int i = 0; i < kWarmPages; ++i) {
        const long long u = u0 + first + (long long)i * stride;
        if (u >= u1) return;
        const CachedHit hit = locate_cached(pg, u, a.Hkv, lane, pad);
        int np = 0;
#pragma unroll
        for (int j = 0; j < kPlanRegs; ++j) {
            const int np_j = __shfl_sync(FULL, pg[j], hit.src);
            if (j == hit.i) np = np_j;
        }
        if (lane != 0 || hit.b < 0 || hit.b >= a.B || np <= 0) continue;
        const long long r = u - hit.excl;
        const int h = (int)(r / (np + pad)), p = (int)(r % (np + pad));
        if (h >= a.Hkv || p >= np || p >= a.maxb) continue;  // past the table, or a virtual unit
        const int blk = __ldcg(a.bt + (long long)hit.b * a.maxb + p);
        if (blk >= 0 && (long long)blk < a.num_blocks)
            for (int q = 0; q < boxes; ++q) tma_prefetch_l2_3d(map, q * box_elems, h, (blk * a.L + a.layer) * (2 * kBS));
    }
}

// Called by a worker after it stored its partial of a cut (sequence, kv
// head) pair whose units are [ps, ps + np).  Worker wk owns units
// [wk*chunk, (wk+1)*chunk), so the pair's partials belong to workers
// ps/chunk .. (ps+np-1)/chunk, every one of them non-empty.  Arrives on the
// pair's counter, tagged with the launch epoch so that a count left by an
// aborted launch, or bytes of another layout that used the same workspace,
// read as zero (a completed pair leaves its counter at zero): a compare-and-swap from `hint`, the counter value read a
// page earlier, which is right on the first try unless another part arrived
// in between.  The last arriving worker merges all partials.  Lane items
// are (head, 8-dim chunk); each lane reads the parts PB at a time with all
// their loads in flight together and folds them into a running (max, sum,
// output), so PB parts cost one round trip to L2.
template <int D, int G>
__device__ __forceinline__ void merge_if_last(const TmaArgs& a, int b, int h, long long ps, int np, long long chunk,
                                              int lane, unsigned long long hint) {
    constexpr unsigned FULL = 0xffffffffu;
    constexpr int CPR = D / 8;     // 8-dim chunks per head row
    constexpr int ITEMS = G * CPR;  // (head, chunk) items
    constexpr int PB = 4;           // parts loaded together
    const long long w0 = ps / chunk, w1 = (ps + np - 1) / chunk;
    const int nparts = (int)(w1 - w0 + 1);
    const long long slot0 = w0 * chunk >= ps ? 2 * w0 : 2 * w0 + 1;  // later parts start inside the pair
    unsigned long long* ctr = a.counters + 1 + (long long)b * a.Hkv + h;
    fence_acq_rel_gpu();  // this lane's partial stores are visible device-wide before the arrival
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        unsigned long long old = hint;
        while (true) {  // every failed attempt means another part arrived: at most nparts rounds
            const unsigned long long nv =
                (unsigned)(old >> 32) == a.epoch ? old + 1 : (((unsigned long long)a.epoch << 32) | 1ull);
            // the last arrival leaves the counter at zero, so that a replay of
            // this launch (a CUDA graph: same tag) counts from zero again
            const bool fin = (int)(nv & 0xffffffffull) == nparts;
            const unsigned long long prev = atomicCAS(ctr, old, fin ? 0ull : nv);
            if (prev == old) {
                last = fin;
                break;
            }
            old = prev;
        }
        if (last) fence_acq_rel_gpu();
    }
    last = __shfl_sync(FULL, last, 0);
    if (!last) return;
    auto slot_of = [&](int j) -> long long { return j == 0 ? slot0 : 2 * (w0 + j); };
#pragma unroll 1
    for (int it = lane; it < ITEMS; it += 32) {
        const int g = it / CPR, c = it % CPR;
        float M = -INFINITY, L = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int j0 = 0; j0 < nparts; j0 += PB) {
            float2 ml[PB];
            float4 x0[PB], x1[PB];
#pragma unroll
            for (int q = 0; q < PB; ++q) {
                ml[q] = make_float2(-INFINITY, 0.f);
                x0[q] = x1[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (j0 + q < nparts) {
                    const long long sl = slot_of(j0 + q);
                    ml[q] = __ldcg(reinterpret_cast<const float2*>(a.ws_ml + (sl * G + g) * 2));
                    const float4* src = reinterpret_cast<const float4*>(a.ws_o + (sl * G + g) * D + c * 8);
                    x0[q] = __ldcg(src);
                    x1[q] = __ldcg(src + 1);
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
                const float xv[8] = {x0[q].x, x0[q].y, x0[q].z, x0[q].w, x1[q].x, x1[q].y, x1[q].z, x1[q].w};
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = acc[e] * sa + xv[e] * sb;
            }
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= inv;
        const long long head = (long long)b * a.H + (long long)h * G + g;
        if (a.out_f16) store8(reinterpret_cast<__half*>(a.out) + head * D + c * 8, acc);
        else store8(reinterpret_cast<float*>(a.out) + head * D + c * 8, acc);
        if (a.lse && c == 0) a.lse[head] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
    }
}

template <int D, int G, int RING, bool ROPE>
__global__ void __launch_bounds__(kNW * 32)
    decode_tma_kernel(const __grid_constant__ CUtensorMap kv_map, const TmaArgs a) {
    using C = TmaCfg<D, G>;
    constexpr int LW = C::LW, RPS = C::RPS, STEPS = C::STEPS, CH = C::CH, N = C::N, NV = C::NV;
    constexpr int CL = C::CL, DUP = C::DUP;
    constexpr unsigned FULL = 0xffffffffu;

    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LW, lq = lane % LW;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint8_t* slots = smem + (size_t)warp * RING * C::SLOT_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kNW * RING * C::SLOT_BYTES) + warp * RING;
    float* p_s = reinterpret_cast<float*>(smem + (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 8) +
                 warp * CH * G;
    float* hs = reinterpret_cast<float*>(smem + (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 8 +
                                         (size_t)kNW * CH * G * 4) +
                warp * 2 * G;
    int* slot_blk = reinterpret_cast<int*>(smem + (size_t)kNW * RING * C::SLOT_BYTES + (size_t)kNW * RING * 8 +
                                           (size_t)kNW * CH * G * 4 + (size_t)kNW * 2 * G * 4) +
                    warp * RING;

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

    // ---- work: static chunk w, then chunks from the queue ----------------
    const long long W = (long long)gridDim.x * kNW;
    const long long w = (long long)blockIdx.x * kNW + warp;
    warm_first_pages<ROPE>(a, &kv_map, w, W, lane, 1, 0);
    grid_dependency_wait();
    grid_dependents_launch();
    const WorkerPlan pl = plan_worker<D, ROPE>(a, w, W, lane);
    const long long U = pl.U, chunk = pl.chunk;
    const long long NC = (U + chunk - 1) / chunk;

    float2 q2[G][4];
    float2 o2[G][4];
    float m_run = -INFINITY, l_own = 0.f;
    const int i0 = (lq * N) / LW;   // first partial index this lane holds after the reduction
    const int gl = i0 / STEPS;      // the head this lane scores

    long long cid = w < NC ? w : NC;
    Cursor cur = pl.cur;
    int kg = 0;  // units consumed by this warp so far (ring slot / phase counter)

    while (cid < NC) {  // one static chunk per warp
        const long long u0 = cid * chunk, u1 = min(u0 + chunk, U);
        const int nu = (int)(u1 - u0);

        // ---- TMA issue: lane 0 owns the issue cursor; the block id of the next
        // unit to issue is loaded one page ahead so its latency hides behind math.
        Cursor ic = cur;
        int blk_next = lane == 0 ? a.bt[(long long)ic.b * a.maxb + ic.p] : 0;
        auto issue = [&](int k) {
            if (lane == 0) {
                const int slot = (kg + k) % RING;
                const int blk = blk_next;
                slot_blk[slot] = blk;
                if (blk < 0 || (long long)blk >= a.num_blocks) {
                    mbar_arrive(&bars[slot]);  // nothing to load; the consumer masks the page
                } else {
                    mbar_arrive_expect_tx(&bars[slot], C::SLOT_BYTES);
                    tma_load_3d(slots + (size_t)slot * C::SLOT_BYTES, &kv_map, &bars[slot], 0, ic.h,
                                (blk * a.L + a.layer) * (2 * kBS));
                }
                cursor_next<ROPE>(ic, a);
                if (k + 1 < nu) blk_next = a.bt[(long long)ic.b * a.maxb + ic.p];
            }
        };
        const int prime = nu < RING ? nu : RING;
        for (int k = 0; k < prime; ++k) issue(k);

        bool seg_open = false;
        int seg_start_p = 0;
        bool seg_first = true;
        unsigned long long ctr_hint = 0;  // arrival counter of the open segment's pair, read a page early
        for (int k = 0; k < nu; ++k) {
            const int slot = (kg + k) % RING;
            const int ctx_b = cur.n;
            if (!seg_open) {
                // ---- segment start: load (and rotate) the group's query rows ----
                seg_open = true;
                seg_first = (k == 0);
                seg_start_p = cur.p;
                ctr_hint = 0;
                m_run = -INFINITY;
                l_own = 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const long long row = ((long long)cur.b * a.H + (long long)cur.h * G + g) * D + lq * 8;
                    float x[8];
                    if (a.q_f16) load8(reinterpret_cast<const __half*>(a.q) + row, x);
                    else load8(reinterpret_cast<const float*>(a.q) + row, x);
                    if (ROPE) {
                        const float4* cs = reinterpret_cast<const float4*>(
                            a.cos_sin + ((long long)(ctx_b - 1) * (D / 2) + lq * 4) * 2);
#pragma unroll
                        for (int pr = 0; pr < 2; ++pr) {
                            const float4 c4 = __ldg(cs + pr);
                            rope_pair(x[4 * pr], x[4 * pr + 1], c4.x, c4.y, x[4 * pr], x[4 * pr + 1]);
                            rope_pair(x[4 * pr + 2], x[4 * pr + 3], c4.z, c4.w, x[4 * pr + 2], x[4 * pr + 3]);
                        }
                        if (a.q_out && cur.p == 0 && grp == 0) {
                            if (a.q_f16) store8(reinterpret_cast<__half*>(a.q_out) + row, x);
                            else store8(reinterpret_cast<float*>(a.q_out) + row, x);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        q2[g][j] = make_float2(x[2 * j] * a.qscale, x[2 * j + 1] * a.qscale);
                        o2[g][j] = make_float2(0.f, 0.f);
                    }
                }
            }

            const bool landed = __all_sync(FULL, mbar_wait_bounded(&bars[slot], ((kg + k) / RING) & 1));
            if (!landed) {
                if (lane == 0) report(a.status, COTTUS_STATUS_TIMEOUT);
                // let the loads still in flight land (bounded) before the warp leaves
                for (int kk = k + 1; kk < k + RING && kk < nu; ++kk)
                    (void)__all_sync(FULL, mbar_wait_bounded(&bars[(kg + kk) % RING], ((kg + kk) / RING) & 1));
                return;
            }
            const int blk = slot_blk[slot];
            const bool blk_ok = blk >= 0 && (long long)blk < a.num_blocks;
            if (!blk_ok && lane == 0) report(a.status, COTTUS_STATUS_BAD_BLOCK_ID);
            int n_valid = blk_ok ? ctx_b - cur.p * kBS : 0;
            n_valid = n_valid > kBS ? kBS : n_valid;
            const uint16_t* kt = reinterpret_cast<const uint16_t*>(slots + (size_t)slot * C::SLOT_BYTES);
            const uint16_t* vt = kt + kBS * D;

            if (ROPE && blk_ok && cur.p == cur.np - 1 && grp == 0) {
                // ---- the new token: rotate k, encode k and v, append -------------
                const int t_new = (ctx_b - 1) % kBS;
                const long long src = ((long long)cur.b * a.Hkv + cur.h) * D + lq * 8;
                float kx[8], vx[8];
                if (a.q_f16) {
                    load8(reinterpret_cast<const __half*>(a.k_new) + src, kx);
                    load8(reinterpret_cast<const __half*>(a.v_new) + src, vx);
                } else {
                    load8(reinterpret_cast<const float*>(a.k_new) + src, kx);
                    load8(reinterpret_cast<const float*>(a.v_new) + src, vx);
                }
                const float4* cs =
                    reinterpret_cast<const float4*>(a.cos_sin + ((long long)(ctx_b - 1) * (D / 2) + lq * 4) * 2);
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
                *reinterpret_cast<uint4*>(const_cast<uint16_t*>(kt) + t_new * D + lq * 8) = k4;
                *reinterpret_cast<uint4*>(const_cast<uint16_t*>(vt) + t_new * D + lq * 8) = v4;
                const long long row0 = ((long long)blk * a.L + a.layer) * (2 * kBS);
                const long long koff = ((row0 + t_new) * a.Hkv + cur.h) * D + lq * 8;
                const long long voff = ((row0 + kBS + t_new) * a.Hkv + cur.h) * D + lq * 8;
                *reinterpret_cast<uint4*>(a.kv + koff) = k4;
                *reinterpret_cast<uint4*>(a.kv + voff) = v4;
            }
            if (ROPE) __syncwarp();

            // ---- the page, CH tokens at a time ------------------------------------
#pragma unroll
            for (int c = 0; c < C::NCH; ++c) {
                const int tb = c * CH;
                float part[N];
#pragma unroll
                for (int s = 0; s < STEPS; ++s) {
                    const int row = tb + s * RPS + grp;
                    const uint4 raw = *reinterpret_cast<const uint4*>(kt + row * D + lq * 8);
                    const float2 k0 = h2_to_f2(raw.x), k1 = h2_to_f2(raw.y), k2 = h2_to_f2(raw.z),
                                 k3 = h2_to_f2(raw.w);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        float2 acc = fmul2(q2[g][0], k0);
                        acc = ffma2(q2[g][1], k1, acc);
                        acc = ffma2(q2[g][2], k2, acc);
                        acc = ffma2(q2[g][3], k3, acc);
                        part[g * STEPS + s] = acc.x + acc.y;
                    }
                }
                TransposeReduce<N, LW / 2>::run(part, lq);

                // scores of this lane (head gl), masked past the context
                float sc[NV];
                bool ok[NV];
                float cmax = -INFINITY;
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                    const int s = (i0 + j) % STEPS;
                    const int t = tb + s * RPS + grp;
                    ok[j] = t < n_valid;
                    sc[j] = ok[j] ? part[j] : -INFINITY;
                    cmax = fmaxf(cmax, sc[j]);
                }
#pragma unroll
                for (int o = 1; o < CL; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(FULL, cmax, o));
#pragma unroll
                for (int o = LW; o < 32; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(FULL, cmax, o));

                const bool upd = cmax > m_run + 8.0f;
                if (__any_sync(FULL, upd)) {
                    const float m_new = upd ? cmax : m_run;
                    const float alpha = upd ? exp2f(m_run - m_new) : 1.0f;
                    l_own *= alpha;
                    m_run = m_new;
                    if (grp == 0 && (lq % CL) == 0) hs[gl] = alpha;
                    __syncwarp();
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float al = hs[g];
                        const float2 al2 = make_float2(al, al);
#pragma unroll
                        for (int j = 0; j < 4; ++j) o2[g][j] = fmul2(o2[g][j], al2);
                    }
                    __syncwarp();
                }
                float psum = 0.f;
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                    const float pj = ok[j] ? exp2f(sc[j] - m_run) : 0.f;
                    psum += pj;
                    const int s = (i0 + j) % STEPS;
                    p_s[(grp * STEPS + s) * G + gl] = pj;
                }
                if (DUP == 1 || (lq % DUP) == 0) l_own += psum;
                __syncwarp();

#pragma unroll
                for (int s = 0; s < STEPS; ++s) {
                    const int row = tb + s * RPS + grp;
                    uint4 raw = *reinterpret_cast<const uint4*>(vt + row * D + lq * 8);
                    if (row >= n_valid) raw = make_uint4(0u, 0u, 0u, 0u);
                    const float2 v0 = h2_to_f2(raw.x), v1 = h2_to_f2(raw.y), v2 = h2_to_f2(raw.z),
                                 v3 = h2_to_f2(raw.w);
                    float pv[G];
#pragma unroll
                    for (int g = 0; g < G; ++g) pv[g] = p_s[(grp * STEPS + s) * G + g];
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float2 p2 = make_float2(pv[g], pv[g]);
                        o2[g][0] = ffma2(p2, v0, o2[g][0]);
                        o2[g][1] = ffma2(p2, v1, o2[g][1]);
                        o2[g][2] = ffma2(p2, v2, o2[g][2]);
                        o2[g][3] = ffma2(p2, v3, o2[g][3]);
                    }
                }
                __syncwarp();
            }

            // ---- refill this slot --------------------------------------------
            if (k + RING < nu) {
                fence_proxy_async_smem();
                issue(k + RING);
            }

            // the next page ends a cut segment of this pair: read the pair's
            // arrival counter now, so the arrival's compare-and-swap finds it
            if (lane == 0 && k + 1 < nu && cur.p + 1 < cur.np && (cur.p + 2 == cur.np || k + 2 == nu) &&
                !(seg_start_p == 0 && cur.p + 2 == cur.np))
                ctr_hint = ld_relaxed_u64(a.counters + 1 + (long long)cur.b * a.Hkv + cur.h);

            // ---- segment end -------------------------------------------------
            const bool seg_end = (cur.p == cur.np - 1) || (k == nu - 1);
            if (seg_end) {
#pragma unroll
                for (int o = LW; o < 32; o <<= 1) {
#pragma unroll
                    for (int g = 0; g < G; ++g) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            o2[g][j].x += __shfl_xor_sync(FULL, o2[g][j].x, o);
                            o2[g][j].y += __shfl_xor_sync(FULL, o2[g][j].y, o);
                        }
                    }
                }
                float lt = l_own;
#pragma unroll
                for (int o = 1; o < CL; o <<= 1) lt += __shfl_xor_sync(FULL, lt, o);
#pragma unroll
                for (int o = LW; o < 32; o <<= 1) lt += __shfl_xor_sync(FULL, lt, o);
                if (grp == 0 && (lq % CL) == 0) {
                    hs[2 * gl] = m_run;
                    hs[2 * gl + 1] = lt;
                }
                __syncwarp();
                const bool whole = seg_start_p == 0 && cur.p == cur.np - 1;
                if (grp == 0) {
                    const long long slot_id = seg_first ? 2 * cid : 2 * cid + 1;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float mg = hs[2 * g], lg = hs[2 * g + 1];
                        const long long head = (long long)cur.b * a.H + (long long)cur.h * G + g;
                        float x[8];
                        if (whole) {
                            const float inv = lg > 0.f ? 1.0f / lg : 0.f;
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                x[2 * j] = o2[g][j].x * inv;
                                x[2 * j + 1] = o2[g][j].y * inv;
                            }
                            if (a.out_f16) store8(reinterpret_cast<__half*>(a.out) + head * D + lq * 8, x);
                            else store8(reinterpret_cast<float*>(a.out) + head * D + lq * 8, x);
                            if (a.lse && lq == 0) a.lse[head] = lg > 0.f ? (mg + log2f(lg)) * kLn2 : -INFINITY;
                        } else {
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                x[2 * j] = o2[g][j].x;
                                x[2 * j + 1] = o2[g][j].y;
                            }
                            store8(a.ws_o + (slot_id * G + g) * D + lq * 8, x);
                            if (lq == 0) {
                                a.ws_ml[(slot_id * G + g) * 2] = mg;
                                a.ws_ml[(slot_id * G + g) * 2 + 1] = lg;
                            }
                        }
                    }
                }
                if (!whole) merge_if_last<D, G>(a, cur.b, cur.h, u0 + k - cur.p, cur.np, chunk, lane, ctr_hint);
                __syncwarp();
                seg_open = false;
            }
            if (k + 1 < nu) cursor_next<ROPE>(cur, a);
        }
        kg += nu;
        cid = NC;
    }
    signal_done(a, lane, &cta_done);
}

// ---------------------------------------------------------------------------
// Host side of one head_dim: tensor map, occupancy cache, launch.
// ---------------------------------------------------------------------------
CUtensorMap make_kv_tensor_map(const DecodeDesc& d, bool swizzle128, cudaError_t* err);
int device_sm_count(int device);
unsigned next_epoch();

// Upper bound on the number of chunks of a launch with W workers.
inline long long max_chunks(long long W) { return W + 1; }

// Launch with programmatic stream serialization: the kernel may begin its
// prologue while the previous kernel of the stream drains; it waits
// (griddepcontrol.wait) before reading any global memory.
template <typename Kern>
inline cudaError_t launch_pdl(Kern kern, int grid, size_t smem, cudaStream_t st, const CUtensorMap& map,
                              const TmaArgs& a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kNW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, map, a);
}

// Kernel arguments of one launch; the workspace holds a reserved word and
// the pair counters, then 2 partial slots per chunk of G x D outputs and
// G x (m, l).
inline TmaArgs make_tma_args(const DecodeDesc& d, long long W, int G, int D) {
    TmaArgs a;
    a.out = d.out;
    a.q = d.q;
    a.bt = d.block_table;
    a.ctx = d.context_lens;
    a.positions = d.positions;
    a.lse = d.lse;
    const size_t ctr_bytes = workspace_zero_prefix_bytes(d.batch, d.num_kv_heads);
    a.counters = reinterpret_cast<unsigned long long*>(d.workspace);
    a.ws_o = reinterpret_cast<float*>(static_cast<uint8_t*>(d.workspace) + ctr_bytes);
    a.ws_ml = a.ws_o + (size_t)2 * max_chunks(W) * G * D;
    a.status = d.status;
    a.epoch = next_epoch();
    a.sig = d.signal;
    a.pm = d.merge;
    a.k_new = d.k_new;
    a.v_new = d.v_new;
    a.cos_sin = d.cos_sin;
    a.q_out = d.q_out;
    a.kv = d.kv_mut;
    a.num_blocks = d.num_blocks;
    a.B = d.batch;
    a.H = d.num_heads;
    a.Hkv = d.num_kv_heads;
    a.L = d.num_layers;
    a.layer = d.layer;
    a.maxb = d.max_blocks;
    a.max_pos = d.max_position;
    a.q_f16 = d.q_f16;
    a.out_f16 = d.out_f16;
    a.qscale = d.scale * kLog2e;
    return a;
}

template <int D, int G, int RING, bool ROPE>
struct TmaLauncher {
    static int blocks_per_sm(int device) {
        static int cache[64] = {0};
        if (device < 0 || device >= 64) return 1;
        if (cache[device] == 0) {
            auto kern = decode_tma_kernel<D, G, RING, ROPE>;
            const size_t smem = tma_smem_bytes<RING, D, G>();
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
        const int grid = (int)(W / kNW);
        cudaError_t err = cudaSuccess;
        const CUtensorMap map = make_kv_tensor_map(d, false, &err);
        if (err != cudaSuccess) return err;
        TmaArgs a = make_tma_args(d, W, G, D);
        return launch_pdl(decode_tma_kernel<D, G, RING, ROPE>, grid, tma_smem_bytes<RING, D, G>(), st, map, a);
    }
};

template <int D, int RING>
cudaError_t dispatch_tma(const DecodeDesc& d, cudaStream_t st) {
    const int G = d.num_heads / d.num_kv_heads;
    if (d.rope) {
        switch (G) {
            case 1: return TmaLauncher<D, 1, RING, true>::launch(d, st);
            case 2: return TmaLauncher<D, 2, RING, true>::launch(d, st);
            case 4: return TmaLauncher<D, 4, RING, true>::launch(d, st);
            case 8: return TmaLauncher<D, 8, RING, true>::launch(d, st);
        }
    } else {
        switch (G) {
            case 1: return TmaLauncher<D, 1, RING, false>::launch(d, st);
            case 2: return TmaLauncher<D, 2, RING, false>::launch(d, st);
            case 4: return TmaLauncher<D, 4, RING, false>::launch(d, st);
            case 8: return TmaLauncher<D, 8, RING, false>::launch(d, st);
        }
    }
    return cudaErrorInvalidValue;
}

template <int D, int RING>
size_t dispatch_workers(const DecodeDesc& d) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int G = d.num_heads / d.num_kv_heads;
    if (d.rope) {
        switch (G) {
            case 1: return TmaLauncher<D, 1, RING, true>::workers(dev);
            case 2: return TmaLauncher<D, 2, RING, true>::workers(dev);
            case 4: return TmaLauncher<D, 4, RING, true>::workers(dev);
            case 8: return TmaLauncher<D, 8, RING, true>::workers(dev);
        }
    } else {
        switch (G) {
            case 1: return TmaLauncher<D, 1, RING, false>::workers(dev);
            case 2: return TmaLauncher<D, 2, RING, false>::workers(dev);
            case 4: return TmaLauncher<D, 4, RING, false>::workers(dev);
            case 8: return TmaLauncher<D, 8, RING, false>::workers(dev);
        }
    }
    return 0;
}

}  // namespace cb200
