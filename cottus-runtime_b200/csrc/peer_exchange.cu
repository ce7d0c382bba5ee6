// Split-context decode across the GPUs of one node without a collective
// library call: the exchange of partial results goes through peer memory
// over NVLink.
//
// Each rank owns one exchange buffer (cudaMalloc'd once, mapped by every
// other rank through CUDA IPC): a flag per rank, the decode's CTA counter,
// a "broken" word, and two slots of partials ([batch][heads][head_dim]
// normalised fp32 outputs and [batch][heads] natural-log LSEs).  A step on
// every rank:
//   1. the decode kernel writes this rank's partials into its own slot
//      (epoch & 1) and, when its last CTA has finished, stores `epoch` into
//      flag[rank] of every rank's buffer (decode_tma.cuh: signal_done);
//   2. every rank waits (bounded) until every rank's flag in its own buffer
//      has reached `epoch`, then reads every rank's slot directly (peer
//      loads) and merges them, the arithmetic of cottus_lse_combine: on the
//      tensor-core path in the decode kernel itself, its CTAs taking the
//      rows in turn (decode_mma.cuh), otherwise in a combine kernel.
// Two slots suffice: a rank overwrites slot s at step n+2 only after its
// merge of step n+1, which waited for every rank's step-n+1 decode, which
// each rank started after its own merge of step n had read slot s.  The
// same chain bounds how far a peer can run ahead: when this rank's merge of
// step n polls, a peer's flag reads n or n+1 (the peer may already have
// finished its decode of step n+1), never more, so the wait accepts any
// flag at or past `epoch` (serial-number comparison, wrap-safe).
//
// Failure handling: a merge whose wait runs out reports
// COTTUS_STATUS_TIMEOUT, writes nothing, and sets the broken word in its own
// buffer and in every peer's; from then on every merge of every rank of
// this exchange reports COTTUS_STATUS_TIMEOUT at once without waiting or
// writing, until the ranks destroy the exchange and create a new one (the
// epochs of the ranks may disagree after a missed step, so no later step of
// the old exchange can be trusted).  The combine kernel also returns the
// decode's CTA counter to zero, which a decode warp that gave up on a wait
// leaves behind (the decode kernel that merges itself resets it when it
// completes normally; after a wait that gave up, the exchange is broken).
// Plain loads and stores only (no bulk or tensor copies of peer memory).
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "cottus_b200.h"
#include "internal.h"

namespace cb200 {
int set_error(int code, const std::string& msg);

namespace {

constexpr size_t kAlign = 256;
constexpr long long kPeerWaitCycles = 2000000000LL;  // default wait limit: about a second at 2 GHz
}  // namespace
}  // namespace cb200

// The merge of a step runs in the decode kernel itself where the shape takes
// the tensor-core kernel (one launch per step); 0 keeps the decode + combine
// kernel pair for every shape.
#ifndef CB200_SPLIT_MERGE_IN_DECODE
#define CB200_SPLIT_MERGE_IN_DECODE 1
#endif

namespace cb200 {
namespace {

size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

struct Layout {
    size_t flags, done, broken, slot0, slot_bytes, part_bytes, total;
};

Layout layout_of(int world, long long heads, int head_dim) {
    Layout l;
    l.flags = 0;
    l.done = align_up(sizeof(uint32_t) * kMaxPeers);
    l.broken = l.done + 64;
    l.slot0 = l.done + kAlign;
    l.part_bytes = align_up((size_t)heads * head_dim * sizeof(float));
    l.slot_bytes = l.part_bytes + align_up((size_t)heads * sizeof(float));
    l.total = l.slot0 + 2 * l.slot_bytes;
    (void)world;
    return l;
}

static_assert(kMaxPeers == kMergeParts, "one merge part per rank");
struct PeerSlots {
    const float* part[kMaxPeers];
    const float* lse[kMaxPeers];
    uint32_t* broken[kMaxPeers];  // every rank's broken word (this rank's own included)
};

// Control words of this rank's buffer for one combine launch.
struct CombineCtl {
    const uint32_t* flags;  // flag per rank
    uint32_t* done;         // the decode's CTA counter
    uint32_t* broken;       // this rank's broken word
    uint32_t epoch;
    long long wait_cycles;
};

// One warp per (sequence, head): merge_head_parts over parts 0..world-1,
// the arithmetic of lse_combine_kernel (same bits as the NCCL path).
__global__ void peer_combine_kernel(const __grid_constant__ PeerSlots src, int world, const CombineCtl ctl,
                                    void* out, int out_f16, float* lse_out, long long heads, int D,
                                    uint32_t* status) {
    __shared__ int ready;
    grid_dependency_wait();    // this rank's decode has completed (its own flag is then set as well)
    grid_dependents_launch();  // the next decode may start its prologue while this merge runs
    if (threadIdx.x == 0) {
        // the decode has completed: its CTA counter is free to reset (a warp
        // that gave up on a wait leaves a count behind)
        if (blockIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(ctl.done) = 0u;
        bool ok = ld_acquire_sys(ctl.broken) == 0u;
        const long long t0 = clock64();
        for (int r = 0; r < world && ok; ++r)
            while ((int32_t)(ld_acquire_sys(ctl.flags + r) - ctl.epoch) < 0)
                if (clock64() - t0 > ctl.wait_cycles) {
                    ok = false;
                    break;
                }
        ready = ok;
        if (!ok && blockIdx.x == 0) {
            report(status, COTTUS_STATUS_TIMEOUT);
            // every later combine of every rank refuses at once
            for (int r = 0; r < world; ++r)
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(src.broken[r]), "r"(1u) : "memory");
        }
    }
    __syncthreads();
    if (!ready) return;
    const long long hw = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (hw >= heads) return;
    merge_head_parts(src.lse, src.part, world, hw, D, lane, out, out_f16, lse_out);
}

__global__ void peer_signal_kernel(PeerSignal sig) {
    __threadfence_system();
    for (int r = 0; r < sig.world; ++r)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(sig.flags[r] + sig.rank), "r"(sig.epoch) : "memory");
}

}  // namespace

cudaError_t launch_peer_signal(const PeerSignal& sig, cudaStream_t st) {
    return launch_kernel(peer_signal_kernel, dim3(1), dim3(1), 0, st, sig);
}
}  // namespace cb200

struct cottus_peer_exchange {
    int world = 0, rank = 0, batch = 0, heads = 0, head_dim = 0;
    cb200::Layout lay{};
    uint8_t* local = nullptr;                 // this rank's buffer
    uint8_t* base[cb200::kMaxPeers] = {};     // every rank's buffer as seen from this GPU
    bool absent[cb200::kMaxPeers] = {};       // stand-in buffer of a rank that takes no part (local allocation)
    bool opened = false;
    uint32_t epoch = 0;
    long long wait_cycles = cb200::kPeerWaitCycles;
};

namespace {

int fail(int code, const std::string& msg) { return cb200::set_error(code, msg); }
int cuda_fail(cudaError_t e) { return fail(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e)); }

}  // namespace

extern "C" {

int cottus_peer_exchange_create(int32_t world, int32_t rank, int32_t batch, int32_t num_heads, int32_t head_dim,
                                cottus_peer_exchange** out, void* ipc_handle) {
    if (!out || !ipc_handle) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (world < 1 || world > cb200::kMaxPeers || rank < 0 || rank >= world)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "world must be in [1, 8] and rank in [0, world)");
    if (batch <= 0 || num_heads <= 0 || head_dim <= 0 || head_dim > 512)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "batch, num_heads and head_dim must be positive (head_dim <= 512)");
    auto* ex = new cottus_peer_exchange;
    ex->world = world;
    ex->rank = rank;
    ex->batch = batch;
    ex->heads = num_heads;
    ex->head_dim = head_dim;
    ex->lay = cb200::layout_of(world, (long long)batch * num_heads, head_dim);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, ex->lay.total);
    if (e == cudaSuccess) e = cudaMemset(p, 0, ex->lay.total);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        delete ex;
        return cuda_fail(e);
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == COTTUS_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(ipc_handle, &h, sizeof h);
    ex->local = static_cast<uint8_t*>(p);
    ex->base[rank] = ex->local;
    *out = ex;
    return COTTUS_OK;
}

int cottus_peer_exchange_open(cottus_peer_exchange* ex, const void* handles) {
    if (!ex || !handles) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL argument");
    if (ex->opened) return fail(COTTUS_ERR_INVALID_ARGUMENT, "exchange already opened");
    const auto* hs = static_cast<const uint8_t*>(handles);
    auto undo = [&](int upto) {
        for (int q = 0; q < upto; ++q) {
            if (q == ex->rank || !ex->base[q]) continue;
            if (ex->absent[q]) cudaFree(ex->base[q]);
            else cudaIpcCloseMemHandle(ex->base[q]);
            ex->base[q] = nullptr;
            ex->absent[q] = false;
        }
    };
    for (int r = 0; r < ex->world; ++r) {
        if (r == ex->rank) continue;
        const uint8_t* hr = hs + (size_t)r * COTTUS_IPC_HANDLE_BYTES;
        bool zero = true;
        for (int i = 0; i < COTTUS_IPC_HANDLE_BYTES; ++i) zero = zero && hr[i] == 0;
        void* p = nullptr;
        cudaError_t e;
        if (zero) {
            // a rank that takes no part: a local stand-in whose flag nothing raises
            e = cudaMalloc(&p, ex->lay.total);
            if (e == cudaSuccess) e = cudaMemset(p, 0, ex->lay.total);
            if (e != cudaSuccess && p) {
                cudaFree(p);
                p = nullptr;
            }
        } else {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, hr, sizeof h);
            e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        }
        if (e != cudaSuccess) {
            undo(r);
            return cuda_fail(e);
        }
        ex->base[r] = static_cast<uint8_t*>(p);
        ex->absent[r] = zero;
    }
    ex->opened = true;
    return COTTUS_OK;
}

int cottus_peer_exchange_set_wait_cycles(cottus_peer_exchange* ex, int64_t cycles) {
    if (!ex) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL argument");
    if (cycles < 1000 || cycles > (int64_t)1e12)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "wait limit must be in [1e3, 1e12] GPU clock cycles");
    ex->wait_cycles = cycles;
    return COTTUS_OK;
}

void cottus_peer_exchange_destroy(cottus_peer_exchange* ex) {
    if (!ex) return;
    for (int r = 0; r < ex->world; ++r) {
        if (r == ex->rank || !ex->base[r]) continue;
        if (ex->absent[r]) cudaFree(ex->base[r]);
        else cudaIpcCloseMemHandle(ex->base[r]);
    }
    if (ex->local) cudaFree(ex->local);
    delete ex;
}

size_t cottus_split_decode_workspace_size(const cottus_paged_decode_params* p) {
    if (!p) return 0;
    cottus_paged_decode_params q = *p;  // the decode runs in partial mode: fp32 outputs and LSEs
    float dummy;
    q.out_dtype = COTTUS_F32;
    q.lse_out = &dummy;
    return cottus_paged_decode_workspace_size(&q);
}

int cottus_split_decode(const cottus_paged_decode_params* p, cottus_peer_exchange* ex, cottus_stream_t stream) {
    if (!p || !ex) return fail(COTTUS_ERR_INVALID_ARGUMENT, "NULL argument");
    if (!ex->opened) return fail(COTTUS_ERR_INVALID_ARGUMENT, "exchange not opened (cottus_peer_exchange_open)");
    if (p->batch != ex->batch || p->num_heads != ex->heads || p->head_dim != ex->head_dim)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "batch, num_heads and head_dim must match the exchange");
    if (p->out_dtype != COTTUS_F32 && p->out_dtype != COTTUS_F16)
        return fail(COTTUS_ERR_INVALID_ARGUMENT, "unsupported dtype");
    const uint32_t epoch = ++ex->epoch;
    const size_t slot = ex->lay.slot0 + (size_t)(epoch & 1u) * ex->lay.slot_bytes;
    // 1. this rank's partials into its own slot, completion flagged to every rank
    cottus_paged_decode_params q = *p;
    q.out = ex->local + slot;
    q.out_dtype = COTTUS_F32;
    q.lse_out = reinterpret_cast<float*>(ex->local + slot + ex->lay.part_bytes);
    cb200::PeerSignal sig;
    for (int r = 0; r < ex->world; ++r) sig.flags[r] = reinterpret_cast<uint32_t*>(ex->base[r] + ex->lay.flags);
    sig.done = reinterpret_cast<uint32_t*>(ex->local + ex->lay.done);
    sig.rank = ex->rank;
    sig.world = ex->world;
    sig.epoch = epoch;
#if CB200_SPLIT_MERGE_IN_DECODE
    // on the tensor-core path the decode kernel merges the ranks' partials itself
    cb200::PeerMerge pm;
    for (int r = 0; r < ex->world; ++r) {
        pm.part[r] = reinterpret_cast<const float*>(ex->base[r] + slot);
        pm.lse[r] = reinterpret_cast<const float*>(ex->base[r] + slot + ex->lay.part_bytes);
        pm.broken[r] = reinterpret_cast<uint32_t*>(ex->base[r] + ex->lay.broken);
    }
    pm.flags = reinterpret_cast<const uint32_t*>(ex->local + ex->lay.flags);
    pm.broken_own = reinterpret_cast<uint32_t*>(ex->local + ex->lay.broken);
    pm.out = p->out;
    pm.out_f16 = p->out_dtype == COTTUS_F16;
    pm.lse_out = p->lse_out;
    pm.wait_cycles = ex->wait_cycles;
    pm.enabled = 1;
    const int rcx = cb200::paged_decode_exchanged(&q, sig, pm, reinterpret_cast<cudaStream_t>(stream));
    if (rcx != COTTUS_ERR_UNSUPPORTED) return rcx;
#endif
    // otherwise: the decode (its completion signalled), then a combine kernel
    const int rc = cb200::paged_decode_signalled(&q, sig, reinterpret_cast<cudaStream_t>(stream));
    if (rc != COTTUS_OK) return rc;
    // 2. wait for every rank's flag, pull and merge
    cb200::PeerSlots src = {};
    for (int r = 0; r < ex->world; ++r) {
        src.part[r] = reinterpret_cast<const float*>(ex->base[r] + slot);
        src.lse[r] = reinterpret_cast<const float*>(ex->base[r] + slot + ex->lay.part_bytes);
        src.broken[r] = reinterpret_cast<uint32_t*>(ex->base[r] + ex->lay.broken);
    }
    cb200::CombineCtl ctl;
    ctl.flags = reinterpret_cast<const uint32_t*>(ex->local + ex->lay.flags);
    ctl.done = reinterpret_cast<uint32_t*>(ex->local + ex->lay.done);
    ctl.broken = reinterpret_cast<uint32_t*>(ex->local + ex->lay.broken);
    ctl.epoch = epoch;
    ctl.wait_cycles = ex->wait_cycles;
    const long long heads = (long long)ex->batch * ex->heads;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((heads * 32 + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, cb200::peer_combine_kernel, src, ex->world, ctl, p->out,
                                             (int)(p->out_dtype == COTTUS_F16), p->lse_out, heads, ex->head_dim,
                                             p->status);
    if (e != cudaSuccess) return cuda_fail(e);
    return COTTUS_OK;
}

}  // extern "C"
