// cottus_paged_decode_static_scratch: the batched paged decode for callers
// that cannot allocate device memory.
//
// Some callers have no way to call cudaMalloc (or any allocating routine)
// at the point where they run attention: code inside a custom allocator or
// memory-pool callback, engines that reserve all device memory up front and
// forbid later allocations, and plugin hosts that hand a plugin only a
// stream and the tensors of one call.  cottus_paged_decode needs a
// caller-provided workspace for split-KV partials; this variant uses a
// fixed scratch array that is part of the library's device image instead.
//
// The array is a file-scope __device__ variable, so every GPU that loads
// the library holds kStaticScratchBytes of it until the process exits.
// Its host-side name is only a stand-in for the symbol: the device address
// is obtained once per device with cudaGetSymbolAddress (the first call on
// a device does this set-up, so that first call should come before any
// stream capture).  All calls on a device share the array and it keeps the
// previous call's contents; the arrival counters that must start at zero
// are cleared (cudaMemsetAsync, no allocation) at every call.  Calls whose
// executions overlap on the GPU (different streams, no ordering between
// them) race on the array.  The looked-up address is kept with the id of
// the context it belongs to; after a device reset (a new primary context)
// the next call looks it up again.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "cottus_b200.h"
#include "internal.h"

namespace cb200 {
int set_error(int code, const std::string& msg);
}

namespace {

constexpr size_t kStaticScratchBytes = (size_t)32 << 20;  // 32 MiB per device

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct ScratchAddress {
    unsigned long long ctx = 0;  // id of the context the address belongs to (0: none yet)
    void* ptr = nullptr;
};
ScratchAddress g_scratch[kMaxDevices];

// Unique id of the calling thread's current context, 0 when there is none
// or the driver does not report it.
unsigned long long current_context_id() {
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    });
    if (!get_current || !get_id) return 0;
    CUcontext c = nullptr;
    if (get_current(&c) != CUDA_SUCCESS || !c) return 0;
    unsigned long long id = 0;
    return get_id(c, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of the scratch array on the current device (looked up with
// that device current, once per device and context).
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cb200::set_error(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return cb200::set_error(COTTUS_ERR_UNSUPPORTED, "device index out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    ScratchAddress& a = g_scratch[dev];
    const unsigned long long ctx = current_context_id();
    if (!a.ptr || ctx == 0 || ctx != a.ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p)
            return cb200::set_error(COTTUS_ERR_CUDA, std::string("CUDA error: cudaGetSymbolAddress of the static "
                                                                 "scratch failed: ") + cudaGetErrorString(e));
        a.ptr = p;
        a.ctx = current_context_id();  // the lookup made the device's primary context current if none was
    }
    *out = a.ptr;
    return COTTUS_OK;
}

}  // namespace

extern "C" int cottus_paged_decode_static_scratch(const cottus_paged_decode_params* p, cottus_stream_t stream) {
    // the arguments are checked before anything is sized or queued
    const int bad = cb200::validate_decode_params(p);
    if (bad) return bad;
    const size_t need = cottus_paged_decode_workspace_size(p);
    if (need > kStaticScratchBytes)
        return cb200::set_error(COTTUS_ERR_WORKSPACE,
                                "this call needs " + std::to_string(need) + " bytes of scratch; the static scratch "
                                "holds " + std::to_string(kStaticScratchBytes) +
                                " bytes (use cottus_paged_decode with a caller-provided workspace)");
    cottus_paged_decode_params q = *p;
    q.workspace = nullptr;
    q.workspace_bytes = 0;
    if (need > 0 && p->batch > 0) {
        void* scratch = nullptr;
        const int rc = scratch_address(&scratch);
        if (rc != COTTUS_OK) return rc;
        // the pair arrival counters lead the workspace and must start at zero
        const size_t zero = cb200::workspace_zero_prefix_bytes(p->batch, p->num_kv_heads);
        const cudaError_t e = cudaMemsetAsync(scratch, 0, zero, reinterpret_cast<cudaStream_t>(stream));
        if (e != cudaSuccess)
            return cb200::set_error(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e));
        q.workspace = scratch;
        q.workspace_bytes = kStaticScratchBytes;
    }
    return cottus_paged_decode(&q, stream);
}
