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
// them) race on the array.
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
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up once per
// device with that device current).
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cb200::set_error(COTTUS_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return cb200::set_error(COTTUS_ERR_UNSUPPORTED, "device index out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p)
            return cb200::set_error(COTTUS_ERR_CUDA, std::string("CUDA error: cudaGetSymbolAddress of the static "
                                                                 "scratch failed: ") + cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return COTTUS_OK;
}

}  // namespace

extern "C" int cottus_paged_decode_static_scratch(const cottus_paged_decode_params* p, cottus_stream_t stream) {
    if (!p) return cb200::set_error(COTTUS_ERR_INVALID_ARGUMENT, "params must not be NULL");
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
