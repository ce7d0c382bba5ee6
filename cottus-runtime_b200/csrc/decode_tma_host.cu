// Host side of the TMA fast path: support predicate, workspace size,
// KV-pool tensor map, per-device SM count, dispatch by head_dim.
#include <cudaTypedefs.h>

#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <mutex>

#include "decode_tma.cuh"

namespace cb200 {

int device_sm_count(int device) {
    static int cache[64] = {0};
    if (device < 0 || device >= 64) return 148;
    if (cache[device] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        cache[device] = n > 0 ? n : 148;
    }
    return cache[device];
}

// Launch tags of the pair arrival counters.  Seeded per process so that a
// counter left behind by an aborted launch of another process is unlikely
// to carry a live tag; 0 is never used.
unsigned next_epoch() {
    static std::atomic<unsigned> ctr{[] {
        const auto t = (unsigned long long)std::chrono::steady_clock::now().time_since_epoch().count();
        return (unsigned)((t * 0x9E3779B97F4A7C15ull) >> 32) ^ ((unsigned)getpid() << 16);
    }()};
    unsigned e;
    do {
        e = ctr.fetch_add(1, std::memory_order_relaxed) + 1;
    } while (e == 0);
    return e;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// View of the pool as rows of head_dim fp16 values:
//   dim0 = head_dim (contiguous), dim1 = kv head (stride head_dim),
//   dim2 = (block, layer, K|V, token) rows (stride num_kv_heads*head_dim).
// One 16 x 2 box row range of dim2 covers the K rows then the V rows of a
// page/layer, so box {head_dim, 1, 32} loads both tiles of one kv head.
CUtensorMap make_kv_tensor_map(const DecodeDesc& d, bool swizzle128, cudaError_t* err) {
    CUtensorMap map;
    std::memset(&map, 0, sizeof map);
    auto fn = encode_fn();
    if (!fn) {
        *err = cudaErrorNotSupported;
        return map;
    }
    const void* base = d.rope ? static_cast<const void*>(d.kv_mut) : static_cast<const void*>(d.kv);
    cuuint64_t dims[3] = {(cuuint64_t)d.head_dim, (cuuint64_t)d.num_kv_heads,
                          (cuuint64_t)d.num_blocks * d.num_layers * 2 * kBS};
    cuuint64_t strides[2] = {(cuuint64_t)d.head_dim * 2, (cuuint64_t)d.num_kv_heads * d.head_dim * 2};
    // plain: one {head_dim, 1, 32} box per page; swizzled: {64, 1, 32} boxes
    // (128-byte rows, 128B swizzle) for conflict-free ldmatrix
    cuuint32_t box[3] = {swizzle128 ? 64u : (cuuint32_t)d.head_dim, 1, 2 * kBS};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    *err = r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
    return map;
}

// 2-D tiled map over a row-major fp16 matrix [outer][inner] (row pitch
// `pitch_bytes`), box {box_inner, box_outer}, optionally 128-byte swizzled.
CUtensorMap make_tensor_map_2d_f16(const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_bytes,
                                   uint32_t box_inner, uint32_t box_outer, bool swizzle128, cudaError_t* err) {
    CUtensorMap map;
    std::memset(&map, 0, sizeof map);
    auto fn = encode_fn();
    if (!fn) {
        *err = cudaErrorNotSupported;
        return map;
    }
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    *err = r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
    return map;
}

// Leading bytes of a decode workspace: a reserved word and one arrival
// counter per (sequence, kv head) pair, rounded to 256 bytes.
size_t workspace_zero_prefix_bytes(int32_t batch, int32_t num_kv_heads) {
    return ((1 + (size_t)batch * (size_t)num_kv_heads) * 8 + 255) & ~size_t(255);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool tma_supported(const DecodeDesc& d) {
    if (d.block_size != kBS) return false;
    if (d.head_dim != 64 && d.head_dim != 128 && d.head_dim != 256) return false;
    if (d.num_kv_heads <= 0 || d.num_heads % d.num_kv_heads != 0) return false;
    const int G = d.num_heads / d.num_kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return false;
    const void* pool = d.rope ? static_cast<const void*>(d.kv_mut) : static_cast<const void*>(d.kv);
    if (!aligned16(pool) || !aligned16(d.q) || !aligned16(d.out)) return false;
    if (d.rope && (!d.cos_sin || !aligned16(d.k_new) || !aligned16(d.v_new) || !aligned16(d.q_out) ||
                   !aligned16(d.cos_sin)))
        return false;
    if (d.num_blocks <= 0 || d.num_blocks * (int64_t)d.num_layers * 2 * kBS >= (int64_t(1) << 31)) return false;
    if ((int64_t)d.batch * d.num_heads >= (int64_t(1) << 31)) return false;
    return true;
}

bool mma_supported(const DecodeDesc& d) {
    if (!tma_supported(d)) return false;
    if (d.head_dim != 64 && d.head_dim != 128) return false;
    // without grouped queries the SIMT kernel is faster (measured: 6.1 vs
    // 5.5 TB/s on the MHA workload)
    // (fp32 outputs split the probabilities into fp16 hi + lo parts)
    return d.num_heads != d.num_kv_heads;
}

static size_t workers(const DecodeDesc& d) {
    if (mma_supported(d)) return d.head_dim == 64 ? mma_workers_d64(d) : mma_workers_d128(d);
    switch (d.head_dim) {
        case 64: return tma_workers_d64(d);
        case 128: return tma_workers_d128(d);
        case 256: return tma_workers_d256(d);
    }
    return 0;
}

size_t tma_workspace_bytes(const DecodeDesc& d) {
    const size_t W = workers(d);
    const size_t G = (size_t)(d.num_heads / d.num_kv_heads);
    const size_t ctr_bytes = workspace_zero_prefix_bytes(d.batch, d.num_kv_heads);
    return ctr_bytes + 2 * (size_t)max_chunks((long long)W) * G * ((size_t)d.head_dim + 2) * sizeof(float) + 256;
}

cudaError_t launch_decode_tma(const DecodeDesc& d, cudaStream_t st) {
    if (mma_supported(d)) return d.head_dim == 64 ? launch_decode_mma_d64(d, st) : launch_decode_mma_d128(d, st);
    switch (d.head_dim) {
        case 64: return launch_decode_tma_d64(d, st);
        case 128: return launch_decode_tma_d128(d, st);
        case 256: return launch_decode_tma_d256(d, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace cb200
