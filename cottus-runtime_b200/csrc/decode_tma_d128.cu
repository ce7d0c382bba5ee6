// Fast-path instantiations for head_dim 128 (ring of 2 pages per warp).
#include "decode_tma.cuh"

#ifndef CB200_RING_D128
#define CB200_RING_D128 2
#endif

namespace cb200 {
cudaError_t launch_decode_tma_d128(const DecodeDesc& d, cudaStream_t st) { return dispatch_tma<128, CB200_RING_D128>(d, st); }
size_t tma_workers_d128(const DecodeDesc& d) { return dispatch_workers<128, CB200_RING_D128>(d); }
}  // namespace cb200
