// Fast-path instantiations for head_dim 64 (ring of 4 pages per warp).
#include "decode_tma.cuh"

#ifndef CB200_RING_D64
#define CB200_RING_D64 4
#endif

namespace cb200 {
cudaError_t launch_decode_tma_d64(const DecodeDesc& d, cudaStream_t st) { return dispatch_tma<64, CB200_RING_D64>(d, st); }
size_t tma_workers_d64(const DecodeDesc& d) { return dispatch_workers<64, CB200_RING_D64>(d); }
}  // namespace cb200
