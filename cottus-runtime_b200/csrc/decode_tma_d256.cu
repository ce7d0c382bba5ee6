// Fast-path instantiations for head_dim 256 (ring of 2 pages per warp).
#include "decode_tma.cuh"

#ifndef CB200_RING_D256
#define CB200_RING_D256 2
#endif

namespace cb200 {
cudaError_t launch_decode_tma_d256(const DecodeDesc& d, cudaStream_t st) { return dispatch_tma<256, CB200_RING_D256>(d, st); }
size_t tma_workers_d256(const DecodeDesc& d) { return dispatch_workers<256, CB200_RING_D256>(d); }
}  // namespace cb200
