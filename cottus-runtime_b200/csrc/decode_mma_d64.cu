// Tensor-core path instantiations for head_dim 64 (ring of 3 pages per warp).
#include "decode_mma.cuh"

#ifndef CB200_MMA_RING_D64
#define CB200_MMA_RING_D64 3
#endif

namespace cb200 {
cudaError_t launch_decode_mma_d64(const DecodeDesc& d, cudaStream_t st) {
    long long W = 0;
    return dispatch_mma<64, CB200_MMA_RING_D64>(d, st, false, &W);
}
size_t mma_workers_d64(const DecodeDesc& d) {
    long long W = 0;
    dispatch_mma<64, CB200_MMA_RING_D64>(d, nullptr, true, &W);
    return (size_t)W;
}
}  // namespace cb200
