// Tensor-core path instantiations for head_dim 128 (ring of 2 pages per warp).
#include "decode_mma.cuh"

#ifndef CB200_MMA_RING_D128
#define CB200_MMA_RING_D128 2
#endif

namespace cb200 {
cudaError_t launch_decode_mma_d128(const DecodeDesc& d, cudaStream_t st) {
    long long W = 0;
    return dispatch_mma<128, CB200_MMA_RING_D128>(d, st, false, &W);
}
size_t mma_workers_d128(const DecodeDesc& d) {
    long long W = 0;
    dispatch_mma<128, CB200_MMA_RING_D128>(d, nullptr, true, &W);
    return (size_t)W;
}
}  // namespace cb200
