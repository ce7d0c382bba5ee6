// Fast-path instantiations for head_dim 128 (ring of 2 pages per warp).
#include "decode_tma.cuh"

namespace cb200 {
cudaError_t launch_decode_tma_d128(const DecodeDesc& d, cudaStream_t st) { return dispatch_tma<128, 2>(d, st); }
size_t tma_workers_d128(const DecodeDesc& d) { return dispatch_workers<128, 2>(d); }
}  // namespace cb200
