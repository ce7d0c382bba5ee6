// Fast-path instantiations for head_dim 64 (ring of 4 pages per warp).
#include "decode_tma.cuh"

namespace cb200 {
cudaError_t launch_decode_tma_d64(const DecodeDesc& d, cudaStream_t st) { return dispatch_tma<64, 4>(d, st); }
size_t tma_workers_d64(const DecodeDesc& d) { return dispatch_workers<64, 4>(d); }
}  // namespace cb200
