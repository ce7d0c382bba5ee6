// Same-signature drop-in for the reference's cottus::ropeCUDA
// (compute_primitives_cuda.h:22-29): device pointers, in place allowed,
// default stream.  (cos, sin) are evaluated on the host with the
// reference's float formula (compute_primitives_cpu.cpp:54-57) and the
// rotation is computed without FMA contraction, so the result equals
// cottus::ropeCPU bit for bit.
#pragma once

#include <cstdint>

namespace cottus {

void ropeCUDA(float* d_output, const float* d_input, int32_t pos, int32_t numHeads, int32_t headDim,
              float theta = 10000.0f);

}  // namespace cottus
