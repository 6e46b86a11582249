// Tensor-core (tcgen05) GEMM entry points.
#pragma once

#include <cuda_runtime.h>

#include "kernels.cuh"

namespace pet {

// Pre-split copies of the B operand of a GEMM: hi = tf32(B), lo = B - hi,
// same layout and leading dimension as GemmArgs::B.
struct TCWeights {
  const float *hi = nullptr;
  const float *lo = nullptr;
};

// True when the shape and alignment fit the tensor-core kernel (N multiple
// of 128, K multiple of 32, 16-byte aligned rows).
bool gemm_tc_supported(const GemmArgs &a);

// C = A B^T (+ epilogue) with 3xTF32 on tcgen05; `err` (device int) is set
// non-zero if a pipeline wait times out.
void gemm_3xtf32(const GemmArgs &a, const TCWeights &w, int *err, cudaStream_t s);

}  // namespace pet
