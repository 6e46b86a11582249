// Tensor-core (tcgen05) GEMM entry points.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "kernels.cuh"

namespace pet {

// Pre-split copies of the B operand of a GEMM: hi = tf32(B), lo = B - hi,
// same layout and leading dimension as GemmArgs::B.
struct TCWeights {
  const float *hi = nullptr;
  const float *lo = nullptr;
};

// fp16 pre-split copies of a B operand for the 3xFP16 kernel: B 2^b_scale
// = hi + lo (both fp16, round-to-nearest), one power-of-two scale per
// weight tensor chosen so that its largest |element| maps into [2^14, 2^15).
struct TCWeights16 {
  const uint16_t *hi = nullptr;
  const uint16_t *lo = nullptr;
  int b_scale = 0;
  // 3: A_hi B_hi + A_hi B_lo + A_lo B_hi (fp32 accuracy); 1: A_hi B_hi only
  // (the reduced-precision mode: 11 significant bits per operand)
  int products = 3;
};

// True when the shape and alignment fit the tensor-core kernel (N multiple
// of 128, K multiple of 32, 16-byte aligned rows).
bool gemm_tc_supported(const GemmArgs &a);
// True when the 3xFP16 kernel applies as well (K a multiple of 128 and at
// most 2048, B rows 16-byte aligned in fp16).
bool gemm_f16_supported(const GemmArgs &a);

// C = A B^T (+ epilogue) with 3xTF32 on tcgen05; `err` (device int) is set
// non-zero if a pipeline wait times out.
void gemm_3xtf32(const GemmArgs &a, const TCWeights &w, int *err, cudaStream_t s);

// C = A B^T (+ epilogue) with 3xFP16 on tcgen05.  A comes in split-fp16
// form (a.a_split; when not a.a_split_ready a pre-pass first writes it from
// the fp32 A, row-gathered): fp16 hi + lo scaled by 2^s per row and
// 128-element k block.  B is pre-split with one scale 2^b_scale.
// A B^T ~= sum over blocks of (A_hi B_hi + A_hi B_lo + A_lo B_hi)
// 2^-(s + b_scale) with fp32 accumulation, operands streamed by TMA.  With
// a.c_split the epilogue also writes the result in split form.
void gemm_3xf16(const GemmArgs &a, const TCWeights16 &w, int *err, cudaStream_t s);

// Failure-detection test hooks.  inject_gemm_stall: the next 3xFP16 launch
// with a plain store epilogue withholds the operand loads of its first CTA,
// whose bounded waits then run out (the launch sets *err = 1; the CTA
// drains its own copies and MMAs and frees its TMEM).  set_gemm_wait_bound_ns:
// the bound of the GEMM kernels' waits on the current device (0: 1 s).
void inject_gemm_stall();
bool gemm_stall_armed();
void set_gemm_wait_bound_ns(uint64_t ns);

// Power-of-two scale exponent s with max|x| 2^s in [2^14, 2^15) (0 for an
// all-zero tensor, clamped to [-120, 120]).
int f16_scale_exponent(float max_abs);

}  // namespace pet
