// "Split fp16" form of an fp32 matrix, the A operand format of the 3xFP16
// tensor-core GEMM: hi = rn(x 2^s), lo = rn(x 2^s - hi) (fp16 each,
// [rows][cols], row-major) with one power-of-two scale exponent s per row and
// 128-column block ([cols / 128][rows] int8), chosen so that the block's
// largest |element| maps into [2^14, 2^15).  hi + lo carries 22 significant
// bits of every element; elements below 2^-17 of their block's maximum keep
// an absolute error under 2^-40 of it.  Kernels that produce a GEMM's A
// operand write this form directly (Split16View in kernels.cuh).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "kernels.cuh"

namespace pet {

// 2^e for e in [-126, 127], built from its IEEE-754 bit pattern (exact).
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// s with mx 2^s in [2^14, 2^15); 0 for mx = 0; clamped to [-120, 120].
__device__ __forceinline__ int split_scale_exponent(float mx) {
  if (!(mx > 0.f)) return 0;
  const int E = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu);
  const int s = 141 - (E > 0 ? E : 0);
  return s < -120 ? -120 : (s > 120 ? 120 : s);
}

// Two scaled values -> packed fp16 hi pair and lo pair.
__device__ __forceinline__ void split2(float a, float b, float f, uint32_t &h, uint32_t &l) {
  const float x0 = a * f, x1 = b * f;
  const __half2 hh = __floats2half2_rn(x0, x1);
  const float2 r = __half22float2(hh);
  const __half2 ll = __floats2half2_rn(x0 - r.x, x1 - r.y);
  h = *reinterpret_cast<const uint32_t *>(&hh);
  l = *reinterpret_cast<const uint32_t *>(&ll);
}

// Warp-wide: lane l holds columns 4l..4l+3 of 128-column block `blk` of
// row `row`; writes the block's split form and its scale.
__device__ __forceinline__ void warp_split_block(const Split16View &o, int row, int blk, float4 v, int lane) {
  float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, k));
  const int s = split_scale_exponent(mx);
  const float f = pow2f(s);
  uint32_t h0, h1, l0, l1;
  split2(v.x, v.y, f, h0, l0);
  split2(v.z, v.w, f, h1, l1);
  const size_t off = static_cast<size_t>(row) * o.cols + blk * 128 + lane * 4;
  *reinterpret_cast<uint2 *>(o.hi + off) = make_uint2(h0, h1);
  if (o.lo) *reinterpret_cast<uint2 *>(o.lo + off) = make_uint2(l0, l1);
  if (lane == 0) o.sc[static_cast<size_t>(blk) * split_ld(o) + row] = static_cast<int8_t>(s);
}

// One thread: n consecutive values (n a multiple of 8) of one row segment
// starting at column c0, all in block c0 / 128, scaled by 2^s.
template <int n>
__device__ __forceinline__ void thread_split_store(const Split16View &o, int row, int c0, const float *v, int s) {
  const float f = pow2f(s);
  uint16_t *hp = o.hi + static_cast<size_t>(row) * o.cols + c0;
  uint16_t *lp = o.lo ? o.lo + static_cast<size_t>(row) * o.cols + c0 : nullptr;
#pragma unroll
  for (int i = 0; i < n; i += 8) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) split2(v[i + 2 * k], v[i + 2 * k + 1], f, h[k], l[k]);
    *reinterpret_cast<uint4 *>(hp + i) = make_uint4(h[0], h[1], h[2], h[3]);
    if (lp) *reinterpret_cast<uint4 *>(lp + i) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

}  // namespace pet
