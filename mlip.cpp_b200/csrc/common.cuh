// Shared helpers for the PET B200 backend: error handling, a grow-only
// device arena, and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

namespace pet {

// Host-side failure carrying an mlipcpp_error_t code (see api.cpp).
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

enum ErrorCode {
  kErrNullPointer = 2,
  kErrOutOfMemory = 4,
  kErrIO = 5,
  kErrComputation = 6,
  kErrInvalidParameter = 7,
  kErrBackend = 8,
  kErrUnsupported = 9,
  kErrInternal = 255,
};

inline void cuda_check(cudaError_t e, const char *what, const char *file, int line) {
  if (e == cudaSuccess) return;
  int code = (e == cudaErrorMemoryAllocation) ? kErrOutOfMemory : kErrBackend;
  throw Error(code, std::string("CUDA error in ") + what + " (" + file + ":" +
                        std::to_string(line) + "): " + cudaGetErrorString(e));
}
// Kernels launched by this library (reported through the C API).
extern std::atomic<long long> g_kernel_launches;
// Device allocations (cudaMalloc calls) this library has made in this process.
extern std::atomic<long long> g_device_allocations;

#define CUDA_CHECK(x) ::pet::cuda_check((x), #x, __FILE__, __LINE__)
#define CUDA_LAUNCH_CHECK()                                                  \
  do {                                                                       \
    ::pet::g_kernel_launches.fetch_add(1, std::memory_order_relaxed);        \
    ::pet::cuda_check(cudaGetLastError(), "kernel launch", __FILE__, __LINE__); \
  } while (0)

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// A grow-only device buffer.  `ensure` reallocates (without preserving the
// contents) only when the requested size exceeds the capacity, so buffers are
// reused across predictions of similar size.
struct DevBuf {
  void *ptr = nullptr;
  size_t cap = 0;
  DevBuf() = default;
  DevBuf(const DevBuf &) = delete;
  DevBuf &operator=(const DevBuf &) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    cap = 0;
  }
  void *ensure(size_t bytes) {
    if (bytes <= cap && ptr) return ptr;
    release();
    size_t want = bytes < 256 ? 256 : bytes;
    g_device_allocations.fetch_add(1, std::memory_order_relaxed);
    CUDA_CHECK(cudaMalloc(&ptr, want));
    cap = want;
    return ptr;
  }
  template <class T> T *as() const { return static_cast<T *>(ptr); }
};

// Pinned host buffer for host<->device staging.
struct HostBuf {
  void *ptr = nullptr;
  size_t cap = 0;
  HostBuf() = default;
  HostBuf(const HostBuf &) = delete;
  HostBuf &operator=(const HostBuf &) = delete;
  ~HostBuf() {
    if (ptr) cudaFreeHost(ptr);
  }
  void *ensure(size_t bytes) {
    if (bytes <= cap && ptr) return ptr;
    if (ptr) cudaFreeHost(ptr);
    ptr = nullptr;
    size_t want = bytes < 256 ? 256 : bytes;
    CUDA_CHECK(cudaMallocHost(&ptr, want));
    cap = want;
    return ptr;
  }
  template <class T> T *as() const { return static_cast<T *>(ptr); }
};

#ifdef __CUDACC__
__device__ __forceinline__ float silu_f(float z) { return z / (1.0f + expf(-z)); }
// d silu / dz = s (1 + z (1 - s)), s = sigmoid(z)
__device__ __forceinline__ float dsilu_f(float z) {
  float s = 1.0f / (1.0f + expf(-z));
  return s * (1.0f + z * (1.0f - s));
}
// silu(z) and silu'(z) from the logistic s = 1 / (1 + e^-z), computed with
// the fast intrinsics __expf and __fdividef (a few ulp: below the 22-bit
// precision of the split-fp16 operands these values feed).  z is clamped
// at -80 so that e^-z stays far below the 2^126 where __fdividef returns 0
// early; silu and silu' there are below 1e-33.
__device__ __forceinline__ void silu_pair(float z, float &y, float &dy) {
  const float s = __fdividef(1.0f, 1.0f + __expf(-fmaxf(z, -80.0f)));
  y = z * s;
  dy = s * (1.0f + z * (1.0f - s));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
#endif

}  // namespace pet
