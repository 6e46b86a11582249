// Exact-fp32 SIMT GEMM with fused epilogues: the correctness baseline and
// the fallback for shapes the tensor-core kernel does not take.  128x128
// CTA tile, 8x8 outputs per thread, register-staged double-buffered smem.
#include "common.cuh"
#include "kernels.cuh"

namespace pet {
namespace {

constexpr int BM = 128, BN = 128, BK = 8;

template <int EPI, bool VEC>
__global__ void __launch_bounds__(256) k_gemm_f32(GemmArgs p) {
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int lr = tid >> 1, lk = (tid & 1) * 4;
  const float *arow = nullptr, *brow = nullptr;
  if (m0 + lr < p.M) {
    const int r = p.a_rows ? p.a_rows[m0 + lr] : (m0 + lr);
    arow = p.A + static_cast<size_t>(r) * p.lda;
  }
  if (n0 + lr < p.N) brow = p.B + static_cast<size_t>(n0 + lr) * p.ldb;

  auto ld4 = [&](const float *row, int k) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!row) return v;
    if (VEC && k + 3 < p.K) return *reinterpret_cast<const float4 *>(row + k);
    if (k < p.K) v.x = row[k];
    if (k + 1 < p.K) v.y = row[k + 1];
    if (k + 2 < p.K) v.z = row[k + 2];
    if (k + 3 < p.K) v.w = row[k + 3];
    return v;
  };
  auto st = [&](int buf, float4 a, float4 b) {
    As[buf][lk + 0][lr] = a.x; As[buf][lk + 1][lr] = a.y;
    As[buf][lk + 2][lr] = a.z; As[buf][lk + 3][lr] = a.w;
    Bs[buf][lk + 0][lr] = b.x; Bs[buf][lk + 1][lr] = b.y;
    Bs[buf][lk + 2][lr] = b.z; Bs[buf][lk + 3][lr] = b.w;
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int ty = tid >> 4, tx = tid & 15;
  float4 ra = ld4(arow, lk), rb = ld4(brow, lk);
  st(0, ra, rb);
  __syncthreads();
  const int nk = (p.K + BK - 1) / BK;
  for (int kt = 0; kt < nk; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < nk) {
      ra = ld4(arow, (kt + 1) * BK + lk);
      rb = ld4(brow, (kt + 1) * BK + lk);
    }
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[cur][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[cur][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[cur][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[cur][kk][64 + tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) st(cur ^ 1, ra, rb);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= p.M) continue;
    const int rc = p.c_rows ? p.c_rows[m] : m;
    float *crow = p.C + static_cast<size_t>(rc) * p.ldc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int nb = n0 + h * 64 + tx * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = nb + j;
        if (n >= p.N) continue;
        float v = acc[i][h * 4 + j];
        if (p.bias) v += p.bias[n];
        if (EPI == EPI_STORE) {
          crow[n] = v;
        } else if (EPI == EPI_SILU) {
          float y, dy;
          silu_pair(v, y, dy);
          if (p.Z) p.Z[static_cast<size_t>(m) * p.ldz + n] = dy;
          crow[n] = y;
        } else if (EPI == EPI_ACCUM) {
          crow[n] += v;
        } else if (EPI == EPI_DSILU) {
          crow[n] = v * p.Z[static_cast<size_t>(m) * p.ldz + n];
        } else {  // EPI_RESID
          crow[n] = v + p.R[static_cast<size_t>(rc) * p.ldr + n];
        }
      }
    }
  }
}

template <int EPI>
void launch(const GemmArgs &a, cudaStream_t s) {
  dim3 grid(ceil_div(a.M, BM), ceil_div(a.N, BN));
  const bool vec = (a.lda % 4 == 0) && (a.ldb % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(a.A) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(a.B) % 16 == 0);
  if (vec) k_gemm_f32<EPI, true><<<grid, 256, 0, s>>>(a);
  else k_gemm_f32<EPI, false><<<grid, 256, 0, s>>>(a);
  CUDA_LAUNCH_CHECK();
}

}  // namespace

void gemm_f32(const GemmArgs &a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return;
  if (a.N > 65535 * BN) throw Error(kErrInvalidParameter, "gemm: N too large");
  switch (a.epi) {
    case EPI_STORE: launch<EPI_STORE>(a, s); break;
    case EPI_SILU: launch<EPI_SILU>(a, s); break;
    case EPI_ACCUM: launch<EPI_ACCUM>(a, s); break;
    case EPI_DSILU: launch<EPI_DSILU>(a, s); break;
    case EPI_RESID: launch<EPI_RESID>(a, s); break;
    default: throw Error(kErrInternal, "gemm: bad epilogue");
  }
}

}  // namespace pet
