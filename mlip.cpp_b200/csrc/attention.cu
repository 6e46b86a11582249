// Per-atom multi-head attention over each atom's own token block (node token
// + its n_i edge tokens), forward and backward, exact fp32.
//
// Reference: build_multi_head_attention, src/models/pet/pet_layers.cpp:318-492
// (softmax(Q K^T / sqrt(hd) + mask) V, mask shared across heads and along
// queries, keys innermost) and the attention masks of
// src/models/pet/pet_batch.cpp:570-666.  The reference pads every atom to a
// global max_neighbors and masks the pads with -inf; those keys get exactly
// zero weight, so processing each atom's real S_i = n_i + 1 tokens only is
// the same computation without the padding.
//
// One CTA per (atom, head): K and V (and for backward Q, dO, P, dS) of that
// head live in shared memory with a +1 pad so lane-per-key and
// lane-per-channel accesses are bank-conflict free.
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"

namespace pet {
namespace {

constexpr int kFwdWarps = 2;
constexpr int kBwdWarps = 4;

size_t fwd_smem(int S, int hd) {
  return sizeof(float) * (2ull * S * (hd + 1) + S + kFwdWarps * hd + kFwdWarps * S);
}
size_t bwd_smem(int S, int hd) {
  return sizeof(float) * (4ull * S * (hd + 1) + S + 2ull * S * (S + 1));
}

template <int HD>
__global__ void __launch_bounds__(32 * kFwdWarps) k_attn_fwd(AttnArgs a) {
  extern __shared__ float sm[];
  const int atom = blockIdx.x, h = blockIdx.y;
  const int e0 = a.offset[atom];
  const int S = a.offset[atom + 1] - e0 + 1;
  const int t0 = e0 + atom;
  const int d = a.d, ld = 3 * d;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float *sK = sm;
  float *sV = sK + S * (HD + 1);
  float *sM = sV + S * (HD + 1);
  float *sQ = sM + S + w * HD;
  float *sP = sM + S + kFwdWarps * HD + w * S;
  for (int idx = threadIdx.x; idx < S * HD; idx += blockDim.x) {
    const int s = idx / HD, c = idx % HD;
    const float *row = a.qkv + static_cast<size_t>(t0 + s) * ld + h * HD + c;
    sK[s * (HD + 1) + c] = row[d];
    sV[s * (HD + 1) + c] = row[2 * d];
  }
  for (int s = threadIdx.x; s < S; s += blockDim.x) sM[s] = s == 0 ? 0.f : a.key_mask[e0 + s - 1];
  __syncthreads();
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  for (int q = w; q < S; q += kFwdWarps) {
    const float *qrow = a.qkv + static_cast<size_t>(t0 + q) * ld + h * HD;
    for (int c = lane; c < HD; c += 32) sQ[c] = qrow[c];
    __syncwarp();
    float mx = -FLT_MAX;
    for (int k = lane; k < S; k += 32) {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < HD; ++c) s = fmaf(sQ[c], sK[k * (HD + 1) + c], s);
      s = s * scale + sM[k];
      sP[k] = s;
      mx = fmaxf(mx, s);
    }
    mx = warp_max(mx);
    float sum = 0.f;
    for (int k = lane; k < S; k += 32) {
      const float p = expf(sP[k] - mx);
      sP[k] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    __syncwarp();
    const float inv = 1.0f / sum;
    float *orow = a.out + static_cast<size_t>(t0 + q) * d + h * HD;
    for (int c = lane; c < HD; c += 32) {
      float o = 0.f;
      for (int k = 0; k < S; ++k) o = fmaf(sP[k], sV[k * (HD + 1) + c], o);
      orow[c] = o * inv;
    }
    __syncwarp();
  }
}

// dV = P^T dO, dP = dO V^T, dS = P (dP - rowsum(P dP)), dQ = s dS K, dK = s dS^T Q.
// The mask is a constant input in the reference (pet.cpp:274-275): no grad.
template <int HD>
__global__ void __launch_bounds__(32 * kBwdWarps) k_attn_bwd(AttnArgs a) {
  extern __shared__ float sm[];
  const int atom = blockIdx.x, h = blockIdx.y;
  const int e0 = a.offset[atom];
  const int S = a.offset[atom + 1] - e0 + 1;
  const int t0 = e0 + atom;
  const int d = a.d, ld = 3 * d;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int P1 = HD + 1, PS = S + 1;
  float *sQ = sm;
  float *sK = sQ + S * P1;
  float *sV = sK + S * P1;
  float *sG = sV + S * P1;  // dO
  float *sM = sG + S * P1;
  float *sP = sM + S;       // [S][S+1]
  float *sD = sP + S * PS;  // dS [S][S+1]
  for (int idx = threadIdx.x; idx < S * HD; idx += blockDim.x) {
    const int s = idx / HD, c = idx % HD;
    const float *row = a.qkv + static_cast<size_t>(t0 + s) * ld + h * HD + c;
    sQ[s * P1 + c] = row[0];
    sK[s * P1 + c] = row[d];
    sV[s * P1 + c] = row[2 * d];
    sG[s * P1 + c] = a.d_out[static_cast<size_t>(t0 + s) * d + h * HD + c];
  }
  for (int s = threadIdx.x; s < S; s += blockDim.x) sM[s] = s == 0 ? 0.f : a.key_mask[e0 + s - 1];
  __syncthreads();
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  for (int q = w; q < S; q += kBwdWarps) {
    float *prow = sP + q * PS;
    float *drow = sD + q * PS;
    float mx = -FLT_MAX;
    for (int k = lane; k < S; k += 32) {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < HD; ++c) s = fmaf(sQ[q * P1 + c], sK[k * P1 + c], s);
      s = s * scale + sM[k];
      prow[k] = s;
      mx = fmaxf(mx, s);
    }
    mx = warp_max(mx);
    float sum = 0.f;
    for (int k = lane; k < S; k += 32) {
      const float p = expf(prow[k] - mx);
      prow[k] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    float dsum = 0.f;
    for (int k = lane; k < S; k += 32) {
      const float p = prow[k] * inv;
      prow[k] = p;
      float dp = 0.f;
#pragma unroll
      for (int c = 0; c < HD; ++c) dp = fmaf(sG[q * P1 + c], sV[k * P1 + c], dp);
      drow[k] = dp;
      dsum = fmaf(p, dp, dsum);
    }
    dsum = warp_sum(dsum);
    for (int k = lane; k < S; k += 32) drow[k] = prow[k] * (drow[k] - dsum);
    __syncwarp();
    float *dq = a.d_qkv + static_cast<size_t>(t0 + q) * ld + h * HD;
    for (int c = lane; c < HD; c += 32) {
      float acc = 0.f;
      for (int k = 0; k < S; ++k) acc = fmaf(drow[k], sK[k * P1 + c], acc);
      dq[c] = acc * scale;
    }
  }
  __syncthreads();
  for (int k = w; k < S; k += kBwdWarps) {
    float *dk = a.d_qkv + static_cast<size_t>(t0 + k) * ld + h * HD;
    for (int c = lane; c < HD; c += 32) {
      float gk = 0.f, gv = 0.f;
      for (int q = 0; q < S; ++q) {
        gk = fmaf(sD[q * PS + k], sQ[q * P1 + c], gk);
        gv = fmaf(sP[q * PS + k], sG[q * P1 + c], gv);
      }
      dk[d + c] = gk * scale;
      dk[2 * d + c] = gv;
    }
  }
}

template <int HD>
void run_fwd(const AttnArgs &a, cudaStream_t s) {
  const size_t sm = fwd_smem(a.max_tokens, HD);
  CUDA_CHECK(cudaFuncSetAttribute(k_attn_fwd<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(sm)));
  k_attn_fwd<HD><<<dim3(a.n_atoms, a.heads), 32 * kFwdWarps, sm, s>>>(a);
  CUDA_LAUNCH_CHECK();
}

template <int HD>
void run_bwd(const AttnArgs &a, cudaStream_t s) {
  const size_t sm = bwd_smem(a.max_tokens, HD);
  CUDA_CHECK(cudaFuncSetAttribute(k_attn_bwd<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(sm)));
  k_attn_bwd<HD><<<dim3(a.n_atoms, a.heads), 32 * kBwdWarps, sm, s>>>(a);
  CUDA_LAUNCH_CHECK();
}

constexpr size_t kSmemLimit = 227 * 1024;

}  // namespace

int attention_max_tokens(int hd) {
  int S = 1;
  while (bwd_smem(S + 1, hd) <= kSmemLimit && fwd_smem(S + 1, hd) <= kSmemLimit) ++S;
  return S;
}

void attention_fwd(const AttnArgs &a, cudaStream_t s) {
  if (a.n_atoms <= 0) return;
  const int hd = a.d / a.heads;
  if (a.max_tokens > attention_max_tokens(hd))
    throw Error(kErrUnsupported, "attention: " + std::to_string(a.max_tokens - 1) +
                                     " neighbours exceed the per-atom limit");
  switch (hd) {
    case 16: run_fwd<16>(a, s); break;
    case 32: run_fwd<32>(a, s); break;
    case 64: run_fwd<64>(a, s); break;
    default: throw Error(kErrUnsupported, "attention: head size " + std::to_string(hd));
  }
}

void attention_bwd(const AttnArgs &a, cudaStream_t s) {
  if (a.n_atoms <= 0) return;
  const int hd = a.d / a.heads;
  if (a.max_tokens > attention_max_tokens(hd))
    throw Error(kErrUnsupported, "attention: " + std::to_string(a.max_tokens - 1) +
                                     " neighbours exceed the per-atom limit");
  switch (hd) {
    case 16: run_bwd<16>(a, s); break;
    case 32: run_bwd<32>(a, s); break;
    case 64: run_bwd<64>(a, s); break;
    default: throw Error(kErrUnsupported, "attention: head size " + std::to_string(hd));
  }
}

// ---------------------------------------------------------------------------
// Layer norm (warp per row)
// ---------------------------------------------------------------------------
namespace {

constexpr float kLnEps = 1e-5f;

__global__ void k_ln_fwd(const float *__restrict__ x, const float *__restrict__ g,
                         const float *__restrict__ b, float *__restrict__ y,
                         float *__restrict__ xhat, float *__restrict__ rstd, int rows, int d) {
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float *xr = x + static_cast<size_t>(row) * d;
  float s = 0.f;
  for (int c = lane; c < d; c += 32) s += xr[c];
  const float inv_d = 1.0f / static_cast<float>(d);
  const float mean = warp_sum(s) * inv_d;
  float v = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float t = xr[c] - mean;
    v = fmaf(t, t, v);
  }
  const float var = warp_sum(v) * inv_d;
  const float sd = sqrtf(var * (1.0f + kLnEps));
  float *yr = y + static_cast<size_t>(row) * d;
  float *hr = xhat + static_cast<size_t>(row) * d;
  for (int c = lane; c < d; c += 32) {
    const float h = (xr[c] - mean) / sd;
    hr[c] = h;
    yr[c] = h * g[c] + b[c];
  }
  if (lane == 0) rstd[row] = 1.0f / sd;
}

__global__ void k_ln_bwd(const float *__restrict__ dy, const float *__restrict__ xhat,
                         const float *__restrict__ rstd, const float *__restrict__ g,
                         float *__restrict__ dx, int rows, int d) {
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float *dyr = dy + static_cast<size_t>(row) * d;
  const float *hr = xhat + static_cast<size_t>(row) * d;
  float s1 = 0.f, s2 = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float gh = dyr[c] * g[c];
    s1 += gh;
    s2 = fmaf(gh, hr[c], s2);
  }
  const float inv_d = 1.0f / static_cast<float>(d);
  const float m1 = warp_sum(s1) * inv_d;
  const float m2 = warp_sum(s2) * inv_d * (1.0f + kLnEps);
  const float r = rstd[row];
  float *dxr = dx + static_cast<size_t>(row) * d;
  for (int c = lane; c < d; c += 32) dxr[c] = r * (dyr[c] * g[c] - m1 - hr[c] * m2);
}

}  // namespace

void layer_norm_fwd(const float *x, const float *g, const float *b, float *y, float *xhat,
                    float *rstd, int rows, int d, cudaStream_t s) {
  if (rows <= 0) return;
  k_ln_fwd<<<ceil_div(static_cast<int64_t>(rows) * 32, 256), 256, 0, s>>>(x, g, b, y, xhat, rstd, rows, d);
  CUDA_LAUNCH_CHECK();
}

void layer_norm_bwd(const float *dy, const float *xhat, const float *rstd, const float *g,
                    float *dx, int rows, int d, cudaStream_t s) {
  if (rows <= 0) return;
  k_ln_bwd<<<ceil_div(static_cast<int64_t>(rows) * 32, 256), 256, 0, s>>>(dy, xhat, rstd, g, dx, rows, d);
  CUDA_LAUNCH_CHECK();
}

}  // namespace pet
