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
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"

namespace pet {
namespace {

// One thread owns one (query token, head) row: its q (forward) or q and dO
// (backward) stay in registers, and the head's K and V rows are read from
// shared memory with 16-byte loads that every thread of a warp shares
// (broadcast), so each load feeds 4-8 FMAs.  A CTA covers one atom and a
// group of HG heads (threads = HG * S).  The forward keeps an online softmax
// and stores each row's log-sum-exp; the backward recomputes P from it.
constexpr size_t kSmemLimit = 227 * 1024;

// Floats between consecutive heads' [S][HD] blocks in shared memory: padded
// to 16 mod 32 so the two heads a warp can straddle read disjoint banks.
__host__ __device__ __forceinline__ int head_stride(int S, int hd) {
  const int n = S * hd;
  return n + ((16 - n % 32) + 32) % 32;
}
size_t fwd_smem(int S, int hd, int hg) {
  return sizeof(float) * (2ull * hg * head_stride(S, hd) + S);
}
// Floats between consecutive heads' [S][S|1] P / dS matrices (16 mod 32).
__host__ __device__ __forceinline__ int mat_stride(int S) {
  const int n = S * (S | 1);
  return n + ((16 - n % 32) + 32) % 32;
}
size_t bwd_smem(int S, int hd, int hg) {
  return sizeof(float) * (2ull * hg * head_stride(S, hd) + 2ull * hg * mat_stride(S) + S +
                          static_cast<size_t>(hg) * S);
}

template <int HD>
__device__ __forceinline__ float dot_row(const float (&q)[HD], const float *__restrict__ krow) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int c = 0; c < HD; c += 4) {
    const float4 k = *reinterpret_cast<const float4 *>(krow + c);
    a0 = fmaf(q[c], k.x, a0);
    a1 = fmaf(q[c + 1], k.y, a1);
    a2 = fmaf(q[c + 2], k.z, a2);
    a3 = fmaf(q[c + 3], k.w, a3);
  }
  return (a0 + a1) + (a2 + a3);
}

template <int HD>
__device__ __forceinline__ void axpy_row(float (&o)[HD], float p, const float *__restrict__ vrow) {
#pragma unroll
  for (int c = 0; c < HD; c += 4) {
    const float4 v = *reinterpret_cast<const float4 *>(vrow + c);
    o[c] = fmaf(p, v.x, o[c]);
    o[c + 1] = fmaf(p, v.y, o[c + 1]);
    o[c + 2] = fmaf(p, v.z, o[c + 2]);
    o[c + 3] = fmaf(p, v.w, o[c + 3]);
  }
}

// Cooperative asynchronous 16-byte copies (cp.async) of the (token,
// head-group) block of one of q/k/v (column offset `col`) or of a [T, d]
// array into smem laid out [HG][S][HD]; every copy of the block is in flight
// at once.  The caller commits and waits (cp_async_wait_all) before use.
template <int HD>
__device__ __forceinline__ void load_block(float *dst, const float *src, int ld, int col, int t0, int S,
                                           int hg) {
  const int per_row = HD / 4, per_head = S * per_row, n = hg * per_head, hs = head_stride(S, HD);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int hh = i / per_head, rem = i - hh * per_head, k = rem / per_row, c = (rem - k * per_row) * 4;
    const uint32_t d32 = static_cast<uint32_t>(__cvta_generic_to_shared(dst + hh * hs + k * HD + c));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d32),
                 "l"(src + static_cast<size_t>(t0 + k) * ld + col + hh * HD + c)
                 : "memory");
  }
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

template <int HD>
__global__ void k_attn_fwd(AttnArgs a, int hg) {
  extern __shared__ __align__(16) float sm[];
  const int atom = blockIdx.x, h0 = blockIdx.y * hg;
  const int e0 = a.offset[atom];
  const int S = a.offset[atom + 1] - e0 + 1;
  const int t0 = e0 + atom;
  const int d = a.d, ld = 3 * d;
  const int hs = head_stride(S, HD);
  float *sK = sm, *sV = sK + hg * hs, *sM = sV + hg * hs;
  load_block<HD>(sK, a.qkv, ld, d + h0 * HD, t0, S, hg);
  load_block<HD>(sV, a.qkv, ld, 2 * d + h0 * HD, t0, S, hg);
  for (int k = threadIdx.x; k < S; k += blockDim.x) sM[k] = k == 0 ? 0.f : a.key_mask[e0 + k - 1];
  cp_async_wait_all();
  __syncthreads();
  const int t = threadIdx.x;
  if (t >= hg * S) return;
  const int hh = t / S, q = t - hh * S, h = h0 + hh;
  float qr[HD], o[HD];
  const float *qsrc = a.qkv + static_cast<size_t>(t0 + q) * ld + h * HD;
#pragma unroll
  for (int c = 0; c < HD; c += 4) {
    const float4 v = *reinterpret_cast<const float4 *>(qsrc + c);
    qr[c] = v.x; qr[c + 1] = v.y; qr[c + 2] = v.z; qr[c + 3] = v.w;
    o[c] = o[c + 1] = o[c + 2] = o[c + 3] = 0.f;
  }
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  const float *K = sK + hh * hs, *V = sV + hh * hs;
  float m = -FLT_MAX, l = 0.f;
  for (int k = 0; k < S; ++k) {
    const float s = dot_row<HD>(qr, K + k * HD) * scale + sM[k];
    if (s > m) {
      const float corr = expf(m - s);
      l *= corr;
#pragma unroll
      for (int c = 0; c < HD; ++c) o[c] *= corr;
      m = s;
    }
    const float p = expf(s - m);
    l += p;
    axpy_row<HD>(o, p, V + k * HD);
  }
  const float inv = 1.0f / l;
  float *dst = a.out + static_cast<size_t>(t0 + q) * d + h * HD;
#pragma unroll
  for (int c = 0; c < HD; c += 4)
    *reinterpret_cast<float4 *>(dst + c) = make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
  a.lse[static_cast<size_t>(t0 + q) * a.heads + h] = m + logf(l);
}

// dS = P (dP - rowsum(P dP)), dQ = s dS K, dK = s dS^T Q, dV = P^T dO.
// The mask is a constant input in the reference (pet.cpp:274-275): no grad.
// Phase A (thread = query row) needs K and V in shared memory and its own q
// and dO rows in registers; phase B (thread = key row) needs Q and dO.  The
// two phases share one [2][HG][S][HD] region (K, V then Q, dO), so a CTA
// holds two row blocks and the P / dS matrices.
template <int HD>
__global__ void k_attn_bwd(AttnArgs a, int hg) {
  extern __shared__ __align__(16) float sm[];
  const int atom = blockIdx.x, h0 = blockIdx.y * hg;
  const int e0 = a.offset[atom];
  const int S = a.offset[atom + 1] - e0 + 1;
  const int t0 = e0 + atom;
  const int d = a.d, ld = 3 * d;
  const int PS = S | 1;
  const int hs = head_stride(S, HD), ms = mat_stride(S);
  float *sA = sm, *sB = sA + hg * hs;  // K, V (phase A) then Q, dO (phase B)
  float *sP = sB + hg * hs, *sD = sP + hg * ms, *sM = sD + hg * ms, *sL = sM + S;
  load_block<HD>(sA, a.qkv, ld, d + h0 * HD, t0, S, hg);
  load_block<HD>(sB, a.qkv, ld, 2 * d + h0 * HD, t0, S, hg);
  for (int k = threadIdx.x; k < S; k += blockDim.x) sM[k] = k == 0 ? 0.f : a.key_mask[e0 + k - 1];
  for (int i = threadIdx.x; i < hg * S; i += blockDim.x) {
    const int hh = i / S, q = i - hh * S;
    sL[i] = a.lse[static_cast<size_t>(t0 + q) * a.heads + h0 + hh];
  }
  const int t = threadIdx.x;
  const bool live = t < hg * S;
  const int hh = live ? t / S : 0, r = live ? t - hh * S : 0, h = h0 + hh;
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  float qr[HD], g[HD];
  if (live) {
    const float *qs = a.qkv + static_cast<size_t>(t0 + r) * ld + h * HD;
    const float *gs = a.d_out + static_cast<size_t>(t0 + r) * d + h * HD;
#pragma unroll
    for (int c = 0; c < HD; c += 4) {
      const float4 v = *reinterpret_cast<const float4 *>(qs + c);
      const float4 w = *reinterpret_cast<const float4 *>(gs + c);
      qr[c] = v.x; qr[c + 1] = v.y; qr[c + 2] = v.z; qr[c + 3] = v.w;
      g[c] = w.x; g[c + 1] = w.y; g[c + 2] = w.z; g[c + 3] = w.w;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  float *P = sP + hh * ms, *Dm = sD + hh * ms;
  if (live) {
    // phase A: thread = query row r
    const float *K = sA + hh * hs, *V = sB + hh * hs;
    float acc[HD];
#pragma unroll
    for (int c = 0; c < HD; ++c) acc[c] = 0.f;
    const float lse = sL[hh * S + r];
    float D = 0.f;
#pragma unroll 2
    for (int k = 0; k < S; ++k) {
      const float p = expf(dot_row<HD>(qr, K + k * HD) * scale + sM[k] - lse);
      const float dp = dot_row<HD>(g, V + k * HD);
      P[r * PS + k] = p;
      Dm[r * PS + k] = dp;
      D = fmaf(p, dp, D);
    }
#pragma unroll 2
    for (int k = 0; k < S; ++k) {
      const float ds = P[r * PS + k] * (Dm[r * PS + k] - D);
      Dm[r * PS + k] = ds;
      axpy_row<HD>(acc, ds, K + k * HD);
    }
    float *dq = a.d_qkv + static_cast<size_t>(t0 + r) * ld + h * HD;
#pragma unroll
    for (int c = 0; c < HD; c += 4)
      *reinterpret_cast<float4 *>(dq + c) =
          make_float4(acc[c] * scale, acc[c + 1] * scale, acc[c + 2] * scale, acc[c + 3] * scale);
  }
  __syncthreads();  // K and V no longer read: bring in Q and dO
  load_block<HD>(sA, a.qkv, ld, h0 * HD, t0, S, hg);
  load_block<HD>(sB, a.d_out, d, h0 * HD, t0, S, hg);
  cp_async_wait_all();
  __syncthreads();
  if (live) {
    // phase B: thread = key row r
    const float *Q = sA + hh * hs, *G = sB + hh * hs;
    float dk[HD], dv[HD];
#pragma unroll
    for (int c = 0; c < HD; ++c) dk[c] = dv[c] = 0.f;
#pragma unroll 2
    for (int q = 0; q < S; ++q) {
      axpy_row<HD>(dk, Dm[q * PS + r], Q + q * HD);
      axpy_row<HD>(dv, P[q * PS + r], G + q * HD);
    }
    float *dst = a.d_qkv + static_cast<size_t>(t0 + r) * ld + h * HD;
#pragma unroll
    for (int c = 0; c < HD; c += 4) {
      *reinterpret_cast<float4 *>(dst + d + c) =
          make_float4(dk[c] * scale, dk[c + 1] * scale, dk[c + 2] * scale, dk[c + 3] * scale);
      *reinterpret_cast<float4 *>(dst + 2 * d + c) = make_float4(dv[c], dv[c + 1], dv[c + 2], dv[c + 3]);
    }
  }
}

// Heads per CTA: the largest of 4, 2, 1 that divides the head count, keeps
// HG * S threads <= 1024 and fits the shared-memory budget `limit`.
int pick_group(int heads, int S, int hd, bool bwd, size_t limit) {
  for (int hg = 4; hg >= 1; hg >>= 1) {
    if (heads % hg) continue;
    if (hg * S > 1024) continue;
    if ((bwd ? bwd_smem(S, hd, hg) : fwd_smem(S, hd, hg)) <= limit) return hg;
  }
  return 0;
}

template <int HD>
void run(const AttnArgs &a, bool bwd, cudaStream_t s) {
  const int S = a.max_tokens;
  // prefer two CTAs per SM for the backward's large footprint
  int hg = pick_group(a.heads, S, HD, bwd, bwd ? kSmemLimit / 2 : kSmemLimit / 4);
  if (!hg) hg = pick_group(a.heads, S, HD, bwd, kSmemLimit);
  if (!hg) throw Error(kErrUnsupported, "attention: too many neighbours for one CTA");
  const size_t smem = bwd ? bwd_smem(S, HD, hg) : fwd_smem(S, HD, hg);
  const int threads = (hg * S + 31) / 32 * 32;
  dim3 grid(a.n_atoms, a.heads / hg);
  if (bwd) {
    CUDA_CHECK(cudaFuncSetAttribute(k_attn_bwd<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    k_attn_bwd<HD><<<grid, threads, smem, s>>>(a, hg);
  } else {
    CUDA_CHECK(cudaFuncSetAttribute(k_attn_fwd<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    k_attn_fwd<HD><<<grid, threads, smem, s>>>(a, hg);
  }
  CUDA_LAUNCH_CHECK();
}

void dispatch(const AttnArgs &a, bool bwd, cudaStream_t s) {
  if (a.n_atoms <= 0) return;
  const int hd = a.d / a.heads;
  if (a.max_tokens > attention_max_tokens(hd))
    throw Error(kErrUnsupported, "attention: " + std::to_string(a.max_tokens - 1) +
                                     " neighbours exceed the per-atom limit");
  switch (hd) {
    case 16: run<16>(a, bwd, s); break;
    case 32: run<32>(a, bwd, s); break;
    case 64: run<64>(a, bwd, s); break;
    default: throw Error(kErrUnsupported, "attention: head size " + std::to_string(hd));
  }
}

}  // namespace

int attention_max_tokens(int hd) {
  int S = 1;
  while (pick_group(1, S + 1, hd, true, kSmemLimit) && pick_group(1, S + 1, hd, false, kSmemLimit)) ++S;
  return S;
}

void attention_fwd(const AttnArgs &a, cudaStream_t s) { dispatch(a, false, s); }
void attention_bwd(const AttnArgs &a, cudaStream_t s) { dispatch(a, true, s); }

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
