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
#include "split16.cuh"

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
  return sizeof(float) * (2ull * hg * head_stride(S, hd) + S + static_cast<size_t>(hg) * S);
}
// Floats between consecutive heads' [S][S|1] P / dS matrices (16 mod 32).
__host__ __device__ __forceinline__ int mat_stride(int S) {
  const int n = S * (S | 1);
  return n + ((16 - n % 32) + 32) % 32;
}
// [2][HG] row blocks, P and dS, key mask [S], log-sum-exp [HG][S] and the
// three [HG][S] arrays of the split outputs' block maxima
size_t bwd_smem(int S, int hd, int hg) {
  return sizeof(float) * (2ull * hg * head_stride(S, hd) + 2ull * hg * mat_stride(S) + S +
                          4ull * hg * S);
}

// Split-fp16 output of a (row, head-group) block: each of the HG threads of
// `row` holds its head's HD values; `mx` (smem, [HG][S]) has been filled with
// every thread's max |value| and synchronised.  Writes the block's split form.
template <int HD>
__device__ __forceinline__ void group_split_store(const Split16View &o, int row, int col, int blk, const float *mx,
                                                  int hg, int S, int r, int hh, float (&v)[HD]) {
  float m = 0.f;
  for (int k = 0; k < hg; ++k) m = fmaxf(m, mx[k * S + r]);
  const int s = split_scale_exponent(m);
  thread_split_store<HD>(o, row, col, v, s);
  if (hh == 0) o.sc[static_cast<size_t>(blk) * split_ld(o) + row] = static_cast<int8_t>(s);
}

template <int HD>
__device__ __forceinline__ float absmax(const float (&v)[HD]) {
  float m = 0.f;
#pragma unroll
  for (int c = 0; c < HD; ++c) m = fmaxf(m, fabsf(v[c]));
  return m;
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
__device__ __forceinline__ void load_block(float *dst, const float *src, int ld, int col, AtomRows tr, int S,
                                           int hg) {
  const int per_row = HD / 4, per_head = S * per_row, n = hg * per_head, hs = head_stride(S, HD);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int hh = i / per_head, rem = i - hh * per_head, k = rem / per_row, c = (rem - k * per_row) * 4;
    const uint32_t d32 = static_cast<uint32_t>(__cvta_generic_to_shared(dst + hh * hs + k * HD + c));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d32),
                 "l"(src + static_cast<size_t>(tr(k)) * ld + col + hh * HD + c)
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
  const AtomRows tr = atom_rows(atom, e0, a.edge_base);
  const int d = a.d, ld = 3 * d;
  const int hs = head_stride(S, HD);
  float *sK = sm, *sV = sK + hg * hs, *sM = sV + hg * hs, *sX = sM + S;
  load_block<HD>(sK, a.qkv, ld, d + h0 * HD, tr, S, hg);
  load_block<HD>(sV, a.qkv, ld, 2 * d + h0 * HD, tr, S, hg);
  for (int k = threadIdx.x; k < S; k += blockDim.x) sM[k] = k == 0 ? 0.f : a.key_mask[e0 + k - 1];
  cp_async_wait_all();
  __syncthreads();
  const int t = threadIdx.x;
  const bool live = t < hg * S;
  const int hh = live ? t / S : 0, q = live ? t - hh * S : 0, h = h0 + hh;
  float o[HD];
  if (live) {
    float qr[HD];
    const float *qsrc = a.qkv + static_cast<size_t>(tr(q)) * ld + h * HD;
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
#pragma unroll
    for (int c = 0; c < HD; ++c) o[c] *= inv;
    a.lse[static_cast<size_t>(tr(q)) * a.heads + h] = m + logf(l);
    if (a.out) {
      float *dst = a.out + static_cast<size_t>(tr(q)) * d + h * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 4) *reinterpret_cast<float4 *>(dst + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
    }
    if (a.out_split.hi) sX[hh * S + q] = absmax<HD>(o);
  }
  if (a.out_split.hi) {
    __syncthreads();
    if (live) group_split_store<HD>(a.out_split, tr(q), h * HD, blockIdx.y, sX, hg, S, q, hh, o);
  }
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
  const AtomRows tr = atom_rows(atom, e0, a.edge_base);
  const int d = a.d, ld = 3 * d;
  const int PS = S | 1;
  const int hs = head_stride(S, HD), ms = mat_stride(S);
  float *sA = sm, *sB = sA + hg * hs;  // K, V (phase A) then Q, dO (phase B)
  float *sP = sB + hg * hs, *sD = sP + hg * ms, *sM = sD + hg * ms, *sL = sM + S, *sX = sL + hg * S;
  load_block<HD>(sA, a.qkv, ld, d + h0 * HD, tr, S, hg);
  load_block<HD>(sB, a.qkv, ld, 2 * d + h0 * HD, tr, S, hg);
  for (int k = threadIdx.x; k < S; k += blockDim.x) sM[k] = k == 0 ? 0.f : a.key_mask[e0 + k - 1];
  for (int i = threadIdx.x; i < hg * S; i += blockDim.x) {
    const int hh = i / S, q = i - hh * S;
    sL[i] = a.lse[static_cast<size_t>(tr(q)) * a.heads + h0 + hh];
  }
  const int t = threadIdx.x;
  const bool live = t < hg * S;
  const int hh = live ? t / S : 0, r = live ? t - hh * S : 0, h = h0 + hh;
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  float qr[HD], g[HD];
  if (live) {
    const float *qs = a.qkv + static_cast<size_t>(tr(r)) * ld + h * HD;
    const float *gs = a.d_out + static_cast<size_t>(tr(r)) * d + h * HD;
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
  const bool split = a.dqkv_split.hi != nullptr;
  float acc[HD];
  if (live) {
    // phase A: thread = query row r
    const float *K = sA + hh * hs, *V = sB + hh * hs;
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
#pragma unroll
    for (int c = 0; c < HD; ++c) acc[c] *= scale;
    if (a.d_qkv) {
      float *dq = a.d_qkv + static_cast<size_t>(tr(r)) * ld + h * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 4)
        *reinterpret_cast<float4 *>(dq + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
    }
    if (split) sX[hh * S + r] = absmax<HD>(acc);
  }
  __syncthreads();  // K and V no longer read: bring in Q and dO
  if (split && live) group_split_store<HD>(a.dqkv_split, tr(r), h * HD, blockIdx.y, sX, hg, S, r, hh, acc);
  load_block<HD>(sA, a.qkv, ld, h0 * HD, tr, S, hg);
  load_block<HD>(sB, a.d_out, d, h0 * HD, tr, S, hg);
  cp_async_wait_all();
  __syncthreads();
  float dk[HD], dv[HD];
  if (live) {
    // phase B: thread = key row r
    const float *Q = sA + hh * hs, *G = sB + hh * hs;
#pragma unroll
    for (int c = 0; c < HD; ++c) dk[c] = dv[c] = 0.f;
#pragma unroll 2
    for (int q = 0; q < S; ++q) {
      axpy_row<HD>(dk, Dm[q * PS + r], Q + q * HD);
      axpy_row<HD>(dv, P[q * PS + r], G + q * HD);
    }
#pragma unroll
    for (int c = 0; c < HD; ++c) dk[c] *= scale;
    if (a.d_qkv) {
      float *dst = a.d_qkv + static_cast<size_t>(tr(r)) * ld + h * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 4) {
        *reinterpret_cast<float4 *>(dst + d + c) = make_float4(dk[c], dk[c + 1], dk[c + 2], dk[c + 3]);
        *reinterpret_cast<float4 *>(dst + 2 * d + c) = make_float4(dv[c], dv[c + 1], dv[c + 2], dv[c + 3]);
      }
    }
    if (split) {
      sX[hg * S + hh * S + r] = absmax<HD>(dk);
      sX[2 * hg * S + hh * S + r] = absmax<HD>(dv);
    }
  }
  if (split) {
    __syncthreads();
    if (live) {
      const int nbq = d / 128;
      group_split_store<HD>(a.dqkv_split, tr(r), d + h * HD, nbq + blockIdx.y, sX + hg * S, hg, S, r, hh, dk);
      group_split_store<HD>(a.dqkv_split, tr(r), 2 * d + h * HD, 2 * nbq + blockIdx.y, sX + 2 * hg * S, hg, S, r,
                            hh, dv);
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
  int hg = 0;
  if (bwd ? a.dqkv_split.hi != nullptr : a.out_split.hi != nullptr) {
    // split output: the CTA's heads form one 128-column block
    hg = 128 / HD;
    if (128 % HD || a.heads % hg || hg * S > 1024 ||
        (bwd ? bwd_smem(S, HD, hg) : fwd_smem(S, HD, hg)) > kSmemLimit)
      throw Error(kErrInternal, "attention: split output needs 128 / head size heads per CTA");
  } else {
    // prefer two CTAs per SM for the backward's large footprint
    hg = pick_group(a.heads, S, HD, bwd, bwd ? kSmemLimit / 2 : kSmemLimit / 4);
    if (!hg) hg = pick_group(a.heads, S, HD, bwd, kSmemLimit);
    if (!hg) throw Error(kErrUnsupported, "attention: too many neighbours for one CTA");
  }
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

int attention_split_max_tokens(int hd) {
  if (hd <= 0 || 128 % hd) return 0;
  const int hg = 128 / hd;
  int S = 0;
  while (hg * (S + 1) <= 1024 && bwd_smem(S + 1, hd, hg) <= kSmemLimit && fwd_smem(S + 1, hd, hg) <= kSmemLimit) ++S;
  return S;
}

void attention_fwd(const AttnArgs &a, cudaStream_t s) { dispatch(a, false, s); }
void attention_bwd(const AttnArgs &a, cudaStream_t s) { dispatch(a, true, s); }

// ---------------------------------------------------------------------------
// Layer norm (warp per row)
// ---------------------------------------------------------------------------
namespace {

constexpr float kLnEps = 1e-5f;

// stats: the row's mean at stats[row], 1 / sd at stats[rows + row]; the
// backward recomputes xhat = (x - mean) / sd from x and these.
__global__ void k_ln_fwd(const float *__restrict__ x, const float *__restrict__ g,
                         const float *__restrict__ b, float *__restrict__ y,
                         float *__restrict__ stats, int rows, int d) {
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
  const float r = 1.0f / sqrtf(var * (1.0f + kLnEps));
  float *yr = y + static_cast<size_t>(row) * d;
  for (int c = lane; c < d; c += 32) yr[c] = (xr[c] - mean) * r * g[c] + b[c];
  if (lane == 0) {
    stats[row] = mean;
    stats[rows + row] = r;
  }
}

__global__ void k_ln_bwd(const float *__restrict__ dy, const float *__restrict__ x,
                         const float *__restrict__ stats, const float *__restrict__ g,
                         float *__restrict__ dx, int rows, int d) {
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float *dyr = dy + static_cast<size_t>(row) * d;
  const float *xr = x + static_cast<size_t>(row) * d;
  const float mean = stats[row], r = stats[rows + row];
  float s1 = 0.f, s2 = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float gh = dyr[c] * g[c];
    s1 += gh;
    s2 = fmaf(gh, (xr[c] - mean) * r, s2);
  }
  const float inv_d = 1.0f / static_cast<float>(d);
  const float m1 = warp_sum(s1) * inv_d;
  const float m2 = warp_sum(s2) * inv_d * (1.0f + kLnEps);
  float *dxr = dx + static_cast<size_t>(row) * d;
  for (int c = lane; c < d; c += 32) dxr[c] = r * (dyr[c] * g[c] - m1 - (xr[c] - mean) * r * m2);
}

// Rows of d = 128 nb columns: lane l holds float4 columns 128 b + 4 l, so
// each 128-column block of the output is one warp-wide split block.
template <int NB>
__global__ void k_ln_fwd4(const float *__restrict__ x, const float *__restrict__ g,
                          const float *__restrict__ b, float *__restrict__ y,
                          float *__restrict__ stats, int rows, Split16View ys) {
  constexpr int d = 128 * NB;
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float *xr = x + static_cast<size_t>(row) * d;
  float4 v[NB];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    v[k] = *reinterpret_cast<const float4 *>(xr + 128 * k + 4 * lane);
    s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  }
  const float inv_d = 1.0f / static_cast<float>(d);
  const float mean = warp_sum(s) * inv_d;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const float t0 = v[k].x - mean, t1 = v[k].y - mean, t2 = v[k].z - mean, t3 = v[k].w - mean;
    q = fmaf(t0, t0, q); q = fmaf(t1, t1, q); q = fmaf(t2, t2, q); q = fmaf(t3, t3, q);
  }
  const float var = warp_sum(q) * inv_d;
  const float r = 1.0f / sqrtf(var * (1.0f + kLnEps));
  float *yr = y ? y + static_cast<size_t>(row) * d : nullptr;  // y null: split output only
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const int c = 128 * k + 4 * lane;
    const float4 gg = __ldg(reinterpret_cast<const float4 *>(g + c));
    const float4 bb = __ldg(reinterpret_cast<const float4 *>(b + c));
    const float4 h = make_float4((v[k].x - mean) * r, (v[k].y - mean) * r, (v[k].z - mean) * r,
                                 (v[k].w - mean) * r);
    const float4 o = make_float4(h.x * gg.x + bb.x, h.y * gg.y + bb.y, h.z * gg.z + bb.z, h.w * gg.w + bb.w);
    if (yr) *reinterpret_cast<float4 *>(yr + c) = o;
    if (ys.hi) warp_split_block(ys, row, k, o, lane);
  }
  if (lane == 0) {
    stats[row] = mean;
    stats[rows + row] = r;
  }
}

template <int NB>
__global__ void k_ln_bwd4(const float *__restrict__ dy, const float *__restrict__ x,
                          const float *__restrict__ stats, const float *__restrict__ g,
                          float *__restrict__ dx, int rows, Split16View dxs) {
  constexpr int d = 128 * NB;
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float *dyr = dy + static_cast<size_t>(row) * d;
  const float *xr = x + static_cast<size_t>(row) * d;
  const float mean = stats[row], r = stats[rows + row];
  float4 gh[NB], hh[NB];
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const int c = 128 * k + 4 * lane;
    const float4 a = *reinterpret_cast<const float4 *>(dyr + c);
    const float4 gg = __ldg(reinterpret_cast<const float4 *>(g + c));
    const float4 xv = *reinterpret_cast<const float4 *>(xr + c);
    hh[k] = make_float4((xv.x - mean) * r, (xv.y - mean) * r, (xv.z - mean) * r, (xv.w - mean) * r);
    gh[k] = make_float4(a.x * gg.x, a.y * gg.y, a.z * gg.z, a.w * gg.w);
    s1 += (gh[k].x + gh[k].y) + (gh[k].z + gh[k].w);
    s2 = fmaf(gh[k].x, hh[k].x, s2); s2 = fmaf(gh[k].y, hh[k].y, s2);
    s2 = fmaf(gh[k].z, hh[k].z, s2); s2 = fmaf(gh[k].w, hh[k].w, s2);
  }
  const float inv_d = 1.0f / static_cast<float>(d);
  const float m1 = warp_sum(s1) * inv_d;
  const float m2 = warp_sum(s2) * inv_d * (1.0f + kLnEps);
  float *dxr = dx ? dx + static_cast<size_t>(row) * d : nullptr;  // dx null: split output only
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const int c = 128 * k + 4 * lane;
    const float4 o = make_float4(r * (gh[k].x - m1 - hh[k].x * m2), r * (gh[k].y - m1 - hh[k].y * m2),
                                 r * (gh[k].z - m1 - hh[k].z * m2), r * (gh[k].w - m1 - hh[k].w * m2));
    if (dxr) *reinterpret_cast<float4 *>(dxr + c) = o;
    if (dxs.hi) warp_split_block(dxs, row, k, o, lane);
  }
}

}  // namespace

void layer_norm_fwd(const float *x, const float *g, const float *b, float *y, float *stats, int rows, int d,
                    cudaStream_t s, const Split16View *ys) {
  if (rows <= 0) return;
  const int grid = ceil_div(static_cast<int64_t>(rows) * 32, 256);
  const Split16View none{};
  const Split16View &o = ys ? *ys : none;
  switch (d % 128 == 0 ? d / 128 : 0) {
    case 1: k_ln_fwd4<1><<<grid, 256, 0, s>>>(x, g, b, y, stats, rows, o); break;
    case 2: k_ln_fwd4<2><<<grid, 256, 0, s>>>(x, g, b, y, stats, rows, o); break;
    case 4: k_ln_fwd4<4><<<grid, 256, 0, s>>>(x, g, b, y, stats, rows, o); break;
    case 8: k_ln_fwd4<8><<<grid, 256, 0, s>>>(x, g, b, y, stats, rows, o); break;
    default:
      if (ys) throw Error(kErrInternal, "layer_norm_fwd: split output needs d in {128, 256, 512, 1024}");
      k_ln_fwd<<<grid, 256, 0, s>>>(x, g, b, y, stats, rows, d);
  }
  CUDA_LAUNCH_CHECK();
}

void layer_norm_bwd(const float *dy, const float *x, const float *stats, const float *g, float *dx, int rows, int d,
                    cudaStream_t s, const Split16View *dxs) {
  if (rows <= 0) return;
  const int grid = ceil_div(static_cast<int64_t>(rows) * 32, 256);
  const Split16View none{};
  const Split16View &o = dxs ? *dxs : none;
  switch (d % 128 == 0 ? d / 128 : 0) {
    case 1: k_ln_bwd4<1><<<grid, 256, 0, s>>>(dy, x, stats, g, dx, rows, o); break;
    case 2: k_ln_bwd4<2><<<grid, 256, 0, s>>>(dy, x, stats, g, dx, rows, o); break;
    case 4: k_ln_bwd4<4><<<grid, 256, 0, s>>>(dy, x, stats, g, dx, rows, o); break;
    case 8: k_ln_bwd4<8><<<grid, 256, 0, s>>>(dy, x, stats, g, dx, rows, o); break;
    default:
      if (dxs) throw Error(kErrInternal, "layer_norm_bwd: split output needs d in {128, 256, 512, 1024}");
      k_ln_bwd<<<grid, 256, 0, s>>>(dy, x, stats, g, dx, rows, d);
  }
  CUDA_LAUNCH_CHECK();
}

}  // namespace pet
