// Per-edge / per-atom kernels of the PET pass.  All are HBM- or
// latency-bound elementwise work; grids are grid-stride over edges or atoms.
#include <cuda_fp16.h>

#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "ops.cuh"
#include "split16.cuh"

namespace pet {
namespace {

constexpr float kPi = 3.14159265358979323846f;

int grid_for(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  if (g < 1) g = 1;
  if (g > 148 * 64) g = 148 * 64;
  return static_cast<int>(g);
}

__global__ void k_edge_prep(EdgePrepArgs a) {
  const float inv_delta = 1.0f / a.width;
  const float off = (a.width - a.cutoff) * inv_delta;
  const int total = a.n_edges > a.n_atoms ? a.n_edges : a.n_atoms;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    if (e >= a.n_edges) continue;
    const int i = a.center[e], j = a.nbr[e];
    const float x = a.vec[3 * e], y = a.vec[3 * e + 1], z = a.vec[3 * e + 2];
    // in-graph distance and cutoff (pet.cpp:208-256)
    const float r = sqrtf(x * x + y * y + z * z);
    const float xx = r * inv_delta + off;
    const float xc = fminf(fmaxf(xx, 0.0f), 1.0f);
    a.r[e] = r;
    a.fc[e] = cosf(xc * kPi) * 0.5f + 0.5f;
    a.dfc_dr[e] = (xx > 0.0f && xx < 1.0f) ? -0.5f * sinf(xc * kPi) * kPi * inv_delta : 0.0f;
    // attention key mask: fp16(log(smooth_cutoff(d_nl))) (pet_batch.cpp:37-47, 628-638);
    // cos/log evaluated in f64 and rounded once, i.e. correctly rounded f32.
    const float dn = a.dist_nl[e];
    float fcm;
    if (dn >= a.cutoff) fcm = 0.0f;
    else if (dn <= a.cutoff - a.width) fcm = 1.0f;
    else {
      const float xm = (dn - a.cutoff + a.width) / a.width;
      fcm = 0.5f + 0.5f * static_cast<float>(cos(static_cast<double>(kPi * xm)));
    }
    a.key_mask[e] = fcm > 0.0f
        ? __half2float(__float2half_rn(static_cast<float>(log(static_cast<double>(fcm)))))
        : -INFINITY;
    a.nbr_species[e] = a.species[j];
    // reverse edge (j -> i, -S); the reference's hash map keeps the last edge
    // inserted under a key, so the last match wins (pet_batch.cpp:416-436)
    const int s0 = a.shift[3 * e], s1 = a.shift[3 * e + 1], s2 = a.shift[3 * e + 2];
    int rv = -1;
    const int kb = j < a.n_atoms ? a.offset[j] : 0, kend = j < a.n_atoms ? a.offset[j + 1] : 0;
    for (int k = kb, ke = kend; k < ke; ++k) {
      if (a.nbr[k] == i && a.shift[3 * k] == -s0 && a.shift[3 * k + 1] == -s1 &&
          a.shift[3 * k + 2] == -s2)
        rv = k;
    }
    a.rev[e] = rv;
  }
}

// Column j of the auxiliary block: x, y, z, r, 1, one-hot(species), zeros.
__device__ __forceinline__ float aux_value(int j, float x, float y, float z, float r, int sp) {
  return j == 0 ? x : j == 1 ? y : j == 2 ? z : j == 3 ? r : j == 4 ? 1.0f : (j - 5 == sp ? 1.0f : 0.0f);
}

// Row of x_prev whose token enters edge e's layer-1 message, or -1.
__device__ __forceinline__ int message_row(const FeaturizeArgs &a, int e) {
  const int m = a.msg_row ? a.msg_row[e] : -1;
  if (m >= 0) return m;
  const int rv = a.rev[e];
  return rv >= 0 ? a.prev_base + rv : -1;
}

__device__ __forceinline__ float feat_value(const FeaturizeArgs &a, int e, int c) {
  const int d = a.d;
  const int sp = a.nbr_species[e];
  if (a.layer > 0) {
    if (c < d) {
      const int row = message_row(a, e);
      const float m0 = a.emb0[static_cast<size_t>(sp) * d + c];
      const float mr = row >= 0 ? a.x_prev[static_cast<size_t>(row) * d + c] : 0.0f;
      return 0.5f * (m0 + mr);
    }
    c -= d;
  }
  return aux_value(c, a.vec[3 * e], a.vec[3 * e + 1], a.vec[3 * e + 2], a.r[e], sp);
}

__global__ void k_featurize(FeaturizeArgs a) {
  const int K = featurize_cols(a.layer, a.d, a.aux);
  const int64_t total = static_cast<int64_t>(a.n_edges) * K;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(t / K), c = static_cast<int>(t % K);
    a.cat[t] = feat_value(a, e, c);
  }
}

// Split-fp16 output: warp per edge, lane l holds columns 4l..4l+3 of each
// 128-column block (d and aux multiples of 128, so a block lies in one part).
__global__ void k_featurize_split(FeaturizeArgs a) {
  const int d = a.d, nbd = a.layer > 0 ? d / 128 : 0;
  const int e = static_cast<int>((blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (e >= a.n_edges) return;
  const int sp = a.nbr_species[e];
  if (a.layer > 0) {  // message: 0.5 (embedding[nbr species] + X0[row(reverse edge)])
    const int row = message_row(a, e);
    const float *m0 = a.emb0 + static_cast<size_t>(sp) * d;
    const float *mr = row >= 0 ? a.x_prev + static_cast<size_t>(row) * d : nullptr;
    for (int k = 0; k < nbd; ++k) {
      const int c = k * 128 + lane * 4;
      const float4 p = __ldg(reinterpret_cast<const float4 *>(m0 + c));
      const float4 q = mr ? *reinterpret_cast<const float4 *>(mr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      warp_split_block(a.cat_split, e, k,
                       make_float4(0.5f * (p.x + q.x), 0.5f * (p.y + q.y), 0.5f * (p.z + q.z), 0.5f * (p.w + q.w)),
                       lane);
    }
  }
  const float x = a.vec[3 * e], y = a.vec[3 * e + 1], z = a.vec[3 * e + 2], r = a.r[e];
  for (int k = 0; k < a.aux / 128; ++k) {
    const int c = k * 128 + lane * 4;
    warp_split_block(a.cat_split, e, nbd + k,
                     make_float4(aux_value(c, x, y, z, r, sp), aux_value(c + 1, x, y, z, r, sp),
                                 aux_value(c + 2, x, y, z, r, sp), aux_value(c + 3, x, y, z, r, sp)),
                     lane);
  }
}

__global__ void k_node_tokens(const float *__restrict__ tab, const int *__restrict__ sp, float *__restrict__ x,
                              int n, int d) {
  const int64_t total = static_cast<int64_t>(n) * d;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(t / d), c = static_cast<int>(t % d);
    x[static_cast<size_t>(i) * d + c] = tab[static_cast<size_t>(sp[i]) * d + c];
  }
}

// Node tokens with the split-fp16 form of the same rows: warp per (atom, block).
__global__ void k_node_tokens_split(const float *__restrict__ tab, const int *__restrict__ sp,
                                    float *__restrict__ x, int n, int d, Split16View xs) {
  const int nb = d / 128;
  const int64_t w = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(n) * nb) return;
  const int i = static_cast<int>(w / nb), blk = static_cast<int>(w % nb);
  const int c = blk * 128 + lane * 4, row = i;
  const float4 v = *reinterpret_cast<const float4 *>(tab + static_cast<size_t>(sp[i]) * d + c);
  if (x) *reinterpret_cast<float4 *>(x + static_cast<size_t>(row) * d + c) = v;  // x null: split only
  warp_split_block(xs, row, blk, v, lane);
}

__global__ void k_head_last(const float *__restrict__ y, const float *__restrict__ w,
                            const float *__restrict__ b, float *__restrict__ pred, int rows, int r) {
  const int lane = threadIdx.x & 31;
  for (int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < rows;
       m += (gridDim.x * blockDim.x) >> 5) {
    const float *yr = y + static_cast<size_t>(m) * r;
    float s = 0.f;
    for (int c = lane; c < r; c += 32) s = fmaf(yr[c], w[c], s);
    s = warp_sum(s);
    if (lane == 0) pred[m] = s + b[0];
  }
}

__global__ void k_head_last_bwd(const float *__restrict__ z, const float *__restrict__ w,
                                const float *__restrict__ scale, float *__restrict__ dz, int rows, int r) {
  const int64_t total = static_cast<int64_t>(rows) * r;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(t / r), c = static_cast<int>(t % r);
    const float sc = scale ? scale[m] : 1.0f;
    dz[t] = w[c] * z[t] * sc;  // z holds silu' from the forward
  }
}

// dz in split-fp16 form only: warp per (row, 128-column block).
__global__ void k_head_last_bwd_split(const float *__restrict__ z, const float *__restrict__ w,
                                      const float *__restrict__ scale, int rows, int r, Split16View dzs) {
  const int nb = r / 128;
  const int64_t wi = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wi >= static_cast<int64_t>(rows) * nb) return;
  const int m = static_cast<int>(wi / nb), blk = static_cast<int>(wi % nb);
  const int c = blk * 128 + lane * 4;
  const float sc = scale ? scale[m] : 1.0f;
  const float4 zz = *reinterpret_cast<const float4 *>(z + static_cast<size_t>(m) * r + c);
  const float4 ww = *reinterpret_cast<const float4 *>(w + c);
  warp_split_block(dzs, m, blk, make_float4(ww.x * zz.x * sc, ww.y * zz.y * sc, ww.z * zz.z * sc, ww.w * zz.w * sc),
                   lane);
}

__global__ void k_atom_energy(const float *__restrict__ np, const float *__restrict__ ep,
                              const float *__restrict__ fc, const int *__restrict__ offset,
                              float *__restrict__ e_atom, int n, int accumulate) {
  const int lane = threadIdx.x & 31;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n;
       i += (gridDim.x * blockDim.x) >> 5) {
    float s = 0.f;
    for (int e = offset[i] + lane; e < offset[i + 1]; e += 32) s = fmaf(ep[e], fc[e], s);
    s = warp_sum(s);
    if (lane == 0) e_atom[i] = (accumulate ? e_atom[i] : 0.0f) + np[i] + s;
  }
}

__global__ void k_add_vec(const float *__restrict__ x, float *__restrict__ y, int n, int accumulate) {
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x)
    y[t] = accumulate ? y[t] + x[t] : x[t];
}

// Split input: lane l owns columns 4l..4l+3 of every 128-column block for
// all the edges it visits, so its H/32 rows of P stay in registers; a warp
// takes U edges per iteration and issues all their loads before the
// arithmetic, so U edges' memory latency overlaps.
template <int NB>
__global__ void k_edge_xyzr_bwd_split(Split16View dzs, const float *__restrict__ P, float *__restrict__ g4,
                                      int n_edges, int accumulate) {
  constexpr int H = 128 * NB, U = NB <= 4 ? 2 : 1;
  const int lane = threadIdx.x & 31;
  float4 w[NB][4];
#pragma unroll
  for (int k = 0; k < NB; ++k)
#pragma unroll
    for (int q = 0; q < 4; ++q) w[k][q] = __ldg(reinterpret_cast<const float4 *>(P + 4 * (128 * k + 4 * lane + q)));
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int e0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; e0 < n_edges; e0 += U * warps) {
    uint2 hv[U][NB], lv[U][NB];
    int8_t sv[U][NB];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * warps;
#pragma unroll
      for (int k = 0; k < NB; ++k) {
        if (e < n_edges) {
          const size_t off = static_cast<size_t>(e) * H + 128 * k + 4 * lane;
          hv[u][k] = *reinterpret_cast<const uint2 *>(dzs.hi + off);
          lv[u][k] = *reinterpret_cast<const uint2 *>(dzs.lo + off);
          sv[u][k] = dzs.sc[static_cast<size_t>(k) * split_ld(dzs) + e];
        } else {
          hv[u][k] = lv[u][k] = make_uint2(0u, 0u);
          sv[u][k] = 0;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * warps;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int k = 0; k < NB; ++k) {
        const float f = pow2f(-static_cast<int>(sv[u][k]));
        const float2 h0 = __half22float2(*reinterpret_cast<const __half2 *>(&hv[u][k].x));
        const float2 h1 = __half22float2(*reinterpret_cast<const __half2 *>(&hv[u][k].y));
        const float2 l0 = __half22float2(*reinterpret_cast<const __half2 *>(&lv[u][k].x));
        const float2 l1 = __half22float2(*reinterpret_cast<const __half2 *>(&lv[u][k].y));
        const float g[4] = {(h0.x + l0.x) * f, (h0.y + l0.y) * f, (h1.x + l1.x) * f, (h1.y + l1.y) * f};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          s0 = fmaf(g[q], w[k][q].x, s0);
          s1 = fmaf(g[q], w[k][q].y, s1);
          s2 = fmaf(g[q], w[k][q].z, s2);
          s3 = fmaf(g[q], w[k][q].w, s3);
        }
      }
      s0 = warp_sum(s0);
      s1 = warp_sum(s1);
      s2 = warp_sum(s2);
      s3 = warp_sum(s3);
      if (lane == 0 && e < n_edges) {
        float4 *o = reinterpret_cast<float4 *>(g4) + e;
        float4 v = make_float4(s0, s1, s2, s3);
        if (accumulate) {
          const float4 p = *o;
          v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
        }
        *o = v;
      }
    }
  }
}

__global__ void k_edge_xyzr_bwd(const float *__restrict__ dz, const float *__restrict__ P, float *__restrict__ g4,
                                int n_edges, int H, int accumulate) {
  const int lane = threadIdx.x & 31;
  for (int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; e < n_edges; e += (gridDim.x * blockDim.x) >> 5) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    const float *gr = dz + static_cast<size_t>(e) * H;
    for (int o = lane; o < H; o += 32) {
      const float g = gr[o];
      const float4 w = __ldg(reinterpret_cast<const float4 *>(P + 4 * o));
      s0 = fmaf(g, w.x, s0);
      s1 = fmaf(g, w.y, s1);
      s2 = fmaf(g, w.z, s2);
      s3 = fmaf(g, w.w, s3);
    }
    s0 = warp_sum(s0);
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    s3 = warp_sum(s3);
    if (lane == 0) {
      float4 *o = reinterpret_cast<float4 *>(g4) + e;
      float4 v = make_float4(s0, s1, s2, s3);
      if (accumulate) {
        const float4 p = *o;
        v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
      }
      *o = v;
    }
  }
}

// Warp per edge, 16-byte accesses along the row (d, ld multiples of 4).
__global__ void k_message_bwd(const float *__restrict__ dmsg, int ld, const int *__restrict__ rev, int base,
                              float *__restrict__ dx, int n_edges,
                              int n_msg, int d) {
  const int lane = threadIdx.x & 31;
  for (int x = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; x < n_edges; x += (gridDim.x * blockDim.x) >> 5) {
    const int rv = rev[x];
    if (rv < 0 || rv >= n_msg) continue;
    const float4 *src = reinterpret_cast<const float4 *>(dmsg + static_cast<size_t>(rv) * ld);
    float4 *dst = reinterpret_cast<float4 *>(dx + static_cast<size_t>(base + x) * d);
    for (int c = lane; c < d / 4; c += 32) {
      const float4 m = src[c];
      float4 v = dst[c];
      v.x = fmaf(0.5f, m.x, v.x);
      v.y = fmaf(0.5f, m.y, v.y);
      v.z = fmaf(0.5f, m.z, v.z);
      v.w = fmaf(0.5f, m.w, v.w);
      dst[c] = v;
    }
  }
}

__global__ void k_edge_grad(const float *__restrict__ g4, const float *__restrict__ gfc,
                            const float *__restrict__ dfc_dr, const float *__restrict__ vec,
                            const float *__restrict__ r, float *__restrict__ g, int n_edges) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_edges; e += gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4 *>(g4)[e];
    const float gr = (a.w + gfc[e] * dfc_dr[e]) / r[e];
    g[3 * e] = a.x + gr * vec[3 * e];
    g[3 * e + 1] = a.y + gr * vec[3 * e + 1];
    g[3 * e + 2] = a.z + gr * vec[3 * e + 2];
  }
}

__global__ void k_forces(const float *__restrict__ g, const int *__restrict__ offset,
                         const int *__restrict__ rev, float *__restrict__ F, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float fx = 0.f, fy = 0.f, fz = 0.f;
    for (int e = offset[i]; e < offset[i + 1]; ++e) {
      fx += g[3 * e];
      fy += g[3 * e + 1];
      fz += g[3 * e + 2];
      const int rv = rev[e];
      if (rv >= 0) {
        fx -= g[3 * rv];
        fy -= g[3 * rv + 1];
        fz -= g[3 * rv + 2];
      }
    }
    F[3 * i] = fx;
    F[3 * i + 1] = fy;
    F[3 * i + 2] = fz;
  }
}

// Edges whose reverse is missing (a pair that only one side sees at the
// cutoff) still push -g onto their neighbour.
__global__ void k_forces_unpaired(const float *__restrict__ g, const int *__restrict__ nbr,
                                  const int *__restrict__ rev, float *__restrict__ F, int n_edges) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_edges; e += gridDim.x * blockDim.x) {
    if (rev[e] >= 0) continue;
    const int j = nbr[e];
    atomicAdd(F + 3 * j, -g[3 * e]);
    atomicAdd(F + 3 * j + 1, -g[3 * e + 1]);
    atomicAdd(F + 3 * j + 2, -g[3 * e + 2]);
  }
}

template <int NV>
__device__ void block_sum(double (&v)[NV], double *sm) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = warp_sum_d(v[k]);
  if (lane == 0)
    for (int k = 0; k < NV; ++k) sm[w * NV + k] = v[k];
  __syncthreads();
  if (w == 0) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      double t = lane < nw ? sm[lane * NV + k] : 0.0;
      v[k] = warp_sum_d(t);
    }
  }
}

__global__ void __launch_bounds__(512) k_reduce_systems(
    const float *__restrict__ vec, const float *__restrict__ g, const float *__restrict__ e_atom,
    const int *__restrict__ offset, const int *__restrict__ sys_begin, double *__restrict__ virial,
    double *__restrict__ energy, int with_virial) {
  __shared__ double sm[16 * 7];
  const int k = blockIdx.x;
  const int a0 = sys_begin[k], a1 = sys_begin[k + 1];
  double v[7] = {0, 0, 0, 0, 0, 0, 0};
  for (int i = a0 + threadIdx.x; i < a1; i += blockDim.x) v[6] += static_cast<double>(e_atom[i]);
  if (with_virial) {
    for (int e = offset[a0] + threadIdx.x; e < offset[a1]; e += blockDim.x) {
      const double ex = vec[3 * e], ey = vec[3 * e + 1], ez = vec[3 * e + 2];
      const double gx = g[3 * e], gy = g[3 * e + 1], gz = g[3 * e + 2];
      v[0] += ex * gx;
      v[1] += ey * gy;
      v[2] += ez * gz;
      v[3] += 0.5 * (ey * gz + ez * gy);
      v[4] += 0.5 * (ex * gz + ez * gx);
      v[5] += 0.5 * (ex * gy + ey * gx);
    }
  }
  block_sum<7>(v, sm);
  if (threadIdx.x == 0) {
    for (int c = 0; c < 6; ++c) virial[6 * k + c] = v[c];
    energy[k] = v[6];
  }
}

// Deterministic two-stage sum of one structure's energy and virial: block b
// sums a fixed chunk of the atoms and of the edges into partial[b][0..6]
// (0: energy, 1..6: Voigt virial), then one block adds the partials in
// block order.  Replaces a single-block pass over a million edges.
__global__ void __launch_bounds__(256) k_reduce_partial(const float *__restrict__ vec, const float *__restrict__ g,
                                                        const float *__restrict__ e_atom, int n_atoms, int n_edges,
                                                        int with_virial, double *__restrict__ partial) {
  __shared__ double sm[8 * 7];
  const int B = gridDim.x, b = blockIdx.x;
  const int ca = (n_atoms + B - 1) / B, ce = (n_edges + B - 1) / B;
  const int a0 = b * ca, a1 = min(n_atoms, a0 + ca), e0 = b * ce, e1 = with_virial ? min(n_edges, e0 + ce) : e0;
  double v[7] = {0, 0, 0, 0, 0, 0, 0};
  for (int i = a0 + threadIdx.x; i < a1; i += blockDim.x) v[0] += static_cast<double>(e_atom[i]);
  for (int e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
    const double ex = vec[3 * e], ey = vec[3 * e + 1], ez = vec[3 * e + 2];
    const double gx = g[3 * e], gy = g[3 * e + 1], gz = g[3 * e + 2];
    v[1] += ex * gx;
    v[2] += ey * gy;
    v[3] += ez * gz;
    v[4] += 0.5 * (ey * gz + ez * gy);
    v[5] += 0.5 * (ex * gz + ez * gx);
    v[6] += 0.5 * (ex * gy + ey * gx);
  }
  block_sum<7>(v, sm);
  if (threadIdx.x == 0)
    for (int c = 0; c < 7; ++c) partial[7 * b + c] = v[c];
}

__global__ void __launch_bounds__(256) k_reduce_final(const double *__restrict__ partial, int n_part,
                                                      double *__restrict__ energy, double *__restrict__ virial) {
  __shared__ double sm[8 * 7];
  double v[7] = {0, 0, 0, 0, 0, 0, 0};
  for (int b = threadIdx.x; b < n_part; b += blockDim.x)
    for (int c = 0; c < 7; ++c) v[c] += partial[7 * b + c];
  block_sum<7>(v, sm);
  if (threadIdx.x == 0) {
    *energy = v[0];
    for (int c = 0; c < 6; ++c) virial[c] = v[1 + c];
  }
}

// ---- non-conservative heads ----------------------------------------------
constexpr int kNcMaxOut = 9;

// p[o] = y . w[o, :] for o < od, summed over the warp (every lane gets all).
__device__ __forceinline__ void nc_row_dots(const float *__restrict__ y, const float *w, int r, int od, int lane,
                                            float (&p)[kNcMaxOut]) {
#pragma unroll
  for (int o = 0; o < kNcMaxOut; ++o) p[o] = 0.f;
  for (int c = lane; c < r; c += 32) {
    const float yv = y[c];
#pragma unroll
    for (int o = 0; o < kNcMaxOut; ++o)
      if (o < od) p[o] = fmaf(yv, w[o * r + c], p[o]);
  }
#pragma unroll
  for (int o = 0; o < kNcMaxOut; ++o)
    if (o < od) p[o] = warp_sum(p[o]);
}

// Warp per atom i: dst[i, o] += yn[i] . wn[o] + bn[o]
//                             + sum_{e in i} fc[e] (ye[e] . we[o] + be[o]).
// The last layers' weights sit in shared memory: [od][r] node, [od][r] edge.
__global__ void __launch_bounds__(256) k_nc_readout(const float *__restrict__ yn, const float *__restrict__ ye,
                                                    const float *__restrict__ wn, const float *__restrict__ bn,
                                                    const float *__restrict__ we, const float *__restrict__ be,
                                                    const float *__restrict__ fc, const int *__restrict__ offset,
                                                    float *__restrict__ dst, int n, int r, int od) {
  extern __shared__ float s_w[];
  const int nw = od * r;
  for (int t = threadIdx.x; t < nw; t += blockDim.x) {
    s_w[t] = wn[t];
    if (ye) s_w[nw + t] = we[t];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += (gridDim.x * blockDim.x) >> 5) {
    float out[kNcMaxOut], p[kNcMaxOut];
    nc_row_dots(yn + static_cast<size_t>(i) * r, s_w, r, od, lane, out);
#pragma unroll
    for (int o = 0; o < kNcMaxOut; ++o)
      if (o < od) out[o] += bn[o];
    if (ye) {
      for (int e = offset[i]; e < offset[i + 1]; ++e) {
        nc_row_dots(ye + static_cast<size_t>(e) * r, s_w + nw, r, od, lane, p);
        const float f = fc[e];
#pragma unroll
        for (int o = 0; o < kNcMaxOut; ++o)
          if (o < od) out[o] = fmaf(f, p[o] + be[o], out[o]);
      }
    }
    float v = 0.f;
#pragma unroll
    for (int o = 0; o < kNcMaxOut; ++o)
      if (o == lane) v = out[o];
    if (lane < od) dst[static_cast<size_t>(i) * od + lane] += v;
  }
}

// Block per system: out[6k + c] = Voigt sum over its atoms of the 3x3
// tensors S[i] (row-major xx xy xz yx yy yz zx zy zz), off-diagonals
// symmetrised in f32 per atom as pet.cpp:644-665 does, summed in f64.
__global__ void __launch_bounds__(256) k_nc_stress_reduce(const float *__restrict__ S,
                                                          const int *__restrict__ sys_begin,
                                                          double *__restrict__ out) {
  __shared__ double sm[8 * 6];
  const int k = blockIdx.x;
  double v[6] = {0, 0, 0, 0, 0, 0};
  for (int i = sys_begin[k] + threadIdx.x; i < sys_begin[k + 1]; i += blockDim.x) {
    const float *t = S + 9 * static_cast<size_t>(i);
    v[0] += t[0];
    v[1] += t[4];
    v[2] += t[8];
    v[3] += 0.5f * (t[5] + t[7]);
    v[4] += 0.5f * (t[2] + t[6]);
    v[5] += 0.5f * (t[1] + t[3]);
  }
  block_sum<6>(v, sm);
  if (threadIdx.x == 0)
    for (int c = 0; c < 6; ++c) out[6 * k + c] = v[c];
}


}  // namespace

void reduce_one(const float *vec, const float *g, const float *e_atom, int n_atoms, int n_edges, bool with_virial,
                double *partial, double *energy, double *virial, cudaStream_t s) {
  const int64_t work = std::max<int64_t>(std::max(n_atoms, with_virial ? n_edges : 0), 1);
  const int B = static_cast<int>(std::min<int64_t>(kReduceMaxParts, (work + 4095) / 4096));
  k_reduce_partial<<<B, 256, 0, s>>>(vec, g, e_atom, n_atoms, n_edges, with_virial ? 1 : 0, partial);
  CUDA_LAUNCH_CHECK();
  k_reduce_final<<<1, 256, 0, s>>>(partial, B, energy, virial);
  CUDA_LAUNCH_CHECK();
}

void reduce_local(const float *vec, const float *g, const float *e_atom, int n_energy, int n_edges,
                  double *out, double *partial, cudaStream_t s) {
  reduce_one(vec, g, e_atom, n_energy, n_edges, n_edges > 0, partial, out, out + 1, s);
}

void edge_prep(const EdgePrepArgs &a, cudaStream_t s) {
  const int total = a.n_edges > a.n_atoms ? a.n_edges : a.n_atoms;
  if (total <= 0) return;
  k_edge_prep<<<grid_for(total, 256), 256, 0, s>>>(a);
  CUDA_LAUNCH_CHECK();
}

void featurize(const FeaturizeArgs &a, cudaStream_t s) {
  const int K = featurize_cols(a.layer, a.d, a.aux);
  const int64_t total = static_cast<int64_t>(a.n_edges) * K;
  if (total <= 0) return;
  if (a.aux < 5) throw Error(kErrInternal, "featurize: the auxiliary block needs at least 5 columns");
  if (a.cat_split.hi) {
    if (a.d % 128 || a.aux % 128)
      throw Error(kErrInternal, "featurize: split output needs d and the auxiliary block multiples of 128");
    k_featurize_split<<<ceil_div(static_cast<int64_t>(a.n_edges) * 32, 256), 256, 0, s>>>(a);
  } else {
    k_featurize<<<grid_for(total, 256), 256, 0, s>>>(a);
  }
  CUDA_LAUNCH_CHECK();
}

void node_tokens(const float *table, const int *species, float *x, int n, int d, cudaStream_t s,
                 const Split16View *xs) {
  if (n <= 0) return;
  if (xs) {
    if (d % 128) throw Error(kErrInternal, "node_tokens: split output needs a multiple of 128 columns");
    k_node_tokens_split<<<ceil_div(static_cast<int64_t>(n) * (d / 128) * 32, 256), 256, 0, s>>>(
        table, species, x, n, d, *xs);
  } else {
    k_node_tokens<<<grid_for(static_cast<int64_t>(n) * d, 256), 256, 0, s>>>(table, species, x, n, d);
  }
  CUDA_LAUNCH_CHECK();
}

void head_last(const float *y, const float *w, const float *b, float *pred, int rows, int r,
               cudaStream_t s) {
  if (rows <= 0) return;
  k_head_last<<<grid_for(static_cast<int64_t>(rows) * 32, 256), 256, 0, s>>>(y, w, b, pred, rows, r);
  CUDA_LAUNCH_CHECK();
}

void head_last_bwd(const float *z, const float *w, const float *scale, float *dz, int rows, int r,
                   cudaStream_t s, const Split16View *dzs) {
  if (rows <= 0) return;
  if (dzs) {
    if (r % 128) throw Error(kErrInternal, "head_last_bwd: split output needs a multiple of 128 columns");
    k_head_last_bwd_split<<<ceil_div(static_cast<int64_t>(rows) * (r / 128) * 32, 256), 256, 0, s>>>(
        z, w, scale, rows, r, *dzs);
  } else {
    k_head_last_bwd<<<grid_for(static_cast<int64_t>(rows) * r, 256), 256, 0, s>>>(z, w, scale, dz, rows, r);
  }
  CUDA_LAUNCH_CHECK();
}

void atom_energy(const float *node_pred, const float *edge_pred, const float *fc, const int *offset,
                 float *e_atom, int n, bool accumulate, cudaStream_t s) {
  if (n <= 0) return;
  k_atom_energy<<<grid_for(static_cast<int64_t>(n) * 32, 256), 256, 0, s>>>(node_pred, edge_pred, fc, offset,
                                                                            e_atom, n, accumulate);
  CUDA_LAUNCH_CHECK();
}

void add_vec(const float *x, float *y, int n, bool accumulate, cudaStream_t s) {
  if (n <= 0) return;
  k_add_vec<<<grid_for(n, 256), 256, 0, s>>>(x, y, n, accumulate);
  CUDA_LAUNCH_CHECK();
}

void edge_xyzr_bwd(const float *dz, const Split16View *dzs, const float *P, float *g4, int n_edges, int H,
                   bool accumulate, cudaStream_t s) {
  if (n_edges <= 0) return;
  const int grid = grid_for(static_cast<int64_t>(n_edges) * 32, 256);
  if (dzs) {
    switch (H % 128 == 0 ? H / 128 : 0) {
      case 1: k_edge_xyzr_bwd_split<1><<<grid, 256, 0, s>>>(*dzs, P, g4, n_edges, accumulate); break;
      case 2: k_edge_xyzr_bwd_split<2><<<grid, 256, 0, s>>>(*dzs, P, g4, n_edges, accumulate); break;
      case 4: k_edge_xyzr_bwd_split<4><<<grid, 256, 0, s>>>(*dzs, P, g4, n_edges, accumulate); break;
      case 8: k_edge_xyzr_bwd_split<8><<<grid, 256, 0, s>>>(*dzs, P, g4, n_edges, accumulate); break;
      default: throw Error(kErrInternal, "edge_xyzr_bwd: split input needs H in {128, 256, 512, 1024}");
    }
  } else {
    k_edge_xyzr_bwd<<<grid, 256, 0, s>>>(dz, P, g4, n_edges, H, accumulate);
  }
  CUDA_LAUNCH_CHECK();
}

void message_bwd(const float *dmsg, int ld, const int *rev, int base, float *dx,
                 int n_edges, int n_msg, int d, cudaStream_t s) {
  if (n_edges <= 0) return;
  if (d % 4 || ld % 4) throw Error(kErrInternal, "message_bwd: rows must be multiples of 4 floats");
  k_message_bwd<<<grid_for(static_cast<int64_t>(n_edges) * 32, 256), 256, 0, s>>>(dmsg, ld, rev, base, dx,
                                                                                  n_edges, n_msg, d);
  CUDA_LAUNCH_CHECK();
}

void edge_grad(const float *g4, const float *gfc, const float *dfc_dr, const float *vec,
               const float *r, float *g, int n_edges, cudaStream_t s) {
  if (n_edges <= 0) return;
  k_edge_grad<<<grid_for(n_edges, 256), 256, 0, s>>>(g4, gfc, dfc_dr, vec, r, g, n_edges);
  CUDA_LAUNCH_CHECK();
}

void forces(const float *g, const int *offset, const int *nbr, const int *rev, float *F, int n,
            int n_edges, cudaStream_t s) {
  if (n <= 0) return;
  k_forces<<<grid_for(n, 128), 128, 0, s>>>(g, offset, rev, F, n);
  CUDA_LAUNCH_CHECK();
  if (n_edges > 0) {
    k_forces_unpaired<<<grid_for(n_edges, 256), 256, 0, s>>>(g, nbr, rev, F, n_edges);
    CUDA_LAUNCH_CHECK();
  }
}

void nc_readout(const float *yn, const float *ye, const float *wn, const float *bn, const float *we,
                const float *be, const float *fc, const int *offset, float *dst, int n, int r, int od,
                cudaStream_t s) {
  if (n <= 0) return;
  if (od < 1 || od > kNcMaxOut) throw Error(kErrInternal, "nc_readout: at most 9 outputs");
  const size_t smem = sizeof(float) * 2 * od * r;
  if (smem > 48 * 1024) throw Error(kErrUnsupported, "nc_readout: head width too large");
  k_nc_readout<<<grid_for(static_cast<int64_t>(n) * 32, 256), 256, smem, s>>>(yn, ye, wn, bn, we, be, fc, offset,
                                                                             dst, n, r, od);
  CUDA_LAUNCH_CHECK();
}

void nc_stress_reduce(const float *S, const int *sys_atom_begin, int n_sys, double *out, cudaStream_t s) {
  if (n_sys <= 0) return;
  k_nc_stress_reduce<<<n_sys, 256, 0, s>>>(S, sys_atom_begin, out);
  CUDA_LAUNCH_CHECK();
}

void reduce_systems(const float *vec, const float *g, const float *e_atom, const int *offset,
                    const int *sys_atom_begin, int n_sys, double *virial, double *energy,
                    bool with_virial, cudaStream_t s, int n_atoms, int n_edges, double *partial) {
  if (n_sys <= 0) return;
  if (n_sys == 1 && partial) {  // one structure: spread over the GPU
    reduce_one(vec, g, e_atom, n_atoms, n_edges, with_virial, partial, energy, virial, s);
    return;
  }
  k_reduce_systems<<<n_sys, 512, 0, s>>>(vec, g, e_atom, offset, sys_atom_begin, virial, energy,
                                         with_virial ? 1 : 0);
  CUDA_LAUNCH_CHECK();
}

}  // namespace pet
