// GPU cell-list neighbour search, bit-exact with mlip.cpp's
// NeighborListBuilder (src/core/neighbor_list.cpp).
//
// Layout in HBM: atoms are binned by a counting sort (bin_start / bin_atoms,
// each bin's atoms in descending index order, which is the order the
// reference's head-inserted linked lists visit them,
// neighbor_list.cpp:97-105).  One warp owns one centre atom.  It walks the
// (2n+1)^3 search bins in the reference's dz, dy, dx order, packs the
// candidates of up to 32 bins into one dense list, and tests 32 candidates
// per step; a ballot keeps hits in candidate order, so each centre's edges
// come out in exactly the reference's slot order.  A count pass sizes the
// CSR offsets, a fill pass writes the edges.
//
// All fp64 arithmetic uses __dmul_rn / __dadd_rn / __dsub_rn so nvcc cannot
// contract it into FMAs; with the same operation order as the reference this
// reproduces its doubles, and __double2float_rn its float casts.
#include "neighbor.cuh"

#include <cmath>
#include <mutex>

namespace pet {

// ---------------------------------------------------------------------------
// Host: grid parameters (CellGrid ctor, neighbor_list.cpp:38-66)
// ---------------------------------------------------------------------------
void cell_inverse_f32(const float m[9], float inv[9]) {
  // Cell::compute_inverse, system.cpp:19-48 (f32 cofactors)
  auto M = [&](int i, int j) { return m[i * 3 + j]; };
  float det = M(0, 0) * (M(1, 1) * M(2, 2) - M(2, 1) * M(1, 2)) -
              M(0, 1) * (M(1, 0) * M(2, 2) - M(1, 2) * M(2, 0)) +
              M(0, 2) * (M(1, 0) * M(2, 1) - M(1, 1) * M(2, 0));
  float invdet = 1.0f / det;
  inv[0] = (M(1, 1) * M(2, 2) - M(2, 1) * M(1, 2)) * invdet;
  inv[1] = (M(0, 2) * M(2, 1) - M(0, 1) * M(2, 2)) * invdet;
  inv[2] = (M(0, 1) * M(1, 2) - M(0, 2) * M(1, 1)) * invdet;
  inv[3] = (M(1, 2) * M(2, 0) - M(1, 0) * M(2, 2)) * invdet;
  inv[4] = (M(0, 0) * M(2, 2) - M(0, 2) * M(2, 0)) * invdet;
  inv[5] = (M(1, 0) * M(0, 2) - M(0, 0) * M(1, 2)) * invdet;
  inv[6] = (M(1, 0) * M(2, 1) - M(2, 0) * M(1, 1)) * invdet;
  inv[7] = (M(2, 0) * M(0, 1) - M(0, 0) * M(2, 1)) * invdet;
  inv[8] = (M(0, 0) * M(1, 1) - M(1, 0) * M(0, 1)) * invdet;
}

void make_grid_params(const float cell[9], const bool pbc[3], float cutoff, GridParams *g) {
  float finv[9];
  cell_inverse_f32(cell, finv);
  for (int k = 0; k < 9; ++k) g->inv[k] = finv[k];
  double cv[3][3];
  for (int a = 0; a < 3; ++a)
    for (int c = 0; c < 3; ++c) cv[a][c] = cell[a * 3 + c];
  auto cross = [](const double *a, const double *b, double *r) {
    r[0] = a[1] * b[2] - a[2] * b[1];
    r[1] = a[2] * b[0] - a[0] * b[2];
    r[2] = a[0] * b[1] - a[1] * b[0];
  };
  auto dot = [](const double *a, const double *b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; };
  double nrm[3][3];
  cross(cv[1], cv[2], nrm[0]);
  cross(cv[2], cv[0], nrm[1]);
  cross(cv[0], cv[1], nrm[2]);
  double vol = std::fabs(dot(cv[2], nrm[2]));
  const double rc = cutoff;
  for (int a = 0; a < 3; ++a) {
    double face = vol / std::sqrt(dot(nrm[a], nrm[a]));
    int nb = static_cast<int>(std::floor(face / rc));
    g->nb[a] = nb > 1 ? nb : 1;
    g->ns[a] = static_cast<int>(std::ceil(rc * g->nb[a] / face));
    double s = 1.0 / g->nb[a];
    for (int c = 0; c < 3; ++c) g->bv[a * 3 + c] = cv[a][c] * s;
    g->pbc[a] = pbc[a] ? 1 : 0;
  }
  g->cutoff_sq = rc * rc;
}

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
namespace {

__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }

__device__ __forceinline__ int wrap_bin(int idx, int n, int periodic) {
  if (periodic) {
    idx = idx % n;
    if (idx < 0) idx += n;
    return idx;
  }
  return idx < 0 ? 0 : (idx > n - 1 ? n - 1 : idx);
}

// position_to_bin, neighbor_list.cpp:68-80
__device__ __forceinline__ void pos_to_bin(const GridParams &g, double x, double y, double z,
                                           int b[3]) {
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    double f = dadd(dadd(dmul(g.inv[k], x), dmul(g.inv[3 + k], y)), dmul(g.inv[6 + k], z));
    b[k] = static_cast<int>(floor(dmul(f, static_cast<double>(g.nb[k]))));
  }
}

// relative_position, neighbor_list.cpp:107-110
__device__ __forceinline__ void rel_pos(const GridParams &g, double x, double y, double z,
                                        const int b[3], double r[3]) {
  const double p[3] = {x, y, z};
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    double v = dsub(p[c], dmul(g.bv[0 * 3 + c], static_cast<double>(b[0])));
    v = dsub(v, dmul(g.bv[1 * 3 + c], static_cast<double>(b[1])));
    r[c] = dsub(v, dmul(g.bv[2 * 3 + c], static_cast<double>(b[2])));
  }
}

template <typename P>
__global__ void k_bin_atoms(const P *__restrict__ pos, int n, GridParams g,
                            int *__restrict__ braw, int *__restrict__ bin_of,
                            int *__restrict__ bin_count) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int b[3];
  pos_to_bin(g, pos[3 * i], pos[3 * i + 1], pos[3 * i + 2], b);
  braw[3 * i] = b[0];
  braw[3 * i + 1] = b[1];
  braw[3 * i + 2] = b[2];
  int w0 = wrap_bin(b[0], g.nb[0], g.pbc[0]);
  int w1 = wrap_bin(b[1], g.nb[1], g.pbc[1]);
  int w2 = wrap_bin(b[2], g.nb[2], g.pbc[2]);
  int idx = w0 + g.nb[0] * (w1 + g.nb[1] * w2);
  bin_of[i] = idx;
  atomicAdd(bin_count + idx, 1);
}

__global__ void k_fill_bins(const int *__restrict__ bin_of, int n, const int *__restrict__ bin_start,
                            int *__restrict__ cursor, int *__restrict__ bin_atoms) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int b = bin_of[i];
  int k = atomicAdd(cursor + b, 1);
  bin_atoms[bin_start[b] + k] = i;
}

// Descending atom index inside each bin (head-insert linked-list order).
__global__ void k_sort_bins(const int *__restrict__ bin_start, int nbins, int *__restrict__ bin_atoms) {
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nbins) return;
  int s = bin_start[b], e = bin_start[b + 1];
  for (int k = s + 1; k < e; ++k) {
    int v = bin_atoms[k];
    int m = k - 1;
    while (m >= s && bin_atoms[m] < v) {
      bin_atoms[m + 1] = bin_atoms[m];
      --m;
    }
    bin_atoms[m + 1] = v;
  }
}

constexpr int kNLWarps = 4;  // warps (centres) per CTA

// Periodic search (build_periodic, neighbor_list.cpp:163-297).
// kFill = false: count edges per centre; true: write them at offset[i].
template <bool kFill, typename P>
__global__ void __launch_bounds__(32 * kNLWarps)
k_periodic(const P *__restrict__ pos, int n, GridParams g, const int *__restrict__ braw,
           const int *__restrict__ bin_start, const int *__restrict__ bin_atoms,
           int *__restrict__ count, const int *__restrict__ offset, int *__restrict__ e_center,
           int *__restrict__ e_nbr, int *__restrict__ e_shift, float *__restrict__ e_vec,
           float *__restrict__ e_dist) {
  __shared__ int s_start[kNLWarps][32];
  __shared__ int s_pre[kNLWarps][33];
  __shared__ int s_d[kNLWarps][32];  // packed (dx, dy, dz) offsets
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int i = blockIdx.x * kNLWarps + w;
  if (i >= n) return;

  int ri[3] = {braw[3 * i], braw[3 * i + 1], braw[3 * i + 2]};
  int bi[3], wi[3];
#pragma unroll
  for (int d = 0; d < 3; ++d) {
    bi[d] = g.pbc[d] ? ri[d] : wrap_bin(ri[d], g.nb[d], 0);
    wi[d] = wrap_bin(ri[d], g.nb[d], g.pbc[d]);
  }
  double rel_i[3];
  rel_pos(g, pos[3 * i], pos[3 * i + 1], pos[3 * i + 2], bi, rel_i);

  const int sx = 2 * g.ns[0] + 1, sy = 2 * g.ns[1] + 1, sz = 2 * g.ns[2] + 1;
  const int n_search_bins = sx * sy * sz;
  int found = 0;
  const int base = kFill ? offset[i] : 0;

  for (int g0 = 0; g0 < n_search_bins; g0 += 32) {
    // lane k describes search bin g0 + k (dz outer, dy, dx inner)
    int q = g0 + lane;
    int cnt = 0, start = 0, packed = 0;
    if (q < n_search_bins) {
      int ix = q % sx, iy = (q / sx) % sy, iz = q / (sx * sy);
      int dx = ix - g.ns[0], dy = iy - g.ns[1], dz = iz - g.ns[2];
      int bz = wi[2] + dz, by = wi[1] + dy, bx = wi[0] + dx;
      bool ok = true;
      if (g.pbc[2]) bz = wrap_bin(bz, g.nb[2], 1); else ok &= (bz >= 0 && bz < g.nb[2]);
      if (g.pbc[1]) by = wrap_bin(by, g.nb[1], 1); else ok &= (by >= 0 && by < g.nb[1]);
      if (g.pbc[0]) bx = wrap_bin(bx, g.nb[0], 1); else ok &= (bx >= 0 && bx < g.nb[0]);
      if (ok) {
        int b = bx + g.nb[0] * (by + g.nb[1] * bz);
        start = bin_start[b];
        cnt = bin_start[b + 1] - start;
      }
      packed = (dx + 512) | ((dy + 512) << 10) | ((dz + 512) << 20);
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    s_start[w][lane] = start;
    s_pre[w][lane] = incl - cnt;
    s_d[w][lane] = packed;
    if (lane == 0) s_pre[w][32] = total;
    __syncwarp();
    const int nb_here = min(32, n_search_bins - g0);
    for (int c0 = 0; c0 < total; c0 += 32) {
      const int c = c0 + lane;
      bool hit = false;
      int j = 0, dxyz = 0;
      double dr[3] = {0, 0, 0}, d2 = 0;
      if (c < total) {
        int lo = 0, hi = nb_here;  // last k with s_pre[k] <= c
        while (lo < hi) {
          int mid = (lo + hi) >> 1;
          if (s_pre[w][mid] <= c) lo = mid + 1; else hi = mid;
        }
        const int k = lo - 1;
        j = bin_atoms[s_start[w][k] + (c - s_pre[w][k])];
        dxyz = s_d[w][k];
        const int dx = (dxyz & 1023) - 512, dy = ((dxyz >> 10) & 1023) - 512,
                  dz = ((dxyz >> 20) & 1023) - 512;
        const bool same = (dx == 0 && dy == 0 && dz == 0);
        if (i != j || !same) {
          int rj[3] = {braw[3 * j], braw[3 * j + 1], braw[3 * j + 2]};
          int bj[3];
#pragma unroll
          for (int d = 0; d < 3; ++d) bj[d] = g.pbc[d] ? rj[d] : wrap_bin(rj[d], g.nb[d], 0);
          double rel_j[3];
          rel_pos(g, pos[3 * j], pos[3 * j + 1], pos[3 * j + 2], bj, rel_j);
#pragma unroll
          for (int cc = 0; cc < 3; ++cc) {
            // offset = ((bv2 dz) + bv1 dy) + bv0 dx  (neighbor_list.cpp:223-243)
            double off = dmul(g.bv[2 * 3 + cc], static_cast<double>(dz));
            off = dadd(off, dmul(g.bv[1 * 3 + cc], static_cast<double>(dy)));
            off = dadd(off, dmul(g.bv[0 * 3 + cc], static_cast<double>(dx)));
            dr[cc] = dadd(dsub(rel_j[cc], rel_i[cc]), off);
          }
          d2 = dadd(dadd(dmul(dr[0], dr[0]), dmul(dr[1], dr[1])), dmul(dr[2], dr[2]));
          hit = d2 < g.cutoff_sq;
        }
      }
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (kFill && hit) {
        const int e = base + found + __popc(m & ((1u << lane) - 1u));
        const int dx = (dxyz & 1023) - 512, dy = ((dxyz >> 10) & 1023) - 512,
                  dz = ((dxyz >> 20) & 1023) - 512;
        const int dl[3] = {dx, dy, dz};
        e_center[e] = i;
        e_nbr[e] = j;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          const int rjd = braw[3 * j + d];
          e_shift[3 * e + d] = (ri[d] - rjd + dl[d]) / g.nb[d];
          e_vec[3 * e + d] = __double2float_rn(dr[d]);
        }
        e_dist[e] = __double2float_rn(__dsqrt_rn(d2));
      }
      found += __popc(m);
    }
    __syncwarp();
  }
  if (!kFill && lane == 0) count[i] = found;
}

// Open-boundary search (build_non_periodic, neighbor_list.cpp:126-161):
// j ascending inside the centre's own system, 1e-16 < d^2 < rc^2 (rc^2 an
// f32 product), i != j.
template <bool kFill>
__global__ void __launch_bounds__(128)
k_open(const float *__restrict__ pos, const int *__restrict__ sys_begin,
       const int *__restrict__ sys_end, int n, double rc2, int *__restrict__ count,
       const int *__restrict__ offset, int *__restrict__ e_center, int *__restrict__ e_nbr,
       int *__restrict__ e_shift, float *__restrict__ e_vec, float *__restrict__ e_dist) {
  const int lane = threadIdx.x & 31;
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (i >= n) return;
  const double xi = pos[3 * i], yi = pos[3 * i + 1], zi = pos[3 * i + 2];
  const int jb = sys_begin[i], je = sys_end[i];
  int found = 0;
  const int base = kFill ? offset[i] : 0;
  for (int j0 = jb; j0 < je; j0 += 32) {
    const int j = j0 + lane;
    bool hit = false;
    double dr[3] = {0, 0, 0}, d2 = 0;
    if (j < je && j != i) {
      dr[0] = dsub(static_cast<double>(pos[3 * j]), xi);
      dr[1] = dsub(static_cast<double>(pos[3 * j + 1]), yi);
      dr[2] = dsub(static_cast<double>(pos[3 * j + 2]), zi);
      d2 = dadd(dadd(dmul(dr[0], dr[0]), dmul(dr[1], dr[1])), dmul(dr[2], dr[2]));
      hit = d2 < rc2 && d2 > 1e-16;
    }
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (kFill && hit) {
      const int e = base + found + __popc(m & ((1u << lane) - 1u));
      e_center[e] = i;
      e_nbr[e] = j;
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        e_shift[3 * e + d] = 0;
        e_vec[3 * e + d] = __double2float_rn(dr[d]);
      }
      e_dist[e] = __double2float_rn(__dsqrt_rn(d2));
    }
    found += __popc(m);
  }
  if (!kFill && lane == 0) count[i] = found;
}

// Single-CTA exclusive scan with max; each thread scans a contiguous chunk.
__global__ void __launch_bounds__(1024) k_scan(const int *__restrict__ in, int *__restrict__ out,
                                               int *__restrict__ max_out, int n) {
  __shared__ int s_sum[32], s_max[32];
  const int t = threadIdx.x, nt = blockDim.x;
  const int chunk = (n + nt - 1) / nt;
  const int a = min(n, t * chunk), b = min(n, a + chunk);
  int sum = 0, mx = 0;
  for (int k = a; k < b; ++k) {
    sum += in[k];
    mx = max(mx, in[k]);
  }
  // block exclusive scan of `sum`
  const int lane = t & 31, w = t >> 5;
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int wm = mx;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wm = max(wm, __shfl_xor_sync(0xffffffffu, wm, o));
  if (lane == 31) s_sum[w] = incl;
  if (lane == 0) s_max[w] = wm;
  __syncthreads();
  if (w == 0) {
    const int nw = nt >> 5;
    int v = lane < nw ? s_sum[lane] : 0;
    int m2 = lane < nw ? s_max[lane] : 0;
    int inc2 = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, inc2, o);
      if (lane >= o) inc2 += u;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m2 = max(m2, __shfl_xor_sync(0xffffffffu, m2, o));
    s_sum[lane] = inc2 - v;  // exclusive warp offsets
    if (lane == 0) s_max[0] = m2;
  }
  __syncthreads();
  int run = s_sum[w] + incl - sum;
  for (int k = a; k < b; ++k) {
    out[k] = run;
    run += in[k];
  }
  if (t == nt - 1) out[n] = run;
  if (t == 0 && max_out) *max_out = s_max[0];
}

}  // namespace

void scan_counts(const int *in, int *out, int *max_out, int n, cudaStream_t stream) {
  k_scan<<<1, 1024, 0, stream>>>(in, out, max_out, n);
  CUDA_LAUNCH_CHECK();
}

// The pair offsets are int32 scans; the largest per-centre count times the
// number of centres bounds the total, so below 2^31 nothing wrapped.
void check_pair_total(int max_count, int n_centers) {
  if (static_cast<int64_t>(max_count) * n_centers > INT32_MAX)
    throw Error(kErrInvalidParameter, "the neighbour list could exceed 2^31 - 1 pairs (" +
                                          std::to_string(n_centers) + " centres with up to " +
                                          std::to_string(max_count) + " neighbours each)");
}

// k_periodic packs each search-bin offset into 10 bits, so at most 511 bins
// are searched on either side along any axis.
void check_search_extent(const GridParams &g) {
  for (int a = 0; a < 3; ++a)
    if (g.ns[a] > kMaxSearchBins)
      throw Error(kErrInvalidParameter, "the cutoff spans " + std::to_string(g.ns[a]) +
                                            " cell widths along one axis (at most " +
                                            std::to_string(kMaxSearchBins) + ")");
}

namespace {
void size_edges(EdgeList &out, int n, cudaStream_t stream) {
  int host[2];
  CUDA_CHECK(cudaMemcpyAsync(&host[0], out.offset.as<int>() + n, sizeof(int), cudaMemcpyDeviceToHost, stream));
  CUDA_CHECK(cudaMemcpyAsync(&host[1], out.offset.as<int>() + n + 1, sizeof(int), cudaMemcpyDeviceToHost, stream));
  CUDA_CHECK(cudaStreamSynchronize(stream));
  check_pair_total(host[1], n);
  out.n_edges = host[0];
  out.max_count = host[1];
  size_t e = static_cast<size_t>(out.n_edges > 0 ? out.n_edges : 1);
  out.center.ensure(e * 4);
  out.nbr.ensure(e * 4);
  out.shift.ensure(e * 12);
  out.vec.ensure(e * 12);
  out.dist.ensure(e * 4);
}
}  // namespace

template <typename P>
void build_grid_nl(const P *pos, int n, int n_centers, const GridParams &g, EdgeList &out, NLScratch &s,
                   cudaStream_t stream) {
  check_search_extent(g);
  out.n_atoms = n_centers;
  const int nbins = g.nb[0] * g.nb[1] * g.nb[2];
  int *braw = static_cast<int *>(s.braw.ensure(sizeof(int) * 3 * (n + 1)));
  int *bin_of = static_cast<int *>(s.bin_of.ensure(sizeof(int) * (n + 1)));
  int *bin_count = static_cast<int *>(s.bin_count.ensure(sizeof(int) * (nbins + 1)));
  int *bin_start = static_cast<int *>(s.bin_start.ensure(sizeof(int) * (nbins + 2)));
  int *cursor = static_cast<int *>(s.bin_cursor.ensure(sizeof(int) * (nbins + 1)));
  int *bin_atoms = static_cast<int *>(s.bin_atoms.ensure(sizeof(int) * (n + 1)));
  int *count = static_cast<int *>(out.count.ensure(sizeof(int) * (n_centers + 1)));
  int *offset = static_cast<int *>(out.offset.ensure(sizeof(int) * (n_centers + 2)));
  CUDA_CHECK(cudaMemsetAsync(bin_count, 0, sizeof(int) * nbins, stream));
  CUDA_CHECK(cudaMemsetAsync(cursor, 0, sizeof(int) * nbins, stream));
  if (n > 0) {
    k_bin_atoms<P><<<ceil_div(n, 256), 256, 0, stream>>>(pos, n, g, braw, bin_of, bin_count);
    CUDA_LAUNCH_CHECK();
  }
  scan_counts(bin_count, bin_start, nullptr, nbins, stream);
  if (n > 0) {
    k_fill_bins<<<ceil_div(n, 256), 256, 0, stream>>>(bin_of, n, bin_start, cursor, bin_atoms);
    CUDA_LAUNCH_CHECK();
    k_sort_bins<<<ceil_div(nbins, 128), 128, 0, stream>>>(bin_start, nbins, bin_atoms);
    CUDA_LAUNCH_CHECK();
  }
  if (n_centers > 0) {
    k_periodic<false, P><<<ceil_div(n_centers, kNLWarps), 32 * kNLWarps, 0, stream>>>(
        pos, n_centers, g, braw, bin_start, bin_atoms, count, nullptr, nullptr, nullptr, nullptr, nullptr,
        nullptr);
    CUDA_LAUNCH_CHECK();
  }
  scan_counts(count, offset, offset + n_centers + 1, n_centers, stream);
  size_edges(out, n_centers, stream);
  if (n_centers > 0 && out.n_edges > 0) {
    k_periodic<true, P><<<ceil_div(n_centers, kNLWarps), 32 * kNLWarps, 0, stream>>>(
        pos, n_centers, g, braw, bin_start, bin_atoms, nullptr, offset, out.center.as<int>(),
        out.nbr.as<int>(), out.shift.as<int>(), out.vec.as<float>(), out.dist.as<float>());
    CUDA_LAUNCH_CHECK();
  }
}

void build_periodic_nl(const float *pos, int n, const GridParams &g, EdgeList &out, NLScratch &s,
                       cudaStream_t stream) {
  build_grid_nl<float>(pos, n, n, g, out, s, stream);
}

void build_local_nl(const double *pos, int n, int n_centers, const GridParams &g, EdgeList &out,
                    NLScratch &s, cudaStream_t stream) {
  build_grid_nl<double>(pos, n, n_centers, g, out, s, stream);
}

__global__ void k_skin_displacement(const float *__restrict__ pos, const float *__restrict__ ref, int n, SkinGeom g,
                                    int *__restrict__ img, unsigned *__restrict__ d_max2) {
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  float d2 = 0.f;
  if (a < n) {
    double d[3], k[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) d[c] = static_cast<double>(ref[3 * a + c]) - static_cast<double>(pos[3 * a + c]);
    // k = round((ref - pos) inv) along periodic axes
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double f = d[0] * g.inv[0 * 3 + c] + d[1] * g.inv[1 * 3 + c] + d[2] * g.inv[2 * 3 + c];
      k[c] = g.pbc[c] ? rint(f) : 0.0;
      img[3 * a + c] = static_cast<int>(k[c]);
    }
    double m = 0.0;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double u = k[0] * g.cell[0 * 3 + c] + k[1] * g.cell[1 * 3 + c] + k[2] * g.cell[2 * 3 + c] - d[c];
      m += u * u;
    }
    d2 = static_cast<float>(m);
  }
  d2 = warp_max(d2);
  if ((threadIdx.x & 31) == 0 && d2 > 0.f) atomicMax(d_max2, __float_as_uint(d2));
}

__global__ void k_refresh_edges(const float *__restrict__ pos, int n_edges, const int *__restrict__ center,
                                const int *__restrict__ nbr, const int *__restrict__ shift,
                                const int *__restrict__ img, SkinGeom g, float *__restrict__ vec,
                                float *__restrict__ dist) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_edges) return;
  const int i = center[e], j = nbr[e];
  double s[3], v[3];
#pragma unroll
  for (int c = 0; c < 3; ++c)
    s[c] = static_cast<double>(shift[3 * e + c] + img[3 * j + c] - img[3 * i + c]);
  double d2 = 0.0;
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    v[c] = (static_cast<double>(pos[3 * j + c]) - static_cast<double>(pos[3 * i + c])) +
           (s[0] * g.cell[0 * 3 + c] + s[1] * g.cell[1 * 3 + c] + s[2] * g.cell[2 * 3 + c]);
    vec[3 * e + c] = __double2float_rn(v[c]);
    d2 += v[c] * v[c];
  }
  dist[e] = __double2float_rn(sqrt(d2));
}

void skin_displacement(const float *pos, const float *ref, int n, const SkinGeom &g, int *img, unsigned *d_max2,
                       cudaStream_t stream) {
  if (n <= 0) return;
  k_skin_displacement<<<ceil_div(n, 256), 256, 0, stream>>>(pos, ref, n, g, img, d_max2);
  CUDA_LAUNCH_CHECK();
}

void refresh_edges(const float *pos, int n_edges, const int *center, const int *nbr, const int *shift,
                   const int *img, const SkinGeom &g, float *vec, float *dist, cudaStream_t stream) {
  if (n_edges <= 0) return;
  k_refresh_edges<<<ceil_div(n_edges, 256), 256, 0, stream>>>(pos, n_edges, center, nbr, shift, img, g, vec, dist);
  CUDA_LAUNCH_CHECK();
}

void build_open_nl(const float *pos, const int *sys_begin, const int *sys_end, int n, float cutoff,
                   EdgeList &out, NLScratch &s, cudaStream_t stream) {
  (void)s;
  out.n_atoms = n;
  int *count = static_cast<int *>(out.count.ensure(sizeof(int) * (n + 1)));
  int *offset = static_cast<int *>(out.offset.ensure(sizeof(int) * (n + 2)));
  const float rc2f = cutoff * cutoff;
  const double rc2 = rc2f;
  if (n > 0) {
    k_open<false><<<ceil_div(static_cast<int64_t>(n) * 32, 128), 128, 0, stream>>>(
        pos, sys_begin, sys_end, n, rc2, count, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
    CUDA_LAUNCH_CHECK();
  }
  scan_counts(count, offset, offset + n + 1, n, stream);
  size_edges(out, n, stream);
  if (n > 0 && out.n_edges > 0) {
    k_open<true><<<ceil_div(static_cast<int64_t>(n) * 32, 128), 128, 0, stream>>>(
        pos, sys_begin, sys_end, n, rc2, nullptr, offset, out.center.as<int>(), out.nbr.as<int>(),
        out.shift.as<int>(), out.vec.as<float>(), out.dist.as<float>());
    CUDA_LAUNCH_CHECK();
  }
}

// ---------------------------------------------------------------------------
// Search without allocation (build_periodic_nl_noalloc)
// ---------------------------------------------------------------------------
// Working memory: one static array per device, as ints
//   braw [3 (A+1)] | bin_of [A+1] | bin_atoms [A+1] | count [A+1] |
//   offset [A+2] | bin_count [B+1] | bin_start [B+2] | cursor [B+1]
// with A = kNoAllocMaxAtoms, B = kNoAllocMaxBins.  bin_count and cursor must
// start at zero and are cleared by every call; every other part is fully
// written before it is read.
namespace {
constexpr size_t kNAAtomSlot = static_cast<size_t>(kNoAllocMaxAtoms) + 1;
constexpr size_t kNABinSlot = static_cast<size_t>(kNoAllocMaxBins) + 1;
constexpr size_t kNAOffBinOf = 3 * kNAAtomSlot;
constexpr size_t kNAOffBinAtoms = kNAOffBinOf + kNAAtomSlot;
constexpr size_t kNAOffCount = kNAOffBinAtoms + kNAAtomSlot;
constexpr size_t kNAOffOffset = kNAOffCount + kNAAtomSlot;
constexpr size_t kNAOffBinCount = kNAOffOffset + kNAAtomSlot + 1;
constexpr size_t kNAOffBinStart = kNAOffBinCount + kNABinSlot;
constexpr size_t kNAOffCursor = kNAOffBinStart + kNABinSlot + 1;
constexpr size_t kNAInts = kNAOffCursor + kNABinSlot;
static_assert(kNAInts == 7 * kNAAtomSlot + 3 * kNABinSlot + 2, "scratch layout");
__device__ __align__(256) int g_nl_noalloc_scratch[kNAInts];

constexpr int kNAMaxDevices = 64;
std::mutex g_nl_noalloc_mu;
int *g_nl_noalloc_ptr[kNAMaxDevices] = {};

// Device address of g_nl_noalloc_scratch on the current device.  The first
// call on a device looks it up (cudaGetSymbolAddress, with that device
// current) and keeps it; later calls only read the table.
int *noalloc_scratch() {
  int dev = 0;
  CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNAMaxDevices) throw Error(kErrUnsupported, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_nl_noalloc_mu);
  if (!g_nl_noalloc_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_nl_noalloc_scratch);
    if (rc != cudaSuccess || !p)
      throw Error(kErrBackend, std::string("cudaGetSymbolAddress of the neighbour-list scratch failed: ") +
                                   cudaGetErrorString(rc));
    g_nl_noalloc_ptr[dev] = static_cast<int *>(p);
  }
  return g_nl_noalloc_ptr[dev];
}
}  // namespace

int64_t build_periodic_nl_noalloc(const float *pos, int n, const GridParams &g, int64_t cap,
                                  int *e_center, int *e_nbr, int *e_shift, float *e_vec, float *e_dist,
                                  cudaStream_t stream) {
  const int64_t nbins = static_cast<int64_t>(g.nb[0]) * g.nb[1] * g.nb[2];
  if (n < 0 || n > kNoAllocMaxAtoms)
    throw Error(kErrInvalidParameter, "the no-allocation neighbour list takes at most " +
                                          std::to_string(kNoAllocMaxAtoms) + " atoms (got " +
                                          std::to_string(n) + ")");
  if (nbins > kNoAllocMaxBins)
    throw Error(kErrInvalidParameter, "the no-allocation neighbour list takes at most " +
                                          std::to_string(kNoAllocMaxBins) + " cutoff-sized bins (this cell needs " +
                                          std::to_string(nbins) + ")");
  check_search_extent(g);
  if (n == 0) return 0;
  int *braw = noalloc_scratch();
  int *bin_of = braw + kNAOffBinOf;
  int *bin_atoms = braw + kNAOffBinAtoms;
  int *count = braw + kNAOffCount;
  int *offset = braw + kNAOffOffset;        // A + 2 entries
  int *bin_count = braw + kNAOffBinCount;
  int *bin_start = braw + kNAOffBinStart;   // B + 2 entries
  int *cursor = braw + kNAOffCursor;
  const int nb = static_cast<int>(nbins);
  CUDA_CHECK(cudaMemsetAsync(bin_count, 0, sizeof(int) * nb, stream));
  CUDA_CHECK(cudaMemsetAsync(cursor, 0, sizeof(int) * nb, stream));
  k_bin_atoms<float><<<ceil_div(n, 256), 256, 0, stream>>>(pos, n, g, braw, bin_of, bin_count);
  CUDA_LAUNCH_CHECK();
  scan_counts(bin_count, bin_start, nullptr, nb, stream);
  k_fill_bins<<<ceil_div(n, 256), 256, 0, stream>>>(bin_of, n, bin_start, cursor, bin_atoms);
  CUDA_LAUNCH_CHECK();
  k_sort_bins<<<ceil_div(nb, 128), 128, 0, stream>>>(bin_start, nb, bin_atoms);
  CUDA_LAUNCH_CHECK();
  k_periodic<false, float><<<ceil_div(n, kNLWarps), 32 * kNLWarps, 0, stream>>>(
      pos, n, g, braw, bin_start, bin_atoms, count, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
  CUDA_LAUNCH_CHECK();
  scan_counts(count, offset, offset + n + 1, n, stream);
  int total_max[2] = {0, 0};  // the scan's total and largest count
  CUDA_CHECK(cudaMemcpyAsync(total_max, offset + n, 2 * sizeof(int), cudaMemcpyDeviceToHost, stream));
  CUDA_CHECK(cudaStreamSynchronize(stream));
  check_pair_total(total_max[1], n);
  const int total = total_max[0];
  if (total > 0 && total <= cap) {
    k_periodic<true, float><<<ceil_div(n, kNLWarps), 32 * kNLWarps, 0, stream>>>(
        pos, n, g, braw, bin_start, bin_atoms, nullptr, offset, e_center, e_nbr, e_shift, e_vec, e_dist);
    CUDA_LAUNCH_CHECK();
    CUDA_CHECK(cudaStreamSynchronize(stream));
  }
  return total;
}

}  // namespace pet
