// Spatial domain decomposition of one periodic cell (see domain.h).  All
// per-atom and per-edge work is in kernels on the model's stream; the host
// reads back only the per-rank counts that size the exchanges.
//
// Determinism: the halo copies of each owned atom are enumerated in a fixed
// order (destination rank, then image shift, x slowest) and placed by scans,
// so the ghosts of a local system, and with them its neighbour list, come in
// the same order every step.  Requests are placed with atomic counters: their
// order only decides where a received token row sits, not what is computed.
#include "domain.h"

#include <chrono>
#include <cmath>
#include <cstring>
#include <string>

#include "ops.cuh"

namespace pet {
namespace {

using Geom = DomainEngine::Geom;

// One halo copy of an owned atom: its position with the image shift applied
// (f64), its index among its owner's owned atoms, its atomic number and the
// image shift G (in cell vectors) of this copy relative to the owner's
// position of the atom.
struct GhostRec {
  double x, y, z;
  int32_t src;
  int32_t z_num;
  int32_t img;
  int32_t pad;
};
static_assert(sizeof(GhostRec) == 40, "ghost record layout");

// A request for the layer-0 token of the owner's edge j -> (copy of the
// requester's atom i) whose neighbour carries image shift T.
struct ReqRec {
  int32_t j, i, img, pad;
};

constexpr int kMaxShift = 511;  // packed image shifts: 10 bits per axis

__host__ __device__ inline int32_t pack3(int a, int b, int c) {
  return (a + 512) | ((b + 512) << 10) | ((c + 512) << 20);
}
__device__ inline void unpack3(int32_t v, int (&o)[3]) {
  o[0] = (v & 1023) - 512;
  o[1] = ((v >> 10) & 1023) - 512;
  o[2] = ((v >> 20) & 1023) - 512;
}
__device__ inline bool fits3(const int (&o)[3]) {
  return abs(o[0]) <= kMaxShift && abs(o[1]) <= kMaxShift && abs(o[2]) <= kMaxShift;
}

__device__ inline int slab_coord(const Geom &g, int r, int a) {
  return a == 0 ? r % g.p[0] : a == 1 ? (r / g.p[0]) % g.p[1] : r / (g.p[0] * g.p[1]);
}

// Fractional coordinates of a position (row vector times the inverse cell).
__device__ inline void frac_of(const Geom &g, double x, double y, double z, double (&f)[3]) {
#pragma unroll
  for (int k = 0; k < 3; ++k) f[k] = x * g.inv[k] + y * g.inv[3 + k] + z * g.inv[6 + k];
}

// Image id 0..26 <-> shift (x slowest, each -1..1).
__device__ inline void image_shift(int id, int (&s)[3]) {
  s[0] = id / 9 - 1;
  s[1] = (id / 3) % 3 - 1;
  s[2] = id % 3 - 1;
}

// Bit mask over image ids of the copies of an atom at wrapped fractional
// position fw that lie in rank r's halo box: the rank's slab widened by the
// halo width along each split axis.  Images shift only along split axes; a
// rank sends no copy of an atom to itself without a shift.
__device__ inline uint32_t halo_mask(const Geom &g, int r, const double (&fw)[3]) {
  uint32_t m = 0;
  for (int id = 0; id < 27; ++id) {
    int s[3];
    image_shift(id, s);
    bool ok = !(r == g.rank && s[0] == 0 && s[1] == 0 && s[2] == 0);
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      if (g.p[a] == 1) {
        ok &= s[a] == 0;
        continue;
      }
      const int c = slab_coord(g, r, a);
      const double lo = static_cast<double>(c) / g.p[a] - g.d1[a], hi = static_cast<double>(c + 1) / g.p[a] + g.d1[a];
      const double v = fw[a] + s[a];
      ok &= v >= lo && v < hi;
    }
    if (ok) m |= 1u << id;
  }
  return m;
}

// Thread per owned atom: wrap shift W = -floor(frac) (packed), and for each
// rank the mask of its copies and their number.
__global__ void k_halo_mask(const float *__restrict__ pos, int n, Geom g, uint32_t *__restrict__ mask,
                            int *__restrict__ cnt, int32_t *__restrict__ wrap, int *__restrict__ flag) {
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= n) return;
  double f[3];
  frac_of(g, pos[3 * a], pos[3 * a + 1], pos[3 * a + 2], f);
  int W[3];
  double fw[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const double fl = floor(f[k]);
    W[k] = fabs(fl) <= kMaxShift ? -static_cast<int>(fl) : 0;
    fw[k] = f[k] + W[k];
  }
  if (!fits3(W) || fabs(f[0]) > kMaxShift || fabs(f[1]) > kMaxShift || fabs(f[2]) > kMaxShift) atomicOr(flag, 1);
  wrap[a] = pack3(W[0], W[1], W[2]);
  for (int r = 0; r < g.world; ++r) {
    const uint32_t m = halo_mask(g, r, fw);
    mask[static_cast<size_t>(r) * n + a] = m;
    cnt[static_cast<size_t>(r) * n + a] = __popc(m);
  }
}

// Thread per owned atom: write its copies for every rank at
// sbase[r] + off[r][a] (rank segments of the send buffer).
__global__ void k_halo_fill(const float *__restrict__ pos, const int32_t *__restrict__ z, int n, Geom g,
                            const uint32_t *__restrict__ mask, const int32_t *__restrict__ wrap,
                            const int *__restrict__ off, const int64_t *__restrict__ sbase,
                            GhostRec *__restrict__ out) {
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= n) return;
  int W[3];
  unpack3(wrap[a], W);
  const double x = pos[3 * a], y = pos[3 * a + 1], zz = pos[3 * a + 2];
  for (int r = 0; r < g.world; ++r) {
    uint32_t m = mask[static_cast<size_t>(r) * n + a];
    int64_t dst = sbase[r] + off[static_cast<size_t>(r) * (n + 1) + a];
    while (m) {
      const int id = __ffs(m) - 1;
      m &= m - 1;
      int s[3];
      image_shift(id, s);
      const int G[3] = {W[0] + s[0], W[1] + s[1], W[2] + s[2]};
      GhostRec rec;
      rec.x = x + G[0] * g.cell[0] + G[1] * g.cell[3] + G[2] * g.cell[6];
      rec.y = y + G[0] * g.cell[1] + G[1] * g.cell[4] + G[2] * g.cell[7];
      rec.z = zz + G[0] * g.cell[2] + G[1] * g.cell[5] + G[2] * g.cell[8];
      rec.src = a;
      rec.z_num = z[a];
      rec.img = pack3(G[0], G[1], G[2]);
      rec.pad = 0;
      out[dst++] = rec;
    }
  }
}

__global__ void k_rank_totals(const int *__restrict__ off, int n, int world, int64_t *__restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < world) out[r] = off[static_cast<size_t>(r) * (n + 1) + n];
}

// Source rank of element q of a buffer whose rank segments start at base[r].
__device__ inline int segment_of(const int64_t *base, int world, int64_t q) {
  int r = 0;
  while (r + 1 < world && base[r + 1] <= q) ++r;
  return r;
}

// Thread per local atom: f64 position in the local frame (owned atoms with
// their wrap shift, ghosts as received), species index, and per ghost its
// owner rank, owner-local index and image shift.
__global__ void k_local_build(const float *__restrict__ pos, const int32_t *__restrict__ wrap,
                              const int *__restrict__ species_own, int n_own, const GhostRec *__restrict__ recv,
                              const int64_t *__restrict__ rbase, int n_ghost, Geom g, const int *__restrict__ zmap,
                              double *__restrict__ posl, int *__restrict__ species, int *__restrict__ ghost_rank,
                              int *__restrict__ ghost_src, int32_t *__restrict__ ghost_img, int *__restrict__ flag) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_own + n_ghost) return;
  double o[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) o[c] = g.origin[0] * g.cell[c] + g.origin[1] * g.cell[3 + c] + g.origin[2] * g.cell[6 + c];
  if (t < n_own) {
    int W[3];
    unpack3(wrap[t], W);
#pragma unroll
    for (int c = 0; c < 3; ++c)
      posl[3 * t + c] = static_cast<double>(pos[3 * t + c]) + W[0] * g.cell[c] + W[1] * g.cell[3 + c] +
                        W[2] * g.cell[6 + c] - o[c];
    species[t] = species_own[t];
  } else {
    const int q = t - n_own;
    const GhostRec rec = recv[q];
    posl[3 * t] = rec.x - o[0];
    posl[3 * t + 1] = rec.y - o[1];
    posl[3 * t + 2] = rec.z - o[2];
    const int sp = (rec.z_num >= 0 && rec.z_num < 128) ? zmap[rec.z_num] : -1;
    if (sp < 0) atomicOr(flag, 2);
    species[t] = sp < 0 ? 0 : sp;
    ghost_rank[q] = segment_of(rbase, g.world, q);
    ghost_src[q] = rec.src;
    ghost_img[q] = rec.img;
  }
}

// Thread per edge: requests per owner rank of edges to ghosts.
__global__ void k_req_count(const int *__restrict__ nbr, int n_edges, int n_own, const int *__restrict__ ghost_rank,
                            int *__restrict__ cnt) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_edges) return;
  const int j = nbr[e];
  if (j >= n_own) atomicAdd(cnt + ghost_rank[j - n_own], 1);
}

// Thread per edge i -> j: for a ghost j, a request to j's owner for the
// token of its edge j -> i with neighbour image T = W_i - G_j - s (s: the
// edge's periodic shift along unsplit axes), so that the two edge vectors
// are exact opposites; msg_row[e] = T0 + its slot (-1 for local j).
__global__ void k_req_fill(const int *__restrict__ center, const int *__restrict__ nbr,
                           const int *__restrict__ shift, int n_edges, int n_own, const int32_t *__restrict__ wrap,
                           const int *__restrict__ ghost_rank, const int *__restrict__ ghost_src,
                           const int32_t *__restrict__ ghost_img, const int64_t *__restrict__ base,
                           int *__restrict__ cursor, int T0, ReqRec *__restrict__ out, int *__restrict__ req_edge,
                           int *__restrict__ msg_row, int *__restrict__ flag) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_edges) return;
  const int j = nbr[e];
  if (j < n_own) {
    msg_row[e] = -1;
    return;
  }
  const int q = j - n_own;
  const int r = ghost_rank[q];
  const int64_t slot = base[r] + atomicAdd(cursor + r, 1);
  int Wi[3], Gj[3];
  unpack3(wrap[center[e]], Wi);
  unpack3(ghost_img[q], Gj);
  int T[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) T[c] = Wi[c] - Gj[c] - shift[3 * e + c];
  if (!fits3(T)) atomicOr(flag, 4);
  out[slot] = ReqRec{ghost_src[q], center[e], pack3(T[0], T[1], T[2]), 0};
  req_edge[slot] = e;
  msg_row[e] = T0 + static_cast<int>(slot);
}

// Thread per received request: the owned centre's edge to the requester's
// atom with the requested image shift (G_k - W_j + s' == T), or -1.
__global__ void k_resolve(const ReqRec *__restrict__ req, int n_req, const int64_t *__restrict__ rbase, int world,
                          const int *__restrict__ offset, const int *__restrict__ nbr, const int *__restrict__ shift,
                          int n_own, const int32_t *__restrict__ wrap, const int *__restrict__ ghost_rank,
                          const int *__restrict__ ghost_src, const int32_t *__restrict__ ghost_img,
                          int *__restrict__ reply_edge) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= n_req) return;
  const ReqRec rq = req[q];
  const int from = segment_of(rbase, world, q);
  int found = -1;
  if (rq.j >= 0 && rq.j < n_own) {
    int T[3], Wj[3];
    unpack3(rq.img, T);
    unpack3(wrap[rq.j], Wj);
    for (int e = offset[rq.j]; e < offset[rq.j + 1]; ++e) {
      const int k = nbr[e];
      if (k < n_own) continue;
      const int gk = k - n_own;
      if (ghost_rank[gk] != from || ghost_src[gk] != rq.i) continue;
      int G[3];
      unpack3(ghost_img[gk], G);
      if (G[0] - Wj[0] + shift[3 * e] == T[0] && G[1] - Wj[1] + shift[3 * e + 1] == T[1] &&
          G[2] - Wj[2] + shift[3 * e + 2] == T[2])
        found = e;
    }
  }
  reply_edge[q] = found;
}

// Warp per row q: dst[q] = scale * src[base + idx[q]] (zeros for idx < 0).
__global__ void k_gather_rows(const float *__restrict__ src, int base, const int *__restrict__ idx, int n, int d,
                              float scale, float *__restrict__ dst) {
  const int lane = threadIdx.x & 31;
  for (int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; q < n; q += (gridDim.x * blockDim.x) >> 5) {
    const int r = idx[q];
    float4 *o = reinterpret_cast<float4 *>(dst + static_cast<size_t>(q) * d);
    if (r < 0) {
      for (int c = lane; c < d / 4; c += 32) o[c] = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    const float4 *in = reinterpret_cast<const float4 *>(src + static_cast<size_t>(base + r) * d);
    for (int c = lane; c < d / 4; c += 32) {
      const float4 v = in[c];
      o[c] = make_float4(scale * v.x, scale * v.y, scale * v.z, scale * v.w);
    }
  }
}

// Warp per row q: dst[base + idx[q]] += src[q] (idx < 0 skipped; no two
// rows share a destination).
__global__ void k_scatter_add_rows(const float *__restrict__ src, const int *__restrict__ idx, int n, int d, int base,
                                   float *__restrict__ dst) {
  const int lane = threadIdx.x & 31;
  for (int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; q < n; q += (gridDim.x * blockDim.x) >> 5) {
    const int r = idx[q];
    if (r < 0) continue;
    const float4 *in = reinterpret_cast<const float4 *>(src + static_cast<size_t>(q) * d);
    float4 *o = reinterpret_cast<float4 *>(dst + static_cast<size_t>(base + r) * d);
    for (int c = lane; c < d / 4; c += 32) {
      const float4 a = in[c];
      float4 v = o[c];
      v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
      o[c] = v;
    }
  }
}

// Thread per owned atom: its local force plus the forces its copies
// received on other ranks (in the fixed copy order), into out.
__global__ void k_owned_forces(const float *__restrict__ F, const float *__restrict__ frecv, int n, int world,
                               const int *__restrict__ cnt, const int *__restrict__ off,
                               const int64_t *__restrict__ sbase, float *__restrict__ out) {
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= n) return;
  float fx = F[3 * a], fy = F[3 * a + 1], fz = F[3 * a + 2];
  for (int r = 0; r < world; ++r) {
    const int c = cnt[static_cast<size_t>(r) * n + a];
    const int64_t b = sbase[r] + off[static_cast<size_t>(r) * (n + 1) + a];
    for (int k = 0; k < c; ++k) {
      fx += frecv[3 * (b + k)];
      fy += frecv[3 * (b + k) + 1];
      fz += frecv[3 * (b + k) + 2];
    }
  }
  out[3 * a] = fx;
  out[3 * a + 1] = fy;
  out[3 * a + 2] = fz;
}

int blocks(int64_t n, int t) { return static_cast<int>(n > 0 ? (n + t - 1) / t : 1); }
int row_blocks(int64_t rows) {
  const int64_t b = (rows * 32 + 255) / 256;
  return static_cast<int>(b < 1 ? 1 : (b > 148 * 32 ? 148 * 32 : b));
}

}  // namespace

DomainEngine::DomainEngine(PETModel &model, const float cell[9], const int grid[3], int rank, float skin,
                           const DomainComm &comm)
    : model_(model), comm_(comm) {
  if (!comm.alltoallv || !comm.allreduce_sum_f64) throw Error(kErrInvalidParameter, "domain exchange callbacks missing");
  int world = 1;
  for (int a = 0; a < 3; ++a) {
    if (grid[a] < 1) throw Error(kErrInvalidParameter, "domain grid entries must be >= 1");
    g_.p[a] = grid[a];
    world *= grid[a];
  }
  if (rank < 0 || rank >= world) throw Error(kErrInvalidParameter, "rank outside the domain grid");
  if (world > 64) throw Error(kErrUnsupported, "at most 64 domains");
  if (!std::isfinite(skin) || skin < 0.0f) throw Error(kErrInvalidParameter, "skin must be finite and >= 0");
  g_.world = world;
  g_.rank = rank;
  double m[3][3];
  for (int k = 0; k < 9; ++k) g_.cell[k] = cell[k];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) m[i][j] = cell[3 * i + j];
  const double det = m[0][0] * (m[1][1] * m[2][2] - m[1][2] * m[2][1]) - m[0][1] * (m[1][0] * m[2][2] - m[1][2] * m[2][0]) +
                     m[0][2] * (m[1][0] * m[2][1] - m[1][1] * m[2][0]);
  if (!(std::fabs(det) > 1e-10)) throw Error(kErrInvalidParameter, "domain cell is singular");
  // inverse: frac = pos . inv (rows of the cell are the lattice vectors)
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      const int i1 = (j + 1) % 3, i2 = (j + 2) % 3, j1 = (i + 1) % 3, j2 = (i + 2) % 3;
      g_.inv[3 * i + j] = (m[i1][j1] * m[i2][j2] - m[i1][j2] * m[i2][j1]) / det;
    }
  // face distances: volume / |a_b x a_c|
  const double vol = std::fabs(det);
  float lcell[9];
  bool pbc[3];
  const double rc = static_cast<double>(model.cutoff()) + skin;
  for (int a = 0; a < 3; ++a) {
    const double *u = m[(a + 1) % 3], *v = m[(a + 2) % 3];
    const double cx = u[1] * v[2] - u[2] * v[1], cy = u[2] * v[0] - u[0] * v[2], cz = u[0] * v[1] - u[1] * v[0];
    const double face = vol / std::sqrt(cx * cx + cy * cy + cz * cz);
    pbc[a] = g_.p[a] == 1;
    // halo width with a relative margin for rounding at the slab faces
    g_.d1[a] = pbc[a] ? 0.0 : rc / face * (1.0 + 1e-9) + 1e-12;
    if (!pbc[a] && g_.d1[a] * 2.0 >= 1.0 / g_.p[a])
      throw Error(kErrInvalidParameter, "cell too small for this domain grid: a slab must be wider than twice "
                                        "the cutoff (plus skin)");
    const int c = a == 0 ? rank % g_.p[0] : a == 1 ? (rank / g_.p[0]) % g_.p[1] : rank / (g_.p[0] * g_.p[1]);
    g_.origin[a] = pbc[a] ? 0.0 : static_cast<double>(c) / g_.p[a] - g_.d1[a];
    // local frame: split axes span the slab plus both halos
    const double w = pbc[a] ? 1.0 : 1.0 / g_.p[a] + 2.0 * g_.d1[a];
    for (int k = 0; k < 3; ++k) lcell[3 * a + k] = static_cast<float>(m[a][k] * w);
  }
  make_grid_params(lcell, pbc, model.cutoff(), &grid_);
  check_search_extent(grid_);
  for (auto &e : ev_) CUDA_CHECK(cudaEventCreate(&e));
}

DomainEngine::~DomainEngine() {
  for (auto &e : ev_)
    if (e) cudaEventDestroy(e);
}

void DomainEngine::set_atoms(int n_own, const int32_t *numbers) {
  if (n_own < 0 || (n_own > 0 && !numbers)) throw Error(kErrInvalidParameter, "owned atoms: bad count or NULL numbers");
  std::vector<int> sp(n_own > 0 ? n_own : 1, 0);
  comp_ = 0.0;
  for (int i = 0; i < n_own; ++i) {
    if (!model_.knows_species(numbers[i]) || numbers[i] < 0 || numbers[i] >= 128)
      throw Error(kErrComputation, "Unknown atomic number " + std::to_string(numbers[i]) +
                                       " not found in species_to_index mapping");
    comp_ += model_.composition_energy(numbers[i]);
  }
  const int *zmap_dev = model_.device_species_map();
  int hz[128];
  CUDA_CHECK(cudaMemcpy(hz, zmap_dev, sizeof(hz), cudaMemcpyDeviceToHost));
  for (int i = 0; i < n_own; ++i) sp[i] = hz[numbers[i]];
  n_own_ = n_own;
  CUDA_CHECK(cudaMemcpy(species_own_.ensure(sizeof(int) * sp.size()), sp.data(), sizeof(int) * sp.size(),
                        cudaMemcpyHostToDevice));
  // the atomic numbers travel with the halo copies
  int32_t *dz = static_cast<int32_t *>(z_own_.ensure(sizeof(int32_t) * (n_own + 1)));
  if (n_own > 0) CUDA_CHECK(cudaMemcpy(dz, numbers, sizeof(int32_t) * n_own, cudaMemcpyHostToDevice));
}

std::vector<int64_t> DomainEngine::exchange_counts(const int64_t *d_send_counts, int64_t *d_recv_counts) {
  const int W = g_.world;
  std::vector<int64_t> ones(W, 1), out(W);
  alltoallv(d_send_counts, ones, d_recv_counts, ones, sizeof(int64_t), model_.stream());
  CUDA_CHECK(cudaMemcpyAsync(out.data(), d_recv_counts, sizeof(int64_t) * W, cudaMemcpyDeviceToHost, model_.stream()));
  CUDA_CHECK(cudaStreamSynchronize(model_.stream()));
  return out;
}

void DomainEngine::alltoallv(const void *send, const std::vector<int64_t> &sc, void *recv,
                             const std::vector<int64_t> &rc, size_t elem_bytes, cudaStream_t s) {
  const int32_t rc_ = comm_.alltoallv(comm_.user, send, sc.data(), recv, rc.data(), static_cast<int64_t>(elem_bytes), s);
  if (rc_ != 0) throw Error(kErrComputation, "domain exchange (alltoallv) failed with code " + std::to_string(rc_));
}

void DomainEngine::step(const float *d_pos, float *d_forces, bool grad, double *energy, double virial[6]) {
  const auto t_host = std::chrono::steady_clock::now();
  cudaStream_t s = model_.stream();
  CUDA_CHECK(cudaSetDevice(model_.device()));
  const int W = g_.world, n = n_own_;
  if (n > 0 && !d_pos) throw Error(kErrNullPointer, "NULL device positions");
  if (!species_own_.ptr) throw Error(kErrInvalidParameter, "domain_set_atoms must come before the first step");
  CUDA_CHECK(cudaEventRecord(ev_[0], s));
  int *flag = static_cast<int *>(flag_.ensure(sizeof(int) * 4));
  CUDA_CHECK(cudaMemsetAsync(flag, 0, sizeof(int), s));

  // ---- 1. halo: copies of owned atoms for every rank --------------------
  const size_t nn = static_cast<size_t>(n) + 1;
  int32_t *wrap = static_cast<int32_t *>(wrap_.ensure(sizeof(int32_t) * nn));
  const int32_t *z_own = z_own_.as<int32_t>();
  // per rank r: mask[r n + a], cnt[r n + a] (atom a's copies for r) and
  // off[r (n + 1) + a] (their exclusive scan, off[r (n + 1) + n] = total)
  uint32_t *mask = static_cast<uint32_t *>(cnt_.ensure(sizeof(uint32_t) * 2 * W * nn));
  int *cnt = reinterpret_cast<int *>(mask + W * nn);
  int *off = static_cast<int *>(off_.ensure(sizeof(int) * W * (nn + 1)));
  int64_t *counts = static_cast<int64_t *>(counts_.ensure(sizeof(int64_t) * 4 * W));
  if (n > 0) {
    k_halo_mask<<<blocks(n, 128), 128, 0, s>>>(d_pos, n, g_, mask, cnt, wrap, flag);
    CUDA_LAUNCH_CHECK();
  }
  for (int r = 0; r < W; ++r)
    scan_counts(cnt + static_cast<size_t>(r) * n, off + static_cast<size_t>(r) * nn, nullptr, n, s);
  k_rank_totals<<<1, 64, 0, s>>>(off, n, W, counts);
  CUDA_LAUNCH_CHECK();
  halo_sc_.assign(W, 0);
  CUDA_CHECK(cudaMemcpyAsync(halo_sc_.data(), counts, sizeof(int64_t) * W, cudaMemcpyDeviceToHost, s));
  halo_rc_ = exchange_counts(counts, counts + W);
  std::vector<int64_t> sb(W + 1, 0), rb(W + 1, 0);
  for (int r = 0; r < W; ++r) {
    sb[r + 1] = sb[r] + halo_sc_[r];
    rb[r + 1] = rb[r] + halo_rc_[r];
  }
  n_sent_ = static_cast<int>(sb[W]);
  n_ghost_ = static_cast<int>(rb[W]);
  int64_t *sbase = static_cast<int64_t *>(sbase_.ensure(sizeof(int64_t) * 2 * (W + 1)));
  int64_t *rbase = sbase + (W + 1);
  CUDA_CHECK(cudaMemcpyAsync(sbase, sb.data(), sizeof(int64_t) * (W + 1), cudaMemcpyHostToDevice, s));
  CUDA_CHECK(cudaMemcpyAsync(rbase, rb.data(), sizeof(int64_t) * (W + 1), cudaMemcpyHostToDevice, s));
  GhostRec *srec = static_cast<GhostRec *>(send_rec_.ensure(sizeof(GhostRec) * (n_sent_ + 1)));
  GhostRec *rrec = static_cast<GhostRec *>(recv_rec_.ensure(sizeof(GhostRec) * (n_ghost_ + 1)));
  if (n > 0) {
    k_halo_fill<<<blocks(n, 128), 128, 0, s>>>(d_pos, z_own, n, g_, mask, wrap, off, sbase, srec);
    CUDA_LAUNCH_CHECK();
  }
  alltoallv(srec, halo_sc_, rrec, halo_rc_, sizeof(GhostRec), s);
  CUDA_CHECK(cudaEventRecord(ev_[1], s));

  // ---- 2. local system, neighbour list, requests -------------------------
  const int n_local = n + n_ghost_;
  double *posl = static_cast<double *>(pos_local_.ensure(sizeof(double) * 3 * (n_local + 1)));
  int *species = static_cast<int *>(species_local_.ensure(sizeof(int) * (n_local + 1)));
  int *grank = static_cast<int *>(ghost_rank_.ensure(sizeof(int) * 2 * (n_ghost_ + 1)));
  int *gsrc = grank + (n_ghost_ + 1);
  int32_t *gimg = static_cast<int32_t *>(ghost_img_.ensure(sizeof(int32_t) * (n_ghost_ + 1)));
  if (n_local > 0) {
    k_local_build<<<blocks(n_local, 128), 128, 0, s>>>(d_pos, wrap, species_own_.as<int>(), n, rrec, rbase, n_ghost_,
                                                       g_, model_.device_species_map(), posl, species, grank, gsrc,
                                                       gimg, flag);
    CUDA_LAUNCH_CHECK();
  }
  const EdgeList &nl = model_.domain_neighbors(posl, n_local, n, grid_);
  const int E = nl.n_edges, T0 = n + E;
  int *rcnt = static_cast<int *>(req_cnt_.ensure(sizeof(int) * 2 * W));
  int *cursor = rcnt + W;
  CUDA_CHECK(cudaMemsetAsync(rcnt, 0, sizeof(int) * 2 * W, s));
  if (E > 0) {
    k_req_count<<<blocks(E, 256), 256, 0, s>>>(nl.nbr.as<int>(), E, n, grank, rcnt);
    CUDA_LAUNCH_CHECK();
  }
  std::vector<int> rc_host(W);
  CUDA_CHECK(cudaMemcpyAsync(rc_host.data(), rcnt, sizeof(int) * W, cudaMemcpyDeviceToHost, s));
  CUDA_CHECK(cudaStreamSynchronize(s));
  req_sc_.assign(rc_host.begin(), rc_host.end());
  std::vector<int64_t> qb(W + 1, 0);
  for (int r = 0; r < W; ++r) qb[r + 1] = qb[r] + req_sc_[r];
  n_req_out_ = static_cast<int>(qb[W]);  // requests sent = token rows received
  int64_t *qbase = static_cast<int64_t *>(req_base_.ensure(sizeof(int64_t) * 2 * (W + 1)));
  int64_t *qrbase = qbase + (W + 1);
  CUDA_CHECK(cudaMemcpyAsync(qbase, qb.data(), sizeof(int64_t) * (W + 1), cudaMemcpyHostToDevice, s));
  ReqRec *qsend = static_cast<ReqRec *>(req_send_.ensure(sizeof(ReqRec) * (n_req_out_ + 1)));
  int *qedge = static_cast<int *>(req_edge_.ensure(sizeof(int) * (n_req_out_ + 1)));
  int *mrow = static_cast<int *>(msg_row_buf_.ensure(sizeof(int) * (E + 1)));
  if (E > 0) {
    k_req_fill<<<blocks(E, 256), 256, 0, s>>>(nl.center.as<int>(), nl.nbr.as<int>(), nl.shift.as<int>(), E, n, wrap,
                                               grank, gsrc, gimg, qbase, cursor, T0, qsend, qedge, mrow, flag);
    CUDA_LAUNCH_CHECK();
  }
  CUDA_CHECK(cudaMemcpyAsync(counts + 2 * W, req_sc_.data(), sizeof(int64_t) * W, cudaMemcpyHostToDevice, s));
  req_rc_ = exchange_counts(counts + 2 * W, counts + 3 * W);
  std::vector<int64_t> qr(W + 1, 0);
  for (int r = 0; r < W; ++r) qr[r + 1] = qr[r] + req_rc_[r];
  n_req_in_ = static_cast<int>(qr[W]);  // requests received = token rows sent
  CUDA_CHECK(cudaMemcpyAsync(qrbase, qr.data(), sizeof(int64_t) * (W + 1), cudaMemcpyHostToDevice, s));
  ReqRec *qrecv = static_cast<ReqRec *>(req_recv_.ensure(sizeof(ReqRec) * (n_req_in_ + 1)));
  alltoallv(qsend, req_sc_, qrecv, req_rc_, sizeof(ReqRec), s);
  int *reply = static_cast<int *>(reply_edge_.ensure(sizeof(int) * (n_req_in_ + 1)));
  if (n_req_in_ > 0) {
    k_resolve<<<blocks(n_req_in_, 128), 128, 0, s>>>(qrecv, n_req_in_, qrbase, W, nl.offset.as<int>(),
                                                     nl.nbr.as<int>(), nl.shift.as<int>(), n, wrap, grank, gsrc, gimg,
                                                     reply);
    CUDA_LAUNCH_CHECK();
  }
  n_in = n_req_out_;
  msg_row = mrow;
  CUDA_CHECK(cudaEventRecord(ev_[2], s));

  // ---- 3. the model (with the token exchanges) ----------------------------
  double *red = static_cast<double *>(red_.ensure(sizeof(double) * 8));
  model_.domain_predict(species, n_local, n, this, grad, red);
  CUDA_CHECK(cudaEventRecord(ev_[3], s));

  // ---- 4. forces on ghosts back to their owners ----------------------------
  if (grad) {
    const float *F = model_.device_forces();
    float *frecv = static_cast<float *>(force_recv_.ensure(sizeof(float) * 3 * (n_sent_ + 1)));
    alltoallv(F + 3 * static_cast<size_t>(n), halo_rc_, frecv, halo_sc_, 3 * sizeof(float), s);
    if (n > 0 && d_forces) {
      k_owned_forces<<<blocks(n, 128), 128, 0, s>>>(F, frecv, n, W, cnt, off, sbase, d_forces);
      CUDA_LAUNCH_CHECK();
    }
  }
  CUDA_CHECK(cudaEventRecord(ev_[4], s));

  // ---- 5. energy (with composition) and virial summed over the ranks ------
  double *hred = static_cast<double *>(h_.ensure(sizeof(double) * 8 + sizeof(int) * 4));
  hred[7] = comp_;
  CUDA_CHECK(cudaMemcpyAsync(red + 7, hred + 7, sizeof(double), cudaMemcpyHostToDevice, s));
  const int32_t ar = comm_.allreduce_sum_f64(comm_.user, red, 8, s);
  if (ar != 0) throw Error(kErrComputation, "domain exchange (allreduce) failed with code " + std::to_string(ar));
  CUDA_CHECK(cudaMemcpyAsync(hred, red, sizeof(double) * 8, cudaMemcpyDeviceToHost, s));
  int *hflag = reinterpret_cast<int *>(hred + 8);
  CUDA_CHECK(cudaMemcpyAsync(hflag, flag, sizeof(int), cudaMemcpyDeviceToHost, s));
  CUDA_CHECK(cudaEventRecord(ev_[5], s));
  CUDA_CHECK(cudaStreamSynchronize(s));
  n_in = 0;
  msg_row = nullptr;
  model_.check_device_error(grad);
  if (*hflag & 1) throw Error(kErrInvalidParameter, "an owned atom lies more than 511 cells from the cell");
  if (*hflag & 2) throw Error(kErrComputation, "a ghost atom has an atomic number the model does not know");
  if (*hflag & 4) throw Error(kErrInvalidParameter, "an edge's image shift exceeds 511 cells");
  *energy = hred[0] + hred[7];
  for (int c = 0; c < 6; ++c) virial[c] = grad ? hred[1 + c] : 0.0;

  float ms = 0.f;
  for (int k = 0; k < 5; ++k) {
    CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[k], ev_[k + 1]));
    stats_.ms[k] = ms;
  }
  CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[0], ev_[5]));
  stats_.ms[5] = ms;
  stats_.ms[6] = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_host).count();
  stats_.n_own = n;
  stats_.n_ghost = n_ghost_;
  stats_.n_edges = E;
  stats_.n_req_out = n_req_out_;
  stats_.n_req_in = n_req_in_;
  stats_.n_sent = n_sent_;
}

void DomainEngine::exchange_tokens(float *x0, int N0, int T0, int d, cudaStream_t s) {
  if (d % 4) throw Error(kErrInternal, "token rows must be multiples of 4 floats");
  float *send = static_cast<float *>(tok_send_.ensure(sizeof(float) * d * (static_cast<size_t>(n_req_in_) + 1)));
  if (n_req_in_ > 0) {
    k_gather_rows<<<row_blocks(n_req_in_), 256, 0, s>>>(x0, N0, reply_edge_.as<int>(), n_req_in_, d, 1.0f, send);
    CUDA_LAUNCH_CHECK();
  }
  alltoallv(send, req_rc_, x0 + static_cast<size_t>(T0) * d, req_sc_, sizeof(float) * d, s);
}

void DomainEngine::exchange_token_grads(const float *dmsg, float *dx, int N0, int d, cudaStream_t s) {
  float *gs = static_cast<float *>(grad_send_.ensure(sizeof(float) * d * (static_cast<size_t>(n_req_out_) + 1)));
  float *gr = static_cast<float *>(grad_recv_.ensure(sizeof(float) * d * (static_cast<size_t>(n_req_in_) + 1)));
  // the message is 0.5 (embedding + token): its token gradient is 0.5 dmsg
  if (n_req_out_ > 0) {
    k_gather_rows<<<row_blocks(n_req_out_), 256, 0, s>>>(dmsg, 0, req_edge_.as<int>(), n_req_out_, d, 0.5f, gs);
    CUDA_LAUNCH_CHECK();
  }
  alltoallv(gs, req_sc_, gr, req_rc_, sizeof(float) * d, s);
  if (n_req_in_ > 0) {
    k_scatter_add_rows<<<row_blocks(n_req_in_), 256, 0, s>>>(gr, reply_edge_.as<int>(), n_req_in_, d, N0, dx);
    CUDA_LAUNCH_CHECK();
  }
}

}  // namespace pet
