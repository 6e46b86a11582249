// GPU cell-list neighbour search, bit-exact with mlip.cpp's
// NeighborListBuilder (src/core/neighbor_list.cpp:126-297).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace pet {

// Bin grid of one periodic cell, computed on the host in fp64 with the
// reference's operation order (CellGrid ctor, neighbor_list.cpp:38-66).
struct GridParams {
  double inv[9];     // f32 cofactor inverse widened to f64 (system.cpp:19-48)
  double bv[9];      // bin vectors: bv[3*a + xyz] = cell[a] * (1.0 / nb[a])
  int nb[3];         // bins per axis
  int ns[3];         // search half-width per axis
  int pbc[3];
  double cutoff_sq;  // (double)cutoff squared in f64 (periodic path)
};

// `cutoff` must be finite and positive (the callers check it).
void make_grid_params(const float cell[9], const bool pbc[3], float cutoff, GridParams *g);

// Largest search half-width per axis (bin offsets are packed in 10 bits).
constexpr int kMaxSearchBins = 511;
// Throws Error(kErrInvalidParameter) when a cutoff spans more than
// kMaxSearchBins bins along an axis.
void check_search_extent(const GridParams &g);
// Throws Error(kErrInvalidParameter) when n_centers x max_count may exceed
// the int32 pair offsets.
void check_pair_total(int max_count, int n_centers);
void cell_inverse_f32(const float m[9], float inv[9]);

// Edges of a neighbour list in centre-major order (the reference's slot
// order inside each centre), SoA, sized by `ensure`.
struct EdgeList {
  int n_atoms = 0;
  int n_edges = 0;
  int max_count = 0;
  DevBuf count, offset;        // [N], [N+1]
  DevBuf center, nbr, shift;   // [E], [E], [3E]
  DevBuf vec, dist;            // [3E] f32, [E] f32
};

struct NLScratch {
  DevBuf braw, bin_of, bin_count, bin_start, bin_cursor, bin_atoms, scan_aux;
};

// Build the full list (no self pairs) for one periodic system.  `pos` is a
// device [N,3] f32 array.  Synchronises once on `stream` to size the edge
// arrays.  Raises Error on failure.
void build_periodic_nl(const float *pos, int n, const GridParams &g, EdgeList &out,
                       NLScratch &s, cudaStream_t stream);

// Local system of a spatial domain: n atoms with f64 positions (owned
// atoms, then ghost shells, images already placed), pairs found with the
// grid search of a non-periodic bounding cell (g.pbc all 0), only for the
// first n_centers atoms (all n atoms are candidate neighbours).
void build_local_nl(const double *pos, int n, int n_centers, const GridParams &g, EdgeList &out,
                    NLScratch &s, cudaStream_t stream);

// Open-boundary O(n^2) search, batched: atom a belongs to the system whose
// atoms are [sys_begin[a], sys_end[a]).  `cutoff_sq_f32` is the f32 product
// cutoff*cutoff the reference compares against (neighbor_list.cpp:131).
void build_open_nl(const float *pos, const int *sys_begin, const int *sys_end, int n,
                   float cutoff, EdgeList &out, NLScratch &s, cudaStream_t stream);

// ---- Verlet lists: a list built with cutoff + skin, kept across calls -------
// Cell geometry of a kept list: the lattice (rows) and its inverse in f64
// and the periodic axes (a non-periodic system has pbc all 0).
struct SkinGeom {
  double cell[9], inv[9];
  int pbc[3];
};
// Displacement of every atom since the list was built, modulo the cell:
// img[a] (3 ints) = the lattice translation k that brings pos[a] + k cell
// nearest to ref[a] along periodic axes, so that wrapping an atom back
// into the cell is not a move.  *d_max2 (device, bits of a non-negative
// float) receives the largest |pos + k cell - ref|^2; the caller zeroes it
// first.
void skin_displacement(const float *pos, const float *ref, int n, const SkinGeom &g, int *img,
                       unsigned *d_max2, cudaStream_t stream);
// Vectors and distances of the kept pairs at the current positions:
// vec = pos[j] - pos[i] + (shift + img[j] - img[i]) cell in f64, rounded to
// f32 (vec) and f32(sqrt) (dist), the arithmetic of a fresh build up to the
// order of its additions.
void refresh_edges(const float *pos, int n_edges, const int *center, const int *nbr, const int *shift,
                   const int *img, const SkinGeom &g, float *vec, float *dist, cudaStream_t stream);

// Periodic (or partially periodic) search that allocates nothing, for
// callers that own all device memory.  Positions and the five pair arrays
// are the caller's device buffers on the current device; the working memory
// is one fixed static device array per device (7 kNoAllocMaxAtoms +
// 3 kNoAllocMaxBins ints, 2.6 MB), whose address the first call on a
// device looks up.  Throws Error(kErrInvalidParameter) above either limit.
// Returns the total pair count; the arrays are written only when it is at
// most `cap`.  Synchronises `stream`, and all of its work has finished when
// it returns.  Calls on one device share the array: calls that overlap in
// time (other host threads) race.
constexpr int kNoAllocMaxAtoms = 65536;
constexpr int kNoAllocMaxBins = 65536;
int64_t build_periodic_nl_noalloc(const float *pos, int n, const GridParams &g, int64_t cap,
                                  int *e_center, int *e_nbr, int *e_shift, float *e_vec, float *e_dist,
                                  cudaStream_t stream);

// Exclusive scan of n int32 counts into out[0..n] (out[n] = total) and the
// maximum count into *max_out (device scalars); single CTA.
void scan_counts(const int *in, int *out, int *max_out, int n, cudaStream_t stream);

}  // namespace pet
