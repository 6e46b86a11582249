// Per-edge and per-atom kernels of the PET pass (graph preparation,
// featuriser, message passing, readout, gradients, forces, virial).
#pragma once

#include <cuda_runtime.h>

#include "kernels.cuh"

namespace pet {

struct EdgePrepArgs {
  int n_atoms, n_edges;
  const int *offset, *center, *nbr, *shift, *species;
  const float *vec, *dist_nl;
  float cutoff, width;
  // outputs
  float *r, *fc, *dfc_dr, *key_mask;
  int *nbr_species, *rev;
};
// r, f_c and df_c/dr in-graph (pet.cpp:208-256); the fp16 log-cutoff key
// mask from the neighbour-list distance (pet_batch.cpp:37-47,603-653); token
// neighbour species; reverse edge (pet_batch.cpp:399-495).
void edge_prep(const EdgePrepArgs &a, cudaStream_t s);

// Input rows of the compression's first linear (build_tokens,
// pet_layers.cpp:685-796).  The reference concatenates the edge embedding
// W_e [x y z r] + b_e (pet_layers.cpp:151-217), the neighbour-species
// embedding (embedding[nbr species] in layer 0, pet.cpp:789-832;
// neighbor_embedder[nbr species] in layer 1) and, in layer 1, the message
// 0.5 (embedding[nbr species] + X0[row(rev e)]) (pet_layers.cpp:608-679).
// The first two enter compress.0 linearly, so the model folds their
// products with its weight into a fused weight at load, and the rows here
// carry only what those products multiply:
//   layer 1: cat[e, 0:d] = the message;
//   then `aux` columns: x, y, z, r, 1, one-hot(nbr species), zeros.
struct FeaturizeArgs {
  int n_edges, d, layer, aux;
  const float *vec, *r;
  const int *nbr_species, *rev;
  const float *emb0, *x_prev;  // x_prev: layer-0 output tokens, edge e at row prev_base + e
  int prev_base;
  // optional [n_edges]: the x_prev row of edge e's message where it is not
  // prev_base + rev[e] (a reverse edge held by another spatial domain, its
  // token received after the layer-0 rows); -1 where rev[e] applies
  const int *msg_row = nullptr;
  float *cat;
  Split16View cat_split;  // if set, cat is written in split-fp16 form only
};
void featurize(const FeaturizeArgs &a, cudaStream_t s);
// Columns of a featurised row: the message (layer 1) plus the auxiliary block.
__host__ __device__ inline int featurize_cols(int layer, int d, int aux) { return (layer > 0 ? d : 0) + aux; }

// X[i, :] = table[species[i], :] for the n node-token rows (xs: the same
// rows in split form too)
void node_tokens(const float *table, const int *species, float *x, int n,
                 int d, cudaStream_t s, const Split16View *xs = nullptr);

// pred[m] = dot(y[m, :], w) + b
void head_last(const float *y, const float *w, const float *b, float *pred, int rows, int r,
               cudaStream_t s);
// dz[m, c] = w[c] z[m, c] scale[m], z = silu' of the forward pre-activation
// (scale null -> 1)
// (dzs: write dz in split form only; dz unused)
void head_last_bwd(const float *z, const float *w, const float *scale, float *dz, int rows, int r,
                   cudaStream_t s, const Split16View *dzs = nullptr);
// e_atom[i] (+)= node_pred[i] + sum_{e in i} edge_pred[e] fc[e]
void atom_energy(const float *node_pred, const float *edge_pred, const float *fc, const int *offset,
                 float *e_atom, int n, bool accumulate, cudaStream_t s);
// gfc[e] (+)= edge_pred[e]
void add_vec(const float *x, float *y, int n, bool accumulate, cudaStream_t s);

// g4[e, 0:4] (+)= P^T dz[e]: the gradient of the compression pre-activation
// with respect to [x y z r] of each edge, P [H][4] being the fused weight's
// x, y, z, r columns (i.e. compress.0's edge-embedding block times W_e).
// dz is [n_edges][H] fp32, or in split form when dzs is given.
void edge_xyzr_bwd(const float *dz, const Split16View *dzs, const float *P, float *g4, int n_edges, int H,
                   bool accumulate, cudaStream_t s);
// dX[base + x, :] += 0.5 dmsg[rev[x], :]   for 0 <= rev[x] < n_msg
void message_bwd(const float *dmsg, int ld, const int *rev, int base, float *dx,
                 int n_edges, int n_msg, int d, cudaStream_t s);
// g[e] = g4[e, 0:3] + (g4[e, 3] + gfc[e] dfc_dr[e]) vec[e] / r[e]
void edge_grad(const float *g4, const float *gfc, const float *dfc_dr, const float *vec,
               const float *r, float *g, int n_edges, cudaStream_t s);
// F[i] = sum_{e in i} g[e] - sum_{e : nbr[e] = i} g[e]   (pet.cpp:965-998)
void forces(const float *g, const int *offset, const int *nbr, const int *rev, float *F, int n,
            int n_edges, cudaStream_t s);
// Per system k: virial[k][6] = sum over its edges of sym(vec (x) g) (Voigt),
// energy[k] = sum of its atomic energies (both in f64).
// A single structure (n_sys == 1 with `partial`, scratch of
// kReduceMaxParts x 7 doubles: n_atoms atoms and n_edges edges) is summed by
// a deterministic two-stage reduction over the whole GPU.
constexpr int kReduceMaxParts = 1024;
void reduce_systems(const float *vec, const float *g, const float *e_atom, const int *offset,
                    const int *sys_atom_begin, int n_sys, double *virial, double *energy,
                    bool with_virial, cudaStream_t s, int n_atoms = 0, int n_edges = 0,
                    double *partial = nullptr);

// Non-conservative property readout of one layer (build_property_output,
// pet_layers.cpp:845-915), warp per atom i < n:
//   dst[i, o] += yn[i] . wn[o] + bn[o] + sum_{e in i} fc[e] (ye[e] . we[o] + be[o])
// yn [n, r], ye [edges, r]: the heads' second hidden layer (ye null: no
// edges); wn, we [od, r] and bn, be [od]: the last layers; od <= 9.
void nc_readout(const float *yn, const float *ye, const float *wn, const float *bn, const float *we,
                const float *be, const float *fc, const int *offset, float *dst, int n, int r, int od,
                cudaStream_t s);
// Per system k: out[6k..6k+5] = Voigt (xx yy zz yz xz xy) sum of the per-atom
// 3x3 tensors S [n, 9] over its atoms, off-diagonals symmetrised
// (pet.cpp:621-666), in f64.
void nc_stress_reduce(const float *S, const int *sys_atom_begin, int n_sys, double *out, cudaStream_t s);

// out[0] = sum of e_atom[0..n_energy), out[1..6] = Voigt sum over edges
// [0, n_edges) of sym(vec (x) g) (f64, two-stage; partial: scratch of
// kReduceMaxParts x 7 doubles).
void reduce_local(const float *vec, const float *g, const float *e_atom, int n_energy, int n_edges,
                  double *out, double *partial, cudaStream_t s);

}  // namespace pet
