// Kernel entry points of the PET forward/backward pass.  Every dense layer
// is one "TN" GEMM  C[m, n] = sum_k A[row_a(m), k] * B[n, k]  (both operands
// K-contiguous; backward passes use pre-transposed weights) with a fused
// epilogue.  Token rows are ragged per atom: atom i owns rows
// [off_i + i, off_i + i + 1 + n_i): its node token, then its n_i edge tokens
// in neighbour-list slot order (no padding to a global max_neighbors).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace pet {

enum Epilogue : int {
  EPI_STORE = 0,    // C = acc + bias
  EPI_SILU = 1,     // z = acc + bias: C = silu(z), Z[m] = silu'(z) (kept for the backward; Z may be null)
  EPI_ACCUM = 2,    // C += acc + bias
  EPI_DSILU = 3,    // C = acc * Z[m]  (Z = silu' from the forward)
  EPI_RESID = 4,    // C = acc + bias + R[row_c(m)]
};

// A matrix in split-fp16 form (split16.cuh): hi, lo [rows][cols] fp16 and
// scale exponents sc [cols / 128][rows].  hi == nullptr: none.  lo ==
// nullptr with hi set: the hi parts only, for a matrix whose only reader is
// a one-product (reduced-precision) GEMM; writers then skip the lo parts.
struct Split16View {
  uint16_t *hi = nullptr;
  uint16_t *lo = nullptr;
  int8_t *sc = nullptr;
  int rows = 0, cols = 0;
  int ld = 0;  // scale entries between consecutive 128-column blocks (0: rows)
};
// Scale of (row, block): sc[block * split_ld(v) + row].
__host__ __device__ inline int split_ld(const Split16View &v) { return v.ld ? v.ld : v.rows; }
// Rows [r0, r0 + n) of v as a view of its own.
inline Split16View split_rows(const Split16View &v, int r0, int n) {
  Split16View o = v;
  o.hi = v.hi + static_cast<size_t>(r0) * v.cols;
  o.lo = v.lo ? v.lo + static_cast<size_t>(r0) * v.cols : nullptr;
  o.sc = v.sc + r0;
  o.rows = n;
  o.ld = split_ld(v);
  return o;
}

struct GemmArgs {
  const float *A = nullptr;
  int lda = 0;
  const int *a_rows = nullptr;  // optional row gather for A
  const float *B = nullptr;     // [N, K] row-major
  int ldb = 0;
  float *C = nullptr;
  int ldc = 0;
  const int *c_rows = nullptr;  // optional row scatter for C (and R)
  int M = 0, N = 0, K = 0;
  const float *bias = nullptr;  // [N] or null
  float *Z = nullptr;           // EPI_SILU (write) / EPI_DSILU (read), rows m
  int ldz = 0;
  const float *R = nullptr;     // EPI_RESID residual, rows row_c(m)
  int ldr = 0;
  int epi = EPI_STORE;
  // 3xFP16 only.  a_split: split form of A ([M, K]); a_split_ready = it
  // already holds A (else the GEMM first writes A, row-gathered, into it).
  // c_split: also write the result in split form (rows row_c(m)); C may
  // then be null.
  Split16View a_split;
  bool a_split_ready = false;
  Split16View c_split;
  Split16View r_split;  // EPI_RESID: residual in split form (rows m) instead of R
  // Failure-detection test hook (3xFP16 kernel): the producer of this CTA
  // issues no loads, so its MMA warp's bounded wait runs out; -1: none.
  int stall_cta = -1;
};

// Dense fp32 GEMM (exact fp32 FFMA accumulation).
void gemm_f32(const GemmArgs &a, cudaStream_t stream);

// ---- attention over each atom's token block -------------------------------
// Token rows of a GNN layer: node token of atom i at row i, the token of
// edge e (CSR order) at row edge_base + e; atom i's sequence is its node
// token, then its edges.
struct AttnArgs {
  const float *qkv;       // [T, 3d]  (q | k | v, heads contiguous)
  float *out;             // [T, d]   forward output
  const float *d_out;     // [T, d]   backward: upstream grad
  float *d_qkv;           // [T, 3d]  backward: result
  float *lse;             // [T, heads] row log-sum-exp (forward writes, backward reads)
  const float *key_mask;  // [E] additive mask of each edge key (node key: 0)
  const int *offset;      // [N+1] edge offsets (CSR)
  int n_atoms, d, heads, max_tokens;
  int edge_base;          // token row of edge 0
  // Optional split-fp16 outputs (then out / d_qkv may be null): the forward
  // output [T, d] and the backward result [T, 3d].  Needs 128 / head size
  // heads per CTA, one 128-column block.
  Split16View out_split;
  Split16View dqkv_split;
  // Optional split of the atoms by sequence length (tensor-core kernels
  // only): the n_short atoms in short_atoms have at most
  // attention_short_tokens() tokens and run on the kernels for short
  // sequences, the n_long in long_atoms on the others.  Null: one class
  // chosen by max_tokens.  `atoms` (set per launch): the atom of each CTA
  // row of the grid, null for the identity.
  const int *short_atoms = nullptr, *long_atoms = nullptr;
  int n_short = 0, n_long = 0;
  const int *atoms = nullptr;
};
// Row of token k (0: the node) of one atom's sequence.
struct AtomRows {
  int node, ebase;  // ebase + k is the row of token k >= 1
  __host__ __device__ int operator()(int k) const { return k == 0 ? node : ebase + k; }
};
__host__ __device__ inline AtomRows atom_rows(int atom, int e0, int edge_base) {
  return AtomRows{atom, edge_base + e0 - 1};
}
void attention_fwd(const AttnArgs &a, cudaStream_t stream);
void attention_bwd(const AttnArgs &a, cudaStream_t stream);
// Tensor-core forward / backward on register-resident split-fp16 products
// (attention_mma.cu): head size 32, at most 64 tokens per atom; split
// outputs need heads in groups of 4 (one cluster per 128-column block).
bool attention_mma_supported(const AttnArgs &a, bool bwd);
void attention_mma(const AttnArgs &a, bool bwd, cudaStream_t stream);
// Longest sequence the short-sequence tensor-core kernels take.
int attention_short_tokens();
// Atoms [0, n) split by sequence length (edges + 1 from the CSR offsets):
// at most `short_tokens` into short_atoms, the rest into long_atoms, in
// ascending order within each warp of 32 atoms; counts[0..1] (device,
// zeroed by the caller) receive the two class sizes.
void attention_classes(const int *offset, int n, int short_tokens, int *short_atoms, int *long_atoms,
                       int *counts, cudaStream_t stream);
// Largest per-atom token count the attention kernels accept for head size hd.
int attention_max_tokens(int hd);
// Largest tokens per atom for which the attention kernels can write
// split-fp16 outputs (128 / hd heads per CTA); 0 if hd does not divide 128.
int attention_split_max_tokens(int hd);

// ---- row-wise ops ---------------------------------------------------------
// y = (x - mean) / sqrt(var * (1 + eps)) * g + b  (pet_layers.cpp:85-145);
// stats [2 rows]: each row's mean, then its 1 / sqrt(var (1 + eps)); y may be
// null when ys is given; ys: also write y in split-fp16 form (d a multiple
// of 128, at most 1024)
void layer_norm_fwd(const float *x, const float *g, const float *b, float *y, float *stats, int rows, int d,
                    cudaStream_t stream, const Split16View *ys = nullptr);
// dx = rstd (dxhat - mean(dxhat) - (1 + eps) xhat mean(dxhat xhat)), dxhat = dy g,
// with xhat = (x - mean) rstd recomputed from the forward's input x and its
// stats; dxs: also write dx in split-fp16 form
void layer_norm_bwd(const float *dy, const float *x, const float *stats, const float *g, float *dx, int rows, int d,
                    cudaStream_t stream, const Split16View *dxs = nullptr);

}  // namespace pet
