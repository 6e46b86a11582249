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
  EPI_SILU = 1,     // z = acc + bias: C = silu(z), Z[m] = silu'(z) (kept for the backward)
  EPI_ACCUM = 2,    // C += acc + bias
  EPI_DSILU = 3,    // C = acc * Z[m]  (Z = silu' from the forward)
  EPI_RESID = 4,    // C = acc + bias + R[row_c(m)]
};

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
};

// Dense fp32 GEMM (exact fp32 FFMA accumulation).
void gemm_f32(const GemmArgs &a, cudaStream_t stream);

// ---- attention over each atom's token block -------------------------------
struct AttnArgs {
  const float *qkv;       // [T, 3d]  (q | k | v, heads contiguous)
  float *out;             // [T, d]   forward output
  const float *d_out;     // [T, d]   backward: upstream grad
  float *d_qkv;           // [T, 3d]  backward: result
  float *lse;             // [T, heads] row log-sum-exp (forward writes, backward reads)
  const float *key_mask;  // [E] additive mask of each edge key (node key: 0)
  const int *offset;      // [N+1] edge offsets (CSR)
  int n_atoms, d, heads, max_tokens;
};
void attention_fwd(const AttnArgs &a, cudaStream_t stream);
void attention_bwd(const AttnArgs &a, cudaStream_t stream);
// Largest per-atom token count the attention kernels accept for head size hd.
int attention_max_tokens(int hd);

// ---- row-wise ops ---------------------------------------------------------
// y = (x - mean) / sqrt(var * (1 + eps)) * g + b  (pet_layers.cpp:85-145)
void layer_norm_fwd(const float *x, const float *g, const float *b, float *y, float *xhat,
                    float *rstd, int rows, int d, cudaStream_t stream);
// dx = rstd (dxhat - mean(dxhat) - (1 + eps) xhat mean(dxhat xhat)), dxhat = dy g
void layer_norm_bwd(const float *dy, const float *xhat, const float *rstd, const float *g,
                    float *dx, int rows, int d, cudaStream_t stream);

}  // namespace pet
