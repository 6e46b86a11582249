// Per-atom multi-head attention, forward and backward, on register-resident
// tensor-core products (mma.sync m16n8k16, fp16 inputs, fp32 accumulation)
// in split-fp16 form: x 2^s = hi + lo and every product is the sum
// hi.lo + lo.hi + hi.hi, which carries about 22 significant bits, as in the
// 3xFP16 GEMM.  Head size 32, at most 64 tokens per atom.
//
// Reference: build_multi_head_attention, src/models/pet/pet_layers.cpp:318-492
// (softmax(Q K^T / sqrt(hd) + mask) V per atom, the key mask shared by all
// queries); each atom attends over its own S = n + 1 tokens only.
//
// Why this form: a per-atom block is at most 64 x 64.  tcgen05 works on 64-
// or 128-row tiles whose accumulators live in tensor memory and whose
// operands must be in shared memory, so every P and dS block would make a
// round trip TMEM -> registers -> shared memory between products (measured:
// 9.4 ms per forward against 6.1 ms for the SIMT kernel, in an earlier
// tcgen05 forward kept in this repository's history).
// Here the scores, P, dP and dS of a 16-row strip stay in the registers of
// one warp, and the accumulator layout of one product is the operand layout
// of the next.
//
// A CTA is one (atom, head), 4 warps.  Q, K, V (and dO) of the head are
// converted once into split-fp16 shared-memory blocks [64][40] (80-byte rows,
// conflict-free for ldmatrix), one power-of-two scale per block.
//   forward, warp w = query rows 16w..16w+15:
//     S = Q K^T, softmax along the row (quad shuffles), lse, O = P V;
//   backward, pass 1, warp w = query rows:
//     S, P (from lse), dP = dO V^T, D = rowsum(P o dP), dS = P o (dP - D),
//     dQ = s dS K;
//   backward, pass 2, warp w = key rows (transposed recomputation):
//     S^T = K Q^T, P^T, dP^T = V dO^T, dS^T, dV = P^T dO, dK = s dS^T Q.
// P enters a product at the fixed scale 2^14; dS with one scale per warp
// strip.  The exponentials of P use the __expf intrinsic: its few-ulp
// error is at the level of the ~22 significant bits P keeps in split form.  Split-fp16 outputs need one scale per (row, 128-column block),
// i.e. per 4 heads: those 4 CTAs form a cluster; each pushes its row
// maxima into every CTA's shared memory (remote atomic max) between the two
// halves of one cluster barrier, so no CTA reads another's memory.
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"
#include "split16.cuh"

namespace pet {
namespace {

constexpr int kHd = 32;
constexpr int kMaxTok = 64;
constexpr int kPitch = 40;                  // halves per shared-memory row (80 bytes)
constexpr int kMat = kMaxTok * kPitch;      // halves per [64][40] block
constexpr int kThreads = 128;

// ---- small helpers --------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], uint32_t a) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], uint32_t a) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
// c += a b  (16 x 8 x 16, fp16 in, fp32 accumulate).  A register-only
// operation: not volatile, so independent products can be interleaved.
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// c += (ah + al)(bh + bl) without the al bl term
__device__ __forceinline__ void mma3(float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0,
                                     uint32_t bh1, uint32_t bl0, uint32_t bl1) {
  mma16816(c, ah, bl0, bl1);
  mma16816(c, al, bh0, bh1);
  mma16816(c, ah, bh0, bh1);
}

// Address for ldmatrix.x4 of the 16 x 16 block at (r0, c0) of a [64][40]
// fp16 block, A-operand order: matrices (r0, c0), (r0 + 8, c0), (r0, c0 + 8),
// (r0 + 8, c0 + 8) -> a0..a3.
__device__ __forceinline__ uint32_t a_addr(uint32_t base, int r0, int c0, int lane) {
  const int j = lane >> 3;
  return base + 2u * static_cast<uint32_t>((r0 + (lane & 7) + 8 * (j & 1)) * kPitch + c0 + 8 * (j >> 1));
}
// B operand of two n-tiles from an [n][k] block (rows = the product's
// columns): matrices (n0, k0), (n0, k0 + 8), (n0 + 8, k0), (n0 + 8, k0 + 8)
// -> b0, b1 of tile n0 and b0, b1 of tile n0 + 8.
__device__ __forceinline__ uint32_t bn_addr(uint32_t base, int n0, int k0, int lane) {
  const int j = lane >> 3;
  return base + 2u * static_cast<uint32_t>((n0 + (lane & 7) + 8 * (j >> 1)) * kPitch + k0 + 8 * (j & 1));
}
// B operand of two n-tiles from a [k][n] block, with ldmatrix.trans:
// matrices (k0, n0), (k0 + 8, n0), (k0, n0 + 8), (k0 + 8, n0 + 8).
__device__ __forceinline__ uint32_t bk_addr(uint32_t base, int k0, int n0, int lane) {
  const int j = lane >> 3;
  return base + 2u * static_cast<uint32_t>((k0 + (lane & 7) + 8 * (j & 1)) * kPitch + n0 + 8 * (j >> 1));
}

// Accumulator tiles (c-layout) 2t and 2t + 1 as the A fragment of k-step t,
// in split form at scale f.
__device__ __forceinline__ void c_to_a(const float (&c0)[4], const float (&c1)[4], float f, uint32_t (&ah)[4],
                                       uint32_t (&al)[4]) {
  split2(c0[0], c0[1], f, ah[0], al[0]);
  split2(c0[2], c0[3], f, ah[1], al[1]);
  split2(c1[0], c1[1], f, ah[2], al[2]);
  split2(c1[2], c1[3], f, ah[3], al[3]);
}

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}
__device__ __forceinline__ float warp_absmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- cluster helpers (split outputs) -----------------------------------------
__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of a cluster barrier: arrive once this CTA's row maxima are
// cleared, wait just before writing into the peers' (they have long arrived).
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// max into the same shared variable of cluster CTA `rank`
__device__ __forceinline__ void red_max_peer(int *local, uint32_t rank, int v) {
  const uint32_t a = smem_addr(local);
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  asm volatile("red.shared::cluster.max.u32 [%0], %1;" ::"r"(r), "r"(v) : "memory");
}

// ---- shared memory -------------------------------------------------------------
struct Smem {
  uint16_t mat[8][kMat];  // Q, K, V, dO: hi then lo ([0..3] hi, [4..7] lo)
  float lse[kMaxTok], mask[kMaxTok], D[kMaxTok];
  int scale[4];           // block scale exponents of Q, K, V, dO
  int rmax[3][kMaxTok];   // row maxima of the outputs (bits of non-negative floats)
};

// Q, K, V (and dO when `grad`) of (atom, head) into split-fp16 blocks; warp
// w converts block w (rows past S are zero) with one scale from its maximum.
__device__ __forceinline__ void load_blocks(Smem &sm, const AttnArgs &a, AtomRows tr, int S, int h, bool grad) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < 3 || grad) {
    float v[8][8];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      if (r < S) {
        const float *src = warp < 3 ? a.qkv + static_cast<size_t>(tr(r)) * 3 * a.d + warp * a.d + h * kHd + c
                                    : a.d_out + static_cast<size_t>(tr(r)) * a.d + h * kHd + c;
        const float4 x0 = *reinterpret_cast<const float4 *>(src), x1 = *reinterpret_cast<const float4 *>(src + 4);
        v[i][0] = x0.x; v[i][1] = x0.y; v[i][2] = x0.z; v[i][3] = x0.w;
        v[i][4] = x1.x; v[i][5] = x1.y; v[i][6] = x1.z; v[i][7] = x1.w;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) mx = fmaxf(mx, fabsf(v[i][k]));
    }
    const int s = split_scale_exponent(warp_absmax(mx));
    const float f = pow2f(s);
    if (lane == 0) sm.scale[warp] = s;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      uint32_t hh[4], ll[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) split2(v[i][2 * k], v[i][2 * k + 1], f, hh[k], ll[k]);
      *reinterpret_cast<uint4 *>(&sm.mat[warp][r * kPitch + c]) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
      *reinterpret_cast<uint4 *>(&sm.mat[4 + warp][r * kPitch + c]) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
    }
  }
}

// Row maxima of a 16-row strip's outputs (4 n-tiles of the c-layout) into
// rm of every CTA of the cluster (quad-reduced, one remote max per row and
// CTA), so that after the next cluster barrier rm holds the block maxima.
__device__ __forceinline__ void strip_rowmax(int *rm, const float (&o)[4][4], int r0, int S, int lane) {
  float m0 = 0.f, m1 = 0.f;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    m0 = fmaxf(m0, fmaxf(fabsf(o[n][0]), fabsf(o[n][1])));
    m1 = fmaxf(m1, fmaxf(fabsf(o[n][2]), fabsf(o[n][3])));
  }
  m0 = quad_max(m0);
  m1 = quad_max(m1);
  const int g = lane >> 2;
  if ((lane & 3) == 0) {
#pragma unroll
    for (uint32_t c = 0; c < 4; ++c) {
      if (r0 + g < S) red_max_peer(rm + r0 + g, c, __float_as_int(m0));
      if (r0 + g + 8 < S) red_max_peer(rm + r0 + g + 8, c, __float_as_int(m1));
    }
  }
}

// Store a 16-row strip (4 n-tiles, columns col0 + 8n + 2 tig) as fp32 into
// dst (row pitch ld) or, when `o` is set, in split form with the block
// scales from the cluster's row maxima `rm`.
__device__ __forceinline__ void strip_store(const float (&v)[4][4], int r0, int S, AtomRows tr, int lane, float *dst,
                                            size_t ld, int col0, const Split16View *o, const int *rm, int blk,
                                            bool write_scale) {
  const int g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = r0 + g + 8 * half;
    if (r >= S) continue;
    if (dst) {
      float *p = dst + static_cast<size_t>(tr(r)) * ld + col0 + 2 * tig;
#pragma unroll
      for (int n = 0; n < 4; ++n) *reinterpret_cast<float2 *>(p + 8 * n) = make_float2(v[n][2 * half], v[n][2 * half + 1]);
    }
    if (o) {
      const int s = split_scale_exponent(__int_as_float(rm[r]));
      const float f = pow2f(s);
      const size_t off = static_cast<size_t>(tr(r)) * o->cols + col0 + 2 * tig;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        uint32_t hh, ll;
        split2(v[n][2 * half], v[n][2 * half + 1], f, hh, ll);
        *reinterpret_cast<uint32_t *>(o->hi + off + 8 * n) = hh;
        if (o->lo) *reinterpret_cast<uint32_t *>(o->lo + off + 8 * n) = ll;
      }
      if (write_scale && tig == 0) o->sc[static_cast<size_t>(blk) * split_ld(*o) + tr(r)] = static_cast<int8_t>(s);
    }
  }
}

// Split-fp16 stores of a warp's 16-row strip through shared memory: the
// 16 x 32 block of one output (hi and lo parts, 1 KB each) is staged with
// the 16-byte chunks of each row XOR-swizzled by (row & 3), then written
// out in 16-byte stores, four lanes per row covering its 64 contiguous
// bytes, instead of 4-byte stores spread over eight rows.  lo == nullptr:
// the hi parts only.  Row scales and their bytes as in strip_store.
__device__ __forceinline__ void strip_stage(const float (&v)[4][4], int r0, int S, AtomRows tr, int lane,
                                            uint16_t *hi, uint16_t *lo, const int *rm, const Split16View &o,
                                            int blk, bool write_scale) {
  const int g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int lr = g + 8 * half, r = r0 + lr;
    const int s = r < S ? split_scale_exponent(__int_as_float(rm[r])) : 0;
    const float f = pow2f(s);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      uint32_t hh, ll;
      split2(v[n][2 * half], v[n][2 * half + 1], f, hh, ll);
      const int off = lr * 32 + ((n ^ (lr & 3)) << 3) + 2 * tig;
      *reinterpret_cast<uint32_t *>(hi + off) = hh;
      if (lo) *reinterpret_cast<uint32_t *>(lo + off) = ll;
    }
    if (write_scale && tig == 0 && r < S) o.sc[static_cast<size_t>(blk) * split_ld(o) + tr(r)] = static_cast<int8_t>(s);
  }
}
// The strip staged by strip_stage into columns col0 .. col0 + 31 of rows
// r0 .. r0 + 15 (those below S) of o.
__device__ __forceinline__ void stage_store(const uint16_t *hi, const uint16_t *lo, int r0, int S, AtomRows tr,
                                            int lane, const Split16View &o, int col0) {
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int c = 32 * it + lane, lr = c >> 2, ch = c & 3, r = r0 + lr;
    const int off = lr * 32 + ((ch ^ (lr & 3)) << 3);
    if (r < S) {
      const size_t go = static_cast<size_t>(tr(r)) * o.cols + col0 + 8 * ch;
      *reinterpret_cast<uint4 *>(o.hi + go) = *reinterpret_cast<const uint4 *>(hi + off);
      if (o.lo) *reinterpret_cast<uint4 *>(o.lo + go) = *reinterpret_cast<const uint4 *>(lo + off);
    }
  }
}

// ---- forward ---------------------------------------------------------------------
// Shared memory of the forward for atoms of at most MT tokens: Q, K, V in
// split form.  MT = 48 (3 warps, 23 KB) covers the usual neighbour counts
// with no idle warp and more CTAs per SM; MT = 64 (4 warps) the rest.
template <int MT>
struct SmemF {
  uint16_t mat[6][MT * kPitch];  // Q, K, V hi, then Q, K, V lo
  float mask[MT];
  int scale[3];
  int rmax[MT];                  // row maxima of the output (bits of non-negative floats)
};

template <bool kSplit, int MT>
__global__ void __launch_bounds__(2 * MT) k_attn_fwd_mma(AttnArgs a) {
  constexpr int kW = MT / 16, kNT = MT / 8, kTh = 32 * kW;  // warps (row strips), 8-key tiles, threads
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SmemF<MT> &sm = *reinterpret_cast<SmemF<MT> *>(smem_raw);
  const int atom = a.atoms ? a.atoms[blockIdx.x] : static_cast<int>(blockIdx.x), h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  const int e0 = a.offset[atom], S = a.offset[atom + 1] - e0 + 1;
  const AtomRows tr = atom_rows(atom, e0, a.edge_base);
  const int NW = (S + 15) >> 4, NK8 = 2 * NW;  // row strips, 8-key tiles
  if (warp < 3) {  // warp w converts block w (Q, K, V; rows past S are zero) at one scale
    float v[MT / 8][8];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < MT / 8; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      if (r < S) {
        const float *src = a.qkv + static_cast<size_t>(tr(r)) * 3 * a.d + warp * a.d + h * kHd + c;
        const float4 x0 = *reinterpret_cast<const float4 *>(src), x1 = *reinterpret_cast<const float4 *>(src + 4);
        v[i][0] = x0.x; v[i][1] = x0.y; v[i][2] = x0.z; v[i][3] = x0.w;
        v[i][4] = x1.x; v[i][5] = x1.y; v[i][6] = x1.z; v[i][7] = x1.w;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) mx = fmaxf(mx, fabsf(v[i][k]));
    }
    const int sc = split_scale_exponent(warp_absmax(mx));
    const float f = pow2f(sc);
    if (lane == 0) sm.scale[warp] = sc;
#pragma unroll
    for (int i = 0; i < MT / 8; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      uint32_t hh[4], ll[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) split2(v[i][2 * k], v[i][2 * k + 1], f, hh[k], ll[k]);
      *reinterpret_cast<uint4 *>(&sm.mat[warp][r * kPitch + c]) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
      *reinterpret_cast<uint4 *>(&sm.mat[3 + warp][r * kPitch + c]) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
    }
  }
  for (int k = threadIdx.x; k < MT; k += kTh) {
    sm.mask[k] = k < S ? (k == 0 ? 0.f : a.key_mask[e0 + k - 1]) : 0.f;
    if (kSplit) sm.rmax[k] = 0;
  }
  __syncthreads();
  if (kSplit) cluster_arrive();
  const uint32_t Qh = smem_addr(sm.mat[0]), Ql = smem_addr(sm.mat[3]), Kh = smem_addr(sm.mat[1]),
                 Kl = smem_addr(sm.mat[4]), Vh = smem_addr(sm.mat[2]), Vl = smem_addr(sm.mat[5]);
  float o[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  const int q0 = 16 * warp;
  const bool act = warp < NW;
  if (act) {
    float s[kNT][4];
#pragma unroll
    for (int n = 0; n < kNT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t ah[4], al[4];
      ldsm4(ah, a_addr(Qh, q0, 16 * ks, lane));
      ldsm4(al, a_addr(Ql, q0, 16 * ks, lane));
#pragma unroll
      for (int p = 0; p < kW; ++p) {
        if (2 * p < NK8) {
          uint32_t bh[4], bl[4];
          ldsm4(bh, bn_addr(Kh, 16 * p, 16 * ks, lane));
          ldsm4(bl, bn_addr(Kl, 16 * p, 16 * ks, lane));
          mma3(s[2 * p], ah, al, bh[0], bh[1], bl[0], bl[1]);
          mma3(s[2 * p + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
        }
      }
    }
    // softmax along each row (rows g and g + 8 of the strip)
    const float fs = pow2f(-(sm.scale[0] + sm.scale[1])) * (1.0f / sqrtf(static_cast<float>(kHd)));
    float m[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
    for (int n = 0; n < kNT; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = q0 + g + 8 * (e >> 1), c = 8 * n + 2 * tig + (e & 1);
        s[n][e] = (n < NK8 && r < S && c < S) ? fmaf(s[n][e], fs, sm.mask[c]) : -FLT_MAX;
        m[e >> 1] = fmaxf(m[e >> 1], s[n][e]);
      }
    }
    m[0] = quad_max(m[0]);
    m[1] = quad_max(m[1]);
    float l[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < kNT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[n][e] = s[n][e] == -FLT_MAX ? 0.f : __expf(s[n][e] - m[e >> 1]);
        l[e >> 1] += s[n][e];
      }
    l[0] = quad_sum(l[0]);
    l[1] = quad_sum(l[1]);
    if (tig == 0) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = q0 + g + 8 * half;
        if (r < S) a.lse[static_cast<size_t>(tr(r)) * a.heads + h] = m[half] + logf(l[half]);
      }
    }
    const float inv[2] = {l[0] > 0.f ? 1.0f / l[0] : 0.f, l[1] > 0.f ? 1.0f / l[1] : 0.f};
#pragma unroll
    for (int n = 0; n < kNT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] *= inv[e >> 1];
    // O = P V, P at the fixed scale 2^14
#pragma unroll
    for (int ks = 0; ks < kW; ++ks) {
      if (ks < NW) {
        uint32_t ah[4], al[4];
        c_to_a(s[2 * ks], s[2 * ks + 1], 16384.f, ah, al);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          uint32_t bh[4], bl[4];
          ldsm4t(bh, bk_addr(Vh, 16 * ks, 16 * p, lane));
          ldsm4t(bl, bk_addr(Vl, 16 * ks, 16 * p, lane));
          mma3(o[2 * p], ah, al, bh[0], bh[1], bl[0], bl[1]);
          mma3(o[2 * p + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
        }
      }
    }
    const float fo = pow2f(-(14 + sm.scale[2]));
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[n][e] *= fo;
    if (a.out) strip_store(o, q0, S, tr, lane, a.out, a.d, h * kHd, nullptr, nullptr, 0, false);
  }
  if (kSplit) {
    cluster_wait();
    if (act) strip_rowmax(sm.rmax, o, q0, S, lane);
    cluster_barrier();  // every CTA's maxima have reached every CTA
    if (act)
      strip_store(o, q0, S, tr, lane, nullptr, 0, h * kHd, &a.out_split, sm.rmax, (h * kHd) / 128,
                  cta_rank_in_cluster() == 0);
  }
}

// ---- forward with split output, one CTA per 128-column block ---------------------
// For atoms of at most 48 tokens: the 128 / 32 = 4 heads of one 128-column
// block of the output share a CTA of 12 warps (head = warp / 3, row strip or
// converted block = warp % 3), so the row maxima that fix the block's split
// scale meet in shared memory instead of crossing a thread-block cluster.
constexpr int kBlkHeads = 128 / kHd;
struct SmemFB {
  uint16_t mat[kBlkHeads][6][48 * kPitch];  // per head: Q, K, V hi, then Q, K, V lo
  float mask[48];
  int scale[kBlkHeads][3];
  int rmax[48];  // row maxima of the block's output (bits of non-negative floats)
};
static_assert(3 * kBlkHeads * 1024 <= kBlkHeads * 6 * 48 * kPitch, "output staging fits in the Q / K / V blocks");

__global__ void __launch_bounds__(32 * 3 * kBlkHeads) k_attn_fwd_mma_blk(AttnArgs a) {
  constexpr int MT = 48, kNT = MT / 8;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SmemFB &sm = *reinterpret_cast<SmemFB *>(smem_raw);
  const int atom = a.atoms ? a.atoms[blockIdx.x] : static_cast<int>(blockIdx.x), blk = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  const int hl = warp / 3, sw = warp % 3, h = blk * kBlkHeads + hl;
  const int e0 = a.offset[atom], S = a.offset[atom + 1] - e0 + 1;
  const AtomRows tr = atom_rows(atom, e0, a.edge_base);
  const int NW = (S + 15) >> 4, NK8 = 2 * NW;
  uint16_t(*mat)[48 * kPitch] = sm.mat[hl];
  {  // warp (hl, sw): block sw (Q, K or V) of head hl, rows past S zero, one scale
    float v[MT / 8][8];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < MT / 8; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      if (r < S) {
        const float *src = a.qkv + static_cast<size_t>(tr(r)) * 3 * a.d + sw * a.d + h * kHd + c;
        const float4 x0 = *reinterpret_cast<const float4 *>(src), x1 = *reinterpret_cast<const float4 *>(src + 4);
        v[i][0] = x0.x; v[i][1] = x0.y; v[i][2] = x0.z; v[i][3] = x0.w;
        v[i][4] = x1.x; v[i][5] = x1.y; v[i][6] = x1.z; v[i][7] = x1.w;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) mx = fmaxf(mx, fabsf(v[i][k]));
    }
    const int sc = split_scale_exponent(warp_absmax(mx));
    const float f = pow2f(sc);
    if (lane == 0) sm.scale[hl][sw] = sc;
#pragma unroll
    for (int i = 0; i < MT / 8; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      uint32_t hh[4], ll[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) split2(v[i][2 * k], v[i][2 * k + 1], f, hh[k], ll[k]);
      *reinterpret_cast<uint4 *>(&mat[sw][r * kPitch + c]) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
      *reinterpret_cast<uint4 *>(&mat[3 + sw][r * kPitch + c]) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
    }
  }
  for (int k = threadIdx.x; k < MT; k += blockDim.x) {
    sm.mask[k] = k < S ? (k == 0 ? 0.f : a.key_mask[e0 + k - 1]) : 0.f;
    sm.rmax[k] = 0;
  }
  __syncthreads();
  const uint32_t Qh = smem_addr(mat[0]), Ql = smem_addr(mat[3]), Kh = smem_addr(mat[1]), Kl = smem_addr(mat[4]),
                 Vh = smem_addr(mat[2]), Vl = smem_addr(mat[5]);
  float o[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  const int q0 = 16 * sw;
  const bool act = sw < NW;
  if (act) {
    float s[kNT][4];
#pragma unroll
    for (int n = 0; n < kNT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t ah[4], al[4];
      ldsm4(ah, a_addr(Qh, q0, 16 * ks, lane));
      ldsm4(al, a_addr(Ql, q0, 16 * ks, lane));
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        if (2 * p < NK8) {
          uint32_t bh[4], bl[4];
          ldsm4(bh, bn_addr(Kh, 16 * p, 16 * ks, lane));
          ldsm4(bl, bn_addr(Kl, 16 * p, 16 * ks, lane));
          mma3(s[2 * p], ah, al, bh[0], bh[1], bl[0], bl[1]);
          mma3(s[2 * p + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
        }
      }
    }
    const float fs = pow2f(-(sm.scale[hl][0] + sm.scale[hl][1])) * (1.0f / sqrtf(static_cast<float>(kHd)));
    float m[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
    for (int n = 0; n < kNT; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = q0 + g + 8 * (e >> 1), c = 8 * n + 2 * tig + (e & 1);
        s[n][e] = (n < NK8 && r < S && c < S) ? fmaf(s[n][e], fs, sm.mask[c]) : -FLT_MAX;
        m[e >> 1] = fmaxf(m[e >> 1], s[n][e]);
      }
    }
    m[0] = quad_max(m[0]);
    m[1] = quad_max(m[1]);
    float l[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < kNT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[n][e] = s[n][e] == -FLT_MAX ? 0.f : __expf(s[n][e] - m[e >> 1]);
        l[e >> 1] += s[n][e];
      }
    l[0] = quad_sum(l[0]);
    l[1] = quad_sum(l[1]);
    if (tig == 0) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = q0 + g + 8 * half;
        if (r < S) a.lse[static_cast<size_t>(tr(r)) * a.heads + h] = m[half] + logf(l[half]);
      }
    }
    const float inv[2] = {l[0] > 0.f ? 1.0f / l[0] : 0.f, l[1] > 0.f ? 1.0f / l[1] : 0.f};
#pragma unroll
    for (int n = 0; n < kNT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] *= inv[e >> 1];
#pragma unroll
    for (int ks = 0; ks < 3; ++ks) {
      if (ks < NW) {
        uint32_t ah[4], al[4];
        c_to_a(s[2 * ks], s[2 * ks + 1], 16384.f, ah, al);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          uint32_t bh[4], bl[4];
          ldsm4t(bh, bk_addr(Vh, 16 * ks, 16 * p, lane));
          ldsm4t(bl, bk_addr(Vl, 16 * ks, 16 * p, lane));
          mma3(o[2 * p], ah, al, bh[0], bh[1], bl[0], bl[1]);
          mma3(o[2 * p + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
        }
      }
    }
    const float fo = pow2f(-(14 + sm.scale[hl][2]));
    float m0 = 0.f, m1 = 0.f;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) o[n][e] *= fo;
      m0 = fmaxf(m0, fmaxf(fabsf(o[n][0]), fabsf(o[n][1])));
      m1 = fmaxf(m1, fmaxf(fabsf(o[n][2]), fabsf(o[n][3])));
    }
    // this head's row maxima into the block's (quad-reduced, one atomic per row)
    m0 = quad_max(m0);
    m1 = quad_max(m1);
    if (tig == 0) {
      if (q0 + g < S) atomicMax(&sm.rmax[q0 + g], __float_as_int(m0));
      if (q0 + g + 8 < S) atomicMax(&sm.rmax[q0 + g + 8], __float_as_int(m1));
    }
  }
  __syncthreads();  // the block's row maxima; every warp is past its products
  if (act) {
    // staging: 2 KB per warp in the Q / K / V blocks, dead after the barrier
    uint16_t *st = reinterpret_cast<uint16_t *>(smem_raw) + (threadIdx.x >> 5) * 1024;
    strip_stage(o, q0, S, tr, lane, st, a.out_split.lo ? st + 512 : nullptr, sm.rmax, a.out_split, blk, hl == 0);
    __syncwarp();
    stage_store(st, st + 512, q0, S, tr, lane, a.out_split, h * kHd);
  }
}

// ---- backward --------------------------------------------------------------------
// Scores and dP of a 16-row strip r0.. against all rows of the other block:
// s = A1 B1^T, dp = A2 B2^T (A from [rows][32] blocks, B likewise).
template <int NT>
__device__ __forceinline__ void strip_scores(float (&s)[NT][4], float (&dp)[NT][4], uint32_t a1h, uint32_t a1l,
                                             uint32_t b1h, uint32_t b1l, uint32_t a2h, uint32_t a2l, uint32_t b2h,
                                             uint32_t b2l, int r0, int NK8, int lane) {
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    uint32_t ah[4], al[4], ch[4], cl[4];
    ldsm4(ah, a_addr(a1h, r0, 16 * ks, lane));
    ldsm4(al, a_addr(a1l, r0, 16 * ks, lane));
    ldsm4(ch, a_addr(a2h, r0, 16 * ks, lane));
    ldsm4(cl, a_addr(a2l, r0, 16 * ks, lane));
#pragma unroll
    for (int p = 0; p < NT / 2; ++p) {
      if (2 * p < NK8) {
        uint32_t bh[4], bl[4];
        ldsm4(bh, bn_addr(b1h, 16 * p, 16 * ks, lane));
        ldsm4(bl, bn_addr(b1l, 16 * p, 16 * ks, lane));
        mma3(s[2 * p], ah, al, bh[0], bh[1], bl[0], bl[1]);
        mma3(s[2 * p + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
        ldsm4(bh, bn_addr(b2h, 16 * p, 16 * ks, lane));
        ldsm4(bl, bn_addr(b2l, 16 * p, 16 * ks, lane));
        mma3(dp[2 * p], ch, cl, bh[0], bh[1], bl[0], bl[1]);
        mma3(dp[2 * p + 1], ch, cl, bh[2], bh[3], bl[2], bl[3]);
      }
    }
  }
}

// acc (16 x 32) += A (16 x SP, the c-layout tiles x, scale f) times the
// [SP][32] block B (via ldmatrix.trans).
template <int NT>
__device__ __forceinline__ void strip_times_block(float (&acc)[4][4], const float (&x)[NT][4], float f, uint32_t bh_,
                                                  uint32_t bl_, int NW, int lane) {
#pragma unroll
  for (int ks = 0; ks < NT / 2; ++ks) {
    if (ks < NW) {
      uint32_t ah[4], al[4];
      c_to_a(x[2 * ks], x[2 * ks + 1], f, ah, al);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        uint32_t bh[4], bl[4];
        ldsm4t(bh, bk_addr(bh_, 16 * ks, 16 * p, lane));
        ldsm4t(bl, bk_addr(bl_, 16 * ks, 16 * p, lane));
        mma3(acc[2 * p], ah, al, bh[0], bh[1], bl[0], bl[1]);
        mma3(acc[2 * p + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
      }
    }
  }
}

template <bool kSplit>
__global__ void __launch_bounds__(kThreads) k_attn_bwd_mma(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  const int atom = a.atoms ? a.atoms[blockIdx.x] : static_cast<int>(blockIdx.x), h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  const int e0 = a.offset[atom], S = a.offset[atom + 1] - e0 + 1;
  const AtomRows tr = atom_rows(atom, e0, a.edge_base);
  const int NW = (S + 15) >> 4, NK8 = 2 * NW;
  const int d = a.d;
  load_blocks(sm, a, tr, S, h, true);
  for (int k = threadIdx.x; k < kMaxTok; k += kThreads) {
    sm.mask[k] = k < S ? (k == 0 ? 0.f : a.key_mask[e0 + k - 1]) : 0.f;
    sm.lse[k] = k < S ? a.lse[static_cast<size_t>(tr(k)) * a.heads + h] : 0.f;
    if (kSplit) sm.rmax[0][k] = sm.rmax[1][k] = sm.rmax[2][k] = 0;
  }
  __syncthreads();
  if (kSplit) cluster_arrive();
  const uint32_t Qh = smem_addr(sm.mat[0]), Ql = smem_addr(sm.mat[4]), Kh = smem_addr(sm.mat[1]),
                 Kl = smem_addr(sm.mat[5]), Vh = smem_addr(sm.mat[2]), Vl = smem_addr(sm.mat[6]),
                 Gh = smem_addr(sm.mat[3]), Gl = smem_addr(sm.mat[7]);
  const float rs = 1.0f / sqrtf(static_cast<float>(kHd));
  const float fs = pow2f(-(sm.scale[0] + sm.scale[1])) * rs;
  const float fdp = pow2f(-(sm.scale[3] + sm.scale[2]));
  const bool act = warp < NW;
  const int r0 = 16 * warp;
  float dq[4][4], dk[4][4], dv[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dq[n][e] = dk[n][e] = dv[n][e] = 0.f;

  // ---- pass 1: warp = query rows r0..r0+15 ----
  if (act) {
    float s[8][4], dp[8][4];
    strip_scores(s, dp, Qh, Ql, Kh, Kl, Gh, Gl, Vh, Vl, r0, NK8, lane);
    float Dp[2] = {0.f, 0.f};
    const float lq[2] = {sm.lse[r0 + g], sm.lse[r0 + g + 8]};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = r0 + g + 8 * (e >> 1), c = 8 * n + 2 * tig + (e & 1);
        const bool v = n < NK8 && r < S && c < S;
        s[n][e] = v ? __expf(fmaf(s[n][e], fs, sm.mask[c]) - lq[e >> 1]) : 0.f;
        dp[n][e] = v ? dp[n][e] * fdp : 0.f;
        Dp[e >> 1] = fmaf(s[n][e], dp[n][e], Dp[e >> 1]);
      }
    Dp[0] = quad_sum(Dp[0]);
    Dp[1] = quad_sum(Dp[1]);
    if (tig == 0) {
      sm.D[r0 + g] = Dp[0];
      sm.D[r0 + g + 8] = Dp[1];
    }
    float mx = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dp[n][e] = s[n][e] * (dp[n][e] - Dp[e >> 1]);  // dS
        mx = fmaxf(mx, fabsf(dp[n][e]));
      }
    const int sd = split_scale_exponent(warp_absmax(mx));
    strip_times_block(dq, dp, pow2f(sd), Kh, Kl, NW, lane);
    const float fq = pow2f(-(sd + sm.scale[1])) * rs;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) dq[n][e] *= fq;
  }
  __syncthreads();  // D of every query row

  // ---- pass 2: warp = key rows r0..r0+15 (transposed) ----
  if (act) {
    float st[8][4], dpt[8][4];
    strip_scores(st, dpt, Kh, Kl, Qh, Ql, Vh, Vl, Gh, Gl, r0, NK8, lane);
    const float mk[2] = {sm.mask[r0 + g], sm.mask[r0 + g + 8]};
    float mx = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = r0 + g + 8 * (e >> 1), c = 8 * n + 2 * tig + (e & 1);  // key r, query c
        const bool v = n < NK8 && r < S && c < S;
        const float p = v ? __expf(fmaf(st[n][e], fs, mk[e >> 1]) - sm.lse[c]) : 0.f;
        dpt[n][e] = v ? p * (dpt[n][e] * fdp - sm.D[c]) : 0.f;  // dS^T
        st[n][e] = p;                                           // P^T
        mx = fmaxf(mx, fabsf(dpt[n][e]));
      }
    strip_times_block(dv, st, 16384.f, Gh, Gl, NW, lane);
    const int sd = split_scale_exponent(warp_absmax(mx));
    strip_times_block(dk, dpt, pow2f(sd), Qh, Ql, NW, lane);
    const float fv = pow2f(-(14 + sm.scale[3])), fk = pow2f(-(sd + sm.scale[0])) * rs;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dv[n][e] *= fv;
        dk[n][e] *= fk;
      }
  }

  const size_t ld = 3 * static_cast<size_t>(d);
  if (act && a.d_qkv) {
    strip_store(dq, r0, S, tr, lane, a.d_qkv, ld, h * kHd, nullptr, nullptr, 0, false);
    strip_store(dk, r0, S, tr, lane, a.d_qkv, ld, d + h * kHd, nullptr, nullptr, 0, false);
    strip_store(dv, r0, S, tr, lane, a.d_qkv, ld, 2 * d + h * kHd, nullptr, nullptr, 0, false);
  }
  if (kSplit) {
    cluster_wait();
    if (act) {
      strip_rowmax(sm.rmax[0], dq, r0, S, lane);
      strip_rowmax(sm.rmax[1], dk, r0, S, lane);
      strip_rowmax(sm.rmax[2], dv, r0, S, lane);
    }
    cluster_barrier();  // every CTA's maxima have reached every CTA
    if (act) {
      const int nb = d / 128, blk = (h * kHd) / 128;
      const bool first = cta_rank_in_cluster() == 0;
      strip_store(dq, r0, S, tr, lane, nullptr, 0, h * kHd, &a.dqkv_split, sm.rmax[0], blk, first);
      strip_store(dk, r0, S, tr, lane, nullptr, 0, d + h * kHd, &a.dqkv_split, sm.rmax[1], nb + blk, first);
      strip_store(dv, r0, S, tr, lane, nullptr, 0, 2 * d + h * kHd, &a.dqkv_split, sm.rmax[2], 2 * nb + blk, first);
    }
  }
}

// ---- backward for atoms of at most 48 tokens ---------------------------------------
// Three warps, one per 16-row strip.  Pass 1 (warp = query rows) computes
// S, P, dP, D and dS in registers and dQ = dS K; pass 2 (warp = key rows)
// reads P and then dS back transposed with ldmatrix.trans as the A operands
// of dV = P^T dO and dK = dS^T Q instead of recomputing the scores.  P and
// dS (split form, P at 2^14, dS at one scale for the whole item from a
// block-wide maximum) take turns in the region that held K and V, which are
// dead once dQ is done, so a CTA needs 32 KB and six fit on an SM.
constexpr int kMT = 48;
constexpr int kW48 = kMT / 16;       // warps
constexpr int kTh48 = 32 * kW48;     // threads
constexpr int kPitchP = 56;          // halves per P / dS row (112 bytes: conflict-free ldmatrix)
constexpr int kMatP = kMT * kPitchP;
constexpr int kMat48 = kMT * kPitch;

struct Smem48 {
  uint16_t qg[4][kMat48];         // Q hi, dO hi, Q lo, dO lo
  uint16_t kv[4 * kMat48];        // K hi, V hi, K lo, V lo; later P or dS: hi [kMatP], lo [kMatP]
  float lse[kMT], mask[kMT];
  int scale[4];                   // block scale exponents of Q, K, V, dO
  int gmax;                       // bits of max |dO|
  int dsmax;                      // bits of the item's max |dS|
  int rmax[3][kMT];
};
static_assert(4 * kMat48 >= 2 * kMatP, "P / dS fit in the K / V region");
static_assert(kW48 * 3072 * 2 <= 8 * kMat48 * 2, "split-output staging fits in the Q / dO / K / V blocks");

// A operand (16 keys x 16 queries) of a transposed product from a stored
// [query][key] block: matrices (q0, k0), (q0, k0 + 8), (q0 + 8, k0),
// (q0 + 8, k0 + 8) loaded with .trans -> a0..a3.
__device__ __forceinline__ uint32_t at_addr(uint32_t base, int k0, int q0, int lane) {
  const int j = lane >> 3;
  return base + 2u * static_cast<uint32_t>((q0 + (lane & 7) + 8 * (j >> 1)) * kPitchP + k0 + 8 * (j & 1));
}

// acc (16 x 32) += A^T (stored [query][key] blocks, rows k0.. as A rows)
// times the [query][32] block B, over NW 16-query steps.
__device__ __forceinline__ void stored_t_times_block(float (&acc)[4][4], uint32_t ah_, uint32_t al_, int k0,
                                                     uint32_t bh_, uint32_t bl_, int NW, int lane) {
#pragma unroll
  for (int ks = 0; ks < 3; ++ks) {
    if (ks < NW) {
      uint32_t ah[4], al[4];
      ldsm4t(ah, at_addr(ah_, k0, 16 * ks, lane));
      ldsm4t(al, at_addr(al_, k0, 16 * ks, lane));
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        uint32_t bh[4], bl[4];
        ldsm4t(bh, bk_addr(bh_, 16 * ks, 16 * p, lane));
        ldsm4t(bl, bk_addr(bl_, 16 * ks, 16 * p, lane));
        mma3(acc[2 * p], ah, al, bh[0], bh[1], bl[0], bl[1]);
        mma3(acc[2 * p + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
      }
    }
  }
}

// c-layout tiles of a 16-row strip into a stored [row][col] split block
__device__ __forceinline__ void strip_to_smem(uint16_t *hi, uint16_t *lo, const float (&x)[6][4], int NK8, int r0,
                                              float f, int lane) {
  const int g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int n = 0; n < 6; ++n) {
    if (n < NK8) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t hh, ll;
        split2(x[n][2 * half], x[n][2 * half + 1], f, hh, ll);
        const int off = (r0 + g + 8 * half) * kPitchP + 8 * n + 2 * tig;
        *reinterpret_cast<uint32_t *>(hi + off) = hh;
        *reinterpret_cast<uint32_t *>(lo + off) = ll;
      }
    }
  }
}

template <bool kSplit>
__global__ void __launch_bounds__(kTh48, 6) k_attn_bwd_mma48(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem48 &sm = *reinterpret_cast<Smem48 *>(smem_raw);
  const int atom = a.atoms ? a.atoms[blockIdx.x] : static_cast<int>(blockIdx.x), h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  const int e0 = a.offset[atom], S = a.offset[atom + 1] - e0 + 1;
  const AtomRows tr = atom_rows(atom, e0, a.edge_base);
  const int NW = (S + 15) >> 4, NK8 = 2 * NW;
  const int d = a.d;
  // this warp's block (Q, K or V) in split form
  uint16_t *const whi = warp == 0 ? sm.qg[0] : sm.kv + (warp - 1) * kMat48;
  uint16_t *const wlo = warp == 0 ? sm.qg[2] : sm.kv + (warp + 1) * kMat48;
  float gv[2][8];
  {  // warp w: block w of Q, K, V (6 row-chunks per lane); all threads: 2 chunks of dO
    float v[6][8];
    float mx = 0.f, gm = 0.f;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      if (r < S) {
        const float *src = a.qkv + static_cast<size_t>(tr(r)) * 3 * d + warp * d + h * kHd + c;
        const float4 x0 = *reinterpret_cast<const float4 *>(src), x1 = *reinterpret_cast<const float4 *>(src + 4);
        v[i][0] = x0.x; v[i][1] = x0.y; v[i][2] = x0.z; v[i][3] = x0.w;
        v[i][4] = x1.x; v[i][5] = x1.y; v[i][6] = x1.z; v[i][7] = x1.w;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) mx = fmaxf(mx, fabsf(v[i][k]));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int task = threadIdx.x + kTh48 * i, r = task >> 2, c = (task & 3) * 8;
      if (r < S) {
        const float *src = a.d_out + static_cast<size_t>(tr(r)) * d + h * kHd + c;
        const float4 x0 = *reinterpret_cast<const float4 *>(src), x1 = *reinterpret_cast<const float4 *>(src + 4);
        gv[i][0] = x0.x; gv[i][1] = x0.y; gv[i][2] = x0.z; gv[i][3] = x0.w;
        gv[i][4] = x1.x; gv[i][5] = x1.y; gv[i][6] = x1.z; gv[i][7] = x1.w;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) gv[i][k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) gm = fmaxf(gm, fabsf(gv[i][k]));
    }
    if (threadIdx.x == 0) {
      sm.gmax = 0;
      sm.dsmax = 0;
    }
    const int sc = split_scale_exponent(warp_absmax(mx));
    const float f = pow2f(sc);
    if (lane == 0) sm.scale[warp] = sc;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const int task = lane + 32 * i, r = task >> 2, c = (task & 3) * 8;
      uint32_t hh[4], ll[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) split2(v[i][2 * k], v[i][2 * k + 1], f, hh[k], ll[k]);
      *reinterpret_cast<uint4 *>(&whi[r * kPitch + c]) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
      *reinterpret_cast<uint4 *>(&wlo[r * kPitch + c]) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
    }
    for (int k = threadIdx.x; k < kMT; k += kTh48) {
      sm.mask[k] = k < S ? (k == 0 ? 0.f : a.key_mask[e0 + k - 1]) : 0.f;
      sm.lse[k] = k < S ? a.lse[static_cast<size_t>(tr(k)) * a.heads + h] : 0.f;
      if (kSplit) sm.rmax[0][k] = sm.rmax[1][k] = sm.rmax[2][k] = 0;
    }
    gm = warp_absmax(gm);
    __syncthreads();  // gmax and dsmax cleared
    if (lane == 0) atomicMax(&sm.gmax, __float_as_int(gm));
    __syncthreads();  // max |dO|
    const int sg = split_scale_exponent(__int_as_float(sm.gmax));
    const float fg = pow2f(sg);
    if (threadIdx.x == 0) sm.scale[3] = sg;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int task = threadIdx.x + kTh48 * i, r = task >> 2, c = (task & 3) * 8;
      uint32_t hh[4], ll[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) split2(gv[i][2 * k], gv[i][2 * k + 1], fg, hh[k], ll[k]);
      *reinterpret_cast<uint4 *>(&sm.qg[1][r * kPitch + c]) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
      *reinterpret_cast<uint4 *>(&sm.qg[3][r * kPitch + c]) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
    }
  }
  __syncthreads();  // every block and scale
  if (kSplit) cluster_arrive();
  const uint32_t Qh = smem_addr(sm.qg[0]), Ql = smem_addr(sm.qg[2]), Gh = smem_addr(sm.qg[1]),
                 Gl = smem_addr(sm.qg[3]), Kh = smem_addr(sm.kv), Vh = smem_addr(sm.kv + kMat48),
                 Kl = smem_addr(sm.kv + 2 * kMat48), Vl = smem_addr(sm.kv + 3 * kMat48);
  const uint32_t Xh = smem_addr(sm.kv), Xl = smem_addr(sm.kv + kMatP);  // P or dS, after K and V
  const float rs = 1.0f / sqrtf(static_cast<float>(kHd));
  const float fs = pow2f(-(sm.scale[0] + sm.scale[1])) * rs;
  const float fdp = pow2f(-(sm.scale[3] + sm.scale[2]));
  const bool act = warp < NW;
  const int r0 = 16 * warp;
  float dq[4][4], dk[4][4], dv[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dq[n][e] = dk[n][e] = dv[n][e] = 0.f;

  // ---- pass 1: warp = query rows: P, dS and dQ in registers ----
  float s[6][4], dp[6][4];
  if (act) {
    strip_scores(s, dp, Qh, Ql, Kh, Kl, Gh, Gl, Vh, Vl, r0, NK8, lane);
    float Dp[2] = {0.f, 0.f};
    const float lq[2] = {sm.lse[r0 + g], sm.lse[r0 + g + 8]};
#pragma unroll
    for (int n = 0; n < 6; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = r0 + g + 8 * (e >> 1), c = 8 * n + 2 * tig + (e & 1);
        const bool v = n < NK8 && r < S && c < S;
        s[n][e] = v ? __expf(fmaf(s[n][e], fs, sm.mask[c]) - lq[e >> 1]) : 0.f;
        dp[n][e] = v ? dp[n][e] * fdp : 0.f;
        Dp[e >> 1] = fmaf(s[n][e], dp[n][e], Dp[e >> 1]);
      }
    Dp[0] = quad_sum(Dp[0]);
    Dp[1] = quad_sum(Dp[1]);
    float mx = 0.f;
#pragma unroll
    for (int n = 0; n < 6; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dp[n][e] = s[n][e] * (dp[n][e] - Dp[e >> 1]);  // dS
        mx = fmaxf(mx, fabsf(dp[n][e]));
      }
    mx = warp_absmax(mx);
    if (lane == 0) atomicMax(&sm.dsmax, __float_as_int(mx));
  }
  __syncthreads();  // the item's max |dS|
  const int sd = split_scale_exponent(__int_as_float(sm.dsmax));
  if (act) {
    strip_times_block(dq, dp, pow2f(sd), Kh, Kl, NW, lane);
    const float fq = pow2f(-(sd + sm.scale[1])) * rs;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) dq[n][e] *= fq;
  }
  __syncthreads();  // K and V are no longer read
  if (act) strip_to_smem(sm.kv, sm.kv + kMatP, s, NK8, r0, 16384.f, lane);
  __syncthreads();  // P of every query row

  // ---- pass 2: warp = key rows r0..r0+15: dV = P^T dO, then dK = dS^T Q ----
  if (act) stored_t_times_block(dv, Xh, Xl, r0, Gh, Gl, NW, lane);
  __syncthreads();  // P is no longer read
  if (act) strip_to_smem(sm.kv, sm.kv + kMatP, dp, NK8, r0, pow2f(sd), lane);
  __syncthreads();  // dS of every query row
  if (act) {
    stored_t_times_block(dk, Xh, Xl, r0, Qh, Ql, NW, lane);
    const float fv = pow2f(-(14 + sm.scale[3])), fk = pow2f(-(sd + sm.scale[0])) * rs;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dv[n][e] *= fv;
        dk[n][e] *= fk;
      }
  }

  const size_t ld = 3 * static_cast<size_t>(d);
  if (act && a.d_qkv) {
    strip_store(dq, r0, S, tr, lane, a.d_qkv, ld, h * kHd, nullptr, nullptr, 0, false);
    strip_store(dk, r0, S, tr, lane, a.d_qkv, ld, d + h * kHd, nullptr, nullptr, 0, false);
    strip_store(dv, r0, S, tr, lane, a.d_qkv, ld, 2 * d + h * kHd, nullptr, nullptr, 0, false);
  }
  if (kSplit) {
    cluster_wait();
    if (act) {
      strip_rowmax(sm.rmax[0], dq, r0, S, lane);
      strip_rowmax(sm.rmax[1], dk, r0, S, lane);
      strip_rowmax(sm.rmax[2], dv, r0, S, lane);
    }
    cluster_barrier();  // every CTA's maxima have reached every CTA
    if (act) {
      const int nb = d / 128, blk = (h * kHd) / 128;
      const bool first = cta_rank_in_cluster() == 0;
      // staging: 6 KB per warp in the Q / dO / K / V blocks, dead once every
      // warp of the cluster has passed the barrier
      uint16_t *st = reinterpret_cast<uint16_t *>(smem_raw) + warp * 3072;
      const bool lo = a.dqkv_split.lo != nullptr;
      strip_stage(dq, r0, S, tr, lane, st, lo ? st + 512 : nullptr, sm.rmax[0], a.dqkv_split, blk, first);
      strip_stage(dk, r0, S, tr, lane, st + 1024, lo ? st + 1536 : nullptr, sm.rmax[1], a.dqkv_split, nb + blk, first);
      strip_stage(dv, r0, S, tr, lane, st + 2048, lo ? st + 2560 : nullptr, sm.rmax[2], a.dqkv_split, 2 * nb + blk,
                  first);
      __syncwarp();
      stage_store(st, st + 512, r0, S, tr, lane, a.dqkv_split, h * kHd);
      stage_store(st + 1024, st + 1536, r0, S, tr, lane, a.dqkv_split, d + h * kHd);
      stage_store(st + 2048, st + 2560, r0, S, tr, lane, a.dqkv_split, 2 * d + h * kHd);
    }
  }
}

// One class of atoms: n CTA rows (a.atoms maps them to atoms; null for
// atoms 0..n-1) on the kernels for short sequences (at most kMT tokens) or
// for any length up to kMaxTok.
template <bool kSplit>
void launch_class(const AttnArgs &a, bool bwd, bool small, int n, cudaStream_t s) {
  if (n <= 0) return;
  size_t smem;
  int threads = kThreads;
  void (*fn)(AttnArgs);
  if (bwd) {
    smem = small ? sizeof(Smem48) : sizeof(Smem);
    threads = small ? kTh48 : kThreads;
    fn = small ? k_attn_bwd_mma48<kSplit> : k_attn_bwd_mma<kSplit>;
  } else if (kSplit && small) {
    // one CTA per (atom, 128-column block): no cluster
    smem = sizeof(SmemFB);
    CUDA_CHECK(cudaFuncSetAttribute(k_attn_fwd_mma_blk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
    k_attn_fwd_mma_blk<<<dim3(n, a.heads / kBlkHeads), 32 * 3 * kBlkHeads, smem, s>>>(a);
    CUDA_LAUNCH_CHECK();
    return;
  } else {
    smem = small ? sizeof(SmemF<kMT>) : sizeof(SmemF<kMaxTok>);
    threads = small ? 2 * kMT : 2 * kMaxTok;
    fn = small ? k_attn_fwd_mma<kSplit, kMT> : k_attn_fwd_mma<kSplit, kMaxTok>;
  }
  CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n, a.heads);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (kSplit) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 128 / kHd;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  CUDA_CHECK(cudaLaunchKernelEx(&cfg, fn, a));
  CUDA_LAUNCH_CHECK();
}

// With atoms longer than kMT tokens and the class lists given, the short
// atoms keep the faster short-sequence kernels and only the long ones take
// the general kernels; otherwise one launch over atoms 0..n_atoms-1.
template <bool kSplit>
void launch_mma(const AttnArgs &a0, bool bwd, cudaStream_t s) {
  AttnArgs a = a0;
  a.atoms = nullptr;
  if (a0.max_tokens <= kMT || !a0.short_atoms || !a0.long_atoms) {
    launch_class<kSplit>(a, bwd, a0.max_tokens <= kMT, a0.n_atoms, s);
    return;
  }
  a.atoms = a0.short_atoms;
  a.max_tokens = kMT;
  launch_class<kSplit>(a, bwd, true, a0.n_short, s);
  a.atoms = a0.long_atoms;
  a.max_tokens = a0.max_tokens;
  launch_class<kSplit>(a, bwd, false, a0.n_long, s);
}

__global__ void k_attention_classes(const int *__restrict__ offset, int n, int short_tokens,
                                    int *__restrict__ short_atoms, int *__restrict__ long_atoms,
                                    int *__restrict__ counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x, lane = threadIdx.x & 31;
  const bool valid = i < n;
  const bool is_short = valid && offset[i + 1] - offset[i] + 1 <= short_tokens;
  const unsigned ms = __ballot_sync(0xffffffffu, is_short), ml = __ballot_sync(0xffffffffu, valid && !is_short);
  int bs = 0, bl = 0;
  if (lane == 0) {
    if (ms) bs = atomicAdd(&counts[0], __popc(ms));
    if (ml) bl = atomicAdd(&counts[1], __popc(ml));
  }
  bs = __shfl_sync(0xffffffffu, bs, 0);
  bl = __shfl_sync(0xffffffffu, bl, 0);
  const unsigned below = (1u << lane) - 1u;
  if (is_short) short_atoms[bs + __popc(ms & below)] = i;
  else if (valid) long_atoms[bl + __popc(ml & below)] = i;
}

}  // namespace

bool attention_mma_supported(const AttnArgs &a, bool bwd) {
  if (a.heads <= 0 || a.d != a.heads * kHd) return false;
  if (a.max_tokens < 1 || a.max_tokens > kMaxTok) return false;
  const bool split = bwd ? a.dqkv_split.hi != nullptr : a.out_split.hi != nullptr;
  if (split && (a.heads % (128 / kHd) || a.d % 128)) return false;
  return bwd ? (a.d_out && a.lse) : a.lse != nullptr;
}

int attention_short_tokens() { return kMT; }

void attention_classes(const int *offset, int n, int short_tokens, int *short_atoms, int *long_atoms, int *counts,
                       cudaStream_t s) {
  if (n <= 0) return;
  k_attention_classes<<<(n + 255) / 256, 256, 0, s>>>(offset, n, short_tokens, short_atoms, long_atoms, counts);
  CUDA_LAUNCH_CHECK();
}

void attention_mma(const AttnArgs &a, bool bwd, cudaStream_t s) {
  if (a.n_atoms <= 0) return;
  if (!attention_mma_supported(a, bwd)) throw Error(kErrInternal, "attention_mma: unsupported shape");
  const bool split = bwd ? a.dqkv_split.hi != nullptr : a.out_split.hi != nullptr;
  if (split) launch_mma<true>(a, bwd, s);
  else launch_mma<false>(a, bwd, s);
}

}  // namespace pet
