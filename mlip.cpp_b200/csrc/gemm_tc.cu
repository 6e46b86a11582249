// fp32-accurate GEMM on the 5th-generation tensor cores (tcgen05, sm_100a):
// "3xTF32" -- every fp32 operand x is split into x_hi = tf32(x) (low 13
// mantissa bits cleared) and x_lo = x - x_hi (exact in fp32), and
//   A B ~= A_hi B_hi + A_hi B_lo + A_lo B_hi
// accumulated in fp32 in tensor memory.  The dropped A_lo B_lo term and the
// truncation of x_lo are below 2^-21 relative, i.e. fp32-level accuracy.
//
// Tile: 128 (M) x 128 (N) x 32 (K, one 128-byte row of fp32 per operand
// row).  Operands live in shared memory in the K-major 128-byte
// swizzled layout UMMA reads (8-row x 128-byte atoms, 16-byte chunk index
// XOR row % 8, atoms 1024 bytes apart).
//  * A (activations, fp32, optionally row-gathered) is loaded by all 128
//    threads with 16-byte loads, split in registers and stored swizzled.
//  * B (weights) are pre-split on the host into hi/lo copies and streamed
//    with cp.async 16-byte copies into the swizzled layout.
//  * One thread issues 4 (k-steps of 8) x 3 tcgen05.mma per k-tile; a
//    tcgen05.commit to the stage's mbarrier frees the stage.
//  * Accumulators (128 lanes x 128 fp32 columns, double-buffered in TMEM)
//    are read back with tcgen05.ld (each warp its 32 lanes = rows) every
//    K-chunk and summed in registers; the epilogue is fused.
//
// "3xFP16" (k_gemm_3xf16) runs the same pipeline on kind::f16 MMAs, which
// have twice the tf32 rate and half its operand bytes per product: A row m
// is scaled by an exact power of two 2^s_m that maps its largest |element|
// into [2^14, 2^15) (a pre-pass computes s_m), B by one power of two per
// weight tensor, and each is split into fp16 hi = rn(x) and lo = rn(x - hi)
// (11 + 11 significant bits, the same as tf32 hi + lo).  The epilogue
// multiplies the fp32 result by 2^-(s_m + s_B), which is exact.  Elements
// below 2^-17 of their row's maximum keep an absolute error under 2^-40 of
// that maximum (fp16 subnormal lo parts).  Tile 128 x 128 x 64 fp16.
//
// Every mbarrier wait is bounded (~1 s of %globaltimer); on expiry the kernel
// records an error code, skips the rest of its work, frees its tensor memory
// and returns, so a fault cannot hang the GPU.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstdlib>
#include <atomic>
#include <cstring>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "split16.cuh"
#include "tc_common.cuh"

namespace pet {
namespace {
using namespace tc;

constexpr int BM = 128, BK = 32;

// Instruction descriptor: fp32 accumulate, tf32 A and B, both K-major,
// N >> 3 in [17,23), M >> 4 in [24,29).
template <int BN>
__device__ __forceinline__ uint32_t idesc_tf32() {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// fp32 accumulate, fp16 A and B, both K-major.
template <int BN>
__device__ __forceinline__ uint32_t idesc_f16() {
  return (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// Warp roles (288 threads, one CTA per SM, persistent over output tiles):
//   warps 0-3  producers: A (load, split, swizzled store) and B (cp.async)
//              into a kStages-deep ring of smem stages;
//   warp 4     MMA issuer (lane 0): for each K-chunk of kChunk k-tiles it
//              accumulates into one of two TMEM buffers, then commits;
//   warps 5-8  accumulators: drain each finished TMEM chunk into fp32
//              registers with round-to-nearest adds, then run the epilogue.
// The tensor core's own fp32 accumulation truncates; summing only kChunk *
// 4 * 3 products per TMEM pass and promoting chunks into registers keeps the
// result at fp32 accuracy for K up to thousands.
constexpr int BN = 128;
constexpr int kStages = 3;
#ifndef PET_GEMM_CHUNK
#define PET_GEMM_CHUNK 4
#endif
constexpr int kChunk = PET_GEMM_CHUNK;  // k-tiles (of 32) per TMEM accumulation pass
constexpr int kStageBytes = 4 * BM * 128;  // A hi, A lo, B hi, B lo
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
constexpr int kWsThreads = 288;

struct Bars {
  uint32_t full, empty, accf, acce, abort_addr;
};

// The two warps that share a TMEM lane quarter, each with 64 columns of a
// 128-column scale block, exchange their maxima through shared memory:
// slot [2 (tile parity)][2 (column half)][32 (lane)], one mbarrier of 64.
struct PairExchange {
  float *slot;
  uint32_t bar;
  int parity, half;
  volatile int *abort_flag;
};

// Epilogue of one thread's row segment [n0, n0 + NC): bias, activation,
// fp32 store (if p.C), and for the 3xFP16 kernel (kScaled) optionally the
// split-fp16 form of the result (p.c_split).  NC = 128: the segment is one
// scale block.  NC = 64: a block is shared with the partner warp (px).
template <int EPI, bool kScaled = false, int NC = BN>
__device__ __forceinline__ void epilogue_store(const GemmArgs &p, int row, int n0, float (&acc)[NC],
                                               float s_row = 1.f, float s_b = 1.f,
                                               const PairExchange *px = nullptr) {
  const bool split = kScaled && p.c_split.hi != nullptr;
  const bool valid = row < p.M;
  constexpr bool kShared = NC < 128;
  if (!valid && !(split && kShared)) return;  // the block exchange needs every thread
  const int rc = valid ? (p.c_rows ? p.c_rows[row] : row) : 0;
  float *crow = (p.C && valid) ? p.C + static_cast<size_t>(rc) * p.ldc : nullptr;
  // EPI_SILU with Z == null: no derivative kept (forward-only passes)
  const float *zrow = ((EPI == EPI_SILU || EPI == EPI_DSILU) && p.Z) ? p.Z + static_cast<size_t>(row) * p.ldz : nullptr;
  const float *rrow = EPI == EPI_RESID ? p.R + static_cast<size_t>(rc) * p.ldr : nullptr;
  // 32 columns at a time: all loads of a group (bias, Z or R, C for ACCUM)
  // are issued before its stores, so a thread waits on memory once per group
#pragma unroll
  for (int g = 0; g < NC; g += 32) {
    if (!valid) break;
    float4 x[8], ld[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = g + 4 * k;
      x[k] = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      if (kScaled) {  // two exact power-of-two multiplies
        x[k].x = (x[k].x * s_row) * s_b; x[k].y = (x[k].y * s_row) * s_b;
        x[k].z = (x[k].z * s_row) * s_b; x[k].w = (x[k].w * s_row) * s_b;
      }
    }
    if (p.bias) {
      float4 b[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) b[k] = __ldg(reinterpret_cast<const float4 *>(p.bias + n0 + g + 4 * k));
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        x[k].x += b[k].x; x[k].y += b[k].y; x[k].z += b[k].z; x[k].w += b[k].w;
      }
    }
    if (EPI == EPI_DSILU || EPI == EPI_RESID || EPI == EPI_ACCUM) {
      const float *src = EPI == EPI_DSILU ? zrow : EPI == EPI_RESID ? rrow : crow;
#pragma unroll
      for (int k = 0; k < 8; ++k) ld[k] = *reinterpret_cast<const float4 *>(src + n0 + g + 4 * k);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int n = n0 + g + 4 * k;
      float4 out;
      if (EPI == EPI_STORE) {
        out = x[k];
      } else if (EPI == EPI_SILU) {
        float4 dy;
        silu_pair(x[k].x, out.x, dy.x); silu_pair(x[k].y, out.y, dy.y);
        silu_pair(x[k].z, out.z, dy.z); silu_pair(x[k].w, out.w, dy.w);
        if (zrow) *reinterpret_cast<float4 *>(const_cast<float *>(zrow) + n) = dy;
      } else if (EPI == EPI_DSILU) {
        out = make_float4(x[k].x * ld[k].x, x[k].y * ld[k].y, x[k].z * ld[k].z, x[k].w * ld[k].w);
      } else {  // EPI_RESID, EPI_ACCUM: x + R or x + C
        out = make_float4(x[k].x + ld[k].x, x[k].y + ld[k].y, x[k].z + ld[k].z, x[k].w + ld[k].w);
      }
      if (crow) *reinterpret_cast<float4 *>(crow + n) = out;
      if (split) {
        const int j = g + 4 * k;
        acc[j] = out.x; acc[j + 1] = out.y; acc[j + 2] = out.z; acc[j + 3] = out.w;
      }
    }
  }
  if (split) {
    float mx = 0.f;
    if (valid) {
#pragma unroll
      for (int j = 0; j < NC; ++j) mx = fmaxf(mx, fabsf(acc[j]));
    }
    if (kShared) {
      const int lane = threadIdx.x & 31;
      float *slot = px->slot + px->parity * 64;
      slot[px->half * 32 + lane] = mx;
      mbar_arrive(px->bar);
      if (!wait_or_abort(px->bar, px->parity, px->abort_flag)) return;
      mx = fmaxf(mx, slot[(1 - px->half) * 32 + lane]);
      if (!valid) return;
    }
    const int s = split_scale_exponent(mx);
    thread_split_store<NC>(p.c_split, rc, n0, acc, s);
    if (!kShared || px->half == 0)
      p.c_split.sc[static_cast<size_t>(n0 / 128) * split_ld(p.c_split) + rc] = static_cast<int8_t>(s);
  }
}

template <int EPI>
__global__ void __launch_bounds__(kWsThreads, 1) k_gemm_3xtf32(GemmArgs p, TCWeights w, int *err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t bars = base + kStages * kStageBytes;
  // mbarriers: full[kStages], empty[kStages], accf[2], acce[2]
  const uint32_t full0 = bars, empty0 = bars + 8 * kStages, accf0 = bars + 16 * kStages,
                 acce0 = accf0 + 16;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kStages * kStageBytes + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + kStages * kStageBytes + 200);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = p.K / BK;
  const int tiles_n = p.N / BN;
  const int tiles = ((p.M + BM - 1) / BM) * tiles_n;

  if (warp == 4) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 128);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // ---------------- producers ----------------
    const int pr = tid >> 3, pc = tid & 7;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
      const float *arow[BM / 16];
#pragma unroll
      for (int i = 0; i < BM / 16; ++i) {
        const int m = m0 + pr + 16 * i;
        arow[i] = nullptr;
        if (m < p.M) arow[i] = p.A + static_cast<size_t>(p.a_rows ? p.a_rows[m] : m) * p.lda;
      }
      const float *bhi = w.hi + static_cast<size_t>(n0) * p.ldb;
      const float *blo = w.lo + static_cast<size_t>(n0) * p.ldb;
      for (int kt = 0; kt < nk; ++kt, ++it) {
        const int s = it % kStages;
        if (!wait_or_abort(empty0 + 8 * s, ((it / kStages) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t st = base + s * kStageBytes;
        const uint32_t sAhi = st, sAlo = st + BM * 128, sBhi = st + 2 * BM * 128, sBlo = st + 3 * BM * 128;
        const int k0 = kt * BK + pc * 4;
#pragma unroll 4
        for (int i = 0; i < BN / 16; ++i) {
          const int r = pr + 16 * i;
          const size_t off = static_cast<size_t>(r) * p.ldb + k0;
          cp_async16(sBhi + swz(r, pc), bhi + off);
          cp_async16(sBlo + swz(r, pc), blo + off);
        }
        float4 va[BM / 16];
#pragma unroll
        for (int i = 0; i < BM / 16; ++i)
          va[i] = arow[i] ? *reinterpret_cast<const float4 *>(arow[i] + k0) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < BM / 16; ++i) {
          const int r = pr + 16 * i;
          float4 h, l;
          h.x = tf32_hi(va[i].x); l.x = va[i].x - h.x;
          h.y = tf32_hi(va[i].y); l.y = va[i].y - h.y;
          h.z = tf32_hi(va[i].z); l.z = va[i].z - h.z;
          h.w = tf32_hi(va[i].w); l.w = va[i].w - h.w;
          *reinterpret_cast<float4 *>(gbase + (sAhi - base) + swz(r, pc)) = h;
          *reinterpret_cast<float4 *>(gbase + (sAlo - base) + swz(r, pc)) = l;
        }
        cp_async_wait_all();
        fence_proxy_async();
        mbar_arrive(full0 + 8 * s);
      }
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32<BN>();
      int it = 0, chunk = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        for (int kt0 = 0; kt0 < nk && ok; kt0 += kChunk, ++chunk) {
          const int b = chunk & 1;
          if (!wait_or_abort(acce0 + 8 * b, ((chunk >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dtm = tmem + static_cast<uint32_t>(b * BN);
          const int kend = kt0 + kChunk < nk ? kt0 + kChunk : nk;
          for (int kt = kt0; kt < kend; ++kt, ++it) {
            const int s = it % kStages;
            if (!wait_or_abort(full0 + 8 * s, (it / kStages) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t st = base + s * kStageBytes;
            const uint32_t sAhi = st, sAlo = st + BM * 128, sBhi = st + 2 * BM * 128, sBlo = st + 3 * BM * 128;
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk) {
              const uint32_t ko = kk * 32;
              mma_tf32(dtm, sw128_desc(sAlo + ko), sw128_desc(sBhi + ko), idesc, (kt > kt0 || kk > 0) ? 1u : 0u);
              mma_tf32(dtm, sw128_desc(sAhi + ko), sw128_desc(sBlo + ko), idesc, 1u);
              mma_tf32(dtm, sw128_desc(sAhi + ko), sw128_desc(sBhi + ko), idesc, 1u);
            }
            mma_commit(empty0 + 8 * s);
          }
          if (ok) mma_commit(accf0 + 8 * b);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- accumulators + epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int chunk = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
      float acc[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = 0.f;
      for (int kt0 = 0; kt0 < nk; kt0 += kChunk, ++chunk) {
        const int b = chunk & 1;
        if (!wait_or_abort(accf0 + 8 * b, (chunk >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BN);
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
          float v[32];
          tmem_ld32(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c0 + j] = __fadd_rn(acc[c0 + j], v[j]);
        }
        tc_fence_before();
        mbar_arrive(acce0 + 8 * b);
      }
      if (ok) epilogue_store<EPI>(p, m0 + q * 32 + lane, n0, acc);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicExch(err, 1);
  if (warp == 4)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
}

// ---------------------------------------------------------------------------
// 3xFP16 with TMA-fed operands
// ---------------------------------------------------------------------------
// A pre-pass (k_split_a) writes A, row-gathered if asked, as "split fp16":
// hi = rn(a 2^s), lo = rn(a 2^s - hi) ([M, K] fp16 each) with one scale
// exponent s per row and 128-element k block ([K/128, M] int8), chosen so
// that the block's largest |element| maps into [2^14, 2^15).  The GEMM
// streams A hi/lo and the pre-split weights B hi/lo with TMA (128-byte
// swizzle, exactly the UMMA K-major layout), and one TMEM pass covers one
// k block, so the accumulator warps promote each pass with its row's block
// scale: acc += pass 2^-s.  The epilogue applies the weight tensor's scale.
constexpr int kSBlock = 128;               // k per A scale block = one TMEM pass (384 products)
constexpr int kMaxSBlocks = 16;            // K <= 2048

// Warp per row: lane l holds elements 4l..4l+3 of every 128-element block.
__global__ void __launch_bounds__(256) k_split_a(const float *__restrict__ A, int lda,
                                                 const int *__restrict__ a_rows, int M, int K, Split16View o) {
  const int m = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (m >= M) return;
  const float *row = A + static_cast<size_t>(a_rows ? a_rows[m] : m) * lda;
  const int nb = K / kSBlock;
  float4 v[kMaxSBlocks];
#pragma unroll
  for (int b = 0; b < kMaxSBlocks; ++b)
    if (b < nb) v[b] = *reinterpret_cast<const float4 *>(row + b * kSBlock + lane * 4);
#pragma unroll
  for (int b = 0; b < kMaxSBlocks; ++b) {
    if (b >= nb) break;
    warp_split_block(o, m, b, v[b], lane);
  }
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// 2D tiled TMA load (box 64 x 128 fp16, 128-byte swizzle) completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// ---- TMA epilogue ------------------------------------------------------------
// Tensor maps of the epilogue's global operands (only those the launch uses
// are encoded): fp32 C, Z (silu'), R (residual) with boxes of 16 columns x
// 32 rows, and the split output's fp16 hi / lo with boxes of 32 x 32; all
// with 64-byte rows and the 64-byte swizzle.
struct EpiMaps {
  CUtensorMap c, z, r, hi, lo;
  CUtensorMap rhi, rlo;  // residual in split form: boxes of 16 fp16 x 32 rows, no swizzle
};

__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
// 16-byte chunk c (0..3) of row r of a 32 x 64-byte staging box (64-byte swizzle)
__device__ __forceinline__ uint32_t sw64(uint32_t buf, int r, int c) {
  return buf + static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N committed bulk groups of this thread still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Per-warp state of the TMA epilogue: two 2 KB staging buffers and their
// load mbarriers; `ph` holds the parity of each buffer's next load wait,
// `pend` (lane 0's copy) the buffers with a load issued and not yet waited
// for, which an aborting warp lets land before the CTA ends.
struct EpiWarp {
  uint32_t buf0, lbar0;
  uint32_t ph;
  uint32_t pend;
};

// epilogue_store for the 3xFP16 kernel when the output rows are not
// scattered (p.c_rows == null): the same arithmetic, with the global
// operands of the epilogue moved by TMA.  Lane = row (row0 + lane); the
// 64 columns [n0, n0 + NC) go in groups of 16 (32 for the split output):
// lanes write a group into a staging buffer, one lane stores it with
// cp.async.bulk.tensor; loads of R / Z / C come the same way, two groups
// ahead (the first two are issued by epi_prefetch before the promotion).
// Rows past p.M are filled with zeros on load and clipped on store.
// Returns false if a wait timed out (the abort flag is then set).
template <int EPI>
__device__ __forceinline__ const CUtensorMap *epi_load_map(const EpiMaps &em) {
  return EPI == EPI_DSILU ? &em.z : EPI == EPI_RESID ? &em.r : &em.c;
}
// Load of one 16-column group of the epilogue input into buffer b: the
// fp32 box (64-byte swizzle), or for a split residual (rs) the hi and lo
// boxes (1 KB each, unswizzled) side by side.
template <int EPI>
__device__ __forceinline__ void epi_issue_load(const EpiMaps &em, EpiWarp &ew, int b, bool rs, int col,
                                               int row0) {
  const uint32_t bar = ew.lbar0 + 8 * b, buf = ew.buf0 + 2048 * b;
  ew.pend |= 1u << b;
  mbar_expect_tx(bar, 2048);
  if (EPI == EPI_RESID && rs) {
    tma_load_2d(buf, &em.rhi, bar, col, row0);
    tma_load_2d(buf + 1024, &em.rlo, bar, col, row0);
  } else {
    tma_load_2d(buf, epi_load_map<EPI>(em), bar, col, row0);
  }
}
template <int EPI>
__device__ __forceinline__ void epi_prefetch(const EpiMaps &em, EpiWarp &ew, bool rs, int row0, int n0,
                                             int lane) {
  if (!(EPI == EPI_DSILU || EPI == EPI_RESID || EPI == EPI_ACCUM)) return;
  if (lane == 0) {
    bulk_wait_read<0>();  // earlier stores no longer read the buffers
#pragma unroll
    for (int b = 0; b < 2; ++b) epi_issue_load<EPI>(em, ew, b, rs, n0 + 16 * b, row0);
  }
  __syncwarp();
}

template <int EPI, int NC>
__device__ __forceinline__ bool epilogue_tma(const GemmArgs &p, const EpiMaps &em, EpiWarp &ew, int row0, int lane,
                                             int n0, float (&acc)[NC], float s_b, const PairExchange *px,
                                             volatile int *abort_flag) {
  static_assert(NC % 32 == 0, "32-column split groups");
  constexpr bool kLoad = EPI == EPI_DSILU || EPI == EPI_RESID || EPI == EPI_ACCUM;
  const int row = row0 + lane;
  const bool valid = row < p.M;
  const bool split = p.c_split.hi != nullptr;
  const bool hasC = p.C != nullptr, hasZ = EPI == EPI_SILU && p.Z != nullptr;
  const bool rs = EPI == EPI_RESID && p.r_split.hi != nullptr;
  // scale of the split residual's 128-column block for this row
  const float rsf = (rs && valid) ? pow2f(-static_cast<int>(p.r_split.sc[static_cast<size_t>(n0 / 128) * split_ld(p.r_split) + row]))
                                  : 0.f;
  if (!kLoad) {  // stores of earlier tiles no longer read the buffers
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  }
#pragma unroll
  for (int g = 0; g < NC / 16; ++g) {
    const int b = g & 1;
    const uint32_t buf = ew.buf0 + 2048 * b;
    float x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = acc[16 * g + j] * s_b;
    if (p.bias) {
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 bb = __ldg(reinterpret_cast<const float4 *>(p.bias + n0 + 16 * g + j));
        x[j] += bb.x; x[j + 1] += bb.y; x[j + 2] += bb.z; x[j + 3] += bb.w;
      }
    }
    if (kLoad) {
      if (!__all_sync(0xffffffffu, wait_or_abort(ew.lbar0 + 8 * b, (ew.ph >> b) & 1u, abort_flag))) return false;
      ew.ph ^= 1u << b;
      ew.pend &= ~(1u << b);
      if (rs) {  // residual = (hi + lo) 2^-s, rows of 32 bytes
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const uint4 hv = lds128(buf + static_cast<uint32_t>(lane * 32 + 16 * m));
          const uint4 lv = lds128(buf + 1024u + static_cast<uint32_t>(lane * 32 + 16 * m));
          const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, lw[4] = {lv.x, lv.y, lv.z, lv.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 h2 = __half22float2(*reinterpret_cast<const __half2 *>(&hw[k]));
            const float2 l2 = __half22float2(*reinterpret_cast<const __half2 *>(&lw[k]));
            x[8 * m + 2 * k] += (h2.x + l2.x) * rsf;
            x[8 * m + 2 * k + 1] += (h2.y + l2.y) * rsf;
          }
        }
        __syncwarp();  // every lane has read the buffer before it is rewritten
      } else {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const uint4 v = lds128(sw64(buf, lane, m));
          const float l4[4] = {u2f(v.x), u2f(v.y), u2f(v.z), u2f(v.w)};
#pragma unroll
          for (int k = 0; k < 4; ++k) x[4 * m + k] = EPI == EPI_DSILU ? x[4 * m + k] * l4[k] : x[4 * m + k] + l4[k];
        }
      }
      // the result goes back into the same buffer, then to C; the buffer
      // then receives the group two ahead (the proxy fence orders this
      // warp's reads and writes of it before those TMA operations)
      if (hasC) {
#pragma unroll
        for (int m = 0; m < 4; ++m)
          sts128(sw64(buf, lane, m), make_uint4(f2u(x[4 * m]), f2u(x[4 * m + 1]), f2u(x[4 * m + 2]), f2u(x[4 * m + 3])));
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        if (hasC) {
          tma_store_2d(&em.c, buf, n0 + 16 * g, row0);
          bulk_commit();
        }
        if (g + 2 < NC / 16) {
          bulk_wait_read<0>();
          epi_issue_load<EPI>(em, ew, b, rs, n0 + 16 * (g + 2), row0);
        }
      }
    } else {
      uint4 zv[4];
      if (EPI == EPI_SILU) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          float y[4], dy[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) silu_pair(x[4 * m + k], y[k], dy[k]);
#pragma unroll
          for (int k = 0; k < 4; ++k) x[4 * m + k] = y[k];
          zv[m] = make_uint4(f2u(dy[0]), f2u(dy[1]), f2u(dy[2]), f2u(dy[3]));
        }
      }
      // one store per buffer and group (Z in buffer 0, C in buffer 1 for the
      // SiLU with both; otherwise buffers alternate by group)
      const int nst = (hasZ ? 1 : 0) + (hasC ? 1 : 0);
      if (nst) {
        if (lane == 0) {
          if (nst == 2) bulk_wait_read<0>();
          else bulk_wait_read<1>();
        }
        __syncwarp();
        const uint32_t bz = nst == 2 ? ew.buf0 : buf, bc = nst == 2 ? ew.buf0 + 2048 : buf;
        if (hasZ) {
#pragma unroll
          for (int m = 0; m < 4; ++m) sts128(sw64(bz, lane, m), zv[m]);
        }
        if (hasC) {
#pragma unroll
          for (int m = 0; m < 4; ++m)
            sts128(sw64(bc, lane, m), make_uint4(f2u(x[4 * m]), f2u(x[4 * m + 1]), f2u(x[4 * m + 2]), f2u(x[4 * m + 3])));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          if (hasZ) tma_store_2d(&em.z, bz, n0 + 16 * g, row0);
          if (hasC) tma_store_2d(&em.c, bc, n0 + 16 * g, row0);
          bulk_commit();
        }
      }
    }
    if (split) {
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[16 * g + j] = x[j];
    }
  }
  if (split) {
    float mx = 0.f;
    if (valid) {
#pragma unroll
      for (int j = 0; j < NC; ++j) mx = fmaxf(mx, fabsf(acc[j]));
    }
    if (NC < 128) {  // the partner warp holds the other half of the scale block
      float *slot = px->slot + px->parity * 64;
      slot[px->half * 32 + lane] = mx;
      mbar_arrive(px->bar);
      if (!__all_sync(0xffffffffu, wait_or_abort(px->bar, px->parity, px->abort_flag))) return false;
      mx = fmaxf(mx, slot[(1 - px->half) * 32 + lane]);
    }
    const int sx = split_scale_exponent(mx);
    const float f = pow2f(sx);
    const bool has_lo = p.c_split.lo != nullptr;
#pragma unroll
    for (int g = 0; g < NC / 32; ++g) {
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      if (has_lo) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          uint32_t h[4], l[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            split2(acc[32 * g + 8 * m + 2 * k], acc[32 * g + 8 * m + 2 * k + 1], f, h[k], l[k]);
          sts128(sw64(ew.buf0, lane, m), make_uint4(h[0], h[1], h[2], h[3]));
          sts128(sw64(ew.buf0 + 2048, lane, m), make_uint4(l[0], l[1], l[2], l[3]));
        }
      } else {  // hi parts only: one rounding per element, no lo store
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          uint32_t h[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const __half2 hh = __floats2half2_rn(acc[32 * g + 8 * m + 2 * k] * f, acc[32 * g + 8 * m + 2 * k + 1] * f);
            h[k] = *reinterpret_cast<const uint32_t *>(&hh);
          }
          sts128(sw64(ew.buf0, lane, m), make_uint4(h[0], h[1], h[2], h[3]));
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&em.hi, ew.buf0, n0 + 32 * g, row0);
        if (has_lo) tma_store_2d(&em.lo, ew.buf0 + 2048, n0 + 32 * g, row0);
        bulk_commit();
      }
    }
    if (valid && (NC == 128 || px->half == 0))
      p.c_split.sc[static_cast<size_t>(n0 / 128) * split_ld(p.c_split) + row] = static_cast<int8_t>(sx);
  }
  return true;
}

// ---- epilogue with scattered output rows (p.c_rows) ----------------------------
// The rows of a warp go to arbitrary destination rows, which TMA tile stores
// cannot express; 64-byte row segments still move through the staging
// buffer (64-byte swizzle) so that a warp instruction covers 8 rows x 64
// contiguous bytes.  drow: this lane's destination row, -1 for none.
__device__ __forceinline__ void rows_store64(uint32_t buf, const uint4 (&v)[4], char *base, size_t pitch, int drow,
                                             int lane) {
#pragma unroll
  for (int m = 0; m < 4; ++m) sts128(sw64(buf, lane, m), v[m]);
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2), c = lane & 3;
    const int dr = __shfl_sync(0xffffffffu, drow, r);
    const uint4 x = lds128(sw64(buf, r, c));
    if (dr >= 0) *reinterpret_cast<uint4 *>(base + static_cast<size_t>(dr) * pitch + 16 * c) = x;
  }
  __syncwarp();
}
__device__ __forceinline__ void rows_load64(uint32_t buf, uint4 (&v)[4], const char *base, size_t pitch, int srow,
                                            int lane) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2), c = lane & 3;
    const int sr = __shfl_sync(0xffffffffu, srow, r);
    sts128(sw64(buf, r, c), sr >= 0 ? *reinterpret_cast<const uint4 *>(base + static_cast<size_t>(sr) * pitch + 16 * c)
                                    : make_uint4(0u, 0u, 0u, 0u));
  }
  __syncwarp();
#pragma unroll
  for (int m = 0; m < 4; ++m) v[m] = lds128(sw64(buf, lane, m));
  __syncwarp();
}

// epilogue_store for the 3xFP16 kernel with scattered output rows: C, R and
// the split output at rows c_rows[row], Z at rows `row`, through the
// staging buffer with plain loads and stores.
template <int EPI, int NC>
__device__ __forceinline__ bool epilogue_rows(const GemmArgs &p, const EpiWarp &ew, int row0, int lane, int n0,
                                              float (&acc)[NC], float s_b, const PairExchange *px) {
  static_assert(NC % 32 == 0, "32-column split groups");
  const int row = row0 + lane;
  const bool valid = row < p.M;
  const int rc = valid ? p.c_rows[row] : -1, rz = valid ? row : -1;
  const bool split = p.c_split.hi != nullptr;
  const uint32_t buf = ew.buf0;
  if (lane == 0) bulk_wait_read<0>();  // no TMA store of this warp still reads the buffer
  __syncwarp();
#pragma unroll
  for (int g = 0; g < NC / 16; ++g) {
    const int c0 = n0 + 16 * g;
    float x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = acc[16 * g + j] * s_b;
    if (p.bias) {
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 bb = __ldg(reinterpret_cast<const float4 *>(p.bias + c0 + j));
        x[j] += bb.x; x[j + 1] += bb.y; x[j + 2] += bb.z; x[j + 3] += bb.w;
      }
    }
    if (EPI == EPI_DSILU || EPI == EPI_RESID || EPI == EPI_ACCUM) {
      uint4 lv[4];
      if (EPI == EPI_DSILU) rows_load64(buf, lv, reinterpret_cast<const char *>(p.Z + c0), sizeof(float) * p.ldz, rz, lane);
      else if (EPI == EPI_RESID) rows_load64(buf, lv, reinterpret_cast<const char *>(p.R + c0), sizeof(float) * p.ldr, rc, lane);
      else rows_load64(buf, lv, reinterpret_cast<const char *>(p.C + c0), sizeof(float) * p.ldc, rc, lane);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float l4[4] = {u2f(lv[m].x), u2f(lv[m].y), u2f(lv[m].z), u2f(lv[m].w)};
#pragma unroll
        for (int k = 0; k < 4; ++k) x[4 * m + k] = EPI == EPI_DSILU ? x[4 * m + k] * l4[k] : x[4 * m + k] + l4[k];
      }
    }
    if (EPI == EPI_SILU) {
      uint4 zv[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        float y[4], dy[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) silu_pair(x[4 * m + k], y[k], dy[k]);
#pragma unroll
        for (int k = 0; k < 4; ++k) x[4 * m + k] = y[k];
        zv[m] = make_uint4(f2u(dy[0]), f2u(dy[1]), f2u(dy[2]), f2u(dy[3]));
      }
      if (p.Z) rows_store64(buf, zv, reinterpret_cast<char *>(p.Z + c0), sizeof(float) * p.ldz, rz, lane);
    }
    if (p.C) {
      uint4 cv[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) cv[m] = make_uint4(f2u(x[4 * m]), f2u(x[4 * m + 1]), f2u(x[4 * m + 2]), f2u(x[4 * m + 3]));
      rows_store64(buf, cv, reinterpret_cast<char *>(p.C + c0), sizeof(float) * p.ldc, rc, lane);
    }
    if (split) {
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[16 * g + j] = x[j];
    }
  }
  if (split) {
    float mx = 0.f;
    if (valid) {
#pragma unroll
      for (int j = 0; j < NC; ++j) mx = fmaxf(mx, fabsf(acc[j]));
    }
    if (NC < 128) {
      float *slot = px->slot + px->parity * 64;
      slot[px->half * 32 + lane] = mx;
      mbar_arrive(px->bar);
      if (!__all_sync(0xffffffffu, wait_or_abort(px->bar, px->parity, px->abort_flag))) return false;
      mx = fmaxf(mx, slot[(1 - px->half) * 32 + lane]);
    }
    const int sx = split_scale_exponent(mx);
    const float f = pow2f(sx);
    const size_t pitch = sizeof(uint16_t) * p.c_split.cols;
#pragma unroll
    for (int g = 0; g < NC / 32; ++g) {
      uint4 hv[4], lv[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) split2(acc[32 * g + 8 * m + 2 * k], acc[32 * g + 8 * m + 2 * k + 1], f, h[k], l[k]);
        hv[m] = make_uint4(h[0], h[1], h[2], h[3]);
        lv[m] = make_uint4(l[0], l[1], l[2], l[3]);
      }
      rows_store64(buf, hv, reinterpret_cast<char *>(p.c_split.hi + n0 + 32 * g), pitch, rc, lane);
      if (p.c_split.lo) rows_store64(buf, lv, reinterpret_cast<char *>(p.c_split.lo + n0 + 32 * g), pitch, rc, lane);
    }
    if (valid && (NC == 128 || px->half == 0))
      p.c_split.sc[static_cast<size_t>(n0 / 128) * split_ld(p.c_split) + rc] = static_cast<int8_t>(sx);
  }
  return true;
}

// Tile shapes of the 3xFP16 kernel.  BN = 128: k-tiles of 64 (128-byte rows,
// 128-byte swizzle), 3 stages of 64 KB, 4 TMEM buffers, 4 accumulator
// warps.  BN = 256: k-tiles of 32 (64-byte rows, 64-byte swizzle), 4 stages
// of 48 KB (a quarter fewer operand bytes per product and one more stage in
// flight), 2 TMEM buffers of 256 columns, 8 accumulator warps (two per TMEM
// lane quarter, 128 columns each).
template <int BN_>
struct F16Cfg {
  static constexpr int BK = BN_ == 256 ? 32 : 64;
  static constexpr int RowBytes = BK * 2;
  static constexpr int ATile = BM * RowBytes;
  static constexpr int BTile = BN_ * RowBytes;
  static constexpr int StageBytes = 2 * ATile + 2 * BTile;
  static constexpr int Stages = (192 * 1024) / StageBytes;
  static constexpr int Chunk = kSBlock / BK;          // k-tiles per TMEM pass (one A scale block)
  static constexpr int TmemBufs = 512 / BN_;
  // 8 accumulator warps, two per TMEM lane quarter, each with NC columns
  static constexpr int AccWarps = 8;
  static constexpr int NC = BN_ / 2;
  static constexpr int Threads = 64 + 32 * AccWarps;
  // 10 warps put 3 on some SM sub-partitions: 168 registers at most
  static constexpr int LaunchBound = 384;
  static constexpr uint32_t Sbo = 8 * RowBytes;      // bytes between 8-row swizzle atoms
  static constexpr uint64_t Layout = BN_ == 256 ? 4 : 2;  // SWIZZLE_64B : SWIZZLE_128B
  // stages, the epilogue warps' staging buffers (2 x 2 KB each), barriers
  // and slots (512 B), the [4][2][2][32] block-max exchange, and up to
  // Slack bytes lost to aligning the base to 1024 (the kernel checks)
  static constexpr int StageOut = 2 * 2048;
  static constexpr int Slack = 512;
  static constexpr int Smem = Stages * StageBytes + AccWarps * StageOut + 512 + 2048 + Slack;
};

template <typename C>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t start) {
  return static_cast<uint64_t>((start >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<uint64_t>(C::Sbo >> 4) << 32) | (1ull << 46) | (C::Layout << 61);
}

template <int EPI, int BNt>
__global__ void __launch_bounds__(F16Cfg<BNt>::LaunchBound, 1)
    k_gemm_3xf16(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                 const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                 const __grid_constant__ EpiMaps em, GemmArgs p, const int8_t *__restrict__ sc, TCWeights16 w,
                 int *err) {
  const int b_scale = w.b_scale;
  using C = F16Cfg<BNt>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  if (base - raw > static_cast<uint32_t>(C::Slack)) {  // shared-memory plan does not fit: fail loudly
    if (threadIdx.x == 0) atomicExch(err, 3);
    return;
  }
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t ostage = base + C::Stages * C::StageBytes;  // epilogue staging, 1024-aligned
  const uint32_t bars = ostage + C::AccWarps * C::StageOut;
  const int small = C::Stages * C::StageBytes + C::AccWarps * C::StageOut;  // byte offset of `bars` from gbase
  // mbarriers: full[Stages], empty[Stages], accf[TmemBufs], acce[TmemBufs],
  // xchg[4] (block-max exchange of the two warps of each lane quarter),
  // eload[2 per epilogue warp] (TMA loads of the epilogue's inputs)
  const uint32_t full0 = bars, empty0 = bars + 8 * C::Stages, accf0 = bars + 16 * C::Stages,
                 acce0 = accf0 + 8 * C::TmemBufs, xchg0 = acce0 + 8 * C::TmemBufs, eload0 = xchg0 + 32;
  // drain: the MMA thread's commit after an abort (its MMAs complete before
  // the TMEM is freed); after eload's 16 x AccWarps bytes, below tmem_slot
  const uint32_t drain = bars + 376;
  static_assert(16 * C::Stages + 16 * C::TmemBufs + 32 + 16 * C::AccWarps <= 376, "mbarrier area");
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + small + 384);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + small + 392);
  float *xslots = reinterpret_cast<float *>(gbase + small + 512);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = p.K / C::BK;
  const int tiles_n = p.N / BNt;
  const int tiles = ((p.M + BM - 1) / BM) * tiles_n;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < C::Stages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < C::TmemBufs; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 32 * C::AccWarps);
    }
    for (int q = 0; q < 4; ++q) mbar_init(xchg0 + 8 * q, 64);
    for (int e = 0; e < 2 * C::AccWarps; ++e) mbar_init(eload0 + 8 * e, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int issued = 0;  // producer: k-stages whose loads it issued

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0;
      // the failure-detection hook: this CTA's producer issues nothing
      bool ok = p.stall_cta != static_cast<int>(blockIdx.x);
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BNt;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % C::Stages;
          if (!wait_or_abort(empty0 + 8 * s, ((it / C::Stages) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t st = base + s * C::StageBytes;
          const uint32_t fb = full0 + 8 * s;
          if (w.products == 1) {  // hi tiles only
            mbar_expect_tx(fb, C::ATile + C::BTile);
            tma_load_2d(st, &tAh, fb, kt * C::BK, m0);
            tma_load_2d(st + 2 * C::ATile, &tBh, fb, kt * C::BK, n0);
          } else {
            mbar_expect_tx(fb, C::StageBytes);
            tma_load_2d(st, &tAh, fb, kt * C::BK, m0);
            tma_load_2d(st + C::ATile, &tAl, fb, kt * C::BK, m0);
            tma_load_2d(st + 2 * C::ATile, &tBh, fb, kt * C::BK, n0);
            tma_load_2d(st + 2 * C::ATile + C::BTile, &tBl, fb, kt * C::BK, n0);
          }
        }
      }
      issued = it;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<BNt>();
      int it = 0, chunk = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        for (int kt0 = 0; kt0 < nk && ok; kt0 += C::Chunk, ++chunk) {
          const int b = chunk % C::TmemBufs;
          if (!wait_or_abort(acce0 + 8 * b, ((chunk / C::TmemBufs) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dtm = tmem + static_cast<uint32_t>(b * BNt);
          for (int kt = kt0; kt < kt0 + C::Chunk; ++kt, ++it) {
            const int s = it % C::Stages;
            if (!wait_or_abort(full0 + 8 * s, (it / C::Stages) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t st = base + s * C::StageBytes;
            const uint32_t sAhi = st, sAlo = st + C::ATile, sBhi = st + 2 * C::ATile,
                           sBlo = st + 2 * C::ATile + C::BTile;
            if (w.products == 1) {
#pragma unroll
              for (int kk = 0; kk < C::BK / 16; ++kk) {
                const uint32_t ko = kk * 32;
                mma_f16(dtm, kmajor_desc<C>(sAhi + ko), kmajor_desc<C>(sBhi + ko), idesc,
                        (kt > kt0 || kk > 0) ? 1u : 0u);
              }
            } else {
#pragma unroll
              for (int kk = 0; kk < C::BK / 16; ++kk) {
                const uint32_t ko = kk * 32;  // 16 fp16 = 32 bytes per MMA k-step
                mma_f16(dtm, kmajor_desc<C>(sAlo + ko), kmajor_desc<C>(sBhi + ko), idesc,
                        (kt > kt0 || kk > 0) ? 1u : 0u);
                mma_f16(dtm, kmajor_desc<C>(sAhi + ko), kmajor_desc<C>(sBlo + ko), idesc, 1u);
                mma_f16(dtm, kmajor_desc<C>(sAhi + ko), kmajor_desc<C>(sBhi + ko), idesc, 1u);
              }
            }
            mma_commit(empty0 + 8 * s);
          }
          if (ok) mma_commit(accf0 + 8 * b);
        }
      }
    }
    __syncwarp();
  } else {
    // ------- accumulators + epilogue: warp -> (TMEM lane quarter, column half of NC) -------
    constexpr int NC = C::NC;
    const int q = warp & 3;
    const int h = (warp - 2) / 4;
    const float sb = pow2f(-b_scale);
    int chunk = 0, ep = 0;
    bool ok = true;
    // A scale exponent of this thread's row for one 128-k chunk (0 beyond
    // the matrix), loaded one chunk ahead: the first chunk of the next tile
    // is requested before this tile's epilogue, so the load's latency
    // overlaps it instead of stalling the promotion
    const int nch = nk / C::Chunk;
    auto scale_of = [&](int tile, int c) -> int {
      const int r = (tile / tiles_n) * BM + q * 32 + lane;
      return (tile < tiles && r < p.M) ? static_cast<int>(sc[static_cast<size_t>(c) * split_ld(p.a_split) + r]) : 0;
    };
    int sc_next = scale_of(blockIdx.x, 0);
    EpiWarp ew{ostage + static_cast<uint32_t>((warp - 2) * C::StageOut), eload0 + 16u * (warp - 2), 0u, 0u};
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++ep) {
      const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BNt + h * NC;
      const int row = m0 + q * 32 + lane;
      if (!p.c_rows) epi_prefetch<EPI>(em, ew, p.r_split.hi != nullptr, m0 + q * 32, n0, lane);
      float acc[NC];
#pragma unroll
      for (int j = 0; j < NC; ++j) acc[j] = 0.f;
      for (int kt0 = 0; kt0 < nk; kt0 += C::Chunk, ++chunk) {
        const int b = chunk % C::TmemBufs;
        const int c = kt0 / C::Chunk;
        const int sc_cur = sc_next;
        sc_next = c + 1 < nch ? scale_of(tile, c + 1) : scale_of(tile + gridDim.x, 0);
        const float sa = row < p.M ? pow2f(-sc_cur) : 0.f;
        if (!__all_sync(0xffffffffu, wait_or_abort(accf0 + 8 * b, (chunk / C::TmemBufs) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr =
            tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BNt + h * NC);
#pragma unroll
        for (int c0 = 0; c0 < NC; c0 += 32) {
          float v[32];
          tmem_ld32(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c0 + j] = __fmaf_rn(v[j], sa, acc[c0 + j]);
        }
        tc_fence_before();
        mbar_arrive(acce0 + 8 * b);
      }
      if (ok) {
        const PairExchange px{xslots + q * 128, xchg0 + 8 * q, ep & 1, h, abort_flag};
        if (p.c_rows)
          ok = epilogue_rows<EPI, NC>(p, ew, m0 + q * 32, lane, n0, acc, sb, &px);
        else
          ok = epilogue_tma<EPI, NC>(p, em, ew, m0 + q * 32, lane, n0, acc, sb, &px, abort_flag);
      }
    }
    if (lane == 0) {
      // after an abort: loads of epilogue inputs still in flight land first
      for (int b = 0; b < 2; ++b)
        if ((ew.pend >> b) & 1u) wait_bounded(ew.lbar0 + 8 * b, (ew.ph >> b) & 1u);
      bulk_wait_all();  // the epilogue's stores are complete before the CTA ends
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // after an abort, this CTA's own asynchronous work completes before it
    // ends: the loads issued for the last stages (earlier ones were
    // consumed) and every MMA issued (before its TMEM is freed)
    if (warp == 0 && lane == 0)
      for (int j = issued > C::Stages ? issued - C::Stages : 0; j < issued; ++j)
        wait_bounded(full0 + 8 * (j % C::Stages), (j / C::Stages) & 1);
    if (warp == 1 && lane == 0) {
      mma_commit(drain);
      wait_bounded(drain, 0);
    }
    __syncwarp();
  }
  if (tid == 0 && *abort_flag) atomicExch(err, 1);
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// ---------------------------------------------------------------------------
// 3xFP16 on an SM pair (cta_group::2): cluster of 2 CTAs, tile 256 x 256.
// Each CTA streams its own 128 rows of A and one 128-row half of B into its
// shared memory (32 KB per k-tile of 32, 6 stages); the leader CTA (rank 0)
// issues M = 256 MMAs that read both CTAs' operands and accumulate each
// CTA's 128 rows in its own tensor memory.  Both CTAs' TMA loads complete on
// the leader's stage barrier; MMA commits arrive on the barriers of both
// CTAs; the peer's accumulator warps release a TMEM buffer by arriving on the
// leader's barrier.  No load uses multicast.
// ---------------------------------------------------------------------------
struct PairCfg {
  static constexpr int BK = 32;                       // fp16 k per tile (64-byte rows)
  static constexpr int RowBytes = 64;
  static constexpr int ATile = BM * RowBytes;         // this CTA's 128 A rows
  static constexpr int BTile = 128 * RowBytes;        // this CTA's half of the 256 B rows
  static constexpr int StageBytes = 2 * ATile + 2 * BTile;  // 32 KB
  static constexpr int Stages = 6;
  static constexpr int Chunk = kSBlock / BK;          // 4 k-tiles per TMEM pass
  static constexpr int TmemBufs = 2;                  // 2 x 256 columns
  static constexpr int AccWarps = 8;
  static constexpr int Threads = 64 + 32 * AccWarps;  // 320
  static constexpr uint32_t Sbo = 8 * RowBytes;
  static constexpr uint64_t Layout = 4;               // SWIZZLE_64B
  static constexpr int Smem = Stages * StageBytes + 1024 + 256;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory that completes on a (possibly peer) barrier.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// Commit of the leader's MMAs, arriving on the barrier at `bar` in both CTAs.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(bar), "h"(mask)
      : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(384, 1)
    k_gemm_3xf16_pair(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                      const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                      GemmArgs p, const int8_t *__restrict__ sc, int b_scale, int *err) {
  using C = PairCfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t bars = base + C::Stages * C::StageBytes;
  // mbarriers: full[Stages], empty[Stages], accf[2], acce[2] (same offsets in both CTAs)
  const uint32_t full0 = bars, empty0 = bars + 8 * C::Stages, accf0 = bars + 16 * C::Stages,
                 acce0 = accf0 + 8 * C::TmemBufs;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + C::Stages * C::StageBytes + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + C::Stages * C::StageBytes + 200);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int nk = p.K / C::BK;
  const int tiles_n = p.N / 256;
  const int tiles = ((p.M + 255) / 256) * tiles_n;
  const int pair = static_cast<int>(cluster_id_x()), npairs = static_cast<int>(num_clusters_x());

  if (tid == 0) {
    for (int s = 0; s < C::Stages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < C::TmemBufs; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 2 * 32 * C::AccWarps);  // both CTAs' accumulator threads
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // barriers and tensor memory of both CTAs exist before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        const int m0 = (tile / tiles_n) * 256 + static_cast<int>(rank) * BM;
        const int n0 = (tile % tiles_n) * 256 + static_cast<int>(rank) * 128;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % C::Stages;
          if (!wait_or_abort(empty0 + 8 * s, ((it / C::Stages) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t st = base + s * C::StageBytes;
          const uint32_t fb = map_to_rank(full0 + 8 * s, 0);
          if (leader) mbar_expect_tx(full0 + 8 * s, 2 * C::StageBytes);
          tma_load_2d_pair(st, &tAh, fb, kt * C::BK, m0);
          tma_load_2d_pair(st + C::ATile, &tAl, fb, kt * C::BK, m0);
          tma_load_2d_pair(st + 2 * C::ATile, &tBh, fb, kt * C::BK, n0);
          tma_load_2d_pair(st + 2 * C::ATile + C::BTile, &tBl, fb, kt * C::BK, n0);
        }
      }
      // tail: wait for the commits that free the last stages, so that no
      // MMA-commit arrival is still headed for this CTA when it exits
      for (int i = it; ok && i < it + C::Stages; ++i) {
        const int s = i % C::Stages;
        ok = wait_or_abort(empty0 + 8 * s, ((i / C::Stages) & 1) ^ 1, abort_flag);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (leader && lane == 0) {
      const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(256 >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);
      int it = 0, chunk = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        for (int kt0 = 0; kt0 < nk && ok; kt0 += C::Chunk, ++chunk) {
          const int b = chunk % C::TmemBufs;
          if (!wait_or_abort(acce0 + 8 * b, ((chunk / C::TmemBufs) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dtm = tmem + static_cast<uint32_t>(b * 256);
          for (int kt = kt0; kt < kt0 + C::Chunk; ++kt, ++it) {
            const int s = it % C::Stages;
            if (!wait_or_abort(full0 + 8 * s, (it / C::Stages) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t st = base + s * C::StageBytes;
            const uint32_t sAhi = st, sAlo = st + C::ATile, sBhi = st + 2 * C::ATile,
                           sBlo = st + 2 * C::ATile + C::BTile;
#pragma unroll
            for (int kk = 0; kk < C::BK / 16; ++kk) {
              const uint32_t ko = kk * 32;
              mma_f16_pair(dtm, kmajor_desc<C>(sAlo + ko), kmajor_desc<C>(sBhi + ko), idesc,
                           (kt > kt0 || kk > 0) ? 1u : 0u);
              mma_f16_pair(dtm, kmajor_desc<C>(sAhi + ko), kmajor_desc<C>(sBlo + ko), idesc, 1u);
              mma_f16_pair(dtm, kmajor_desc<C>(sAhi + ko), kmajor_desc<C>(sBhi + ko), idesc, 1u);
            }
            mma_commit_pair(empty0 + 8 * s);
          }
          if (ok) mma_commit_pair(accf0 + 8 * b);
        }
      }
    }
    __syncwarp();
  } else {
    // ------- accumulators + epilogue (both CTAs): warp -> (lane quarter, column half) -------
    const int q = warp & 3;
    const int h = (warp - 2) / 4;
    const float sb = pow2f(-b_scale);
    int chunk = 0;
    bool ok = true;
    for (int tile = pair; tile < tiles && ok; tile += npairs) {
      const int m0 = (tile / tiles_n) * 256 + static_cast<int>(rank) * BM;
      const int n0 = (tile % tiles_n) * 256 + h * 128;
      const int row = m0 + q * 32 + lane;
      float acc[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) acc[j] = 0.f;
      for (int kt0 = 0; kt0 < nk; kt0 += C::Chunk, ++chunk) {
        const int b = chunk % C::TmemBufs;
        const float sa = row < p.M ? pow2f(-static_cast<int>(sc[static_cast<size_t>(kt0 / C::Chunk) * split_ld(p.a_split) + row])) : 0.f;
        if (!wait_or_abort(accf0 + 8 * b, (chunk / C::TmemBufs) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr =
            tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 256 + h * 128);
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          float v[32];
          tmem_ld32(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c0 + j] = __fmaf_rn(v[j], sa, acc[c0 + j]);
        }
        tc_fence_before();
        mbar_arrive_cluster(map_to_rank(acce0 + 8 * b, 0));
      }
      if (ok) epilogue_store<EPI, true>(p, row, n0, acc, 1.f, sb);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicExch(err, 1);
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

int g_num_sms = 0;

template <int EPI>
void launch(const GemmArgs &a, const TCWeights &w, int *err, cudaStream_t s) {
  if (g_num_sms == 0) {
    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    CUDA_CHECK(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  CUDA_CHECK(cudaFuncSetAttribute(k_gemm_3xtf32<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  const int tiles = ceil_div(a.M, BM) * (a.N / BN);
  const int grid = tiles < g_num_sms ? tiles : g_num_sms;
  k_gemm_3xtf32<EPI><<<grid, kWsThreads, kSmemBytes, s>>>(a, w, err);
  CUDA_LAUNCH_CHECK();
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
// Tile of the 3xFP16 GEMM.  By default 128 x 128 (3 stages, 4 TMEM
// buffers: the MMA runs furthest ahead of the epilogue; fastest on most PET
// layer shapes), and 128 x 256 for wide plain-store layers (see launch16).
// MLIPCPP_B200_F16_TILE forces 128 (128 x 128), 256 (one-SM 128 x 256) or
// 512 (the SM-pair 256 x 256) where N allows.
const int g_f16_bn = [] {
  const char *e = std::getenv("MLIPCPP_B200_F16_TILE");
  return e ? std::atoi(e) : 0;
}();

// Row-major [rows, cols] fp16 matrix with leading dimension ld (elements):
// boxes of box_k x box_rows, 128- or 64-byte swizzle, zero fill outside.
void resolve_encoder() {
  if (g_encode_tiled) return;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (!fn || q != cudaDriverEntryPointSuccess) throw Error(kErrBackend, "cuTensorMapEncodeTiled unavailable");
  g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

CUtensorMap make_map_f16(const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_k,
                         uint32_t box_rows) {
  resolve_encoder();
  CUtensorMap m;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {box_k, box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUtensorMapSwizzle sw = box_k * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUresult r = g_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides,
                                    box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(kErrBackend, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return m;
}

// Map of an epilogue operand: [rows][cols] of `elem`-byte elements with
// leading dimension ld, box (32 x 64 bytes), 64-byte swizzle.
CUtensorMap make_map_epi(const void *ptr, CUtensorMapDataType type, uint32_t elem, uint64_t rows, uint64_t cols,
                         uint64_t ld, uint32_t box_bytes = 64) {
  resolve_encoder();
  CUtensorMap m;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * elem};
  const cuuint32_t box[2] = {box_bytes / elem, 32};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = g_encode_tiled(&m, type, 2, const_cast<void *>(ptr), dims, strides, box, es,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(kErrBackend, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return m;
}

std::atomic<bool> g_gemm_stall{false};

// The epilogue maps a launch uses (unscattered output rows only).
EpiMaps make_epi_maps(const GemmArgs &a) {
  EpiMaps e;
  std::memset(&e, 0, sizeof(e));
  if (a.c_rows) return e;
  const auto F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32, F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (a.C) e.c = make_map_epi(a.C, F32, 4, a.M, a.N, a.ldc);
  if (a.Z && (a.epi == EPI_SILU || a.epi == EPI_DSILU)) e.z = make_map_epi(a.Z, F32, 4, a.M, a.N, a.ldz);
  if (a.epi == EPI_RESID && a.r_split.hi) {
    e.rhi = make_map_epi(a.r_split.hi, F16, 2, a.M, a.N, a.r_split.cols, 32);
    e.rlo = make_map_epi(a.r_split.lo, F16, 2, a.M, a.N, a.r_split.cols, 32);
  } else if (a.epi == EPI_RESID) {
    e.r = make_map_epi(a.R, F32, 4, a.M, a.N, a.ldr);
  }
  if (a.c_split.hi) {
    e.hi = make_map_epi(a.c_split.hi, F16, 2, a.M, a.N, a.c_split.cols);
    if (a.c_split.lo) e.lo = make_map_epi(a.c_split.lo, F16, 2, a.M, a.N, a.c_split.cols);
  }
  return e;
}

template <int EPI, int BNt>
void launch16_bn(const GemmArgs &a, const TCWeights16 &w, int *err, cudaStream_t s) {
  const Split16View &sp = a.a_split;
  using C = F16Cfg<BNt>;
  // a hi-only A (sp.lo null) is read by one-product launches only, which
  // never load the lo map
  const CUtensorMap ah = make_map_f16(sp.hi, a.M, a.K, a.K, C::BK, BM),
                    al = make_map_f16(sp.lo ? sp.lo : sp.hi, a.M, a.K, a.K, C::BK, BM);
  const CUtensorMap bh = make_map_f16(w.hi, a.N, a.K, a.ldb, C::BK, BNt),
                    bl = make_map_f16(w.lo, a.N, a.K, a.ldb, C::BK, BNt);
  CUDA_CHECK(cudaFuncSetAttribute(k_gemm_3xf16<EPI, BNt>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::Smem));
  const int tiles = ceil_div(a.M, BM) * (a.N / BNt);
  const int grid = tiles < g_num_sms ? tiles : g_num_sms;
  const EpiMaps em = make_epi_maps(a);
  GemmArgs args = a;
  // failure-detection hook: a store epilogue with unscattered rows reads no
  // global inputs, so the stalled CTA only has its mainloop to drain
  if (EPI == EPI_STORE && !a.c_rows && g_gemm_stall.exchange(false)) args.stall_cta = 0;
  k_gemm_3xf16<EPI, BNt><<<grid, C::Threads, C::Smem, s>>>(ah, al, bh, bl, em, args, sp.sc, w, err);
  CUDA_LAUNCH_CHECK();
}

template <int EPI>
void launch16_pair(const GemmArgs &a, const TCWeights16 &w, int *err, cudaStream_t s) {
  const Split16View &sp = a.a_split;
  using C = PairCfg;
  // a hi-only A (sp.lo null) is read by one-product launches only, which
  // never load the lo map
  const CUtensorMap ah = make_map_f16(sp.hi, a.M, a.K, a.K, C::BK, BM),
                    al = make_map_f16(sp.lo ? sp.lo : sp.hi, a.M, a.K, a.K, C::BK, BM);
  const CUtensorMap bh = make_map_f16(w.hi, a.N, a.K, a.ldb, C::BK, 128),
                    bl = make_map_f16(w.lo, a.N, a.K, a.ldb, C::BK, 128);
  CUDA_CHECK(cudaFuncSetAttribute(k_gemm_3xf16_pair<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::Smem));
  const int tiles = ceil_div(a.M, 256) * (a.N / 256);
  int pairs = g_num_sms / 2;
  if (tiles < pairs) pairs = tiles;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(C::Threads);
  cfg.dynamicSmemBytes = C::Smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_gemm_3xf16_pair<EPI>, ah, al, bh, bl, a,
                                static_cast<const int8_t *>(sp.sc), w.b_scale, err));
  ::pet::g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

template <int EPI>
void launch16(const GemmArgs &a, const TCWeights16 &w, int *err, cudaStream_t s) {
  if (g_num_sms == 0) {
    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    CUDA_CHECK(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  if (!a.a_split_ready) {
    k_split_a<<<ceil_div(a.M, 8), 256, 0, s>>>(a.A, a.lda, a.a_rows, a.M, a.K, a.a_split);
    CUDA_LAUNCH_CHECK();
  }
  // default tile: 128 x 128; plain fp32-store layers run faster on 128 x 256,
  // whose B-tile reuse halves the A traffic per product (32k cell, ms per
  // launch: QKV N = 1536 4.29 -> 3.92, N = 512 K = 512 1.48 -> 1.33,
  // N = 512 K = 256 0.87 -> 0.84), while the layers with split outputs,
  // SiLU or residual epilogues ran slower there (their epilogue, 128 columns
  // per warp, sets the pace)
  const bool wide = EPI == EPI_STORE && !a.c_split.hi && !a.c_rows && a.N % 256 == 0;
  const int bn = g_f16_bn ? g_f16_bn : (wide ? 256 : 128);
  if (a.N % 256 == 0 && bn == 512 && w.products == 3 && !a.r_split.hi) launch16_pair<EPI>(a, w, err, s);
  else if (a.N % 256 == 0 && bn == 256) launch16_bn<EPI, 256>(a, w, err, s);
  else launch16_bn<EPI, 128>(a, w, err, s);
}

}  // namespace

int f16_scale_exponent(float mx) {
  if (!(mx > 0.f)) return 0;
  uint32_t u;
  std::memcpy(&u, &mx, 4);
  const int E = static_cast<int>((u >> 23) & 0xFFu);
  const int s = 141 - (E > 0 ? E : 0);
  return s < -120 ? -120 : (s > 120 ? 120 : s);
}

bool gemm_f16_supported(const GemmArgs &a) {
  return gemm_tc_supported(a) && a.K % kSBlock == 0 && a.K <= kSBlock * kMaxSBlocks && a.ldb % 8 == 0;
}

void inject_gemm_stall() { g_gemm_stall.store(true); }

bool gemm_stall_armed() { return g_gemm_stall.load(); }

void set_gemm_wait_bound_ns(uint64_t ns) {
  const uint64_t v = ns ? ns : tc::kWaitNs;
  CUDA_CHECK(cudaMemcpyToSymbol(tc::g_wait_ns, &v, sizeof(v)));
}

void gemm_3xf16(const GemmArgs &a, const TCWeights16 &w, int *err, cudaStream_t s) {
  const Split16View &sp = a.a_split;
  if (!sp.hi || sp.rows != a.M || sp.cols != a.K)
    throw Error(kErrInternal, "gemm_3xf16: split A view does not match the GEMM shape");
  if (a.c_split.hi && (a.c_split.cols != a.N || a.N % 128 != 0))
    throw Error(kErrInternal, "gemm_3xf16: split output view does not match the GEMM shape");
  if (reinterpret_cast<uintptr_t>(w.hi) % 16 || reinterpret_cast<uintptr_t>(w.lo) % 16 ||
      reinterpret_cast<uintptr_t>(sp.hi) % 16 || reinterpret_cast<uintptr_t>(sp.lo) % 16 ||
      (a.c_split.hi && (reinterpret_cast<uintptr_t>(a.c_split.hi) % 16 || reinterpret_cast<uintptr_t>(a.c_split.lo) % 16)))
    throw Error(kErrInternal, "gemm_3xf16: fp16 operands not 16-byte aligned");
  if (!sp.lo && w.products != 1)
    throw Error(kErrInternal, "gemm_3xf16: an A operand without lo parts needs the one-product mode");
  if (a.r_split.hi && !a.r_split.lo) throw Error(kErrInternal, "gemm_3xf16: a split residual needs its lo parts");
  if (a.r_split.hi && (a.epi != EPI_RESID || a.c_rows || a.r_split.rows < a.M || a.r_split.cols != a.N ||
                       reinterpret_cast<uintptr_t>(a.r_split.hi) % 16 || reinterpret_cast<uintptr_t>(a.r_split.lo) % 16))
    throw Error(kErrInternal, "gemm_3xf16: split residual view does not match the GEMM");
  switch (a.epi) {
    case EPI_STORE: launch16<EPI_STORE>(a, w, err, s); break;
    case EPI_SILU: launch16<EPI_SILU>(a, w, err, s); break;
    case EPI_ACCUM: launch16<EPI_ACCUM>(a, w, err, s); break;
    case EPI_DSILU: launch16<EPI_DSILU>(a, w, err, s); break;
    case EPI_RESID: launch16<EPI_RESID>(a, w, err, s); break;
    default: throw Error(kErrInternal, "gemm_tc: bad epilogue");
  }
}

bool gemm_tc_supported(const GemmArgs &a) {
  const bool aligned = (a.lda % 4 == 0) && (a.ldb % 4 == 0) && (a.ldc % 4 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.A) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.C) % 16 == 0) &&
                       (!a.Z || (a.ldz % 4 == 0 && reinterpret_cast<uintptr_t>(a.Z) % 16 == 0)) &&
                       (!a.R || (a.ldr % 4 == 0 && reinterpret_cast<uintptr_t>(a.R) % 16 == 0)) &&
                       (!a.bias || reinterpret_cast<uintptr_t>(a.bias) % 16 == 0);
  return aligned && a.M > 0 && a.K > 0 && a.K % BK == 0 && a.N % 128 == 0;
}

void gemm_3xtf32(const GemmArgs &a, const TCWeights &w, int *err, cudaStream_t s) {
  switch (a.epi) {
    case EPI_STORE: launch<EPI_STORE>(a, w, err, s); break;
    case EPI_SILU: launch<EPI_SILU>(a, w, err, s); break;
    case EPI_ACCUM: launch<EPI_ACCUM>(a, w, err, s); break;
    case EPI_DSILU: launch<EPI_DSILU>(a, w, err, s); break;
    case EPI_RESID: launch<EPI_RESID>(a, w, err, s); break;
    default: throw Error(kErrInternal, "gemm_tc: bad epilogue");
  }
}

}  // namespace pet
