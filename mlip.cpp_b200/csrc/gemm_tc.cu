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
#include <cuda_fp16.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"

namespace pet {
namespace {

constexpr int BM = 128, BK = 32;
constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s bound on every wait

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// K-major, 128-byte swizzle smem descriptor (tile base 1024-byte aligned):
// start >> 4 in [0,14), LBO (unused for this layout) = 1, SBO = 1024 bytes
// between 8-row atoms, version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t start) {
  return static_cast<uint64_t>((start >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

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

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(r[k]);
}

__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// Byte offset of 16-byte chunk c (0..7) of row r in a swizzled tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
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

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// 2^e for e in [-126, 127], built from its IEEE-754 bit pattern (exact).
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

template <int EPI, bool kScaled = false>
__device__ __forceinline__ void epilogue_store(const GemmArgs &p, int row, int n0, const float (&acc)[BN],
                                               float s_row = 1.f, float s_b = 1.f) {
  if (row >= p.M) return;
  const int rc = p.c_rows ? p.c_rows[row] : row;
  float *crow = p.C + static_cast<size_t>(rc) * p.ldc;
#pragma unroll
  for (int j = 0; j < BN; j += 4) {
    const int n = n0 + j;
    float4 x = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    if (kScaled) {  // two exact power-of-two multiplies
      x.x = (x.x * s_row) * s_b; x.y = (x.y * s_row) * s_b;
      x.z = (x.z * s_row) * s_b; x.w = (x.w * s_row) * s_b;
    }
    if (p.bias) {
      const float4 b = *reinterpret_cast<const float4 *>(p.bias + n);
      x.x += b.x; x.y += b.y; x.z += b.z; x.w += b.w;
    }
    float4 *dst = reinterpret_cast<float4 *>(crow + n);
    if (EPI == EPI_STORE) {
      *dst = x;
    } else if (EPI == EPI_SILU) {
      *reinterpret_cast<float4 *>(p.Z + static_cast<size_t>(row) * p.ldz + n) = x;
      *dst = make_float4(silu_f(x.x), silu_f(x.y), silu_f(x.z), silu_f(x.w));
    } else if (EPI == EPI_ACCUM) {
      const float4 o = *dst;
      *dst = make_float4(o.x + x.x, o.y + x.y, o.z + x.z, o.w + x.w);
    } else if (EPI == EPI_DSILU) {
      const float4 z = *reinterpret_cast<const float4 *>(p.Z + static_cast<size_t>(row) * p.ldz + n);
      *dst = make_float4(x.x * dsilu_f(z.x), x.y * dsilu_f(z.y), x.z * dsilu_f(z.z), x.w * dsilu_f(z.w));
    } else {  // EPI_RESID
      const float4 r = *reinterpret_cast<const float4 *>(p.R + static_cast<size_t>(rc) * p.ldr + n);
      *dst = make_float4(x.x + r.x, x.y + r.y, x.z + r.z, x.w + r.w);
    }
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
// 3xFP16: same roles and pipeline as k_gemm_3xtf32, k-tiles of 64 fp16
// ---------------------------------------------------------------------------
constexpr int BK16 = 64;
#ifndef PET_GEMM_CHUNK16
#define PET_GEMM_CHUNK16 2
#endif
// k-tiles (of 64) per TMEM accumulation pass: 2 x 64 x 3 = 384 products, as
// many as 4 tf32 k-tiles of 32
constexpr int kChunk16 = PET_GEMM_CHUNK16;

// Row pre-pass: rs[m] = s with max_k |A[m, k]| 2^s in [2^14, 2^15).
__device__ __forceinline__ int scale_exponent_dev(float mx) {
  if (!(mx > 0.f)) return 0;
  const int E = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu);
  int s = 141 - (E > 0 ? E : 0);
  return s < -120 ? -120 : (s > 120 ? 120 : s);
}

__global__ void __launch_bounds__(256) k_row_scale(const float *__restrict__ A, int lda,
                                                   const int *__restrict__ a_rows, int M, int K,
                                                   int *__restrict__ rs) {
  const int m = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (m >= M) return;
  const float *row = A + static_cast<size_t>(a_rows ? a_rows[m] : m) * lda;
  float mx = 0.f;
  for (int k = lane * 4; k < K; k += 128) {
    const float4 v = *reinterpret_cast<const float4 *>(row + k);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) rs[m] = scale_exponent_dev(mx);
}

// 8 scaled fp32 values -> 8 fp16 hi (rn) and 8 fp16 lo = rn(x - hi), packed
// in element order (lower k at the lower address).
__device__ __forceinline__ void split_f16x8(const float4 &a, const float4 &b, float sc, uint4 &hi, uint4 &lo) {
  const float x[8] = {a.x * sc, a.y * sc, a.z * sc, a.w * sc, b.x * sc, b.y * sc, b.z * sc, b.w * sc};
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 hh = __floats2half2_rn(x[2 * j], x[2 * j + 1]);
    const float2 hf = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(x[2 * j] - hf.x, x[2 * j + 1] - hf.y);
    h[j] = *reinterpret_cast<const uint32_t *>(&hh);
    l[j] = *reinterpret_cast<const uint32_t *>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int EPI>
__global__ void __launch_bounds__(kWsThreads, 1)
    k_gemm_3xf16(GemmArgs p, TCWeights16 w, const int *__restrict__ rs, int *err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t bars = base + kStages * kStageBytes;
  const uint32_t full0 = bars, empty0 = bars + 8 * kStages, accf0 = bars + 16 * kStages,
                 acce0 = accf0 + 16;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kStages * kStageBytes + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + kStages * kStageBytes + 200);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = p.K / BK16;
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
      float asc[BM / 16];
#pragma unroll
      for (int i = 0; i < BM / 16; ++i) {
        const int m = m0 + pr + 16 * i;
        arow[i] = nullptr;
        asc[i] = 1.f;
        if (m < p.M) {
          arow[i] = p.A + static_cast<size_t>(p.a_rows ? p.a_rows[m] : m) * p.lda;
          asc[i] = pow2f(rs[m]);
        }
      }
      const uint16_t *bhi = w.hi + static_cast<size_t>(n0) * p.ldb;
      const uint16_t *blo = w.lo + static_cast<size_t>(n0) * p.ldb;
      for (int kt = 0; kt < nk; ++kt, ++it) {
        const int s = it % kStages;
        if (!wait_or_abort(empty0 + 8 * s, ((it / kStages) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t st = base + s * kStageBytes;
        const uint32_t sAhi = st, sAlo = st + BM * 128, sBhi = st + 2 * BM * 128, sBlo = st + 3 * BM * 128;
        const int k0 = kt * BK16 + pc * 8;
#pragma unroll 4
        for (int i = 0; i < BN / 16; ++i) {
          const int r = pr + 16 * i;
          const size_t off = static_cast<size_t>(r) * p.ldb + k0;
          cp_async16(sBhi + swz(r, pc), bhi + off);
          cp_async16(sBlo + swz(r, pc), blo + off);
        }
        float4 va[BM / 16][2];
#pragma unroll
        for (int i = 0; i < BM / 16; ++i) {
          if (arow[i]) {
            va[i][0] = *reinterpret_cast<const float4 *>(arow[i] + k0);
            va[i][1] = *reinterpret_cast<const float4 *>(arow[i] + k0 + 4);
          } else {
            va[i][0] = va[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int i = 0; i < BM / 16; ++i) {
          const int r = pr + 16 * i;
          uint4 h, l;
          split_f16x8(va[i][0], va[i][1], asc[i], h, l);
          *reinterpret_cast<uint4 *>(gbase + (sAhi - base) + swz(r, pc)) = h;
          *reinterpret_cast<uint4 *>(gbase + (sAlo - base) + swz(r, pc)) = l;
        }
        cp_async_wait_all();
        fence_proxy_async();
        mbar_arrive(full0 + 8 * s);
      }
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<BN>();
      int it = 0, chunk = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        for (int kt0 = 0; kt0 < nk && ok; kt0 += kChunk16, ++chunk) {
          const int b = chunk & 1;
          if (!wait_or_abort(acce0 + 8 * b, ((chunk >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dtm = tmem + static_cast<uint32_t>(b * BN);
          const int kend = kt0 + kChunk16 < nk ? kt0 + kChunk16 : nk;
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
            for (int kk = 0; kk < BK16 / 16; ++kk) {
              const uint32_t ko = kk * 32;  // 16 fp16 = 32 bytes per MMA k-step
              mma_f16(dtm, sw128_desc(sAlo + ko), sw128_desc(sBhi + ko), idesc, (kt > kt0 || kk > 0) ? 1u : 0u);
              mma_f16(dtm, sw128_desc(sAhi + ko), sw128_desc(sBlo + ko), idesc, 1u);
              mma_f16(dtm, sw128_desc(sAhi + ko), sw128_desc(sBhi + ko), idesc, 1u);
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
    const int q = warp & 3;
    const float sb = pow2f(-w.b_scale);
    int chunk = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
      float acc[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = 0.f;
      for (int kt0 = 0; kt0 < nk; kt0 += kChunk16, ++chunk) {
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
      const int row = m0 + q * 32 + lane;
      if (ok) epilogue_store<EPI, true>(p, row, n0, acc, row < p.M ? pow2f(-rs[row]) : 1.f, sb);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicExch(err, 1);
  if (warp == 4)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
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

template <int EPI>
void launch16(const GemmArgs &a, const TCWeights16 &w, int *rs, int *err, cudaStream_t s) {
  if (g_num_sms == 0) {
    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    CUDA_CHECK(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  k_row_scale<<<ceil_div(a.M, 8), 256, 0, s>>>(a.A, a.lda, a.a_rows, a.M, a.K, rs);
  CUDA_LAUNCH_CHECK();
  CUDA_CHECK(cudaFuncSetAttribute(k_gemm_3xf16<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  const int tiles = ceil_div(a.M, BM) * (a.N / BN);
  const int grid = tiles < g_num_sms ? tiles : g_num_sms;
  k_gemm_3xf16<EPI><<<grid, kWsThreads, kSmemBytes, s>>>(a, w, rs, err);
  CUDA_LAUNCH_CHECK();
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
  return gemm_tc_supported(a) && a.K % BK16 == 0 && a.ldb % 8 == 0;
}

void gemm_3xf16(const GemmArgs &a, const TCWeights16 &w, int *rs, int *err, cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(w.hi) % 16 || reinterpret_cast<uintptr_t>(w.lo) % 16)
    throw Error(kErrInternal, "gemm_3xf16: fp16 weight copies not 16-byte aligned");
  switch (a.epi) {
    case EPI_STORE: launch16<EPI_STORE>(a, w, rs, err, s); break;
    case EPI_SILU: launch16<EPI_SILU>(a, w, rs, err, s); break;
    case EPI_ACCUM: launch16<EPI_ACCUM>(a, w, rs, err, s); break;
    case EPI_DSILU: launch16<EPI_DSILU>(a, w, rs, err, s); break;
    case EPI_RESID: launch16<EPI_RESID>(a, w, rs, err, s); break;
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
