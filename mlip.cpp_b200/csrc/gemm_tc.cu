// fp32-accurate GEMM on the 5th-generation tensor cores (tcgen05, sm_100a):
// "3xTF32" -- every fp32 operand x is split into x_hi = tf32(x) (low 13
// mantissa bits cleared) and x_lo = x - x_hi (exact in fp32), and
//   A B ~= A_hi B_hi + A_hi B_lo + A_lo B_hi
// accumulated in fp32 in tensor memory.  The dropped A_lo B_lo term and the
// truncation of x_lo are below 2^-21 relative, i.e. fp32-level accuracy.
//
// Tile: 128 (M) x BN (N, 128 or 256) x 32 (K, one 128-byte row of fp32 per
// operand row).  Operands live in shared memory in the K-major 128-byte
// swizzled layout UMMA reads (8-row x 128-byte atoms, 16-byte chunk index
// XOR row % 8, atoms 1024 bytes apart).
//  * A (activations, fp32, optionally row-gathered) is loaded by all 128
//    threads with 16-byte loads, split in registers and stored swizzled.
//  * B (weights) are pre-split on the host into hi/lo copies and streamed
//    with cp.async 16-byte copies into the swizzled layout.
//  * One thread issues 4 (k-steps of 8) x 3 tcgen05.mma per k-tile; a
//    tcgen05.commit to the stage's mbarrier frees the stage.
//  * The accumulator (128 lanes x BN fp32 columns) is read back with
//    tcgen05.ld (each warp its 32 lanes = rows) and the epilogue is fused.
// Every mbarrier wait is bounded (~1 s of %globaltimer); on expiry the kernel
// records an error code, skips the rest of its work, frees its tensor memory
// and returns, so a fault cannot hang the GPU.
#include <cstdint>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"

namespace pet {
namespace {

constexpr int BM = 128, BK = 32;
constexpr int kThreads = 128;
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

// Bounded wait; returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) return false;
  }
  return true;
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

template <int BN>
struct Smem {
  static constexpr int kA = BM * 128;       // bytes of one A operand tile
  static constexpr int kB = BN * 128;       // bytes of one B operand tile
  static constexpr int kStage = 2 * kA + 2 * kB;
  static constexpr int kStages = BN == 256 ? 2 : 3;
  static constexpr int kBytes = kStages * kStage + 1024 /*align*/ + 256 /*barriers*/;
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_3xtf32(GemmArgs p, TCWeights w, int *err) {
  using S = Smem<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + S::kStages * S::kStage;  // kStages mbarriers (8 B each)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + S::kStages * S::kStage + 64);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int nk = p.K / BK;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < S::kStages; ++s) mbar_init(bar0 + 8 * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Producer mapping: 8 threads cover one 128-byte row (one 16 B chunk each).
  const int pr = tid >> 3, pc = tid & 7;
  const float *arow[BM / 16];
#pragma unroll
  for (int i = 0; i < BM / 16; ++i) {
    const int m = m0 + pr + 16 * i;
    arow[i] = nullptr;
    if (m < p.M) {
      const int r = p.a_rows ? p.a_rows[m] : m;
      arow[i] = p.A + static_cast<size_t>(r) * p.lda;
    }
  }
  const float *bhi = w.hi + static_cast<size_t>(n0) * p.ldb;
  const float *blo = w.lo + static_cast<size_t>(n0) * p.ldb;
  const uint32_t idesc = idesc_tf32<BN>();
  bool ok = true;

  for (int kt = 0; kt < nk && ok; ++kt) {
    const int s = kt % S::kStages;
    const uint32_t st = base + s * S::kStage;
    const uint32_t sAhi = st, sAlo = st + S::kA, sBhi = st + 2 * S::kA, sBlo = sBhi + S::kB;
    if (kt >= S::kStages) {
      // thread 0 waits for the MMAs that read this stage; the verdict is
      // made uniform so the whole CTA takes the same path
      bool w_ok = true;
      if (tid == 0) w_ok = mbar_wait(bar0 + 8 * s, ((kt / S::kStages) - 1) & 1);
      if (!__syncthreads_and(w_ok)) {
        ok = false;
        break;
      }
    }
    const int k0 = kt * BK + pc * 4;
    // B: pre-split hi/lo weight rows via cp.async
#pragma unroll 4
    for (int i = 0; i < BN / 16; ++i) {
      const int r = pr + 16 * i;
      const size_t off = static_cast<size_t>(r) * p.ldb + k0;
      cp_async16(sBhi + swz(r, pc), bhi + off);
      cp_async16(sBlo + swz(r, pc), blo + off);
    }
    // A: load, split, store swizzled
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
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint32_t ko = kk * 32;  // 8 tf32 = 32 bytes along K
        const uint32_t acc0 = (kt > 0 || kk > 0) ? 1u : 0u;
        mma_tf32(tmem, sw128_desc(sAlo + ko), sw128_desc(sBhi + ko), idesc, acc0);
        mma_tf32(tmem, sw128_desc(sAhi + ko), sw128_desc(sBlo + ko), idesc, 1u);
        mma_tf32(tmem, sw128_desc(sAhi + ko), sw128_desc(sBhi + ko), idesc, 1u);
      }
      mma_commit(bar0 + 8 * s);
    }
  }
  // all MMAs done: the last commit tracks every earlier MMA of this thread
  if (ok && nk > 0) {
    const int s = (nk - 1) % S::kStages;
    bool w_ok = true;
    if (tid == 0) w_ok = mbar_wait(bar0 + 8 * s, ((nk - 1) / S::kStages) & 1);
    ok = __syncthreads_and(w_ok);
  }
  if (!ok) {
    if (lane == 0) atomicExch(err, 1);
  } else {
    tc_fence_after();
    const int row = m0 + warp * 32 + lane;
    const bool live = row < p.M;
    const int rc = live ? (p.c_rows ? p.c_rows[row] : row) : 0;
    float *crow = p.C + static_cast<size_t>(rc) * p.ldc;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
      const int nb = n0 + c0;
      if (!live || nb >= p.N) continue;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 x = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        if (p.bias) {
          const float4 b = *reinterpret_cast<const float4 *>(p.bias + nb + j);
          x.x += b.x; x.y += b.y; x.z += b.z; x.w += b.w;
        }
        float4 *dst = reinterpret_cast<float4 *>(crow + nb + j);
        if (EPI == EPI_STORE) {
          *dst = x;
        } else if (EPI == EPI_SILU) {
          *reinterpret_cast<float4 *>(p.Z + static_cast<size_t>(row) * p.ldz + nb + j) = x;
          *dst = make_float4(silu_f(x.x), silu_f(x.y), silu_f(x.z), silu_f(x.w));
        } else if (EPI == EPI_ACCUM) {
          const float4 o = *dst;
          *dst = make_float4(o.x + x.x, o.y + x.y, o.z + x.z, o.w + x.w);
        } else if (EPI == EPI_DSILU) {
          const float4 z = *reinterpret_cast<const float4 *>(p.Z + static_cast<size_t>(row) * p.ldz + nb + j);
          *dst = make_float4(x.x * dsilu_f(z.x), x.y * dsilu_f(z.y), x.z * dsilu_f(z.z), x.w * dsilu_f(z.w));
        } else {  // EPI_RESID
          const float4 r = *reinterpret_cast<const float4 *>(p.R + static_cast<size_t>(rc) * p.ldr + nb + j);
          *dst = make_float4(x.x + r.x, x.y + r.y, x.z + r.z, x.w + r.w);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
}

template <int BN, int EPI>
void launch(const GemmArgs &a, const TCWeights &w, int *err, cudaStream_t s) {
  const int bytes = Smem<BN>::kBytes;
  CUDA_CHECK(cudaFuncSetAttribute(k_gemm_3xtf32<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  dim3 grid(ceil_div(a.M, BM), a.N / BN);
  k_gemm_3xtf32<BN, EPI><<<grid, kThreads, bytes, s>>>(a, w, err);
  CUDA_LAUNCH_CHECK();
}

template <int BN>
void dispatch(const GemmArgs &a, const TCWeights &w, int *err, cudaStream_t s) {
  switch (a.epi) {
    case EPI_STORE: launch<BN, EPI_STORE>(a, w, err, s); break;
    case EPI_SILU: launch<BN, EPI_SILU>(a, w, err, s); break;
    case EPI_ACCUM: launch<BN, EPI_ACCUM>(a, w, err, s); break;
    case EPI_DSILU: launch<BN, EPI_DSILU>(a, w, err, s); break;
    case EPI_RESID: launch<BN, EPI_RESID>(a, w, err, s); break;
    default: throw Error(kErrInternal, "gemm_tc: bad epilogue");
  }
}

}  // namespace

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
  if (a.N % 256 == 0) dispatch<256>(a, w, err, s);
  else dispatch<128>(a, w, err, s);
}

}  // namespace pet
