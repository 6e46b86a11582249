// Per-atom attention on the 5th-generation tensor cores (tcgen05), head
// size 32, at most 64 tokens per atom.
//
// Reference: build_multi_head_attention, src/models/pet/pet_layers.cpp:318-492
// (softmax(Q K^T / sqrt(hd) + mask) V per atom, the key mask shared by all
// queries).  As in the SIMT kernels of attention.cu, each atom attends over
// its own S_i = n_i + 1 tokens only.
//
// Two atoms share one M = 128 tile: rows 0-63 are atom a's tokens, rows
// 64-127 atom b's (zero rows beyond each atom's S).  For every head, one CTA
//   1. converts Q, K (per-row power-of-two scales) and V^T (one scale per
//      head block) from fp32 into split-fp16 (hi + lo) shared-memory tiles;
//   2. issues S = Q K^T as 3 x 2 kind::f16 MMAs (M = N = 128, K = 32) into
//      tensor memory; the two off-diagonal 64 x 64 blocks are not used;
//   3. runs the softmax with one thread per row (= TMEM lane): it reads the
//      64 scores of its own atom, applies scales, 1/sqrt(hd) and the key
//      mask, and writes P (fixed scale 2^14) as split fp16 into the A tile of
//      the next product, with zeros in the other atom's key panel;
//   4. issues O = P V as 3 x 8 MMAs (M = 128, N = 32, K = 128 keys);
//   5. divides by the row sum and stores O (fp32, or split fp16 once the
//      4 heads of a 128-column block are done) and the row log-sum-exp.
// The P tile overlays the Q / K tiles, which the S MMAs have finished reading
// (80 KB of tiles, two CTAs per SM).  Every wait is bounded.
//
// Measured on the 32k-atom cell (hd 32, 16 heads): correct to the fp32
// tolerances, but 9.4 ms per launch against 6.1 ms for the SIMT kernel: each
// CTA runs the five phases of its 16 heads back to back with 8 warps per SM,
// and the tensor pipe is busy 6% of the time.  It is selected with
// MLIPCPP_B200_ATTN=tc.
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"
#include "split16.cuh"
#include "tc_common.cuh"

namespace pet {
namespace {
using namespace tc;

constexpr int kHd = 32;                // head size
constexpr int kThreads = 128;          // one thread per row / TMEM lane (two atoms x 64)
// shared-memory tiles (bytes from a 1024-aligned base)
constexpr int kQh = 0, kQl = 8192;     // Q: 128 rows x 64 B, 64-byte swizzle
constexpr int kKh = 16384, kKl = 24576;  // K: same
constexpr int kPh = 0, kPl = 32768;    // P: 2 key panels of 128 rows x 128 B (128-byte swizzle), over Q / K
constexpr int kVh = 65536, kVl = 73728;  // V^T: 2 key panels of 32 rows x 128 B
constexpr int kTiles = 81920;
// after the tiles: key scale exponents [128] int, key mask [128] float, then
// max |V| bits, the two mbarriers, the TMEM address and the abort flag
constexpr int kKScale = kTiles, kMask = kTiles + 512, kVMax = kTiles + 1024, kBars = kTiles + 1040,
              kTmemSlot = kTiles + 1056, kAbort = kTiles + 1064;
constexpr int kSmall = 1088;
constexpr int kSmem = kTiles + kSmall + 1024;  // + alignment of the base
constexpr float kPScale = 16384.f;     // P in [0, 1] -> [0, 2^14]

// 16-byte chunk c of row r in a 64-byte-swizzled tile with 64-byte rows.
__device__ __forceinline__ uint32_t swz64(int r, int c) {
  return static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// Write 32 values (one row of a K-major 64-byte-row tile) in split form.
__device__ __forceinline__ void store_row32(uint8_t *hi, uint8_t *lo, int r, const float (&v)[kHd], float f) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) split2(v[8 * c + 2 * k], v[8 * c + 2 * k + 1], f, h[k], l[k]);
    *reinterpret_cast<uint4 *>(hi + swz64(r, c)) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(lo + swz64(r, c)) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

template <int HDB>
__device__ __forceinline__ float row_absmax(const float (&v)[HDB]) {
  float m = 0.f;
#pragma unroll
  for (int c = 0; c < HDB; ++c) m = fmaxf(m, fabsf(v[c]));
  return m;
}

__global__ void __launch_bounds__(kThreads, 2) k_attn_fwd_tc(AttnArgs a, int *err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *g = smem_raw + (base - raw);
  int *s_kscale = reinterpret_cast<int *>(g + kKScale);
  float *s_mask = reinterpret_cast<float *>(g + kMask);
  int *s_vmax = reinterpret_cast<int *>(g + kVMax);  // bits of max |V| (non-negative floats order as ints)
  const uint32_t bar_s = base + kBars, bar_o = bar_s + 8;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(g + kTmemSlot);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(g + kAbort);

  const int t = threadIdx.x, warp = t >> 5;
  const int pair = blockIdx.x;
  const int own = t >> 6, r = t & 63;  // atom of this row (0: a, 1: b), token within it
  const int atom = 2 * pair + own;
  const bool has_atom = atom < a.n_atoms;
  const int e0 = has_atom ? a.offset[atom] : 0;
  const int S = has_atom ? a.offset[atom + 1] - e0 + 1 : 0;
  const bool valid = r < S;
  const int tr = atom_rows(atom, e0, a.edge_base)(r);  // token row
  const int d = a.d, ld = 3 * d;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (t == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // key mask: 0 for the node token, the fp16 log-cutoff mask of each edge,
  // -inf for the rows beyond the atom
  s_mask[t] = valid ? (r == 0 ? 0.f : a.key_mask[e0 + r - 1]) : -FLT_MAX;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_o = tmem + 128;  // S: columns [0, 128), O: [128, 160)
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const float qk_scale = rsqrtf(static_cast<float>(kHd));
  const uint32_t idesc_s = idesc_f16(128, 128), idesc_o = idesc_f16(128, kHd);

  // For the split output, the fp32 O of the 4 heads of a 128-column block
  // waits in the block's own hi / lo row segments (256 + 256 bytes = 128
  // floats) until the block is converted in place.
  for (int hg = 0; hg < a.heads / 4; ++hg) {
#pragma unroll 1
    for (int hb = 0; hb < 4; ++hb) {
      const int h = 4 * hg + hb;
      const int ph = h & 1;  // phase of both barriers for this head
      // ---- 1. Q, K, V^T of head h into split-fp16 tiles ----
      float q[kHd], k[kHd], v[kHd];
      if (valid) {
        const float *src = a.qkv + static_cast<size_t>(tr) * ld + h * kHd;
#pragma unroll
        for (int c = 0; c < kHd; c += 4) {
          const float4 x = *reinterpret_cast<const float4 *>(src + c);
          const float4 y = *reinterpret_cast<const float4 *>(src + d + c);
          const float4 z = *reinterpret_cast<const float4 *>(src + 2 * d + c);
          q[c] = x.x; q[c + 1] = x.y; q[c + 2] = x.z; q[c + 3] = x.w;
          k[c] = y.x; k[c + 1] = y.y; k[c + 2] = y.z; k[c + 3] = y.w;
          v[c] = z.x; v[c + 1] = z.y; v[c + 2] = z.z; v[c + 3] = z.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < kHd; ++c) q[c] = k[c] = v[c] = 0.f;
      }
      if (t == 0) *s_vmax = 0;
      const int sq = split_scale_exponent(row_absmax<kHd>(q));
      const int sk = split_scale_exponent(row_absmax<kHd>(k));
      store_row32(g + kQh, g + kQl, t, q, pow2f(sq));
      store_row32(g + kKh, g + kKl, t, k, pow2f(sk));
      s_kscale[t] = sk;
      __syncthreads();  // s_vmax reset seen by all
      {
        float vm = row_absmax<kHd>(v);
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, o2));
        if ((t & 31) == 0) atomicMax(s_vmax, __float_as_int(vm));
      }
      __syncthreads();
      const int sv = split_scale_exponent(__int_as_float(*s_vmax));
      {
        const float fv = pow2f(sv);
        // V^T: row = dim c, column = key t, in key panel t / 64
        uint8_t *vh = g + kVh + (t >> 6) * 4096, *vl = g + kVl + (t >> 6) * 4096;
        const int kk = t & 63;
#pragma unroll
        for (int c = 0; c < kHd; c += 2) {
          uint32_t hh, ll;
          split2(v[c], v[c + 1], fv, hh, ll);
          const uint32_t o0 = static_cast<uint32_t>(c * 128 + (((kk >> 3) ^ (c & 7)) << 4) + (kk & 7) * 2);
          const uint32_t o1 =
              static_cast<uint32_t>((c + 1) * 128 + (((kk >> 3) ^ ((c + 1) & 7)) << 4) + (kk & 7) * 2);
          *reinterpret_cast<uint16_t *>(vh + o0) = static_cast<uint16_t>(hh & 0xFFFFu);
          *reinterpret_cast<uint16_t *>(vh + o1) = static_cast<uint16_t>(hh >> 16);
          *reinterpret_cast<uint16_t *>(vl + o0) = static_cast<uint16_t>(ll & 0xFFFFu);
          *reinterpret_cast<uint16_t *>(vl + o1) = static_cast<uint16_t>(ll >> 16);
        }
      }
      fence_proxy_async();
      __syncthreads();
      // ---- 2. S = Q K^T ----
      if (t == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint32_t ko = kk * 32;
          mma_f16(t_s, kmajor_desc(base + kQl + ko, 512, 4), kmajor_desc(base + kKh + ko, 512, 4), idesc_s,
                  kk > 0 ? 1u : 0u);
          mma_f16(t_s, kmajor_desc(base + kQh + ko, 512, 4), kmajor_desc(base + kKl + ko, 512, 4), idesc_s, 1u);
          mma_f16(t_s, kmajor_desc(base + kQh + ko, 512, 4), kmajor_desc(base + kKh + ko, 512, 4), idesc_s, 1u);
        }
        mma_commit(bar_s);
      }
      // ---- 3. softmax of the row over its own atom's 64 keys ----
      wait_or_abort(bar_s, ph, abort_flag);
      tc_fence_after();
      float m = -FLT_MAX, l = 0.f;
      float s0[32], s1[32];
      tmem_ld32(t_s + lane_base + own * 64, s0);
      tmem_ld32(t_s + lane_base + own * 64 + 32, s1);
      tc_fence_before();
      {
        const float sqf = pow2f(-sq) * qk_scale;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          s0[j] = s0[j] * (sqf * pow2f(-s_kscale[own * 64 + j])) + s_mask[own * 64 + j];
          s1[j] = s1[j] * (sqf * pow2f(-s_kscale[own * 64 + 32 + j])) + s_mask[own * 64 + 32 + j];
          m = fmaxf(m, fmaxf(s0[j], s1[j]));
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          s0[j] = s_mask[own * 64 + j] == -FLT_MAX ? 0.f : expf(s0[j] - m);
          s1[j] = s_mask[own * 64 + 32 + j] == -FLT_MAX ? 0.f : expf(s1[j] - m);
          l += s0[j] + s1[j];
        }
      }
      __syncthreads();  // every row has read S; the Q / K tiles are free for P
      {
        // P row t: own key panel from the scores, the other panel zero
        uint8_t *pw = g + kPh + own * 16384, *plw = g + kPl + own * 16384;
        uint8_t *zh = g + kPh + (1 - own) * 16384, *zl = g + kPl + (1 - own) * 16384;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float *sv8 = c < 4 ? s0 + 8 * c : s1 + 8 * (c - 4);
          uint32_t hh[4], ll[4];
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) split2(sv8[2 * kq], sv8[2 * kq + 1], kPScale, hh[kq], ll[kq]);
          *reinterpret_cast<uint4 *>(pw + swz(t, c)) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
          *reinterpret_cast<uint4 *>(plw + swz(t, c)) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
          *reinterpret_cast<uint4 *>(zh + swz(t, c)) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4 *>(zl + swz(t, c)) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async();
      __syncthreads();
      // ---- 4. O = P V ----
      if (t == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int panel = kk >> 2;
          const uint32_t ko = (kk & 3) * 32;
          const uint32_t pa = base + kPh + panel * 16384 + ko, pla = base + kPl + panel * 16384 + ko;
          const uint32_t vb = base + kVh + panel * 4096 + ko, vlb = base + kVl + panel * 4096 + ko;
          mma_f16(t_o, kmajor_desc(pla, 1024, 2), kmajor_desc(vb, 1024, 2), idesc_o, kk > 0 ? 1u : 0u);
          mma_f16(t_o, kmajor_desc(pa, 1024, 2), kmajor_desc(vlb, 1024, 2), idesc_o, 1u);
          mma_f16(t_o, kmajor_desc(pa, 1024, 2), kmajor_desc(vb, 1024, 2), idesc_o, 1u);
        }
        mma_commit(bar_o);
      }
      // ---- 5. O / l, log-sum-exp ----
      wait_or_abort(bar_o, ph, abort_flag);
      tc_fence_after();
      float o[kHd];
      tmem_ld32(t_o + lane_base, o);
      tc_fence_before();
      const float f = pow2f(-sv) / (kPScale * l);
#pragma unroll
      for (int c = 0; c < kHd; ++c) o[c] *= f;
      if (valid) {
        a.lse[static_cast<size_t>(tr) * a.heads + h] = m + logf(l);
        if (a.out) {
          float *dst = a.out + static_cast<size_t>(tr) * d + h * kHd;
#pragma unroll
          for (int c = 0; c < kHd; c += 4)
            *reinterpret_cast<float4 *>(dst + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
        }
      }
      if (a.out_split.hi && valid) {
        uint16_t *seg = (hb < 2 ? a.out_split.hi : a.out_split.lo) + static_cast<size_t>(tr) * a.out_split.cols +
                        hg * 128;
        float *dst = reinterpret_cast<float *>(seg) + (hb & 1) * kHd;
#pragma unroll
        for (int c = 0; c < kHd; c += 4) *reinterpret_cast<float4 *>(dst + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
      }
      __syncthreads();  // the next head overwrites every tile
    }
    if (a.out_split.hi && valid) {
      const size_t off = static_cast<size_t>(tr) * a.out_split.cols + hg * 128;
      const float *f0 = reinterpret_cast<const float *>(a.out_split.hi + off);
      const float *f1 = reinterpret_cast<const float *>(a.out_split.lo + off);
      float ob[128];
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
        const float4 x = *reinterpret_cast<const float4 *>(f0 + c);
        const float4 y = *reinterpret_cast<const float4 *>(f1 + c);
        ob[c] = x.x; ob[c + 1] = x.y; ob[c + 2] = x.z; ob[c + 3] = x.w;
        ob[64 + c] = y.x; ob[64 + c + 1] = y.y; ob[64 + c + 2] = y.z; ob[64 + c + 3] = y.w;
      }
      const int s = split_scale_exponent(row_absmax<128>(ob));
      thread_split_store<128>(a.out_split, tr, hg * 128, ob, s);
      a.out_split.sc[static_cast<size_t>(hg) * split_ld(a.out_split) + tr] = static_cast<int8_t>(s);
    }
    if (*abort_flag) break;  // read after a barrier: the same for every thread
  }
  tc_fence_before();
  __syncthreads();
  if (t == 0 && *abort_flag) atomicExch(err, 1);
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
}

}  // namespace

bool attention_tc_supported(const AttnArgs &a) {
  return a.d == a.heads * kHd && a.max_tokens <= 64 && a.heads % 4 == 0 && a.lse &&
         (!a.out_split.hi || a.out_split.cols == a.d);
}

void attention_fwd_tc(const AttnArgs &a, int *err, cudaStream_t s) {
  if (a.n_atoms <= 0) return;
  if (!attention_tc_supported(a)) throw Error(kErrInternal, "attention_fwd_tc: unsupported shape");
  CUDA_CHECK(cudaFuncSetAttribute(k_attn_fwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
  k_attn_fwd_tc<<<(a.n_atoms + 1) / 2, kThreads, kSmem, s>>>(a, err);
  CUDA_LAUNCH_CHECK();
}

}  // namespace pet
