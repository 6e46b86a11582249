// PET forward pass and hand-written backward pass to the edge vectors, on
// ragged per-atom token blocks.  Replaces mlip.cpp's ggml graph
// (src/models/pet/pet.cpp, pet_layers.cpp) and ggml autograd
// (pet.cpp:292-320) with explicit kernels.
//
// Data layout in HBM (T = N + E token rows, row-major [T, d] fp32):
//   atom i owns rows [off_i + i, off_i + i + 1 + n_i): its node token then
//   its n_i edge tokens in neighbour-list slot order.  All dense layers run
//   on all T rows at once; attention runs per atom on its own rows.
// Stored for the backward pass (per transformer block): QKV [T,3d],
// LN-normalised inputs and 1/sigma of both layer norms, the FFN
// pre-activation [T,f]; per GNN layer the compress pre-activation [E,H] and
// the readout pre-activations.  Nothing else: no dW is needed, so GEMM
// inputs of linear layers are never kept.
#include "model.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include <cuda_fp16.h>

#include "gemm_tc.cuh"
#include "gguf.h"
#include "kernels.cuh"
#include "ops.cuh"

namespace pet {

namespace {

// Bump allocator run twice: once to size (base == nullptr), once to assign.
struct Plan {
  char *base = nullptr;
  size_t off = 0;
  template <class T> T *take(size_t n) {
    const size_t b = (n * sizeof(T) + 255) / 256 * 256;
    T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
    off += b;
    return p;
  }
};

struct BlockW {
  const float *Win, *bin, *Wout, *bout, *ga, *ba, *gm, *bm, *W0, *b0, *W3, *b3;
  const float *WinT, *WoutT, *W0T, *W3T;
};
struct HeadW {
  const float *H0, *h0, *H2, *h2, *HL, *hl, *H0T, *H2T;
};
// A forward-only property head (PropertyHead, pet_types.h:83-107):
// node and edge MLPs d -> dh -> dh -> od.
struct PropW {
  HeadW node{}, edge{};
  bool loaded = false;
};
struct LayerW {
  const float *node_emb, *C2, *c2, *C2T;
  // compress.0 with the edge and neighbour-species embeddings folded in
  // ([hid][featurised columns], bias included), its x, y, z, r columns as
  // [hid][4] for the backward, and (layer 1) the transpose of compress.0,
  // whose message rows give the message gradient
  const float *C0f, *C0xyzr, *C0T;
  BlockW blk[2];
  HeadW node, edge;
  PropW nc[2];  // non-conservative heads: [0] forces (od 3), [1] stress (od 9)
};

struct Acts {
  // graph
  float *r, *fc, *dfc_dr, *key_mask;
  int *nbr_species, *rev;
  // kept for backward
  float *qkv[4], *xa[4], *ra[4], *zf[4], *xm[4], *rm[4], *lse[4];
  float *zc[2], *zn1[2], *zn2[2], *ze1[2], *ze2[2];
  float *gfc, *e_atom;
  // non-conservative outputs per atom: forces [N1, 3], stress [N1, 9]
  float *ncF, *ncS;
  // forward scratch
  float *cat, *hc, *xin, *xmid, *xl[2], *o, *x1, *hf, *yn1, *yn2, *ye1, *ye2, *node_pred,
      *edge_pred;
  // backward scratch
  float *dx, *dx2, *du, *dout, *dqkv, *dx1, *dhf, *dz1, *dz2, *dzc, *dmsg, *g4, *g, *F;
};


GemmArgs make_gemm(const float *A, int lda, const int *a_rows, const float *B, int ldb, float *C, int ldc,
                   const int *c_rows, int M, int N, int K, const float *bias, int epi,
                   float *Z = nullptr, int ldz = 0, const float *R = nullptr, int ldr = 0) {
  GemmArgs g;
  g.A = A; g.lda = lda; g.a_rows = a_rows;
  g.B = B; g.ldb = ldb;
  g.C = C; g.ldc = ldc; g.c_rows = c_rows;
  g.M = M; g.N = N; g.K = K;
  g.bias = bias; g.epi = epi; g.Z = Z; g.ldz = ldz; g.R = R; g.ldr = ldr;
  return g;
}

// Algorithmic HBM bytes of one GEMM: A and C once, B once, plus epilogue
// side streams (Z written or read, residual read).
double gemm_bytes(const GemmArgs &g) {
  double b = 4.0 * (static_cast<double>(g.M) * g.K + static_cast<double>(g.N) * g.K +
                    static_cast<double>(g.M) * g.N);
  if (g.epi == EPI_SILU || g.epi == EPI_DSILU || g.epi == EPI_RESID || g.epi == EPI_ACCUM)
    b += 4.0 * static_cast<double>(g.M) * g.N;
  return b;
}

}  // namespace

struct PETModel::Internals {
  Acts a;
  LayerW lw[2];
};

int g_default_device = -1;  // set by mlipcpp_b200_set_device

PETModel::PETModel() : in_(new Internals()) {
  if (g_default_device >= 0) CUDA_CHECK(cudaSetDevice(g_default_device));
  CUDA_CHECK(cudaGetDevice(&device_));
  CUDA_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  for (auto &e : ev_) CUDA_CHECK(cudaEventCreate(&e));
}

PETModel::~PETModel() {
  if (gexec_) cudaGraphExecDestroy(gexec_);
  for (auto &e : ev_)
    if (e) cudaEventDestroy(e);
  for (auto &e : ev_pool_) cudaEventDestroy(e);
  if (stream_) cudaStreamDestroy(stream_);
}

void PETModel::mark_begin(cudaEvent_t &a) {
  if (ev_used_ + 2 > ev_pool_.size()) {
    for (int k = 0; k < 64; ++k) {
      cudaEvent_t e;
      CUDA_CHECK(cudaEventCreate(&e));
      ev_pool_.push_back(e);
    }
  }
  a = ev_pool_[ev_used_++];
  CUDA_CHECK(cudaEventRecord(a, stream_));
}

void PETModel::mark_end(int cls, cudaEvent_t a, double flops, double bytes) {
  cudaEvent_t b = ev_pool_[ev_used_++];
  CUDA_CHECK(cudaEventRecord(b, stream_));
  marks_.push_back({cls, a, b, flops, bytes});
}

void PETModel::collect_marks() {
  for (const Mark &m : marks_) {
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, m.a, m.b));
    KernelStat &k = kstats_[m.cls];
    k.launches += 1;
    k.ms += ms;
    k.flops += m.flops;
    k.bytes += m.bytes;
  }
  marks_.clear();
  ev_used_ = 0;
}

const float *PETModel::w(const std::string &name) const {
  auto it = wptr_.find(name);
  if (it == wptr_.end()) throw Error(kErrIO, "Required tensor '" + name + "' not found");
  return it->second;
}

const float *PETModel::device_forces() const { return in_->a.F; }

size_t PETModel::device_bytes() const {
  return wbuf_.cap + persist_.cap + scratch_.cap + sp_[0].cap + sp_[1].cap + sp_[2].cap + nl_.center.cap * 10;
}

// ---------------------------------------------------------------------------
// Weights (PETModel::load_from_gguf, pet.cpp:1100-1312)
// ---------------------------------------------------------------------------
namespace {
uint16_t float_to_half_bits(float x) {
  const __half h = __float2half_rn(x);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}
float half_bits_to_float(uint16_t b) {
  __half h;
  std::memcpy(&h, &b, 2);
  return __half2float(h);
}
}  // namespace

Split16View PETModel::split_view(int i, int rows, int cols) {
  const size_t n = static_cast<size_t>(rows) * cols;
  if (sp_[i].cap < n * 4 + n / 128) throw Error(kErrInternal, "split-fp16 buffer too small");
  Split16View v;
  v.hi = sp_[i].as<uint16_t>();
  v.lo = v.hi + n;
  v.sc = reinterpret_cast<int8_t *>(v.lo + n);
  v.rows = rows;
  v.cols = cols;
  return v;
}

int PETModel::weight_scale(size_t elem) const {
  auto it = std::upper_bound(wscale_.begin(), wscale_.end(), elem,
                             [](size_t e, const WScale &w) { return e < w.begin; });
  if (it == wscale_.begin() || elem >= (it - 1)->end) throw Error(kErrInternal, "weight pointer outside every tensor");
  return (it - 1)->scale;
}

void PETModel::load(const std::string &path, float cutoff_override) {
  GGUFFile f(path);
  const auto *emb = f.tensor("model.embedding.weight");
  if (!emb) throw Error(kErrIO, "Required tensor 'model.embedding.weight' not found");
  Hypers h;
  // pet.cpp:1178-1187; like the reference, a cutoff override set before the
  // load only survives when the file carries no pet.cutoff key.
  h.cutoff = f.get_f32("pet.cutoff", cutoff_override > 0.0f ? cutoff_override : 4.5f);
  h.heads = f.get_i32("pet.num_heads", 8);
  h.gnn_layers = f.get_i32("pet.num_gnn_layers", 2);
  h.ff = f.get_i32("pet.d_feedforward", 512);
  h.dh = f.get_i32("pet.d_head", 128);
  h.width = f.get_f32("pet.cutoff_width", 0.5f);
  h.d = static_cast<int>(emb->ne[0]);
  if (!std::isfinite(h.cutoff) || h.cutoff <= 0.0f || !std::isfinite(h.width) || h.width <= 0.0f)
    throw Error(kErrIO, "pet.cutoff and pet.cutoff_width must be finite and positive");
  if (h.gnn_layers != 2) throw Error(kErrUnsupported, "pet layout supports exactly 2 GNN layers");
  if (h.d % h.heads != 0) throw Error(kErrIO, "d_pet not divisible by num_heads");
  const auto *c0 = f.tensor("model.gnn.0.compress.0.weight");
  if (!c0) throw Error(kErrIO, "Required tensor 'model.gnn.0.compress.0.weight' not found");
  h.hid = static_cast<int>(c0->ne[1]);
  const auto *w0 = f.tensor("model.gnn.0.tl.0.mlp.0.weight");
  if (w0) h.ff = static_cast<int>(w0->ne[1]);
  const auto *hd = f.tensor("model.node_heads.energy.0.0.weight");
  if (hd) h.dh = static_cast<int>(hd->ne[1]);

  // Device copies: every f32 tensor, plus [in, out] transposes of the
  // linears the backward pass multiplies by (dX = dY W).
  std::vector<std::pair<std::string, std::vector<float>>> host;
  for (const auto &kv : f.tensors()) {
    const GGUFTensor &t = kv.second;
    if (t.type != 0) continue;
    std::vector<float> v(t.numel());
    std::memcpy(v.data(), t.data.data(), v.size() * 4);
    host.emplace_back(kv.first, std::move(v));
  }
  auto transpose_of = [&](const std::string &name) {
    const GGUFTensor *t = f.tensor(name);
    if (!t || t->ne.size() != 2) throw Error(kErrIO, "Required tensor '" + name + "' not found");
    const int64_t in = t->ne[0], out = t->ne[1];
    const float *src = reinterpret_cast<const float *>(t->data.data());
    std::vector<float> v(in * out);
    for (int64_t o = 0; o < out; ++o)
      for (int64_t i = 0; i < in; ++i) v[i * out + o] = src[o * in + i];
    host.emplace_back(name + ".T", std::move(v));
  };
  for (int l = 0; l < 2; ++l) {
    const std::string p = "model.gnn." + std::to_string(l) + ".";
    if (l > 0) transpose_of(p + "compress.0.weight");
    transpose_of(p + "compress.2.weight");
    for (int t = 0; t < 2; ++t) {
      const std::string q = p + "tl." + std::to_string(t) + ".";
      transpose_of(q + "attn.in.weight");
      transpose_of(q + "attn.out.weight");
      transpose_of(q + "mlp.0.weight");
      transpose_of(q + "mlp.3.weight");
    }
    for (const char *kind : {"node", "edge"}) {
      const std::string hp = std::string("model.") + kind + "_heads.energy." + std::to_string(l) + ".";
      transpose_of(hp + "0.weight");
      transpose_of(hp + "2.weight");
    }
  }
  // Fused compress.0 weights.  The reference feeds compress.0 the
  // concatenation [W_e (x y z r) + b_e | table[nbr species] | message]
  // (pet_layers.cpp:151-217, 685-796); the first two parts are linear in
  // per-edge data that has 5 + (table rows) degrees of freedom, so their
  // products with compress.0 are computed here once, in double precision:
  //   fused[:, msg]     = C0[:, 2d:3d]                           (layer 1)
  //   fused[:, x y z r] = C0[:, 0:d] W_e
  //   fused[:, 1]       = C0[:, 0:d] b_e + c0
  //   fused[:, 5 + s]   = C0[:, d:2d] table[s]
  // and the featuriser writes rows [msg | x y z r 1 one-hot(s) 0...].
  {
    const GGUFTensor *e0t = f.tensor("model.embedding.weight");
    const int64_t d = h.d, H = h.hid, n_tab = e0t->ne[1];
    h.aux = static_cast<int>((5 + n_tab + 127) / 128 * 128);
    auto data = [&](const std::string &name, int64_t numel) {
      const GGUFTensor *t = f.tensor(name);
      if (!t || t->type != 0 || static_cast<int64_t>(t->numel()) != numel)
        throw Error(kErrIO, "Required tensor '" + name + "' not found or of an unexpected shape");
      return reinterpret_cast<const float *>(t->data.data());
    };
    const float *emb0 = data("model.embedding.weight", n_tab * d);
    for (int l = 0; l < 2; ++l) {
      const std::string p = "model.gnn." + std::to_string(l) + ".";
      const int64_t Kin = (l == 0 ? 2 : 3) * d, K = (l == 0 ? 0 : d) + h.aux;
      const float *C0 = data(p + "compress.0.weight", H * Kin), *c0 = data(p + "compress.0.bias", H);
      const float *We = data(p + "edge_embedder.weight", 4 * d), *be = data(p + "edge_embedder.bias", d);
      const float *tab = l == 0 ? emb0 : data(p + "neighbor_embedder.weight", n_tab * d);
      std::vector<float> fw(H * K, 0.0f), px(H * 4);
      for (int64_t o = 0; o < H; ++o) {
        const float *row = C0 + o * Kin;
        float *dst = fw.data() + o * K;
        if (l > 0)
          for (int64_t c = 0; c < d; ++c) dst[c] = row[2 * d + c];
        float *aux = dst + (l == 0 ? 0 : d);
        for (int j = 0; j < 4; ++j) {
          double acc = 0.0;
          for (int64_t c = 0; c < d; ++c) acc += static_cast<double>(row[c]) * We[4 * c + j];
          aux[j] = px[4 * o + j] = static_cast<float>(acc);
        }
        double bias = c0[o];
        for (int64_t c = 0; c < d; ++c) bias += static_cast<double>(row[c]) * be[c];
        aux[4] = static_cast<float>(bias);
        for (int64_t sidx = 0; sidx < n_tab; ++sidx) {
          double acc = 0.0;
          for (int64_t c = 0; c < d; ++c) acc += static_cast<double>(row[d + c]) * tab[sidx * d + c];
          aux[5 + sidx] = static_cast<float>(acc);
        }
      }
      host.emplace_back(p + "compress.0.fused", std::move(fw));
      host.emplace_back(p + "compress.0.xyzr", std::move(px));
    }
  }
  // One arena holding five copies with identical element layout: fp32, its
  // tf32 truncation (hi) and the remainder (lo), then fp16 hi = rn(w 2^s)
  // and lo = rn(w 2^s - hi) with one power-of-two scale s per tensor, so the
  // split operands of any weight pointer (sub-blocks included) sit at fixed
  // offsets from it.
  size_t total = 0;
  for (auto &kv : host) total += (kv.second.size() * 4 + 255) / 256 * 256;
  wbuf_.ensure(4 * total);
  wspan_ = total / 4;
  wptr_.clear();
  wscale_.clear();
  std::vector<char> staging(4 * total, 0);
  uint16_t *hi16 = reinterpret_cast<uint16_t *>(staging.data() + 3 * total);
  uint16_t *lo16 = hi16 + wspan_;
  size_t off = 0;
  for (auto &kv : host) {
    std::memcpy(staging.data() + off, kv.second.data(), kv.second.size() * 4);
    float *hi = reinterpret_cast<float *>(staging.data() + total + off);
    float *lo = reinterpret_cast<float *>(staging.data() + 2 * total + off);
    float mx = 0.f;
    for (size_t k = 0; k < kv.second.size(); ++k) {
      uint32_t u;
      std::memcpy(&u, &kv.second[k], 4);
      u &= 0xFFFFE000u;
      std::memcpy(&hi[k], &u, 4);
      lo[k] = kv.second[k] - hi[k];
      mx = std::max(mx, std::fabs(kv.second[k]));
    }
    const int sc = f16_scale_exponent(mx);
    const size_t e0 = off / 4;
    for (size_t k = 0; k < kv.second.size(); ++k) {
      const float x = std::ldexp(kv.second[k], sc);
      const float xh = half_bits_to_float(hi16[e0 + k] = float_to_half_bits(x));
      lo16[e0 + k] = float_to_half_bits(x - xh);
    }
    wscale_.push_back({e0, e0 + kv.second.size(), sc});
    wptr_[kv.first] = reinterpret_cast<const float *>(wbuf_.as<char>() + off);
    off += (kv.second.size() * 4 + 255) / 256 * 256;
  }
  CUDA_CHECK(cudaMemcpy(wbuf_.ptr, staging.data(), 4 * total, cudaMemcpyHostToDevice));
  {
    const char *gr = std::getenv("MLIPCPP_B200_GRAPH");
    use_graph_ = !(gr && std::string(gr) == "0");
  }
  const char *g = std::getenv("MLIPCPP_B200_GEMM");
  use_tc_ = !(g && std::string(g) == "simt");
  use_f16_ = use_tc_ && !(g && std::string(g) == "tf32");
  {
    const char *at = std::getenv("MLIPCPP_B200_ATTN");
    use_attn_rows_ = at && (std::string(at) == "rows" || std::string(at) == "simt");
  }
  {
    // chain mode: every dense layer's K and N a multiple of 128 (K <= 2048),
    // 128 / head-size heads form one 128-column block, layer norms of <= 1024
    const int hd = h.d / h.heads;
    const bool m128 = h.d % 128 == 0 && h.ff % 128 == 0 && h.hid % 128 == 0 && h.dh % 128 == 0;
    chain_ok_ = use_f16_ && m128 && 3 * h.d <= 2048 && h.ff <= 2048 && h.hid <= 2048 && h.d <= 1024 &&
                hd > 0 && 128 % hd == 0 && h.heads % (128 / hd) == 0;
    const char *c = std::getenv("MLIPCPP_B200_CHAIN");
    if (c && std::string(c) == "0") chain_ok_ = false;
  }

  // composition map and species index (pet.cpp:1280-1303)
  species_index_.clear();
  composition_.clear();
  const auto *zt = f.tensor("composition.atomic_numbers");
  const auto *et = f.tensor("composition.energies");
  if (zt && et) {
    const int ns = static_cast<int>(zt->ne[0]);
    const int32_t *z = reinterpret_cast<const int32_t *>(zt->data.data());
    const float *e = reinterpret_cast<const float *>(et->data.data());
    for (int i = 0; i < ns; ++i) {
      composition_[z[i]] = e[i];
      species_index_[z[i]] = i;
    }
    h.n_species = ns;
  }
  for (int z = 0; z < kZTable; ++z) {
    auto si = species_index_.find(z);
    auto ci = composition_.find(z);
    zidx_[z] = si == species_index_.end() ? -1 : si->second;
    zcomp_[z] = ci == composition_.end() ? 0.0f : ci->second;
  }
  h_ = h;

  // resolve pointers once
  for (int l = 0; l < 2; ++l) {
    const std::string p = "model.gnn." + std::to_string(l) + ".";
    LayerW &L = in_->lw[l];
    L.node_emb = w(p + "node_embedder.weight");
    L.C2 = w(p + "compress.2.weight");
    L.c2 = w(p + "compress.2.bias");
    L.C0T = l > 0 ? w(p + "compress.0.weight.T") : nullptr;
    L.C0f = w(p + "compress.0.fused");
    L.C0xyzr = w(p + "compress.0.xyzr");
    L.C2T = w(p + "compress.2.weight.T");
    for (int t = 0; t < 2; ++t) {
      const std::string q = p + "tl." + std::to_string(t) + ".";
      BlockW &B = L.blk[t];
      B.Win = w(q + "attn.in.weight"); B.bin = w(q + "attn.in.bias");
      B.Wout = w(q + "attn.out.weight"); B.bout = w(q + "attn.out.bias");
      B.ga = w(q + "norm_a.weight"); B.ba = w(q + "norm_a.bias");
      B.gm = w(q + "norm_m.weight"); B.bm = w(q + "norm_m.bias");
      B.W0 = w(q + "mlp.0.weight"); B.b0 = w(q + "mlp.0.bias");
      B.W3 = w(q + "mlp.3.weight"); B.b3 = w(q + "mlp.3.bias");
      B.WinT = w(q + "attn.in.weight.T"); B.WoutT = w(q + "attn.out.weight.T");
      B.W0T = w(q + "mlp.0.weight.T"); B.W3T = w(q + "mlp.3.weight.T");
    }
    for (int k = 0; k < 2; ++k) {
      const std::string kind = k == 0 ? "node" : "edge";
      const std::string hp = "model." + kind + "_heads.energy." + std::to_string(l) + ".";
      const std::string lp = "model." + kind + "_last_layers.energy." + std::to_string(l) + ".energy___0.";
      HeadW &H = k == 0 ? L.node : L.edge;
      H.H0 = w(hp + "0.weight"); H.h0 = w(hp + "0.bias");
      H.H2 = w(hp + "2.weight"); H.h2 = w(hp + "2.bias");
      H.HL = w(lp + "weight"); H.hl = w(lp + "bias");
      H.H0T = w(hp + "0.weight.T"); H.H2T = w(hp + "2.weight.T");
    }
  }
  // Non-conservative property heads (pet.cpp:1263-1269, names
  // pet_types.h:130-138).  A layer's head counts when its node_heads.*.0
  // weight exists (PropertyHead::is_loaded); the property is used when
  // layer 0 has one (PETWeights::has_property).
  static const char *const kProp[2] = {"nc_forces", "nc_stress"};
  static const char *const kLast[2] = {"nc_f", "nc_s"};
  static const int kOut[2] = {3, 9};
  for (int p = 0; p < 2; ++p) {
    for (int l = 0; l < 2; ++l) {
      PropW &P = in_->lw[l].nc[p];
      P = PropW{};
      const std::string ls = std::to_string(l);
      if (!f.tensor(std::string("model.node_heads.") + kProp[p] + "." + ls + ".0.weight")) continue;
      for (int k = 0; k < 2; ++k) {
        const std::string kind = k == 0 ? "node" : "edge";
        const std::string hp = "model." + kind + "_heads." + kProp[p] + "." + ls + ".";
        const std::string lp = "model." + kind + "_last_layers." + kProp[p] + "." + ls + "." + kLast[p] + ".";
        auto shape_is = [&](const std::string &name, int64_t in, int64_t out) {
          const GGUFTensor *t = f.tensor(name);
          if (!t) throw Error(kErrIO, "Required tensor '" + name + "' not found");
          if (t->ne.size() < 2 || t->ne[0] != in || t->ne[1] != out)
            throw Error(kErrUnsupported, "tensor '" + name + "' has an unsupported shape (expected [" +
                                             std::to_string(out) + ", " + std::to_string(in) + "])");
        };
        shape_is(hp + "0.weight", h.d, h.dh);
        shape_is(hp + "2.weight", h.dh, h.dh);
        shape_is(lp + "weight", h.dh, kOut[p]);
        HeadW &H = k == 0 ? P.node : P.edge;
        H.H0 = w(hp + "0.weight"); H.h0 = w(hp + "0.bias");
        H.H2 = w(hp + "2.weight"); H.h2 = w(hp + "2.bias");
        H.HL = w(lp + "weight"); H.hl = w(lp + "bias");
      }
      P.loaded = true;
    }
  }
  has_ncf_ = in_->lw[0].nc[0].loaded;
  has_ncs_ = in_->lw[0].nc[1].loaded;
  (void)w("model.embedding.weight");
}

// ---------------------------------------------------------------------------
// Memory plan
// ---------------------------------------------------------------------------
// Sizes: n_local atoms in the system, layer 0 runs on the first N0 atoms
// (E0 edges, T0 = N0 + E0 tokens), layer 1 and the readout on the first N1
// (E1, T1).  A whole structure has n_local = N0 = N1.
struct Counts {
  int n_local, N0, E0, N1, E1;
  int n_in;  // layer-0 token rows received from other domains (after the T0 rows)
};

static void plan_memory(Plan &P, Plan &S, Acts &a, const Hypers &h, const Counts &c, bool grad, bool chain,
                        bool ncf, bool ncs) {
  const size_t d = h.d, f = h.ff, r = h.dh, H = h.hid;
  const size_t E0 = std::max(c.E0, 1), N0 = std::max(c.N0, 1), E1 = std::max(c.E1, 1),
               N1 = std::max(c.N1, 1), NL = std::max(c.n_local, 1);
  const size_t T0 = N0 + E0, T1 = N1 + E1;
  // persistent (graph + activations kept for backward)
  a.r = P.take<float>(E0); a.fc = P.take<float>(E0); a.dfc_dr = P.take<float>(E0);
  a.key_mask = P.take<float>(E0);
  a.nbr_species = P.take<int>(E0);
  a.rev = P.take<int>(E0);
  for (int b = 0; b < 4; ++b) {
    const size_t T = b < 2 ? T0 : T1;
    a.qkv[b] = P.take<float>(T * 3 * d);
    a.lse[b] = P.take<float>(T * h.heads);
    // LN inputs (the residual sums) and their per-row mean and 1 / sd,
    // from which the backward recomputes the normalised rows
    a.xa[b] = P.take<float>(T * d); a.ra[b] = P.take<float>(2 * T);
    a.zf[b] = P.take<float>(T * f);
    a.xm[b] = P.take<float>(T * d); a.rm[b] = P.take<float>(2 * T);
  }
  for (int l = 0; l < 2; ++l) {
    a.zc[l] = P.take<float>((l == 0 ? E0 : E1) * H);
    a.zn1[l] = P.take<float>(N1 * r); a.zn2[l] = P.take<float>(N1 * r);
    a.ze1[l] = P.take<float>(E1 * r); a.ze2[l] = P.take<float>(E1 * r);
  }
  a.gfc = P.take<float>(E0);
  a.e_atom = P.take<float>(N1);
  a.F = P.take<float>(3 * NL);
  a.ncF = ncf ? P.take<float>(3 * N1) : nullptr;
  a.ncS = ncs ? P.take<float>(9 * N1) : nullptr;
  a.g = P.take<float>(3 * E0);
  a.g4 = P.take<float>(4 * E0);
  // forward scratch
  Plan fs = S;
  // chain mode keeps GEMM-only operands (cat, hc, o, hf, yn1, ye1; dqkv,
  // dhf, dzc, dz1, dz2) in the split buffers alone
  auto ftake = [&](Plan &pl, size_t n) -> float * { return chain ? nullptr : pl.take<float>(n); };
  a.cat = ftake(fs, E0 * featurize_cols(1, h.d, h.aux)); a.hc = ftake(fs, E0 * H);
  a.xin = fs.take<float>(T0 * d); a.xmid = fs.take<float>(T0 * d);
  a.xl[0] = fs.take<float>((T0 + c.n_in) * d); a.xl[1] = fs.take<float>(T1 * d);
  a.o = ftake(fs, T0 * d); a.x1 = fs.take<float>(T0 * d);
  a.hf = ftake(fs, T0 * f);
  a.yn1 = ftake(fs, N1 * r); a.yn2 = fs.take<float>(N1 * r);
  a.ye1 = ftake(fs, E1 * r); a.ye2 = fs.take<float>(E1 * r);
  a.node_pred = fs.take<float>(N1); a.edge_pred = fs.take<float>(E1);
  size_t fwd_end = fs.off;
  // backward scratch (aliases the forward scratch)
  Plan bs = S;
  if (grad) {
    a.dx = bs.take<float>(T0 * d); a.dx2 = bs.take<float>(T0 * d); a.du = bs.take<float>(T0 * d);
    a.dout = bs.take<float>(T0 * d); a.dqkv = ftake(bs, T0 * 3 * d); a.dx1 = bs.take<float>(T0 * d);
    a.dhf = ftake(bs, T0 * f);
    const size_t rows = std::max(N1, E1);
    a.dz1 = ftake(bs, rows * r); a.dz2 = ftake(bs, rows * r);
    a.dzc = ftake(bs, E0 * H); a.dmsg = bs.take<float>(E1 * d);
  }
  S.off = std::max(fwd_end, bs.off);
}

// ---------------------------------------------------------------------------
// Forward + backward
// ---------------------------------------------------------------------------
void PETModel::forward_backward(bool grad) {
  const Acts &a = in_->a;
  const LayerW *g_lw = in_->lw;
  const Hypers &h = h_;
  const int d = h.d, f = h.ff, r = h.dh, H = h.hid;
  const int N1 = Nl_[1], E1 = El_[1], E0 = El_[0], T0 = Tl_[0];
  int N = Nl_[0], E = El_[0], T = Tl_[0];  // the layer being processed
  cudaStream_t s = stream_;
  const int *offset = nl_.offset.as<int>();
  const int *species = species_;
  const float *emb0 = w("model.embedding.weight");
  const bool ch = chain_;
  // silu' is kept for the backward only
  auto keep = [grad](float *z) { return grad ? z : nullptr; };

  // Split-fp16 operands of the chain mode: each producer takes the next
  // buffer; the GEMM that consumes it runs before the buffer comes round
  // again, and a GEMM that writes a split result writes the other buffer.
  int next_sp = 0, last_sp = 0;
  auto take_split = [&](int rows, int cols) {
    const Split16View v = split_view(next_sp, rows, cols);
    last_sp = next_sp;
    next_sp ^= 1;
    return v;
  };
  // A split buffer whose only reader is the next GEMM's A operand: in the
  // reduced-precision mode that GEMM multiplies the hi parts alone, so the
  // lo parts are neither computed nor stored.
  auto operand = [this](Split16View v) {
    if (reduced_) v.lo = nullptr;
    return v;
  };
  struct SplitIO {
    const Split16View *a = nullptr;  // A operand in split form
    bool a_ready = true;             // ... already written (else: write it from fp32 A first)
    const Split16View *c = nullptr;  // also write C in split form
    const Split16View *r = nullptr;  // EPI_RESID: residual in split form (R unused)
  };

  auto gemm = [&](const float *A, int lda, const int *a_rows, const float *B, int ldb, float *C, int ldc,
                  const int *c_rows, int M, int N, int K, const float *bias, int epi, cudaStream_t st,
                  float *Z = nullptr, int ldz = 0, const float *R = nullptr, int ldr = 0, SplitIO io = {}) {
    GemmArgs g = make_gemm(A, lda, a_rows, B, ldb, C, ldc, c_rows, M, N, K, bias, epi, Z, ldz, R, ldr);
    const float *wb = wbuf_.as<float>();
    const bool in_arena = B >= wb && B < wb + wspan_;
    const bool tc = use_tc_ && in_arena && gemm_tc_supported(g);
    const size_t eoff = in_arena ? static_cast<size_t>(B - wb) : 0;
    const bool f16 = tc && use_f16_ && gemm_f16_supported(g) && eoff % 8 == 0;
    cudaEvent_t e0 = nullptr;
    if (kprof_) mark_begin(e0);
    if (f16) {
      const uint16_t *h16 = reinterpret_cast<const uint16_t *>(wb + 3 * wspan_);
      if (io.a) {
        g.a_split = *io.a;
        g.a_split_ready = io.a_ready;
      } else {
        g.a_split = operand(split_view(0, M, K));
        g.a_split_ready = false;
      }
      if (io.c) g.c_split = *io.c;
      if (io.r) g.r_split = *io.r;
      gemm_3xf16(g, TCWeights16{h16 + eoff, h16 + wspan_ + eoff, weight_scale(eoff), reduced_ ? 1 : 3},
                 d_err_.as<int>(), st);
    } else if (io.c || io.r || (io.a && io.a_ready)) {
      throw Error(kErrInternal, "split-fp16 operands need the 3xFP16 GEMM");
    } else if (tc) {
      gemm_3xtf32(g, TCWeights{B + wspan_, B + 2 * wspan_}, d_err_.as<int>(), st);
    } else {
      gemm_f32(g, st);
    }
    if (kprof_)
      mark_end(f16 ? KC_GEMM_F16 : tc ? KC_GEMM_TC : KC_GEMM_SIMT, e0, 2.0 * M * N * static_cast<double>(K),
               gemm_bytes(g));
  };
  auto attn = [&](bool backward, const AttnArgs &x) {
    cudaEvent_t e0 = nullptr;
    if (kprof_) mark_begin(e0);
    if (!use_attn_rows_ && attention_mma_supported(x, backward)) attention_mma(x, backward, s);
    else if (backward) attention_bwd(x, s);
    else attention_fwd(x, s);
    if (kprof_) mark_end(KC_ATTENTION, e0, 0.0, 4.0 * T * (backward ? 7.0 : 4.0) * d);
    (void)x;
  };
  AttnArgs at{};
  at.key_mask = a.key_mask;
  at.offset = offset;
  at.n_atoms = N;
  at.d = d;
  at.heads = h.heads;
  at.max_tokens = max_tok_;
  at.edge_base = N;
  if (n_short_ + n_long_ > 0) {
    at.short_atoms = attn_cls_.as<int>();
    at.long_atoms = attn_cls_.as<int>() + Nl_[0];
    at.n_short = n_short_;
    at.n_long = n_long_;
  }

  // Transformer block b on input x (its split form sx in chain mode); the
  // output goes to `out` when non-null, and in chain mode also to *sout when
  // non-null.
  auto block_fwd = [&](int b, const float *x, const Split16View *sx, float *out, Split16View *sout) {
    const BlockW &B = g_lw[b / 2].blk[b % 2];
    gemm(x, d, nullptr, B.Win, d, a.qkv[b], 3 * d, nullptr, T, 3 * d, d, B.bin, EPI_STORE, s, nullptr, 0, nullptr,
         0, SplitIO{sx});
    at.qkv = a.qkv[b];
    at.lse = a.lse[b];
    at.out = a.o;
    Split16View so, sx1, shf;
    if (ch) {
      so = operand(take_split(T, d));
      at.out_split = so;
    }
    attn(false, at);
    at.out_split = Split16View{};
    // in chain mode the residuals come from the split forms, so the fp32
    // block input and x1 are not written at all
    gemm(a.o, d, nullptr, B.Wout, d, a.xa[b], d, nullptr, T, d, d, B.bout, EPI_RESID, s, nullptr, 0, ch ? nullptr : x, d,
         SplitIO{ch ? &so : nullptr, true, nullptr, ch ? sx : nullptr});
    if (ch) sx1 = take_split(T, d);
    layer_norm_fwd(a.xa[b], B.ga, B.ba, ch ? nullptr : a.x1, a.ra[b], T, d, s, ch ? &sx1 : nullptr);
    if (ch) shf = operand(take_split(T, f));
    gemm(a.x1, d, nullptr, B.W0, d, a.hf, f, nullptr, T, f, d, B.b0, EPI_SILU, s, keep(a.zf[b]), f, nullptr, 0,
         SplitIO{ch ? &sx1 : nullptr, true, ch ? &shf : nullptr});
    gemm(a.hf, f, nullptr, B.W3, f, a.xm[b], d, nullptr, T, d, f, B.b3, EPI_RESID, s, nullptr, 0, ch ? nullptr : a.x1, d,
         SplitIO{ch ? &shf : nullptr, true, nullptr, ch ? &sx1 : nullptr});
    if (ch && sout) *sout = take_split(T, d);
    layer_norm_fwd(a.xm[b], B.gm, B.bm, out, a.rm[b], T, d, s, ch ? sout : nullptr);
  };
  // Energy head (node or edge) on rows [row0, row0 + M) of the layer output:
  // x in fp32, or in chain mode its split form sxl (in split buffer fin_sp;
  // the head's hidden layer takes the other buffer).
  Split16View sxl;
  int fin_sp = 0;
  auto head_fwd = [&](const float *x, int row0, int M, const HeadW &hw, float *y1, float *y2, float *z1,
                      float *z2) {
    Split16View sa, sy;
    if (ch) {
      sa = split_rows(sxl, row0, M);
      sy = operand(split_view(fin_sp ^ 1, M, r));
    }
    gemm(x ? x + static_cast<size_t>(row0) * d : nullptr, d, nullptr, hw.H0, d, y1, r, nullptr, M, r, d, hw.h0,
         EPI_SILU, s, keep(z1), r, nullptr, 0, SplitIO{ch ? &sa : nullptr, true, ch ? &sy : nullptr});
    gemm(y1, r, nullptr, hw.H2, r, y2, r, nullptr, M, r, r, hw.h2, EPI_SILU, s, keep(z2), r, nullptr, 0,
         SplitIO{ch ? &sy : nullptr});
  };

  if (E0 > E1) CUDA_CHECK(cudaMemsetAsync(a.gfc, 0, sizeof(float) * E0, s));
  if (ncf_) CUDA_CHECK(cudaMemsetAsync(a.ncF, 0, sizeof(float) * 3 * N1, s));
  if (ncs_) CUDA_CHECK(cudaMemsetAsync(a.ncS, 0, sizeof(float) * 9 * N1, s));
  for (int l = 0; l < 2; ++l) {
    const LayerW &L = g_lw[l];
    const int K = featurize_cols(l, d, h.aux);
    N = Nl_[l];
    E = El_[l];
    T = Tl_[l];
    at.n_atoms = N;
    at.edge_base = N;
    Split16View sx;
    // layer-0 tokens of reverse edges held by other domains (collective)
    if (l == 1 && rm_) rm_->exchange_tokens(a.xl[0], Nl_[0], Tl_[0], d, s);
    if (E > 0) {
      FeaturizeArgs fa{};
      fa.n_edges = E; fa.d = d; fa.layer = l; fa.aux = h.aux;
      fa.vec = nl_.vec.as<float>(); fa.r = a.r;
      fa.nbr_species = a.nbr_species; fa.rev = a.rev;
      fa.emb0 = emb0; fa.x_prev = a.xl[0]; fa.prev_base = Nl_[0];
      fa.msg_row = (l == 1 && rm_) ? rm_->msg_row : nullptr;
      fa.cat = a.cat;
      Split16View scat, shc;
      if (ch) {
        scat = operand(take_split(E, K));
        fa.cat_split = scat;
      }
      featurize(fa, s);
      if (ch) shc = operand(take_split(E, H));
      gemm(a.cat, K, nullptr, L.C0f, K, a.hc, H, nullptr, E, H, K, nullptr, EPI_SILU, s, keep(a.zc[l]), H, nullptr, 0,
           SplitIO{ch ? &scat : nullptr, true, ch ? &shc : nullptr});
      // edge tokens: rows [N, N + E) of the layer's tokens
      Split16View sxe;
      if (ch) {
        sx = take_split(T, d);
        sxe = split_rows(sx, N, E);
      }
      gemm(a.hc, H, nullptr, L.C2, H, ch ? nullptr : a.xin + static_cast<size_t>(N) * d, d, nullptr, E, d, H, L.c2,
           EPI_STORE, s, nullptr, 0, nullptr, 0, SplitIO{ch ? &shc : nullptr, true, ch ? &sxe : nullptr});
    } else if (ch) {
      sx = take_split(T, d);
    }
    node_tokens(L.node_emb, species, ch ? nullptr : a.xin, N, d, s, ch ? &sx : nullptr);
    Split16View smid;
    block_fwd(2 * l, a.xin, ch ? &sx : nullptr, ch ? nullptr : a.xmid, ch ? &smid : nullptr);
    // layer output: fp32 for the next layer's messages (layer 0) and the
    // fp32 path; in chain mode the readout reads its split form
    block_fwd(2 * l + 1, a.xmid, ch ? &smid : nullptr, (ch && l > 0) ? nullptr : a.xl[l], ch ? &sxl : nullptr);
    fin_sp = last_sp;
    const float *xo = ch ? nullptr : a.xl[l];
    // readout (pet_layers.cpp:920-1015) of the N1 atoms whose energy counts:
    // node rows [0, N1), edge rows [N, N + E1)
    head_fwd(xo, 0, N1, L.node, a.yn1, a.yn2, a.zn1[l], a.zn2[l]);
    head_last(a.yn2, L.node.HL, L.node.hl, a.node_pred, N1, r, s);
    if (E1 > 0) {
      head_fwd(xo, N, E1, L.edge, a.ye1, a.ye2, a.ze1[l], a.ze2[l]);
      head_last(a.ye2, L.edge.HL, L.edge.hl, a.edge_pred, E1, r, s);
      add_vec(a.edge_pred, a.gfc, E1, l > 0, s);
    }
    atom_energy(a.node_pred, a.edge_pred, a.fc, offset, a.e_atom, N1, l > 0, s);
    // non-conservative heads of this layer (build_property_output,
    // pet_layers.cpp:845-915), summed over the layers per atom
    for (int p = 0; p < 2; ++p) {
      const PropW &P = L.nc[p];
      if (!P.loaded || !(p == 0 ? ncf_ : ncs_)) continue;
      head_fwd(xo, 0, N1, P.node, a.yn1, a.yn2, nullptr, nullptr);
      if (E1 > 0) head_fwd(xo, N, E1, P.edge, a.ye1, a.ye2, nullptr, nullptr);
      nc_readout(a.yn2, E1 > 0 ? a.ye2 : nullptr, P.node.HL, P.node.hl, P.edge.HL, P.edge.hl, a.fc, offset,
                 p == 0 ? a.ncF : a.ncS, N1, r, p == 0 ? 3 : 9, s);
    }
  }
  if (timing_) record_phase(4);
  if (!grad) return;

  // ---- backward ----------------------------------------------------------
  // gradient of the head's input into rows [row0, row0 + M) of dst
  auto head_bwd = [&](const HeadW &hw, const float *z1, const float *z2, const float *scale, int row0, int M,
                      float *dst) {
    Split16View s2, s1;
    if (ch) s2 = operand(take_split(M, r));
    head_last_bwd(z2, hw.HL, scale, a.dz2, M, r, s, ch ? &s2 : nullptr);
    if (ch) s1 = operand(take_split(M, r));
    gemm(a.dz2, r, nullptr, hw.H2T, r, a.dz1, r, nullptr, M, r, r, nullptr, EPI_DSILU, s, const_cast<float *>(z1), r,
         nullptr, 0, SplitIO{ch ? &s2 : nullptr, true, ch ? &s1 : nullptr});
    gemm(a.dz1, r, nullptr, hw.H0T, r, dst + static_cast<size_t>(row0) * d, d, nullptr, M, d, r, nullptr, EPI_STORE,
         s, nullptr, 0, nullptr, 0, SplitIO{ch ? &s1 : nullptr});
  };
  auto readout_bwd = [&](int l, float *dst) {
    const LayerW &L = g_lw[l];
    head_bwd(L.node, a.zn1[l], a.zn2[l], nullptr, 0, N1, dst);
    if (E1 > 0) head_bwd(L.edge, a.ze1[l], a.ze2[l], a.fc, Nl_[l], E1, dst);
  };
  // dxin: the block input's gradient in fp32; in chain mode it goes instead
  // to *sdxin in split form when that is given
  auto block_bwd = [&](int b, const float *dy, float *dxin, const Split16View *sdxin = nullptr) {
    const BlockW &B = g_lw[b / 2].blk[b % 2];
    Split16View sdu, sdhf, sdu2, sdq;
    if (ch) sdu = take_split(T, d);
    // chain mode: du is read only in split form (GEMM operand and residual)
    layer_norm_bwd(dy, a.xm[b], a.rm[b], B.gm, ch ? nullptr : a.du, T, d, s, ch ? &sdu : nullptr);
    if (ch) sdhf = operand(take_split(T, f));
    gemm(a.du, d, nullptr, B.W3T, d, a.dhf, f, nullptr, T, f, d, nullptr, EPI_DSILU, s, a.zf[b], f, nullptr, 0,
         SplitIO{ch ? &sdu : nullptr, true, ch ? &sdhf : nullptr});
    gemm(a.dhf, f, nullptr, B.W0T, f, a.dx1, d, nullptr, T, d, f, nullptr, EPI_RESID, s, nullptr, 0,
         ch ? nullptr : a.du, d, SplitIO{ch ? &sdhf : nullptr, true, nullptr, ch ? &sdu : nullptr});
    if (ch) sdu2 = take_split(T, d);
    layer_norm_bwd(a.dx1, a.xa[b], a.ra[b], B.ga, ch ? nullptr : a.du, T, d, s, ch ? &sdu2 : nullptr);
    gemm(a.du, d, nullptr, B.WoutT, d, a.dout, d, nullptr, T, d, d, nullptr, EPI_STORE, s, nullptr, 0, nullptr, 0,
         SplitIO{ch ? &sdu2 : nullptr});
    at.qkv = a.qkv[b];
    at.lse = a.lse[b];
    at.d_out = a.dout;
    at.d_qkv = a.dqkv;
    if (ch) {
      sdq = operand(take_split(T, 3 * d));
      at.dqkv_split = sdq;
    }
    attn(true, at);
    at.dqkv_split = Split16View{};
    const bool sout = ch && sdxin;
    gemm(a.dqkv, 3 * d, nullptr, B.WinT, 3 * d, sout ? nullptr : dxin, d, nullptr, T, d, 3 * d, nullptr, EPI_RESID, s,
         nullptr, 0, ch ? nullptr : a.du, d,
         SplitIO{ch ? &sdq : nullptr, true, sout ? sdxin : nullptr, ch ? &sdu2 : nullptr});
  };
  // dtok: the token gradient (fp32; in chain mode its split form sdtok)
  auto compress_bwd = [&](int l, const float *dtok, const Split16View *sdtok, bool accumulate) {
    const LayerW &L = g_lw[l];
    Split16View sa, sz;
    if (ch) {
      sa = split_rows(*sdtok, Nl_[l], E);  // the edge rows
      sz = take_split(E, H);
    }
    gemm(ch ? nullptr : dtok + static_cast<size_t>(Nl_[l]) * d, d, nullptr, L.C2T, d, a.dzc, H, nullptr, E, H, d,
         nullptr, EPI_DSILU, s, a.zc[l], H, nullptr, 0, SplitIO{ch ? &sa : nullptr, true, ch ? &sz : nullptr});
    if (l == 1)
      gemm(a.dzc, H, nullptr, L.C0T + static_cast<size_t>(2) * d * H, H, a.dmsg, d, nullptr, E, d, H, nullptr,
           EPI_STORE, s, nullptr, 0, nullptr, 0, SplitIO{ch ? &sz : nullptr});
    // d/d[x y z r] through the fused weight's edge-embedding columns
    edge_xyzr_bwd(a.dzc, ch ? &sz : nullptr, L.C0xyzr, a.g4, E, H, accumulate, s);
  };

  // layer 1 (its N1 atoms), then layer 0 (N0 atoms); layer-0 tokens of
  // atoms beyond N1 receive gradient only through the reversed messages.
  N = N1; E = E1; T = Tl_[1];
  at.n_atoms = N;
  at.edge_base = N;
  if (E0 > 0) CUDA_CHECK(cudaMemsetAsync(a.g4, 0, sizeof(float) * 4 * E0, s));
  readout_bwd(1, a.dx);
  block_bwd(3, a.dx, a.dx2);
  // the first block's input gradient feeds only the compression backward
  Split16View sdx;
  if (ch) sdx = operand(split_view(2, T, d));
  block_bwd(2, a.dx2, a.dx, ch ? &sdx : nullptr);
  if (E > 0) compress_bwd(1, a.dx, ch ? &sdx : nullptr, true);
  N = Nl_[0]; E = E0; T = T0;
  at.n_atoms = N;
  at.edge_base = N;
  if (T0 > Tl_[1]) CUDA_CHECK(cudaMemsetAsync(a.dx, 0, sizeof(float) * static_cast<size_t>(T0) * d, s));
  readout_bwd(0, a.dx);
  if (E1 > 0) message_bwd(a.dmsg, d, a.rev, Nl_[0], a.dx, E0, E1, d, s);
  // gradients of the messages whose tokens came from other domains go back
  // to them, and theirs for this domain's tokens come in (collective)
  if (rm_) rm_->exchange_token_grads(a.dmsg, a.dx, Nl_[0], d, s);
  block_bwd(1, a.dx, a.dx2);
  if (ch) sdx = operand(split_view(2, T, d));
  block_bwd(0, a.dx2, a.dx, ch ? &sdx : nullptr);
  if (E0 > 0) {
    compress_bwd(0, a.dx, ch ? &sdx : nullptr, true);
    edge_grad(a.g4, a.gfc, a.dfc_dr, nl_.vec.as<float>(), a.r, a.g, E0, s);
  }
  if (n_local_ > Nl_[0]) CUDA_CHECK(cudaMemsetAsync(a.F, 0, sizeof(float) * 3 * n_local_, s));
  forces(a.g, offset, nl_.nbr.as<int>(), a.rev, a.F, Nl_[0], E0, s);
  if (timing_) record_phase(5);
}

// ---------------------------------------------------------------------------
// Prediction
// ---------------------------------------------------------------------------
// Everything the launches of forward_backward depend on: shapes, modes and
// the addresses of every buffer they touch.  Equal keys launch identical
// work, so a graph captured under one key replays for the next.
std::vector<uintptr_t> PETModel::graph_key(bool grad) const {
  auto p = [](const void *x) { return reinterpret_cast<uintptr_t>(x); };
  return {static_cast<uintptr_t>(n_local_), static_cast<uintptr_t>(Nl_[0]), static_cast<uintptr_t>(Nl_[1]),
          static_cast<uintptr_t>(El_[0]), static_cast<uintptr_t>(El_[1]), static_cast<uintptr_t>(max_tok_),
          (grad ? 1u : 0u) | (ncf_ ? 2u : 0u) | (ncs_ ? 4u : 0u) | (chain_ ? 8u : 0u) | (reduced_ ? 16u : 0u) |
              (timing_ ? 32u : 0u),
          p(persist_.ptr), p(scratch_.ptr), p(sp_[0].ptr), p(sp_[1].ptr), p(sp_[2].ptr), p(wbuf_.ptr),
          p(nl_.offset.ptr), p(nl_.center.ptr), p(nl_.nbr.ptr), p(nl_.shift.ptr), p(nl_.vec.ptr), p(nl_.dist.ptr),
          p(species_), p(d_err_.ptr), static_cast<uintptr_t>(n_short_), p(attn_cls_.ptr)};
}

// Phase boundary i of the step's timing.  Inside a capture the record
// becomes a node of the graph, so that each replay records the event.
void PETModel::record_phase(int i) {
  if (capturing_) CUDA_CHECK(cudaEventRecordWithFlags(ev_[i], stream_, cudaEventRecordExternal));
  else CUDA_CHECK(cudaEventRecord(ev_[i], stream_));
}

// forward_backward is about 110 launches.  For small structures their
// launch latency is a large part of a step, so when a prediction has the
// same key as the one before it (the same shapes in the same buffers, as
// when a structure is evaluated again or strained in place), the launches
// are captured once into a CUDA graph and replayed from then on.  A first
// or changed key runs eagerly, so one-off shapes pay no capture.  Kernel
// profiling, the domain path's exchanges and an armed failure-test stall
// always run eagerly.  If the capture fails, graphs are switched off for
// this model and the step runs eagerly.
void PETModel::run_forward_backward(bool grad) {
  if (!use_graph_ || kprof_ || rm_ || gemm_stall_armed()) {
    forward_backward(grad);
    return;
  }
  std::vector<uintptr_t> key = graph_key(grad);
  if (gexec_ && key == gkey_) {
    CUDA_CHECK(cudaGraphLaunch(gexec_, stream_));
    g_kernel_launches.fetch_add(graph_kernels_, std::memory_order_relaxed);
    return;
  }
  if (key != last_key_) {
    last_key_ = std::move(key);
    forward_backward(grad);
    return;
  }
  const long long k0 = g_kernel_launches.load();
  cudaGraph_t graph = nullptr;
  CUDA_CHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
  capturing_ = true;
  try {
    forward_backward(grad);
    capturing_ = false;
  } catch (...) {
    capturing_ = false;
    cudaStreamEndCapture(stream_, &graph);
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    use_graph_ = false;
    forward_backward(grad);
    return;
  }
  if (cudaStreamEndCapture(stream_, &graph) != cudaSuccess || !graph) {
    cudaGetLastError();
    use_graph_ = false;
    forward_backward(grad);
    return;
  }
  graph_kernels_ = g_kernel_launches.load() - k0;
  bool updated = false;
  if (gexec_) {
    cudaGraphExecUpdateResultInfo info;
    updated = cudaGraphExecUpdate(gexec_, graph, &info) == cudaSuccess;
    if (!updated) {
      cudaGetLastError();
      cudaGraphExecDestroy(gexec_);
      gexec_ = nullptr;
    }
  }
  if (!updated) CUDA_CHECK(cudaGraphInstantiate(&gexec_, graph, 0));
  cudaGraphDestroy(graph);
  gkey_ = last_key_;
  CUDA_CHECK(cudaGraphLaunch(gexec_, stream_));
}

void PETModel::setup_graph(int n_local, int N0, int E0, int N1, int E1, const int *d_species, bool grad, int n_in) {
  n_local_ = n_local;
  Nl_[0] = N0; El_[0] = E0; Tl_[0] = N0 + E0;
  Nl_[1] = N1; El_[1] = E1; Tl_[1] = N1 + E1;
  max_tok_ = nl_.max_count + 1;
  species_ = d_species;
  if (max_tok_ > attention_max_tokens(h_.d / h_.heads))
    throw Error(kErrUnsupported, "an atom has " + std::to_string(nl_.max_count) +
                                     (skin_ > 0.f ? " neighbours within the cutoff plus the neighbour-list skin"
                                                  : " neighbours") +
                                     ", above the supported maximum of " +
                                     std::to_string(attention_max_tokens(h_.d / h_.heads) - 1));
  chain_ = chain_ok_ && max_tok_ <= attention_split_max_tokens(h_.d / h_.heads);
  // atoms with more tokens than the short-sequence attention kernels take:
  // split the atoms into two classes so that only those run on the general
  // kernels (one host read of the class sizes)
  n_short_ = n_long_ = 0;
  if (!use_attn_rows_ && max_tok_ > attention_short_tokens() && N0 == N1 && N0 > 0) {
    int *cls = static_cast<int *>(attn_cls_.ensure(sizeof(int) * (2 * static_cast<size_t>(N0) + 2)));
    int *counts = cls + 2 * static_cast<size_t>(N0);
    CUDA_CHECK(cudaMemsetAsync(counts, 0, 2 * sizeof(int), stream_));
    attention_classes(nl_.offset.as<int>(), N0, attention_short_tokens(), cls, cls + N0, counts, stream_);
    int hc[2] = {0, 0};
    CUDA_CHECK(cudaMemcpyAsync(hc, counts, sizeof(hc), cudaMemcpyDeviceToHost, stream_));
    CUDA_CHECK(cudaStreamSynchronize(stream_));
    n_short_ = hc[0];
    n_long_ = hc[1];
  }
  // memory plan: size, allocate, assign
  const Counts c{n_local, N0, E0, N1, E1, n_in};
  Plan P, S;
  plan_memory(P, S, in_->a, h_, c, grad, chain_, ncf_, ncs_);
  persist_.ensure(P.off);
  scratch_.ensure(S.off);
  if (use_f16_) {  // largest A operand of a 3xFP16 GEMM: [tokens, max(3d, ff, hid)]
    const size_t kmax = static_cast<size_t>(std::max({3 * h_.d, h_.ff, h_.hid, featurize_cols(1, h_.d, h_.aux)}));
    const size_t mk = static_cast<size_t>(std::max(Tl_[0], Tl_[1])) * kmax;
    sp_[0].ensure(mk * 4 + mk / 128 + 256);
    if (chain_) sp_[1].ensure(mk * 4 + mk / 128 + 256);
    const size_t md = static_cast<size_t>(std::max(Tl_[0], Tl_[1])) * h_.d;
    if (chain_ && grad) sp_[2].ensure(md * 4 + md / 128 + 256);
  }
  P = Plan{persist_.as<char>(), 0};
  S = Plan{scratch_.as<char>(), 0};
  plan_memory(P, S, in_->a, h_, c, grad, chain_, ncf_, ncs_);
  const Acts &a = in_->a;
  EdgePrepArgs ep{};
  ep.n_atoms = N0; ep.n_edges = E0;
  ep.offset = nl_.offset.as<int>(); ep.center = nl_.center.as<int>(); ep.nbr = nl_.nbr.as<int>();
  ep.shift = nl_.shift.as<int>(); ep.species = d_species;
  ep.vec = nl_.vec.as<float>(); ep.dist_nl = nl_.dist.as<float>();
  ep.cutoff = h_.cutoff; ep.width = h_.width;
  ep.r = a.r; ep.fc = a.fc; ep.dfc_dr = a.dfc_dr; ep.key_mask = a.key_mask;
  ep.nbr_species = a.nbr_species; ep.rev = a.rev;
  edge_prep(ep, stream_);
}

const int *PETModel::device_species_map() {
  if (!d_zmap_.ptr) {
    int h[128];
    for (int z = 0; z < 128; ++z) {
      h[z] = species_of(z);
    }
    CUDA_CHECK(cudaMemcpy(d_zmap_.ensure(sizeof(h)), h, sizeof(h), cudaMemcpyHostToDevice));
  }
  return d_zmap_.as<int>();
}

bool PETModel::skin_list(const float *d_pos, int n, const SystemView &sys, cudaStream_t s) {
  const bool periodic = sys.cell != nullptr;
  SkinGeom sg{};
  if (periodic) {
    for (int k = 0; k < 9; ++k) sg.cell[k] = sys.cell[k];
    const double *m = sg.cell;
    const double det = m[0] * (m[4] * m[8] - m[5] * m[7]) - m[1] * (m[3] * m[8] - m[5] * m[6]) +
                       m[2] * (m[3] * m[7] - m[4] * m[6]);
    const double c[9] = {m[4] * m[8] - m[5] * m[7], m[2] * m[7] - m[1] * m[8], m[1] * m[5] - m[2] * m[4],
                         m[5] * m[6] - m[3] * m[8], m[0] * m[8] - m[2] * m[6], m[2] * m[3] - m[0] * m[5],
                         m[3] * m[7] - m[4] * m[6], m[1] * m[6] - m[0] * m[7], m[0] * m[4] - m[1] * m[3]};
    for (int k = 0; k < 9; ++k) sg.inv[k] = det != 0.0 ? c[k] / det : 0.0;
    for (int a = 0; a < 3; ++a) sg.pbc[a] = sys.pbc[a] && det != 0.0 ? 1 : 0;
  }
  bool keep = vl_valid_ && vl_n_ == n && vl_periodic_ == periodic &&
              (!periodic || (std::memcmp(vl_cell_, sys.cell, sizeof(vl_cell_)) == 0 &&
                             vl_pbc_[0] == sys.pbc[0] && vl_pbc_[1] == sys.pbc[1] && vl_pbc_[2] == sys.pbc[2]));
  if (keep) {
    unsigned *dmax = static_cast<unsigned *>(vl_max_.ensure(sizeof(unsigned)));
    CUDA_CHECK(cudaMemsetAsync(dmax, 0, sizeof(unsigned), s));
    skin_displacement(d_pos, vl_ref_.as<float>(), n, sg, vl_img_.as<int>(), dmax, s);
    unsigned bits = 0;
    CUDA_CHECK(cudaMemcpyAsync(&bits, dmax, sizeof(bits), cudaMemcpyDeviceToHost, s));
    CUDA_CHECK(cudaStreamSynchronize(s));
    float m2;
    std::memcpy(&m2, &bits, sizeof(m2));
    const float half = 0.5f * skin_;
    keep = m2 <= half * half;
  }
  if (keep) {
    refresh_edges(d_pos, nl_.n_edges, nl_.center.as<int>(), nl_.nbr.as<int>(), nl_.shift.as<int>(),
                  vl_img_.as<int>(), sg, nl_.vec.as<float>(), nl_.dist.as<float>(), s);
    return true;
  }
  const float rc = h_.cutoff + skin_;
  if (periodic) {
    GridParams g;
    make_grid_params(sys.cell, sys.pbc, rc, &g);
    build_periodic_nl(d_pos, n, g, nl_, nls_, s);
  } else {
    std::vector<int> b(n, 0), e(n, n);
    int *db = static_cast<int *>(d_sys_begin_.ensure(sizeof(int) * (n + 1)));
    int *de = static_cast<int *>(d_sys_end_.ensure(sizeof(int) * (n + 1)));
    CUDA_CHECK(cudaMemcpyAsync(db, b.data(), sizeof(int) * n, cudaMemcpyHostToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(de, e.data(), sizeof(int) * n, cudaMemcpyHostToDevice, s));
    build_open_nl(d_pos, db, de, n, rc, nl_, nls_, s);
  }
  CUDA_CHECK(cudaMemcpyAsync(vl_ref_.ensure(sizeof(float) * 3 * n), d_pos, sizeof(float) * 3 * n,
                             cudaMemcpyDeviceToDevice, s));
  vl_img_.ensure(sizeof(int) * 3 * n);
  vl_valid_ = true;
  vl_n_ = n;
  vl_periodic_ = periodic;
  if (periodic) {
    std::memcpy(vl_cell_, sys.cell, sizeof(vl_cell_));
    for (int a = 0; a < 3; ++a) vl_pbc_[a] = sys.pbc[a];
  }
  ++nl_builds_;
  return false;
}

const EdgeList &PETModel::domain_neighbors(const double *d_pos, int n_local, int n_own, const GridParams &g) {
  if (wptr_.empty()) throw Error(3, "Model weights not loaded");
  CUDA_CHECK(cudaSetDevice(device_));
  vl_valid_ = false;
  ++nl_builds_;
  int *derr = static_cast<int *>(d_err_.ensure(sizeof(int) * 4));
  CUDA_CHECK(cudaMemsetAsync(derr, 0, sizeof(int), stream_));
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[0], stream_));
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[1], stream_));
  build_local_nl(d_pos, n_local, n_own, g, nl_, nls_, stream_);
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[2], stream_));
  return nl_;
}

void PETModel::domain_predict(const int *d_species, int n_local, int n_own, RemoteMessages *rm, bool grad,
                              double *d_red) {
  cudaStream_t s = stream_;
  ncf_ = ncs_ = false;
  rm_ = rm;
  try {
    setup_graph(n_local, n_own, nl_.n_edges, n_own, nl_.n_edges, d_species, grad, rm ? rm->n_in : 0);
    if (timing_) CUDA_CHECK(cudaEventRecord(ev_[3], s));
    forward_backward(grad);
  } catch (...) {
    rm_ = nullptr;
    throw;
  }
  rm_ = nullptr;
  double *red = static_cast<double *>(d_red_.ensure(sizeof(double) * (16 + 7 * kReduceMaxParts)));
  reduce_local(nl_.vec.as<float>(), in_->a.g, in_->a.e_atom, n_own, grad ? El_[0] : 0, red, red + 16, s);
  CUDA_CHECK(cudaMemcpyAsync(d_red, red, sizeof(double) * 7, cudaMemcpyDeviceToDevice, s));
  if (timing_) {
    CUDA_CHECK(cudaEventRecord(ev_[6], s));
    CUDA_CHECK(cudaEventRecord(ev_[7], s));
  }
}

void PETModel::check_device_error(bool grad) {
  int herr = 0;
  CUDA_CHECK(cudaMemcpy(&herr, d_err_.ptr, sizeof(int), cudaMemcpyDeviceToHost));
  if (kprof_) collect_marks();
  if (herr != 0)
    throw Error(kErrComputation, "a tensor-core pipeline wait timed out (device error " + std::to_string(herr) + ")");
  if (timing_) read_times(grad);
}

void PETModel::read_times(bool grad) {
  float ms;
  CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[0], ev_[1])); times_.h2d = ms;
  CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[1], ev_[2])); times_.nl = ms;
  CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[2], ev_[3])); times_.prep = ms;
  CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[3], ev_[4])); times_.forward = ms;
  times_.backward = 0.f;
  if (grad) { CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[4], ev_[5])); times_.backward = ms; }
  CUDA_CHECK(cudaEventElapsedTime(&ms, grad ? ev_[5] : ev_[4], ev_[6])); times_.reduce = ms;
  CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[6], ev_[7])); times_.d2h = ms;
  CUDA_CHECK(cudaEventElapsedTime(&ms, ev_[0], ev_[7])); times_.total = ms;
}

void PETModel::run_group(const float *d_pos, int n_atoms, const std::vector<const SystemView *> &systems,
                         const std::vector<int> &atom_begin, bool grad, std::vector<Result *> &results,
                         bool copy_forces, bool nc) {
  cudaStream_t s = stream_;
  const int n_sys = static_cast<int>(systems.size());
  n_sys_ = n_sys;
  // pet.cpp:281-282: a property's heads run when asked for and present
  ncf_ = nc && has_ncf_;
  ncs_ = nc && has_ncs_;
  int *derr = static_cast<int *>(d_err_.ensure(sizeof(int) * 4));
  CUDA_CHECK(cudaMemsetAsync(derr, 0, sizeof(int), s));
  // species indices (pet_batch.cpp:146-167): unknown Z is an error
  int *hsp = static_cast<int *>(h_species_.ensure(sizeof(int) * (n_atoms + 1) + sizeof(int) * (n_sys + 1)));
  for (int k = 0; k < n_sys; ++k) {
    const SystemView &sv = *systems[k];
    for (int i = 0; i < sv.n_atoms; ++i) {
      const int si = species_of(sv.numbers[i]);
      if (si < 0)
        throw Error(kErrComputation, "Unknown atomic number " + std::to_string(sv.numbers[i]) +
                                         " not found in species_to_index mapping");
      hsp[atom_begin[k] + i] = si;
    }
  }
  int *hsb = hsp + n_atoms + 1;
  for (int k = 0; k <= n_sys; ++k) hsb[k] = atom_begin[k];
  int *dsp = static_cast<int *>(d_species_.ensure(sizeof(int) * (n_atoms + 1)));
  int *dsb = static_cast<int *>(d_sys_atoms_.ensure(sizeof(int) * (n_sys + 1)));
  CUDA_CHECK(cudaMemcpyAsync(dsp, hsp, sizeof(int) * n_atoms, cudaMemcpyHostToDevice, s));
  CUDA_CHECK(cudaMemcpyAsync(dsb, hsb, sizeof(int) * (n_sys + 1), cudaMemcpyHostToDevice, s));
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[1], s));

  // neighbour list
  const bool periodic = systems[0]->cell != nullptr;
  if (n_sys == 1 && skin_ > 0.f) {
    skin_list(d_pos, n_atoms, *systems[0], s);
  } else if (periodic) {
    if (n_sys != 1) throw Error(kErrInternal, "periodic systems run one per group");
    vl_valid_ = false;
    ++nl_builds_;
    GridParams g;
    make_grid_params(systems[0]->cell, systems[0]->pbc, h_.cutoff, &g);
    build_periodic_nl(d_pos, n_atoms, g, nl_, nls_, s);
  } else {
    vl_valid_ = false;
    ++nl_builds_;
    std::vector<int> b(n_atoms), e(n_atoms);
    for (int k = 0; k < n_sys; ++k)
      for (int i = atom_begin[k]; i < atom_begin[k + 1]; ++i) {
        b[i] = atom_begin[k];
        e[i] = atom_begin[k + 1];
      }
    int *db = static_cast<int *>(d_sys_begin_.ensure(sizeof(int) * (n_atoms + 1)));
    int *de = static_cast<int *>(d_sys_end_.ensure(sizeof(int) * (n_atoms + 1)));
    CUDA_CHECK(cudaMemcpyAsync(db, b.data(), sizeof(int) * n_atoms, cudaMemcpyHostToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(de, e.data(), sizeof(int) * n_atoms, cudaMemcpyHostToDevice, s));
    build_open_nl(d_pos, db, de, n_atoms, h_.cutoff, nl_, nls_, s);
  }
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[2], s));
  setup_graph(n_atoms, n_atoms, nl_.n_edges, n_atoms, nl_.n_edges, dsp, grad);
  const Acts &a = in_->a;
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[3], s));

  run_forward_backward(grad);

  // per-system energy and virial in f64 (pet.cpp:542-548, 1041-1077); then
  // the per-system Voigt sums of the non-conservative stress
  const size_t nred = static_cast<size_t>(ncs_ ? 13 : 7) * n_sys;
  double *red = static_cast<double *>(d_red_.ensure(sizeof(double) * (nred + 8 + 7 * kReduceMaxParts)));
  reduce_systems(nl_.vec.as<float>(), a.g, a.e_atom, nl_.offset.as<int>(), dsb, n_sys, red + n_sys, red,
                 grad && El_[0] > 0, s, n_atoms, El_[0], red + nred + 8);
  if (ncs_) nc_stress_reduce(a.ncS, dsb, n_sys, red + 7 * n_sys, s);
  // pet.cpp:601-617: non-conservative forces added to the gradient forces
  if (ncf_) add_vec(a.ncF, a.F, 3 * n_atoms, grad, s);
  const bool have_forces = grad || ncf_;
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[6], s));
  const size_t fbytes = (have_forces && copy_forces) ? sizeof(float) * 3 * n_atoms : 0;
  char *hout = static_cast<char *>(h_out_.ensure(sizeof(double) * nred + fbytes + 16));
  int *herr = reinterpret_cast<int *>(hout + sizeof(double) * nred + fbytes);
  CUDA_CHECK(cudaMemcpyAsync(herr, d_err_.ptr, sizeof(int), cudaMemcpyDeviceToHost, s));
  CUDA_CHECK(cudaMemcpyAsync(hout, red, sizeof(double) * nred, cudaMemcpyDeviceToHost, s));
  if (fbytes)
    CUDA_CHECK(cudaMemcpyAsync(hout + sizeof(double) * nred, a.F, fbytes, cudaMemcpyDeviceToHost, s));
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[7], s));
  CUDA_CHECK(cudaStreamSynchronize(s));
  if (kprof_) collect_marks();
  if (*herr != 0)
    throw Error(kErrComputation, "a tensor-core pipeline wait timed out (device error " +
                                     std::to_string(*herr) + ")");

  const double *he = reinterpret_cast<const double *>(hout);
  const double *hv = he + n_sys;
  const double *hs = he + 7 * n_sys;
  const float *hF = reinterpret_cast<const float *>(hout + sizeof(double) * nred);
  for (int k = 0; k < n_sys; ++k) {
    const SystemView &sv = *systems[k];
    Result &R = *results[k];
    double tot = he[k];
    for (int i = 0; i < sv.n_atoms; ++i) tot += composition_energy(sv.numbers[i]);
    R.energy = static_cast<float>(tot);
    R.has_forces = false;
    R.has_stress = false;
    R.forces.clear();
    R.stress.clear();
    if (have_forces) {
      R.has_forces = true;
      if (copy_forces) R.forces.assign(hF + 3 * atom_begin[k], hF + 3 * atom_begin[k + 1]);
    }
    // pet.cpp:1079-1097: f32 determinant, stress only when |V| > 1e-10
    const float *m = sv.cell;
    const bool periodic = m && (sv.pbc[0] || sv.pbc[1] || sv.pbc[2]);
    float vol = 0.f;
    if (periodic)
      vol = std::fabs(m[0] * (m[4] * m[8] - m[5] * m[7]) - m[1] * (m[3] * m[8] - m[5] * m[6]) +
                      m[2] * (m[3] * m[7] - m[4] * m[6]));
    if (grad) {
      R.stress.assign(6, 0.0f);
      if (periodic && vol > 1e-10f) {
        for (int c = 0; c < 6; ++c) R.stress[c] = static_cast<float>(hv[6 * k + c]) / vol;
        R.has_stress = true;
      }
    }
    if (ncs_) {
      // pet.cpp:627-686: the per-atom tensors' Voigt sum is added to the
      // stress already there and the sum divided by the volume, as the
      // reference does (with gradients on as well, that divides the
      // gradient stress a second time; the mlipcpp API never asks for both)
      if (R.stress.empty()) R.stress.assign(6, 0.0f);
      for (int c = 0; c < 6; ++c) R.stress[c] += static_cast<float>(hs[6 * k + c]);
      if (periodic && vol > 1e-10f) {
        for (int c = 0; c < 6; ++c) R.stress[c] /= vol;
        R.has_stress = true;
      }
    }
  }
  if (timing_) read_times(grad);
}

std::vector<Result> PETModel::predict(const std::vector<SystemView> &systems, bool grad, bool nc) {
  std::vector<Result> out(systems.size());
  if (systems.empty()) return out;
  if (wptr_.empty()) throw Error(3, "Model weights not loaded");
  CUDA_CHECK(cudaSetDevice(device_));
  auto run = [&](const std::vector<int> &idx) {
    std::vector<const SystemView *> sv;
    std::vector<Result *> rs;
    std::vector<int> begin{0};
    for (int k : idx) {
      sv.push_back(&systems[k]);
      rs.push_back(&out[k]);
      begin.push_back(begin.back() + systems[k].n_atoms);
    }
    const int n = begin.back();
    float *hp = static_cast<float *>(h_pos_.ensure(sizeof(float) * 3 * (n + 1)));
    for (size_t k = 0; k < sv.size(); ++k)
      std::memcpy(hp + 3 * begin[k], sv[k]->positions, sizeof(float) * 3 * sv[k]->n_atoms);
    float *dp = static_cast<float *>(d_pos_.ensure(sizeof(float) * 3 * (n + 1)));
    if (timing_) CUDA_CHECK(cudaEventRecord(ev_[0], stream_));
    CUDA_CHECK(cudaMemcpyAsync(dp, hp, sizeof(float) * 3 * n, cudaMemcpyHostToDevice, stream_));
    run_group(dp, n, sv, begin, grad, rs, true, nc);
  };
  std::vector<int> open;
  for (size_t k = 0; k < systems.size(); ++k) {
    if (systems[k].n_atoms <= 0) continue;
    if (systems[k].cell) run({static_cast<int>(k)});
    else open.push_back(static_cast<int>(k));
  }
  if (!open.empty()) run(open);
  return out;
}

void PETModel::predict_device(const float *d_pos, const SystemView &sys, bool grad, Result &out,
                              bool copy_forces, bool nc) {
  if (wptr_.empty()) throw Error(3, "Model weights not loaded");
  std::vector<const SystemView *> sv{&sys};
  std::vector<Result *> rs{&out};
  std::vector<int> begin{0, sys.n_atoms};
  if (timing_) CUDA_CHECK(cudaEventRecord(ev_[0], stream_));
  run_group(d_pos, sys.n_atoms, sv, begin, grad, rs, copy_forces, nc);
}

}  // namespace pet
