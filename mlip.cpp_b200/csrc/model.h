// PET energy / force / stress model on one B200: the replacement for
// mlip.cpp's PETModel (src/models/pet/pet.{h,cpp}) behind the mlipcpp C API.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "neighbor.cuh"

namespace pet {

struct Hypers {
  int d = 256, heads = 8, ff = 512, dh = 128, hid = 256;  // hid: compress hidden width
  int gnn_layers = 2, attn_layers = 2, n_species = 0;
  // columns of the featurised rows' auxiliary block (x, y, z, r, 1 and one
  // per embedding row, rounded up to 128): see FeaturizeArgs
  int aux = 128;
  float cutoff = 4.5f, width = 0.5f;
};

// One structure as the C API receives it (host pointers, not owned).
struct SystemView {
  int n_atoms = 0;
  const float *positions = nullptr;    // [n, 3]
  const int32_t *numbers = nullptr;    // [n]
  const float *cell = nullptr;         // [9] row-major or null
  bool pbc[3] = {true, true, true};
};

struct Result {
  float energy = 0.0f;
  std::vector<float> forces;  // [n, 3]
  std::vector<float> stress;  // [6] Voigt xx yy zz yz xz xy
  bool has_forces = false;
  bool has_stress = false;
};

// Kernel classes timed individually when kernel profiling is on.
enum KernelClass {
  KC_GEMM_TC = 0,    // 3xTF32 tensor-core GEMM
  KC_GEMM_SIMT = 1,  // fp32 SIMT GEMM
  KC_ATTENTION = 2,
  KC_NEIGHBOR = 3,
  KC_OTHER = 4,
  KC_GEMM_F16 = 5,   // 3xFP16 tensor-core GEMM (with its row-scale pre-pass)
  KC_COUNT = 6
};

struct KernelStat {
  long long launches = 0;
  double ms = 0.0, flops = 0.0, bytes = 0.0;
};

// Per-phase CUDA-event timings of the last predict (milliseconds).
struct PhaseTimes {
  float h2d = 0, nl = 0, prep = 0, forward = 0, backward = 0, reduce = 0, d2h = 0, total = 0;
};

// Layer-1 messages of a spatial domain whose reverse edges live on other
// ranks (implemented by DomainEngine, domain.cu).  The message of a layer-1
// edge i -> j reads the layer-0 token of j -> i (pet_layers.cpp:608-679);
// when j is a ghost that token is computed by j's owner.  Both calls are
// collective over the ranks and made exactly once per prediction.
struct RemoteMessages {
  virtual ~RemoteMessages() = default;
  int n_in = 0;                  // remote tokens received after the T0 layer-0 rows
  const int *msg_row = nullptr;  // [E1]: x_prev row of each edge's message, -1: its local reverse
  // After the layer-0 forward: x0 = the T0 layer-0 token rows (d floats
  // each, node rows then edge rows from N0); fill x0 rows [T0, T0 + n_in).
  virtual void exchange_tokens(float *x0, int N0, int T0, int d, cudaStream_t s) = 0;
  // After the layer-1 compression backward: dmsg [E1][d] holds the message
  // gradients; add the gradients other ranks' messages send back into the
  // layer-0 token gradient rows dx (edge rows from N0).
  virtual void exchange_token_grads(const float *dmsg, float *dx, int N0, int d, cudaStream_t s) = 0;
};

class PETModel {
 public:
  PETModel();
  ~PETModel();
  PETModel(const PETModel &) = delete;
  PETModel &operator=(const PETModel &) = delete;

  // PETModel::load_from_gguf (pet.cpp:1100-1312)
  void load(const std::string &path, float cutoff_override = 0.0f);
  float cutoff() const { return h_.cutoff; }
  const Hypers &hypers() const { return h_; }

  // predict_batch (pet.cpp:125-694).  With compute_grad the result carries
  // forces, and stress for periodic systems.  With nc the non-conservative
  // heads the model has run in the forward pass (pet.cpp:742-784): their
  // per-atom forces are added to the result's forces and their per-atom
  // stress, summed per system, to its stress (pet.cpp:576-686).
  std::vector<Result> predict(const std::vector<SystemView> &systems, bool compute_grad, bool nc = false);
  // The model carries non-conservative force / stress heads (layer 0 present,
  // PETWeights::has_force_heads / has_stress_heads, pet_types.h:247-254).
  bool has_nc_forces() const { return has_ncf_; }
  bool has_nc_stress() const { return has_ncs_; }

  // A spatial domain whose layer-0 messages cross to other ranks
  // (DomainEngine).  domain_neighbors: the neighbour list of the local
  // system (n_own owned atoms, then ghosts; f64 device positions; only the
  // owned atoms are centres).  domain_predict: both layers and the readout
  // on the owned atoms with `rm` supplying the remote messages; gradient
  // forces on all n_local atoms (device_forces), and the owned energy and
  // the local virial into d_red[0..6] (device f64).  Synchronises nothing:
  // the caller reads d_red after a stream synchronisation and then calls
  // check_device_error.
  const EdgeList &domain_neighbors(const double *d_pos, int n_local, int n_own, const GridParams &g);
  void domain_predict(const int *d_species, int n_local, int n_own, RemoteMessages *rm, bool grad, double *d_red);
  void check_device_error(bool grad);
  int device() const { return device_; }
  // species index of every atomic number 0..127 (-1: not in the model), device
  const int *device_species_map();
  double composition_energy(int z) const {
    if (z >= 0 && z < kZTable) return zcomp_[z];
    auto it = composition_.find(z);
    return it == composition_.end() ? 0.0 : it->second;
  }
  // species index of atomic number z, -1 when the model does not know it
  int species_of(int z) const {
    if (z >= 0 && z < kZTable) return zidx_[z];
    auto it = species_index_.find(z);
    return it == species_index_.end() ? -1 : it->second;
  }
  bool knows_species(int z) const { return species_of(z) >= 0; }

  // Device-resident entry for benchmarks: positions already on the device.
  void predict_device(const float *d_pos, const SystemView &sys, bool compute_grad, Result &out,
                      bool copy_forces, bool nc = false);

  // Forces [n, 3] of the last prediction in device memory (valid until the
  // next call on this model).
  const float *device_forces() const;
  const PhaseTimes &last_times() const { return times_; }
  // Per-launch CUDA events around GEMM and attention launches, accumulated
  // into kernel_stats() after each predict (cumulative until reset).
  void set_kernel_profiling(bool on) { kprof_ = on; }
  const KernelStat *kernel_stats() const { return kstats_; }
  void reset_kernel_stats() { for (auto &k : kstats_) k = KernelStat{}; }
  int last_atoms() const { return n_local_; }
  int last_edges() const { return El_[0]; }
  int last_max_neighbors() const { return max_tok_ - 1; }
  void set_timing(bool on) { timing_ = on; }
  // Verlet list for single-structure predictions: with skin > 0 the list is
  // built with cutoff + skin and kept across calls (vectors and distances
  // refreshed from the new positions) until an atom has moved more than
  // skin / 2 since the build, the atom count, cell or pbc change, or another
  // call rebuilds the list.  Pairs beyond the cutoff get f_c = 0 and a -inf
  // key mask, the reference's padding, so results are unchanged.  0: a new
  // list every call (the default).
  void set_neighbor_skin(float skin) {
    skin_ = skin;
    vl_valid_ = false;
  }
  float neighbor_skin() const { return skin_; }
  // neighbour lists built by this model so far (kept lists not counted again)
  long long neighbor_builds() const { return nl_builds_; }
  cudaStream_t stream() const { return stream_; }
  size_t device_bytes() const;

 private:
  struct Group;  // systems that share one neighbour-list launch
  void run_group(const float *d_pos, int n_atoms, const std::vector<const SystemView *> &systems,
                 const std::vector<int> &atom_begin, bool compute_grad,
                 std::vector<Result *> &results, bool copy_forces, bool nc);
  void forward_backward(bool compute_grad);
  // forward_backward through a CUDA graph when the same shapes and buffers
  // come back (see model.cu)
  void run_forward_backward(bool compute_grad);
  std::vector<uintptr_t> graph_key(bool compute_grad) const;
  void record_phase(int i);
  void setup_graph(int n_local, int N0, int E0, int N1, int E1, const int *d_species, bool grad, int n_in = 0);
  void read_times(bool grad);
  const float *w(const std::string &name) const;
  // neighbour list of a single structure through the kept Verlet list
  // (builds it when it cannot be kept); true when the list was kept
  bool skin_list(const float *d_pos, int n_atoms, const SystemView &sys, cudaStream_t s);

  struct Internals;  // device pointers of weights and activations (model.cu)
  std::unique_ptr<Internals> in_;
  Hypers h_;
  cudaStream_t stream_ = nullptr;
  int device_ = 0;
  DevBuf wbuf_;          // [fp32 | tf32 hi | lo] copies of every weight
  size_t wspan_ = 0;     // floats between the three copies
  bool use_tc_ = true;   // tensor-core GEMMs (MLIPCPP_B200_GEMM=simt disables)
  bool use_f16_ = true;  // 3xFP16 where it applies (MLIPCPP_B200_GEMM=tf32 keeps 3xTF32)
  // attention kernels: forward and backward on the tensor-core kernels of
  // attention_mma.cu where they apply (head size 32, up to 64 tokens), else
  // on the SIMT kernels; MLIPCPP_B200_ATTN=rows (or simt): SIMT for both
  bool use_attn_rows_ = false;
  // MLIPCPP_PRECISION_F16: dense layers with the hi x hi product only
  bool reduced_ = false;
  // non-conservative heads in the file / run in the current prediction
  bool has_ncf_ = false, has_ncs_ = false;
  bool ncf_ = false, ncs_ = false;

 public:
  void set_reduced_precision(bool on) { reduced_ = on; }
  bool reduced_precision() const { return reduced_; }

 private:
  // fp16 hi / lo copies after the three fp32 copies, same element offsets;
  // one power-of-two scale per tensor: {first element, end element, scale}
  struct WScale { size_t begin, end; int scale; };
  std::vector<WScale> wscale_;
  // Split-fp16 buffers.  sp_[0]: the A operand a 3xFP16 GEMM converts from
  // fp32.  In chain mode (every dense layer on 3xFP16) the kernels that
  // produce a GEMM's A operand write it in split form, alternating between
  // sp_[0] and sp_[1]; each is consumed by the next GEMM.
  // sp_[2] (chain mode): the split gradient of a layer's first block input,
  // whose edge rows the compression backward reads
  DevBuf sp_[3];
  bool chain_ok_ = false;  // the model's shapes allow chain mode (set at load)
  bool chain_ = false;     // chain mode for the current prediction
  Split16View split_view(int i, int rows, int cols);
  int weight_scale(size_t elem) const;
  DevBuf d_err_;         // device error word written by bounded waits
  std::map<std::string, const float *> wptr_;
  std::map<int, int> species_index_;
  std::map<int, float> composition_;
  // the same for Z < kZTable as flat tables (per-atom lookups on the host)
  static constexpr int kZTable = 128;
  int zidx_[kZTable];
  float zcomp_[kZTable];

  // per-call device state
  DevBuf d_pos_, d_species_, d_sys_begin_, d_sys_end_, d_sys_atoms_, d_zmap_;
  RemoteMessages *rm_ = nullptr;  // set during domain_predict
  // CUDA graph of forward_backward (MLIPCPP_B200_GRAPH=0 disables): the key
  // of the last prediction, the key and executable of the captured graph,
  // and the kernels it launches (added to the launch counter on replay)
  bool use_graph_ = true;
  std::vector<uintptr_t> last_key_, gkey_;
  cudaGraphExec_t gexec_ = nullptr;
  long long graph_kernels_ = 0;
  bool capturing_ = false;
  // Verlet list state (set_neighbor_skin): positions at the build, per-atom
  // image offsets, the device maximum of the displacements, and the
  // geometry the list was built for
  float skin_ = 0.f;
  bool vl_valid_ = false;
  int vl_n_ = 0;
  bool vl_periodic_ = false;
  float vl_cell_[9] = {};
  bool vl_pbc_[3] = {};
  DevBuf vl_ref_, vl_img_, vl_max_;
  long long nl_builds_ = 0;
  // attention atom classes of the current prediction (short_atoms, then
  // long_atoms, then two counts); both sizes 0 when one class holds all
  DevBuf attn_cls_;
  int n_short_ = 0, n_long_ = 0;
  const int *species_ = nullptr;  // species index of every local atom (device), set by setup_graph
  EdgeList nl_;
  NLScratch nls_;
  DevBuf persist_, scratch_;
  DevBuf d_red_;  // per-system energy (f64) + virial (f64 x 6)
  HostBuf h_pos_, h_species_, h_out_;
  int n_local_ = 0, Nl_[2] = {0, 0}, El_[2] = {0, 0}, Tl_[2] = {0, 0}, max_tok_ = 0, n_sys_ = 0;
  bool timing_ = false;
  bool kprof_ = false;
  KernelStat kstats_[KC_COUNT];
  struct Mark { int cls; cudaEvent_t a, b; double flops, bytes; };
  std::vector<Mark> marks_;
  std::vector<cudaEvent_t> ev_pool_;
  size_t ev_used_ = 0;
  void mark_begin(cudaEvent_t &a);
  void mark_end(int cls, cudaEvent_t a, double flops, double bytes);
  void collect_marks();
  PhaseTimes times_;
  cudaEvent_t ev_[8] = {};
};

}  // namespace pet
