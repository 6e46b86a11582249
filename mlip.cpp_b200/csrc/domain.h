// Spatial domain decomposition of one periodic cell over several ranks (one
// GPU each), with halo exchanges over the caller's collectives.  The
// reference evaluates a structure on one device (PETModel::predict_batch,
// src/models/pet/pet.cpp:125-694); this splits that evaluation so that every
// rank runs both GNN layers on its owned atoms only.
//
// Per step, on the model's stream:
//   1. halo: each rank sends the positions of its owned atoms that lie within
//      cutoff (+ skin) of another rank's slab (periodic images included) to
//      that rank; the received atoms are the ghosts of the local system;
//   2. the neighbour list of the owned atoms over owned + ghost atoms;
//   3. requests: a layer-1 message of edge i -> j reads the layer-0 token of
//      the reverse edge j -> i (pet_layers.cpp:608-679); for a ghost j that
//      edge belongs to j's owner, which receives a request (j, i, image
//      shift) and resolves it to one of its edges;
//   4. the model, with two exchanges inside it: the owners send the
//      requested layer-0 tokens (d floats each) after layer 0, and the
//      requesters send the gradients of those tokens back after the layer-1
//      backward;
//   5. forces computed on ghost atoms go back to their owners and are added
//      there (the reverse halo);
//   6. one sum over ranks of (energy, virial, composition energy).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "model.h"
#include "neighbor.cuh"

namespace pet {

// Collectives among the ranks that share one cell, supplied by the caller
// (torch.distributed over NCCL, or an in-process emulation).  All buffers
// are device memory on the model's device.  alltoallv: rank r's segment of
// d_send (send_counts[r] elements of elem_bytes bytes, segments in rank
// order) arrives in rank r's d_recv in this rank's segment (recv_counts
// elements per source rank, in rank order).  allreduce_sum_f64: in-place
// sum of n doubles over the ranks.  Both must be ordered on `stream` (the
// send data is what the stream's earlier work produced; later work on the
// stream sees the received data) and return 0 on success.
struct DomainComm {
  void *user = nullptr;
  int32_t (*alltoallv)(void *user, const void *d_send, const int64_t *send_counts, void *d_recv,
                       const int64_t *recv_counts, int64_t elem_bytes, void *stream) = nullptr;
  int32_t (*allreduce_sum_f64)(void *user, double *d_buf, int64_t n, void *stream) = nullptr;
};

// Per-phase device times of the last step (CUDA events on the model's
// stream, milliseconds): halo, neighbour list + requests, model (with its
// two token exchanges), reverse halo of forces, sum over ranks; the whole
// step; and the host wall-clock of the call.  Counts of the last step.
struct DomainStats {
  double ms[7] = {};
  int64_t n_own = 0, n_ghost = 0, n_edges = 0, n_req_out = 0, n_req_in = 0, n_sent = 0;
};

class DomainEngine : public RemoteMessages {
 public:
  // cell: row-major lattice vectors of the whole cell (periodic along all
  // three axes); grid: slabs per axis (their product is the number of
  // ranks); rank: this rank, at slab (rank % g0, rank / g0 % g1,
  // rank / (g0 g1)); skin: extra width of the halo beyond the cutoff, for
  // owned atoms that have moved since the ownership was assigned.
  DomainEngine(PETModel &model, const float cell[9], const int grid[3], int rank, float skin,
               const DomainComm &comm);
  ~DomainEngine() override;
  DomainEngine(const DomainEngine &) = delete;
  DomainEngine &operator=(const DomainEngine &) = delete;

  // The owned atoms' atomic numbers (host); their positions come with each
  // step in the same order.  Throws Error(kErrComputation) for a Z the model
  // does not know.
  void set_atoms(int n_own, const int32_t *numbers);
  // One energy + forces + virial evaluation.  d_pos: the owned atoms'
  // positions (device, [3 n_own] f32); d_forces: their forces (device, may
  // be null); energy and virial (Voigt, not divided by the volume) are sums
  // over all ranks.  Collective: every rank calls it once per step.
  void step(const float *d_pos, float *d_forces, bool grad, double *energy, double virial[6]);
  const DomainStats &stats() const { return stats_; }

  void exchange_tokens(float *x0, int N0, int T0, int d, cudaStream_t s) override;
  void exchange_token_grads(const float *dmsg, float *dx, int N0, int d, cudaStream_t s) override;

  // Geometry shared with the kernels.
  struct Geom {
    double cell[9], inv[9];
    double d1[3];      // halo width per axis in fractional units (0 along unsplit axes)
    double origin[3];  // this rank's local frame origin (fractional)
    int p[3];
    int world, rank;
  };

 private:
  std::vector<int64_t> exchange_counts(const int64_t *d_send_counts, int64_t *d_recv_counts);
  void alltoallv(const void *send, const std::vector<int64_t> &sc, void *recv, const std::vector<int64_t> &rc,
                 size_t elem_bytes, cudaStream_t s);

  PETModel &model_;
  DomainComm comm_;
  Geom g_{};
  GridParams grid_{};  // neighbour search of the local frame
  int n_own_ = 0, n_ghost_ = 0, n_req_out_ = 0, n_req_in_ = 0, n_sent_ = 0;
  double comp_ = 0.0;  // composition energy of the owned atoms
  std::vector<int64_t> halo_sc_, halo_rc_, req_sc_, req_rc_;
  DevBuf species_own_, z_own_, cnt_, off_, wrap_, send_rec_, recv_rec_, sbase_, counts_;
  DevBuf pos_local_, species_local_, ghost_rank_, ghost_src_, ghost_img_;
  DevBuf req_cnt_, req_base_, req_send_, req_recv_, req_edge_, msg_row_buf_, reply_edge_;
  DevBuf tok_send_, grad_send_, grad_recv_, force_recv_, red_, flag_;
  HostBuf h_;
  cudaEvent_t ev_[6] = {};
  DomainStats stats_;
};

}  // namespace pet
