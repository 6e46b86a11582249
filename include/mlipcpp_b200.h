/*
 * Extensions of the mlipcpp C API provided by the B200 backend.
 *
 * The reference exposes batched prediction only through C++
 * (PETModel::predict_batch, src/models/pet/pet.h:140-143); it is made
 * available to C callers here.  The remaining entry points serve
 * benchmarking and MD drivers that keep positions on the GPU.
 */
#ifndef MLIPCPP_B200_H
#define MLIPCPP_B200_H

#include "mlipcpp.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Predict a batch of independent structures in one call
 * (PETModel::predict_batch, src/models/pet/pet.cpp:125-694).  Non-periodic
 * structures are evaluated together; periodic ones one after another.
 * results[k] receives a handle that owns its data (valid until freed with
 * mlipcpp_result_free). */
mlipcpp_error_t mlipcpp_predict_batch(mlipcpp_model_t model, int32_t n_systems,
                                      const mlipcpp_system_t *systems,
                                      const mlipcpp_predict_options_t *options,
                                      mlipcpp_result_t *results);

/* The same batch from packed arrays, with the results written straight into
 * the caller's arrays (no result handles), for callers that hold many
 * structures as one block (data loaders, screening loops).  Structure k has
 * n_atoms[k] > 0 atoms; its positions ([3 n_atoms[k]] float) and atomic
 * numbers follow those of structure k - 1 in `positions` and `numbers`.
 * cells: [9 n_systems] row-major lattices, or NULL when every structure is
 * non-periodic; pbc: [3 n_systems], or NULL for periodic along all axes when
 * cells are given.  Out: energies [n_systems]; forces [3 sum n_atoms] (NULL:
 * not copied out); stress [6 n_systems], Voigt (NULL: not copied out).
 * Outputs the options do not ask for, and stress of a non-periodic
 * structure, are written as zeros. */
mlipcpp_error_t mlipcpp_b200_predict_packed(mlipcpp_model_t model, int32_t n_systems, const int32_t *n_atoms,
                                            const float *positions, const int32_t *numbers, const float *cells,
                                            const bool *pbc, const mlipcpp_predict_options_t *options,
                                            float *energies, float *forces, float *stress);

/* Predict one structure whose positions are already in device memory
 * (d_positions: device pointer to [3n] float).  atomic_numbers, cell and pbc
 * are host pointers.  Forces are copied back only when copy_forces is true.
 * Same result-handle semantics as mlipcpp_predict. */
mlipcpp_error_t mlipcpp_b200_predict_device(mlipcpp_model_t model, int32_t n_atoms,
                                            const float *d_positions,
                                            const int32_t *atomic_numbers, const float *cell,
                                            const bool *pbc,
                                            const mlipcpp_predict_options_t *options,
                                            bool copy_forces, mlipcpp_result_t *result);

/* No counterpart in the reference (its Python MD loop copies positions and
 * forces through the host each step, python/mlipcpp/ase.py:123-183).  As
 * mlipcpp_b200_predict_device, but the forces stay on the device: they are
 * written to d_forces (device, [3n] float, may be NULL) and the energy
 * (eV, composition included) to *energy; stress (host [6], Voigt, may be
 * NULL) and *has_stress (may be NULL) as in the result of
 * mlipcpp_predict_with_options.  Forces asked for from a model that cannot
 * give them (use_nc_forces without force heads, compute_forces off) return
 * MLIPCPP_ERROR_INVALID_PARAMETER when d_forces is set.  For MD drivers that
 * keep positions, velocities and forces on the GPU. */
mlipcpp_error_t mlipcpp_b200_predict_device_forces(mlipcpp_model_t model, int32_t n_atoms,
                                                   const float *d_positions, const int32_t *atomic_numbers,
                                                   const float *cell, const bool *pbc,
                                                   const mlipcpp_predict_options_t *options, float *d_forces,
                                                   double *energy, float stress[6], bool *has_stress);

/* Verlet neighbour list for repeated single-structure predictions (MD):
 * the reference builds a new list every call (PETModel::predict_batch,
 * src/models/pet/pet.cpp:125-694).  With skin > 0 (Angstrom) the list is
 * built with cutoff + skin and kept across calls, its vectors and distances
 * recomputed from the new positions, until an atom has moved more than
 * skin / 2 since the build (a move by a lattice vector along a periodic
 * axis, as when an integrator wraps positions into the cell, does not
 * count), the atom count, cell or pbc change, or a batch or another call
 * rebuilds the list.  The extra pairs lie beyond the cutoff, where the
 * smooth cutoff is 0 and the key mask -inf, like the reference's padding,
 * so results agree with fresh lists to rounding.  A kept list also keeps
 * the shapes, so the model's kernels replay from a CUDA graph.  0 (the
 * default) rebuilds every call.  A skin that is negative or not finite is
 * MLIPCPP_ERROR_INVALID_PARAMETER. */
mlipcpp_error_t mlipcpp_b200_set_neighbor_skin(mlipcpp_model_t model, float skin);

/* Neighbour lists this model has built so far (kept lists count once);
 * -1 for an invalid or unloaded model. */
int64_t mlipcpp_b200_neighbor_builds(mlipcpp_model_t model);

/* Enable per-phase CUDA-event timing of later predictions. */
mlipcpp_error_t mlipcpp_b200_set_timing(mlipcpp_model_t model, bool enable);

/* Phase times (ms) of the last prediction: h2d, neighbour list, graph prep,
 * forward, backward, reductions, d2h, total. */
mlipcpp_error_t mlipcpp_b200_last_timings(mlipcpp_model_t model, float times_ms[8]);

/* Size of the last prediction: atoms, edges, max neighbours, device bytes
 * held by the model (MiB). */
mlipcpp_error_t mlipcpp_b200_last_shape(mlipcpp_model_t model, int64_t shape[4]);

/* Full neighbour list (no self pairs) of one structure computed on the GPU,
 * bit-identical to the reference's NeighborListBuilder
 * (src/core/neighbor_list.cpp:118-297), in its enumeration order.  Host
 * pointers in and out; writes at most `cap` pairs into the (optional)
 * arrays and returns the total pair count, or -(error code) on failure, so
 * a call with cap = 0 sizes the buffers.  shifts: [3 * pairs] int32,
 * vectors: [3 * pairs] float, distances: [pairs] float. */
int64_t mlipcpp_b200_neighbor_list(int32_t n_atoms, const float *positions, const float *cell,
                                   const bool *pbc, float cutoff, int64_t cap, int32_t *centers,
                                   int32_t *neighbors, int32_t *shifts, float *vectors,
                                   float *distances);

/* No counterpart in the reference.  The periodic (or partially periodic)
 * neighbour list of mlipcpp_b200_neighbor_list, same pairs in the same
 * order, for callers that cannot let a library allocate GPU memory: an MD
 * engine or host framework that hands out every device buffer from its own
 * pool, and code running where a cudaMalloc would stall other streams or is
 * not permitted.  It allocates nothing.  `d_positions` ([3 n_atoms] float)
 * and the five pair arrays are the caller's device buffers on the calling
 * thread's current device; `cell` and `pbc` are host arrays as in
 * mlipcpp_b200_neighbor_list (cell is required).  The working memory is a
 * fixed static device array of 2.6 MB inside this library, which limits a
 * call to at most 65536 atoms and 65536 cutoff-sized bins; larger requests
 * return -MLIPCPP_ERROR_INVALID_PARAMETER with a message naming the limit,
 * before any device work; so do a cutoff that is not finite and positive,
 * one that spans more than 511 cell widths along an axis, and a list that
 * could exceed 2^31 - 1 pairs.  The first call on each device looks up that
 * array's address (cudaGetSymbolAddress), so make it before any stream
 * capture.  All calls on one device share the array, and each call clears
 * the parts that must start at zero: calls that overlap in time (from
 * several host threads or streams) race, so serialise them.
 * Work runs on `stream` (NULL: the legacy default stream).  Every call
 * copies the pair count to the host and synchronises `stream` before it
 * returns, so its work there has finished by then.  Returns the total pair
 * count; the arrays are written only when it is at most `cap` (else call
 * again with larger arrays), or -(error code) on failure. */
int64_t mlipcpp_b200_neighbor_list_noalloc(int32_t n_atoms, const float *d_positions, const float *cell,
                                           const bool *pbc, float cutoff, int64_t cap, int32_t *d_centers,
                                           int32_t *d_neighbors, int32_t *d_shifts, float *d_vectors,
                                           float *d_distances, void *stream);

/* ---- Spatial domain decomposition of one periodic cell (no counterpart in
 * the reference, which evaluates a structure on one device:
 * PETModel::predict_batch, src/models/pet/pet.cpp:125-694) ----------------
 * One rank per GPU, each with its own model.  The cell is split into
 * grid[0] x grid[1] x grid[2] fractional slabs; rank r owns slab
 * (r % g0, r / g0 % g1, r / (g0 g1)) and the atoms assigned to it.  Every
 * step: owned atoms within cutoff + skin of another slab are sent there as
 * ghosts (periodic images included); each rank runs both GNN layers and the
 * readout on its owned atoms only; a layer-1 message that needs the layer-0
 * token of an edge held by another rank gets it from that rank, and the
 * token's gradient goes back; forces on ghosts return to their owners; the
 * energy and virial are summed over the ranks.  The exchanges are the
 * caller's collectives (mlipcpp_b200_comm_t), e.g. torch.distributed over
 * NCCL: alltoallv sends rank r the send_counts[r] elements of elem_bytes
 * bytes of d_send's r-th segment and receives recv_counts[r] elements from
 * rank r into d_recv's r-th segment (segments in rank order);
 * allreduce_sum_f64 sums n doubles in place.  Buffers are device memory of
 * the model's device; both calls must be ordered on `stream` (a cudaStream_t)
 * and return 0 on success.  Every call of domain_step is collective. */
typedef struct {
  void *user;
  int32_t (*alltoallv)(void *user, const void *d_send, const int64_t *send_counts, void *d_recv,
                       const int64_t *recv_counts, int64_t elem_bytes, void *stream);
  int32_t (*allreduce_sum_f64)(void *user, double *d_buf, int64_t n, void *stream);
} mlipcpp_b200_comm_t;

typedef struct mlipcpp_b200_domain_impl *mlipcpp_b200_domain_t;

/* This rank's domain.  cell: row-major lattice of the whole cell (periodic);
 * skin: halo width beyond the cutoff (A) for atoms that moved since
 * ownership was assigned.  Returns NULL on failure (message in
 * mlipcpp_get_last_error), e.g. when a slab is not wider than twice the
 * cutoff plus skin. */
mlipcpp_b200_domain_t mlipcpp_b200_domain_create(mlipcpp_model_t model, const float cell[9],
                                                 const int32_t grid[3], int32_t rank, float skin,
                                                 const mlipcpp_b200_comm_t *comm);
void mlipcpp_b200_domain_free(mlipcpp_b200_domain_t domain);
/* The owned atoms' atomic numbers (host), in the order of the positions of
 * every step.  An unknown Z returns MLIPCPP_ERROR_COMPUTATION. */
mlipcpp_error_t mlipcpp_b200_domain_set_atoms(mlipcpp_b200_domain_t domain, int32_t n_owned,
                                              const int32_t *atomic_numbers);
/* One evaluation: d_positions [3 n_owned] f32 device; d_forces [3 n_owned]
 * f32 device (may be NULL); energy (eV, composition included) and virial
 * (Voigt xx yy zz yz xz xy, sum_e e (x) dE/de, not divided by the volume)
 * over the whole cell, on every rank. */
mlipcpp_error_t mlipcpp_b200_domain_step(mlipcpp_b200_domain_t domain, const float *d_positions,
                                         float *d_forces, bool compute_forces, double *energy,
                                         double virial[6]);
/* Last step: device ms of halo, neighbour list + requests, model (with the
 * token exchanges), reverse force halo, sum over ranks, whole step; host ms
 * of the call; then owned atoms, ghosts, edges, token rows received, token
 * rows sent, halo copies sent -> stats[0..12]. */
mlipcpp_error_t mlipcpp_b200_domain_stats(mlipcpp_b200_domain_t domain, double stats[13]);

/* Number of CUDA kernels this library has launched in this process. */
int64_t mlipcpp_b200_kernel_launches(void);

/* Number of device allocations (cudaMalloc calls) this library has made in
 * this process. */
int64_t mlipcpp_b200_device_allocations(void);

/* Failure-detection test hooks (no counterpart in the reference).  Every
 * wait of the tensor-core GEMM pipelines is bounded; on expiry the CTA
 * stops, lets its own copies and MMAs complete, frees its tensor memory and
 * records a device error that the call returns as MLIPCPP_ERROR_COMPUTATION;
 * the model stays usable.  set_wait_bound_ns sets that bound on the current
 * device (0: the default of 1 s).  inject_gemm_stall makes the next GEMM
 * launch with a plain store epilogue withhold the operand loads of its
 * first CTA, so that CTA's waits run out. */
mlipcpp_error_t mlipcpp_b200_set_wait_bound_ns(uint64_t ns);
mlipcpp_error_t mlipcpp_b200_inject_gemm_stall(void);

/* CUDA device ordinal used by models created afterwards (default: the
 * calling thread's current device). */
mlipcpp_error_t mlipcpp_b200_set_device(int32_t device);

/* Time every GEMM and attention launch with CUDA events on the model's
 * stream (also resets the statistics). */
mlipcpp_error_t mlipcpp_b200_set_kernel_profiling(mlipcpp_model_t model, bool enable);

/* Cumulative per-class statistics since profiling was enabled: for classes
 * 3xTF32 tensor-core GEMM, SIMT GEMM, attention, neighbour list, other,
 * 3xFP16 tensor-core GEMM (with its row-scale pre-pass):
 * {launches, total ms, algorithmic FLOPs, algorithmic HBM bytes}
 * -> stats[4 * class + 0..3]. */
mlipcpp_error_t mlipcpp_b200_kernel_stats(mlipcpp_model_t model, double stats[24]);

#ifdef __cplusplus
}
#endif

#endif /* MLIPCPP_B200_H */
