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

/* One spatial domain of a large periodic cell (multi-GPU domain
 * decomposition).  d_positions: device pointer to [3 * n_local] double, the
 * owned atoms first, then the ghost atoms within one cutoff of the owned
 * region, then the other ghosts (periodic images already placed);
 * atomic_numbers is a host array.  Layer 0 runs on the first n_layer0
 * atoms, layer 1 and the readout on the first n_owned.  cell: row-major
 * cell of the search grid; pbc: per axis, whether the local system is
 * periodic along it (an axis the decomposition does not split) or open
 * (NULL: open along all three).  Along open axes the local positions should
 * lie inside the cell, for an even spread over the bins.
 * Outputs: energy of the owned atoms (host, eV, f64, composition included),
 * gradient forces on every local atom (d_forces: device [3 * n_local] float,
 * may be NULL), and the local virial sum_e e (x) dE/de in Voigt order (host,
 * f64, not divided by a volume).  Summing energies, virials and the forces
 * of each atom over all domains gives the whole cell's results. */
mlipcpp_error_t mlipcpp_b200_predict_local(mlipcpp_model_t model, int32_t n_local,
                                           const double *d_positions,
                                           const int32_t *atomic_numbers, int32_t n_layer0,
                                           int32_t n_owned, const float cell[9],
                                           const bool *pbc, bool compute_forces, float *d_forces, double *energy,
                                           double virial[6]);

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

/* Number of CUDA kernels this library has launched in this process. */
int64_t mlipcpp_b200_kernel_launches(void);

/* Number of device allocations (cudaMalloc calls) this library has made in
 * this process. */
int64_t mlipcpp_b200_device_allocations(void);

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
