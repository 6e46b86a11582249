/*
 * mlipcpp C API, implemented by the B200 backend (libmlipcpp_b200.so).
 *
 * Drop-in for mlip.cpp's include/mlipcpp/mlipcpp.h: every function, enum
 * value and struct layout below matches that header so existing callers
 * (the Fortran module, C programs, ctypes/cffi bindings) relink unchanged.
 * Each declaration cites the reference declaration it replaces.
 *
 * Behaviour that differs by design:
 *  - Only NVIDIA GPUs (sm_100a) are served.  There is no CPU fallback:
 *    selecting MLIPCPP_BACKEND_CPU (or another vendor's backend) makes
 *    mlipcpp_model_load fail with MLIPCPP_ERROR_BACKEND.
 *  - Only the "pet" GGUF architecture is implemented; "pet-graph" files load
 *    with MLIPCPP_ERROR_UNSUPPORTED.
 *
 * Thread safety: as in the reference, a model handle is not thread-safe; the
 * last error message is thread-local.
 */
#ifndef MLIPCPP_H
#define MLIPCPP_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library version "MAJOR.MINOR.PATCH" of the API implemented.
 * Replaces mlipcpp.h:36. */
const char *mlipcpp_version(void);

/* Error codes.  Replaces mlipcpp.h:46-58 (same values). */
typedef enum {
  MLIPCPP_OK = 0,
  MLIPCPP_ERROR_INVALID_HANDLE = 1,
  MLIPCPP_ERROR_NULL_POINTER = 2,
  MLIPCPP_ERROR_MODEL_NOT_LOADED = 3,
  MLIPCPP_ERROR_OUT_OF_MEMORY = 4,
  MLIPCPP_ERROR_IO = 5,
  MLIPCPP_ERROR_COMPUTATION = 6,
  MLIPCPP_ERROR_INVALID_PARAMETER = 7,
  MLIPCPP_ERROR_BACKEND = 8,
  MLIPCPP_ERROR_UNSUPPORTED = 9,
  MLIPCPP_ERROR_INTERNAL = 255
} mlipcpp_error_t;

/* Static description of an error code (never NULL).  Replaces mlipcpp.h:65. */
const char *mlipcpp_error_string(mlipcpp_error_t error);

/* Thread-local message of the last failure, NULL after a success.
 * Replaces mlipcpp.h:74. */
const char *mlipcpp_get_last_error(void);

/* Backend selection.  Replaces mlipcpp.h:84-94 (same values). */
typedef enum {
  MLIPCPP_BACKEND_AUTO = 0,
  MLIPCPP_BACKEND_CPU = 1,
  MLIPCPP_BACKEND_CUDA = 2,
  MLIPCPP_BACKEND_HIP = 3,
  MLIPCPP_BACKEND_METAL = 4,
  MLIPCPP_BACKEND_VULKAN = 5,
  MLIPCPP_BACKEND_SYCL = 6,
  MLIPCPP_BACKEND_CANN = 7,
  MLIPCPP_BACKEND_WEBGPU = 8
} mlipcpp_backend_t;

/* Global backend for models loaded afterwards.  Replaces mlipcpp.h:103. */
void mlipcpp_set_backend(mlipcpp_backend_t backend);
/* Name of the active backend ("CUDA").  Replaces mlipcpp.h:113. */
const char *mlipcpp_get_backend_name(void);
/* True when a CUDA device serves predictions.  Replaces mlipcpp.h:119. */
bool mlipcpp_backend_is_gpu(void);
/* True for AUTO and CUDA when a CUDA device is present; false otherwise.
 * Replaces mlipcpp.h:131. */
bool mlipcpp_is_backend_available(mlipcpp_backend_t backend);
/* Accepted for compatibility; this library does not log.  Replaces
 * mlipcpp.h:140. */
void mlipcpp_suppress_logging(void);

/* Compute precision.  Replaces mlipcpp.h:145-149 (same values).
 * F32: fp32-accurate arithmetic.  F16: accepted, computed as F32. */
typedef enum {
  MLIPCPP_PRECISION_F32 = 0,
  MLIPCPP_PRECISION_F16 = 1
} mlipcpp_precision_t;

/* Opaque handles.  Replace mlipcpp.h:159,167. */
typedef struct mlipcpp_model_impl *mlipcpp_model_t;
typedef struct mlipcpp_result_impl *mlipcpp_result_t;

/* Model options.  Replaces mlipcpp.h:177-181 (same layout). */
typedef struct {
  mlipcpp_backend_t backend;
  mlipcpp_precision_t precision;
  float cutoff_override; /* as in the reference, only used when the GGUF has no pet.cutoff */
} mlipcpp_model_options_t;

/* Defaults: AUTO, F32, 0.0.  Replaces mlipcpp.h:193. */
mlipcpp_error_t mlipcpp_model_options_default(mlipcpp_model_options_t *options);

/* One structure.  Replaces mlipcpp.h:216-222 (same layout): positions
 * [3n] (x,y,z per atom, Angstrom), atomic numbers [n], cell [9] row-major
 * with lattice vectors as rows or NULL (non-periodic), pbc [3] or NULL
 * (all periodic when a cell is given). */
typedef struct {
  int32_t n_atoms;
  const float *positions;
  const int32_t *atomic_numbers;
  const float *cell;
  const bool *pbc;
} mlipcpp_system_t;

/* Model lifecycle.  Replace mlipcpp.h:237,248,257,268. */
mlipcpp_model_t mlipcpp_model_create(const mlipcpp_model_options_t *options);
mlipcpp_error_t mlipcpp_model_load(mlipcpp_model_t model, const char *path);
void mlipcpp_model_free(mlipcpp_model_t model);
mlipcpp_error_t mlipcpp_model_get_cutoff(mlipcpp_model_t model, float *cutoff);

/* Prediction options.  Replaces mlipcpp.h:278-283 (same layout). */
typedef struct {
  bool compute_forces;
  bool compute_stress;
  bool use_nc_forces;
} mlipcpp_predict_options_t;

/* Defaults: forces on, stress off, nc off.  Replaces mlipcpp.h:295. */
mlipcpp_error_t mlipcpp_predict_options_default(mlipcpp_predict_options_t *options);

/* Prediction.  Replace mlipcpp.h:317,336,358,378.  `compute_forces` (or
 * forces/stress options) runs the backward pass; stress is produced for
 * periodic systems.  The returned handle refers to the model's last result:
 * it is valid until the model's next prediction or free, and is released
 * with mlipcpp_result_free. */
mlipcpp_error_t mlipcpp_predict(mlipcpp_model_t model, const mlipcpp_system_t *system,
                                bool compute_forces, mlipcpp_result_t *result);
mlipcpp_error_t mlipcpp_predict_ptr(mlipcpp_model_t model, int32_t n_atoms,
                                    const float *positions, const int32_t *atomic_numbers,
                                    const float *cell, const bool *pbc, bool compute_forces,
                                    mlipcpp_result_t *result);
mlipcpp_error_t mlipcpp_predict_with_options(mlipcpp_model_t model,
                                             const mlipcpp_system_t *system,
                                             const mlipcpp_predict_options_t *options,
                                             mlipcpp_result_t *result);
mlipcpp_error_t mlipcpp_predict_ptr_with_options(mlipcpp_model_t model, int32_t n_atoms,
                                                 const float *positions,
                                                 const int32_t *atomic_numbers,
                                                 const float *cell, const bool *pbc,
                                                 const mlipcpp_predict_options_t *options,
                                                 mlipcpp_result_t *result);

/* Result access.  Replace mlipcpp.h:396,410,424,433,442,451,463.
 * Energy in eV, forces [n*3] in eV/A, stress [6] Voigt (xx,yy,zz,yz,xz,xy)
 * in eV/A^3. */
mlipcpp_error_t mlipcpp_result_get_energy(mlipcpp_result_t result, float *energy);
mlipcpp_error_t mlipcpp_result_get_forces(mlipcpp_result_t result, float *forces, int32_t n_atoms);
mlipcpp_error_t mlipcpp_result_get_stress(mlipcpp_result_t result, float stress[6]);
mlipcpp_error_t mlipcpp_result_n_atoms(mlipcpp_result_t result, int32_t *n_atoms);
mlipcpp_error_t mlipcpp_result_has_forces(mlipcpp_result_t result, bool *has_forces);
mlipcpp_error_t mlipcpp_result_has_stress(mlipcpp_result_t result, bool *has_stress);
void mlipcpp_result_free(mlipcpp_result_t result);

#ifdef __cplusplus
}
#endif

#endif /* MLIPCPP_H */
