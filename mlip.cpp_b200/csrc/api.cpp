// mlipcpp C API over the B200 PET backend.  Mirrors the reference
// implementation's contract (src/api/c/mlipcpp_api.cpp): argument checks and
// their error codes, thread-local error messages, no exception crossing the
// ABI, and a result handle that refers to the model's last result.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "mlipcpp.h"
#include "mlipcpp_b200.h"
#include "domain.h"
#include "gemm_tc.cuh"
#include "gguf.h"
#include "model.h"

namespace pet {
std::atomic<long long> g_kernel_launches{0};
std::atomic<long long> g_device_allocations{0};
extern int g_default_device;
}

struct mlipcpp_model_impl {
  std::unique_ptr<pet::PETModel> model;
  mlipcpp_model_options_t options{};
  pet::Result last;
  bool loaded = false;
};

struct mlipcpp_b200_domain_impl {
  std::unique_ptr<pet::DomainEngine> engine;
};

struct mlipcpp_result_impl {
  const pet::Result *result = nullptr;  // the model's last result, or `own`
  pet::Result own;
  int32_t n_atoms = 0;
};

namespace {

thread_local std::string g_last_error;
std::mutex g_backend_mutex;
mlipcpp_backend_t g_backend = MLIPCPP_BACKEND_AUTO;

void set_error(const std::string &m) { g_last_error = m; }
void clear_error() { g_last_error.clear(); }

bool have_cuda_device() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

bool backend_served(mlipcpp_backend_t b) {
  return (b == MLIPCPP_BACKEND_AUTO || b == MLIPCPP_BACKEND_CUDA) && have_cuda_device();
}

// Build a SystemView the way the reference builds its AtomicSystem
// (mlipcpp_api.cpp:438-460): a cell with NULL pbc means all periodic.
pet::SystemView make_view(const mlipcpp_system_t *s) {
  pet::SystemView v;
  v.n_atoms = s->n_atoms;
  v.positions = s->positions;
  v.numbers = s->atomic_numbers;
  v.cell = s->cell;
  if (s->cell && s->pbc) {
    v.pbc[0] = s->pbc[0];
    v.pbc[1] = s->pbc[1];
    v.pbc[2] = s->pbc[2];
  }
  return v;
}

mlipcpp_error_t check_model(mlipcpp_model_t model) {
  if (!model) {
    set_error("Invalid model handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!model->loaded) {
    set_error("Model weights not loaded");
    return MLIPCPP_ERROR_MODEL_NOT_LOADED;
  }
  return MLIPCPP_OK;
}

mlipcpp_error_t check_system(const mlipcpp_system_t *system) {
  if (system->n_atoms <= 0) {
    set_error("Invalid number of atoms");
    return MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (!system->positions || !system->atomic_numbers) {
    set_error("NULL positions or atomic_numbers");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  return MLIPCPP_OK;
}

mlipcpp_error_t map_exception(const std::exception &e, const char *what, int dflt) {
  set_error(std::string(what) + e.what());
  if (auto *pe = dynamic_cast<const pet::Error *>(&e)) return static_cast<mlipcpp_error_t>(pe->code);
  return static_cast<mlipcpp_error_t>(dflt);
}

// predict_with_options semantics (mlipcpp_api.cpp:569-593): gradient when
// forces or stress are wanted and nc forces are not; unrequested outputs
// cleared afterwards.
void finish_options(pet::Result &r, const mlipcpp_predict_options_t &o) {
  if (!o.compute_forces) {
    r.forces.clear();
    r.has_forces = false;
  }
  if (!o.compute_stress) {
    r.stress.clear();
    r.has_stress = false;
  }
}

}  // namespace

extern "C" {

const char *mlipcpp_version(void) { return "0.1.2"; }

const char *mlipcpp_error_string(mlipcpp_error_t error) {
  switch (error) {
    case MLIPCPP_OK: return "Success";
    case MLIPCPP_ERROR_INVALID_HANDLE: return "Invalid model or result handle";
    case MLIPCPP_ERROR_NULL_POINTER: return "NULL pointer passed to function";
    case MLIPCPP_ERROR_MODEL_NOT_LOADED: return "Model weights not loaded";
    case MLIPCPP_ERROR_OUT_OF_MEMORY: return "Memory allocation failed";
    case MLIPCPP_ERROR_IO: return "File I/O error";
    case MLIPCPP_ERROR_COMPUTATION: return "Computation graph execution failed";
    case MLIPCPP_ERROR_INVALID_PARAMETER: return "Invalid parameter value";
    case MLIPCPP_ERROR_BACKEND: return "Backend initialization failed";
    case MLIPCPP_ERROR_UNSUPPORTED: return "Operation not supported";
    case MLIPCPP_ERROR_INTERNAL: return "Internal error (bug in mlipcpp)";
    default: return "Unknown error";
  }
}

const char *mlipcpp_get_last_error(void) { return g_last_error.empty() ? nullptr : g_last_error.c_str(); }

void mlipcpp_set_backend(mlipcpp_backend_t backend) {
  std::lock_guard<std::mutex> lock(g_backend_mutex);
  g_backend = backend;
}

const char *mlipcpp_get_backend_name(void) { return "CUDA"; }

bool mlipcpp_backend_is_gpu(void) { return have_cuda_device(); }

bool mlipcpp_is_backend_available(mlipcpp_backend_t backend) { return backend_served(backend); }

void mlipcpp_suppress_logging(void) {}

mlipcpp_error_t mlipcpp_model_options_default(mlipcpp_model_options_t *options) {
  if (!options) {
    set_error("NULL pointer for options");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  options->backend = MLIPCPP_BACKEND_AUTO;
  options->precision = MLIPCPP_PRECISION_F32;
  options->cutoff_override = 0.0f;
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_model_t mlipcpp_model_create(const mlipcpp_model_options_t *options) {
  try {
    mlipcpp_model_options_t dflt;
    if (!options) {
      mlipcpp_model_options_default(&dflt);
      options = &dflt;
    }
    auto impl = std::make_unique<mlipcpp_model_impl>();
    impl->options = *options;
    if (options->backend != MLIPCPP_BACKEND_AUTO) mlipcpp_set_backend(options->backend);
    clear_error();
    return impl.release();
  } catch (const std::exception &e) {
    set_error(std::string("Failed to create model: ") + e.what());
    return nullptr;
  }
}

mlipcpp_error_t mlipcpp_model_load(mlipcpp_model_t model, const char *path) {
  if (!model) {
    set_error("Invalid model handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!path) {
    set_error("NULL path");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  try {
    mlipcpp_backend_t b;
    {
      std::lock_guard<std::mutex> lock(g_backend_mutex);
      b = g_backend;
    }
    if (!backend_served(b)) {
      set_error(b == MLIPCPP_BACKEND_AUTO || b == MLIPCPP_BACKEND_CUDA
                    ? "No CUDA device available (this backend has no CPU fallback)"
                    : "Requested backend is not available in the B200 build (CUDA only)");
      return MLIPCPP_ERROR_BACKEND;
    }
    std::string arch;
    {
      pet::GGUFFile f(path);
      arch = f.get_string("general.architecture", "");
    }
    if (arch == "pet-graph") {
      set_error("Unsupported model architecture: pet-graph (not implemented by the B200 backend)");
      return MLIPCPP_ERROR_UNSUPPORTED;
    }
    if (arch != "pet") {
      set_error("Unsupported model architecture: " + arch);
      return MLIPCPP_ERROR_UNSUPPORTED;
    }
    auto m = std::make_unique<pet::PETModel>();
    m->load(path, model->options.cutoff_override);
    m->set_reduced_precision(model->options.precision == MLIPCPP_PRECISION_F16);
    model->model = std::move(m);
    model->loaded = true;
    clear_error();
    return MLIPCPP_OK;
  } catch (const pet::Error &e) {
    set_error(std::string("Error loading model: ") + e.what());
    return e.code == pet::kErrBackend || e.code == pet::kErrOutOfMemory || e.code == pet::kErrUnsupported
               ? static_cast<mlipcpp_error_t>(e.code) : MLIPCPP_ERROR_IO;
  } catch (const std::exception &e) {
    set_error(std::string("Error loading model: ") + e.what());
    return MLIPCPP_ERROR_IO;
  } catch (...) {
    set_error("Error loading model: unknown error");
    return MLIPCPP_ERROR_INTERNAL;
  }
}

void mlipcpp_model_free(mlipcpp_model_t model) { delete model; }

mlipcpp_error_t mlipcpp_model_get_cutoff(mlipcpp_model_t model, float *cutoff) {
  if (!model) {
    set_error("Invalid model handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!cutoff) {
    set_error("NULL cutoff pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  if (!model->loaded) {
    set_error("Model weights not loaded");
    return MLIPCPP_ERROR_MODEL_NOT_LOADED;
  }
  *cutoff = model->model->cutoff();
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_predict_options_default(mlipcpp_predict_options_t *options) {
  if (!options) {
    set_error("NULL pointer for options");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  options->compute_forces = true;
  options->compute_stress = false;
  options->use_nc_forces = false;
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_predict(mlipcpp_model_t model, const mlipcpp_system_t *system,
                                bool compute_forces, mlipcpp_result_t *result) {
  if (!model) {
    set_error("Invalid model handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!system) {
    set_error("NULL system pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  if (!result) {
    set_error("NULL result pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  if (auto e = check_model(model)) return e;
  if (auto e = check_system(system)) return e;
  try {
    std::vector<pet::SystemView> v{make_view(system)};
    auto out = model->model->predict(v, compute_forces);
    model->last = std::move(out[0]);
    auto r = std::make_unique<mlipcpp_result_impl>();
    r->result = &model->last;
    r->n_atoms = system->n_atoms;
    *result = r.release();
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Prediction failed: ", MLIPCPP_ERROR_COMPUTATION);
  } catch (...) {
    set_error("Prediction failed: unknown error");
    return MLIPCPP_ERROR_INTERNAL;
  }
}

mlipcpp_error_t mlipcpp_predict_ptr(mlipcpp_model_t model, int32_t n_atoms, const float *positions,
                                    const int32_t *atomic_numbers, const float *cell, const bool *pbc,
                                    bool compute_forces, mlipcpp_result_t *result) {
  mlipcpp_system_t s{n_atoms, positions, atomic_numbers, cell, pbc};
  return mlipcpp_predict(model, &s, compute_forces, result);
}

mlipcpp_error_t mlipcpp_predict_with_options(mlipcpp_model_t model, const mlipcpp_system_t *system,
                                             const mlipcpp_predict_options_t *options,
                                             mlipcpp_result_t *result) {
  if (!model) {
    set_error("Invalid model handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!system) {
    set_error("NULL system pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  if (!result) {
    set_error("NULL result pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  if (auto e = check_model(model)) return e;
  mlipcpp_predict_options_t dflt;
  if (!options) {
    mlipcpp_predict_options_default(&dflt);
    options = &dflt;
  }
  if (auto e = check_system(system)) return e;
  try {
    const bool grad = (options->compute_forces || options->compute_stress) && !options->use_nc_forces;
    std::vector<pet::SystemView> v{make_view(system)};
    auto out = model->model->predict(v, grad, options->use_nc_forces);
    model->last = std::move(out[0]);
    finish_options(model->last, *options);
    auto r = std::make_unique<mlipcpp_result_impl>();
    r->result = &model->last;
    r->n_atoms = system->n_atoms;
    *result = r.release();
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Prediction failed: ", MLIPCPP_ERROR_COMPUTATION);
  } catch (...) {
    set_error("Prediction failed: unknown error");
    return MLIPCPP_ERROR_INTERNAL;
  }
}

mlipcpp_error_t mlipcpp_predict_ptr_with_options(mlipcpp_model_t model, int32_t n_atoms,
                                                 const float *positions, const int32_t *atomic_numbers,
                                                 const float *cell, const bool *pbc,
                                                 const mlipcpp_predict_options_t *options,
                                                 mlipcpp_result_t *result) {
  mlipcpp_system_t s{n_atoms, positions, atomic_numbers, cell, pbc};
  return mlipcpp_predict_with_options(model, &s, options, result);
}

mlipcpp_error_t mlipcpp_result_get_energy(mlipcpp_result_t result, float *energy) {
  if (!result) {
    set_error("Invalid result handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!energy) {
    set_error("NULL energy pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  *energy = result->result->energy;
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_result_get_forces(mlipcpp_result_t result, float *forces, int32_t n_atoms) {
  if (!result) {
    set_error("Invalid result handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!forces) {
    set_error("NULL forces pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  if (n_atoms != result->n_atoms) {
    set_error("n_atoms mismatch");
    return MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (!result->result->has_forces || result->result->forces.size() < static_cast<size_t>(n_atoms) * 3) {
    set_error("Forces not available (compute_forces was false)");
    return MLIPCPP_ERROR_UNSUPPORTED;
  }
  std::memcpy(forces, result->result->forces.data(), sizeof(float) * 3 * n_atoms);
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_result_get_stress(mlipcpp_result_t result, float stress[6]) {
  if (!result) {
    set_error("Invalid result handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!stress) {
    set_error("NULL stress pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  if (!result->result->has_stress) {
    set_error("Stress not available");
    return MLIPCPP_ERROR_UNSUPPORTED;
  }
  std::memcpy(stress, result->result->stress.data(), sizeof(float) * 6);
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_result_n_atoms(mlipcpp_result_t result, int32_t *n_atoms) {
  if (!result) {
    set_error("Invalid result handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!n_atoms) {
    set_error("NULL n_atoms pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  *n_atoms = result->n_atoms;
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_result_has_forces(mlipcpp_result_t result, bool *has_forces) {
  if (!result) {
    set_error("Invalid result handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!has_forces) {
    set_error("NULL has_forces pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  *has_forces = result->result->has_forces;
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_result_has_stress(mlipcpp_result_t result, bool *has_stress) {
  if (!result) {
    set_error("Invalid result handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!has_stress) {
    set_error("NULL has_stress pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  *has_stress = result->result->has_stress;
  clear_error();
  return MLIPCPP_OK;
}

void mlipcpp_result_free(mlipcpp_result_t result) { delete result; }

// ---------------------------------------------------------------------------
// Extensions (include/mlipcpp_b200.h)
// ---------------------------------------------------------------------------
mlipcpp_error_t mlipcpp_predict_batch(mlipcpp_model_t model, int32_t n_systems,
                                      const mlipcpp_system_t *systems,
                                      const mlipcpp_predict_options_t *options,
                                      mlipcpp_result_t *results) {
  if (auto e = check_model(model)) return e;
  if (n_systems < 0) {
    set_error("Invalid number of systems");
    return MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (n_systems > 0 && (!systems || !results)) {
    set_error("NULL systems or results pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  mlipcpp_predict_options_t dflt;
  if (!options) {
    mlipcpp_predict_options_default(&dflt);
    options = &dflt;
  }
  for (int k = 0; k < n_systems; ++k)
    if (auto e = check_system(&systems[k])) return e;
  try {
    const bool grad = (options->compute_forces || options->compute_stress) && !options->use_nc_forces;
    std::vector<pet::SystemView> v;
    for (int k = 0; k < n_systems; ++k) v.push_back(make_view(&systems[k]));
    auto out = model->model->predict(v, grad, options->use_nc_forces);
    for (int k = 0; k < n_systems; ++k) {
      auto r = std::make_unique<mlipcpp_result_impl>();
      r->own = std::move(out[k]);
      finish_options(r->own, *options);
      r->result = &r->own;
      r->n_atoms = systems[k].n_atoms;
      results[k] = r.release();
    }
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Prediction failed: ", MLIPCPP_ERROR_COMPUTATION);
  } catch (...) {
    set_error("Prediction failed: unknown error");
    return MLIPCPP_ERROR_INTERNAL;
  }
}

mlipcpp_error_t mlipcpp_b200_predict_packed(mlipcpp_model_t model, int32_t n_systems, const int32_t *n_atoms,
                                            const float *positions, const int32_t *numbers, const float *cells,
                                            const bool *pbc, const mlipcpp_predict_options_t *options,
                                            float *energies, float *forces, float *stress) {
  if (auto e = check_model(model)) return e;
  if (n_systems < 0) {
    set_error("Invalid number of systems");
    return MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (n_systems > 0 && (!n_atoms || !positions || !numbers || !energies)) {
    set_error("NULL n_atoms, positions, atomic_numbers or energies pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  mlipcpp_predict_options_t dflt;
  if (!options) {
    mlipcpp_predict_options_default(&dflt);
    options = &dflt;
  }
  std::vector<pet::SystemView> v(static_cast<size_t>(n_systems));
  std::vector<int64_t> first(static_cast<size_t>(n_systems) + 1, 0);
  for (int k = 0; k < n_systems; ++k) {
    if (n_atoms[k] <= 0) {
      set_error("Invalid number of atoms");
      return MLIPCPP_ERROR_INVALID_PARAMETER;
    }
    pet::SystemView &s = v[k];
    s.n_atoms = n_atoms[k];
    s.positions = positions + 3 * first[k];
    s.numbers = numbers + first[k];
    if (cells) {
      s.cell = cells + 9 * static_cast<size_t>(k);
      if (pbc)
        for (int c = 0; c < 3; ++c) s.pbc[c] = pbc[3 * static_cast<size_t>(k) + c];
    }
    first[k + 1] = first[k] + n_atoms[k];
  }
  try {
    const bool grad = (options->compute_forces || options->compute_stress) && !options->use_nc_forces;
    auto out = model->model->predict(v, grad, options->use_nc_forces);
    for (int k = 0; k < n_systems; ++k) {
      pet::Result &r = out[k];
      finish_options(r, *options);
      energies[k] = r.energy;
      if (forces) {
        float *f = forces + 3 * first[k];
        const size_t n3 = 3 * static_cast<size_t>(n_atoms[k]);
        if (r.has_forces && r.forces.size() == n3) std::memcpy(f, r.forces.data(), sizeof(float) * n3);
        else std::memset(f, 0, sizeof(float) * n3);
      }
      if (stress) {
        float *st = stress + 6 * static_cast<size_t>(k);
        if (r.has_stress && r.stress.size() == 6) std::memcpy(st, r.stress.data(), sizeof(float) * 6);
        else std::memset(st, 0, sizeof(float) * 6);
      }
    }
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Prediction failed: ", MLIPCPP_ERROR_COMPUTATION);
  } catch (...) {
    set_error("Prediction failed: unknown error");
    return MLIPCPP_ERROR_INTERNAL;
  }
}

mlipcpp_error_t mlipcpp_b200_predict_device(mlipcpp_model_t model, int32_t n_atoms, const float *d_positions,
                                            const int32_t *atomic_numbers, const float *cell, const bool *pbc,
                                            const mlipcpp_predict_options_t *options, bool copy_forces,
                                            mlipcpp_result_t *result) {
  if (auto e = check_model(model)) return e;
  if (!result) {
    set_error("NULL result pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  mlipcpp_system_t s{n_atoms, d_positions, atomic_numbers, cell, pbc};
  if (auto e = check_system(&s)) return e;
  mlipcpp_predict_options_t dflt;
  if (!options) {
    mlipcpp_predict_options_default(&dflt);
    options = &dflt;
  }
  try {
    const bool grad = (options->compute_forces || options->compute_stress) && !options->use_nc_forces;
    pet::SystemView v = make_view(&s);
    model->model->predict_device(d_positions, v, grad, model->last, copy_forces, options->use_nc_forces);
    finish_options(model->last, *options);
    auto r = std::make_unique<mlipcpp_result_impl>();
    r->result = &model->last;
    r->n_atoms = n_atoms;
    *result = r.release();
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Prediction failed: ", MLIPCPP_ERROR_COMPUTATION);
  }
}

mlipcpp_error_t mlipcpp_b200_predict_device_forces(mlipcpp_model_t model, int32_t n_atoms, const float *d_positions,
                                                   const int32_t *atomic_numbers, const float *cell,
                                                   const bool *pbc, const mlipcpp_predict_options_t *options,
                                                   float *d_forces, double *energy, float stress[6],
                                                   bool *has_stress) {
  if (auto e = check_model(model)) return e;
  if (!energy) {
    set_error("NULL energy pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  mlipcpp_system_t s{n_atoms, d_positions, atomic_numbers, cell, pbc};
  if (auto e = check_system(&s)) return e;
  mlipcpp_predict_options_t dflt;
  if (!options) {
    mlipcpp_predict_options_default(&dflt);
    options = &dflt;
  }
  try {
    const bool grad = (options->compute_forces || options->compute_stress) && !options->use_nc_forces;
    pet::SystemView v = make_view(&s);
    model->model->predict_device(d_positions, v, grad, model->last, false, options->use_nc_forces);
    finish_options(model->last, *options);
    *energy = model->last.energy;
    if (d_forces) {
      if (!model->last.has_forces) {
        set_error("No forces: compute_forces is off or the model has no force heads");
        return MLIPCPP_ERROR_INVALID_PARAMETER;
      }
      CUDA_CHECK(cudaMemcpyAsync(d_forces, model->model->device_forces(), sizeof(float) * 3 * n_atoms,
                                 cudaMemcpyDeviceToDevice, model->model->stream()));
      CUDA_CHECK(cudaStreamSynchronize(model->model->stream()));
    }
    if (has_stress) *has_stress = model->last.has_stress;
    if (stress && model->last.has_stress)
      for (int c = 0; c < 6; ++c) stress[c] = model->last.stress[c];
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Prediction failed: ", MLIPCPP_ERROR_COMPUTATION);
  }
}

static_assert(sizeof(mlipcpp_b200_comm_t) == sizeof(pet::DomainComm), "comm layout");

mlipcpp_b200_domain_t mlipcpp_b200_domain_create(mlipcpp_model_t model, const float cell[9], const int32_t grid[3],
                                                 int32_t rank, float skin, const mlipcpp_b200_comm_t *comm) {
  if (check_model(model)) return nullptr;
  if (!cell || !grid || !comm) {
    set_error("NULL pointer argument");
    return nullptr;
  }
  try {
    pet::DomainComm c;
    c.user = comm->user;
    c.alltoallv = comm->alltoallv;
    c.allreduce_sum_f64 = comm->allreduce_sum_f64;
    const int g[3] = {grid[0], grid[1], grid[2]};
    auto *d = new mlipcpp_b200_domain_impl();
    try {
      d->engine.reset(new pet::DomainEngine(*model->model, cell, g, rank, skin, c));
    } catch (...) {
      delete d;
      throw;
    }
    clear_error();
    return d;
  } catch (const std::exception &e) {
    map_exception(e, "Domain set-up failed: ", MLIPCPP_ERROR_INVALID_PARAMETER);
    return nullptr;
  }
}

void mlipcpp_b200_domain_free(mlipcpp_b200_domain_t domain) { delete domain; }

mlipcpp_error_t mlipcpp_b200_domain_set_atoms(mlipcpp_b200_domain_t domain, int32_t n_owned,
                                              const int32_t *atomic_numbers) {
  if (!domain) {
    set_error("Invalid domain handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (n_owned < 0 || (n_owned > 0 && !atomic_numbers)) {
    set_error("owned atoms: negative count or NULL atomic numbers");
    return MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  try {
    domain->engine->set_atoms(n_owned, atomic_numbers);
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Domain set-up failed: ", MLIPCPP_ERROR_COMPUTATION);
  }
}

mlipcpp_error_t mlipcpp_b200_domain_step(mlipcpp_b200_domain_t domain, const float *d_positions, float *d_forces,
                                         bool compute_forces, double *energy, double virial[6]) {
  if (!domain) {
    set_error("Invalid domain handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!energy || !virial) {
    set_error("NULL energy or virial pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  try {
    domain->engine->step(d_positions, d_forces, compute_forces, energy, virial);
    clear_error();
    return MLIPCPP_OK;
  } catch (const std::exception &e) {
    return map_exception(e, "Prediction failed: ", MLIPCPP_ERROR_COMPUTATION);
  }
}

mlipcpp_error_t mlipcpp_b200_domain_stats(mlipcpp_b200_domain_t domain, double stats[13]) {
  if (!domain) {
    set_error("Invalid domain handle");
    return MLIPCPP_ERROR_INVALID_HANDLE;
  }
  if (!stats) {
    set_error("NULL stats pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  const pet::DomainStats &st = domain->engine->stats();
  for (int k = 0; k < 7; ++k) stats[k] = st.ms[k];
  stats[7] = static_cast<double>(st.n_own);
  stats[8] = static_cast<double>(st.n_ghost);
  stats[9] = static_cast<double>(st.n_edges);
  stats[10] = static_cast<double>(st.n_req_out);
  stats[11] = static_cast<double>(st.n_req_in);
  stats[12] = static_cast<double>(st.n_sent);
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_b200_set_neighbor_skin(mlipcpp_model_t model, float skin) {
  if (auto e = check_model(model)) return e;
  if (!(skin >= 0.f) || !std::isfinite(skin)) {
    set_error("Invalid neighbour-list skin");
    return MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  model->model->set_neighbor_skin(skin);
  clear_error();
  return MLIPCPP_OK;
}

int64_t mlipcpp_b200_neighbor_builds(mlipcpp_model_t model) {
  if (check_model(model)) return -1;
  return model->model->neighbor_builds();
}

mlipcpp_error_t mlipcpp_b200_set_timing(mlipcpp_model_t model, bool enable) {
  if (auto e = check_model(model)) return e;
  model->model->set_timing(enable);
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_b200_last_timings(mlipcpp_model_t model, float t[8]) {
  if (auto e = check_model(model)) return e;
  if (!t) {
    set_error("NULL timings pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  const auto &p = model->model->last_times();
  const float v[8] = {p.h2d, p.nl, p.prep, p.forward, p.backward, p.reduce, p.d2h, p.total};
  std::memcpy(t, v, sizeof(v));
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_b200_last_shape(mlipcpp_model_t model, int64_t shape[4]) {
  if (auto e = check_model(model)) return e;
  if (!shape) {
    set_error("NULL shape pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  shape[0] = model->model->last_atoms();
  shape[1] = model->model->last_edges();
  shape[2] = model->model->last_max_neighbors();
  shape[3] = static_cast<int64_t>(model->model->device_bytes() >> 20);
  clear_error();
  return MLIPCPP_OK;
}

int64_t mlipcpp_b200_neighbor_list(int32_t n_atoms, const float *positions, const float *cell,
                                   const bool *pbc, float cutoff, int64_t cap, int32_t *centers,
                                   int32_t *neighbors, int32_t *shifts, float *vectors,
                                   float *distances) {
  if (n_atoms < 0) {
    set_error("Invalid number of atoms");
    return -MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (n_atoms > 0 && !positions) {
    set_error("NULL positions");
    return -MLIPCPP_ERROR_NULL_POINTER;
  }
  if (!std::isfinite(cutoff) || cutoff <= 0.0f) {
    set_error("The cutoff must be finite and positive");
    return -MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (!have_cuda_device()) {
    set_error("No CUDA device available (this backend has no CPU fallback)");
    return -MLIPCPP_ERROR_BACKEND;
  }
  try {
    struct Ctx {
      cudaStream_t s = nullptr;
      pet::EdgeList nl;
      pet::NLScratch scr;
      pet::DevBuf pos, b, e;
      ~Ctx() { if (s) cudaStreamDestroy(s); }
    };
    thread_local Ctx ctx;
    if (!ctx.s) CUDA_CHECK(cudaStreamCreateWithFlags(&ctx.s, cudaStreamNonBlocking));
    float *dp = static_cast<float *>(ctx.pos.ensure(sizeof(float) * 3 * (n_atoms + 1)));
    if (n_atoms > 0)
      CUDA_CHECK(cudaMemcpyAsync(dp, positions, sizeof(float) * 3 * n_atoms, cudaMemcpyHostToDevice, ctx.s));
    if (cell) {
      bool p[3] = {true, true, true};
      if (pbc) { p[0] = pbc[0]; p[1] = pbc[1]; p[2] = pbc[2]; }
      pet::GridParams g;
      pet::make_grid_params(cell, p, cutoff, &g);
      pet::build_periodic_nl(dp, n_atoms, g, ctx.nl, ctx.scr, ctx.s);
    } else {
      std::vector<int> b(n_atoms + 1, 0), e(n_atoms + 1, n_atoms);
      int *db = static_cast<int *>(ctx.b.ensure(sizeof(int) * (n_atoms + 1)));
      int *de = static_cast<int *>(ctx.e.ensure(sizeof(int) * (n_atoms + 1)));
      CUDA_CHECK(cudaMemcpyAsync(db, b.data(), sizeof(int) * (n_atoms + 1), cudaMemcpyHostToDevice, ctx.s));
      CUDA_CHECK(cudaMemcpyAsync(de, e.data(), sizeof(int) * (n_atoms + 1), cudaMemcpyHostToDevice, ctx.s));
      pet::build_open_nl(dp, db, de, n_atoms, cutoff, ctx.nl, ctx.scr, ctx.s);
    }
    const int64_t m = ctx.nl.n_edges;
    const int64_t k = m < cap ? m : cap;
    if (k > 0) {
      if (centers) CUDA_CHECK(cudaMemcpyAsync(centers, ctx.nl.center.ptr, 4 * k, cudaMemcpyDeviceToHost, ctx.s));
      if (neighbors) CUDA_CHECK(cudaMemcpyAsync(neighbors, ctx.nl.nbr.ptr, 4 * k, cudaMemcpyDeviceToHost, ctx.s));
      if (shifts) CUDA_CHECK(cudaMemcpyAsync(shifts, ctx.nl.shift.ptr, 12 * k, cudaMemcpyDeviceToHost, ctx.s));
      if (vectors) CUDA_CHECK(cudaMemcpyAsync(vectors, ctx.nl.vec.ptr, 12 * k, cudaMemcpyDeviceToHost, ctx.s));
      if (distances) CUDA_CHECK(cudaMemcpyAsync(distances, ctx.nl.dist.ptr, 4 * k, cudaMemcpyDeviceToHost, ctx.s));
    }
    CUDA_CHECK(cudaStreamSynchronize(ctx.s));
    clear_error();
    return m;
  } catch (const pet::Error &e) {
    set_error(std::string("Neighbour list failed: ") + e.what());
    return -static_cast<int64_t>(e.code);
  } catch (const std::exception &e) {
    set_error(std::string("Neighbour list failed: ") + e.what());
    return -MLIPCPP_ERROR_COMPUTATION;
  }
}

int64_t mlipcpp_b200_neighbor_list_noalloc(int32_t n_atoms, const float *d_positions, const float *cell,
                                           const bool *pbc, float cutoff, int64_t cap, int32_t *d_centers,
                                           int32_t *d_neighbors, int32_t *d_shifts, float *d_vectors,
                                           float *d_distances, void *stream) {
  if (n_atoms < 0 || cap < 0) {
    set_error("Invalid number of atoms or pair capacity");
    return -MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (!cell) {
    set_error("The no-allocation neighbour list needs a cell (open boundaries: mlipcpp_b200_neighbor_list)");
    return -MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if (!std::isfinite(cutoff) || cutoff <= 0.0f) {
    set_error("The cutoff must be finite and positive");
    return -MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  bool p[3] = {true, true, true};
  if (pbc) { p[0] = pbc[0]; p[1] = pbc[1]; p[2] = pbc[2]; }
  pet::GridParams g;
  pet::make_grid_params(cell, p, cutoff, &g);
  // size limits before any device work, so an oversized call touches nothing
  if (g.ns[0] > pet::kMaxSearchBins || g.ns[1] > pet::kMaxSearchBins || g.ns[2] > pet::kMaxSearchBins) {
    set_error("The cutoff spans more than " + std::to_string(pet::kMaxSearchBins) +
              " cell widths along one axis");
    return -MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  const int64_t nbins = static_cast<int64_t>(g.nb[0]) * g.nb[1] * g.nb[2];
  if (n_atoms > pet::kNoAllocMaxAtoms || nbins > pet::kNoAllocMaxBins) {
    set_error("The no-allocation neighbour list takes at most " + std::to_string(pet::kNoAllocMaxAtoms) +
              " atoms and " + std::to_string(pet::kNoAllocMaxBins) + " cutoff-sized bins (got " +
              std::to_string(n_atoms) + " atoms, " + std::to_string(nbins) + " bins)");
    return -MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  if ((n_atoms > 0 && !d_positions) ||
      (cap > 0 && (!d_centers || !d_neighbors || !d_shifts || !d_vectors || !d_distances))) {
    set_error("NULL device pointer");
    return -MLIPCPP_ERROR_NULL_POINTER;
  }
  if (!have_cuda_device()) {
    set_error("No CUDA device available (this backend has no CPU fallback)");
    return -MLIPCPP_ERROR_BACKEND;
  }
  try {
    const int64_t m = pet::build_periodic_nl_noalloc(d_positions, n_atoms, g, cap, d_centers, d_neighbors,
                                                     d_shifts, d_vectors, d_distances,
                                                     static_cast<cudaStream_t>(stream));
    clear_error();
    return m;
  } catch (const pet::Error &e) {
    set_error(std::string("Neighbour list failed: ") + e.what());
    return -static_cast<int64_t>(e.code);
  } catch (const std::exception &e) {
    set_error(std::string("Neighbour list failed: ") + e.what());
    return -MLIPCPP_ERROR_COMPUTATION;
  }
}

int64_t mlipcpp_b200_kernel_launches(void) { return pet::g_kernel_launches.load(); }

int64_t mlipcpp_b200_device_allocations(void) { return pet::g_device_allocations.load(); }

mlipcpp_error_t mlipcpp_b200_set_wait_bound_ns(uint64_t ns) {
  if (!have_cuda_device()) {
    set_error("No CUDA device available (this backend has no CPU fallback)");
    return MLIPCPP_ERROR_BACKEND;
  }
  try {
    pet::set_gemm_wait_bound_ns(ns);
  } catch (const pet::Error &e) {
    set_error(e.what());
    return static_cast<mlipcpp_error_t>(e.code);
  }
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_b200_inject_gemm_stall(void) {
  pet::inject_gemm_stall();
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_b200_set_device(int32_t device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    set_error("Invalid CUDA device ordinal");
    return MLIPCPP_ERROR_INVALID_PARAMETER;
  }
  pet::g_default_device = device;
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_b200_set_kernel_profiling(mlipcpp_model_t model, bool enable) {
  if (auto e = check_model(model)) return e;
  model->model->set_kernel_profiling(enable);
  model->model->reset_kernel_stats();
  clear_error();
  return MLIPCPP_OK;
}

mlipcpp_error_t mlipcpp_b200_kernel_stats(mlipcpp_model_t model, double stats[24]) {
  if (auto e = check_model(model)) return e;
  if (!stats) {
    set_error("NULL stats pointer");
    return MLIPCPP_ERROR_NULL_POINTER;
  }
  const pet::KernelStat *k = model->model->kernel_stats();
  for (int c = 0; c < pet::KC_COUNT; ++c) {
    stats[4 * c + 0] = static_cast<double>(k[c].launches);
    stats[4 * c + 1] = k[c].ms;
    stats[4 * c + 2] = k[c].flops;
    stats[4 * c + 3] = k[c].bytes;
  }
  clear_error();
  return MLIPCPP_OK;
}

}  // extern "C"
