/* C++ interface of the B200 PET backend: the mlipcpp::Predictor API
 * (replaces the reference's include/mlipcpp/mlipcpp.hpp:22-303 and its
 * implementation src/api/cpp/mlipcpp_cpp.cpp:102-500) as a header-only
 * wrapper over the C ABI in mlipcpp.h, so a C++ caller of the reference
 * compiles unchanged against this header and links libmlipcpp_b200.so.
 *
 * Same names, overloads and semantics:
 *  - predict(..., bool compute_forces) runs the gradient path, which also
 *    yields the stress of periodic systems (mlipcpp_cpp.cpp:157-169);
 *  - predict(..., const PredictOptions &) computes gradients only for
 *    forces or stress (and not with use_nc_forces), keeps only the
 *    requested outputs, and with fd_stress replaces the stress by the
 *    4th-order finite difference of the energy under symmetric Voigt strain
 *    (mlipcpp_cpp.cpp:174-302);
 *  - errors throw: std::invalid_argument for bad arguments, std::runtime_error
 *    for load and prediction failures (with the C API's last error message).
 * A Predictor is not thread-safe (one CUDA stream per model).  Requires
 * C++20 (std::span). */
#ifndef MLIPCPP_HPP
#define MLIPCPP_HPP

#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

#include <unistd.h>

#include "mlipcpp.h"

namespace mlipcpp {

class Predictor;

/* mlipcpp.hpp:31-41; same order as mlipcpp_backend_t's names. */
enum class Backend { Auto, CPU, CUDA, HIP, Metal, Vulkan, WebGPU, SYCL, CANN };

/* mlipcpp.hpp:46-57 */
struct Result {
  float energy = 0.0f;
  std::vector<float> forces;  // [n_atoms * 3] (fx, fy, fz)
  std::vector<float> stress;  // [6] Voigt (xx, yy, zz, yz, xz, xy), eV/A^3

  bool has_forces() const { return !forces.empty(); }
  bool has_stress() const { return !stress.empty(); }
  std::span<const float, 3> force(size_t i) const { return std::span<const float, 3>(forces.data() + i * 3, 3); }
};

/* mlipcpp.hpp:62-65.  `precision` is this backend's extension (the C
 * API's mlipcpp_precision_t: 0 = F32, 1 = F16 reduced precision). */
struct ModelOptions {
  Backend backend = Backend::Auto;
  float cutoff_override = 0.0f;  // used only when the GGUF has no pet.cutoff
  int precision = 0;
};

/* mlipcpp.hpp:81-98: one captured intermediate tensor. */
struct NodeActivation {
  int node_id = 0;
  std::string name;
  std::string dtype;
  std::vector<int64_t> shape;
  std::vector<uint8_t> data;
};

struct ActivationResult {
  Result prediction;
  std::vector<NodeActivation> activations;
};

/* mlipcpp.hpp:103-116 */
struct PredictOptions {
  bool compute_forces = true;
  bool compute_stress = false;
  bool use_nc_forces = false;  // forces / stress from the model's non-conservative heads
  bool fd_stress = false;      // stress by finite differences of the energy (12 predictions)
};

namespace detail {

inline mlipcpp_backend_t to_c(Backend b) {
  switch (b) {
    case Backend::Auto: return MLIPCPP_BACKEND_AUTO;
    case Backend::CPU: return MLIPCPP_BACKEND_CPU;
    case Backend::CUDA: return MLIPCPP_BACKEND_CUDA;
    case Backend::HIP: return MLIPCPP_BACKEND_HIP;
    case Backend::Metal: return MLIPCPP_BACKEND_METAL;
    case Backend::Vulkan: return MLIPCPP_BACKEND_VULKAN;
    case Backend::WebGPU: return MLIPCPP_BACKEND_WEBGPU;
    case Backend::SYCL: return MLIPCPP_BACKEND_SYCL;
    case Backend::CANN: return MLIPCPP_BACKEND_CANN;
  }
  return MLIPCPP_BACKEND_AUTO;
}

inline std::string last_error(mlipcpp_error_t code) {
  const char *m = mlipcpp_get_last_error();
  return std::string(m ? m : mlipcpp_error_string(code));
}

inline void check(mlipcpp_error_t code, const char *what) {
  if (code != MLIPCPP_OK) throw std::runtime_error(std::string(what) + ": " + last_error(code));
}

// Copies a result handle's outputs into a Result and frees the handle.
inline Result take(mlipcpp_result_t h, int32_t n_atoms) {
  struct Guard {
    mlipcpp_result_t h;
    ~Guard() { mlipcpp_result_free(h); }
  } guard{h};
  Result r;
  check(mlipcpp_result_get_energy(h, &r.energy), "Prediction failed");
  bool hf = false, hs = false;
  check(mlipcpp_result_has_forces(h, &hf), "Prediction failed");
  check(mlipcpp_result_has_stress(h, &hs), "Prediction failed");
  if (hf && n_atoms > 0) {
    r.forces.resize(static_cast<size_t>(n_atoms) * 3);
    check(mlipcpp_result_get_forces(h, r.forces.data(), n_atoms), "Prediction failed");
  }
  if (hs) {
    r.stress.resize(6);
    check(mlipcpp_result_get_stress(h, r.stress.data()), "Prediction failed");
  }
  return r;
}

}  // namespace detail

/* mlipcpp.hpp:132-250: RAII owner of one loaded model. */
class Predictor {
 public:
  explicit Predictor(const std::string &path, const ModelOptions &options = {}) { open(path, options); }

  /* Loads a GGUF image held in memory.  The C API loads from a path, so the
   * bytes go to a temporary file that is removed again after the load. */
  Predictor(const uint8_t *data, size_t size, const ModelOptions &options = {}) {
    if (!data || size == 0) throw std::invalid_argument("GGUF buffer must not be empty");
    const char *dir = std::getenv("TMPDIR");
    std::string path = std::string(dir && *dir ? dir : "/tmp") + "/mlipcpp_gguf_XXXXXX";
    const int fd = mkstemp(path.data());
    if (fd < 0) throw std::runtime_error("cannot create a temporary GGUF file in " + path);
    FILE *f = fdopen(fd, "wb");
    if (!f) {
      close(fd);
      std::remove(path.c_str());
      throw std::runtime_error("cannot write a temporary GGUF file: " + path);
    }
    const bool ok = std::fwrite(data, 1, size, f) == size;
    std::fclose(f);
    try {
      if (!ok) throw std::runtime_error("cannot write a temporary GGUF file: " + path);
      open(path, options);
    } catch (...) {
      std::remove(path.c_str());
      throw;
    }
    std::remove(path.c_str());
  }

  ~Predictor() {
    if (model_) mlipcpp_model_free(model_);
  }
  Predictor(Predictor &&o) noexcept : model_(std::exchange(o.model_, nullptr)) {}
  Predictor &operator=(Predictor &&o) noexcept {
    if (this != &o) {
      if (model_) mlipcpp_model_free(model_);
      model_ = std::exchange(o.model_, nullptr);
    }
    return *this;
  }
  Predictor(const Predictor &) = delete;
  Predictor &operator=(const Predictor &) = delete;

  float cutoff() const {
    float c = 0.0f;
    detail::check(mlipcpp_model_get_cutoff(model_, &c), "cutoff");
    return c;
  }

  std::string_view model_type() const { return "PET"; }

  /* Non-periodic system (mlipcpp_cpp.cpp:316-330). */
  Result predict(std::span<const float> positions, std::span<const int32_t> atomic_numbers,
                 bool compute_forces = true) {
    if (positions.size() != atomic_numbers.size() * 3)
      throw std::invalid_argument("positions.size() must be 3 * atomic_numbers.size()");
    return run(static_cast<int32_t>(atomic_numbers.size()), positions.data(), atomic_numbers.data(), nullptr,
               nullptr, compute_forces);
  }

  /* Periodic system (mlipcpp_cpp.cpp:332-354). */
  Result predict(std::span<const float> positions, std::span<const int32_t> atomic_numbers,
                 std::span<const float, 9> cell, std::array<bool, 3> pbc, bool compute_forces = true) {
    if (positions.size() != atomic_numbers.size() * 3)
      throw std::invalid_argument("positions.size() must be 3 * atomic_numbers.size()");
    return run(static_cast<int32_t>(atomic_numbers.size()), positions.data(), atomic_numbers.data(), cell.data(),
               pbc.data(), compute_forces);
  }

  /* Raw pointers; cell == nullptr: non-periodic; pbc == nullptr with a
   * cell: periodic along all three axes (mlipcpp_cpp.cpp:356-390). */
  Result predict(int32_t n_atoms, const float *positions, const int32_t *atomic_numbers,
                 const float *cell = nullptr, const bool *pbc = nullptr, bool compute_forces = true) {
    if (!positions || !atomic_numbers)
      throw std::invalid_argument("positions and atomic_numbers must not be null");
    return run(n_atoms, positions, atomic_numbers, cell, pbc, compute_forces);
  }

  /* Full options (mlipcpp_cpp.cpp:262-302, 455-486). */
  Result predict(int32_t n_atoms, const float *positions, const int32_t *atomic_numbers, const float *cell,
                 const bool *pbc, const PredictOptions &options) {
    if (!positions || !atomic_numbers)
      throw std::invalid_argument("positions and atomic_numbers must not be null");
    const bool flags[3] = {pbc ? pbc[0] : true, pbc ? pbc[1] : true, pbc ? pbc[2] : true};
    const mlipcpp_system_t sys{n_atoms, positions, atomic_numbers, cell, cell ? flags : nullptr};
    mlipcpp_predict_options_t o{options.compute_forces, options.compute_stress, options.use_nc_forces};
    mlipcpp_result_t h = nullptr;
    const mlipcpp_error_t rc = mlipcpp_predict_with_options(model_, &sys, &o, &h);
    if (rc != MLIPCPP_OK) throw std::runtime_error("Prediction failed: " + detail::last_error(rc));
    Result r = detail::take(h, n_atoms);
    if (options.compute_stress && options.fd_stress) r.stress = fd_stress(n_atoms, positions, atomic_numbers, cell, flags);
    return r;
  }

  /* Intermediate tensors exist only for "pet-graph" models
   * (mlipcpp_cpp.cpp:488-503); this backend serves the "pet" layout, so the
   * call always throws, as the reference does for that layout. */
  ActivationResult predict_with_activations(int32_t n_atoms, const float *positions,
                                            const int32_t *atomic_numbers, const float *cell = nullptr,
                                            const bool *pbc = nullptr) {
    (void)cell;
    (void)pbc;
    (void)n_atoms;
    if (!positions || !atomic_numbers)
      throw std::invalid_argument("positions and atomic_numbers must not be null");
    throw std::runtime_error("predict_with_activations is only supported for graph-based models (pet-graph)");
  }

 private:
  void open(const std::string &path, const ModelOptions &options) {
    mlipcpp_model_options_t o;
    mlipcpp_model_options_default(&o);
    o.backend = detail::to_c(options.backend);
    o.precision = options.precision ? MLIPCPP_PRECISION_F16 : MLIPCPP_PRECISION_F32;
    o.cutoff_override = options.cutoff_override;
    model_ = mlipcpp_model_create(&o);
    if (!model_) throw std::runtime_error("Failed to create a model handle");
    const mlipcpp_error_t rc = mlipcpp_model_load(model_, path.c_str());
    if (rc != MLIPCPP_OK) {
      const std::string msg = detail::last_error(rc);
      mlipcpp_model_free(model_);
      model_ = nullptr;
      throw std::runtime_error("Failed to load PET model from: " + path + " (" + msg + ")");
    }
  }

  Result run(int32_t n_atoms, const float *positions, const int32_t *atomic_numbers, const float *cell,
             const bool *pbc, bool compute_forces) {
    const bool flags[3] = {pbc ? pbc[0] : true, pbc ? pbc[1] : true, pbc ? pbc[2] : true};
    const mlipcpp_system_t sys{n_atoms, positions, atomic_numbers, cell, cell ? flags : nullptr};
    mlipcpp_result_t h = nullptr;
    const mlipcpp_error_t rc = mlipcpp_predict(model_, &sys, compute_forces, &h);
    if (rc != MLIPCPP_OK) throw std::runtime_error("Prediction failed: " + detail::last_error(rc));
    return detail::take(h, n_atoms);
  }

  /* 4th-order central difference of the energy in each symmetric Voigt
   * strain component, delta = 5e-3: sigma_k = [8 (E(+d) - E(-d)) -
   * (E(+2d) - E(-2d))] / (12 V d), with cell rows and positions mapped by
   * the strain matrix (mlipcpp_cpp.cpp:174-259).  Empty for open systems
   * and volumes below 1e-10. */
  std::vector<float> fd_stress(int32_t n, const float *pos, const int32_t *z, const float *cell,
                               const bool pbc[3], float delta = 5e-3f) {
    if (!cell) return {};
    auto m = [&](int i, int j) { return static_cast<double>(cell[3 * i + j]); };
    double vol = m(0, 0) * (m(1, 1) * m(2, 2) - m(1, 2) * m(2, 1)) - m(0, 1) * (m(1, 0) * m(2, 2) - m(1, 2) * m(2, 0)) +
                 m(0, 2) * (m(1, 0) * m(2, 1) - m(1, 1) * m(2, 0));
    vol = std::fabs(vol);
    if (vol < 1e-10) return {};
    std::vector<float> sp(static_cast<size_t>(n) * 3);
    float sc[9];
    auto energy_at = [&](int k, double scale) {
      float eta[6] = {0, 0, 0, 0, 0, 0};
      eta[k] = static_cast<float>(delta * scale);
      const double e[3][3] = {{1.0 + eta[0], 0.5 * eta[5], 0.5 * eta[4]},
                              {0.5 * eta[5], 1.0 + eta[1], 0.5 * eta[3]},
                              {0.5 * eta[4], 0.5 * eta[3], 1.0 + eta[2]}};
      for (int i = 0; i < 3; ++i)
        for (int a = 0; a < 3; ++a)
          sc[3 * i + a] = static_cast<float>(e[a][0] * cell[3 * i] + e[a][1] * cell[3 * i + 1] + e[a][2] * cell[3 * i + 2]);
      for (int32_t i = 0; i < n; ++i)
        for (int a = 0; a < 3; ++a)
          sp[3 * i + a] = static_cast<float>(e[a][0] * pos[3 * i] + e[a][1] * pos[3 * i + 1] + e[a][2] * pos[3 * i + 2]);
      return static_cast<double>(run(n, sp.data(), z, sc, pbc, false).energy);
    };
    std::vector<float> stress(6, 0.0f);
    for (int k = 0; k < 6; ++k) {
      const double ep1 = energy_at(k, 1.0), em1 = energy_at(k, -1.0);
      const double ep2 = energy_at(k, 2.0), em2 = energy_at(k, -2.0);
      stress[k] = static_cast<float>((8.0 * (ep1 - em1) - (ep2 - em2)) / (12.0 * vol * delta));
    }
    return stress;
  }

  mlipcpp_model_t model_ = nullptr;
};

/* mlipcpp.hpp:255-301 */
inline const char *version() { return mlipcpp_version(); }
inline void set_backend(Backend backend) { mlipcpp_set_backend(detail::to_c(backend)); }
inline const char *get_backend_name() { return mlipcpp_get_backend_name(); }
inline bool backend_is_gpu() { return mlipcpp_backend_is_gpu(); }
inline bool is_backend_available(Backend backend) { return mlipcpp_is_backend_available(detail::to_c(backend)); }
inline void suppress_logging() { mlipcpp_suppress_logging(); }

}  // namespace mlipcpp

#endif  // MLIPCPP_HPP
