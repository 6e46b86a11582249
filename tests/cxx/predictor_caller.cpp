// A C++ caller of mlipcpp::Predictor, written against the reference's
// interface (include/mlipcpp/mlipcpp.hpp): it compiles against
// include/mlipcpp.hpp and links libmlipcpp_b200.so unchanged.
//
//   predictor_caller                  API checks that need no GPU
//   predictor_caller MODEL XYZ_BIN    one prediction per overload; prints
//                                     energies, forces and stresses
// XYZ_BIN: int32 n, int32 periodic, float cell[9], float pos[3n], int32 z[n].
#include <cstdio>
#include <fstream>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "mlipcpp.hpp"

static int api_checks() {
  int bad = 0;
  if (std::string(mlipcpp::version()).size() < 5) ++bad;
  if (mlipcpp::is_backend_available(mlipcpp::Backend::CPU)) ++bad;  // no CPU fallback here
  mlipcpp::suppress_logging();
  try {
    mlipcpp::Predictor p("/nonexistent/model.gguf");
    ++bad;
  } catch (const std::runtime_error &e) {
    std::cout << "load error: " << e.what() << "\n";
  }
  std::cout << "api " << (bad ? "FAIL" : "OK") << "\n";
  return bad;
}

int main(int argc, char **argv) {
  if (argc < 3) return api_checks();
  std::ifstream in(argv[2], std::ios::binary);
  int32_t n = 0, periodic = 0;
  float cell[9];
  in.read(reinterpret_cast<char *>(&n), 4);
  in.read(reinterpret_cast<char *>(&periodic), 4);
  in.read(reinterpret_cast<char *>(cell), 36);
  std::vector<float> pos(3 * n);
  std::vector<int32_t> z(n);
  in.read(reinterpret_cast<char *>(pos.data()), 12 * n);
  in.read(reinterpret_cast<char *>(z.data()), 4 * n);
  if (!in) {
    std::cerr << "bad input\n";
    return 2;
  }
  mlipcpp::Predictor model(argv[1]);
  std::printf("cutoff %.6f type %s\n", model.cutoff(), std::string(model.model_type()).c_str());
  auto dump = [&](const char *tag, const mlipcpp::Result &r) {
    std::printf("%s energy %.9g forces %d stress %d\n", tag, r.energy, r.has_forces() ? 1 : 0,
                r.has_stress() ? 1 : 0);
    if (r.has_forces())
      for (int i = 0; i < n; ++i) {
        auto f = r.force(i);
        std::printf("%s F %.9g %.9g %.9g\n", tag, f[0], f[1], f[2]);
      }
    if (r.has_stress())
      std::printf("%s S %.9g %.9g %.9g %.9g %.9g %.9g\n", tag, r.stress[0], r.stress[1], r.stress[2],
                  r.stress[3], r.stress[4], r.stress[5]);
  };
  std::span<const float> ps(pos);
  std::span<const int32_t> zs(z);
  if (periodic) {
    dump("span", model.predict(ps, zs, std::span<const float, 9>(cell, 9), {true, true, true}, true));
    dump("raw", model.predict(n, pos.data(), z.data(), cell, nullptr, true));
    mlipcpp::PredictOptions o;
    o.compute_forces = false;
    o.compute_stress = true;
    dump("opts", model.predict(n, pos.data(), z.data(), cell, nullptr, o));
    o.fd_stress = true;
    dump("fd", model.predict(n, pos.data(), z.data(), cell, nullptr, o));
  } else {
    dump("span", model.predict(ps, zs, true));
    dump("raw", model.predict(n, pos.data(), z.data()));
  }
  try {
    model.predict(std::span<const float>(pos.data(), 3), zs, true);
    std::puts("size check FAIL");
    return 1;
  } catch (const std::invalid_argument &) {
    std::puts("size check OK");
  }
  return 0;
}
