// TEST INFRASTRUCTURE -- C shim over the reference's own neighbour-list
// sources (src/core/neighbor_list.cpp, src/core/system.cpp), compiled as-is
// from the read-only reference tree by oracle/Makefile into
// oracle/_ref/libnl_ref.so.  It exists only to pin oracle/nl_oracle.c and the
// fixtures in tests/golden/ against the reference's real output.
#include "mlipcpp/neighbor_list.h"
#include "mlipcpp/system.h"
#include <cstdint>
#include <cstring>
#include <vector>

using namespace mlipcpp;

// Same contract as nlo_build() in nl_oracle.c: returns the pair count and
// writes at most `cap` pairs.  Calls NeighborListBuilder::build
// (src/core/neighbor_list.cpp:118-124) on an AtomicSystem built like the C
// API does (src/api/c/mlipcpp_api.cpp:438-460).
extern "C" int64_t nlref_build(int n, const float *pos, const float *cell,
                               const int *pbc, float cutoff, int full_list,
                               int self_interaction, int64_t cap,
                               int32_t *centers, int32_t *neighbors,
                               int32_t *shifts, float *vecs, float *dists) {
  Cell c;
  const Cell *cp = nullptr;
  if (cell) {
    float lat[3][3];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) lat[i][j] = cell[i * 3 + j];
    bool p[3] = {true, true, true};
    if (pbc) { p[0] = pbc[0]; p[1] = pbc[1]; p[2] = pbc[2]; }
    c = Cell(lat, p[0], p[1], p[2]);
    cp = &c;
  }
  std::vector<int32_t> z(n > 0 ? n : 1, 0); // species do not affect the list
  AtomicSystem sys(n, pos, z.data(), cp);
  NeighborListOptions opt;
  opt.cutoff = cutoff;
  opt.full_list = full_list != 0;
  opt.self_interaction = self_interaction != 0;
  NeighborList nl = NeighborListBuilder(opt).build(sys);
  int64_t m = nl.num_pairs();
  for (int64_t k = 0; k < m && k < cap; ++k) {
    if (centers) centers[k] = nl.centers[k];
    if (neighbors) neighbors[k] = nl.neighbors[k];
    if (shifts) std::memcpy(shifts + 3 * k, nl.cell_shifts[k].data(), 12);
    if (vecs) std::memcpy(vecs + 3 * k, nl.edge_vectors[k].data(), 12);
    if (dists) dists[k] = nl.distances[k];
  }
  return m;
}

// f32 Cell::compute_inverse (src/core/system.cpp:19-48) for pinning.
extern "C" void nlref_cell_inverse(const float m[9], float inv[9]) {
  float lat[3][3];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) lat[i][j] = m[i * 3 + j];
  Cell c(lat, true, true, true);
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) inv[i * 3 + j] = c.inverse[i][j];
}
