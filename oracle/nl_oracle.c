/*
 * TEST INFRASTRUCTURE -- CPU oracle for the neighbour list.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this; the
 * product path never does.
 *
 * A plain-C restatement of mlip.cpp's cell-list neighbour search, written to be
 * bit-exact with it: same fp64 operation order, no FMA contraction (build with
 * -ffp-contract=off), same per-centre enumeration order.
 *
 *   Cell::compute_inverse ........ src/core/system.cpp:19-48  (f32 cofactors)
 *   CellGrid ctor ................ src/core/neighbor_list.cpp:38-66
 *   CellGrid::position_to_bin .... src/core/neighbor_list.cpp:68-80
 *   CellGrid::wrap_bin ........... src/core/neighbor_list.cpp:82-91
 *   CellGrid::insert_atom ........ src/core/neighbor_list.cpp:97-105 (head insert)
 *   CellGrid::relative_position .. src/core/neighbor_list.cpp:107-110
 *   build_non_periodic ........... src/core/neighbor_list.cpp:126-161
 *   build_periodic ............... src/core/neighbor_list.cpp:163-297
 *
 * Pinned bit-exactly against the reference sources compiled by
 * oracle/Makefile (oracle/_ref/libnl_ref.so) in tests/test_oracle_nl.py and
 * against the committed fixtures in tests/golden/.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct { double x, y, z; } v3;

static v3 v3_add(v3 a, v3 b) { v3 r = {a.x + b.x, a.y + b.y, a.z + b.z}; return r; }
static v3 v3_sub(v3 a, v3 b) { v3 r = {a.x - b.x, a.y - b.y, a.z - b.z}; return r; }
static v3 v3_scale(v3 a, double s) { v3 r = {a.x * s, a.y * s, a.z * s}; return r; }
static double v3_dot(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static v3 v3_cross(v3 a, v3 b) {
  v3 r = {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
  return r;
}

/* f32 cofactor inverse of a row-major lattice (rows are lattice vectors). */
void nlo_cell_inverse(const float m[9], float inv[9]) {
#define M(i, j) m[(i)*3 + (j)]
  float det = M(0, 0) * (M(1, 1) * M(2, 2) - M(2, 1) * M(1, 2)) -
              M(0, 1) * (M(1, 0) * M(2, 2) - M(1, 2) * M(2, 0)) +
              M(0, 2) * (M(1, 0) * M(2, 1) - M(1, 1) * M(2, 0));
  float invdet = 1.0f / det;
  inv[0] = (M(1, 1) * M(2, 2) - M(2, 1) * M(1, 2)) * invdet;
  inv[1] = (M(0, 2) * M(2, 1) - M(0, 1) * M(2, 2)) * invdet;
  inv[2] = (M(0, 1) * M(1, 2) - M(0, 2) * M(1, 1)) * invdet;
  inv[3] = (M(1, 2) * M(2, 0) - M(1, 0) * M(2, 2)) * invdet;
  inv[4] = (M(0, 0) * M(2, 2) - M(0, 2) * M(2, 0)) * invdet;
  inv[5] = (M(1, 0) * M(0, 2) - M(0, 0) * M(1, 2)) * invdet;
  inv[6] = (M(1, 0) * M(2, 1) - M(2, 0) * M(1, 1)) * invdet;
  inv[7] = (M(2, 0) * M(0, 1) - M(0, 0) * M(2, 1)) * invdet;
  inv[8] = (M(0, 0) * M(1, 1) - M(1, 0) * M(0, 1)) * invdet;
#undef M
}

typedef struct {
  v3 cv[3], bv[3];
  double inv[9];
  int pbc[3], nb[3], ns[3];
} grid_t;

static void grid_init(grid_t *g, const float cell[9], const int pbc[3], double cutoff) {
  float finv[9];
  nlo_cell_inverse(cell, finv);
  for (int i = 0; i < 3; ++i) {
    g->cv[i].x = cell[i * 3 + 0];
    g->cv[i].y = cell[i * 3 + 1];
    g->cv[i].z = cell[i * 3 + 2];
    g->pbc[i] = pbc[i] != 0;
  }
  for (int k = 0; k < 9; ++k) g->inv[k] = finv[k];
  v3 nrm[3] = {v3_cross(g->cv[1], g->cv[2]), v3_cross(g->cv[2], g->cv[0]),
               v3_cross(g->cv[0], g->cv[1])};
  double vol = fabs(v3_dot(g->cv[2], nrm[2]));
  for (int i = 0; i < 3; ++i) {
    double face = vol / sqrt(v3_dot(nrm[i], nrm[i]));
    int nb = (int)floor(face / cutoff);
    g->nb[i] = nb > 1 ? nb : 1;
    g->ns[i] = (int)ceil(cutoff * g->nb[i] / face);
    g->bv[i] = v3_scale(g->cv[i], 1.0 / g->nb[i]);
  }
}

static void grid_bin(const grid_t *g, v3 p, int b[3]) {
  for (int i = 0; i < 3; ++i) {
    double f = g->inv[0 * 3 + i] * p.x + g->inv[1 * 3 + i] * p.y + g->inv[2 * 3 + i] * p.z;
    b[i] = (int)floor(f * g->nb[i]);
  }
}

static int wrap(int idx, int n, int periodic) {
  if (periodic) {
    idx = idx % n;
    if (idx < 0) idx += n;
    return idx;
  }
  return idx < 0 ? 0 : (idx > n - 1 ? n - 1 : idx);
}

static v3 grid_rel(const grid_t *g, v3 p, const int b[3]) {
  return v3_sub(v3_sub(v3_sub(p, v3_scale(g->bv[0], b[0])), v3_scale(g->bv[1], b[1])),
                v3_scale(g->bv[2], b[2]));
}

typedef struct {
  int64_t n, cap;
  int32_t *centers, *neighbors, *shifts;
  float *vecs, *dists;
} out_t;

static void emit(out_t *o, int i, int j, const int s[3], v3 dr, double d2) {
  int64_t k = o->n++;
  if (k >= o->cap) return;
  if (o->centers) o->centers[k] = i;
  if (o->neighbors) o->neighbors[k] = j;
  if (o->shifts) { o->shifts[3 * k] = s[0]; o->shifts[3 * k + 1] = s[1]; o->shifts[3 * k + 2] = s[2]; }
  if (o->vecs) { o->vecs[3 * k] = (float)dr.x; o->vecs[3 * k + 1] = (float)dr.y; o->vecs[3 * k + 2] = (float)dr.z; }
  if (o->dists) o->dists[k] = (float)sqrt(d2);
}

static v3 load_pos(const float *pos, int i) {
  v3 p = {pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]};
  return p;
}

static void build_open(out_t *o, int n, const float *pos, float cutoff, int full, int self) {
  const float rc2 = cutoff * cutoff; /* f32 product, compared in f64 */
  static const int zero[3] = {0, 0, 0};
  for (int i = 0; i < n; ++i) {
    v3 pi = load_pos(pos, i);
    for (int j = 0; j < n; ++j) {
      if (!self && i == j) continue;
      if (!full && j <= i) continue;
      v3 dr = v3_sub(load_pos(pos, j), pi);
      double d2 = v3_dot(dr, dr);
      if (d2 < rc2 && d2 > 1e-16) emit(o, i, j, zero, dr, d2);
    }
  }
}

static void build_periodic(out_t *o, int n, const float *pos, const float cell[9],
                           const int pbc[3], float cutoff_f, int full) {
  if (n == 0) return;
  const double rc = cutoff_f, rc2 = rc * rc;
  grid_t g;
  grid_init(&g, cell, pbc, rc);
  int nbins = g.nb[0] * g.nb[1] * g.nb[2];
  int *head = (int *)malloc(sizeof(int) * nbins);
  int *next = (int *)malloc(sizeof(int) * (n > 0 ? n : 1));
  int *braw = (int *)malloc(sizeof(int) * 3 * (n > 0 ? n : 1));
  for (int b = 0; b < nbins; ++b) head[b] = -1;
  for (int i = 0; i < n; ++i) {
    int b[3];
    grid_bin(&g, load_pos(pos, i), b);
    for (int d = 0; d < 3; ++d) braw[3 * i + d] = b[d];
    int w[3];
    for (int d = 0; d < 3; ++d) w[d] = wrap(b[d], g.nb[d], g.pbc[d]);
    int idx = w[0] + g.nb[0] * (w[1] + g.nb[1] * w[2]);
    next[i] = head[idx];
    head[idx] = i;
  }
  for (int i = 0; i < n; ++i) {
    v3 pi = load_pos(pos, i);
    const int *ri = braw + 3 * i;
    int bi[3], wi[3];
    for (int d = 0; d < 3; ++d) {
      bi[d] = g.pbc[d] ? ri[d] : wrap(ri[d], g.nb[d], 0);
      wi[d] = wrap(ri[d], g.nb[d], g.pbc[d]);
    }
    v3 rel_i = grid_rel(&g, pi, bi);
    for (int dz = -g.ns[2]; dz <= g.ns[2]; ++dz) {
      int bz = wi[2] + dz;
      if (g.pbc[2]) bz = wrap(bz, g.nb[2], 1);
      else if (bz < 0 || bz >= g.nb[2]) continue;
      v3 oz = v3_scale(g.bv[2], dz);
      for (int dy = -g.ns[1]; dy <= g.ns[1]; ++dy) {
        int by = wi[1] + dy;
        if (g.pbc[1]) by = wrap(by, g.nb[1], 1);
        else if (by < 0 || by >= g.nb[1]) continue;
        v3 oyz = v3_add(oz, v3_scale(g.bv[1], dy));
        for (int dx = -g.ns[0]; dx <= g.ns[0]; ++dx) {
          int bx = wi[0] + dx;
          if (g.pbc[0]) bx = wrap(bx, g.nb[0], 1);
          else if (bx < 0 || bx >= g.nb[0]) continue;
          v3 off = v3_add(oyz, v3_scale(g.bv[0], dx));
          int same = (dx == 0 && dy == 0 && dz == 0);
          for (int j = head[bx + g.nb[0] * (by + g.nb[1] * bz)]; j >= 0; j = next[j]) {
            /* The reference skips the i == j same-image pair before its
             * self_interaction test, so that option never adds a pair here. */
            if (i == j && same) continue;
            const int *rj = braw + 3 * j;
            int bj[3];
            for (int d = 0; d < 3; ++d) bj[d] = g.pbc[d] ? rj[d] : wrap(rj[d], g.nb[d], 0);
            v3 dr = v3_add(v3_sub(grid_rel(&g, load_pos(pos, j), bj), rel_i), off);
            double d2 = v3_dot(dr, dr);
            if (!(d2 < rc2)) continue;
            if (!full) {
              if (j < i) continue;
              if (j == i && (dz < 0 || (dz == 0 && dy < 0) || (dz == 0 && dy == 0 && dx < 0)))
                continue;
            }
            int s[3], dl[3] = {dx, dy, dz};
            for (int d = 0; d < 3; ++d) s[d] = (ri[d] - rj[d] + dl[d]) / g.nb[d];
            emit(o, i, j, s, dr, d2);
          }
        }
      }
    }
  }
  free(head);
  free(next);
  free(braw);
}

/*
 * Full neighbour list in the reference's enumeration order.
 * cell == NULL selects the open-boundary O(N^2) search; otherwise pbc[3]
 * gives per-axis periodicity (NULL = all periodic).  Writes at most `cap`
 * pairs into the (optional) output arrays and returns the total number of
 * pairs, so a call with cap = 0 sizes the buffers.
 */
int64_t nlo_build(int n, const float *pos, const float *cell, const int *pbc, float cutoff,
                  int full_list, int self_interaction, int64_t cap, int32_t *centers,
                  int32_t *neighbors, int32_t *shifts, float *vecs, float *dists) {
  out_t o = {0, cap, centers, neighbors, shifts, vecs, dists};
  if (cell) {
    int p[3] = {1, 1, 1};
    if (pbc) { p[0] = pbc[0]; p[1] = pbc[1]; p[2] = pbc[2]; }
    build_periodic(&o, n, pos, cell, p, cutoff, full_list);
  } else {
    build_open(&o, n, pos, cutoff, full_list, self_interaction);
  }
  return o.n;
}

/* Bin grid parameters (n_bins[3], n_search[3]) for a cell and cutoff. */
void nlo_grid_shape(const float cell[9], const int pbc[3], float cutoff, int nb[3], int ns[3]) {
  grid_t g;
  int p[3] = {1, 1, 1};
  if (pbc) { p[0] = pbc[0]; p[1] = pbc[1]; p[2] = pbc[2]; }
  grid_init(&g, cell, p, (double)cutoff);
  for (int d = 0; d < 3; ++d) { nb[d] = g.nb[d]; ns[d] = g.ns[d]; }
}
