/*
 * npa_oracle.c -- CPU restatement of the burn_automata NPA rollout path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); the CUDA
 * product never calls it.  See npa_oracle.h for the list of reference files.
 *
 * f32 semantics follow the reference's Rust code exactly:
 *   - built with -ffp-contract=off: a*b+c is a rounded multiply then a rounded
 *     add, as rustc emits it;
 *   - sums run left to right in the reference's loop order;
 *   - f32::powi(n) is LLVM's binary exponentiation (ora_powi below);
 *   - `x as isize` saturates and maps NaN to 0 (f2i64_sat);
 *   - f32::ln_1p / exp / tanh / sqrt call the same libm entry points rustc
 *     binds (log1pf, expf, tanhf, sqrtf);
 *   - f32::max / f32::clamp keep Rust's NaN behaviour.
 * Per-particle loops run under OpenMP like the reference's rayon loops; each
 * particle's arithmetic is independent of the thread schedule, so results
 * are deterministic.  The hashgrid build stays serial, as in the reference.
 */
#include "npa_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BOUNDARY_PERIODIC 0
#define BOUNDARY_CLAMPED 1
#define MODE_GRID 0
#define MODE_PARTICLE 1

static const float ORA_PI = 3.14159274101257324219f; /* std::f32::consts::PI */

static int g_threads = 0;
/* 0: f32::ln_1p as the reference binds it (the host libm's log1pf);
 * 1: ln(1 + x) evaluated in f64 and rounded once to f32, the CUDA library's
 *    choice.  Mode 1 predicts the device's arithmetic exactly, so the GPU
 *    can be compared bit for bit even with log-normalisation on; mode 0 is
 *    the reference and the default. */
static int g_log1p_mode = 0;

void ora_set_threads(int threads) { g_threads = threads; }
void ora_set_log1p_mode(int mode) { g_log1p_mode = mode; }

static float ln_1p_f32(float x) {
  return g_log1p_mode ? (float)log1p((double)x) : log1pf(x);
}

/* f32::ln_1p as the reference binds it (the host libm's log1pf), elementwise. */
void ora_ln_1p(const float* x, int64_t count, float* out) {
#pragma omp parallel for schedule(static) num_threads(ora_get_threads())
  for (int64_t i = 0; i < count; ++i) out[i] = log1pf(x[i]);
}

int ora_get_threads(void) {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* Rust scalar semantics                                                     */
/* ------------------------------------------------------------------------ */

/* `f as isize` (saturating, NaN -> 0). */
static int64_t f2i64_sat(float x) {
  if (x != x) return 0;
  if (x >= 9223372036854775808.0f) return INT64_MAX;
  if (x <= -9223372036854775808.0f) return INT64_MIN;
  return (int64_t)x;
}

/* f32::powi with a constant exponent: LLVM expands it by binary
 * exponentiation, multiplying the running product by successive squares. */
static float ora_powi(float x, int n) {
  float result = 1.0f;
  int have = 0;
  float square = x;
  while (n) {
    if (n & 1) {
      result = have ? result * square : square;
      have = 1;
    }
    n >>= 1;
    if (n) square = square * square;
  }
  return have ? result : 1.0f;
}

/* f32::clamp (min <= max asserted by the caller's validation). */
static float clampf_rs(float v, float lo, float hi) {
  if (v < lo) v = lo;
  if (v > hi) v = hi;
  return v;
}

/* f32::max: returns the other operand when one is NaN. */
static float maxf_rs(float a, float b) { return fmaxf(a, b); }

static int64_t rem_euclid_i64(int64_t a, int64_t b) {
  int64_t r = a % b;
  return r < 0 ? r + b : r;
}

static int64_t clamp_i64(int64_t v, int64_t lo, int64_t hi) {
  if (v < lo) return lo;
  if (v > hi) return hi;
  return v;
}

static int64_t wrapping_add_i64(int64_t a, int64_t b) {
  return (int64_t)((uint64_t)a + (uint64_t)b);
}

/* RecipFinite::recip_finite (reference/kernels.rs:156-165). */
static float recip_finite(float x) {
  if (fabsf(x) <= 1e-20f || !isfinite(x)) return 0.0f;
  return 1.0f / x;
}

/* ------------------------------------------------------------------------ */
/* HashGridConfig (config.rs:65-93)                                          */
/* ------------------------------------------------------------------------ */

int ora_grid_validate(const ora_grid_config* cfg) {
  if (!cfg) return ORA_ERR_INVALID_ARGUMENT;
  if (!(cfg->dim == 2 || cfg->dim == 3)) return ORA_ERR_INVALID_DIM;
  if (!isfinite(cfg->eps) || cfg->eps <= 0.0f) return ORA_ERR_INVALID_EPS;
  if (!(cfg->mode == MODE_GRID || cfg->mode == MODE_PARTICLE)) return ORA_ERR_INVALID_ARGUMENT;
  if (!(cfg->boundary == BOUNDARY_PERIODIC || cfg->boundary == BOUNDARY_CLAMPED))
    return ORA_ERR_INVALID_ARGUMENT;
  for (int axis = 0; axis < cfg->dim; ++axis) {
    int64_t s = cfg->grid_size[axis];
    if (s <= 0) return ORA_ERR_INVALID_GRID_SIZE;
    if (cfg->mode == MODE_PARTICLE && (s & (s - 1)) != 0)
      return ORA_ERR_PARTICLE_MODE_REQUIRES_POW2;
  }
  return ORA_OK;
}

int64_t ora_cell_count(const ora_grid_config* cfg) {
  int64_t c = 1;
  for (int axis = 0; axis < cfg->dim; ++axis) c *= cfg->grid_size[axis];
  return c;
}

/* ------------------------------------------------------------------------ */
/* Cell math (hashgrid.rs:71-193)                                            */
/* ------------------------------------------------------------------------ */

/* mix_coord (hashgrid.rs:155-163): `value as i32 as u32` keeps the low 32 bits. */
static uint32_t mix_coord(int64_t value, uint32_t salt) {
  uint32_t x = ((uint32_t)(uint64_t)value) ^ salt;
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

/* particle_cell_hash (hashgrid.rs:147-153). */
static int64_t particle_cell_hash(const int64_t coords[3], const ora_grid_config* cfg,
                                  int64_t cell_count) {
  uint32_t h = mix_coord(coords[0], 0x9e3779b9u) ^ mix_coord(coords[1], 0x85ebca6bu);
  if (cfg->dim == 3) h ^= mix_coord(coords[2], 0xc2b2ae35u);
  return (int64_t)((uint64_t)h % (uint64_t)cell_count);
}

/* Grid-mode cell of one coordinate (hashgrid.rs:80-90 / :106-116). */
static int64_t grid_axis_cell(const ora_grid_config* cfg, int axis, float coordinate) {
  int64_t size = cfg->grid_size[axis];
  float extent = cfg->eps * (float)size;
  float half = extent * 0.5f;
  int64_t cell = f2i64_sat(floorf((coordinate + half) / cfg->eps));
  if (cfg->boundary == BOUNDARY_PERIODIC) return rem_euclid_i64(cell, size);
  return clamp_i64(cell, 0, size - 1);
}

/* cell_coords_for_position (hashgrid.rs:98-121). */
static void cell_coords_for_position(const ora_grid_config* cfg, const float* p,
                                     int64_t out[3]) {
  out[0] = out[1] = out[2] = 0;
  for (int axis = 0; axis < cfg->dim; ++axis) {
    if (cfg->mode == MODE_PARTICLE) {
      out[axis] = f2i64_sat(floorf(p[axis] / cfg->eps));
    } else {
      out[axis] = grid_axis_cell(cfg, axis, p[axis]);
    }
  }
}

/* cell_for_position (hashgrid.rs:71-96). */
static int64_t cell_for_position(const ora_grid_config* cfg, const float* p,
                                 int64_t cell_count) {
  int64_t coords[3];
  cell_coords_for_position(cfg, p, coords);
  if (cfg->mode == MODE_PARTICLE) return particle_cell_hash(coords, cfg, cell_count);
  uint64_t stride = 1, hash = 0;
  for (int axis = 0; axis < cfg->dim; ++axis) {
    hash += (uint64_t)coords[axis] * stride;
    stride *= (uint64_t)cfg->grid_size[axis];
  }
  return (int64_t)hash;
}

int64_t ora_cell_for_position(const ora_grid_config* cfg, const float* pos4) {
  return cell_for_position(cfg, pos4, ora_cell_count(cfg));
}

/* cell_index_from_coords (hashgrid.rs:123-145); returns -1 for None. */
static int64_t cell_index_from_coords(const ora_grid_config* cfg, const int64_t coords[3],
                                      int64_t cell_count) {
  if (cfg->mode == MODE_PARTICLE) return particle_cell_hash(coords, cfg, cell_count);
  uint64_t stride = 1, hash = 0;
  for (int axis = 0; axis < cfg->dim; ++axis) {
    int64_t size = cfg->grid_size[axis];
    int64_t cell;
    if (cfg->boundary == BOUNDARY_PERIODIC) {
      cell = rem_euclid_i64(coords[axis], size);
    } else {
      if (coords[axis] < 0 || coords[axis] >= size) return -1;
      cell = coords[axis];
    }
    hash += (uint64_t)cell * stride;
    stride *= (uint64_t)size;
  }
  return (int64_t)hash;
}

/* neighbor_delta (hashgrid.rs:165-181). */
static void neighbor_delta(const float* lhs, const float* rhs, const ora_grid_config* cfg,
                           float delta[4]) {
  delta[0] = delta[1] = delta[2] = delta[3] = 0.0f;
  for (int axis = 0; axis < cfg->dim; ++axis) {
    float d = rhs[axis] - lhs[axis];
    if (cfg->boundary == BOUNDARY_PERIODIC) {
      float extent = (float)cfg->grid_size[axis] * cfg->eps;
      float half = extent * 0.5f;
      if (d > half) {
        d -= extent;
      } else if (d < -half) {
        d += extent;
      }
    }
    delta[axis] = d;
  }
}

/* wrap_position (hashgrid.rs:183-193); f32::rem_euclid = fmod + fix-up. */
static void wrap_position(float p[4], const ora_grid_config* cfg) {
  if (cfg->boundary != BOUNDARY_PERIODIC) return;
  for (int axis = 0; axis < cfg->dim; ++axis) {
    float extent = (float)cfg->grid_size[axis] * cfg->eps;
    float half = extent * 0.5f;
    float v = p[axis] + half;
    float r = fmodf(v, extent);
    if (r < 0.0f) r = r + fabsf(extent);
    p[axis] = r - half;
  }
}

/* ------------------------------------------------------------------------ */
/* build_hashgrid (hashgrid.rs:16-69): serial two-pass counting sort          */
/* ------------------------------------------------------------------------ */

int ora_build_hashgrid(const ora_grid_config* cfg, const float* positions, int64_t batch,
                       int64_t n, int64_t* bin_offsets, int64_t* permutation,
                       int64_t* inverse_permutation) {
  int st = ora_grid_validate(cfg);
  if (st) return st;
  if (batch < 0 || n < 0) return ORA_ERR_INVALID_ARGUMENT;
  int64_t cells = ora_cell_count(cfg);
  int64_t total_bins = batch * cells;
  int64_t* counts = (int64_t*)calloc((size_t)(total_bins > 0 ? total_bins : 1), sizeof(int64_t));
  int64_t* heads = (int64_t*)malloc((size_t)(total_bins + 1) * sizeof(int64_t));
  if (!counts || !heads) {
    free(counts);
    free(heads);
    return ORA_ERR_INVALID_ARGUMENT;
  }
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t p = 0; p < n; ++p) {
      int64_t idx = b * n + p;
      counts[b * cells + cell_for_position(cfg, positions + 4 * idx, cells)] += 1;
    }
  bin_offsets[0] = 0;
  for (int64_t i = 0; i < total_bins; ++i) bin_offsets[i + 1] = bin_offsets[i] + counts[i];
  memcpy(heads, bin_offsets, (size_t)(total_bins + 1) * sizeof(int64_t));
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t p = 0; p < n; ++p) {
      int64_t idx = b * n + p;
      int64_t bin = b * cells + cell_for_position(cfg, positions + 4 * idx, cells);
      int64_t dst = heads[bin]++;
      permutation[dst] = p;
      inverse_permutation[idx] = dst - b * n;
    }
  free(counts);
  free(heads);
  return ORA_OK;
}

/* ------------------------------------------------------------------------ */
/* Neighbour walk (reference/neighbor.rs:3-44)                               */
/* ------------------------------------------------------------------------ */

typedef struct {
  const ora_grid_config* cfg;
  const float* positions;
  const int64_t* bin_offsets;
  const int64_t* permutation;
  int64_t n, cells;
  float eps2;
} walk_ctx;

/* Visits every j with r2 < eps^2 in dz, dy, dx cell order and ascending
 * permutation order inside a bin, calling VISIT(j, delta, r2). */
#define FOR_EACH_NEIGHBOR(CTX, IDX, J, DELTA, R2, ...)                                   \
  do {                                                                                   \
    const walk_ctx* w__ = (CTX);                                                         \
    int64_t batch__ = (IDX) / w__->n;                                                    \
    int64_t base__ = batch__ * w__->n;                                                   \
    const float* pi__ = w__->positions + 4 * (IDX);                                      \
    int64_t center__[3];                                                                 \
    cell_coords_for_position(w__->cfg, pi__, center__);                                  \
    int zmin__ = w__->cfg->dim == 3 ? -1 : 0, zmax__ = w__->cfg->dim == 3 ? 1 : 0;       \
    for (int dz__ = zmin__; dz__ <= zmax__; ++dz__)                                      \
      for (int dy__ = -1; dy__ <= 1; ++dy__)                                             \
        for (int dx__ = -1; dx__ <= 1; ++dx__) {                                         \
          int64_t coords__[3] = {wrapping_add_i64(center__[0], dx__),                    \
                                 wrapping_add_i64(center__[1], dy__),                    \
                                 wrapping_add_i64(center__[2], dz__)};                   \
          int64_t cell__ = cell_index_from_coords(w__->cfg, coords__, w__->cells);       \
          if (cell__ < 0) continue;                                                      \
          int64_t bin__ = batch__ * w__->cells + cell__;                                 \
          for (int64_t q__ = w__->bin_offsets[bin__]; q__ < w__->bin_offsets[bin__ + 1]; \
               ++q__) {                                                                  \
            int64_t J = base__ + w__->permutation[q__];                                  \
            const float* pj__ = w__->positions + 4 * J;                                  \
            if (w__->cfg->mode == MODE_PARTICLE) {                                       \
              int64_t cj__[3];                                                           \
              cell_coords_for_position(w__->cfg, pj__, cj__);                            \
              if (cj__[0] != coords__[0] || cj__[1] != coords__[1] ||                    \
                  cj__[2] != coords__[2])                                                \
                continue;                                                                \
            }                                                                            \
            float DELTA[4];                                                              \
            neighbor_delta(pi__, pj__, w__->cfg, DELTA);                                 \
            float R2 = 0.0f;                                                             \
            for (int a__ = 0; a__ < w__->cfg->dim; ++a__) R2 = R2 + DELTA[a__] * DELTA[a__]; \
            if (R2 < w__->eps2) {                                                        \
              __VA_ARGS__                                                                \
            }                                                                            \
          }                                                                              \
        }                                                                                \
  } while (0)

/* ------------------------------------------------------------------------ */
/* SPH kernels (reference/kernels.rs)                                        */
/* ------------------------------------------------------------------------ */

typedef struct {
  float eps, eps2;
  float poly6_norm;  /* smoothing_poly6_normalization, kernels.rs:128-134 */
  float spiky_norm;  /* gradient_spiky_normalization, kernels.rs:136-142 */
  int dim;
} sph_consts;

static sph_consts make_sph(const ora_grid_config* cfg) {
  sph_consts k;
  k.eps = cfg->eps;
  k.eps2 = cfg->eps * cfg->eps;
  k.dim = cfg->dim;
  if (cfg->dim == 2) {
    k.poly6_norm = 4.0f / (ORA_PI * ora_powi(cfg->eps, 8));
    k.spiky_norm = 10.0f / (ORA_PI * ora_powi(cfg->eps, 5));
  } else {
    k.poly6_norm = 315.0f / (64.0f * ORA_PI * ora_powi(cfg->eps, 9));
    k.spiky_norm = 15.0f / (ORA_PI * ora_powi(cfg->eps, 6));
  }
  return k;
}

/* smoothing_poly6_kernel (kernels.rs:53-60). */
static float poly6(float r2, const sph_consts* k) {
  if (r2 >= k->eps2) return 0.0f;
  float x = k->eps2 - r2;
  return k->poly6_norm * x * x * x;
}

/* spiky_gradient_kernel (kernels.rs:81-98). */
static void spiky(const float delta[4], float r2, const sph_consts* k, float coeff,
                  float out[4]) {
  out[0] = out[1] = out[2] = out[3] = 0.0f;
  if (r2 <= 0.0f || r2 >= k->eps2) return;
  float r = sqrtf(r2);
  float t = k->eps - r;
  float mag = coeff * k->spiky_norm * 3.0f * (t * t) / r;
  for (int a = 0; a < k->dim; ++a) out[a] = mag * delta[a];
}

/* safe_inverse_symmetric (kernels.rs:3-51). */
static void safe_inverse_symmetric(const float* m, int dim, float out[9]) {
  const float TOL = 1e-3f;
  for (int i = 0; i < 9; ++i) out[i] = 0.0f;
  if (dim == 2) {
    float a = m[0], b = m[1], d = m[3];
    float det = a * d - b * b;
    if (fabsf(det) < TOL) {
      out[0] = 1.0f;
      out[3] = 1.0f;
      return;
    }
    float inv_det = 1.0f / det;
    out[0] = d * inv_det;
    out[1] = -b * inv_det;
    out[2] = -b * inv_det;
    out[3] = a * inv_det;
    return;
  }
  float a = m[0], b = m[1], c = m[2], d = m[4], e = m[5], f = m[8];
  float t1 = d * f - e * e;
  float t2 = c * e - b * f;
  float t3 = b * e - c * d;
  float det = a * t1 + b * t2 + c * t3;
  if (fabsf(det) < TOL) {
    out[0] = 1.0f;
    out[4] = 1.0f;
    out[8] = 1.0f;
    return;
  }
  float inv_det = 1.0f / det;
  out[0] = t1 * inv_det;
  out[1] = t2 * inv_det;
  out[2] = t3 * inv_det;
  out[3] = t2 * inv_det;
  out[4] = (a * f - c * c) * inv_det;
  out[5] = (b * c - a * e) * inv_det;
  out[6] = t3 * inv_det;
  out[7] = (b * c - a * e) * inv_det;
  out[8] = (a * d - b * b) * inv_det;
}

/* log_normalize_vector (normalize.rs:60-69). */
static void log_normalize_vector(float* v, int len) {
  float s = 0.0f;
  for (int i = 0; i < len; ++i) s = s + v[i] * v[i];
  const float e = 1.0e-6f;
  float norm = maxf_rs(sqrtf(s + e * e), e);
  float scale = ln_1p_f32(norm) / norm;
  for (int i = 0; i < len; ++i) v[i] = v[i] * scale;
}

/* ------------------------------------------------------------------------ */
/* Perception (reference/forward.rs)                                         */
/* ------------------------------------------------------------------------ */

int64_t ora_feature_dims(const ora_grid_config* cfg, const ora_perception_options* opt,
                         int64_t c) {
  return c * 2 + (opt->state_grad ? c * cfg->dim : 0) + (opt->density_grad ? cfg->dim : 0) +
         (opt->position_features ? cfg->dim : 0);
}

static int check_shapes_basic(int64_t batch, int64_t n, int64_t c) {
  if (batch < 0 || n < 0 || c < 0) return ORA_ERR_INVALID_ARGUMENT;
  return ORA_OK;
}

int ora_perceive(const ora_grid_config* cfg, const ora_perception_options* opt,
                 const float* positions, const float* states, int64_t batch, int64_t n,
                 int64_t c, float* features, float* density_out, float* blurred_out,
                 float* sgrad_out, float* dgrad_out) {
  int st = check_shapes_basic(batch, n, c);
  if (st) return st;
  st = ora_grid_validate(cfg);
  if (st) return st;
  const int dim = cfg->dim;
  const int64_t total = batch * n;
  const int64_t cells = ora_cell_count(cfg);
  int64_t* offsets = (int64_t*)malloc((size_t)(batch * cells + 1) * sizeof(int64_t));
  int64_t* perm = (int64_t*)malloc((size_t)(total > 0 ? total : 1) * sizeof(int64_t));
  int64_t* inv = (int64_t*)malloc((size_t)(total > 0 ? total : 1) * sizeof(int64_t));
  float* density = (float*)malloc((size_t)(total > 0 ? total : 1) * sizeof(float));
  float* blurred = (float*)calloc((size_t)(total * c > 0 ? total * c : 1), sizeof(float));
  float* sgrad = (float*)calloc((size_t)(total * c * dim > 0 ? total * c * dim : 1), sizeof(float));
  float* dgrad = (float*)calloc((size_t)(total * dim > 0 ? total * dim : 1), sizeof(float));
  if (!offsets || !perm || !inv || !density || !blurred || !sgrad || !dgrad) {
    st = ORA_ERR_INVALID_ARGUMENT;
    goto done;
  }
  st = ora_build_hashgrid(cfg, positions, batch, n, offsets, perm, inv);
  if (st) goto done;

  walk_ctx w = {cfg, positions, offsets, perm, n, cells, cfg->eps * cfg->eps};
  sph_consts k = make_sph(cfg);

  /* density (forward.rs:145-160) */
#pragma omp parallel for schedule(dynamic, 256) num_threads(ora_get_threads())
  for (int64_t idx = 0; idx < total; ++idx) {
    float rho = 0.0f;
    FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, { (void)j; (void)delta; rho = rho + poly6(r2, &k); });
    density[idx] = rho;
  }

  const int both = opt->state_grad && opt->density_grad;
  const int hybrid = opt->hybrid_state_gradient;
  /* Second pass.  second_pass_particle (forward.rs:249-295) when both grads are
   * on; otherwise blur_state (:162), compute_state_gradient (:297),
   * moment_matrix (:357) and compute_density_gradient (:335).  Those separate
   * walks visit neighbours in the same order, so one walk that updates every
   * accumulator yields the same per-accumulator sums. */
#pragma omp parallel for schedule(dynamic, 256) num_threads(ora_get_threads())
  for (int64_t idx = 0; idx < total; ++idx) {
    float* blur = blurred + idx * c;
    float* sg = sgrad + idx * c * dim;
    float* dg = dgrad + idx * dim;
    float moment[9] = {0};
    const float* si = states + idx * c;
    FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
      float vol = recip_finite(density[j]);
      float smooth = poly6(r2, &k);
      const float* sj = states + j * c;
      if (both) {
        for (int64_t ch = 0; ch < c; ++ch) blur[ch] = blur[ch] + sj[ch] * smooth * vol;
      } else {
        float wgt = smooth * vol;
        for (int64_t ch = 0; ch < c; ++ch) blur[ch] = blur[ch] + sj[ch] * wgt;
      }
      if (j != idx) {
        if (opt->density_grad) {
          float g1[4];
          spiky(delta, r2, &k, 1.0f, g1);
          for (int a = 0; a < dim; ++a) dg[a] = dg[a] + g1[a];
        }
        if (opt->state_grad) {
          float gv[4];
          spiky(delta, r2, &k, vol, gv);
          for (int64_t ch = 0; ch < c; ++ch) {
            float diff = sj[ch] - si[ch];
            for (int a = 0; a < dim; ++a) sg[ch * dim + a] = sg[ch * dim + a] + diff * gv[a];
          }
          if (hybrid)
            for (int r = 0; r < dim; ++r)
              for (int col = 0; col < dim; ++col)
                moment[r * dim + col] = moment[r * dim + col] + delta[r] * gv[col];
        }
      }
    });
    if (opt->state_grad) {
      if (hybrid) {
        /* apply_moment_correction (normalize.rs:93-118) */
        float inv_m[9];
        safe_inverse_symmetric(moment, dim, inv_m);
        for (int64_t ch = 0; ch < c; ++ch) {
          float corrected[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int oa = 0; oa < dim; ++oa)
            for (int ia = 0; ia < dim; ++ia)
              corrected[oa] = corrected[oa] + sg[ch * dim + ia] * inv_m[ia * dim + oa];
          for (int a = 0; a < dim; ++a) sg[ch * dim + a] = corrected[a];
        }
      }
      /* normalize_state_gradient (normalize.rs:5-30) */
      float eps0 = maxf_rs(opt->eps0, 1.17549435e-38f);
      float scale = opt->scale_equivariance ? cfg->eps / eps0 : 1.0f;
      for (int64_t ch = 0; ch < c; ++ch) {
        for (int a = 0; a < dim; ++a) sg[ch * dim + a] = sg[ch * dim + a] * scale;
        if (opt->log_norm_grad) log_normalize_vector(sg + ch * dim, dim);
      }
    }
    if (opt->density_grad) {
      /* normalize_density_gradient (normalize.rs:32-58) */
      float eps0 = maxf_rs(opt->eps0, 1.17549435e-38f);
      float a_scale = opt->scale_equivariance ? ora_powi(cfg->eps / eps0, 1 + dim) : 1.0f;
      float b_scale = opt->particle_density_equivariance ? 1.0f / (float)(n > 1 ? n : 1) : 1.0f;
      float scale = a_scale * b_scale;
      for (int a = 0; a < dim; ++a) dg[a] = dg[a] * scale;
      if (opt->log_norm_density_grad) log_normalize_vector(dg, dim);
    }
  }

  /* feature assembly (forward.rs:100-133) */
  {
    const int64_t fd = ora_feature_dims(cfg, opt, c);
#pragma omp parallel for schedule(static) num_threads(ora_get_threads())
    for (int64_t idx = 0; idx < total; ++idx) {
      float* f = features + idx * fd;
      int64_t cur = 0;
      for (int64_t ch = 0; ch < c; ++ch) f[cur++] = states[idx * c + ch];
      for (int64_t ch = 0; ch < c; ++ch) f[cur++] = blurred[idx * c + ch];
      if (opt->state_grad)
        for (int64_t g = 0; g < c * dim; ++g) f[cur++] = sgrad[idx * c * dim + g];
      if (opt->density_grad)
        for (int a = 0; a < dim; ++a) f[cur++] = dgrad[idx * dim + a];
      if (opt->position_features)
        for (int a = 0; a < dim; ++a) f[cur++] = positions[4 * idx + a];
    }
  }
  if (density_out) memcpy(density_out, density, (size_t)total * sizeof(float));
  if (blurred_out) memcpy(blurred_out, blurred, (size_t)(total * c) * sizeof(float));
  if (sgrad_out && opt->state_grad) memcpy(sgrad_out, sgrad, (size_t)(total * c * dim) * sizeof(float));
  if (dgrad_out && opt->density_grad) memcpy(dgrad_out, dgrad, (size_t)(total * dim) * sizeof(float));

done:
  free(offsets);
  free(perm);
  free(inv);
  free(density);
  free(blurred);
  free(sgrad);
  free(dgrad);
  return st;
}

/* Determinant of each particle's hybrid moment matrix M_i = sum over j != i of
 * delta (x) spiky(V_j) (moment_matrix, forward.rs:357-382; V_j =
 * recip_finite(density_j)), computed as safe_inverse_symmetric
 * (kernels.rs:3-51) computes it before comparing |det| with its 1e-3 switch.
 * Test infrastructure: the parity tests count particles whose det lies near
 * the switch, where a last-bit difference in M can flip the branch. */
int ora_moment_det(const ora_grid_config* cfg, const float* positions, int64_t batch, int64_t n,
                   float* det_out) {
  int st = check_shapes_basic(batch, n, 0);
  if (st) return st;
  st = ora_grid_validate(cfg);
  if (st) return st;
  const int dim = cfg->dim;
  const int64_t total = batch * n;
  const int64_t cells = ora_cell_count(cfg);
  int64_t* offsets = (int64_t*)malloc((size_t)(batch * cells + 1) * sizeof(int64_t));
  int64_t* perm = (int64_t*)malloc((size_t)(total > 0 ? total : 1) * sizeof(int64_t));
  int64_t* inv = (int64_t*)malloc((size_t)(total > 0 ? total : 1) * sizeof(int64_t));
  float* density = (float*)malloc((size_t)(total > 0 ? total : 1) * sizeof(float));
  if (!offsets || !perm || !inv || !density) {
    st = ORA_ERR_INVALID_ARGUMENT;
    goto done;
  }
  st = ora_build_hashgrid(cfg, positions, batch, n, offsets, perm, inv);
  if (st) goto done;
  walk_ctx w = {cfg, positions, offsets, perm, n, cells, cfg->eps * cfg->eps};
  sph_consts k = make_sph(cfg);
#pragma omp parallel for schedule(dynamic, 256) num_threads(ora_get_threads())
  for (int64_t idx = 0; idx < total; ++idx) {
    float rho = 0.0f;
    FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, { (void)j; (void)delta; rho = rho + poly6(r2, &k); });
    density[idx] = rho;
  }
#pragma omp parallel for schedule(dynamic, 256) num_threads(ora_get_threads())
  for (int64_t idx = 0; idx < total; ++idx) {
    float m[9] = {0};
    FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
      if (j != idx) {
        float gv[4];
        spiky(delta, r2, &k, recip_finite(density[j]), gv);
        for (int r = 0; r < dim; ++r)
          for (int col = 0; col < dim; ++col) m[r * dim + col] = m[r * dim + col] + delta[r] * gv[col];
      }
    });
    if (dim == 2) {
      det_out[idx] = m[0] * m[3] - m[1] * m[1];
    } else {
      float a = m[0], b = m[1], c = m[2], d = m[4], e = m[5], f = m[8];
      float t1 = d * f - e * e;
      float t2 = c * e - b * f;
      float t3 = b * e - c * d;
      det_out[idx] = a * t1 + b * t2 + c * t3;
    }
  }
done:
  free(offsets);
  free(perm);
  free(inv);
  free(density);
  return st;
}

/* ------------------------------------------------------------------------ */
/* MLP (model.rs:900-940)                                                    */
/* ------------------------------------------------------------------------ */

int ora_forward_update(const float* features, int64_t rows, int64_t in_dims,
                       int64_t hidden_dims, int64_t out_dims, const float* w1, const float* b1,
                       const float* w2, const float* b2, float* update) {
  if (rows < 0 || in_dims <= 0 || hidden_dims <= 0 || out_dims <= 0)
    return ORA_ERR_INVALID_ARGUMENT;
#pragma omp parallel num_threads(ora_get_threads())
  {
    float* hidden = (float*)malloc((size_t)hidden_dims * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t row = 0; row < rows; ++row) {
      const float* f = features + row * in_dims;
      for (int64_t h = 0; h < hidden_dims; ++h) {
        float sum = b1[h];
        const float* w = w1 + h * in_dims;
        for (int64_t i = 0; i < in_dims; ++i) sum = sum + w[i] * f[i];
        hidden[h] = maxf_rs(sum, 0.0f);
      }
      float* u = update + row * out_dims;
      for (int64_t o = 0; o < out_dims; ++o) {
        float sum = b2[o];
        const float* w = w2 + o * hidden_dims;
        for (int64_t h = 0; h < hidden_dims; ++h) sum = sum + w[h] * hidden[h];
        u[o] = sum;
      }
    }
    free(hidden);
  }
  return ORA_OK;
}

/* ------------------------------------------------------------------------ */
/* Euler step (reference/step.rs:4-55)                                       */
/* ------------------------------------------------------------------------ */

int ora_euler_step(const ora_grid_config* cfg, const float* positions, const float* states,
                   const float* dx, const float* ds, int64_t batch, int64_t n, int64_t c,
                   float dt, const float* update_mask, float* next_positions,
                   float* next_states) {
  int st = check_shapes_basic(batch, n, c);
  if (st) return st;
  const int64_t total = batch * n;
  const int mem_dims = cfg->dim == 3 ? 4 : 2;
#pragma omp parallel for schedule(static) num_threads(ora_get_threads())
  for (int64_t idx = 0; idx < total; ++idx) {
    float mask = update_mask ? update_mask[idx] : 1.0f;
    float p[4];
    for (int a = 0; a < 4; ++a) p[a] = positions[4 * idx + a];
    for (int a = 0; a < mem_dims; ++a) p[a] = p[a] + dt * dx[4 * idx + a] * mask;
    wrap_position(p, cfg);
    for (int a = 0; a < 4; ++a) next_positions[4 * idx + a] = p[a];
    for (int64_t ch = 0; ch < c; ++ch) {
      float next = states[idx * c + ch] + dt * ds[idx * c + ch] * mask;
      if (cfg->dim == 3 && c > 3 && (ch == 3 || (c > 8 && ch == 8)))
        next = clampf_rs(next, -8.0f, 24.0f);
      next_states[idx * c + ch] = next;
    }
  }
  return ORA_OK;
}

/* ------------------------------------------------------------------------ */
/* NpaModel::step_cpu (model.rs:768-858)                                     */
/* ------------------------------------------------------------------------ */

int64_t ora_model_perception_dims(const ora_model_config* m) {
  return (int64_t)m->state_dims * 2 +
         (m->state_grad ? (int64_t)m->state_dims * m->spatial_dims : 0) +
         (m->density_grad ? m->spatial_dims : 0) +
         (m->position_features ? m->spatial_dims : 0) + m->auxiliary_input_dims;
}

static float maturity_gate(float liveness) {
  /* position_conditioned_3d_maturity_gate (rollout/mod.rs:67-69) */
  return clampf_rs((4.0f - liveness) * 2.0f, 0.0f, 1.0f);
}

static float motion_gate(float liveness, float signed_distance, int anchored) {
  /* position_conditioned_3d_motion_gate (rollout/mod.rs:78-90) */
  if (anchored) return 0.0f;
  float s = maturity_gate(liveness);
  float d = clampf_rs((fabsf(signed_distance) - 0.01f) / 0.02f, 0.0f, 1.0f);
  return s * d;
}

int ora_step(const ora_model_config* m, const float* w1, const float* b1, const float* w2,
             const float* b2, const ora_grid_config* grid, const float* positions,
             const float* states, int64_t batch, int64_t n, float dt, const float* update_mask,
             float* next_positions, float* next_states, float* dx_out, float* ds_out,
             float* features_out, float* density_out) {
  if (!(m->spatial_dims == 2 || m->spatial_dims == 3)) return ORA_ERR_INVALID_MODEL;
  if (m->state_dims <= 0 || m->hidden_dims <= 0) return ORA_ERR_INVALID_MODEL;
  if (m->auxiliary_input_dims != 0) return ORA_ERR_INVALID_ARGUMENT;
  if (grid->dim != m->spatial_dims) return ORA_ERR_INVALID_ARGUMENT;
  const int64_t c = m->state_dims, dim = m->spatial_dims, hdim = m->hidden_dims;
  const int64_t total = batch * n;
  const int scale_eq = m->equivariance == 2;
  const int pde = m->equivariance == 1 || m->equivariance == 2;
  ora_perception_options opt;
  memset(&opt, 0, sizeof opt);
  opt.state_grad = m->state_grad;
  opt.density_grad = m->density_grad;
  opt.eps0 = m->eps0;
  opt.scale_equivariance = (uint8_t)scale_eq;
  opt.particle_density_equivariance = (uint8_t)pde;
  opt.log_norm_grad = m->log_norm_grad;
  opt.log_norm_density_grad = m->log_norm_density_grad;
  opt.hybrid_state_gradient = 1;
  opt.position_features = m->position_features;
  const int64_t fd = ora_feature_dims(grid, &opt, c);
  const int64_t od = dim + c;
  float* features = (float*)malloc((size_t)(total * fd > 0 ? total * fd : 1) * sizeof(float));
  float* update = (float*)malloc((size_t)(total * od > 0 ? total * od : 1) * sizeof(float));
  float* dx = (float*)calloc((size_t)(total > 0 ? total : 1) * 4, sizeof(float));
  float* ds = (float*)malloc((size_t)(total * c > 0 ? total * c : 1) * sizeof(float));
  int st = ORA_OK;
  if (!features || !update || !dx || !ds) {
    st = ORA_ERR_INVALID_ARGUMENT;
    goto done;
  }
  st = ora_perceive(grid, &opt, positions, states, batch, n, c, features, density_out, NULL,
                    NULL, NULL);
  if (st) goto done;
  st = ora_forward_update(features, total, fd, hdim, od, w1, b1, w2, b2, update);
  if (st) goto done;
  {
    /* forward_from_features_with_eps (model.rs:867-898) */
    const float motion_eps = scale_eq ? grid->eps : m->eps0;
#pragma omp parallel for schedule(static) num_threads(ora_get_threads())
    for (int64_t row = 0; row < total; ++row) {
      const float* u = update + row * od;
      float norm = 0.0f;
      for (int64_t a = 0; a < dim; ++a) norm = norm + u[a] * u[a];
      norm = sqrtf(norm);
      for (int64_t a = 0; a < dim; ++a) dx[4 * row + a] = m->alpha * u[a] * motion_eps / (1.0f + norm);
      for (int64_t ch = 0; ch < c; ++ch) ds[row * c + ch] = u[dim + ch];
    }
  }
  if (dim == 3 && m->position_features && c > 3) {
    /* model.rs:806-837; the reference indexes channel 7 of each row. */
    if (c <= 7) {
      st = ORA_ERR_INVALID_ARGUMENT;
      goto done;
    }
    for (int64_t row = 0; row < total; ++row) {
      float liveness = states[row * c + 3];
      float sd = states[row * c + 7];
      float sgate = maturity_gate(liveness);
      float mgate = motion_gate(liveness, sd, positions[4 * row + 3] >= 0.5f);
      for (int64_t a = 0; a < dim; ++a) dx[4 * row + a] = dx[4 * row + a] * mgate;
      for (int64_t ch = 0; ch < c; ++ch) ds[row * c + ch] = ds[row * c + ch] * sgate;
    }
  }
  st = ora_euler_step(grid, positions, states, dx, ds, batch, n, c, dt, update_mask,
                      next_positions, next_states);
  if (dx_out) memcpy(dx_out, dx, (size_t)total * 4 * sizeof(float));
  if (ds_out) memcpy(ds_out, ds, (size_t)(total * c) * sizeof(float));
  if (features_out) memcpy(features_out, features, (size_t)(total * fd) * sizeof(float));
done:
  free(features);
  free(update);
  free(dx);
  free(ds);
  return st;
}

/* ------------------------------------------------------------------------ */
/* Rollout loop (rollout/mod.rs:240-283)                                     */
/* ------------------------------------------------------------------------ */

int ora_rollout(const ora_model_config* m, const float* w1, const float* b1, const float* w2,
                const float* b2, const ora_grid_config* grid, float* positions, float* states,
                int64_t batch, int64_t n, int64_t steps, float dt, const float* masks,
                float* mean_dx) {
  const int64_t total = batch * n;
  const int64_t c = m->state_dims;
  float* np = (float*)malloc((size_t)(total > 0 ? total : 1) * 4 * sizeof(float));
  float* ns = (float*)malloc((size_t)(total * c > 0 ? total * c : 1) * sizeof(float));
  float* dx = (float*)malloc((size_t)(total > 0 ? total : 1) * 4 * sizeof(float));
  int st = ORA_OK;
  if (!np || !ns || !dx) {
    st = ORA_ERR_INVALID_ARGUMENT;
    goto done;
  }
  for (int64_t s = 0; s < steps; ++s) {
    const float* mask = masks ? masks + s * total : NULL;
    st = ora_step(m, w1, b1, w2, b2, grid, positions, states, batch, n, dt, mask, np, ns, dx,
                  NULL, NULL, NULL);
    if (st) goto done;
    if (mean_dx) {
      float sum = 0.0f;
      for (int64_t r = 0; r < total; ++r) {
        const float* v = dx + 4 * r;
        sum = sum + sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
      }
      mean_dx[s] = sum / (float)(total > 1 ? total : 1);
    }
    memcpy(positions, np, (size_t)total * 4 * sizeof(float));
    memcpy(states, ns, (size_t)(total * c) * sizeof(float));
  }
done:
  free(np);
  free(ns);
  free(dx);
  return st;
}

/* ------------------------------------------------------------------------ */
/* decode_gaussians_3d (gaussian.rs:53-223)                                  */
/* ------------------------------------------------------------------------ */

static int64_t sh_coeffs(const ora_decode_config* cfg) {
  if (cfg->mode == 3) return (int64_t)(cfg->sh_degree + 1) * (cfg->sh_degree + 1);
  return 1;
}

int64_t ora_gaussian_record_floats(const ora_decode_config* cfg) {
  return 12 + 3 * sh_coeffs(cfg);
}

static float sigmoid_rs(float v) { return 1.0f / (1.0f + expf(-v)); }

int ora_decode_gaussians(const ora_decode_config* cfg, const float* positions,
                         const float* states, int64_t count, int64_t c, float* out) {
  if (cfg->mode < 0 || cfg->mode > 3 || cfg->sh_degree < 0) return ORA_ERR_INVALID_ARGUMENT;
  const int64_t k = sh_coeffs(cfg);
  /* validate_decode_layout (gaussian.rs:102-125), an assert! in the reference */
  if ((cfg->mode <= 1 && c < 3) || (cfg->mode == 2 && c < 5) || (cfg->mode == 3 && c < k * 3 + 8))
    return ORA_ERR_STATE_SHAPE;
  if (!(cfg->min_scale <= cfg->max_scale) || !(cfg->min_opacity <= cfg->max_opacity))
    return ORA_ERR_INVALID_ARGUMENT;
  const int64_t rec = 12 + 3 * k;
#pragma omp parallel for schedule(static) num_threads(ora_get_threads())
  for (int64_t idx = 0; idx < count; ++idx) {
    const float* s = states + idx * c;
    const float* p = positions + 4 * idx;
    float* o = out + idx * rec;
    o[0] = p[0];
    o[1] = p[1];
    o[2] = p[2];
    o[3] = 1.0f;
    int64_t color_start = cfg->mode == 3 ? c - k * 3 : c - 3;
    for (int64_t q = 0; q < k; ++q) {
      int64_t base = color_start + q * 3;
      for (int e = 0; e < 3; ++e) o[12 + q * 3 + e] = clampf_rs(s[base + e] + 0.5f, 0.0f, 1.0f);
    }
    if (cfg->mode == 3) {
      int64_t rs = color_start - 4;
      float qv[4] = {s[rs], s[rs + 1], s[rs + 2], s[rs + 3]};
      float norm = sqrtf(qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3]);
      if (norm <= 1e-8f) {
        qv[0] = 1.0f;
        qv[1] = qv[2] = qv[3] = 0.0f;
      } else {
        for (int e = 0; e < 4; ++e) qv[e] = qv[e] / norm;
      }
      for (int e = 0; e < 4; ++e) o[4 + e] = qv[e];
    } else {
      o[4] = 1.0f;
      o[5] = o[6] = o[7] = 0.0f;
    }
    float* so = o + 8;
    switch (cfg->mode) {
      case 0: {
        float scale = maxf_rs(cfg->min_scale, 1.0e-6f);
        so[0] = so[1] = so[2] = scale;
        so[3] = 1.0f;
        break;
      }
      case 1: {
        float scale = clampf_rs(cfg->sigma, cfg->min_scale, cfg->max_scale);
        so[0] = so[1] = so[2] = scale;
        so[3] = clampf_rs(cfg->opacity_scale, cfg->min_opacity, cfg->max_opacity);
        break;
      }
      case 2: {
        float scale_logit = clampf_rs(s[c - 5], -8.0f, 8.0f);
        float opacity_logit = clampf_rs(s[c - 4], -12.0f, 12.0f);
        float scale = clampf_rs(cfg->sigma * expf(scale_logit), cfg->min_scale, cfg->max_scale);
        float opacity = clampf_rs(sigmoid_rs(opacity_logit), cfg->min_opacity, cfg->max_opacity) *
                        cfg->opacity_scale;
        so[0] = so[1] = so[2] = scale;
        so[3] = clampf_rs(opacity, cfg->min_opacity, cfg->max_opacity);
        break;
      }
      default: {
        int64_t anis = color_start - 8;
        float mdiv = maxf_rs(cfg->max_anisotropy, 1e-6f);
        float ax = tanhf(s[anis] / mdiv) * cfg->max_anisotropy;
        float ay = tanhf(s[anis + 1] / mdiv) * cfg->max_anisotropy;
        float az = tanhf(s[anis + 2] / mdiv) * cfg->max_anisotropy;
        float ol = tanhf(s[anis + 3] / mdiv) * cfg->max_anisotropy;
        so[0] = clampf_rs(cfg->sigma * expf(ax), cfg->min_scale, cfg->max_scale);
        so[1] = clampf_rs(cfg->sigma * expf(ay), cfg->min_scale, cfg->max_scale);
        so[2] = clampf_rs(cfg->sigma * expf(az), cfg->min_scale, cfg->max_scale);
        so[3] = clampf_rs(cfg->opacity_scale * expf(ol), cfg->min_opacity, cfg->max_opacity);
        break;
      }
    }
  }
  return ORA_OK;
}

/* ---- GPU executor stochastic update mask ----
 * Host twin of the reference's WGSL update_mask (crates/burn_automata/src/
 * gpu_step.wgsl:1019-1056) as restated by its test helper gpu_update_mask /
 * gpu_random01 / hash_u32 (crates/burn_automata/tests/gpu_wgpu/common.rs:
 * 115-137), extended to batches with the executor's lane seeds
 * (crates/burn_automata/src/gpu/executor/state.rs:1282-1312). */
static uint32_t ora_mask_hash(uint32_t value) {
  uint32_t x = value;
  x = (x ^ 61u) ^ (x >> 16);
  x = x + (x << 3);
  x ^= x >> 4;
  x = x * 0x27d4eb2du;
  return x ^ (x >> 15);
}

static float ora_mask_random01(uint32_t particle, uint32_t step, uint32_t seed) {
  uint32_t mixed = ora_mask_hash(particle ^ ora_mask_hash(step + 0x9e3779b9u) ^ seed);
  return (float)(mixed >> 8) * (1.0f / 16777216.0f);
}

int ora_gpu_update_mask(int64_t batch, int64_t n, float update_prob, uint32_t step,
                        const uint32_t* lane_seeds, float* out) {
  if (batch < 0 || n < 0) return ORA_ERR_INVALID_ARGUMENT;
  for (int64_t lane = 0; lane < batch; ++lane) {
    for (int64_t i = 0; i < n; ++i) {
      float m;
      if (update_prob >= 1.0f) m = 1.0f;
      else if (update_prob <= 0.0f) m = 0.0f;
      else m = ora_mask_random01((uint32_t)i, step, lane_seeds[lane]) < update_prob ? 1.0f : 0.0f;
      out[lane * n + i] = m;
    }
  }
  return ORA_OK;
}

/* ---- the CPU rollout's StdRng update masks (rollout/mod.rs:222-238, :644-651) ----
 * Restated third-party algorithms (crates absent from the reference tree; the
 * versions are its Cargo.lock's):
 *   rand_core 0.9 SeedableRng::seed_from_u64: a PCG32 generator (O'Neill 2014,
 *     XSH-RR 64/32 output) whose 64-bit LCG state (multiplier
 *     6364136223846793005, increment 11634580027462260723) is stepped before
 *     each output; eight outputs, little-endian, are the 32-byte seed.
 *   rand_chacha 0.9.0 ChaCha12Rng::from_seed: Bernstein's ChaCha with 12
 *     rounds; words 0-3 the "expand 32-byte k" constants, 4-11 the seed as
 *     little-endian words, 12-13 a 64-bit block counter from 0, 14-15 the
 *     stream (0).  The generator's u32 outputs are the blocks' 16 words in
 *     order, blocks in counter order.
 *   rand 0.9.4 random::<f32>() (StandardUniform): (next_u32() >> 8) * 2^-24.
 * stochastic_mask draws one value per particle in index order, so the mask of
 * rollout step s (0-based) for particle i uses stream word s * count + i; with
 * update_prob >= 1 it returns ones and draws nothing. */
static uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

void ora_stdrng_key(uint64_t rng_seed, uint32_t key[8]) {
  uint64_t state = rng_seed;
  for (int k = 0; k < 8; ++k) {
    state = state * 6364136223846793005ull + 11634580027462260723ull;
    const uint32_t xorshifted = (uint32_t)(((state >> 18) ^ state) >> 27);
    const uint32_t rot = (uint32_t)(state >> 59);
    key[k] = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
  }
}

#define ORA_QR(a, b, c, d)                \
  do {                                    \
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 16); \
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 12); \
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 8);  \
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 7);  \
  } while (0)

void ora_chacha_block(const uint32_t key[8], uint64_t counter, int rounds, uint32_t out[16]) {
  uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
  for (int k = 0; k < 8; ++k) in[4 + k] = key[k];
  in[12] = (uint32_t)counter;
  in[13] = (uint32_t)(counter >> 32);
  in[14] = 0;
  in[15] = 0;
  uint32_t x[16];
  memcpy(x, in, sizeof(x));
  for (int r = 0; r < rounds; r += 2) {
    ORA_QR(0, 4, 8, 12);
    ORA_QR(1, 5, 9, 13);
    ORA_QR(2, 6, 10, 14);
    ORA_QR(3, 7, 11, 15);
    ORA_QR(0, 5, 10, 15);
    ORA_QR(1, 6, 11, 12);
    ORA_QR(2, 7, 8, 13);
    ORA_QR(3, 4, 9, 14);
  }
  for (int k = 0; k < 16; ++k) out[k] = x[k] + in[k];
}
#undef ORA_QR

/* stochastic_mask draws of StdRng::seed_from_u64(rng_seed) for `steps` steps
 * of `count` particles from step first_step. */
static int stdrng_masks(uint64_t rng_seed, float update_prob, int64_t count, int64_t first_step,
                        int64_t steps, float* out) {
  if (count < 0 || steps < 0 || first_step < 0) return ORA_ERR_INVALID_ARGUMENT;
  if (update_prob >= 1.0f) {
    for (int64_t i = 0; i < count * steps; ++i) out[i] = 1.0f;
    return ORA_OK;
  }
  uint32_t key[8], block[16];
  ora_stdrng_key(rng_seed, key);
  uint64_t have = UINT64_MAX;
  for (int64_t k = 0; k < steps; ++k) {
    for (int64_t i = 0; i < count; ++i) {
      const uint64_t w = (uint64_t)(first_step + k) * (uint64_t)count + (uint64_t)i;
      if (w / 16 != have) {
        have = w / 16;
        ora_chacha_block(key, have, 12, block);
      }
      const float u = (float)(block[w % 16] >> 8) * (1.0f / 16777216.0f);
      out[k * count + i] = u < update_prob ? 1.0f : 0.0f;
    }
  }
  return ORA_OK;
}

int ora_rollout_masks(uint64_t rollout_seed, float update_prob, int64_t count,
                      int64_t first_step, int64_t steps, float* out) {
  return stdrng_masks(rollout_seed ^ 0x5eedull, update_prob, count, first_step, steps, out);
}

/* ------------------------------------------------------------------------ */
/* Training rollout (crates/burn_automata/src/target2d.rs, training.rs)      */
/* ------------------------------------------------------------------------ */

/* mlp_backward_from_output_gradients (training.rs:558-640): per row the
 * forward pass again (pre-activation and ReLU), then the hidden and input
 * adjoints; the weight gradients are summed over the rows in row order. */
int ora_mlp_backward(const float* features, int64_t rows, int64_t in_dims, int64_t hidden,
                     int64_t out_dims, const float* w1, const float* b1, const float* w2,
                     const float* output_gradients, float* gw1, float* gb1, float* gw2,
                     float* gb2, float* gfeatures) {
  if (rows <= 0 || in_dims <= 0 || hidden <= 0 || out_dims <= 0) return ORA_ERR_INVALID_ARGUMENT;
  memset(gw1, 0, (size_t)(hidden * in_dims) * sizeof(float));
  memset(gb1, 0, (size_t)hidden * sizeof(float));
  memset(gw2, 0, (size_t)(out_dims * hidden) * sizeof(float));
  memset(gb2, 0, (size_t)out_dims * sizeof(float));
  memset(gfeatures, 0, (size_t)(rows * in_dims) * sizeof(float));
  float* pre = (float*)malloc((size_t)hidden * sizeof(float));
  float* hid = (float*)malloc((size_t)hidden * sizeof(float));
  float* dh = (float*)malloc((size_t)hidden * sizeof(float));
  if (!pre || !hid || !dh) {
    free(pre);
    free(hid);
    free(dh);
    return ORA_ERR_INVALID_ARGUMENT;
  }
  for (int64_t row = 0; row < rows; ++row) {
    for (int64_t h = 0; h < hidden; ++h) dh[h] = 0.0f;
    const float* f = features + row * in_dims;
    for (int64_t h = 0; h < hidden; ++h) {
      float sum = b1[h];
      for (int64_t i = 0; i < in_dims; ++i) sum = sum + w1[h * in_dims + i] * f[i];
      pre[h] = sum;
      hid[h] = maxf_rs(sum, 0.0f);
    }
    const float* g = output_gradients + row * out_dims;
    for (int64_t o = 0; o < out_dims; ++o) {
      const float d = g[o];
      gb2[o] = gb2[o] + d;
      for (int64_t h = 0; h < hidden; ++h) {
        gw2[o * hidden + h] = gw2[o * hidden + h] + d * hid[h];
        dh[h] = dh[h] + d * w2[o * hidden + h];
      }
    }
    for (int64_t h = 0; h < hidden; ++h) {
      const float dp = pre[h] > 0.0f ? dh[h] : 0.0f;
      gb1[h] = gb1[h] + dp;
      for (int64_t i = 0; i < in_dims; ++i) {
        gw1[h * in_dims + i] = gw1[h * in_dims + i] + dp * f[i];
        gfeatures[row * in_dims + i] = gfeatures[row * in_dims + i] + dp * w1[h * in_dims + i];
      }
    }
  }
  free(pre);
  free(hid);
  free(dh);
  return ORA_OK;
}

/* raw_motion_adjoint (target2d.rs:3644-3673): the adjoint of
 * dx = scale * raw / (1 + |raw|) with respect to raw, added into out. */
static void raw_motion_adjoint(const float* raw, const float* dx_adj, int dims, float scale,
                               float* out) {
  float norm = 0.0f;
  for (int a = 0; a < dims; ++a) norm = norm + raw[a] * raw[a];
  norm = sqrtf(norm);
  const float denom = 1.0f + norm;
  float dot = 0.0f;
  for (int a = 0; a < dims; ++a) dot = dot + raw[a] * dx_adj[a];
  for (int a = 0; a < dims; ++a) {
    float grad = dx_adj[a] / denom;
    if (norm > 0.0f) grad = grad - raw[a] * dot / (norm * denom * denom);
    out[a] = out[a] + scale * grad;
  }
}

/* add_dx_norm_regularizer_adjoint (target2d.rs:3675-3722). */
static void dx_norm_regularizer_adjoint(const float* raw, int dims, float scale, float weight,
                                        float* out) {
  if (weight == 0.0f) return;
  float norm = 0.0f;
  for (int a = 0; a < dims; ++a) norm = norm + raw[a] * raw[a];
  norm = sqrtf(norm);
  float dx[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int a = 0; a < dims; ++a) dx[a] = scale * raw[a] / (1.0f + norm);
  float dx_norm = 0.0f;
  for (int a = 0; a < dims; ++a) dx_norm = dx_norm + dx[a] * dx[a];
  dx_norm = sqrtf(dx_norm);
  if (dx_norm == 0.0f) return;
  float adj[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int a = 0; a < dims; ++a) adj[a] = weight * dx[a] / dx_norm;
  raw_motion_adjoint(raw, adj, dims, scale, out);
}

/* rollout_for_training (target2d.rs:3414-3466): `steps` steps with dt = 1 and
 * the masks of StdRng::seed_from_u64(seed ^ 0x5eed2d); every step's input
 * positions, states and mask are recorded; mean_dx_norm_sum adds each step's
 * mean |dx| (spatial axes) in f32. */
int ora_rollout_for_training(const ora_model_config* m, const float* w1, const float* b1,
                             const float* w2, const float* b2, const ora_grid_config* grid,
                             const float* positions, const float* states, int64_t batch,
                             int64_t n, int64_t steps, float update_prob, uint64_t seed,
                             float* snap_positions, float* snap_states, float* snap_masks,
                             float* final_positions, float* final_states,
                             float* mean_dx_norm_sum) {
  const int64_t total = batch * n, c = m->state_dims;
  float* masks = (float*)malloc((size_t)(total * steps > 0 ? total * steps : 1) * sizeof(float));
  float* pos = (float*)malloc((size_t)(total > 0 ? total : 1) * 4 * sizeof(float));
  float* st = (float*)malloc((size_t)(total * c > 0 ? total * c : 1) * sizeof(float));
  float* np = (float*)malloc((size_t)(total > 0 ? total : 1) * 4 * sizeof(float));
  float* ns = (float*)malloc((size_t)(total * c > 0 ? total * c : 1) * sizeof(float));
  float* dx = (float*)malloc((size_t)(total > 0 ? total : 1) * 4 * sizeof(float));
  int rc = ORA_OK;
  if (!masks || !pos || !st || !np || !ns || !dx) {
    rc = ORA_ERR_INVALID_ARGUMENT;
    goto done;
  }
  rc = stdrng_masks(seed ^ 0x5eed2dull, update_prob, total, 0, steps, masks);
  if (rc) goto done;
  memcpy(pos, positions, (size_t)total * 4 * sizeof(float));
  memcpy(st, states, (size_t)(total * c) * sizeof(float));
  float sum = 0.0f;
  for (int64_t k = 0; k < steps; ++k) {
    memcpy(snap_positions + k * total * 4, pos, (size_t)total * 4 * sizeof(float));
    memcpy(snap_states + k * total * c, st, (size_t)(total * c) * sizeof(float));
    memcpy(snap_masks + k * total, masks + k * total, (size_t)total * sizeof(float));
    rc = ora_step(m, w1, b1, w2, b2, grid, pos, st, batch, n, 1.0f, masks + k * total, np, ns,
                  dx, NULL, NULL, NULL);
    if (rc) goto done;
    /* mean_dx_norm (target2d.rs:3536-3548) */
    float norms = 0.0f;
    for (int64_t i = 0; i < total; ++i) {
      float s = 0.0f;
      for (int a = 0; a < m->spatial_dims; ++a) s = s + dx[4 * i + a] * dx[4 * i + a];
      norms = norms + sqrtf(s);
    }
    sum = sum + norms / (float)(total > 1 ? total : 1);
    float* t = pos;
    pos = np;
    np = t;
    t = st;
    st = ns;
    ns = t;
  }
  memcpy(final_positions, pos, (size_t)total * 4 * sizeof(float));
  memcpy(final_states, st, (size_t)(total * c) * sizeof(float));
  *mean_dx_norm_sum = sum;
done:
  free(masks);
  free(pos);
  free(st);
  free(np);
  free(ns);
  free(dx);
  return rc;
}

/* bptt_gradients (target2d.rs:3550-3642): back through the recorded steps in
 * reverse; per step the features and raw update again, the output adjoint
 * (raw_motion_adjoint of the masked position adjoint, the optional
 * displacement regularizer, the masked state adjoint), the MLP backward, and
 * the perception adjoint added to the running position / state adjoints
 * (unless stopped).  The Euler step is differentiated as the reference does:
 * identity plus the masked update (no wrap or clamp terms). */
int ora_bptt_gradients(const ora_model_config* m, const float* w1, const float* b1,
                       const float* w2, const float* b2, const ora_grid_config* grid,
                       const float* snap_positions, const float* snap_states,
                       const float* snap_masks, int64_t batch, int64_t n, int64_t steps,
                       const float* position_gradients, const float* state_gradients,
                       float regularizer_weight, int stopgrad_pos, int stopgrad_state,
                       float* gw1, float* gb1, float* gw2, float* gb2, float* pos_adj_out,
                       float* state_adj_out) {
  const int64_t total = batch * n, c = m->state_dims, dim = m->spatial_dims;
  const int64_t hdim = m->hidden_dims, od = dim + c;
  const int scale_eq = m->equivariance == 2;
  const int pde = m->equivariance == 1 || m->equivariance == 2;
  ora_perception_options opt;
  memset(&opt, 0, sizeof opt);
  opt.state_grad = m->state_grad;
  opt.density_grad = m->density_grad;
  opt.eps0 = m->eps0;
  opt.scale_equivariance = (uint8_t)scale_eq;
  opt.particle_density_equivariance = (uint8_t)pde;
  opt.log_norm_grad = m->log_norm_grad;
  opt.log_norm_density_grad = m->log_norm_density_grad;
  opt.hybrid_state_gradient = 1;
  opt.position_features = m->position_features;
  const int64_t fd = ora_feature_dims(grid, &opt, c);
  const float motion_eps = scale_eq ? grid->eps : m->eps0;
  const float scale = m->alpha * motion_eps;
  const float reg_scale =
      regularizer_weight == 0.0f ? 0.0f : regularizer_weight / (float)(total > 1 ? total : 1);
  float* pos_adj = (float*)malloc((size_t)(total > 0 ? total : 1) * 4 * sizeof(float));
  float* st_adj = (float*)malloc((size_t)(total * c > 0 ? total * c : 1) * sizeof(float));
  float* feat = (float*)malloc((size_t)(total * fd > 0 ? total * fd : 1) * sizeof(float));
  float* upd = (float*)malloc((size_t)(total * od > 0 ? total * od : 1) * sizeof(float));
  float* oadj = (float*)malloc((size_t)(total * od > 0 ? total * od : 1) * sizeof(float));
  float* sw1 = (float*)malloc((size_t)(hdim * fd) * sizeof(float));
  float* sb1 = (float*)malloc((size_t)hdim * sizeof(float));
  float* sw2 = (float*)malloc((size_t)(od * hdim) * sizeof(float));
  float* sb2 = (float*)malloc((size_t)od * sizeof(float));
  float* gfeat = (float*)malloc((size_t)(total * fd > 0 ? total * fd : 1) * sizeof(float));
  float* pst = (float*)malloc((size_t)(total * c > 0 ? total * c : 1) * sizeof(float));
  float* ppos = (float*)malloc((size_t)(total > 0 ? total : 1) * 4 * sizeof(float));
  int rc = ORA_OK;
  if (!pos_adj || !st_adj || !feat || !upd || !oadj || !sw1 || !sb1 || !sw2 || !sb2 || !gfeat ||
      !pst || !ppos) {
    rc = ORA_ERR_INVALID_ARGUMENT;
    goto done;
  }
  memcpy(pos_adj, position_gradients, (size_t)total * 4 * sizeof(float));
  memcpy(st_adj, state_gradients, (size_t)(total * c) * sizeof(float));
  memset(gw1, 0, (size_t)(hdim * fd) * sizeof(float));
  memset(gb1, 0, (size_t)hdim * sizeof(float));
  memset(gw2, 0, (size_t)(od * hdim) * sizeof(float));
  memset(gb2, 0, (size_t)od * sizeof(float));
  for (int64_t k = steps - 1; k >= 0; --k) {
    const float* sp = snap_positions + k * total * 4;
    const float* ss = snap_states + k * total * c;
    const float* sm = snap_masks + k * total;
    rc = ora_perceive(grid, &opt, sp, ss, batch, n, c, feat, NULL, NULL, NULL, NULL);
    if (rc) goto done;
    rc = ora_forward_update(feat, total, fd, hdim, od, w1, b1, w2, b2, upd);
    if (rc) goto done;
    for (int64_t row = 0; row < total; ++row) {
      float* o = oadj + row * od;
      for (int64_t j = 0; j < od; ++j) o[j] = 0.0f;
      const float mask = sm[row];
      float dxa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int64_t a = 0; a < dim; ++a) dxa[a] = pos_adj[4 * row + a] * mask;
      dx_norm_regularizer_adjoint(upd + row * od, (int)dim, scale, reg_scale, o);
      raw_motion_adjoint(upd + row * od, dxa, (int)dim, scale, o);
      for (int64_t ch = 0; ch < c; ++ch) o[dim + ch] = o[dim + ch] + st_adj[row * c + ch] * mask;
    }
    rc = ora_mlp_backward(feat, total, fd, hdim, od, w1, b1, w2, oadj, sw1, sb1, sw2, sb2, gfeat);
    if (rc) goto done;
    for (int64_t i = 0; i < hdim * fd; ++i) gw1[i] = gw1[i] + sw1[i];
    for (int64_t i = 0; i < hdim; ++i) gb1[i] = gb1[i] + sb1[i];
    for (int64_t i = 0; i < od * hdim; ++i) gw2[i] = gw2[i] + sw2[i];
    for (int64_t i = 0; i < od; ++i) gb2[i] = gb2[i] + sb2[i];
    rc = ora_perceive_adjoint(grid, &opt, sp, ss, batch, n, c, gfeat, pst, ppos);
    if (rc) goto done;
    if (!stopgrad_pos)
      for (int64_t row = 0; row < total; ++row)
        for (int64_t a = 0; a < dim; ++a) pos_adj[4 * row + a] = pos_adj[4 * row + a] + ppos[4 * row + a];
    if (!stopgrad_state)
      for (int64_t i = 0; i < total * c; ++i) st_adj[i] = st_adj[i] + pst[i];
  }
  if (pos_adj_out) memcpy(pos_adj_out, pos_adj, (size_t)total * 4 * sizeof(float));
  if (state_adj_out) memcpy(state_adj_out, st_adj, (size_t)(total * c) * sizeof(float));
done:
  free(pos_adj);
  free(st_adj);
  free(feat);
  free(upd);
  free(oadj);
  free(sw1);
  free(sb1);
  free(sw2);
  free(sb2);
  free(gfeat);
  free(pst);
  free(ppos);
  return rc;
}

/* ---- splat_particles_2d (crates/burn_automata_kernels/src/splat.rs:30-93) ----
 * Each particle adds colour * w to the pixels of its (2r+1)^2 footprint, with
 * w = exp(-(dx^2 + dy^2) / (2 sigma^2)) / (footprint weight sum) * norm_scale
 * when normalize_color; every pixel's sums run in particle order. */
int ora_splat_particles_2d(const ora_splat2d_config* cfg, const float* positions,
                           const float* colors, int64_t count, float* out) {
  const int64_t size = cfg->image_size;
  if (size < 0 || count < 0) return ORA_ERR_INVALID_ARGUMENT;
  for (int64_t i = 0; i < size * size * 4; ++i) out[i] = 0.0f;
  const float fsize = (float)size;
  float sigma = cfg->sigma;
  if (cfg->normalize_color) sigma = sigma * fsize * cfg->pixel_size / (cfg->hi - cfg->lo);
  const int64_t radius = f2i64_sat(maxf_rs(ceilf(5.0f * sigma), 1.0f));
  float norm_scale = 1.0f;
  if (cfg->normalize_color) {
    const float r = fsize * cfg->pixel_size / (cfg->hi - cfg->lo);
    norm_scale = r * r; /* powi(2) */
  }
  const float two_s2 = 2.0f * sigma * sigma;
  for (int64_t p = 0; p < count; ++p) {
    const float* pos = positions + p * 4;
    const float* color = colors + p * 3;
    const float px = (pos[0] - cfg->lo) / (cfg->hi - cfg->lo) * (fsize - 1.0f);
    float py = (pos[1] - cfg->lo) / (cfg->hi - cfg->lo) * (fsize - 1.0f);
    if (cfg->y_up) py = (fsize - 1.0f) - py;
    const int64_t base_x = f2i64_sat(floorf(px));
    const int64_t base_y = f2i64_sat(floorf(py));
    const float frac_x = px - (float)base_x;
    const float frac_y = py - (float)base_y;
    float weight_sum = 0.0f;
    for (int64_t oy = -radius; oy <= radius; ++oy)
      for (int64_t ox = -radius; ox <= radius; ++ox) {
        const int64_t x = base_x + ox, y = base_y + oy;
        if (x < 0 || y < 0 || x >= size || y >= size) continue;
        const float dx = (float)ox - frac_x, dy = (float)oy - frac_y;
        float t = dx * dx;
        t = t + dy * dy;
        weight_sum = weight_sum + expf(-t / two_s2);
      }
    const float denom = cfg->normalize_color ? maxf_rs(weight_sum, 1e-8f) : 1.0f;
    for (int64_t oy = -radius; oy <= radius; ++oy)
      for (int64_t ox = -radius; ox <= radius; ++ox) {
        const int64_t x = base_x + ox, y = base_y + oy;
        if (x < 0 || y < 0 || x >= size || y >= size) continue;
        const float dx = (float)ox - frac_x, dy = (float)oy - frac_y;
        float t = dx * dx;
        t = t + dy * dy;
        const float w = expf(-t / two_s2) / denom * norm_scale;
        float* px_out = out + (y * size + x) * 4;
        px_out[0] = px_out[0] + color[0] * w;
        px_out[1] = px_out[1] + color[1] * w;
        px_out[2] = px_out[2] + color[2] * w;
        px_out[3] = px_out[3] + w;
      }
  }
  return ORA_OK;
}

/* ------------------------------------------------------------------------ */
/* Perception adjoint (reference/adjoint.rs:28-489), serial as the reference */
/* ------------------------------------------------------------------------ */

/* smoothing_poly6_delta_adjoint (kernels.rs:62-79). */
static void poly6_delta_adjoint(const float delta[4], float r2, const sph_consts* k,
                                float output_adjoint, float out[4]) {
  out[0] = out[1] = out[2] = out[3] = 0.0f;
  if (r2 >= k->eps2) return;
  const float x = k->eps2 - r2;
  const float dk = -3.0f * k->poly6_norm * x * x;
  for (int a = 0; a < k->dim; ++a) out[a] = output_adjoint * dk * 2.0f * delta[a];
}

/* spiky_gradient_delta_adjoint (kernels.rs:100-126). */
static void spiky_delta_adjoint(const float delta[4], float r2, const sph_consts* k, float coeff,
                                const float adj[4], float out[4]) {
  out[0] = out[1] = out[2] = out[3] = 0.0f;
  if (r2 <= 0.0f || r2 >= k->eps2) return;
  const float r = sqrtf(r2);
  const float norm = coeff * k->spiky_norm * 3.0f;
  const float t = k->eps - r;
  const float scale = norm * (t * t) / r;
  const float dscale_dr = norm * (1.0f - (k->eps * k->eps) / r2);
  float dot = 0.0f;
  for (int a = 0; a < k->dim; ++a) dot = dot + adj[a] * delta[a];
  for (int a = 0; a < k->dim; ++a) out[a] = scale * adj[a] + dscale_dr * dot * delta[a] / r;
}

/* log_normalize_adjoint (normalize.rs:71-91); input_adjoint starts at zero. */
static void log_normalize_adjoint(const float* input, const float* out_adj, float* in_adj,
                                  int len) {
  const float e = 1.0e-6f;
  float s = 0.0f;
  for (int i = 0; i < len; ++i) s = s + input[i] * input[i];
  const float norm = maxf_rs(sqrtf(s + e * e), e);
  const float l = ln_1p_f32(norm);
  const float scale = l / norm;
  const float dscale = (norm / (1.0f + norm) - l) / (norm * norm);
  float dot = 0.0f;
  for (int i = 0; i < len; ++i) dot = dot + input[i] * out_adj[i];
  const float radial = dscale * dot / norm;
  for (int i = 0; i < len; ++i) in_adj[i] = in_adj[i] + (scale * out_adj[i] + radial * input[i]);
}

/* accumulate_volume_density_adjoint (adjoint.rs:425-435). */
static void volume_density_adjoint(const float* density, float* density_adjoint, int64_t idx,
                                   float volume_adjoint) {
  const float rho = density[idx];
  if (fabsf(rho) <= 1.0e-20f || !isfinite(rho)) return;
  density_adjoint[idx] = density_adjoint[idx] - volume_adjoint / (rho * rho);
}

/* add_delta_position_adjoint (adjoint.rs:437-448). */
static void delta_position_adjoint(float* pos_adj, int64_t lhs, int64_t rhs, int dim,
                                   const float d[4]) {
  for (int a = 0; a < dim; ++a) {
    pos_adj[4 * rhs + a] = pos_adj[4 * rhs + a] + d[a];
    pos_adj[4 * lhs + a] = pos_adj[4 * lhs + a] - d[a];
  }
}

int ora_perceive_adjoint(const ora_grid_config* cfg, const ora_perception_options* opt,
                         const float* positions, const float* states, int64_t batch, int64_t n,
                         int64_t c, const float* feature_adjoint, float* state_adjoint,
                         float* position_adjoint) {
  int st = check_shapes_basic(batch, n, c);
  if (st) return st;
  st = ora_grid_validate(cfg);
  if (st) return st;
  const int dim = cfg->dim;
  const int64_t total = batch * n;
  const int64_t fd = ora_feature_dims(cfg, opt, c);
  const int64_t cells = ora_cell_count(cfg);
  int64_t* offsets = (int64_t*)malloc((size_t)(batch * cells + 1) * sizeof(int64_t));
  int64_t* perm = (int64_t*)malloc((size_t)(total > 0 ? total : 1) * sizeof(int64_t));
  int64_t* inv = (int64_t*)malloc((size_t)(total > 0 ? total : 1) * sizeof(int64_t));
  float* density = (float*)malloc((size_t)(total > 0 ? total : 1) * sizeof(float));
  float* density_adjoint = (float*)calloc((size_t)(total > 0 ? total : 1), sizeof(float));
  float* raw = (float*)malloc((size_t)(c * dim > 0 ? c * dim : 1) * sizeof(float));
  float* raw_adj = (float*)malloc((size_t)(c * dim > 0 ? c * dim : 1) * sizeof(float));
  if (!offsets || !perm || !inv || !density || !density_adjoint || !raw || !raw_adj) {
    st = ORA_ERR_INVALID_ARGUMENT;
    goto done;
  }
  for (int64_t i = 0; i < total * c; ++i) state_adjoint[i] = 0.0f;
  for (int64_t i = 0; i < total * 4; ++i) position_adjoint[i] = 0.0f;
  st = ora_build_hashgrid(cfg, positions, batch, n, offsets, perm, inv);
  if (st) goto done;
  walk_ctx w = {cfg, positions, offsets, perm, n, cells, cfg->eps * cfg->eps};
  sph_consts k = make_sph(cfg);
#pragma omp parallel for schedule(dynamic, 256) num_threads(ora_get_threads())
  for (int64_t idx = 0; idx < total; ++idx) {
    float rho = 0.0f;
    FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, { (void)j; (void)delta; rho = rho + poly6(r2, &k); });
    density[idx] = rho;
  }
  const float eps0 = maxf_rs(opt->eps0, 1.17549435e-38f);
  const float grad_scale = opt->scale_equivariance ? cfg->eps / eps0 : 1.0f;
  float dens_scale = opt->scale_equivariance ? ora_powi(cfg->eps / eps0, 1 + dim) : 1.0f;
  dens_scale = dens_scale * (opt->particle_density_equivariance ? 1.0f / (float)(n > 1 ? n : 1)
                                                                : 1.0f);

  for (int64_t idx = 0; idx < total; ++idx) {
    const float* fa = feature_adjoint + idx * fd;
    int64_t cur = 0;
    const int64_t si = idx * c;
    for (int64_t ch = 0; ch < c; ++ch) state_adjoint[si + ch] = state_adjoint[si + ch] + fa[ch];
    cur += c;
    /* accumulate_blurred_state_adjoint (adjoint.rs:138-166) */
    {
      const float* badj = fa + cur;
      FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
        const float vol = recip_finite(density[j]);
        const float kern = poly6(r2, &k);
        const float weight = kern * vol;
        const int64_t sj = j * c;
        float wadj = 0.0f;
        for (int64_t ch = 0; ch < c; ++ch) {
          state_adjoint[sj + ch] = state_adjoint[sj + ch] + badj[ch] * weight;
          wadj = wadj + badj[ch] * states[sj + ch];
        }
        float da[4];
        poly6_delta_adjoint(delta, r2, &k, wadj * vol, da);
        delta_position_adjoint(position_adjoint, idx, j, dim, da);
        volume_density_adjoint(density, density_adjoint, j, wadj * kern);
      });
    }
    cur += c;
    if (opt->state_grad) {
      /* accumulate_state_gradient_adjoint (adjoint.rs:168-343) */
      const float* gadj = fa + cur;
      const int64_t gd = c * dim;
      for (int64_t g = 0; g < gd; ++g) raw[g] = 0.0f;
      float moment[9] = {0};
      FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
        if (j != idx) {
          const float vol = recip_finite(density[j]);
          float gv[4];
          spiky(delta, r2, &k, vol, gv);
          const int64_t sj = j * c;
          for (int64_t ch = 0; ch < c; ++ch) {
            const float diff = states[sj + ch] - states[si + ch];
            for (int a = 0; a < dim; ++a) raw[ch * dim + a] = raw[ch * dim + a] + diff * gv[a];
          }
          if (opt->hybrid_state_gradient)
            for (int r = 0; r < dim; ++r)
              for (int col = 0; col < dim; ++col)
                moment[r * dim + col] = moment[r * dim + col] + delta[r] * gv[col];
        }
      });
      float inverse[9];
      const int hybrid = opt->hybrid_state_gradient;
      if (hybrid) safe_inverse_symmetric(moment, dim, inverse);
      float inv_adj[9] = {0};
      for (int64_t ch = 0; ch < c; ++ch) {
        float corrected[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int64_t gb = ch * dim;
        for (int a = 0; a < dim; ++a) corrected[a] = raw[gb + a];
        if (hybrid) {
          float mc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int oa = 0; oa < dim; ++oa)
            for (int ia = 0; ia < dim; ++ia) mc[oa] = mc[oa] + corrected[ia] * inverse[ia * dim + oa];
          for (int a = 0; a < 4; ++a) corrected[a] = mc[a];
        }
        float ninput[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int a = 0; a < dim; ++a) ninput[a] = corrected[a] * grad_scale;
        float cadj[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (opt->log_norm_grad)
          log_normalize_adjoint(ninput, gadj + gb, cadj, dim);
        else
          for (int a = 0; a < dim; ++a) cadj[a] = gadj[gb + a];
        for (int a = 0; a < dim; ++a) cadj[a] = cadj[a] * grad_scale;
        float radj[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (hybrid) {
          for (int ia = 0; ia < dim; ++ia)
            for (int oa = 0; oa < dim; ++oa)
              radj[ia] = radj[ia] + cadj[oa] * inverse[ia * dim + oa];
        } else {
          for (int a = 0; a < dim; ++a) radj[a] = cadj[a];
        }
        for (int a = 0; a < dim; ++a) raw_adj[gb + a] = radj[a];
        if (hybrid)
          for (int ia = 0; ia < dim; ++ia)
            for (int oa = 0; oa < dim; ++oa)
              inv_adj[ia * dim + oa] = inv_adj[ia * dim + oa] + raw[gb + ia] * cadj[oa];
      }
      float m_adj[9] = {0};
      if (hybrid) {
        /* inverse_matrix_adjoint (adjoint.rs:450-469) */
        for (int row = 0; row < dim; ++row)
          for (int col = 0; col < dim; ++col) {
            float value = 0.0f;
            for (int ir = 0; ir < dim; ++ir)
              for (int ic = 0; ic < dim; ++ic)
                value = value + inverse[ir * dim + row] * inv_adj[ir * dim + ic] * inverse[col * dim + ic];
            m_adj[row * dim + col] = m_adj[row * dim + col] - value;
          }
      }
      FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
        if (j != idx) {
          const float vol = recip_finite(density[j]);
          float vg[4], ug[4];
          spiky(delta, r2, &k, vol, vg);
          spiky(delta, r2, &k, 1.0f, ug);
          const int64_t sj = j * c;
          for (int64_t ch = 0; ch < c; ++ch) {
            const int64_t gb = ch * dim;
            const float diff = states[sj + ch] - states[si + ch];
            float contrib = 0.0f;
            for (int a = 0; a < dim; ++a) contrib = contrib + raw_adj[gb + a] * vg[a];
            state_adjoint[sj + ch] = state_adjoint[sj + ch] + contrib;
            state_adjoint[si + ch] = state_adjoint[si + ch] - contrib;
            float gadj2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int a = 0; a < dim; ++a) gadj2[a] = raw_adj[gb + a] * diff;
            float da[4];
            spiky_delta_adjoint(delta, r2, &k, vol, gadj2, da);
            delta_position_adjoint(position_adjoint, idx, j, dim, da);
            float vadj = 0.0f;
            for (int a = 0; a < dim; ++a) vadj = vadj + gadj2[a] * ug[a];
            volume_density_adjoint(density, density_adjoint, j, vadj);
          }
          if (hybrid) {
            float dda[4] = {0.0f, 0.0f, 0.0f, 0.0f}, gadj2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int row = 0; row < dim; ++row)
              for (int col = 0; col < dim; ++col) {
                const float adj = m_adj[row * dim + col];
                dda[row] = dda[row] + adj * vg[col];
                gadj2[col] = gadj2[col] + adj * delta[row];
              }
            float gda[4];
            spiky_delta_adjoint(delta, r2, &k, vol, gadj2, gda);
            for (int a = 0; a < dim; ++a) dda[a] = dda[a] + gda[a];
            delta_position_adjoint(position_adjoint, idx, j, dim, dda);
            float vadj = 0.0f;
            for (int a = 0; a < dim; ++a) vadj = vadj + gadj2[a] * ug[a];
            volume_density_adjoint(density, density_adjoint, j, vadj);
          }
        }
      });
      cur += gd;
    }
    if (opt->density_grad) {
      /* accumulate_density_gradient_position_adjoint (adjoint.rs:345-392) */
      const float* dadj = fa + cur;
      float rawd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
        if (j != idx) {
          float g1[4];
          spiky(delta, r2, &k, 1.0f, g1);
          for (int a = 0; a < dim; ++a) rawd[a] = rawd[a] + g1[a];
        }
      });
      float ninput[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int a = 0; a < dim; ++a) ninput[a] = rawd[a] * dens_scale;
      float radj[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (opt->log_norm_density_grad) {
        log_normalize_adjoint(ninput, dadj, radj, dim);
        for (int a = 0; a < dim; ++a) radj[a] = radj[a] * dens_scale;
      } else {
        for (int a = 0; a < dim; ++a) radj[a] = dadj[a] * dens_scale;
      }
      FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
        if (j != idx) {
          float da[4];
          spiky_delta_adjoint(delta, r2, &k, 1.0f, radj, da);
          delta_position_adjoint(position_adjoint, idx, j, dim, da);
        }
      });
      cur += dim;
    }
    if (opt->position_features)
      for (int a = 0; a < dim; ++a)
        position_adjoint[4 * idx + a] = position_adjoint[4 * idx + a] + fa[cur + a];
  }
  /* accumulate_density_kernel_position_adjoint (adjoint.rs:394-412) */
  for (int64_t idx = 0; idx < total; ++idx) {
    const float adj = density_adjoint[idx];
    if (adj == 0.0f) continue;
    FOR_EACH_NEIGHBOR(&w, idx, j, delta, r2, {
      float da[4];
      poly6_delta_adjoint(delta, r2, &k, adj, da);
      delta_position_adjoint(position_adjoint, idx, j, dim, da);
    });
  }
done:
  free(offsets);
  free(perm);
  free(inv);
  free(density);
  free(density_adjoint);
  free(raw);
  free(raw_adj);
  return st;
}
