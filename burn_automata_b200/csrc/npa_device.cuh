// npa_device.cuh -- device-side semantics shared by every kernel.
//
// Each helper restates one function of the reference's CPU path with the same
// f32 operation order.  The library is compiled with --fmad=false, IEEE
// division and IEEE square root (no fast-math), so `a * b + c` is a rounded
// multiply followed by a rounded add, exactly as rustc emits it.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace npa {

constexpr int kBoundaryPeriodic = 0;
constexpr int kBoundaryClamped = 1;
constexpr int kModeGrid = 0;
constexpr int kModeParticle = 1;

// Grid constants for the kernels.  Host code fills it from npa_grid_config so
// that every derived f32 constant is computed once, in the reference's order.
struct GridParams {
  int dim;
  int boundary;
  int mode;
  int grid_size[3];
  uint32_t cells;      // HashGridConfig::cell_count (config.rs:86-88)
  uint32_t cells_mask; // cells - 1 when cells is a power of two (always in Particle mode), else 0
  float eps;
  float eps2;          // eps * eps (neighbor.rs:25)
  float extent[3];     // grid_size[axis] as f32 * eps (hashgrid.rs:170 / :80)
  float half[3];       // extent * 0.5
  float poly6_norm;    // smoothing_poly6_normalization (kernels.rs:128-134)
  float spiky_norm;    // gradient_spiky_normalization (kernels.rs:136-142)
};

// `f as isize`: saturating conversion with NaN -> 0 (Rust semantics).  The
// hardware conversion maps NaN to INT64_MIN, so NaN and the range ends are
// handled explicitly.
__device__ __forceinline__ long long f2ll_sat(float integral) {
  if (integral != integral) return 0;
  if (integral >= 9223372036854775808.0f) return 0x7fffffffffffffffLL;
  if (integral <= -9223372036854775808.0f) return static_cast<long long>(0x8000000000000000ULL);
  return static_cast<long long>(integral);
}

// `f as isize as i32`: the saturated value's low 32 bits.
__device__ __forceinline__ int f2i_low32(float integral) {
  return static_cast<int>(static_cast<unsigned long long>(f2ll_sat(integral)) & 0xffffffffULL);
}

// mix_coord (hashgrid.rs:155-163).
__device__ __forceinline__ uint32_t mix_coord(int value_low32, uint32_t salt) {
  uint32_t x = static_cast<uint32_t>(value_low32) ^ salt;
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// particle_cell_hash (hashgrid.rs:147-153).  DIM: the grid's dimension when
// the caller knows it at compile time (equal to g.dim), 0 to read g.dim.
template <int DIM = 0>
__device__ __forceinline__ uint32_t particle_cell_hash(const GridParams& g, int cx, int cy, int cz) {
  uint32_t h = mix_coord(cx, 0x9e3779b9u) ^ mix_coord(cy, 0x85ebca6bu);
  if ((DIM ? DIM : g.dim) == 3) h ^= mix_coord(cz, 0xc2b2ae35u);
  // h % cells; for a power-of-two cell count (Particle mode validates one)
  // the mask gives the same value without an integer division.
  return g.cells_mask ? (h & g.cells_mask) : (h % g.cells);
}

// Grid-mode axis cell (hashgrid.rs:80-90 / :106-116).
__device__ __forceinline__ int grid_axis_cell(const GridParams& g, int axis, float coordinate) {
  long long cell = f2ll_sat(floorf((coordinate + g.half[axis]) / g.eps));
  long long size = g.grid_size[axis];
  if (g.boundary == kBoundaryPeriodic) {
    long long r = cell % size;
    return static_cast<int>(r < 0 ? r + size : r);
  }
  if (cell < 0) cell = 0;
  if (cell > size - 1) cell = size - 1;
  return static_cast<int>(cell);
}

// cell_coords_for_position (hashgrid.rs:98-121); low 32 bits of each coordinate.
__device__ __forceinline__ int3 cell_coords(const GridParams& g, float4 p) {
  int c[3] = {0, 0, 0};
  const float v[3] = {p.x, p.y, p.z};
#pragma unroll
  for (int axis = 0; axis < 3; ++axis) {
    if (axis < g.dim) {
      if (g.mode == kModeParticle) {
        c[axis] = f2i_low32(floorf(v[axis] / g.eps));
      } else {
        c[axis] = grid_axis_cell(g, axis, v[axis]);
      }
    }
  }
  return make_int3(c[0], c[1], c[2]);
}

// cell_index_from_coords (hashgrid.rs:123-145); returns -1 for None.  DIM as
// for particle_cell_hash.
template <int DIM = 0>
__device__ __forceinline__ long long cell_index(const GridParams& g, int cx, int cy, int cz) {
  if (g.mode == kModeParticle) return particle_cell_hash<DIM>(g, cx, cy, cz);
  const int c[3] = {cx, cy, cz};
  unsigned long long stride = 1, hash = 0;
#pragma unroll
  for (int axis = 0; axis < 3; ++axis) {
    if (axis < (DIM ? DIM : g.dim)) {
      int size = g.grid_size[axis];
      int cell;
      if (g.boundary == kBoundaryPeriodic) {
        int r = c[axis] % size;
        cell = r < 0 ? r + size : r;
      } else {
        if (c[axis] < 0 || c[axis] >= size) return -1;
        cell = c[axis];
      }
      hash += static_cast<unsigned long long>(cell) * stride;
      stride *= static_cast<unsigned long long>(size);
    }
  }
  return static_cast<long long>(hash);
}

// cell_for_position (hashgrid.rs:71-96).
__device__ __forceinline__ uint32_t cell_for_position(const GridParams& g, float4 p) {
  int3 c = cell_coords(g, p);
  if (g.mode == kModeParticle) return particle_cell_hash(g, c.x, c.y, c.z);
  return static_cast<uint32_t>(cell_index(g, c.x, c.y, c.z));
}

// neighbor_delta (hashgrid.rs:165-181).  DIM as for particle_cell_hash.
template <int DIM = 0>
__device__ __forceinline__ float4 neighbor_delta(const GridParams& g, float4 lhs, float4 rhs) {
  float d[3] = {rhs.x - lhs.x, rhs.y - lhs.y, rhs.z - lhs.z};
  float out[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int axis = 0; axis < 3; ++axis) {
    if (axis < (DIM ? DIM : g.dim)) {
      float v = d[axis];
      if (g.boundary == kBoundaryPeriodic) {
        if (v > g.half[axis]) {
          v -= g.extent[axis];
        } else if (v < -g.half[axis]) {
          v += g.extent[axis];
        }
      }
      out[axis] = v;
    }
  }
  return make_float4(out[0], out[1], out[2], 0.0f);
}

// wrap_position (hashgrid.rs:183-193): (c + half).rem_euclid(extent) - half.
__device__ __forceinline__ float4 wrap_position(const GridParams& g, float4 p) {
  if (g.boundary != kBoundaryPeriodic) return p;
  float v[3] = {p.x, p.y, p.z};
#pragma unroll
  for (int axis = 0; axis < 3; ++axis) {
    if (axis < g.dim) {
      float a = v[axis] + g.half[axis];
      float r = fmodf(a, g.extent[axis]);
      if (r < 0.0f) r = r + fabsf(g.extent[axis]);
      v[axis] = r - g.half[axis];
    }
  }
  return make_float4(v[0], v[1], v[2], p.w);
}

// RecipFinite::recip_finite (kernels.rs:156-165).
__device__ __forceinline__ float recip_finite(float x) {
  if (fabsf(x) <= 1e-20f || !isfinite(x)) return 0.0f;
  return 1.0f / x;
}

// smoothing_poly6_kernel (kernels.rs:53-60).
__device__ __forceinline__ float poly6(const GridParams& g, float r2) {
  if (r2 >= g.eps2) return 0.0f;
  float x = g.eps2 - r2;
  return g.poly6_norm * x * x * x;
}

// spiky_gradient_kernel magnitude (kernels.rs:81-98): coeff * k * 3 * (eps-r)^2 / r;
// the gradient is mag * delta[axis].  Zero for r2 <= 0 or r2 >= eps^2.
__device__ __forceinline__ float spiky_mag(const GridParams& g, float r2, float coeff) {
  if (r2 <= 0.0f || r2 >= g.eps2) return 0.0f;
  float r = sqrtf(r2);
  float t = g.eps - r;
  return coeff * g.spiky_norm * 3.0f * (t * t) / r;
}

// safe_inverse_symmetric (kernels.rs:3-51); reads m[0], m[1], m[3] (2D) or
// m[0], m[1], m[2], m[4], m[5], m[8] (3D), i.e. the upper triangle.
__device__ __forceinline__ void safe_inverse_symmetric(const float* m, int dim, float* out) {
  const float TOL = 1e-3f;
#pragma unroll
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

// The host C library's log1pf, bit for bit (f32::ln_1p of the reference; the
// table and how it is built: host_log1p.cu): CUDA's f32 log1pf corrected by a
// 2-bit code per input (0 same, 1 one ulp up, 2 one ulp down, 3 the result is
// stored in a sorted list).
struct Log1pTable {
  const uint32_t* codes;  // 16 codes per word, input (u - base) at bits 2 (i % 16)
  const uint2* side;      // {input bits, host result bits}, ascending inputs
  uint32_t base;          // bits of the smallest tabulated input
  uint32_t nbits;         // tabulated inputs: [base, base + nbits)
  int nside;
  float min_input;        // inputs below are not tabulated (CUDA's log1pf is returned)
};

// The code word holding input x's code (0 when x is not tabulated); loaded
// apart from log1p_host_word so that callers can issue several loads at once.
__device__ __forceinline__ uint32_t log1p_word(float x, const Log1pTable& t) {
  const uint32_t i = __float_as_uint(x) - t.base;
  if (!t.codes || !(x >= t.min_input) || !(i < t.nbits)) return 0u;
  return __ldg(t.codes + (i >> 4));
}

// log1pf(x) of the host given x's code word (from log1p_word).
__device__ __forceinline__ float log1p_host_word(float x, uint32_t word, const Log1pTable& t) {
  const float f = log1pf(x);
  const uint32_t u = __float_as_uint(x);
  const uint32_t i = u - t.base;
  if (!t.codes || !(x >= t.min_input) || !(i < t.nbits)) return f;
  const uint32_t code = (word >> (2u * (i & 15u))) & 3u;
  if (code != 3u)
    return __uint_as_float(__float_as_uint(f) + (code == 1u ? 1u : code == 2u ? ~0u : 0u));
  // lower bound of u among the stored results (every code-3 input is there)
  int lo = 0, n = t.nside;
  while (n > 0) {
    const int half = n >> 1;
    if (__ldg(t.side + lo + half).x < u) {
      lo += half + 1;
      n -= half + 1;
    } else {
      n = half;
    }
  }
  const uint2 e = lo < t.nside ? __ldg(t.side + lo) : make_uint2(0u, 0u);
  return e.x == u ? __uint_as_float(e.y) : f;
}

__device__ __forceinline__ float log1p_host(float x, const Log1pTable& t) {
  return log1p_host_word(x, log1p_word(x, t), t);
}

// f32::clamp (NaN passes through).
__device__ __forceinline__ float clamp_rs(float v, float lo, float hi) {
  if (v < lo) v = lo;
  if (v > hi) v = hi;
  return v;
}

// The GPU executor's counter-based stochastic update mask
// (crates/burn_automata/src/gpu_step.wgsl:1019-1056; host twin
// crates/burn_automata/tests/gpu_wgpu/common.rs:115-137): a particle updates
// in a step when random01(local index, step index, lane seed) < update_prob.
__host__ __device__ inline uint32_t mask_hash_u32(uint32_t x) {
  x = (x ^ 61u) ^ (x >> 16);
  x = x + (x << 3);
  x = x ^ (x >> 4);
  x = x * 0x27d4eb2du;
  x = x ^ (x >> 15);
  return x;
}

__host__ __device__ inline float mask_random01(uint32_t particle, uint32_t step, uint32_t seed) {
  const uint32_t mixed = mask_hash_u32(particle ^ mask_hash_u32(step + 0x9e3779b9u) ^ seed);
  return static_cast<float>(mixed >> 8) * (1.0f / 16777216.0f);
}

// update_mask without the reference's material / coarse-material extensions.
__host__ __device__ inline float stochastic_update_mask(float prob, uint32_t particle,
                                                        uint32_t step, uint32_t seed) {
  if (prob >= 1.0f) return 1.0f;
  if (prob <= 0.0f) return 0.0f;
  return mask_random01(particle, step, seed) < prob ? 1.0f : 0.0f;
}

// Sorted-slot view of the hashgrid used by every neighbour walk.
struct SortedGrid {
  const uint32_t* bin_offsets;  // [B*cells + 1], global sorted slots
  const uint32_t* permutation;  // [B*N] local index of each sorted slot
  const float4* srec;           // [B*N] 2D {x, y, cx, cy}; 3D {x, y, z, cx} (cells as int bits)
  const int2* scyz;             // [B*N] 3D only: {cy, cz}
  const float4* positions;      // [B*N] caller-order positions (own position, w included)
  // [B*N] or null: the processing order of the kernels that walk neighbours
  // (thread / tile row t handles sorted slot order[t]; null = the sorted order
  // itself).  Hit lists and feature tiles are indexed by t.
  const uint32_t* order;
  uint32_t n;                   // particles per batch
  uint32_t total;               // B*N: sorted slots are < total
};

// Neighbour record of sorted slot q: position (xyz) and cell coordinates.
template <int DIM>
__device__ __forceinline__ void load_record(const SortedGrid& s, uint32_t q, float4& pos,
                                            int3& cell) {
  const float4 r = __ldg(s.srec + q);
  if (DIM == 2) {
    pos = make_float4(r.x, r.y, 0.0f, 0.0f);
    cell = make_int3(__float_as_int(r.z), __float_as_int(r.w), 0);
  } else {
    const int2 yz = __ldg(s.scyz + q);
    pos = make_float4(r.x, r.y, r.z, 0.0f);
    cell = make_int3(__float_as_int(r.w), yz.x, yz.y);
  }
}

// Offsets of neighbour bin b in walk order (dz, dy, dx nested).
template <int DIM>
__device__ __forceinline__ int3 bin_delta(int b) {
  if (DIM == 3) return make_int3(b % 3 - 1, (b / 3) % 3 - 1, b / 9 - 1);
  return make_int3(b % 3 - 1, b / 3 - 1, 0);
}

__device__ __forceinline__ int3 add_wrapping(int3 c, int3 d) {
  return make_int3(static_cast<int>(static_cast<uint32_t>(c.x) + static_cast<uint32_t>(d.x)),
                   static_cast<int>(static_cast<uint32_t>(c.y) + static_cast<uint32_t>(d.y)),
                   static_cast<int>(static_cast<uint32_t>(c.z) + static_cast<uint32_t>(d.z)));
}

// for_each_neighbor (neighbor.rs:3-44): cells in dz, dy, dx order, bin ranges
// in permutation order, Particle-mode collision filter on exact coordinates,
// keeps r2 < eps^2 including the particle itself.  The candidates of all
// bins are walked as one flattened sequence (same order), so the threads of a
// warp iterate max(total candidates) rather than the per-bin maximum once per
// bin, and the records of KB consecutive candidates are loaded before any is
// tested, so their round trips to L2 overlap.  visit(q, delta, r2) receives
// the neighbour's sorted slot, in walk order.
template <int DIM, int KB = 4, class Visit>
__device__ __forceinline__ void for_each_neighbor(const GridParams& g, const SortedGrid& s,
                                                  uint32_t batch, float4 pi, int3 center,
                                                  Visit&& visit) {
  constexpr int NB = DIM == 3 ? 27 : 9;
  const uint32_t bin_base = batch * g.cells;
  uint32_t beg[NB], cum[NB];
  uint32_t ncand = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int3 nc = add_wrapping(center, bin_delta<DIM>(b));
    const long long cell = cell_index<DIM>(g, nc.x, nc.y, nc.z);
    uint32_t lo = 0, cnt = 0;
    if (cell >= 0) {
      const uint32_t bin = bin_base + static_cast<uint32_t>(cell);
      lo = __ldg(s.bin_offsets + bin);
      const uint32_t hi = min(__ldg(s.bin_offsets + bin + 1), s.total);
      cnt = hi > lo ? hi - lo : 0u;
    }
    beg[b] = lo;
    ncand += cnt;
    cum[b] = ncand;
  }
  int b = 0;
  uint32_t cur_beg = beg[0], cur_lo = 0, cur_hi = cum[0];
  for (uint32_t v0 = 0; v0 < ncand; v0 += KB) {
    uint32_t qs[KB];
    int bs[KB];
    float4 pj[KB];
    int3 cj[KB];
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      const uint32_t v = v0 + u;
      qs[u] = 0;
      bs[u] = b;
      if (v < ncand) {
        while (v >= cur_hi) {  // advance to the bin holding candidate v
          ++b;
          cur_lo = cur_hi;
#pragma unroll
          for (int k = 1; k < NB; ++k)
            if (k == b) {
              cur_beg = beg[k];
              cur_hi = cum[k];
            }
        }
        bs[u] = b;
        qs[u] = cur_beg + (v - cur_lo);
        load_record<DIM>(s, qs[u], pj[u], cj[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      if (v0 + u >= ncand) break;
      if (g.mode == kModeParticle) {
        const int3 want = add_wrapping(center, bin_delta<DIM>(bs[u]));
        if (cj[u].x != want.x || cj[u].y != want.y || cj[u].z != want.z) continue;
      }
      const float4 d = neighbor_delta<DIM>(g, pi, pj[u]);
      float r2 = d.x * d.x;
      r2 = r2 + d.y * d.y;
      if (DIM == 3) r2 = r2 + d.z * d.z;
      if (r2 < g.eps2) visit(qs[u], d, r2);
    }
  }
}

// for_each_neighbor with one candidate in flight and the per-bin starts and
// running counts in shared memory (`tab` is this thread's column of a
// [2 NB][stride] table): a bin change reads two words instead of selecting
// from register arrays, and the walk keeps 18 fewer registers live (2D
// density: 28 instead of 40, eight 256-thread blocks per SM instead of six;
// cfg2 density 0.134 vs 0.180 ms, cfg1 0.236 vs 0.293 ms).
template <int DIM, class Visit>
__device__ __forceinline__ void for_each_neighbor_tab(const GridParams& g, const SortedGrid& s,
                                                      uint32_t batch, float4 pi, int3 center,
                                                      uint32_t* tab, uint32_t stride,
                                                      Visit&& visit) {
  constexpr int NB = DIM == 3 ? 27 : 9;
  const uint32_t bin_base = batch * g.cells;
  uint32_t ncand = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int3 nc = add_wrapping(center, bin_delta<DIM>(b));
    const long long cell = cell_index<DIM>(g, nc.x, nc.y, nc.z);
    uint32_t lo = 0, cnt = 0;
    if (cell >= 0) {
      const uint32_t bin = bin_base + static_cast<uint32_t>(cell);
      lo = __ldg(s.bin_offsets + bin);
      const uint32_t hi = min(__ldg(s.bin_offsets + bin + 1), s.total);
      cnt = hi > lo ? hi - lo : 0u;
    }
    tab[b * stride] = lo;
    ncand += cnt;
    tab[(NB + b) * stride] = ncand;
  }
  int b = 0;
  uint32_t cur_beg = tab[0], cur_lo = 0, cur_hi = tab[NB * stride];
  for (uint32_t v = 0; v < ncand; ++v) {
    while (v >= cur_hi) {
      ++b;
      cur_lo = cur_hi;
      cur_beg = tab[b * stride];
      cur_hi = tab[(NB + b) * stride];
    }
    const uint32_t q = cur_beg + (v - cur_lo);
    float4 pj;
    int3 cj;
    load_record<DIM>(s, q, pj, cj);
    if (g.mode == kModeParticle) {
      const int3 want = add_wrapping(center, bin_delta<DIM>(b));
      if (cj.x != want.x || cj.y != want.y || cj.z != want.z) continue;
    }
    const float4 d = neighbor_delta<DIM>(g, pi, pj);
    float r2 = d.x * d.x;
    r2 = r2 + d.y * d.y;
    if (DIM == 3) r2 = r2 + d.z * d.z;
    if (r2 < g.eps2) visit(q, d, r2);
  }
}

// Per-warp staging of the cooperative walk: one 32-candidate window.
struct WarpWindow {
  float4 rec[32];     // candidate position; w = 1 when its cell is the visited cell
  uint32_t slot[32];  // candidate sorted slot
  float vol[32];      // payload of the perception walk
  uint32_t row[32];
};

// Lanes of this (converged, fully populated) warp with the same batch and
// cell as this lane; their neighbour candidate sequences are identical.
__device__ __forceinline__ uint32_t warp_cell_peers(uint32_t batch, int3 c) {
  return __match_any_sync(0xffffffffu, c.x) & __match_any_sync(0xffffffffu, c.y) &
         __match_any_sync(0xffffffffu, c.z) & __match_any_sync(0xffffffffu, batch);
}

// Number of distinct (batch, cell) groups among the warp's lanes.
__device__ __forceinline__ int warp_cell_groups(uint32_t peers) {
  const uint32_t lane = threadIdx.x & 31u;
  return __popc(__ballot_sync(0xffffffffu, lane == static_cast<uint32_t>(__ffs(peers) - 1)));
}

// for_each_neighbor, done by a whole warp for the lanes `peers` of one
// (batch, cell) group (the calling lanes' own group when mine is set): the
// candidate sequence of that cell is the same for every member, so lane L
// fetches candidate v0 + L of each 32-candidate window (record, exact-cell
// test, and stage(L, q) for a caller payload) into shared memory, and each
// member then tests the window's candidates in order from there.  The per-lane
// bin bookkeeping and record loads of for_each_neighbor are done once per
// candidate per warp instead of once per lane.  Same visits in the same
// order; visit(j, q, delta, r2) also receives the window index j.
template <int DIM, class Stage, class Visit>
__device__ __forceinline__ void walk_cell_warp(const GridParams& g, const SortedGrid& s,
                                               uint32_t batch, int3 center, bool mine, float4 pi,
                                               WarpWindow& win, Stage& stage, Visit& visit) {
  constexpr int NB = DIM == 3 ? 27 : 9;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t bin_base = batch * g.cells;
  uint32_t beg[NB], cum[NB];
  uint32_t ncand = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int3 nc = add_wrapping(center, bin_delta<DIM>(b));
    const long long cell = cell_index<DIM>(g, nc.x, nc.y, nc.z);
    uint32_t lo = 0, cnt = 0;
    if (cell >= 0) {
      const uint32_t bin = bin_base + static_cast<uint32_t>(cell);
      lo = __ldg(s.bin_offsets + bin);
      const uint32_t hi = min(__ldg(s.bin_offsets + bin + 1), s.total);
      cnt = hi > lo ? hi - lo : 0u;
    }
    beg[b] = lo;
    ncand += cnt;
    cum[b] = ncand;
  }
  int b = 0;
  uint32_t cur_beg = beg[0], cur_lo = 0, cur_hi = cum[0];
  for (uint32_t v0 = 0; v0 < ncand; v0 += 32) {
    const uint32_t v = v0 + lane;
    if (v < ncand) {
      while (v >= cur_hi) {  // advance to the bin holding candidate v
        ++b;
        cur_lo = cur_hi;
#pragma unroll
        for (int k = 1; k < NB; ++k)
          if (k == b) {
            cur_beg = beg[k];
            cur_hi = cum[k];
          }
      }
      const uint32_t q = cur_beg + (v - cur_lo);
      float4 pj;
      int3 cj;
      load_record<DIM>(s, q, pj, cj);
      bool match = true;
      if (g.mode == kModeParticle) {
        const int3 want = add_wrapping(center, bin_delta<DIM>(b));
        match = cj.x == want.x && cj.y == want.y && cj.z == want.z;
      }
      pj.w = match ? 1.0f : 0.0f;
      win.rec[lane] = pj;
      win.slot[lane] = q;
      if (match) stage(lane, q);
    }
    __syncwarp();
    if (mine) {
      const uint32_t nv = min(32u, ncand - v0);
      for (uint32_t j = 0; j < nv; ++j) {
        const float4 pj = win.rec[j];
        if (pj.w == 0.0f) continue;
        const float4 d = neighbor_delta<DIM>(g, pi, pj);
        float r2 = d.x * d.x;
        r2 = r2 + d.y * d.y;
        if (DIM == 3) r2 = r2 + d.z * d.z;
        if (r2 < g.eps2) visit(j, win.slot[j], d, r2);
      }
    }
    __syncwarp();
  }
}

// Every (batch, cell) group of the warp in turn (peers from warp_cell_peers):
// each lane visits exactly its own cell's neighbours, in walk order.
template <int DIM, class Stage, class Visit>
__device__ __forceinline__ void for_each_neighbor_warp(const GridParams& g, const SortedGrid& s,
                                                       uint32_t batch, float4 pi, int3 center,
                                                       uint32_t peers, WarpWindow& win,
                                                       Stage&& stage, Visit&& visit) {
  const uint32_t lane = threadIdx.x & 31u;
  uint32_t pending = 0xffffffffu;
  while (pending) {
    const int leader = __ffs(pending) - 1;
    const uint32_t members = __shfl_sync(0xffffffffu, peers, leader);
    pending &= ~members;
    const uint32_t gb = __shfl_sync(0xffffffffu, batch, leader);
    const int3 gc = make_int3(__shfl_sync(0xffffffffu, center.x, leader),
                              __shfl_sync(0xffffffffu, center.y, leader),
                              __shfl_sync(0xffffffffu, center.z, leader));
    walk_cell_warp<DIM>(g, s, gb, gc, ((members >> lane) & 1u) != 0, pi, win, stage, visit);
  }
}

// At most this many cell groups per warp take the cooperative walk (each
// group costs the warp one full walk); more diverse warps walk per lane.
constexpr int kMaxWarpCellGroups = 4;

// Neighbour lists recorded by the density pass: the sorted slots of a
// particle's hits in walk order, at most `cap` per particle; a particle with
// more hits stores count = cap + 1 and is walked again from the hashgrid.
// Hit e of slot q lives at slots[e * stride + q], so the threads of a warp
// (consecutive slots) write and read consecutive words.
struct HitLists {
  uint32_t* slots;   // [cap][stride]
  uint32_t* count;   // [B*N]
  int cap;
  uint32_t stride;   // >= B*N
};

// Sorted slot handled by processing index t.
__device__ __forceinline__ uint32_t slot_of(const SortedGrid& s, uint32_t t) {
  return s.order ? __ldg(s.order + t) : t;
}

// Cell coordinates of sorted slot q (from its record).
template <int DIM>
__device__ __forceinline__ int3 slot_cell(const SortedGrid& s, uint32_t q) {
  float4 p;
  int3 c;
  load_record<DIM>(s, q, p, c);
  return c;
}

}  // namespace npa
