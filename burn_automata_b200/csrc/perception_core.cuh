// perception_core.cuh -- per-particle SPH perception shared by the perception kernels.
//
// Restates, for one particle and one chunk of CH state channels:
//   second pass             forward.rs:249-295 (state_grad && density_grad) or
//                           blur_state :162, compute_state_gradient :297,
//                           moment_matrix :357, compute_density_gradient :335
//   moment correction       normalize.rs:93-118
//   gradient normalisation  normalize.rs:5-58
// One neighbour walk updates every accumulator; each accumulator receives its
// terms in the reference's walk order, so each sum is the reference's sum.
// DIM and CH are compile-time so every accumulator lives in registers.
#pragma once

#include "npa_internal.h"

namespace npa {

template <int DIM, int CH>
struct PerceptionAcc {
  float blur[CH];
  float sgrad[CH][DIM];
  float dgrad[DIM];
};

// log_normalize_vector (normalize.rs:60-69) on every channel of a chunk:
//   norm = max(sqrt(|v|^2 + 1e-12), 1e-6);  v *= ln_1p(norm) / norm
// with the host libm's log1pf (log1p_host_word).  The norms come first and
// their lookup words are loaded together, so the loads' latencies overlap;
// the f64 log1p, the correction and the division stay out of line (one copy
// serves every channel: inlined per channel they crowded the perception
// kernels out of the instruction cache, cfg2 perception 0.437 -> 0.406 ms).
static __device__ __noinline__ float log_norm_scale(float norm, uint32_t word,
                                                  const Log1pTable t) {
  return log1p_host_word(norm, word, t) / norm;
}

template <int DIM, int N>
__device__ __forceinline__ void log_normalize_rows(float (&v)[N][DIM], const Log1pTable& t) {
  const float e = 1.0e-6f;
  float norm[N];
  uint32_t word[N];
#pragma unroll
  for (int c = 0; c < N; ++c) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < DIM; ++i) s = s + v[c][i] * v[c][i];
    norm[c] = fmaxf(sqrtf(s + e * e), e);
  }
#pragma unroll
  for (int c = 0; c < N; ++c) word[c] = log1p_word(norm[c], t);
#pragma unroll
  for (int c = 0; c < N; ++c) {
    const float scale = log_norm_scale(norm[c], word[c], t);
#pragma unroll
    for (int i = 0; i < DIM; ++i) v[c][i] = v[c][i] * scale;
  }
}

// Accumulators of one particle's chunk plus the moment matrix.
template <int DIM, int CH>
struct ChunkState {
  PerceptionAcc<DIM, CH> acc;
  float moment[DIM][DIM];
};

template <int DIM, int CH>
__device__ __forceinline__ void chunk_init(ChunkState<DIM, CH>& st) {
#pragma unroll
  for (int r = 0; r < DIM; ++r)
#pragma unroll
    for (int c = 0; c < DIM; ++c) st.moment[r][c] = 0.0f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    st.acc.blur[c] = 0.0f;
#pragma unroll
    for (int a = 0; a < DIM; ++a) st.acc.sgrad[c][a] = 0.0f;
  }
#pragma unroll
  for (int a = 0; a < DIM; ++a) st.acc.dgrad[a] = 0.0f;
}

// Loads CH channels of state row `row` (float4 when aligned and whole).
template <int CH>
__device__ __forceinline__ void load_row(const float* __restrict__ states, size_t row, int C,
                                         int c0, bool vec4, float (&out)[CH]) {
  const float* sj = states + row * C + c0;
  if (vec4) {
#pragma unroll
    for (int c = 0; c < CH; c += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(sj + c));
      out[c] = v.x;
      out[c + 1] = v.y;
      out[c + 2] = v.z;
      out[c + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int c = 0; c < CH; ++c) out[c] = (c0 + c < C) ? __ldg(sj + c) : 0.0f;
  }
}

// One neighbour's terms (second_pass_particle, forward.rs:249-295, or the
// separate passes of the other branch), added in the reference's order.
// OPT = 1 fixes the rollout models' options at compile time (state gradient
// and hybrid moment on, density gradient off; p must hold the same), OPT = 2
// the full growing_2d set (state and density gradients, hybrid moment), which
// drops the per-pair option branches; OPT = 0 reads them from p.
template <int DIM, int CH, int OPT = 0>
__device__ __forceinline__ void chunk_add(const GridParams& g, const PerceptionParams& p,
                                          bool self, float4 d, float r2, float vol,
                                          const float (&sjv)[CH], const float (&si)[CH],
                                          ChunkState<DIM, CH>& st) {
  const bool sg = OPT ? true : p.state_grad;
  const bool dg = OPT == 2 ? true : (OPT ? false : p.density_grad);
  const bool hy = OPT ? true : p.hybrid;
  const float smooth = poly6(g, r2);
  if (sg && dg) {
#pragma unroll
    for (int c = 0; c < CH; ++c) st.acc.blur[c] = st.acc.blur[c] + sjv[c] * smooth * vol;
  } else {
    const float w = smooth * vol;
#pragma unroll
    for (int c = 0; c < CH; ++c) st.acc.blur[c] = st.acc.blur[c] + sjv[c] * w;
  }
  if (self) return;
  const float dv[3] = {d.x, d.y, d.z};
  if (dg) {
    const float m1 = spiky_mag(g, r2, 1.0f);
#pragma unroll
    for (int a = 0; a < DIM; ++a) st.acc.dgrad[a] = st.acc.dgrad[a] + m1 * dv[a];
  }
  if (sg) {
    const float mv = spiky_mag(g, r2, vol);
    float gv[DIM];
#pragma unroll
    for (int a = 0; a < DIM; ++a) gv[a] = mv * dv[a];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const float diff = sjv[c] - si[c];
#pragma unroll
      for (int a = 0; a < DIM; ++a) st.acc.sgrad[c][a] = st.acc.sgrad[c][a] + diff * gv[a];
    }
    if (hy) {
#pragma unroll
      for (int r = 0; r < DIM; ++r)
#pragma unroll
        for (int col = 0; col < DIM; ++col)
          st.moment[r][col] = st.moment[r][col] + dv[r] * gv[col];
    }
  }
}

// Moment correction (normalize.rs:93-118) and gradient normalisation (:5-58).
template <int DIM, int CH, int OPT = 0>
__device__ __forceinline__ void chunk_finish(const PerceptionParams& p, ChunkState<DIM, CH>& st) {
  const bool sg = OPT ? true : p.state_grad;
  const bool dg = OPT == 2 ? true : (OPT ? false : p.density_grad);
  const bool hy = OPT ? true : p.hybrid;
  if (sg) {
    if (hy) {
      float m9[9], inv[9];
#pragma unroll
      for (int r = 0; r < DIM; ++r)
#pragma unroll
        for (int c = 0; c < DIM; ++c) m9[r * DIM + c] = st.moment[r][c];
      safe_inverse_symmetric(m9, DIM, inv);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        float corrected[DIM];
#pragma unroll
        for (int oa = 0; oa < DIM; ++oa) {
          corrected[oa] = 0.0f;
#pragma unroll
          for (int ia = 0; ia < DIM; ++ia)
            corrected[oa] = corrected[oa] + st.acc.sgrad[c][ia] * inv[ia * DIM + oa];
        }
#pragma unroll
        for (int a = 0; a < DIM; ++a) st.acc.sgrad[c][a] = corrected[a];
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
      for (int a = 0; a < DIM; ++a) st.acc.sgrad[c][a] = st.acc.sgrad[c][a] * p.state_scale;
    if (p.log_norm_grad) log_normalize_rows<DIM, CH>(st.acc.sgrad, p.l1p);
  }
  if (dg) {
#pragma unroll
    for (int a = 0; a < DIM; ++a) st.acc.dgrad[a] = st.acc.dgrad[a] * p.density_scale;
    if (p.log_norm_density_grad) {
      float row[1][DIM];
#pragma unroll
      for (int a = 0; a < DIM; ++a) row[0][a] = st.acc.dgrad[a];
      log_normalize_rows<DIM, 1>(row, p.l1p);
#pragma unroll
      for (int a = 0; a < DIM; ++a) st.acc.dgrad[a] = row[0][a];
    }
  }
}

// CH channels [c0, c0 + CH) of the particle in sorted slot q.  `states` is the
// caller-order state matrix [B*N][C]; `volume` is recip_finite(density) per
// sorted slot; `si` holds the particle's own channels.  Channels >= C stay 0.
// The neighbours come from the density pass's hit list when it holds them all,
// otherwise from a fresh hashgrid walk; both give the walk order.  `hit_row`
// is the processing index under which the density pass wrote the particle's
// hit list.  `win` is set (warp-uniformly) when the warp's lanes fall into few
// (batch, cell) groups (`peers`: this lane's group): then a walk, if any lane
// needs one, is the warp-cooperative walk of each group.
template <int DIM, int CH, int OPT = 0, bool PIPE = false>
__device__ __forceinline__ void perceive_chunk(const GridParams& g, const PerceptionParams& p,
                                               const SortedGrid& s, const HitLists& hl,
                                               uint32_t batch, uint32_t q, uint32_t hit_row,
                                               float4 pi,
                                               int3 center, const float* __restrict__ states,
                                               int C, int c0, const float* __restrict__ volume,
                                               const float (&si)[CH],
                                               PerceptionAcc<DIM, CH>& out,
                                               WarpWindow* win = nullptr, uint32_t peers = 0) {
  const uint32_t batch_base = batch * s.n;
  const bool vec4 = p.vec_states && ((C & 3) == 0) && ((c0 & 3) == 0) && (CH % 4 == 0) &&
                    (c0 + CH <= C);
  ChunkState<DIM, CH> st;
  chunk_init(st);
  const uint32_t nh = hl.slots ? __ldg(hl.count + hit_row) : uint32_t(hl.cap + 1);
  if (win && __any_sync(0xffffffffu, nh > uint32_t(hl.cap))) {
    for_each_neighbor_warp<DIM>(
        g, s, batch, pi, center, peers, *win,
        [&](uint32_t lane, uint32_t qn) {
          win->vol[lane] = __ldg(volume + qn);
          // qn is in the walked group's rollout, which need not be this lane's
          win->row[lane] = qn / s.n * s.n + __ldg(s.permutation + qn);
        },
        [&](uint32_t j, uint32_t qn, float4 d, float r2) {
          float sjv[CH];
          load_row<CH>(states, win->row[j], C, c0, vec4, sjv);
          chunk_add<DIM, CH, OPT>(g, p, qn == q, d, r2, win->vol[j], sjv, si, st);
        });
  } else if (nh <= uint32_t(hl.cap)) {
    const uint32_t* list = hl.slots + hit_row;
    // PIPE: the list entries of the next pair are loaded one pair ahead, so
    // an iteration waits on two dependent round trips (record / volume /
    // permutation, then state rows) instead of three.  Measured on cfg2's
    // step perception: 0.407 vs 0.433 ms; the API perception kernel (generic
    // options, more registers live) keeps the plain loop.
    uint32_t qn[2] = {q, q};
    if (PIPE) {
#pragma unroll
      for (int u = 0; u < 2; ++u)
        qn[u] = (uint32_t(u) < nh) ? __ldg(list + size_t(u) * hl.stride) : q;
    }
    for (uint32_t e0 = 0; e0 < nh; e0 += 2) {
      uint32_t qj[2];
      float4 pj[2];
      int3 cj[2];
      float vol[2];
      uint32_t prow[2];
      if (PIPE) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          qj[u] = qn[u];
          qn[u] = (e0 + 2 + u < nh) ? __ldg(list + size_t(e0 + 2 + u) * hl.stride) : q;
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!PIPE) qj[u] = (e0 + u < nh) ? __ldg(list + size_t(e0 + u) * hl.stride) : q;
        load_record<DIM>(s, qj[u], pj[u], cj[u]);
        vol[u] = __ldg(volume + qj[u]);
        prow[u] = batch_base + __ldg(s.permutation + qj[u]);
      }
      float sj[2][CH];
#pragma unroll
      for (int u = 0; u < 2; ++u) load_row<CH>(states, prow[u], C, c0, vec4, sj[u]);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (e0 + u >= nh) break;
        const float4 d = neighbor_delta<DIM>(g, pi, pj[u]);
        float r2 = d.x * d.x;
        r2 = r2 + d.y * d.y;
        if (DIM == 3) r2 = r2 + d.z * d.z;
        chunk_add<DIM, CH, OPT>(g, p, qj[u] == q, d, r2, vol[u], sj[u], si, st);
      }
    }
  } else {
    for_each_neighbor<DIM>(g, s, batch, pi, center, [&](uint32_t qn, float4 d, float r2) {
      float sjv[CH];
      load_row<CH>(states, batch_base + __ldg(s.permutation + qn), C, c0, vec4, sjv);
      chunk_add<DIM, CH, OPT>(g, p, qn == q, d, r2, __ldg(volume + qn), sjv, si, st);
    });
  }
  chunk_finish<DIM, CH, OPT>(p, st);
  out = st.acc;
}

// Visits the feature row [s | blur | grad (c*DIM+a) | dgrad? | pos?] of one
// chunk as emit(feature_index, value) (forward.rs:100-133).
template <int DIM, int CH, class Emit>
__device__ __forceinline__ void emit_features(const PerceptionParams& p, int C, int c0, bool lead,
                                              const float (&si)[CH],
                                              const PerceptionAcc<DIM, CH>& a, float4 pi,
                                              Emit&& emit) {
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int ch = c0 + c;
    if (ch < C) {
      emit(ch, si[c]);
      emit(C + ch, a.blur[c]);
      if (p.state_grad) {
#pragma unroll
        for (int d = 0; d < DIM; ++d) emit(2 * C + ch * DIM + d, a.sgrad[c][d]);
      }
    }
  }
  if (lead) {
    int cursor = 2 * C + (p.state_grad ? C * DIM : 0);
    if (p.density_grad) {
#pragma unroll
      for (int d = 0; d < DIM; ++d) emit(cursor + d, a.dgrad[d]);
      cursor += DIM;
    }
    if (p.position_features) {
      const float pv[3] = {pi.x, pi.y, pi.z};
#pragma unroll
      for (int d = 0; d < DIM; ++d) emit(cursor + d, pv[d]);
    }
  }
}

}  // namespace npa
