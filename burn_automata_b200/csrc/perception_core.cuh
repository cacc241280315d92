// perception_core.cuh -- per-particle SPH perception shared by the standalone
// perception kernel and the fused step kernel.
//
// Restates, for one particle and one chunk of CH state channels:
//   density pass            forward.rs:145-160 (done by density_kernel)
//   second pass             forward.rs:249-295 (state_grad && density_grad) or
//                           blur_state :162, compute_state_gradient :297,
//                           moment_matrix :357, compute_density_gradient :335
//   moment correction       normalize.rs:93-118
//   gradient normalisation  normalize.rs:5-58
// One neighbour walk updates every accumulator; each accumulator receives its
// terms in the reference's walk order, so each sum is the reference's sum.
#pragma once

#include "npa_internal.h"

namespace npa {

struct PerceptionOut {
  float blur[8];
  float sgrad[8 * 3];  // [channel][axis]
  float dgrad[3];
};

// CH channels starting at c0 of particle slot q (original row `row`).
// `states` is the original-order state matrix [B*N][C]; `volume` is
// recip_finite(density) per sorted slot.  Channels >= C are left zero.
template <int CH>
__device__ __forceinline__ void perceive_chunk(const GridParams& g, const PerceptionParams& p,
                                               const SortedGrid& s, uint32_t batch, uint32_t q,
                                               float4 pi, int3 center, const float* __restrict__ states,
                                               int C, int c0, const float* __restrict__ volume,
                                               const float* si, PerceptionOut& out) {
  const int dim = g.dim;
  const bool both = p.state_grad && p.density_grad;
  const uint32_t batch_base = batch * s.n;
  float moment[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) moment[i] = 0.0f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    out.blur[c] = 0.0f;
#pragma unroll
    for (int a = 0; a < 3; ++a) out.sgrad[c * 3 + a] = 0.0f;
  }
#pragma unroll
  for (int a = 0; a < 3; ++a) out.dgrad[a] = 0.0f;

  for_each_neighbor(g, s, batch, pi, center, [&](uint32_t qj, float4 d, float r2) {
    const float vol = __ldg(volume + qj);
    const float smooth = poly6(g, r2);
    const float* sj = states + size_t(batch_base + __ldg(s.permutation + qj)) * C + c0;
    float sjv[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) sjv[c] = (c0 + c < C) ? __ldg(sj + c) : 0.0f;
    if (both) {
#pragma unroll
      for (int c = 0; c < CH; ++c) out.blur[c] = out.blur[c] + sjv[c] * smooth * vol;
    } else {
      const float w = smooth * vol;
#pragma unroll
      for (int c = 0; c < CH; ++c) out.blur[c] = out.blur[c] + sjv[c] * w;
    }
    if (qj == q) return;
    const float dv[3] = {d.x, d.y, d.z};
    if (p.density_grad) {
      const float m1 = spiky_mag(g, r2, 1.0f);
#pragma unroll
      for (int a = 0; a < 3; ++a)
        if (a < dim) out.dgrad[a] = out.dgrad[a] + m1 * dv[a];
    }
    if (p.state_grad) {
      const float mv = spiky_mag(g, r2, vol);
      float gv[3];
#pragma unroll
      for (int a = 0; a < 3; ++a) gv[a] = mv * dv[a];
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const float diff = sjv[c] - si[c];
#pragma unroll
        for (int a = 0; a < 3; ++a)
          if (a < dim) out.sgrad[c * 3 + a] = out.sgrad[c * 3 + a] + diff * gv[a];
      }
      if (p.hybrid) {
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int col = 0; col < 3; ++col)
            if (r < dim && col < dim) moment[r * dim + col] = moment[r * dim + col] + dv[r] * gv[col];
      }
    }
  });

  if (p.state_grad) {
    if (p.hybrid) {
      float inv[9];
      safe_inverse_symmetric(moment, dim, inv);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        float corrected[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int oa = 0; oa < 3; ++oa)
#pragma unroll
          for (int ia = 0; ia < 3; ++ia)
            if (oa < dim && ia < dim)
              corrected[oa] = corrected[oa] + out.sgrad[c * 3 + ia] * inv[ia * dim + oa];
#pragma unroll
        for (int a = 0; a < 3; ++a) out.sgrad[c * 3 + a] = corrected[a];
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
#pragma unroll
      for (int a = 0; a < 3; ++a) out.sgrad[c * 3 + a] = out.sgrad[c * 3 + a] * p.state_scale;
      if (p.log_norm_grad) log_normalize(&out.sgrad[c * 3], dim);
    }
  }
  if (p.density_grad) {
#pragma unroll
    for (int a = 0; a < 3; ++a) out.dgrad[a] = out.dgrad[a] * p.density_scale;
    if (p.log_norm_density_grad) log_normalize(out.dgrad, dim);
  }
}

}  // namespace npa
