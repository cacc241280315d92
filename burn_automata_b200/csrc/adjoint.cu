// adjoint.cu -- perceive_adjoint_with_options
// (crates/burn_automata_kernels/src/reference/adjoint.rs:28-489): the
// reverse-mode derivative of the perception features with respect to the
// particles' states and positions, for a given feature adjoint.
//
// The reference runs one serial loop over particles that scatters into its
// neighbours' adjoints.  Here every particle is a thread and the scatter is
// done with float atomics, in three passes:
//   adjoint_prep_kernel     per particle: the raw state gradient and moment
//                           matrix (one walk), then the per-channel adjoint
//                           of the moment correction / scaling / log-norm,
//                           the moment matrix's adjoint and the density
//                           gradient's (one more walk) -> scratch rows
//   adjoint_scatter_kernel  per particle, one walk: blur, state-gradient,
//                           moment and density-gradient terms into the state,
//                           position and density adjoints of both ends
//   adjoint_density_kernel  per particle with a nonzero density adjoint, one
//                           walk: the density kernel's position terms
// Each term is the reference's expression; only the order in which the terms
// of one adjoint entry are added differs (atomics), so results agree to f32
// summation error rather than bit for bit.
#include "npa_internal.h"

namespace npa {
namespace {

// smoothing_poly6_delta_adjoint (kernels.rs:62-79).
__device__ __forceinline__ void poly6_delta_adjoint(const GridParams& g, const float (&d)[3],
                                                    float r2, float out_adj, float (&out)[3],
                                                    int dim) {
  out[0] = out[1] = out[2] = 0.0f;
  if (r2 >= g.eps2) return;
  const float x = g.eps2 - r2;
  const float dk = -3.0f * g.poly6_norm * x * x;
  for (int a = 0; a < dim; ++a) out[a] = out_adj * dk * 2.0f * d[a];
}

// spiky_gradient_delta_adjoint (kernels.rs:100-126).
__device__ __forceinline__ void spiky_delta_adjoint(const GridParams& g, const float (&d)[3],
                                                    float r2, float coeff, const float (&adj)[3],
                                                    float (&out)[3], int dim) {
  out[0] = out[1] = out[2] = 0.0f;
  if (r2 <= 0.0f || r2 >= g.eps2) return;
  const float r = sqrtf(r2);
  const float norm = coeff * g.spiky_norm * 3.0f;
  const float t = g.eps - r;
  const float scale = norm * (t * t) / r;
  const float dscale_dr = norm * (1.0f - (g.eps * g.eps) / r2);
  float dot = 0.0f;
  for (int a = 0; a < dim; ++a) dot = dot + adj[a] * d[a];
  for (int a = 0; a < dim; ++a) out[a] = scale * adj[a] + dscale_dr * dot * d[a] / r;
}

// log_normalize_adjoint (normalize.rs:71-91) from a zero input adjoint.
__device__ __forceinline__ void log_normalize_adjoint(const float (&in)[3], const float* out_adj,
                                                      float (&in_adj)[3], int dim,
                                                      const Log1pTable& l1p) {
  const float e = 1.0e-6f;
  float s = 0.0f;
  for (int a = 0; a < dim; ++a) s = s + in[a] * in[a];
  const float norm = fmaxf(sqrtf(s + e * e), e);
  const float l = log1p_host(norm, l1p);
  const float scale = l / norm;
  const float dscale = (norm / (1.0f + norm) - l) / (norm * norm);
  float dot = 0.0f;
  for (int a = 0; a < dim; ++a) dot = dot + in[a] * out_adj[a];
  const float radial = dscale * dot / norm;
  for (int a = 0; a < dim; ++a) in_adj[a] = 0.0f + (scale * out_adj[a] + radial * in[a]);
}

// accumulate_volume_density_adjoint (adjoint.rs:425-435), atomically.
__device__ __forceinline__ void volume_density_adjoint(const float* density, float* dens_adj,
                                                       size_t j, float volume_adjoint) {
  const float rho = density[j];
  if (fabsf(rho) <= 1.0e-20f || !isfinite(rho)) return;
  atomicAdd(dens_adj + j, -(volume_adjoint / (rho * rho)));
}

__device__ __forceinline__ void spiky_vec(const GridParams& g, const float (&d)[3], float r2,
                                          float coeff, float (&out)[3]) {
  const float m = spiky_mag(g, r2, coeff);
  out[0] = m * d[0];
  out[1] = m * d[1];
  out[2] = m * d[2];
}

// Per-particle scratch rows (floats): raw gradient [C*D], its adjoint [C*D],
// moment adjoint [9], density-gradient adjoint [3].
struct AdjScratch {
  float* raw;
  float* raw_adj;
  float* m_adj;
  float* d_adj;
};

struct AdjArgs {
  GridParams g;
  PerceptionParams p;
  SortedGrid s;
  const uint32_t* inverse;  // [B*N] local sorted slot of each particle
  const float* states;      // [B*N][C]
  const float* density;     // [B*N] caller order
  const float* fa;          // feature adjoint [B*N][F]
  int C;
  uint32_t total;
  AdjScratch sc;
  float* state_adj;  // [B*N][C]
  float* pos_adj;    // [B*N][4]
  float* dens_adj;   // [B*N]
};

// Walks idx's neighbours: visit(j (caller order), delta[3], r2).
template <int DIM, class Visit>
__device__ __forceinline__ void walk(const AdjArgs& A, uint32_t idx, float4& pi, Visit&& visit) {
  const uint32_t batch = idx / A.s.n;
  const uint32_t base = batch * A.s.n;
  const uint32_t q = base + A.inverse[idx];
  int3 c;
  load_record<DIM>(A.s, q, pi, c);
  for_each_neighbor<DIM, 4>(A.g, A.s, batch, pi, c, [&](uint32_t qj, float4 d4, float r2) {
    const float d[3] = {d4.x, d4.y, d4.z};
    visit(base + __ldg(A.s.permutation + qj), d, r2);
  });
}

template <int DIM>
__global__ void __launch_bounds__(128) adjoint_prep_kernel(AdjArgs A) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= A.total) return;
  const int C = A.C;
  const size_t gd = size_t(C) * DIM;
  const float* fa = A.fa + size_t(idx) * A.p.feature_dims;
  const float* si = A.states + size_t(idx) * C;
  for (int ch = 0; ch < C; ++ch) atomicAdd(A.state_adj + size_t(idx) * C + ch, fa[ch]);
  float4 pi;
  size_t cur = 2 * size_t(C);
  if (A.p.state_grad) {
    float* raw = A.sc.raw + size_t(idx) * gd;
    float* raw_adj = A.sc.raw_adj + size_t(idx) * gd;
    for (size_t k = 0; k < gd; ++k) raw[k] = 0.0f;
    float moment[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    walk<DIM>(A, idx, pi, [&](size_t j, const float (&d)[3], float r2) {
      if (j == idx) return;
      float gv[3];
      spiky_vec(A.g, d, r2, recip_finite(A.density[j]), gv);
      const float* sj = A.states + j * C;
      for (int ch = 0; ch < C; ++ch) {
        const float diff = sj[ch] - si[ch];
        for (int a = 0; a < DIM; ++a) raw[ch * DIM + a] = raw[ch * DIM + a] + diff * gv[a];
      }
      if (A.p.hybrid)
        for (int r = 0; r < DIM; ++r)
          for (int c2 = 0; c2 < DIM; ++c2)
            moment[r * DIM + c2] = moment[r * DIM + c2] + d[r] * gv[c2];
    });
    float inv[9];
    if (A.p.hybrid) safe_inverse_symmetric(moment, DIM, inv);
    float inv_adj[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    const float* gadj = fa + cur;
    for (int ch = 0; ch < C; ++ch) {
      float corrected[3] = {0.0f, 0.0f, 0.0f};
      for (int a = 0; a < DIM; ++a) corrected[a] = raw[ch * DIM + a];
      if (A.p.hybrid) {
        float mc[3] = {0.0f, 0.0f, 0.0f};
        for (int oa = 0; oa < DIM; ++oa)
          for (int ia = 0; ia < DIM; ++ia) mc[oa] = mc[oa] + corrected[ia] * inv[ia * DIM + oa];
        for (int a = 0; a < 3; ++a) corrected[a] = mc[a];
      }
      float nin[3] = {0.0f, 0.0f, 0.0f};
      for (int a = 0; a < DIM; ++a) nin[a] = corrected[a] * A.p.state_scale;
      float cadj[3] = {0.0f, 0.0f, 0.0f};
      if (A.p.log_norm_grad)
        log_normalize_adjoint(nin, gadj + ch * DIM, cadj, DIM, A.p.l1p);
      else
        for (int a = 0; a < DIM; ++a) cadj[a] = gadj[ch * DIM + a];
      for (int a = 0; a < DIM; ++a) cadj[a] = cadj[a] * A.p.state_scale;
      float radj[3] = {0.0f, 0.0f, 0.0f};
      if (A.p.hybrid) {
        for (int ia = 0; ia < DIM; ++ia)
          for (int oa = 0; oa < DIM; ++oa) radj[ia] = radj[ia] + cadj[oa] * inv[ia * DIM + oa];
        for (int ia = 0; ia < DIM; ++ia)
          for (int oa = 0; oa < DIM; ++oa)
            inv_adj[ia * DIM + oa] = inv_adj[ia * DIM + oa] + raw[ch * DIM + ia] * cadj[oa];
      } else {
        for (int a = 0; a < DIM; ++a) radj[a] = cadj[a];
      }
      for (int a = 0; a < DIM; ++a) raw_adj[ch * DIM + a] = radj[a];
    }
    float* m_adj = A.sc.m_adj + size_t(idx) * 9;
    for (int k = 0; k < 9; ++k) m_adj[k] = 0.0f;
    if (A.p.hybrid) {
      // inverse_matrix_adjoint (adjoint.rs:450-469)
      for (int row = 0; row < DIM; ++row)
        for (int col = 0; col < DIM; ++col) {
          float value = 0.0f;
          for (int ir = 0; ir < DIM; ++ir)
            for (int ic = 0; ic < DIM; ++ic)
              value = value + inv[ir * DIM + row] * inv_adj[ir * DIM + ic] * inv[col * DIM + ic];
          m_adj[row * DIM + col] = 0.0f - value;
        }
    }
    cur += gd;
  }
  if (A.p.density_grad) {
    float rawd[3] = {0.0f, 0.0f, 0.0f};
    walk<DIM>(A, idx, pi, [&](size_t j, const float (&d)[3], float r2) {
      if (j == idx) return;
      float g1[3];
      spiky_vec(A.g, d, r2, 1.0f, g1);
      for (int a = 0; a < DIM; ++a) rawd[a] = rawd[a] + g1[a];
    });
    const float* dadj = fa + cur;
    float nin[3] = {0.0f, 0.0f, 0.0f}, radj[3] = {0.0f, 0.0f, 0.0f};
    for (int a = 0; a < DIM; ++a) nin[a] = rawd[a] * A.p.density_scale;
    if (A.p.log_norm_density_grad) {
      log_normalize_adjoint(nin, dadj, radj, DIM, A.p.l1p);
      for (int a = 0; a < DIM; ++a) radj[a] = radj[a] * A.p.density_scale;
    } else {
      for (int a = 0; a < DIM; ++a) radj[a] = dadj[a] * A.p.density_scale;
    }
    float* out = A.sc.d_adj + size_t(idx) * 3;
    out[0] = radj[0];
    out[1] = radj[1];
    out[2] = radj[2];
    cur += DIM;
  }
  if (A.p.position_features)
    for (int a = 0; a < DIM; ++a) atomicAdd(A.pos_adj + size_t(idx) * 4 + a, fa[cur + a]);
}

template <int DIM>
__global__ void __launch_bounds__(128) adjoint_scatter_kernel(AdjArgs A) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= A.total) return;
  const int C = A.C;
  const size_t gd = size_t(C) * DIM;
  const float* fa = A.fa + size_t(idx) * A.p.feature_dims;
  const float* badj = fa + C;
  const float* si = A.states + size_t(idx) * C;
  const float* raw_adj = A.sc.raw_adj + size_t(idx) * gd;
  const float* m_adj = A.sc.m_adj + size_t(idx) * 9;
  float dradj[3] = {0.0f, 0.0f, 0.0f};
  if (A.p.density_grad)
    for (int a = 0; a < 3; ++a) dradj[a] = A.sc.d_adj[size_t(idx) * 3 + a];
  float own_pos[3] = {0.0f, 0.0f, 0.0f};
  auto move = [&](size_t j, const float (&da)[3]) {
    for (int a = 0; a < DIM; ++a) {
      atomicAdd(A.pos_adj + j * 4 + a, da[a]);
      own_pos[a] = own_pos[a] - da[a];
    }
  };
  float4 pi;
  walk<DIM>(A, idx, pi, [&](size_t j, const float (&d)[3], float r2) {
    const float vol = recip_finite(A.density[j]);
    const float* sj = A.states + j * C;
    {  // accumulate_blurred_state_adjoint (adjoint.rs:138-166)
      const float kern = poly6(A.g, r2);
      const float weight = kern * vol;
      float wadj = 0.0f;
      for (int ch = 0; ch < C; ++ch) {
        atomicAdd(A.state_adj + j * C + ch, badj[ch] * weight);
        wadj = wadj + badj[ch] * sj[ch];
      }
      float da[3];
      poly6_delta_adjoint(A.g, d, r2, wadj * vol, da, DIM);
      move(j, da);
      volume_density_adjoint(A.density, A.dens_adj, j, wadj * kern);
    }
    if (j == idx) return;
    float vg[3], ug[3];
    if (A.p.state_grad) {  // accumulate_state_gradient_adjoint, second walk (adjoint.rs:271-342)
      spiky_vec(A.g, d, r2, vol, vg);
      spiky_vec(A.g, d, r2, 1.0f, ug);
      for (int ch = 0; ch < C; ++ch) {
        const float diff = sj[ch] - si[ch];
        float contrib = 0.0f;
        for (int a = 0; a < DIM; ++a) contrib = contrib + raw_adj[ch * DIM + a] * vg[a];
        atomicAdd(A.state_adj + j * C + ch, contrib);
        atomicAdd(A.state_adj + size_t(idx) * C + ch, -contrib);
        float gadj[3] = {0.0f, 0.0f, 0.0f};
        for (int a = 0; a < DIM; ++a) gadj[a] = raw_adj[ch * DIM + a] * diff;
        float da[3];
        spiky_delta_adjoint(A.g, d, r2, vol, gadj, da, DIM);
        move(j, da);
        float vadj = 0.0f;
        for (int a = 0; a < DIM; ++a) vadj = vadj + gadj[a] * ug[a];
        volume_density_adjoint(A.density, A.dens_adj, j, vadj);
      }
      if (A.p.hybrid) {
        float dda[3] = {0.0f, 0.0f, 0.0f}, gadj[3] = {0.0f, 0.0f, 0.0f};
        for (int row = 0; row < DIM; ++row)
          for (int col = 0; col < DIM; ++col) {
            const float adj = m_adj[row * DIM + col];
            dda[row] = dda[row] + adj * vg[col];
            gadj[col] = gadj[col] + adj * d[row];
          }
        float gda[3];
        spiky_delta_adjoint(A.g, d, r2, vol, gadj, gda, DIM);
        for (int a = 0; a < DIM; ++a) dda[a] = dda[a] + gda[a];
        move(j, dda);
        float vadj = 0.0f;
        for (int a = 0; a < DIM; ++a) vadj = vadj + gadj[a] * ug[a];
        volume_density_adjoint(A.density, A.dens_adj, j, vadj);
      }
    }
    if (A.p.density_grad) {  // accumulate_density_gradient_position_adjoint (adjoint.rs:345-392)
      float da[3];
      spiky_delta_adjoint(A.g, d, r2, 1.0f, dradj, da, DIM);
      move(j, da);
    }
  });
  for (int a = 0; a < DIM; ++a) atomicAdd(A.pos_adj + size_t(idx) * 4 + a, own_pos[a]);
}

// accumulate_density_kernel_position_adjoint (adjoint.rs:394-412).
template <int DIM>
__global__ void __launch_bounds__(128) adjoint_density_kernel(AdjArgs A) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= A.total) return;
  const float adj = A.dens_adj[idx];
  if (adj == 0.0f) return;
  float own_pos[3] = {0.0f, 0.0f, 0.0f};
  float4 pi;
  walk<DIM>(A, idx, pi, [&](size_t j, const float (&d)[3], float r2) {
    float da[3];
    poly6_delta_adjoint(A.g, d, r2, adj, da, DIM);
    for (int a = 0; a < DIM; ++a) {
      atomicAdd(A.pos_adj + j * 4 + a, da[a]);
      own_pos[a] = own_pos[a] - da[a];
    }
  });
  for (int a = 0; a < DIM; ++a) atomicAdd(A.pos_adj + size_t(idx) * 4 + a, own_pos[a]);
}

}  // namespace

size_t adjoint_scratch_floats(uint32_t total, int state_dims, int dim) {
  return size_t(total) * (2 * size_t(state_dims) * dim + 9 + 3);
}

npa_status launch_perception_adjoint(const GridParams& g, const PerceptionParams& p,
                                     const SortedGrid& s, const uint32_t* inverse,
                                     uint32_t batch, const float* states, int state_dims,
                                     const float* density, const float* feature_adjoint,
                                     float* scratch, float* state_adjoint, float4* position_adjoint,
                                     float* density_adjoint, cudaStream_t stream) {
  const uint32_t total = batch * s.n;
  if (total == 0) return NPA_OK;
  Log1pTable l1p{};
  if (p.log_norm_grad || p.log_norm_density_grad) NPA_TRY(device_log1p_table(&l1p, stream));
  if (state_dims > 0)
    NPA_CUDA(cudaMemsetAsync(state_adjoint, 0, size_t(total) * state_dims * 4, stream),
             "cudaMemsetAsync");
  NPA_CUDA(cudaMemsetAsync(position_adjoint, 0, size_t(total) * 16, stream), "cudaMemsetAsync");
  NPA_CUDA(cudaMemsetAsync(density_adjoint, 0, size_t(total) * 4, stream), "cudaMemsetAsync");
  AdjArgs A;
  A.g = g;
  A.p = p;
  A.p.l1p = l1p;
  A.s = s;
  A.inverse = inverse;
  A.states = states;
  A.density = density;
  A.fa = feature_adjoint;
  A.C = state_dims;
  A.total = total;
  const size_t gd = size_t(total) * state_dims * g.dim;
  A.sc.raw = scratch;
  A.sc.raw_adj = scratch + gd;
  A.sc.m_adj = scratch + 2 * gd;
  A.sc.d_adj = scratch + 2 * gd + size_t(total) * 9;
  A.state_adj = state_adjoint;
  A.pos_adj = reinterpret_cast<float*>(position_adjoint);
  A.dens_adj = density_adjoint;
  const unsigned blocks = grid_for(total, 128);
  if (g.dim == 2) {
    adjoint_prep_kernel<2><<<blocks, 128, 0, stream>>>(A);
    NPA_TRY(after_launch("adjoint_prep_kernel"));
    adjoint_scatter_kernel<2><<<blocks, 128, 0, stream>>>(A);
    NPA_TRY(after_launch("adjoint_scatter_kernel"));
    adjoint_density_kernel<2><<<blocks, 128, 0, stream>>>(A);
  } else {
    adjoint_prep_kernel<3><<<blocks, 128, 0, stream>>>(A);
    NPA_TRY(after_launch("adjoint_prep_kernel"));
    adjoint_scatter_kernel<3><<<blocks, 128, 0, stream>>>(A);
    NPA_TRY(after_launch("adjoint_scatter_kernel"));
    adjoint_density_kernel<3><<<blocks, 128, 0, stream>>>(A);
  }
  return after_launch("adjoint_density_kernel");
}

}  // namespace npa
