// decode.cu -- decode_gaussians_3d (crates/burn_automata_kernels/src/gaussian.rs:53-223).
//
// One thread per particle writes one record
//   [position_visibility 4][rotation 4][scale_opacity 4][spherical_harmonic 3*k]
// exp / tanh / the sigmoid's exp are evaluated in f64 and rounded once to f32;
// the reference calls the host libm's expf / tanhf.
#include "npa_internal.h"

namespace npa {
namespace {

__device__ __forceinline__ float exp_f32(float x) { return static_cast<float>(exp(double(x))); }
__device__ __forceinline__ float tanh_f32(float x) { return static_cast<float>(tanh(double(x))); }
__device__ __forceinline__ float sigmoid_f32(float v) { return 1.0f / (1.0f + exp_f32(-v)); }

__global__ void decode_kernel(npa_gaussian_decode_config cfg, const float4* __restrict__ pos,
                              const float* __restrict__ states, uint32_t count, int C, int k,
                              float* __restrict__ out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const int rec = 12 + 3 * k;
  const float* s = states + size_t(i) * C;
  float* o = out + size_t(i) * rec;
  const float4 p = pos[i];
  // Records are 12 + 3k floats: not 16-byte aligned per particle, so scalar stores.
  o[0] = p.x;
  o[1] = p.y;
  o[2] = p.z;
  o[3] = 1.0f;
  const bool oriented = cfg.mode == NPA_DECODE_SH0_ORIENTED;
  const int color_start = oriented ? C - k * 3 : C - 3;
  // decode_sh (gaussian.rs:134-158)
  for (int q = 0; q < k; ++q)
    for (int e = 0; e < 3; ++e)
      o[12 + q * 3 + e] = clamp_rs(s[color_start + q * 3 + e] + 0.5f, 0.0f, 1.0f);
  // rotation (gaussian.rs:76-89, normalize_quat :214-223)
  float4 rot = make_float4(1.0f, 0.0f, 0.0f, 0.0f);
  if (oriented) {
    const int rs = color_start - 4;
    float qv[4] = {s[rs], s[rs + 1], s[rs + 2], s[rs + 3]};
    float nsq = qv[0] * qv[0];
    nsq = nsq + qv[1] * qv[1];
    nsq = nsq + qv[2] * qv[2];
    nsq = nsq + qv[3] * qv[3];
    const float norm = sqrtf(nsq);
    if (norm <= 1e-8f) {
      qv[0] = 1.0f;
      qv[1] = qv[2] = qv[3] = 0.0f;
    } else {
      for (int e = 0; e < 4; ++e) qv[e] = qv[e] / norm;
    }
    rot = make_float4(qv[0], qv[1], qv[2], qv[3]);
  }
  o[4] = rot.x;
  o[5] = rot.y;
  o[6] = rot.z;
  o[7] = rot.w;
  // decode_scale_opacity (gaussian.rs:160-208)
  float4 so;
  switch (cfg.mode) {
    case NPA_DECODE_PARTICLE_POINT: {
      const float scale = fmaxf(cfg.min_scale, 1.0e-6f);
      so = make_float4(scale, scale, scale, 1.0f);
      break;
    }
    case NPA_DECODE_SH0_FIXED_SCALE: {
      const float scale = clamp_rs(cfg.sigma, cfg.min_scale, cfg.max_scale);
      so = make_float4(scale, scale, scale,
                       clamp_rs(cfg.opacity_scale, cfg.min_opacity, cfg.max_opacity));
      break;
    }
    case NPA_DECODE_SH0_LEARNED_SCALE: {
      const float scale_logit = clamp_rs(s[C - 5], -8.0f, 8.0f);
      const float opacity_logit = clamp_rs(s[C - 4], -12.0f, 12.0f);
      const float scale = clamp_rs(cfg.sigma * exp_f32(scale_logit), cfg.min_scale, cfg.max_scale);
      const float opacity =
          clamp_rs(sigmoid_f32(opacity_logit), cfg.min_opacity, cfg.max_opacity) * cfg.opacity_scale;
      so = make_float4(scale, scale, scale, clamp_rs(opacity, cfg.min_opacity, cfg.max_opacity));
      break;
    }
    default: {
      const int anis = color_start - 8;
      const float mdiv = fmaxf(cfg.max_anisotropy, 1e-6f);
      const float ax = tanh_f32(s[anis] / mdiv) * cfg.max_anisotropy;
      const float ay = tanh_f32(s[anis + 1] / mdiv) * cfg.max_anisotropy;
      const float az = tanh_f32(s[anis + 2] / mdiv) * cfg.max_anisotropy;
      const float ol = tanh_f32(s[anis + 3] / mdiv) * cfg.max_anisotropy;
      so = make_float4(clamp_rs(cfg.sigma * exp_f32(ax), cfg.min_scale, cfg.max_scale),
                       clamp_rs(cfg.sigma * exp_f32(ay), cfg.min_scale, cfg.max_scale),
                       clamp_rs(cfg.sigma * exp_f32(az), cfg.min_scale, cfg.max_scale),
                       clamp_rs(cfg.opacity_scale * exp_f32(ol), cfg.min_opacity, cfg.max_opacity));
      break;
    }
  }
  o[8] = so.x;
  o[9] = so.y;
  o[10] = so.z;
  o[11] = so.w;
}

}  // namespace

npa_status launch_decode(const npa_gaussian_decode_config& cfg, const float4* positions,
                         const float* states, uint32_t count, int state_dims, float* out,
                         cudaStream_t stream) {
  if (count == 0) return NPA_OK;
  const int k = cfg.mode == NPA_DECODE_SH0_ORIENTED ? (cfg.sh_degree + 1) * (cfg.sh_degree + 1) : 1;
  decode_kernel<<<grid_for(count, 128), 128, 0, stream>>>(cfg, positions, states, count,
                                                          state_dims, k, out);
  return after_launch("decode_kernel");
}

}  // namespace npa
