// perception.cu -- density pass and the standalone perception operator
// (perceive_with_options, crates/burn_automata_kernels/src/reference/forward.rs:26-143).
//
// Both kernels run one thread per sorted slot (the standalone perception
// kernel one thread per slot and 8-channel chunk), so threads of a warp walk
// neighbouring bins and read the sorted position / coordinate views
// contiguously.  Results are written back in the caller's original particle
// order through the permutation.
#include "perception_core.cuh"

namespace npa {
namespace {

constexpr int kChunk = 8;

__global__ void __launch_bounds__(256)
density_kernel(GridParams g, SortedGrid s, uint32_t total, float* __restrict__ volume,
               float* __restrict__ density_out) {
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= total) return;
  const uint32_t batch = q / s.n;
  const float4 pi = s.spos[q];
  const int4 c4 = s.scoord[q];
  float rho = 0.0f;
  for_each_neighbor(g, s, batch, pi, make_int3(c4.x, c4.y, c4.z),
                    [&](uint32_t, float4, float r2) { rho = rho + poly6(g, r2); });
  volume[q] = recip_finite(rho);
  if (density_out) density_out[size_t(batch) * s.n + s.permutation[q]] = rho;
}

__global__ void __launch_bounds__(128)
perception_kernel(GridParams g, PerceptionParams p, SortedGrid s, uint32_t total,
                  const float* __restrict__ states, int C, int chunks,
                  const float* __restrict__ volume, float* __restrict__ features,
                  float* __restrict__ blurred, float* __restrict__ state_gradient,
                  float* __restrict__ density_gradient) {
  const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= uint64_t(total) * chunks) return;
  const uint32_t q = static_cast<uint32_t>(t / chunks);
  const int chunk = static_cast<int>(t - uint64_t(q) * chunks);
  const int c0 = chunk * kChunk;
  const uint32_t batch = q / s.n;
  const size_t row = size_t(batch) * s.n + s.permutation[q];
  const float4 pi = s.spos[q];
  const int4 c4 = s.scoord[q];
  float si[kChunk];
#pragma unroll
  for (int c = 0; c < kChunk; ++c) si[c] = (c0 + c < C) ? states[row * C + c0 + c] : 0.0f;
  PerceptionOut out;
  perceive_chunk<kChunk>(g, p, s, batch, q, pi, make_int3(c4.x, c4.y, c4.z), states, C, c0,
                         volume, si, out);
  const int dim = g.dim;
  const size_t F = p.feature_dims;
  float* f = features + row * F;
#pragma unroll
  for (int c = 0; c < kChunk; ++c) {
    const int ch = c0 + c;
    if (ch < C) {
      f[ch] = si[c];
      f[C + ch] = out.blur[c];
      if (blurred) blurred[row * C + ch] = out.blur[c];
      if (p.state_grad) {
        for (int a = 0; a < dim; ++a) {
          f[2 * C + ch * dim + a] = out.sgrad[c * 3 + a];
          if (state_gradient) state_gradient[(row * C + ch) * dim + a] = out.sgrad[c * 3 + a];
        }
      }
    }
  }
  if (chunk == 0) {
    int cursor = 2 * C + (p.state_grad ? C * dim : 0);
    if (p.density_grad) {
      for (int a = 0; a < dim; ++a) {
        f[cursor + a] = out.dgrad[a];
        if (density_gradient) density_gradient[row * dim + a] = out.dgrad[a];
      }
      cursor += dim;
    }
    if (p.position_features) {
      const float pv[3] = {pi.x, pi.y, pi.z};
      for (int a = 0; a < dim; ++a) f[cursor + a] = pv[a];
    }
  }
}

// f32::powi by binary exponentiation (LLVM's expansion for constant exponents).
float powi_f32(float x, int n) {
  float result = 1.0f;
  bool have = false;
  float square = x;
  while (n) {
    if (n & 1) {
      result = have ? result * square : square;
      have = true;
    }
    n >>= 1;
    if (n) square = square * square;
  }
  return have ? result : 1.0f;
}

}  // namespace

PerceptionParams make_perception_params(const GridParams& g, const npa_perception_options& o,
                                        uint32_t n, int state_dims) {
  PerceptionParams p{};
  p.state_grad = o.state_grad != 0;
  p.density_grad = o.density_grad != 0;
  p.scale_eq = o.scale_equivariance != 0;
  p.pde = o.particle_density_equivariance != 0;
  p.log_norm_grad = o.log_norm_grad != 0;
  p.log_norm_density_grad = o.log_norm_density_grad != 0;
  p.hybrid = o.hybrid_state_gradient != 0;
  p.position_features = o.position_features != 0;
  // normalize.rs:11-15 and :38-46 (eps0 = options.eps0.max(f32::MIN_POSITIVE)).
  const float eps0 = fmaxf(o.eps0, 1.17549435e-38f);
  p.state_scale = p.scale_eq ? g.eps / eps0 : 1.0f;
  const float a = p.scale_eq ? powi_f32(g.eps / eps0, 1 + g.dim) : 1.0f;
  const float b = p.pde ? 1.0f / static_cast<float>(n > 1 ? n : 1) : 1.0f;
  p.density_scale = a * b;
  p.feature_dims = state_dims * 2 + (p.state_grad ? state_dims * g.dim : 0) +
                   (p.density_grad ? g.dim : 0) + (p.position_features ? g.dim : 0);
  return p;
}

npa_status launch_density(const GridParams& g, const SortedGrid& s, uint32_t batch,
                          float* volume_sorted, float* density_out, cudaStream_t stream) {
  const uint32_t total = batch * s.n;
  if (total == 0) return NPA_OK;
  density_kernel<<<grid_for(total, 256), 256, 0, stream>>>(g, s, total, volume_sorted,
                                                           density_out);
  return after_launch("density_kernel");
}

npa_status launch_perception(const GridParams& g, const PerceptionParams& p, const SortedGrid& s,
                             uint32_t batch, const float* states, int state_dims,
                             const float* volume_sorted, float* features, float* blurred,
                             float* state_gradient, float* density_gradient,
                             cudaStream_t stream) {
  const uint32_t total = batch * s.n;
  if (total == 0) return NPA_OK;
  const int chunks = state_dims > 0 ? (state_dims + kChunk - 1) / kChunk : 1;
  const uint64_t threads = uint64_t(total) * chunks;
  perception_kernel<<<grid_for(threads, 128), 128, 0, stream>>>(
      g, p, s, total, states, state_dims, chunks, volume_sorted, features, blurred,
      state_gradient, density_gradient);
  return after_launch("perception_kernel");
}

}  // namespace npa
