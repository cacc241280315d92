// train.cu -- the training rollout's backward pass (crates/burn_automata/src/target2d.rs:3550-3722,
// crates/burn_automata/src/training.rs:558-640).
//
//   output_adjoint_kernel    per row: the adjoint of the raw update from the
//                            masked position adjoint (raw_motion_adjoint,
//                            target2d.rs:3644), the displacement regularizer
//                            (add_dx_norm_regularizer_adjoint, :3675) and the
//                            masked state adjoint
//   mlp_backward_rows_kernel per row (mlp_backward_from_output_gradients): the
//                            pre-activation again, the hidden adjoint (sum over
//                            outputs in order), the input adjoint (sum over
//                            hidden units in order); stores the row's hidden
//                            values and pre-activation adjoints for the weights
//   weight_grads_kernel      one thread per weight or bias entry, summing the
//                            rows in row order and adding the sum to the
//                            running total -- the reference's sequential f32
//                            sums, so the gradients are bit for bit its own
//   add_adjoint_kernel       running position / state adjoints += the
//                            perception adjoint's
// Rows are the caller's particles.  Weights are read from global memory with
// every lane of a warp on the same address (broadcast).
#include <algorithm>

#include "npa_internal.h"

namespace npa {
namespace {

__device__ __forceinline__ void raw_motion_adjoint_row(const float* raw, const float (&dxa)[3],
                                                       int dims, float scale, float* out) {
  float norm = 0.0f;
  for (int a = 0; a < dims; ++a) norm = norm + raw[a] * raw[a];
  norm = sqrtf(norm);
  const float denom = 1.0f + norm;
  float dot = 0.0f;
  for (int a = 0; a < dims; ++a) dot = dot + raw[a] * dxa[a];
  for (int a = 0; a < dims; ++a) {
    float grad = dxa[a] / denom;
    if (norm > 0.0f) grad = grad - raw[a] * dot / (norm * denom * denom);
    out[a] = out[a] + scale * grad;
  }
}

__global__ void output_adjoint_kernel(const float* __restrict__ update, const float4* __restrict__ pos_adj,
                                      const float* __restrict__ state_adj,
                                      const float* __restrict__ mask, uint32_t rows, int dims,
                                      int C, float scale, float reg, float* __restrict__ out) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int O = dims + C;
  const float* raw = update + size_t(r) * O;
  float* o = out + size_t(r) * O;
  for (int j = 0; j < O; ++j) o[j] = 0.0f;
  const float m = mask ? mask[r] : 1.0f;
  const float4 pa = pos_adj[r];
  const float pv[3] = {pa.x, pa.y, pa.z};
  if (reg != 0.0f) {  // add_dx_norm_regularizer_adjoint
    float norm = 0.0f;
    for (int a = 0; a < dims; ++a) norm = norm + raw[a] * raw[a];
    norm = sqrtf(norm);
    float dx[3] = {0.0f, 0.0f, 0.0f};
    for (int a = 0; a < dims; ++a) dx[a] = scale * raw[a] / (1.0f + norm);
    float dn = 0.0f;
    for (int a = 0; a < dims; ++a) dn = dn + dx[a] * dx[a];
    dn = sqrtf(dn);
    if (dn != 0.0f) {
      float adj[3] = {0.0f, 0.0f, 0.0f};
      for (int a = 0; a < dims; ++a) adj[a] = reg * dx[a] / dn;
      raw_motion_adjoint_row(raw, adj, dims, scale, o);
    }
  }
  float dxa[3] = {0.0f, 0.0f, 0.0f};
  for (int a = 0; a < dims; ++a) dxa[a] = pv[a] * m;
  raw_motion_adjoint_row(raw, dxa, dims, scale, o);
  const float* sa = state_adj + size_t(r) * C;
  for (int c = 0; c < C; ++c) o[dims + c] = o[dims + c] + sa[c] * m;
}

// One thread per row; the row's per-unit values live in shared memory,
// unit-major ([unit][row of the block]) so that a warp's accesses are
// consecutive words.
constexpr int kBackRows = 64;

__global__ void __launch_bounds__(kBackRows)
mlp_backward_rows_kernel(const float* __restrict__ features, const float* __restrict__ out_adj,
                         uint32_t rows, int F, int H, int O, const float* __restrict__ w1t,
                         int Hp, const float* __restrict__ b1, const float* __restrict__ w2,
                         float* __restrict__ hidden, float* __restrict__ dpre,
                         float* __restrict__ gfeat) {
  extern __shared__ float sm[];
  float* pre = sm;                     // [H][kBackRows]
  float* dh = sm + H * kBackRows;      // [H][kBackRows]
  const int t = threadIdx.x;
  const uint32_t r = blockIdx.x * kBackRows + t;
  if (r >= rows) return;
  const float* f = features + size_t(r) * F;
  for (int h = 0; h < H; ++h) {
    float sum = __ldg(b1 + h);
    for (int i = 0; i < F; ++i) sum = sum + __ldg(w1t + size_t(i) * Hp + h) * f[i];
    pre[h * kBackRows + t] = sum;
    dh[h * kBackRows + t] = 0.0f;
    hidden[size_t(r) * H + h] = fmaxf(sum, 0.0f);
  }
  const float* g = out_adj + size_t(r) * O;
  for (int o = 0; o < O; ++o) {
    const float d = g[o];
    const float* w = w2 + size_t(o) * H;
    for (int h = 0; h < H; ++h) dh[h * kBackRows + t] = dh[h * kBackRows + t] + d * __ldg(w + h);
  }
  float* gf = gfeat + size_t(r) * F;
  for (int i = 0; i < F; ++i) gf[i] = 0.0f;
  for (int h = 0; h < H; ++h) {
    const float dp = pre[h * kBackRows + t] > 0.0f ? dh[h * kBackRows + t] : 0.0f;
    dpre[size_t(r) * H + h] = dp;
    for (int i = 0; i < F; ++i) gf[i] = gf[i] + dp * __ldg(w1t + size_t(i) * Hp + h);
  }
}

// Entry e of [gw1 (H x F) | gb1 (H) | gw2 (O x H) | gb2 (O)]: the sum over
// rows, in row order, of its per-row term, added to the running total.
__global__ void weight_grads_kernel(const float* __restrict__ features,
                                    const float* __restrict__ out_adj,
                                    const float* __restrict__ hidden,
                                    const float* __restrict__ dpre, uint32_t rows, int F, int H,
                                    int O, float* __restrict__ gw1, float* __restrict__ gb1,
                                    float* __restrict__ gw2, float* __restrict__ gb2) {
  const uint32_t n1 = uint32_t(H) * F, n2 = n1 + H, n3 = n2 + uint32_t(O) * H, n4 = n3 + O;
  const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n4) return;
  float s = 0.0f;
  if (e < n1) {
    const int h = e / F, i = e - h * F;
    for (uint32_t r = 0; r < rows; ++r) s = s + dpre[size_t(r) * H + h] * features[size_t(r) * F + i];
    gw1[e] = gw1[e] + s;
  } else if (e < n2) {
    const int h = e - n1;
    for (uint32_t r = 0; r < rows; ++r) s = s + dpre[size_t(r) * H + h];
    gb1[h] = gb1[h] + s;
  } else if (e < n3) {
    const int k = e - n2, o = k / H, h = k - o * H;
    for (uint32_t r = 0; r < rows; ++r) s = s + out_adj[size_t(r) * O + o] * hidden[size_t(r) * H + h];
    gw2[k] = gw2[k] + s;
  } else {
    const int o = e - n3;
    for (uint32_t r = 0; r < rows; ++r) s = s + out_adj[size_t(r) * O + o];
    gb2[o] = gb2[o] + s;
  }
}

__global__ void add_adjoint_kernel(float4* __restrict__ pos_adj, float* __restrict__ state_adj,
                                   const float4* __restrict__ dpos, const float* __restrict__ dstate,
                                   uint32_t rows, int dims, int C, int add_pos, int add_state) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  if (add_pos) {
    float4 p = pos_adj[r];
    const float4 q = dpos[r];
    p.x = p.x + q.x;
    p.y = p.y + q.y;
    if (dims == 3) p.z = p.z + q.z;
    pos_adj[r] = p;
  }
  if (add_state)
    for (int c = 0; c < C; ++c) state_adj[size_t(r) * C + c] = state_adj[size_t(r) * C + c] + dstate[size_t(r) * C + c];
}

// Sets *flag when any of count values is not finite.
__global__ void finite_check_kernel(const float* __restrict__ v, uint64_t count,
                                    int* __restrict__ flag, int code) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
       i += uint64_t(gridDim.x) * blockDim.x)
    if (!isfinite(v[i])) atomicOr(flag, code);
}

}  // namespace

npa_status launch_output_adjoint(const float* update, const float4* pos_adj, const float* state_adj,
                                 const float* mask, uint32_t rows, int dims, int C, float scale,
                                 float reg, float* out, cudaStream_t stream) {
  if (rows == 0) return NPA_OK;
  output_adjoint_kernel<<<grid_for(rows, 128), 128, 0, stream>>>(update, pos_adj, state_adj, mask,
                                                                 rows, dims, C, scale, reg, out);
  return after_launch("output_adjoint_kernel");
}

npa_status launch_mlp_backward(const DeviceModel& m, const float* features, const float* out_adj,
                               uint32_t rows, float* hidden, float* dpre, float* gfeat,
                               float* gw1, float* gb1, float* gw2, float* gb2,
                               cudaStream_t stream) {
  if (rows == 0) return NPA_OK;
  const int F = m.feature_dims, H = m.hidden_dims, O = m.update_dims;
  const size_t smem = size_t(2) * H * kBackRows * sizeof(float);
  NPA_CUDA(cudaFuncSetAttribute(mlp_backward_rows_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
           "cudaFuncSetAttribute");
  // w1 is read from the model's transposed copy w1t [F][hidden_padded]
  mlp_backward_rows_kernel<<<grid_for(rows, kBackRows), kBackRows, smem, stream>>>(
      features, out_adj, rows, F, H, O, m.w1t, m.hidden_padded, m.b1, m.w2, hidden, dpre, gfeat);
  NPA_TRY(after_launch("mlp_backward_rows_kernel"));
  const uint32_t entries = uint32_t(H) * F + H + uint32_t(O) * H + O;
  weight_grads_kernel<<<grid_for(entries, 128), 128, 0, stream>>>(
      features, out_adj, hidden, dpre, rows, F, H, O, gw1, gb1, gw2, gb2);
  return after_launch("weight_grads_kernel");
}

npa_status launch_add_adjoint(float4* pos_adj, float* state_adj, const float4* dpos,
                              const float* dstate, uint32_t rows, int dims, int C, bool add_pos,
                              bool add_state, cudaStream_t stream) {
  if (rows == 0 || (!add_pos && !add_state)) return NPA_OK;
  add_adjoint_kernel<<<grid_for(rows, 128), 128, 0, stream>>>(pos_adj, state_adj, dpos, dstate,
                                                              rows, dims, C, add_pos, add_state);
  return after_launch("add_adjoint_kernel");
}

npa_status launch_finite_check(const float* v, uint64_t count, int* flag, int code,
                               cudaStream_t stream) {
  if (count == 0) return NPA_OK;
  const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>((count + 255) / 256, 148u * 8u));
  finite_check_kernel<<<blocks, 256, 0, stream>>>(v, count, flag, code);
  return after_launch("finite_check_kernel");
}

}  // namespace npa
