// step.cu -- the update MLP, the Euler step and the fused rollout step.
//
// MLP: NpaModel::forward_update_from_features (crates/burn_automata/src/model.rs:900-940)
//   hidden[h] = max(b1[h] + sum_i w1[h][i] * f[i], 0);  u[o] = b2[o] + sum_h w2[o][h] * hidden[h]
// Each sum starts at the bias and adds one rounded product at a time in
// ascending index order, exactly as the reference's loops.  That order is a
// hard requirement: a 64-step rollout of the 2D configuration amplifies an
// FMA-contracted (or tensor-core) MLP to ~2.6e-3 normwise state error while
// the reference-order MLP stays at ~3.5e-4, so the MLP runs on the FP32
// pipe as separate multiply and add (the library is built with --fmad=false).
//
// Work layout (both MLP kernels): a tile of 64 rows per block of 256 threads.
//   layer 1: thread = 4 rows x 8 hidden units per 128-unit column block, k
//            streamed through shared memory in 16-wide slices of w1^T;
//   layer 2: thread = 1 row x ceil(O/4) outputs, sequential over h.
// Fused step (one kernel after hashgrid + density): each tile first runs SPH
// perception (4 threads per particle, channel-split) into the transposed
// feature tile in shared memory, then the MLP, then forward_from_features_with_eps
// (model.rs:867-898), the 3D position gates (model.rs:806-837) and euler_step
// (crates/burn_automata_kernels/src/reference/step.rs:4-55).
#include <algorithm>

#include "perception_core.cuh"

namespace npa {
namespace {

constexpr int kM = 64;          // rows per tile
constexpr int kThreads = 256;   // threads per block
constexpr int kKC = 16;         // k slice staged per iteration
constexpr int kMaxOutPerThread = 16;  // ceil(O / 4) <= 16  ->  O <= 64

struct MlpShape {
  int F, H, Hp, O;
  int hid_stride;  // Hp + 4
  int w2_stride;   // Hp + 4
  int out_stride;  // O + 1
};

struct SmemLayout {
  size_t ft, hid, w1s, w2s, outs, total;  // offsets in floats
};

__host__ __device__ inline SmemLayout smem_layout(const MlpShape& s) {
  SmemLayout l;
  size_t off = 0;
  auto take = [&](size_t floats) {
    size_t o = off;
    off += (floats + 3) & ~size_t(3);
    return o;
  };
  l.ft = take(size_t(s.F) * kM);
  l.hid = take(size_t(kM) * s.hid_stride);
  l.w1s = take(size_t(kKC) * s.Hp);
  l.w2s = take(size_t(s.O) * s.w2_stride);
  l.outs = take(size_t(kM) * s.out_stride);
  l.total = off;
  return l;
}

// Layer 1 for the tile held transposed in ft[F][kM]; writes relu'd hidden units.
template <int HCH>
__device__ __forceinline__ void mlp_layer1(const MlpShape& s, const float* __restrict__ w1t,
                                           const float* __restrict__ b1, const float* ft,
                                           float* hid, float* w1s) {
  const int t = threadIdx.x;
  const int rg = t >> 4;       // rows rg*4 .. rg*4+3
  const int hg = t & 15;       // hidden h = hch*128 + hg*8 .. +7
  float acc[HCH][4][8];
#pragma unroll
  for (int hc = 0; hc < HCH; ++hc) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int h = hc * 128 + hg * 8 + j;
      const float bias = h < s.H ? __ldg(b1 + h) : 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[hc][i][j] = bias;
    }
  }
  const int hp4 = s.Hp >> 2;
  for (int kc = 0; kc < s.F; kc += kKC) {
    const int kn = min(kKC, s.F - kc);
    __syncthreads();  // previous slice consumed
    const float4* src = reinterpret_cast<const float4*>(w1t + size_t(kc) * s.Hp);
    float4* dst = reinterpret_cast<float4*>(w1s);
    for (int e = t; e < kn * hp4; e += kThreads) dst[e] = __ldg(src + e);
    __syncthreads();
    for (int kk = 0; kk < kn; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(ft + (kc + kk) * kM + rg * 4);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int hc = 0; hc < HCH; ++hc) {
        const float* wrow = w1s + kk * s.Hp + hc * 128 + hg * 8;
        const float4 b0 = *reinterpret_cast<const float4*>(wrow);
        const float4 b1v = *reinterpret_cast<const float4*>(wrow + 4);
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1v.x, b1v.y, b1v.z, b1v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[hc][i][j] = acc[hc][i][j] + bv[j] * av[i];
      }
    }
  }
#pragma unroll
  for (int hc = 0; hc < HCH; ++hc) {
    const int h0 = hc * 128 + hg * 8;
    if (h0 < s.Hp) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float* row = hid + (rg * 4 + i) * s.hid_stride + h0;
        float4 v0 = make_float4(fmaxf(acc[hc][i][0], 0.0f), fmaxf(acc[hc][i][1], 0.0f),
                                fmaxf(acc[hc][i][2], 0.0f), fmaxf(acc[hc][i][3], 0.0f));
        float4 v1 = make_float4(fmaxf(acc[hc][i][4], 0.0f), fmaxf(acc[hc][i][5], 0.0f),
                                fmaxf(acc[hc][i][6], 0.0f), fmaxf(acc[hc][i][7], 0.0f));
        *reinterpret_cast<float4*>(row) = v0;
        *reinterpret_cast<float4*>(row + 4) = v1;
      }
    }
  }
}

// Layer 2: out[r][o] = b2[o] + sum_h w2[o][h] * hid[r][h], sequential in h.
__device__ __forceinline__ void mlp_layer2(const MlpShape& s, const float* __restrict__ b2,
                                           const float* hid, const float* w2s, float* outs) {
  const int t = threadIdx.x;
  const int r = t >> 2;
  const int j = t & 3;
  float acc[kMaxOutPerThread];
  const int nout = (s.O - j + 3) >> 2;  // outputs o = j, j+4, ... < O
#pragma unroll
  for (int u = 0; u < kMaxOutPerThread; ++u) acc[u] = (u < nout) ? __ldg(b2 + j + 4 * u) : 0.0f;
  const float* hrow = hid + r * s.hid_stride;
  const int H4 = s.H & ~3;
  for (int h = 0; h < H4; h += 4) {
    const float4 hv = *reinterpret_cast<const float4*>(hrow + h);
#pragma unroll
    for (int u = 0; u < kMaxOutPerThread; ++u) {
      if (u < nout) {
        const float4 w = *reinterpret_cast<const float4*>(w2s + (j + 4 * u) * s.w2_stride + h);
        float a = acc[u];
        a = a + w.x * hv.x;
        a = a + w.y * hv.y;
        a = a + w.z * hv.z;
        a = a + w.w * hv.w;
        acc[u] = a;
      }
    }
  }
  for (int h = H4; h < s.H; ++h) {
    const float hv = hrow[h];
#pragma unroll
    for (int u = 0; u < kMaxOutPerThread; ++u)
      if (u < nout) acc[u] = acc[u] + w2s[(j + 4 * u) * s.w2_stride + h] * hv;
  }
#pragma unroll
  for (int u = 0; u < kMaxOutPerThread; ++u)
    if (u < nout) outs[r * s.out_stride + j + 4 * u] = acc[u];
}

__device__ __forceinline__ void load_w2(const MlpShape& s, const float* __restrict__ w2,
                                        float* w2s) {
  for (int e = threadIdx.x; e < s.O * s.H; e += kThreads) {
    const int o = e / s.H, h = e - o * s.H;
    w2s[o * s.w2_stride + h] = __ldg(w2 + e);
  }
}

template <int HCH>
__global__ void __launch_bounds__(kThreads)
forward_update_kernel(MlpShape s, const float* __restrict__ w1t, const float* __restrict__ b1,
                      const float* __restrict__ w2, const float* __restrict__ b2,
                      const float* __restrict__ features, uint32_t rows,
                      float* __restrict__ update) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const SmemLayout L = smem_layout(s);
  float* ft = smem + L.ft;
  float* hid = smem + L.hid;
  float* w1s = smem + L.w1s;
  float* w2s = smem + L.w2s;
  float* outs = smem + L.outs;
  load_w2(s, w2, w2s);
  const uint32_t tiles = (rows + kM - 1) / kM;
  for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    __syncthreads();
    const uint32_t row0 = tile * kM;
    for (int e = threadIdx.x; e < kM * s.F; e += kThreads) {
      const int r = e / s.F, f = e - r * s.F;
      const uint32_t row = row0 + r;
      ft[f * kM + r] = row < rows ? __ldg(features + size_t(row) * s.F + f) : 0.0f;
    }
    mlp_layer1<HCH>(s, w1t, b1, ft, hid, w1s);
    __syncthreads();
    mlp_layer2(s, b2, hid, w2s, outs);
    __syncthreads();
    for (int e = threadIdx.x; e < kM * s.O; e += kThreads) {
      const int r = e / s.O, o = e - r * s.O;
      const uint32_t row = row0 + r;
      if (row < rows) update[size_t(row) * s.O + o] = outs[r * s.out_stride + o];
    }
  }
}

struct EulerParams {
  float dt;
  int mem_dims;     // spatial_mem_dims (config.rs:90-92)
  int clamp3d;      // dim == 3 && C > 3 (step.rs:48)
};

// euler_step (step.rs:4-55) for one row.
__device__ __forceinline__ float4 euler_position(const GridParams& g, const EulerParams& e,
                                                 float4 p, const float dx[4], float mask) {
  float v[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int a = 0; a < 4; ++a)
    if (a < e.mem_dims) v[a] = v[a] + e.dt * dx[a] * mask;
  return wrap_position(g, make_float4(v[0], v[1], v[2], v[3]));
}

__device__ __forceinline__ float euler_state(const EulerParams& e, int C, int ch, float s,
                                             float ds, float mask) {
  float next = s + e.dt * ds * mask;
  if (e.clamp3d && (ch == 3 || (C > 8 && ch == 8))) next = clamp_rs(next, -8.0f, 24.0f);
  return next;
}

__global__ void euler_kernel(GridParams g, EulerParams e, const float4* __restrict__ pos,
                             const float* __restrict__ states, const float4* __restrict__ dx,
                             const float* __restrict__ ds, uint32_t total, int C,
                             const float* __restrict__ mask, float4* __restrict__ next_pos,
                             float* __restrict__ next_states) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const float m = mask ? mask[i] : 1.0f;
  const float4 d = dx[i];
  const float dv[4] = {d.x, d.y, d.z, d.w};
  next_pos[i] = euler_position(g, e, pos[i], dv, m);
  for (int c = 0; c < C; ++c) {
    const size_t k = size_t(i) * C + c;
    next_states[k] = euler_state(e, C, c, states[k], ds[k], m);
  }
}

struct FusedParams {
  float alpha;
  float motion_eps;  // NpaConfig::motion_eps (config.rs:156-162)
  int gates3d;       // dim == 3 && position_features && C > 3 (model.rs:806-809)
};

// Fused rollout step over sorted slots; CH = channels per perception thread.
template <int CH, int HCH>
__global__ void __launch_bounds__(kThreads)
fused_step_kernel(MlpShape s, GridParams g, PerceptionParams p, SortedGrid sg, uint32_t total,
                  int C, const float* __restrict__ w1t, const float* __restrict__ b1,
                  const float* __restrict__ w2, const float* __restrict__ b2,
                  const float4* __restrict__ positions, const float* __restrict__ states,
                  const float* __restrict__ volume, FusedParams fp, EulerParams ep,
                  const float* __restrict__ mask, float4* __restrict__ next_pos,
                  float* __restrict__ next_states, float4* __restrict__ dx_out,
                  float* __restrict__ ds_out, float* __restrict__ features_out) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const SmemLayout L = smem_layout(s);
  float* ft = smem + L.ft;
  float* hid = smem + L.hid;
  float* w1s = smem + L.w1s;
  float* w2s = smem + L.w2s;
  float* outs = smem + L.outs;
  load_w2(s, w2, w2s);
  const int D = g.dim;
  const uint32_t tiles = (total + kM - 1) / kM;
  const int r = threadIdx.x >> 2;    // particle within the tile
  const int part = threadIdx.x & 3;  // channel chunk
  const int c0 = part * CH;
  for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    __syncthreads();  // previous tile's epilogue done with ft / outs
    const uint32_t q = tile * kM + r;
    const bool live = q < total;
    // ---- perception into ft[F][kM] ----
    if (live) {
      const uint32_t batch = q / sg.n;
      const size_t row = size_t(batch) * sg.n + sg.permutation[q];
      const float4 pi = sg.spos[q];
      const int4 c4 = sg.scoord[q];
      float si[CH];
#pragma unroll
      for (int c = 0; c < CH; ++c) si[c] = (c0 + c < C) ? __ldg(states + row * C + c0 + c) : 0.0f;
      PerceptionOut po;
      perceive_chunk<CH>(g, p, sg, batch, q, pi, make_int3(c4.x, c4.y, c4.z), states, C, c0,
                         volume, si, po);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int ch = c0 + c;
        if (ch < C) {
          ft[ch * kM + r] = si[c];
          ft[(C + ch) * kM + r] = po.blur[c];
          if (p.state_grad)
            for (int a = 0; a < D; ++a) ft[(2 * C + ch * D + a) * kM + r] = po.sgrad[c * 3 + a];
        }
      }
      if (part == 0) {
        int cursor = 2 * C + (p.state_grad ? C * D : 0);
        if (p.density_grad) {
          for (int a = 0; a < D; ++a) ft[(cursor + a) * kM + r] = po.dgrad[a];
          cursor += D;
        }
        if (p.position_features) {
          const float pv[3] = {pi.x, pi.y, pi.z};
          for (int a = 0; a < D; ++a) ft[(cursor + a) * kM + r] = pv[a];
        }
      }
    } else {
      for (int f = part; f < s.F; f += 4) ft[f * kM + r] = 0.0f;
    }
    // ---- MLP ----
    mlp_layer1<HCH>(s, w1t, b1, ft, hid, w1s);
    __syncthreads();
    mlp_layer2(s, b2, hid, w2s, outs);
    __syncthreads();
    // ---- forward_from_features_with_eps + gates + euler_step ----
    if (live) {
      const uint32_t batch = q / sg.n;
      const size_t row = size_t(batch) * sg.n + sg.permutation[q];
      const float* u = outs + r * s.out_stride;
      float norm = 0.0f;
      for (int a = 0; a < D; ++a) norm = norm + u[a] * u[a];
      norm = sqrtf(norm);
      float dx[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int a = 0; a < D; ++a) dx[a] = fp.alpha * u[a] * fp.motion_eps / (1.0f + norm);
      const float4 pi = sg.spos[q];
      float state_gate = 1.0f;
      bool gated = false;
      if (fp.gates3d) {
        // position_conditioned_3d_{maturity,motion}_gate (rollout/mod.rs:67-90)
        const float liveness = ft[3 * kM + r];
        const float sd = ft[7 * kM + r];
        state_gate = clamp_rs((4.0f - liveness) * 2.0f, 0.0f, 1.0f);
        float motion_gate = 0.0f;
        if (!(pi.w >= 0.5f)) {
          const float dg = clamp_rs((fabsf(sd) - 0.01f) / 0.02f, 0.0f, 1.0f);
          motion_gate = state_gate * dg;
        }
        for (int a = 0; a < D; ++a) dx[a] = dx[a] * motion_gate;
        gated = true;
      }
      const float m = mask ? __ldg(mask + row) : 1.0f;
      if (part == 0) {
        next_pos[row] = euler_position(g, ep, pi, dx, m);
        if (dx_out) dx_out[row] = make_float4(dx[0], dx[1], dx[2], dx[3]);
      }
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int ch = c0 + c;
        if (ch < C) {
          float dsv = u[D + ch];
          if (gated) dsv = dsv * state_gate;
          const float sv = ft[ch * kM + r];
          next_states[row * C + ch] = euler_state(ep, C, ch, sv, dsv, m);
          if (ds_out) ds_out[row * C + ch] = dsv;
        }
      }
      if (features_out)
        for (int f = part; f < s.F; f += 4) features_out[row * s.F + f] = ft[f * kM + r];
    }
  }
}

MlpShape make_shape(const DeviceModel& m) {
  MlpShape s;
  s.F = m.feature_dims;
  s.H = m.hidden_dims;
  s.Hp = (m.hidden_dims + 127) / 128 * 128;
  s.O = m.update_dims;
  s.hid_stride = s.Hp + 4;
  s.w2_stride = s.Hp + 4;
  s.out_stride = s.O + 1;
  return s;
}

struct LaunchCfg {
  unsigned grid;
  size_t smem;
};

template <class K>
npa_status plan(K kernel, const MlpShape& s, uint64_t tiles, LaunchCfg* out) {
  const size_t smem = smem_layout(s).total * sizeof(float);
  int dev = 0;
  NPA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  int max_optin = 0, sms = 0;
  NPA_CUDA(cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev),
           "cudaDeviceGetAttribute");
  NPA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
           "cudaDeviceGetAttribute");
  if (smem > size_t(max_optin))
    return fail(NPA_ERR_UNSUPPORTED, "MLP shape needs more shared memory than a block has");
  NPA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
           "cudaFuncSetAttribute");
  int per_sm = 0;
  NPA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem),
           "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  if (per_sm < 1) return fail(NPA_ERR_UNSUPPORTED, "MLP kernel cannot be resident");
  const uint64_t slots = uint64_t(per_sm) * sms;
  out->grid = static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>(tiles, slots)));
  out->smem = smem;
  return NPA_OK;
}

}  // namespace

bool fused_step_supported(const DeviceModel& m) {
  return m.state_dims >= 0 && m.state_dims <= 32 && m.update_dims <= 4 * kMaxOutPerThread &&
         m.hidden_dims >= 1 && m.hidden_dims <= 256 && m.feature_dims >= 1;
}

npa_status launch_forward_update(const DeviceModel& m, const float* features, uint32_t rows,
                                 float* update, cudaStream_t stream) {
  if (rows == 0) return NPA_OK;
  const MlpShape s = make_shape(m);
  if (s.O > 4 * kMaxOutPerThread || s.Hp > 256)
    return fail(NPA_ERR_UNSUPPORTED, "MLP shape outside the supported range (H <= 256, O <= 64)");
  const uint64_t tiles = (uint64_t(rows) + kM - 1) / kM;
  LaunchCfg lc;
  if (s.Hp <= 128) {
    NPA_TRY(plan(forward_update_kernel<1>, s, tiles, &lc));
    forward_update_kernel<1><<<lc.grid, kThreads, lc.smem, stream>>>(s, m.w1t, m.b1, m.w2, m.b2,
                                                                     features, rows, update);
  } else {
    NPA_TRY(plan(forward_update_kernel<2>, s, tiles, &lc));
    forward_update_kernel<2><<<lc.grid, kThreads, lc.smem, stream>>>(s, m.w1t, m.b1, m.w2, m.b2,
                                                                     features, rows, update);
  }
  return after_launch("forward_update_kernel");
}

npa_status launch_euler(const GridParams& g, const float4* positions, const float* states,
                        const float4* dx, const float* ds, uint32_t total, int state_dims,
                        float dt, const float* mask, float4* next_positions, float* next_states,
                        cudaStream_t stream) {
  if (total == 0) return NPA_OK;
  EulerParams e{dt, g.dim == 3 ? 4 : 2, (g.dim == 3 && state_dims > 3) ? 1 : 0};
  euler_kernel<<<grid_for(total, 256), 256, 0, stream>>>(g, e, positions, states, dx, ds, total,
                                                         state_dims, mask, next_positions,
                                                         next_states);
  return after_launch("euler_kernel");
}

npa_status launch_fused_step(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                             const SortedGrid& sgrid, uint32_t batch, const float4* positions,
                             const float* states, const float* volume_sorted, float dt,
                             const float* mask, const StepOutputs& out, cudaStream_t stream) {
  const uint32_t total = batch * sgrid.n;
  if (total == 0) return NPA_OK;
  if (!fused_step_supported(m))
    return fail(NPA_ERR_UNSUPPORTED, "step shape outside the fused kernel's range (C <= 32, H <= 256)");
  const MlpShape s = make_shape(m);
  FusedParams fp;
  fp.alpha = m.alpha;
  fp.motion_eps = m.equivariance == NPA_EQUIV_PARTICLE_DENSITY_AND_SCALE ? g.eps : m.eps0;
  fp.gates3d = (g.dim == 3 && m.position_features && m.state_dims > 3) ? 1 : 0;
  EulerParams e{dt, g.dim == 3 ? 4 : 2, (g.dim == 3 && m.state_dims > 3) ? 1 : 0};
  const uint64_t tiles = (uint64_t(total) + kM - 1) / kM;
  LaunchCfg lc;
#define NPA_FUSED(CH, HCH)                                                                     \
  do {                                                                                         \
    NPA_TRY(plan(fused_step_kernel<CH, HCH>, s, tiles, &lc));                                  \
    fused_step_kernel<CH, HCH><<<lc.grid, kThreads, lc.smem, stream>>>(                        \
        s, g, p, sgrid, total, m.state_dims, m.w1t, m.b1, m.w2, m.b2, positions, states,      \
        volume_sorted, fp, e, mask, out.next_positions, out.next_states, out.dx, out.ds,       \
        out.features);                                                                         \
  } while (0)
  const bool small_c = m.state_dims <= 16;
  const bool small_h = s.Hp <= 128;
  if (small_c && small_h) NPA_FUSED(4, 1);
  else if (small_c) NPA_FUSED(4, 2);
  else if (small_h) NPA_FUSED(8, 1);
  else NPA_FUSED(8, 2);
#undef NPA_FUSED
  return after_launch("fused_step_kernel");
}

}  // namespace npa
