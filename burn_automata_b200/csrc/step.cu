// step.cu -- the update MLP, the Euler step and the MLP stage of the rollout step.
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
// Work layout: NT threads per block (the rollout step: two 192-thread blocks
// per SM with the hidden rows over the feature tile, for hidden widths up to
// 128; otherwise 384, or 256 when a 384-thread tile does not fit in shared
// memory), HG x RG thread grid with
// HG = Hp / kTH hidden groups and RG = NT / HG row groups; a tile holds
// M = 8 * RG rows.
//   layer 1: each thread owns an 8 rows x kTH hidden-unit register tile (the
//            lane layout is described at layer1_hidden_group) and
//            walks k = 0..F-1 in order (features of the tile feature-major in
//            shared memory, w1 transposed in shared memory);
//   layer 2: R NT / M threads per group of R rows (R = 2 or 3), each owning
//            ceil(O / (R NT / M)) outputs of the group's rows, sequential over h.
// The rollout's MLP stage consumes the feature tiles written by
// perception_tiles_kernel ([tile][F][M], sorted order) through one shared
// buffer: once layer 2 is done, one thread starts a bulk (TMA) copy of the next
// tile that completes on an mbarrier, behind the epilogue and the bounded wait
// at the top of the loop (one buffer instead of two
// is what lets 12 warps per SM fit; measured 1.017 vs 1.067 ms at 8 warps
// double-buffered on cfg2).  Each row finishes with forward_from_features_with_eps
// (model.rs:867-898), the 3D position gates (model.rs:806-837) and euler_step
// (crates/burn_automata_kernels/src/reference/step.rs:4-55), writing the next
// position / state in the caller's particle order.
#include <algorithm>
#include <type_traits>

#include "perception_core.cuh"

namespace npa {
namespace {

constexpr int kThreadsWide = 384;    // 12 warps per SM: 3 per scheduler
constexpr int kThreadsNarrow = 256;  // when the wide tile does not fit in shared memory
constexpr int kTwoBlockThreads = 192;  // two blocks per SM, hidden rows over the feature tile
constexpr int kTH = 8;         // hidden units per thread in layer 1
constexpr int kKC = 16;              // k slice when w1 is streamed
constexpr int kMaxOut = 64;          // outputs per row-owning thread (layer 2 runs in passes)
constexpr size_t kSmemBudget = 220 * 1024;

struct MlpShape {
  int NT;          // threads per block
  int F, H, Hp, O;
  int M;           // rows per tile
  int tpr;         // layer-2 threads per row (NT / M)
  int hid_stride;  // Hp + 4
  int w2_stride;   // Hp + 4
  int out_stride;  // O + 1
  int w1_resident; // w1^T [F][Hp] kept in shared memory for the whole kernel
  int l2_rows;     // layer-2 rows per thread: 2, or 3 when M splits into triples with less waste
  int alias;       // the feature tile and the hidden rows share one region (fused step)
};

struct SmemLayout {
  size_t ft0, hid, w1, w2, outs, bar, total;  // offsets in floats
};

__host__ __device__ inline SmemLayout smem_layout(const MlpShape& s) {
  SmemLayout l;
  size_t off = 0;
  auto take = [&](size_t floats) {
    size_t o = off;
    off += (floats + 3) & ~size_t(3);
    return o;
  };
  if (s.alias) {
    const size_t ft_floats = size_t(s.F) * s.M, hid_floats = size_t(s.M) * s.hid_stride;
    l.ft0 = take(ft_floats > hid_floats ? ft_floats : hid_floats);
    l.hid = l.ft0;
  } else {
    l.ft0 = take(size_t(s.F) * s.M);
    l.hid = take(size_t(s.M) * s.hid_stride);
  }
  l.w1 = take(size_t(s.w1_resident ? s.F : kKC) * s.Hp);
  l.w2 = take(size_t(s.O) * s.w2_stride);
  l.outs = take(size_t(s.M) * s.out_stride);
  l.bar = take(4);  // the feature-tile mbarrier (8 bytes, 16-byte aligned)
  l.total = off;
  return l;
}

// ---- bulk (TMA) copy of a feature tile, completed on an mbarrier ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(bar)) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
// One elected thread: expect `bytes` on the barrier and start the copy in
// pieces of at most kBulkPiece bytes (sizes and addresses multiples of 16).
constexpr uint32_t kBulkPiece = 16384;
__device__ __forceinline__ void bulk_tile_load(float* dst, const float* src, uint32_t bytes,
                                               uint64_t* bar) {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
  for (uint32_t off = 0; off < bytes; off += kBulkPiece) {
    const uint32_t n = bytes - off < kBulkPiece ? bytes - off : kBulkPiece;
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(reinterpret_cast<char*>(dst) + off)),
        "l"(reinterpret_cast<const char*>(src) + off), "r"(n), "r"(smem_u32(bar))
        : "memory");
  }
}
// Waits for phase `parity` of the barrier for at most about two seconds of
// global time; false (and a count in g_bulk_copy_timeouts) when it gave up.
__device__ unsigned long long g_bulk_copy_timeouts = 0;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t0));
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    if (t - t0 > 2000000000ull) return false;
  }
}

// The threads that run an MLP tile: the whole block, or a block's consumer
// warps in the warp-specialised step (their own index and named barrier).
struct BlockGroup {
  static __device__ __forceinline__ int tid() { return threadIdx.x; }
  static __device__ __forceinline__ int size() { return blockDim.x; }
  static __device__ __forceinline__ void sync() { __syncthreads(); }
  static __device__ __forceinline__ bool sync_or(bool p) { return __syncthreads_or(p); }
};

// Weights into shared memory: w2 [O][H] -> rows of w2_stride; w1^T when resident.
template <class G = BlockGroup>
__device__ __forceinline__ void load_weights(const MlpShape& s, const float* __restrict__ w1t,
                                             const float* __restrict__ w2, float* w1s,
                                             float* w2s) {
  for (int e = G::tid(); e < s.O * s.H; e += G::size()) {
    const int o = e / s.H, h = e - o * s.H;
    w2s[o * s.w2_stride + h] = __ldg(w2 + e);
  }
  if (s.w1_resident) {
    const float4* src = reinterpret_cast<const float4*>(w1t);
    float4* dst = reinterpret_cast<float4*>(w1s);
    const int n4 = s.F * s.Hp / 4;
    for (int e = G::tid(); e < n4; e += G::size()) dst[e] = __ldg(src + e);
  }
}

// One k step of the 8 x 8 register tile: acc[i][j] += w[j] * f[i], each a
// rounded product then a rounded sum.  All 64 products are formed before the
// 64 sums so no sum waits on the product issued just before it.  (The packed
// mul.rn.f32x2 / add.rn.f32x2 pair was measured not to reproduce the scalar
// results bit for bit, so the scalar form stays.)
__device__ __forceinline__ void micro_tile(float (&acc)[8][kTH], float4 a0, float4 a1,
                                           const float4 (&bq)[kTH / 4]) {
  const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  float bv[kTH];
#pragma unroll
  for (int j4 = 0; j4 < kTH / 4; ++j4) {
    bv[4 * j4] = bq[j4].x;
    bv[4 * j4 + 1] = bq[j4].y;
    bv[4 * j4 + 2] = bq[j4].z;
    bv[4 * j4 + 3] = bq[j4].w;
  }
  float p[8][kTH];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < kTH; ++j) p[i][j] = bv[j] * av[i];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < kTH; ++j) acc[i][j] = acc[i][j] + p[i][j];
}

// Layer 1 for the tile in ft[F][M]: hid[r][h] = max(b1[h] + sum_k w1[h][k] f[r][k], 0).
//
// Thread layout: HG = Hp / 8 hidden groups times NT / HG row groups.  A warp
// spans 8 hidden groups (lanes % 8) of 4 row groups (lanes / 8); hidden group
// hg owns units (j4 HG + hg) 4 + e, j4 in {0, 1}, e in [0, 4), so each
// 16-byte weight load of a warp reads 128 contiguous bytes and each feature
// load four 32-byte-spaced rows: one shared-memory wavefront apiece.
template <int HG, class G = BlockGroup>
__device__ __forceinline__ int layer1_hidden_group() {
  const int lane = G::tid() & 31, warp = G::tid() >> 5;
  return (warp % (HG / 8)) * 8 + (lane & 7);
}
template <int HG, class G = BlockGroup>
__device__ __forceinline__ int layer1_row_group() {
  const int lane = G::tid() & 31, warp = G::tid() >> 5;
  return (warp / (HG / 8)) * 4 + (lane >> 3);
}
static_assert(kTH == 8, "layer1_unit assumes two float4 groups per thread");
__host__ __device__ constexpr int layer1_unit(int HG, int hg, int j4) { return (j4 * HG + hg) * 4; }

// The layer-1 biases of this thread's hidden units (constant over tiles).
template <int HG, class G = BlockGroup>
__device__ __forceinline__ void load_bias1(const MlpShape& s, const float* __restrict__ b1,
                                           float (&bias)[kTH]) {
  const int hg = layer1_hidden_group<HG, G>();
#pragma unroll
  for (int j = 0; j < kTH; ++j) {
    const int h = layer1_unit(HG, hg, j / 4) + (j & 3);
    bias[j] = h < s.H ? __ldg(b1 + h) : 0.0f;
  }
}

// ALIAS: hid overlays ft, so the block synchronises before the hidden rows
// are stored.
template <int HG, int NT, bool ALIAS = false, class G = BlockGroup>
__device__ __forceinline__ void mlp_layer1(const MlpShape& s, const float* __restrict__ w1t,
                                           const float (&bias)[kTH], const float* ft,
                                           float* w1s, float* hid) {
  static_assert(HG % 8 == 0 && (NT / 32) % (HG / 8) == 0, "layer-1 thread layout");
  constexpr int RG = NT / HG;
  constexpr int M = RG * 8;
  const int t = G::tid();
  const int rg = layer1_row_group<HG, G>();
  const int hg = layer1_hidden_group<HG, G>();
  float acc[8][kTH];
#pragma unroll
  for (int j = 0; j < kTH; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][j] = bias[j];
  const float* arow = ft + rg * 8;
  if (s.w1_resident) {
#pragma unroll 1
    for (int k = 0; k < s.F; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(arow + k * M);
      const float4 a1 = *reinterpret_cast<const float4*>(arow + k * M + 4);
      float4 bq[kTH / 4];
#pragma unroll
      for (int j4 = 0; j4 < kTH / 4; ++j4)
        bq[j4] = *reinterpret_cast<const float4*>(w1s + k * s.Hp + layer1_unit(HG, hg, j4));
      micro_tile(acc, a0, a1, bq);
    }
  } else {
    const int hp4 = s.Hp >> 2;
    for (int kc = 0; kc < s.F; kc += kKC) {
      const int kn = min(kKC, s.F - kc);
      G::sync();  // previous slice consumed
      const float4* src = reinterpret_cast<const float4*>(w1t + size_t(kc) * s.Hp);
      float4* dst = reinterpret_cast<float4*>(w1s);
      for (int e = t; e < kn * hp4; e += NT) dst[e] = __ldg(src + e);
      G::sync();
      for (int kk = 0; kk < kn; ++kk) {
        const int k = kc + kk;
        const float4 a0 = *reinterpret_cast<const float4*>(arow + k * M);
        const float4 a1 = *reinterpret_cast<const float4*>(arow + k * M + 4);
        float4 bq[kTH / 4];
#pragma unroll
        for (int j4 = 0; j4 < kTH / 4; ++j4)
          bq[j4] = *reinterpret_cast<const float4*>(w1s + kk * s.Hp + layer1_unit(HG, hg, j4));
        micro_tile(acc, a0, a1, bq);
      }
    }
  }
  if constexpr (ALIAS) G::sync();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float* row = hid + (rg * 8 + i) * s.hid_stride;
#pragma unroll
    for (int j4 = 0; j4 < kTH / 4; ++j4)
      *reinterpret_cast<float4*>(row + layer1_unit(HG, hg, j4)) =
          make_float4(fmaxf(acc[i][4 * j4], 0.0f), fmaxf(acc[i][4 * j4 + 1], 0.0f),
                      fmaxf(acc[i][4 * j4 + 2], 0.0f), fmaxf(acc[i][4 * j4 + 3], 0.0f));
  }
}

__device__ __forceinline__ float lane_of(const float4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// Layer 2: outs[r][o] = b2[o] + sum_h w2[o][h] * hid[r][h], sequential in h.
// R rows per thread: R * tpr threads per row group, thread j owning outputs
// o = j + R tpr u (u in [u0, u0 + NOUT)) of the group's R rows; each weight
// load serves R rows.  Group g holds rows g + i M / R (i < R), so the rows a
// warp reads at one h fall in distinct shared-memory banks.  Outputs past O
// are computed on a valid row, not stored.
template <int R, int NOUT, class G = BlockGroup>
__device__ __forceinline__ void mlp_layer2_rows(const MlpShape& s, const float* __restrict__ b2,
                                                const float* hid, const float* w2s, float* outs,
                                                int u0) {
  const int tpg = R * s.tpr;
  const int t = G::tid();
  const int rg = t / tpg;
  const int j = t - rg * tpg;
  const int ngroups = s.M / R;
  float acc[R][NOUT];
  int woff[NOUT];
#pragma unroll
  for (int u = 0; u < NOUT; ++u) {
    const int o = j + tpg * (u0 + u);
    const int oo = o < s.O ? o : 0;
    const float bias = __ldg(b2 + oo);
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i][u] = bias;
    woff[u] = oo * s.w2_stride;
  }
  int hoff[R];
#pragma unroll
  for (int i = 0; i < R; ++i) hoff[i] = (rg + i * ngroups) * s.hid_stride;
  const int H4 = s.H & ~3;
#pragma unroll 2
  for (int h = 0; h < H4; h += 4) {
    float4 hv[R];
#pragma unroll
    for (int i = 0; i < R; ++i) hv[i] = *reinterpret_cast<const float4*>(hid + hoff[i] + h);
    float4 wv[NOUT];
#pragma unroll
    for (int u = 0; u < NOUT; ++u) wv[u] = *reinterpret_cast<const float4*>(w2s + woff[u] + h);
    // each product is added as soon as it is formed: batching the products
    // first, as layer 1 does, is slower here (cfg2 MLP 0.922 vs 0.897 ms)
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int u = 0; u < NOUT; ++u)
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i][u] = acc[i][u] + lane_of(wv[u], k) * lane_of(hv[i], k);
  }
  for (int h = H4; h < s.H; ++h) {
#pragma unroll
    for (int u = 0; u < NOUT; ++u) {
      const float w = w2s[woff[u] + h];
#pragma unroll
      for (int i = 0; i < R; ++i) acc[i][u] = acc[i][u] + w * hid[hoff[i] + h];
    }
  }
#pragma unroll
  for (int u = 0; u < NOUT; ++u) {
    const int o = j + tpg * (u0 + u);
    if (o < s.O) {
#pragma unroll
      for (int i = 0; i < R; ++i) outs[(rg + i * ngroups) * s.out_stride + o] = acc[i][u];
    }
  }
}

// Outputs per thread per pass over the hidden rows (bounds the products'
// registers: R * NOUT * 4 of them).
template <int R, class G = BlockGroup>
__device__ __forceinline__ void mlp_layer2_r(const MlpShape& s, const float* __restrict__ b2,
                                             const float* hid, const float* w2s, float* outs) {
  constexpr int kChunk = R == 2 ? 8 : 4;
  const int per_thread = (s.O + R * s.tpr - 1) / (R * s.tpr);
  for (int u0 = 0; u0 < per_thread; u0 += kChunk) {
    switch (min(kChunk, per_thread - u0)) {
#define NPA_L2(N)                                                  \
  case N:                                                          \
    if constexpr (N <= kChunk) mlp_layer2_rows<R, N, G>(s, b2, hid, w2s, outs, u0); \
    break;
      NPA_L2(1) NPA_L2(2) NPA_L2(3) NPA_L2(4) NPA_L2(5) NPA_L2(6) NPA_L2(7) NPA_L2(8)
#undef NPA_L2
      default:
        break;
    }
  }
}

template <class G = BlockGroup>
__device__ __forceinline__ void mlp_layer2_any(const MlpShape& s, const float* __restrict__ b2,
                                               const float* hid, const float* w2s, float* outs) {
  if (s.l2_rows == 3)
    mlp_layer2_r<3, G>(s, b2, hid, w2s, outs);
  else
    mlp_layer2_r<2, G>(s, b2, hid, w2s, outs);
}

// API MLP: rows of the caller's row-major feature matrix.
template <int HG, int NT>
__global__ void __launch_bounds__(NT, 1)
forward_update_kernel(MlpShape s, const float* __restrict__ w1t, const float* __restrict__ b1,
                      const float* __restrict__ w2, const float* __restrict__ b2,
                      const float* __restrict__ features, uint32_t rows,
                      float* __restrict__ update) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const SmemLayout L = smem_layout(s);
  float* ft = smem + L.ft0;
  float* hid = smem + L.hid;
  float* w1s = smem + L.w1;
  float* w2s = smem + L.w2;
  float* outs = smem + L.outs;
  load_weights(s, w1t, w2, w1s, w2s);
  float bias1[kTH];
  load_bias1<HG>(s, b1, bias1);
  const uint32_t tiles = (rows + s.M - 1) / s.M;
  for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    __syncthreads();
    const uint32_t row0 = tile * s.M;
    for (int e = threadIdx.x; e < s.M * s.F; e += NT) {
      const int r = e / s.F, f = e - r * s.F;
      const uint32_t row = row0 + r;
      ft[f * s.M + r] = row < rows ? __ldg(features + size_t(row) * s.F + f) : 0.0f;
    }
    __syncthreads();
    mlp_layer1<HG, NT>(s, w1t, bias1, ft, w1s, hid);
    __syncthreads();
    mlp_layer2_any(s, b2, hid, w2s, outs);
    __syncthreads();
    for (int e = threadIdx.x; e < s.M * s.O; e += NT) {
      const int r = e / s.O, o = e - r * s.O;
      const uint32_t row = row0 + r;
      if (row < rows) update[size_t(row) * s.O + o] = outs[r * s.out_stride + o];
    }
  }
}

struct EulerParams {
  float dt;
  int mem_dims;  // spatial_mem_dims (config.rs:90-92)
  int clamp3d;   // dim == 3 && C > 3 (step.rs:48)
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

struct StepParams {
  float alpha;
  float motion_eps;  // NpaConfig::motion_eps (config.rs:156-162)
  int gates3d;       // dim == 3 && position_features && C > 3 (model.rs:806-809)
  int C;
  int D;
  const float* states;  // the step's input states [B*N][C] (caller order)
  // Stochastic update mask of the GPU executor (when lane_seeds is set):
  // mask = stochastic_update_mask(update_prob, local index, *step_counter,
  // lane_seeds[batch]).
  float update_prob;
  const uint32_t* lane_seeds;    // [B] or null
  const uint32_t* step_counter;  // device step index (read once per launch)
};

// Own-state channels a thread keeps in registers between layer 1 and the
// epilogue (each of a row's threads owns a contiguous run of ceil(C / TPR)
// channels; beyond kStateRegs of them the rest are read in the epilogue).
constexpr int kStateRegs = 8;

// One tile of the MLP stage: rows tile * M + [0, M) of the sorted order,
// features in ft [F][M].  Layer 1, layer 2, then
// forward_from_features_with_eps + gates + euler_step with TPR threads per
// row; after_layer2() runs once layer 2 has finished with ft and hid.
// `arrived`: this thread saw the tile's copy complete.  The block decides at
// the barrier after layer 1 (so a thread may start layer 1 while others
// finish the previous tile's epilogue); false for any thread -> the tile is
// abandoned and mlp_tile returns false.
template <int HG, int NT, bool ALIAS, class AfterLayer2, class G = BlockGroup,
          class AfterLayer1 = void (*)()>
__device__ __forceinline__ bool mlp_tile(bool arrived,
    const MlpShape& s, const GridParams& g, const SortedGrid& sg, uint32_t total, uint32_t tile,
    const float (&bias1)[kTH], const float* __restrict__ w1t, const float* __restrict__ b2,
    const StepParams& sp, const EulerParams& ep, const float* __restrict__ mask,
    float4* __restrict__ next_pos, float* __restrict__ next_states, float4* __restrict__ dx_out,
    float* __restrict__ ds_out, float* __restrict__ features_out, uint32_t step_index, float* ft,
    float* w1s, float* hid, float* w2s, float* outs, AfterLayer2&& after_layer2,
    AfterLayer1 after_layer1 = nullptr) {
  constexpr int TPR = HG / 8;  // layer-2 / epilogue threads per row (NT / M)
  const int C = sp.C, D = sp.D;
  const int r = G::tid() / TPR;
  const int part = G::tid() - r * TPR;
  // Each of a row's TPR threads owns a contiguous run of cpt channels, read
  // and written as float4 when the rows are 16-byte aligned.
  const int cpt = (C + TPR - 1) / TPR;
  const int c0 = part * cpt;
  const int cend = min(C, c0 + cpt);
  const bool vec = (C % 4 == 0) && (cpt % 4 == 0) && cpt <= kStateRegs &&
                   ((reinterpret_cast<uintptr_t>(sp.states) | reinterpret_cast<uintptr_t>(next_states) |
                     reinterpret_cast<uintptr_t>(ds_out)) & 15u) == 0;
  // The epilogue's position / mask reads are issued before layer 1 so
  // their latency is hidden behind it.  Tile row r is processing index t.
  const uint32_t t = tile * s.M + r;
  const bool live = t < total;
  size_t row = 0;
  float4 pi = make_float4(0.f, 0.f, 0.f, 0.f);
  float m = 1.0f;
  if (live) {
    const uint32_t q = slot_of(sg, t);
    const uint32_t batch = q / sg.n;
    const uint32_t local = __ldg(sg.permutation + q);
    row = size_t(batch) * sg.n + local;
    pi = __ldg(sg.positions + row);
    if (sp.lane_seeds)
      m = stochastic_update_mask(sp.update_prob, local, step_index, __ldg(sp.lane_seeds + batch));
    else if (mask)
      m = __ldg(mask + row);
  }
  if (features_out && live)
    for (int f = part; f < s.F; f += TPR) features_out[row * s.F + f] = ft[f * s.M + r];
  mlp_layer1<HG, NT, ALIAS, G>(s, w1t, bias1, ft, w1s, hid);
  if (G::sync_or(!arrived)) return false;
  if constexpr (!std::is_pointer<AfterLayer1>::value) after_layer1();
  // own state for the Euler update, hidden behind layer 2
  float sv[kStateRegs];
  if (vec) {
#pragma unroll
    for (int j4 = 0; j4 < kStateRegs / 4; ++j4) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live && 4 * j4 < cpt) v = __ldg(reinterpret_cast<const float4*>(sp.states + row * C + c0) + j4);
      sv[4 * j4] = v.x;
      sv[4 * j4 + 1] = v.y;
      sv[4 * j4 + 2] = v.z;
      sv[4 * j4 + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kStateRegs; ++j) {
      const int ch = c0 + j;
      sv[j] = (live && ch < cend) ? __ldg(sp.states + row * C + ch) : 0.0f;
    }
  }
  float liveness = 0.0f, sd = 0.0f;
  if (sp.gates3d && live) {
    liveness = __ldg(sp.states + row * C + 3);
    sd = __ldg(sp.states + row * C + 7);
  }
  mlp_layer2_any<G>(s, b2, hid, w2s, outs);
  G::sync();
  after_layer2();
  // forward_from_features_with_eps + gates + euler_step, TPR threads per row
  if (live) {
    const float* u = outs + r * s.out_stride;
    float norm = 0.0f;
#pragma unroll
    for (int a = 0; a < 3; ++a)
      if (a < D) norm = norm + u[a] * u[a];
    norm = sqrtf(norm);
    float dx[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int a = 0; a < 3; ++a)
      if (a < D) dx[a] = sp.alpha * u[a] * sp.motion_eps / (1.0f + norm);
    float state_gate = 1.0f;
    if (sp.gates3d) {
      // position_conditioned_3d_{maturity,motion}_gate (rollout/mod.rs:67-90)
      state_gate = clamp_rs((4.0f - liveness) * 2.0f, 0.0f, 1.0f);
      float motion_gate = 0.0f;
      if (!(pi.w >= 0.5f)) motion_gate = state_gate * clamp_rs((fabsf(sd) - 0.01f) / 0.02f, 0.0f, 1.0f);
#pragma unroll
      for (int a = 0; a < 4; ++a) dx[a] = dx[a] * motion_gate;
    }
    if (part == 0) {
      next_pos[row] = euler_position(g, ep, pi, dx, m);
      if (dx_out) dx_out[row] = make_float4(dx[0], dx[1], dx[2], dx[3]);
    }
    float nsv[kStateRegs], dsa[kStateRegs];
#pragma unroll
    for (int j = 0; j < kStateRegs; ++j) {
      const int ch = c0 + j;
      nsv[j] = 0.0f;
      dsa[j] = 0.0f;
      if (ch < cend) {
        float dsv = u[D + ch];
        if (sp.gates3d) dsv = dsv * state_gate;
        nsv[j] = euler_state(ep, C, ch, sv[j], dsv, m);
        dsa[j] = dsv;
      }
    }
    if (vec) {
#pragma unroll
      for (int j4 = 0; j4 < kStateRegs / 4; ++j4)
        if (4 * j4 < cpt) {
          reinterpret_cast<float4*>(next_states + row * C + c0)[j4] =
              make_float4(nsv[4 * j4], nsv[4 * j4 + 1], nsv[4 * j4 + 2], nsv[4 * j4 + 3]);
          if (ds_out)
            reinterpret_cast<float4*>(ds_out + row * C + c0)[j4] =
                make_float4(dsa[4 * j4], dsa[4 * j4 + 1], dsa[4 * j4 + 2], dsa[4 * j4 + 3]);
        }
    } else {
#pragma unroll
      for (int j = 0; j < kStateRegs; ++j) {
        const int ch = c0 + j;
        if (ch < cend) {
          next_states[row * C + ch] = nsv[j];
          if (ds_out) ds_out[row * C + ch] = dsa[j];
        }
      }
    }
    for (int ch = c0 + kStateRegs; ch < cend; ++ch) {
      float dsv = u[D + ch];
      if (sp.gates3d) dsv = dsv * state_gate;
      next_states[row * C + ch] = euler_state(ep, C, ch, __ldg(sp.states + row * C + ch), dsv, m);
      if (ds_out) ds_out[row * C + ch] = dsv;
    }
  }
  return true;
}

// The rollout step's MLP stage over feature tiles in sorted order.
template <int HG, int NT, int BLOCKS = 1>
__global__ void __launch_bounds__(NT, BLOCKS)
mlp_step_kernel(MlpShape s, GridParams g, SortedGrid sg, uint32_t total, uint32_t tile_begin,
                uint32_t tile_end, const float* __restrict__ tiles_in, const float* __restrict__ w1t,
                const float* __restrict__ b1, const float* __restrict__ w2,
                const float* __restrict__ b2, StepParams sp, EulerParams ep,
                const float* __restrict__ mask, float4* __restrict__ next_pos,
                float* __restrict__ next_states, float4* __restrict__ dx_out,
                float* __restrict__ ds_out, float* __restrict__ features_out) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  // One feature-tile buffer, filled by a bulk (TMA) copy on an mbarrier: the
  // next tile is fetched while the epilogue of this one runs (the tile is
  // dead once layer 1 has read it).
  const SmemLayout L = smem_layout(s);
  float* ft = smem + L.ft0;
  float* hid = smem + L.hid;
  float* w1s = smem + L.w1;
  float* w2s = smem + L.w2;
  float* outs = smem + L.outs;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
  const uint32_t tiles = tile_end;
  const uint32_t tile_bytes = uint32_t(s.F) * uint32_t(s.M) * 4u;  // a multiple of 16
  auto issue = [&](uint32_t t) {
    if (threadIdx.x == 0) bulk_tile_load(ft, tiles_in + size_t(t) * s.F * s.M, tile_bytes, bar);
  };
  uint32_t phase = 0;
  uint32_t tile = tile_begin + blockIdx.x;
  if (threadIdx.x == 0) mbar_init(bar);
  __syncthreads();
  if (tile < tiles) issue(tile);
  load_weights(s, w1t, w2, w1s, w2s);
  float bias1[kTH];
  load_bias1<HG>(s, b1, bias1);
  const uint32_t step_index = sp.lane_seeds ? __ldg(sp.step_counter) : 0u;
  __syncthreads();  // the weights in shared memory are complete before any layer 1
  // No barrier at the top of a tile: a thread waits for the tile's copy on
  // the mbarrier itself and goes on into layer 1 while slower threads finish
  // the previous tile's epilogue (which reads neither ft nor hid); the block's
  // decision on a copy that did not complete comes at the barrier after
  // layer 1.
  for (; tile < tiles; tile += gridDim.x) {
    const bool arrived = mbar_wait(bar, phase);
    const bool done = mlp_tile<HG, NT, (BLOCKS > 1)>(
        arrived, s, g, sg, total, tile, bias1, w1t, b2, sp, ep, mask, next_pos, next_states,
        dx_out, ds_out, features_out, step_index, ft, w1s, hid, w2s, outs, [&] {
          const uint32_t next = tile + gridDim.x;
          if (next < tiles) issue(next);
        });
    if (!done) {
      // The copy did not complete in time (for some thread): the whole block
      // counts it, gives the copy a last bounded wait so nothing lands in its
      // shared memory after it exits, and leaves the remaining tiles undone.
      if (threadIdx.x == 0) {
        atomicAdd(&g_bulk_copy_timeouts, 1ull);
        mbar_wait(bar, phase);
      }
      return;
    }
    phase ^= 1u;
  }
}

// The fused step: perception and the MLP stage in one kernel, the feature
// tile never leaving shared memory.  Each block loops over tiles of M sorted
// slots: its threads first compute the tile's feature rows (one thread per
// slot and CH-channel chunk, the perception kernels' per-particle code) into
// ft [F][M], then run mlp_tile on them.  hid overlays ft, which keeps a block
// under half of the SM's shared memory: two blocks per SM, so one block's
// neighbour gathers overlap the other's FP32 work.
constexpr int kFusedThreads = 192;

template <int HG, int DIM, int CH, int OPT>
__global__ void __launch_bounds__(kFusedThreads, 2)
fused_step_kernel(MlpShape s, GridParams g, PerceptionParams pp, SortedGrid sg, HitLists hl,
                  const float* __restrict__ volume, int chunks, uint32_t total,
                  uint32_t tile_begin, uint32_t tile_end, const float* __restrict__ w1t,
                  const float* __restrict__ b1, const float* __restrict__ w2,
                  const float* __restrict__ b2, StepParams sp, EulerParams ep,
                  const float* __restrict__ mask, float4* __restrict__ next_pos,
                  float* __restrict__ next_states, float4* __restrict__ dx_out,
                  float* __restrict__ ds_out, float* __restrict__ features_out) {
  constexpr int NT = kFusedThreads;
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const SmemLayout L = smem_layout(s);
  float* ft = smem + L.ft0;
  float* hid = smem + L.hid;
  float* w1s = smem + L.w1;
  float* w2s = smem + L.w2;
  float* outs = smem + L.outs;
  load_weights(s, w1t, w2, w1s, w2s);
  float bias1[kTH];
  load_bias1<HG>(s, b1, bias1);
  const uint32_t step_index = sp.lane_seeds ? __ldg(sp.step_counter) : 0u;
  const int C = sp.C;
  const int items = s.M * chunks;
  for (uint32_t tile = tile_begin + blockIdx.x; tile < tile_end; tile += gridDim.x) {
    for (int it = threadIdx.x; it < items; it += NT) {
      const int rr = it / chunks;
      const int chunk = it - rr * chunks;
      const int c0 = chunk * CH;
      const uint32_t t = tile * s.M + rr;  // processing index
      float* col = ft + rr;
      if (t >= total) {
        for (int k = chunk; k < s.F; k += chunks) col[k * s.M] = 0.0f;
        continue;
      }
      const uint32_t q = slot_of(sg, t);
      const uint32_t batch = q / sg.n;
      const size_t row = size_t(batch) * sg.n + sg.permutation[q];
      const float4 pi = __ldg(sg.positions + row);
      const int3 c = slot_cell<DIM>(sg, q);
      float si[CH];
      load_row<CH>(sp.states, row, C, c0, false, si);
      PerceptionAcc<DIM, CH> a;
      perceive_chunk<DIM, CH, OPT>(g, pp, sg, hl, batch, q, t, pi, c, sp.states, C, c0, volume,
                                   si, a);
      emit_features<DIM, CH>(pp, C, c0, chunk == 0, si, a, pi,
                             [&](int k, float v) { col[k * s.M] = v; });
    }
    __syncthreads();
    // mlp_tile synchronises after layer 2, so the next tile's feature rows
    // (which overwrite hid) wait for it.
    mlp_tile<HG, NT, true>(true, s, g, sg, total, tile, bias1, w1t, b2, sp, ep, mask, next_pos,
                           next_states, dx_out, ds_out, features_out, step_index, ft, w1s, hid,
                           w2s, outs, [] {});
  }
}

// ---- the warp-specialised step ----
// One 512-thread block per SM: warps 0-7 (producers, 80 registers) compute
// the perception of a tile of 128 sorted slots (one thread per slot and
// 8-channel chunk) into one of two shared feature buffers; warps 8-15
// (consumers, 176 registers) run the MLP tile on the other buffer.  The
// buffers hand over on mbarriers (full: 256 producer arrivals; empty: one
// consumer arrival once layer 1 has read the buffer), so the producers'
// neighbour gathers overlap the consumers' FP32 work on the same SM, and
// each role has the register budget its code needs (setmaxnreg: 256 x 80 +
// 256 x 176 = the block's 512 x 128).  Every wait is bounded; a wait that
// gives up sets the block's abort flag, which every other wait also checks,
// and counts in g_ws_timeouts.
constexpr int kWsThreads = 512;
constexpr int kWsProducers = 256;
constexpr int kWsConsumers = 256;
__device__ unsigned long long g_ws_timeouts = 0;

struct ConsumerGroup {
  static __device__ __forceinline__ int tid() { return int(threadIdx.x) - kWsProducers; }
  static __device__ __forceinline__ int size() { return kWsConsumers; }
  static __device__ __forceinline__ void sync() {
    asm volatile("bar.sync 1, %0;\n" ::"n"(kWsConsumers) : "memory");
  }
  static __device__ __forceinline__ bool sync_or(bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n bar.red.or.pred b, 1, %2, a;\n"
        " selp.u32 %0, 1, 0, b;\n}\n"
        : "=r"(r)
        : "r"(uint32_t(p)), "n"(kWsConsumers)
        : "memory");
    return r != 0;
  }
};

__device__ __forceinline__ void mbar_init_count(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// Waits for phase `parity` for at most about two seconds, giving up early
// when the block's abort flag is set; false (flag set) when it gave up.
__device__ __forceinline__ bool ws_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t0));
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if (*abort_flag) return false;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    if (t - t0 > 2000000000ull) {
      *abort_flag = 1;
      return false;
    }
  }
}

struct WsLayout {
  size_t ft, hid, w1, w2, outs, bar, total;  // offsets in floats
};
__host__ __device__ inline WsLayout ws_layout(const MlpShape& s) {
  WsLayout l;
  size_t off = 0;
  auto take = [&](size_t floats) {
    size_t o = off;
    off += (floats + 3) & ~size_t(3);
    return o;
  };
  l.ft = take(2 * size_t(s.F) * s.M);
  l.hid = take(size_t(s.M) * s.hid_stride);
  l.w1 = take(size_t(s.F) * s.Hp);
  l.w2 = take(size_t(s.O) * s.w2_stride);
  l.outs = take(size_t(s.M) * s.out_stride);
  l.bar = take(12);  // full[2], empty[2] (8 bytes each), the abort flag
  l.total = off;
  return l;
}

template <int HG, int CH, int OPT>
__global__ void __launch_bounds__(kWsThreads, 1)
ws_step_kernel(MlpShape s, GridParams g, PerceptionParams pp, SortedGrid sg, HitLists hl,
               const float* __restrict__ volume, int chunks, uint32_t total, uint32_t ntiles,
               const float* __restrict__ w1t, const float* __restrict__ b1,
               const float* __restrict__ w2, const float* __restrict__ b2, StepParams sp,
               EulerParams ep, const float* __restrict__ mask, float4* __restrict__ next_pos,
               float* __restrict__ next_states) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const WsLayout L = ws_layout(s);
  float* ft0 = smem + L.ft;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
  uint64_t* empty = full + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 4);
  if (threadIdx.x == 0) {
    mbar_init_count(&full[0], kWsProducers);
    mbar_init_count(&full[1], kWsProducers);
    mbar_init_count(&empty[0], 1);
    mbar_init_count(&empty[1], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  const size_t FM = size_t(s.F) * s.M;
  if (threadIdx.x < kWsProducers) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 80;\n" ::: "memory");
    const int C = sp.C;
    const int rr = int(threadIdx.x) / chunks;  // this thread's row of every tile
    const int chunk = int(threadIdx.x) - rr * chunks;
    const int c0 = chunk * CH;
    uint32_t k = 0;
    for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++k) {
      const uint32_t b = k & 1u, use = k >> 1;
      if (use > 0 && !ws_wait(&empty[b], (use - 1u) & 1u, abort_flag)) break;
      float* col = ft0 + b * FM + rr;
      const uint32_t t = tile * s.M + rr;  // processing index
      if (rr >= s.M) {
        // no row (one chunk per particle: threads past the tile's rows)
      } else if (t >= total) {
        for (int f = chunk; f < s.F; f += chunks) col[size_t(f) * s.M] = 0.0f;
      } else {
        const uint32_t q = slot_of(sg, t);
        const uint32_t batch = q / sg.n;
        const size_t row = size_t(batch) * sg.n + sg.permutation[q];
        const float4 pi = __ldg(sg.positions + row);
        const int3 c = slot_cell<2>(sg, q);
        float si[CH];
        load_row<CH>(sp.states, row, C, c0, false, si);
        PerceptionAcc<2, CH> a;
        perceive_chunk<2, CH, OPT>(g, pp, sg, hl, batch, q, t, pi, c, sp.states, C, c0, volume,
                                   si, a);
        emit_features<2, CH>(pp, C, c0, chunk == 0, si, a, pi,
                             [&](int f, float v) { col[size_t(f) * s.M] = v; });
      }
      mbar_arrive(&full[b]);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 176;\n" ::: "memory");
    float* hid = smem + L.hid;
    float* w1s = smem + L.w1;
    float* w2s = smem + L.w2;
    float* outs = smem + L.outs;
    load_weights<ConsumerGroup>(s, w1t, w2, w1s, w2s);
    float bias1[kTH];
    load_bias1<HG, ConsumerGroup>(s, b1, bias1);
    const uint32_t step_index = sp.lane_seeds ? __ldg(sp.step_counter) : 0u;
    ConsumerGroup::sync();  // the weights are complete before any layer 1
    uint32_t k = 0;
    for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++k) {
      const uint32_t b = k & 1u, use = k >> 1;
      const bool arrived = ws_wait(&full[b], use & 1u, abort_flag);
      auto nothing = [] {};
      auto release = [&] {
        // layer 1 is done with the buffer: the producers may refill it
        if (ConsumerGroup::tid() == 0) mbar_arrive(&empty[b]);
      };
      const bool ok =
          mlp_tile<HG, kWsConsumers, false, decltype(nothing)&, ConsumerGroup, decltype(release)>(
              arrived, s, g, sg, total, tile, bias1, w1t, b2, sp, ep, mask, next_pos,
              next_states, nullptr, nullptr, nullptr, step_index, ft0 + b * FM, w1s, hid, w2s,
              outs, nothing, release);
      if (!ok) {
        if (ConsumerGroup::tid() == 0) {
          *abort_flag = 1;
          atomicAdd(&g_ws_timeouts, 1ull);
        }
        break;
      }
    }
  }
}

MlpShape shape_with(const DeviceModel& m, int nt) {
  MlpShape s;
  s.NT = nt;
  s.F = m.feature_dims;
  s.H = m.hidden_dims;
  s.Hp = m.hidden_padded;
  s.O = m.update_dims;
  const int HG = s.Hp / kTH;
  s.M = (nt / HG) * 8;
  s.tpr = nt / s.M;
  s.hid_stride = s.Hp + 4;
  s.w2_stride = s.Hp + 4;
  s.out_stride = s.O + 1;
  s.alias = 0;
  s.w1_resident = 1;
  if (smem_layout(s).total * sizeof(float) > kSmemBudget) s.w1_resident = 0;
  // Layer-2 output slots per row: R tpr ceil(O / (R tpr)).  Triples when M
  // splits into them, they waste no more slots than pairs, and a row group's
  // R tpr threads read at most 8 distinct weight rows (8 x 16 bytes: one
  // shared-memory wavefront per load).  Measured: cfg2 (tpr 2) MLP 0.927 vs
  // 0.954 ms with triples; cfg3 (tpr 4, 12 weight rows) 0.0996 vs 0.0983 ms.
  auto slots = [&](int r) { return r * s.tpr * ((s.O + r * s.tpr - 1) / (r * s.tpr)); };
  s.l2_rows = (s.M % 3 == 0 && 3 * s.tpr <= 8 && slots(3) <= slots(2)) ? 3 : 2;
  return s;
}

// The 384-thread shape when its tile fits in shared memory and its waves of
// tiles (one tile per SM at a time, 148 SMs) take no longer than the 256-thread
// shape's: waves x rows per tile, the narrow tile's rows costing 5 % more
// (8 instead of 12 warps per SM).  So batches of rollouts take wide tiles,
// while a single small rollout spreads smaller tiles over more SMs.  rows = 0
// asks for the narrow shape.
MlpShape make_shape(const DeviceModel& m, uint64_t rows) {
  const MlpShape wide = shape_with(m, kThreadsWide);
  const MlpShape narrow = shape_with(m, kThreadsNarrow);
  if (rows == 0 || smem_layout(wide).total * sizeof(float) > kSmemBudget) return narrow;
  auto waves = [&](const MlpShape& s) { return (rows + 148u * s.M - 1) / (148u * s.M); };
  const double t_wide = double(waves(wide)) * wide.M;
  const double t_narrow = double(waves(narrow)) * narrow.M * 1.05;
  return t_wide <= t_narrow ? wide : narrow;
}

// The fused kernel's shape: 192 threads, hid over ft, at most half of an
// SM's shared memory per block (w1 streamed when its resident copy does not
// fit).
constexpr size_t kFusedSmemBudget = 112 * 1024;
MlpShape fused_shape(const DeviceModel& m) {
  MlpShape s = shape_with(m, kFusedThreads);
  s.alias = 1;
  s.w1_resident = 1;
  if (smem_layout(s).total * sizeof(float) > kFusedSmemBudget) s.w1_resident = 0;
  return s;
}

struct LaunchCfg {
  unsigned grid;
  size_t smem;
};

template <class K>
npa_status plan(K kernel, const MlpShape& s, uint64_t tiles, LaunchCfg* out) {
  const size_t smem = smem_layout(s).total * sizeof(float);
  int per_sm = 0, sms = 0;
  NPA_TRY(kernel_occupancy(reinterpret_cast<const void*>(kernel), s.NT, smem, &per_sm, &sms));
  if (per_sm < 1) return fail(NPA_ERR_UNSUPPORTED, "MLP kernel cannot be resident");
  const uint64_t slots = uint64_t(per_sm) * sms;
  out->grid = static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>(tiles, slots)));
  out->smem = smem;
  return NPA_OK;
}

bool shape_ok(const DeviceModel& m) {
  if (m.hidden_padded != 64 && m.hidden_padded != 128 && m.hidden_padded != 256) return false;
  const MlpShape s = make_shape(m, 0);  // the narrow shape: it fits whenever any does
  return (m.update_dims + s.tpr - 1) / s.tpr <= kMaxOut && m.feature_dims >= 1 &&
         smem_layout(s).total * sizeof(float) <= kSmemBudget;
}

}  // namespace

int hidden_padded_for(int hidden) { return hidden <= 64 ? 64 : (hidden <= 128 ? 128 : 256); }

// The rollout step's MLP shape: two 192-thread blocks per SM whose hidden
// rows overlay the feature tile (each block under half of the SM's shared
// memory), so one block's barriers and tile waits are covered by the other
// block's FP32 work.  Measured against one 384-thread block per SM (cfg2
// MLP stage 0.884 vs 0.896 ms; 32 rollouts 0.132 vs 0.139 ms; cfg0 0.0248 vs
// 0.0267 ms).  Hidden width 256 keeps the one-block shapes (its layer-1
// thread grid needs a multiple of four warps per block; 192 threads have six).
MlpShape make_step_shape(const DeviceModel& m, uint64_t rows) {
  if (rows > 0 && m.hidden_padded <= 128) {
    MlpShape s = shape_with(m, kTwoBlockThreads);
    s.alias = 1;
    s.w1_resident = 1;
    if (2 * (smem_layout(s).total * sizeof(float) + 1024) <= 227 * 1024) return s;
  }
  return make_shape(m, rows);
}

int step_tile_rows(const DeviceModel& m, uint64_t rows) { return make_step_shape(m, rows).M; }

bool mlp_step_supported(const DeviceModel& m) {
  return m.state_dims >= 0 && m.hidden_dims >= 1 && m.hidden_dims <= 256 && shape_ok(m);
}

npa_status launch_forward_update(const DeviceModel& m, const float* features, uint32_t rows,
                                 float* update, cudaStream_t stream) {
  if (rows == 0) return NPA_OK;
  if (!mlp_step_supported(m))
    return fail(NPA_ERR_UNSUPPORTED, "MLP shape outside the supported range");
  const MlpShape s = make_shape(m, rows);
  const uint64_t tiles = (uint64_t(rows) + s.M - 1) / s.M;
  LaunchCfg lc;
#define NPA_FWD(HGV, NTV)                                                                     \
  do {                                                                                        \
    NPA_TRY(plan(forward_update_kernel<HGV, NTV>, s, tiles, &lc));                            \
    forward_update_kernel<HGV, NTV><<<lc.grid, NTV, lc.smem, stream>>>(s, m.w1t, m.b1, m.w2,  \
                                                                       m.b2, features, rows,  \
                                                                       update);               \
  } while (0)
#define NPA_FWD_NT(NTV)                          \
  do {                                           \
    if (s.Hp == 64) NPA_FWD(64 / kTH, NTV);      \
    else if (s.Hp == 128) NPA_FWD(128 / kTH, NTV); \
    else NPA_FWD(256 / kTH, NTV);                \
  } while (0)
  if (s.NT == kThreadsWide) NPA_FWD_NT(kThreadsWide);
  else NPA_FWD_NT(kThreadsNarrow);
#undef NPA_FWD_NT
#undef NPA_FWD
  return after_launch("forward_update_kernel");
}

__global__ void advance_step_kernel(uint32_t* counter) { counter[0] += 1u; }

// mean_dx of run_rollout (rollout/mod.rs:276-283): the mean over particles of
// |dx| = sqrt(dx0^2 + dx1^2 + dx2^2), each norm in the reference's f32 order.
// The sum runs in f64 in a fixed order (contiguous block ranges, then the
// block partials in index order), so it is deterministic and at least as
// accurate as the reference's sequential f32 sum.
constexpr int kNormThreads = 256;
constexpr int kNormBlocks = 148;

__device__ __forceinline__ double block_sum(double v, double* sh) {
  sh[threadIdx.x] = v;
  __syncthreads();
  for (int stride = kNormThreads / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) sh[threadIdx.x] += sh[threadIdx.x + stride];
    __syncthreads();
  }
  return sh[0];
}

__global__ void __launch_bounds__(kNormThreads)
norm_partials_kernel(const float4* __restrict__ dx, uint32_t total, double* __restrict__ partials) {
  __shared__ double sh[kNormThreads];
  const uint32_t per = (total + gridDim.x - 1) / gridDim.x;
  const uint32_t lo = min(total, blockIdx.x * per), hi = min(total, lo + per);
  double acc = 0.0;
  for (uint32_t i = lo + threadIdx.x; i < hi; i += kNormThreads) {
    const float4 v = __ldg(dx + i);
    float n2 = v.x * v.x;
    n2 = n2 + v.y * v.y;
    n2 = n2 + v.z * v.z;
    acc += static_cast<double>(sqrtf(n2));
  }
  const double sum = block_sum(acc, sh);
  if (threadIdx.x == 0) partials[blockIdx.x] = sum;
}

__global__ void __launch_bounds__(kNormThreads)
norm_final_kernel(const double* __restrict__ partials, int count, uint32_t total,
                  float* __restrict__ out) {
  __shared__ double sh[kNormThreads];
  const double v = threadIdx.x < count ? partials[threadIdx.x] : 0.0;
  const double sum = block_sum(v, sh);
  if (threadIdx.x == 0)
    out[0] = static_cast<float>(sum) / static_cast<float>(total > 1 ? total : 1u);
}

npa_status launch_mean_norm(const float4* dx, uint32_t total, double* partials, float* out,
                            cudaStream_t stream) {
  norm_partials_kernel<<<kNormBlocks, kNormThreads, 0, stream>>>(dx, total, partials);
  NPA_TRY(after_launch("norm_partials_kernel"));
  norm_final_kernel<<<1, kNormThreads, 0, stream>>>(partials, kNormBlocks, total, out);
  return after_launch("norm_final_kernel");
}

size_t mean_norm_scratch_bytes() { return kNormBlocks * sizeof(double); }

npa_status launch_advance_step(uint32_t* counter, cudaStream_t stream) {
  advance_step_kernel<<<1, 1, 0, stream>>>(counter);
  return after_launch("advance_step_kernel");
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

uint64_t bulk_copy_timeouts() {
  unsigned long long v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bulk_copy_timeouts, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return v;
}

namespace {
StepParams step_params(const DeviceModel& m, const GridParams& g, const float* states,
                       const StochasticMask& sm) {
  StepParams sp;
  sp.states = states;
  sp.update_prob = sm.update_prob;
  sp.lane_seeds = sm.lane_seeds;
  sp.step_counter = sm.step_counter;
  sp.alpha = m.alpha;
  sp.motion_eps = m.equivariance == NPA_EQUIV_PARTICLE_DENSITY_AND_SCALE ? g.eps : m.eps0;
  sp.gates3d = (g.dim == 3 && m.position_features && m.state_dims > 3) ? 1 : 0;
  sp.C = m.state_dims;
  sp.D = g.dim;
  return sp;
}
}  // namespace

npa_status launch_mlp_step(const DeviceModel& m, const GridParams& g, const SortedGrid& sgrid,
                           uint32_t batch, const float* tiles, const float* states, float dt,
                           const float* mask, const StochasticMask& sm,
                           const StepOutputs& out, cudaStream_t stream, uint32_t tile_begin,
                           uint32_t tile_end) {
  const uint32_t total = batch * sgrid.n;
  if (total == 0) return NPA_OK;
  if (!mlp_step_supported(m))
    return fail(NPA_ERR_UNSUPPORTED, "MLP shape outside the supported range");
  // the bulk copies of the feature tiles start on 16-byte boundaries
  if (reinterpret_cast<uintptr_t>(tiles) & 15u)
    return fail(NPA_ERR_INVALID_ARGUMENT, "step workspace must be 16-byte aligned");
  const MlpShape s = make_step_shape(m, total);
  const StepParams sp = step_params(m, g, states, sm);
  const EulerParams e{dt, g.dim == 3 ? 4 : 2, (g.dim == 3 && m.state_dims > 3) ? 1 : 0};
  const uint32_t ntiles_all = static_cast<uint32_t>((uint64_t(total) + s.M - 1) / s.M);
  tile_end = std::min(tile_end, ntiles_all);
  if (tile_end <= tile_begin) return NPA_OK;
  const uint64_t ntiles = tile_end - tile_begin;
  LaunchCfg lc;
#define NPA_MLP(HGV, NTV)                                                                     \
  do {                                                                                        \
    constexpr int kBlocks = NTV == kTwoBlockThreads ? 2 : 1;                                  \
    NPA_TRY(plan(mlp_step_kernel<HGV, NTV, kBlocks>, s, ntiles, &lc));                        \
    mlp_step_kernel<HGV, NTV, kBlocks><<<lc.grid, NTV, lc.smem, stream>>>(                    \
        s, g, sgrid, total, tile_begin, tile_end, tiles, m.w1t, m.b1, m.w2, m.b2, sp, e, mask, \
        out.next_positions, out.next_states, out.dx, out.ds, out.features);                   \
  } while (0)
#define NPA_MLP_NT(NTV)                          \
  do {                                           \
    if (s.Hp == 64) NPA_MLP(64 / kTH, NTV);      \
    else if (s.Hp == 128) NPA_MLP(128 / kTH, NTV); \
    else NPA_MLP(256 / kTH, NTV);                \
  } while (0)
  if (s.NT == kThreadsWide) NPA_MLP_NT(kThreadsWide);
  else if (s.NT == kTwoBlockThreads) {
    if (s.Hp == 64) NPA_MLP(64 / kTH, kTwoBlockThreads);
    else NPA_MLP(128 / kTH, kTwoBlockThreads);
  }
  else NPA_MLP_NT(kThreadsNarrow);
#undef NPA_MLP_NT
#undef NPA_MLP
  return after_launch("mlp_step_kernel");
}

bool fused_step_supported(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                          uint32_t batch, uint32_t total) {
  if (g.dim != 2 || m.state_dims <= 4 || !mlp_step_supported(m)) return false;
  if (m.hidden_padded != 64 && m.hidden_padded != 128) return false;
  if (p.feature_dims != m.feature_dims) return false;
  // the dense-cell (warp-cooperative) walk is not part of the fused kernel
  if (uint64_t(total) >= uint64_t(8) * batch * g.cells) return false;
  const MlpShape s = fused_shape(m);
  return (m.update_dims + s.tpr - 1) / s.tpr <= kMaxOut &&
         smem_layout(s).total * sizeof(float) <= kFusedSmemBudget;
}

npa_status launch_fused_step(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                             const SortedGrid& sgrid, const HitLists& hl, uint32_t batch,
                             const float* states, const float* volume_sorted, float dt,
                             const float* mask, const StochasticMask& sm, const StepOutputs& out,
                             cudaStream_t stream) {
  const uint32_t total = batch * sgrid.n;
  if (total == 0) return NPA_OK;
  if (!fused_step_supported(m, g, p, batch, total))
    return fail(NPA_ERR_UNSUPPORTED, "fused step outside the supported range");
  PerceptionParams pp = p;
  pp.vec_states = (reinterpret_cast<uintptr_t>(states) % 16) == 0;
  if (p.log_norm_grad || p.log_norm_density_grad) NPA_TRY(device_log1p_table(&pp.l1p, stream));
  const MlpShape s = fused_shape(m);
  const StepParams sp = step_params(m, g, states, sm);
  const EulerParams e{dt, 2, 0};
  const int chunks = (m.state_dims + 7) / 8;
  const uint32_t ntiles = static_cast<uint32_t>((uint64_t(total) + s.M - 1) / s.M);
  const bool fixed_opts = p.state_grad && !p.density_grad && p.hybrid;
  LaunchCfg lc;
#define NPA_FUSED(HGV, OPTV)                                                                    \
  do {                                                                                          \
    NPA_TRY(plan(fused_step_kernel<HGV, 2, 8, OPTV>, s, ntiles, &lc));                          \
    fused_step_kernel<HGV, 2, 8, OPTV><<<lc.grid, kFusedThreads, lc.smem, stream>>>(             \
        s, g, pp, sgrid, hl, volume_sorted, chunks, total, 0, ntiles, m.w1t, m.b1, m.w2, m.b2,   \
        sp, e, mask, out.next_positions, out.next_states, out.dx, out.ds, out.features);         \
  } while (0)
  if (s.Hp == 64) {
    if (fixed_opts) NPA_FUSED(64 / kTH, 1); else NPA_FUSED(64 / kTH, 0);
  } else {
    if (fixed_opts) NPA_FUSED(128 / kTH, 1); else NPA_FUSED(128 / kTH, 0);
  }
#undef NPA_FUSED
  return after_launch("fused_step_kernel");
}

bool ws_step_supported(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                       uint32_t batch, uint32_t total) {
  if (g.dim != 2 || m.state_dims < 1 || m.state_dims > 16 || !mlp_step_supported(m)) return false;
  if (m.hidden_padded != 128 || p.feature_dims != m.feature_dims) return false;
  if (uint64_t(total) >= uint64_t(8) * batch * g.cells) return false;  // dense cells
  const MlpShape s = shape_with(m, kWsConsumers);
  return s.M == 128 && (m.update_dims + s.tpr - 1) / s.tpr <= kMaxOut &&
         ws_layout(s).total * sizeof(float) <= kSmemBudget;
}

npa_status launch_ws_step(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                          const SortedGrid& sgrid, const HitLists& hl, uint32_t batch,
                          const float* states, const float* volume_sorted, float dt,
                          const float* mask, const StochasticMask& sm, const StepOutputs& out,
                          cudaStream_t stream) {
  const uint32_t total = batch * sgrid.n;
  if (total == 0) return NPA_OK;
  if (!ws_step_supported(m, g, p, batch, total))
    return fail(NPA_ERR_UNSUPPORTED, "warp-specialised step outside the supported range");
  PerceptionParams pp = p;
  pp.vec_states = (reinterpret_cast<uintptr_t>(states) % 16) == 0;
  if (p.log_norm_grad || p.log_norm_density_grad) NPA_TRY(device_log1p_table(&pp.l1p, stream));
  MlpShape s = shape_with(m, kWsConsumers);
  s.w1_resident = 1;
  const StepParams sp = step_params(m, g, states, sm);
  const EulerParams e{dt, 2, 0};
  const int ch = m.state_dims <= 4 ? 4 : 8;
  const int chunks = (m.state_dims + ch - 1) / ch;
  const uint32_t ntiles = static_cast<uint32_t>((uint64_t(total) + s.M - 1) / s.M);
  const bool fixed_opts = p.state_grad && !p.density_grad && p.hybrid;
  const size_t smem = ws_layout(s).total * sizeof(float);
  int per_sm = 0, sms = 0;
#define NPA_WS(CHV, OPTV)                                                                      \
  do {                                                                                         \
    NPA_TRY(kernel_occupancy(reinterpret_cast<const void*>(ws_step_kernel<16, CHV, OPTV>),     \
                             kWsThreads, smem, &per_sm, &sms));                                \
    if (per_sm < 1) return fail(NPA_ERR_UNSUPPORTED, "warp-specialised step cannot be resident"); \
    const unsigned grid = static_cast<unsigned>(std::min<uint64_t>(ntiles, uint64_t(sms))); \
    ws_step_kernel<16, CHV, OPTV><<<grid, kWsThreads, smem, stream>>>(                         \
        s, g, pp, sgrid, hl, volume_sorted, chunks, total, ntiles, m.w1t, m.b1, m.w2, m.b2,     \
        sp, e, mask, out.next_positions, out.next_states);                                     \
  } while (0)
  if (ch == 4) {
    if (fixed_opts) NPA_WS(4, 1); else NPA_WS(4, 0);
  } else {
    if (fixed_opts) NPA_WS(8, 1); else NPA_WS(8, 0);
  }
#undef NPA_WS
  return after_launch("ws_step_kernel");
}

uint64_t ws_step_timeouts() {
  unsigned long long v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ws_timeouts, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return v;
}

}  // namespace npa
