// perception.cu -- density pass and SPH perception
// (perceive_with_options, crates/burn_automata_kernels/src/reference/forward.rs:26-143).
//
// All kernels run one thread per sorted slot and 8-channel chunk, so the threads of a warp walk neighbouring bins and read the
// sorted neighbour records contiguously.  DIM (2 or 3) and the channel chunk
// CH are template parameters: every accumulator is a register.
//   density_kernel          rho and 1/rho per sorted slot (forward.rs:145-160)
//   perception_kernel       API output: features and intermediates in the
//                           caller's particle order
//   perception_tiles_kernel step path: the feature rows of `tile_rows` sorted
//                           slots stored feature-major ([tile][F][rows]), the
//                           layout the MLP kernel stages into shared memory
#include <algorithm>

#include "perception_core.cuh"

namespace npa {
namespace {

// 2D: six 128-thread blocks per SM (80 registers, a few spills to L1): the
// neighbour gathers are latency-bound, and 24 warps per SM beat 16 at 127
// registers (cfg2 perception 0.446 vs 0.538 ms; 5 blocks 0.485, 8 blocks
// 0.512).  3D keeps more accumulators (3 gradient axes, a 3 x 3 moment) and
// spills too much at 80 registers (cfg3 perception 0.261 ms); four blocks
// (128 registers) give 0.167 ms, no bound (196 registers) 0.176 ms.
template <int DIM>
struct PerceptionBlocks {
  static constexpr int value = DIM == 2 ? 6 : 4;
};

// KB = candidates whose records are in flight per thread in the flattened
// walk: 4 hides the gathers' latency when few warps run (single small
// rollouts), 1 issues fewer instructions when the launch fills the GPU
// (cfg2 density 0.185 vs 0.202 ms; cfg3 0.101 vs 0.090 ms the other way).
template <int DIM, bool COOP, int KB>
__global__ void __launch_bounds__(256)
density_kernel(GridParams g, SortedGrid s, uint32_t total, float* __restrict__ volume,
               float* __restrict__ density_out, HitLists hl) {
  __shared__ WarpWindow windows[COOP ? 256 / 32 : 1];
  // 2D, one candidate in flight: the walk's bin table, one column per thread
  __shared__ uint32_t tab[(DIM == 2 && KB == 1) ? 18 * 256 : 1];
  // processing index t (hit lists are indexed by it), sorted slot q
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  // Whole warp in range (warp-uniform), so warp collectives below are safe.
  const bool full_warp = (t | 31u) < total;
  if (t >= total) return;
  const uint32_t q = slot_of(s, t);
  const uint32_t batch = q / s.n;
  float4 pi;
  int3 c;
  load_record<DIM>(s, q, pi, c);
  float rho = 0.0f;
  uint32_t hits = 0;
  uint32_t* list = hl.slots ? hl.slots + t : nullptr;
  auto visit = [&](uint32_t qj, float r2) {
    rho = rho + poly6(g, r2);
    if (list && hits < uint32_t(hl.cap)) list[size_t(hits) * hl.stride] = qj;
    ++hits;
  };
  uint32_t peers = 0;
  if (COOP && full_warp) peers = warp_cell_peers(batch, c);
  if (COOP && full_warp && warp_cell_groups(peers) <= kMaxWarpCellGroups) {
    for_each_neighbor_warp<DIM>(g, s, batch, pi, c, peers, windows[threadIdx.x >> 5],
                                [](uint32_t, uint32_t) {},
                                [&](uint32_t, uint32_t qj, float4, float r2) { visit(qj, r2); });
  } else {
    if constexpr (DIM == 2 && KB == 1)
      for_each_neighbor_tab<DIM>(g, s, batch, pi, c, tab + threadIdx.x, 256u,
                                 [&](uint32_t qj, float4, float r2) { visit(qj, r2); });
    else
      for_each_neighbor<DIM, KB>(g, s, batch, pi, c,
                                [&](uint32_t qj, float4, float r2) { visit(qj, r2); });
  }
  if (list) hl.count[t] = min(hits, uint32_t(hl.cap + 1));
  volume[q] = recip_finite(rho);
  if (density_out) density_out[size_t(batch) * s.n + s.permutation[q]] = rho;
}

template <int CH>
__device__ __forceinline__ void load_own(const float* __restrict__ states, size_t row, int C,
                                         int c0, float (&si)[CH]) {
#pragma unroll
  for (int c = 0; c < CH; ++c) si[c] = (c0 + c < C) ? __ldg(states + row * C + c0 + c) : 0.0f;
}

template <int DIM, int CH, bool COOP, int OPT = 0>
__global__ void __launch_bounds__(128, PerceptionBlocks<DIM>::value)
perception_kernel(GridParams g, PerceptionParams p, SortedGrid s, HitLists hl, uint32_t total,
                  const float* __restrict__ states, int C, int chunks,
                  const float* __restrict__ volume, float* __restrict__ features,
                  float* __restrict__ blurred, float* __restrict__ state_gradient,
                  float* __restrict__ density_gradient) {
  __shared__ WarpWindow windows[COOP ? 128 / 32 : 1];
  const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool full_warp = (t | 31u) < uint64_t(total) * chunks;  // warp-uniform
  if (t >= uint64_t(total) * chunks) return;
  const uint32_t pt = static_cast<uint32_t>(t / chunks);  // processing index
  const int chunk = static_cast<int>(t - uint64_t(pt) * chunks);
  const int c0 = chunk * CH;
  const uint32_t q = slot_of(s, pt);
  const uint32_t batch = q / s.n;
  const size_t row = size_t(batch) * s.n + s.permutation[q];
  const float4 pi = __ldg(s.positions + row);
  const int3 c = slot_cell<DIM>(s, q);
  WarpWindow* win = nullptr;
  uint32_t peers = 0;
  if (COOP && full_warp) {
    peers = warp_cell_peers(batch, c);
    if (warp_cell_groups(peers) <= kMaxWarpCellGroups) win = &windows[threadIdx.x >> 5];
  }
  float si[CH];
  load_own<CH>(states, row, C, c0, si);
  PerceptionAcc<DIM, CH> a;
  perceive_chunk<DIM, CH, OPT>(g, p, s, hl, batch, q, pt, pi, c, states, C, c0, volume, si, a, win,
                          peers);
  const size_t F = p.feature_dims;
  float* f = features + row * F;
  emit_features<DIM, CH>(p, C, c0, chunk == 0, si, a, pi, [&](int k, float v) { f[k] = v; });
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int ch = c0 + k;
    if (ch < C) {
      if (blurred) blurred[row * C + ch] = a.blur[k];
      if (state_gradient && p.state_grad)
#pragma unroll
        for (int d = 0; d < DIM; ++d) state_gradient[(row * C + ch) * DIM + d] = a.sgrad[k][d];
    }
  }
  if (chunk == 0 && density_gradient && p.density_grad)
#pragma unroll
    for (int d = 0; d < DIM; ++d) density_gradient[row * DIM + d] = a.dgrad[d];
}

template <int DIM, int CH, bool COOP, int OPT>
__global__ void __launch_bounds__(128, PerceptionBlocks<DIM>::value)
perception_tiles_kernel(GridParams g, PerceptionParams p, SortedGrid s, HitLists hl,
                        uint32_t total, uint32_t q_begin, uint32_t q_end,
                        const float* __restrict__ states, int C, int chunks,
                        const float* __restrict__ volume, int tile_rows,
                        float* __restrict__ tiles) {
  __shared__ WarpWindow windows[COOP ? 128 / 32 : 1];
  const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  // warp-uniform: every lane in range and on a real particle
  const bool full_warp = (t | 31u) < uint64_t(q_end - q_begin) * chunks &&
                         q_begin + static_cast<uint32_t>((t | 31u) / chunks) < total;
  if (t >= uint64_t(q_end - q_begin) * chunks) return;
  // processing index pt: tile row pt, sorted slot q
  const uint32_t pt = q_begin + static_cast<uint32_t>(t / chunks);
  const int chunk = static_cast<int>(t - uint64_t(pt - q_begin) * chunks);
  const int c0 = chunk * CH;
  const size_t F = p.feature_dims;
  float* tile = tiles + size_t(pt / tile_rows) * F * tile_rows + (pt % tile_rows);
  if (pt >= total) {
    for (int k = chunk; k < int(F); k += chunks) tile[size_t(k) * tile_rows] = 0.0f;
    return;
  }
  const uint32_t q = slot_of(s, pt);
  const uint32_t batch = q / s.n;
  const size_t row = size_t(batch) * s.n + s.permutation[q];
  const float4 pi = __ldg(s.positions + row);
  const int3 c = slot_cell<DIM>(s, q);
  WarpWindow* win = nullptr;
  uint32_t peers = 0;
  if (COOP && full_warp) {
    peers = warp_cell_peers(batch, c);
    if (warp_cell_groups(peers) <= kMaxWarpCellGroups) win = &windows[threadIdx.x >> 5];
  }
  float si[CH];
  load_own<CH>(states, row, C, c0, si);
  PerceptionAcc<DIM, CH> a;
  perceive_chunk<DIM, CH, OPT, true>(g, p, s, hl, batch, q, pt, pi, c, states, C, c0, volume, si, a,
                               win, peers);
  emit_features<DIM, CH>(p, C, c0, chunk == 0, si, a, pi,
                         [&](int k, float v) { tile[size_t(k) * tile_rows] = v; });
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

// The warp-cooperative walk pays off when cells hold whole warps of
// particles; its kernels are only launched when the mean occupancy of the
// bins is at least 8 (cfg4's clusters: ~1000 per bin; cfg1: 4; cfg2: 1),
// since the extra code costs the sparse kernels registers (cfg2 perception
// 0.477 vs 0.437 ms).  Both variants give identical results.
bool dense_cells(const GridParams& g, uint32_t batch, uint32_t total) {
  return uint64_t(total) >= uint64_t(8) * batch * g.cells;
}

// Channels per thread: 8 (measured on cfg2: two threads of 8 channels per
// particle beat one of 16 -- 0.54 vs 0.72 ms -- through twice the occupancy).
int chunk_channels(int C) { return C <= 4 ? 4 : 8; }

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
                          float* volume_sorted, float* density_out, const HitLists& hl,
                          cudaStream_t stream) {
  const uint32_t total = batch * s.n;
  if (total == 0) return NPA_OK;
#define NPA_DENS(D, CO, KB)                                                          \
  density_kernel<D, CO, KB><<<grid_for(total, 256), 256, 0, stream>>>(g, s, total,      \
                                                                      volume_sorted,    \
                                                                      density_out, hl)
#define NPA_DENS_KB(D, CO)                      \
  do {                                          \
    if (wide) NPA_DENS(D, CO, 1);               \
    else NPA_DENS(D, CO, 4);                    \
  } while (0)
  const bool coop = dense_cells(g, batch, total);
  // One candidate in flight: in 2D (bin table in shared memory) from 65,536
  // particles (measured: 32 rollouts of 4,096 density 0.035 vs 0.039 ms, 64
  // rollouts 0.046 vs 0.062 ms; one rollout 0.029 vs 0.026 ms the other way),
  // in 3D from two waves of resident 256-thread blocks (four per SM).
  const bool wide = g.dim == 2 ? total >= 65536u : total >= 2u * 148u * 4u * 256u;
  if (g.dim == 2) {
    if (coop) NPA_DENS_KB(2, true); else NPA_DENS_KB(2, false);
  } else {
    if (coop) NPA_DENS_KB(3, true); else NPA_DENS_KB(3, false);
  }
#undef NPA_DENS_KB
#undef NPA_DENS
  return after_launch("density_kernel");
}

npa_status launch_perception(const GridParams& g, const PerceptionParams& p, const SortedGrid& s,
                             const HitLists& hl, uint32_t batch, const float* states, int state_dims,
                             const float* volume_sorted, float* features, float* blurred,
                             float* state_gradient, float* density_gradient,
                             cudaStream_t stream) {
  const uint32_t total = batch * s.n;
  if (total == 0) return NPA_OK;
  PerceptionParams pp = p;
  pp.vec_states = (reinterpret_cast<uintptr_t>(states) % 16) == 0;
  if (p.log_norm_grad || p.log_norm_density_grad) NPA_TRY(device_log1p_table(&pp.l1p, stream));
  const int ch = chunk_channels(state_dims);
  const int chunks = state_dims > 0 ? (state_dims + ch - 1) / ch : 1;
  const unsigned blocks = grid_for(uint64_t(total) * chunks, 128);
  // the full growing_2d option set compiled in (2D): cfg1's perception
  const bool full_opts = p.state_grad && p.density_grad && p.hybrid;
#define NPA_PERC(D, CHV, CO)                                                                  \
  do {                                                                                        \
    if (D == 2 && full_opts)                                                                  \
      perception_kernel<D, CHV, CO, (D == 2 ? 2 : 0)><<<blocks, 128, 0, stream>>>(            \
          g, pp, s, hl, total, states, state_dims, chunks, volume_sorted, features, blurred,  \
          state_gradient, density_gradient);                                                  \
    else                                                                                      \
      perception_kernel<D, CHV, CO><<<blocks, 128, 0, stream>>>(                              \
          g, pp, s, hl, total, states, state_dims, chunks, volume_sorted, features, blurred,  \
          state_gradient, density_gradient);                                                  \
  } while (0)
#define NPA_PERC_CH(D, CO)                                   \
  do {                                                       \
    if (ch == 4) NPA_PERC(D, 4, CO); else NPA_PERC(D, 8, CO); \
  } while (0)
  const bool coop = dense_cells(g, batch, total);
  if (g.dim == 2) {
    if (coop) NPA_PERC_CH(2, true); else NPA_PERC_CH(2, false);
  } else {
    if (coop) NPA_PERC_CH(3, true); else NPA_PERC_CH(3, false);
  }
#undef NPA_PERC_CH
#undef NPA_PERC
  return after_launch("perception_kernel");
}

npa_status launch_perception_tiles(const GridParams& g, const PerceptionParams& p,
                                   const SortedGrid& s, const HitLists& hl, uint32_t batch, const float* states,
                                   int state_dims, const float* volume_sorted, int tile_rows,
                                   float* tiles, cudaStream_t stream, uint32_t tile_begin,
                                   uint32_t tile_end) {
  const uint32_t total = batch * s.n;
  if (total == 0) return NPA_OK;
  const uint32_t padded = (total + tile_rows - 1) / tile_rows * tile_rows;
  const uint32_t q_begin =
      static_cast<uint32_t>(std::min<uint64_t>(padded, uint64_t(tile_begin) * tile_rows));
  const uint32_t q_end =
      static_cast<uint32_t>(std::min<uint64_t>(padded, uint64_t(tile_end) * tile_rows));
  if (q_end <= q_begin) return NPA_OK;
  PerceptionParams pp = p;
  pp.vec_states = (reinterpret_cast<uintptr_t>(states) % 16) == 0;
  if (p.log_norm_grad || p.log_norm_density_grad) NPA_TRY(device_log1p_table(&pp.l1p, stream));
  const int ch = chunk_channels(state_dims);
  const int chunks = state_dims > 0 ? (state_dims + ch - 1) / ch : 1;
  const unsigned blocks = grid_for(uint64_t(q_end - q_begin) * chunks, 128);
#define NPA_TILES(D, CHV, CO)                                                                 \
  do {                                                                                        \
    if (fixed_opts)                                                                           \
      perception_tiles_kernel<D, CHV, CO, 1><<<blocks, 128, 0, stream>>>(                     \
          g, pp, s, hl, total, q_begin, q_end, states, state_dims, chunks, volume_sorted,     \
          tile_rows, tiles);                                                                  \
    else                                                                                      \
      perception_tiles_kernel<D, CHV, CO, 0><<<blocks, 128, 0, stream>>>(                     \
          g, pp, s, hl, total, q_begin, q_end, states, state_dims, chunks, volume_sorted,     \
          tile_rows, tiles);                                                                  \
  } while (0)
#define NPA_TILES_CH(D, CO)                                    \
  do {                                                         \
    if (ch == 4) NPA_TILES(D, 4, CO); else NPA_TILES(D, 8, CO); \
  } while (0)
  const bool coop = dense_cells(g, batch, total);
  // the rollout models' options: state gradient, hybrid moment, no density gradient
  const bool fixed_opts = p.state_grad && !p.density_grad && p.hybrid;
  if (g.dim == 2) {
    if (coop) NPA_TILES_CH(2, true); else NPA_TILES_CH(2, false);
  } else {
    if (coop) NPA_TILES_CH(3, true); else NPA_TILES_CH(3, false);
  }
#undef NPA_TILES_CH
#undef NPA_TILES
  return after_launch("perception_tiles_kernel");
}

}  // namespace npa
