// npa_internal.h -- host-side plumbing shared by the library's translation units.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "../../include/npa_b200.h"
#include "npa_device.cuh"

namespace npa {

// Thread-local last-error text (npa_last_error_message).
void set_error(const std::string& msg);
npa_status fail(npa_status st, const std::string& msg);
// Maps a CUDA error to NPA_ERR_CUDA / NPA_ERR_OUT_OF_MEMORY with its text.
npa_status cuda_fail(cudaError_t err, const char* what);
// Counts kernel launches (npa_kernel_launch_count) and checks the launch.
npa_status after_launch(const char* kernel, int launches = 1);

#define NPA_TRY(expr)                    \
  do {                                   \
    npa_status st__ = (expr);            \
    if (st__ != NPA_OK) return st__;     \
  } while (0)

#define NPA_CUDA(expr, what)                          \
  do {                                                \
    cudaError_t e__ = (expr);                         \
    if (e__ != cudaSuccess) return cuda_fail(e__, what); \
  } while (0)

// Validation mirroring HashGridConfig::validate (config.rs:65-84) plus the
// limits of this implementation (cell counts and indices fit in uint32).
npa_status validate_grid(const npa_grid_config* cfg);
GridParams make_grid_params(const npa_grid_config& cfg);

// Bump allocator over a caller workspace; every block is 256-byte aligned.
struct Carve {
  char* base;
  size_t used = 0;
  size_t cap;
  explicit Carve(void* p, size_t bytes) : base(static_cast<char*>(p)), cap(bytes) {}
  template <class T>
  T* take(size_t count) {
    size_t off = (used + 255) & ~size_t(255);
    used = off + count * sizeof(T) + 0;
    return reinterpret_cast<T*>(base ? base + off : nullptr);
  }
  bool fits() const { return used <= cap; }
};

// ---- hashgrid (hashgrid.cu) ----
struct HashgridBuffers {
  uint32_t* bin_offsets;   // [B*cells + 1]
  uint32_t* permutation;   // [B*N]
  uint32_t* inverse;       // [B*N]
  float4* srec;            // [B*N] sorted neighbour records (position + cell)
  int2* scyz;              // [B*N] 3D cell y, z (unused in 2D)
  // [B*N] optional: a processing order for the neighbour walks, a permutation
  // of the sorted slots that groups spatially adjacent particles (written by
  // the device-wide sort only; see hashgrid_orders).
  uint32_t* order = nullptr;
};
// Whether launch_hashgrid writes a processing order for this shape (the
// device-wide sort path: large rollouts, whose hash order scatters the
// neighbour gathers over DRAM); the per-rollout path's data stays in L2.
bool hashgrid_orders(const GridParams& g, uint32_t batch, uint32_t n);
// Blocks of `kernel` resident per SM at `threads` threads and `smem` bytes of
// dynamic shared memory, and the SM count; sets the kernel's dynamic shared
// memory limit first.  Cached per (device, context, kernel, threads, smem).
npa_status kernel_occupancy(const void* kernel, int threads, size_t smem, int* per_sm, int* sms);
// Bytes of scratch the sort needs beyond HashgridBuffers.
size_t hashgrid_scratch_bytes(const GridParams& g, uint32_t batch, uint32_t n);
// Size of the sorted views (srec + scyz).
size_t sorted_view_bytes(uint32_t batch, uint32_t n);
npa_status launch_hashgrid(const GridParams& g, const float4* positions, uint32_t batch,
                           uint32_t n, const HashgridBuffers& out, void* scratch,
                           size_t scratch_bytes, cudaStream_t stream);

// ---- the host libm's log1pf on the device (host_log1p.cu) ----
// Builds (or loads from its cache) the host-side list of inputs where the host
// log1pf differs from the correctly rounded value.
npa_status prepare_host_log1p();
// The current device's lookup tables, uploaded on the first call on that
// device.  That first call allocates and copies, so it fails (instead of
// breaking a capture) when `stream` is capturing.
npa_status device_log1p_table(Log1pTable* out, cudaStream_t stream = nullptr);
// Number of tabulated inputs whose host result differs from the correctly rounded one.
size_t host_log1p_exceptions();
// out[i] = the host libm's log1pf(x[i]) computed on the device.
npa_status launch_ln_1p(const float* x, uint64_t count, float* out, cudaStream_t stream);

// ---- perception (perception.cu) ----
struct PerceptionParams {
  int state_grad, density_grad, scale_eq, pde, log_norm_grad, log_norm_density_grad, hybrid,
      position_features;
  float state_scale;    // normalize_state_gradient scale (normalize.rs:11-15)
  float density_scale;  // normalize_density_gradient scale (normalize.rs:38-46)
  int feature_dims;
  int vec_states;       // state rows may be read as float4 (16-byte aligned, C % 4 == 0)
  Log1pTable l1p;       // the host libm's log1pf on this device (set by the launchers)
};
PerceptionParams make_perception_params(const GridParams& g, const npa_perception_options& o,
                                        uint32_t n, int state_dims);
// density + volume per sorted slot; density_out (original order) optional;
// hit lists recorded when hl.slots is set.
npa_status launch_density(const GridParams& g, const SortedGrid& s, uint32_t batch,
                          float* volume_sorted, float* density_out, const HitLists& hl,
                          cudaStream_t stream);
// Standalone perception writing features / intermediates in original order.
npa_status launch_perception(const GridParams& g, const PerceptionParams& p, const SortedGrid& s,
                             const HitLists& hl, uint32_t batch, const float* states, int state_dims,
                             const float* volume_sorted, float* features, float* blurred,
                             float* state_gradient, float* density_gradient,
                             cudaStream_t stream);
// Step path: feature rows of `tile_rows` sorted slots stored feature-major per
// tile ([tile][F][tile_rows]); rows past B*N are zero.
npa_status launch_perception_tiles(const GridParams& g, const PerceptionParams& p,
                                   const SortedGrid& s, const HitLists& hl, uint32_t batch, const float* states,
                                   int state_dims, const float* volume_sorted, int tile_rows,
                                   float* tiles, cudaStream_t stream, uint32_t tile_begin = 0,
                                   uint32_t tile_end = 0xffffffffu);

// ---- model / step (step.cu) ----
struct DeviceModel {
  int spatial_dims, state_dims, hidden_dims, feature_dims, update_dims;
  float eps0, alpha;
  int equivariance;
  int density_grad, state_grad, log_norm_grad, log_norm_density_grad, position_features;
  int device;
  int hidden_padded;  // H rounded up to 64, 128 or 256 (the MLP's thread grid)
  float* w1t;  // [F][hidden_padded], w1 transposed and zero-padded
  float* b1;   // [H]
  float* w2;   // [O][H]
  float* b2;   // [O]
};
npa_status launch_forward_update(const DeviceModel& m, const float* features, uint32_t rows,
                                 float* update, cudaStream_t stream);
npa_status launch_euler(const GridParams& g, const float4* positions, const float* states,
                        const float4* dx, const float* ds, uint32_t total, int state_dims,
                        float dt, const float* mask, float4* next_positions, float* next_states,
                        cudaStream_t stream);
struct StepOutputs {
  float4* next_positions;
  float* next_states;
  float4* dx;        // optional
  float* ds;         // optional
  float* features;   // optional
};
int hidden_padded_for(int hidden);
// Rows per feature tile of the MLP stage for a step over `rows` particles
// (depends on the padded hidden width, the feature width and the row count).
int step_tile_rows(const DeviceModel& m, uint64_t rows);
bool mlp_step_supported(const DeviceModel& m);
// The GPU executor's stochastic update mask (inactive when lane_seeds is null).
struct StochasticMask {
  float update_prob = 1.0f;
  const uint32_t* lane_seeds = nullptr;    // [B] device
  const uint32_t* step_counter = nullptr;  // device step index
};
// Feature-tile bulk copies that timed out in the MLP step kernel (device counter).
uint64_t bulk_copy_timeouts();
// step_counter[0] += 1 (after a step that used the stochastic mask).
npa_status launch_advance_step(uint32_t* counter, cudaStream_t stream);
// out[0] = mean over i < total of |dx[i].xyz| (run_rollout's mean_dx entry);
// partials: mean_norm_scratch_bytes() of device scratch.
npa_status launch_mean_norm(const float4* dx, uint32_t total, double* partials, float* out,
                            cudaStream_t stream);
size_t mean_norm_scratch_bytes();
// MLP + dx/ds (+3D gates) + Euler over feature tiles in sorted order.
// Tiles [tile_begin, tile_end) of the step (default: all).
npa_status launch_mlp_step(const DeviceModel& m, const GridParams& g, const SortedGrid& s,
                           uint32_t batch, const float* tiles, const float* states, float dt,
                           const float* mask, const StochasticMask& sm,
                           const StepOutputs& out, cudaStream_t stream, uint32_t tile_begin = 0,
                           uint32_t tile_end = 0xffffffffu);

// The fused step (perception + MLP + Euler in one kernel, after the density
// pass): supported for 2D models with more than 4 channels, hidden width up
// to 128 and sparse cells; the same results as perception tiles + MLP step.
bool fused_step_supported(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                          uint32_t batch, uint32_t total);
npa_status launch_fused_step(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                             const SortedGrid& s, const HitLists& hl, uint32_t batch,
                             const float* states, const float* volume_sorted, float dt,
                             const float* mask, const StochasticMask& sm, const StepOutputs& out,
                             cudaStream_t stream);

// The warp-specialised step (perception producer warps and MLP consumer warps
// in one 512-thread block per SM, feature tiles handed over in shared
// memory): 2D models with at most 16 channels, hidden width 128, sparse
// cells; the same results as the split kernels.
bool ws_step_supported(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                       uint32_t batch, uint32_t total);
npa_status launch_ws_step(const DeviceModel& m, const GridParams& g, const PerceptionParams& p,
                          const SortedGrid& s, const HitLists& hl, uint32_t batch,
                          const float* states, const float* volume_sorted, float dt,
                          const float* mask, const StochasticMask& sm, const StepOutputs& out,
                          cudaStream_t stream);
// Bounded waits of the warp-specialised step that gave up (device counter).
uint64_t ws_step_timeouts();

// ---- training rollout backward (train.cu) ----
// out[r][O] = adjoint of row r's raw update (target2d.rs:3566-3604): the masked
// position adjoint through raw_motion_adjoint, the displacement regularizer
// (reg = weight / rows; 0 = off) and the masked state adjoint.
npa_status launch_output_adjoint(const float* update, const float4* pos_adj, const float* state_adj,
                                 const float* mask, uint32_t rows, int dims, int C, float scale,
                                 float reg, float* out, cudaStream_t stream);
// mlp_backward_from_output_gradients (training.rs:558-640) over `rows` rows:
// the input adjoint into gfeat and the weight / bias gradients ADDED to
// gw1 [H][F], gb1, gw2 [O][H], gb2; hidden / dpre are [rows][H] scratch.
npa_status launch_mlp_backward(const DeviceModel& m, const float* features, const float* out_adj,
                               uint32_t rows, float* hidden, float* dpre, float* gfeat,
                               float* gw1, float* gb1, float* gw2, float* gb2,
                               cudaStream_t stream);
npa_status launch_add_adjoint(float4* pos_adj, float* state_adj, const float4* dpos,
                              const float* dstate, uint32_t rows, int dims, int C, bool add_pos,
                              bool add_state, cudaStream_t stream);
// *flag |= code when any of the count values is not finite.
npa_status launch_finite_check(const float* v, uint64_t count, int* flag, int code,
                               cudaStream_t stream);

// ---- perception adjoint (adjoint.cu) ----
// Scratch floats launch_perception_adjoint needs beyond its outputs.
size_t adjoint_scratch_floats(uint32_t total, int state_dims, int dim);
// perceive_adjoint_with_options over a built hashgrid (sorted view s, local
// inverse permutation) and the caller-order density; zeroes and fills the
// state / position / density adjoints.
npa_status launch_perception_adjoint(const GridParams& g, const PerceptionParams& p,
                                     const SortedGrid& s, const uint32_t* inverse,
                                     uint32_t batch, const float* states, int state_dims,
                                     const float* density, const float* feature_adjoint,
                                     float* scratch, float* state_adjoint, float4* position_adjoint,
                                     float* density_adjoint, cudaStream_t stream);

// ---- splat (splat.cu) ----
size_t splat_workspace_bytes(uint32_t count);
npa_status launch_splat_2d(const npa_splat2d_config& cfg, const float4* positions,
                           const float* colors, uint32_t count, float4* out, void* workspace,
                           cudaStream_t stream);

// ---- the CPU rollout's StdRng update masks (stdrng.cu) ----
struct ChachaKey {
  uint32_t k[8];
};
// StdRng::seed_from_u64(rng_seed) as ChaCha12 key words.
ChachaKey stdrng_key(uint64_t rng_seed);
// mask[i] = (stream word word0 + i, as random::<f32>()) < update_prob, i < count.
npa_status launch_stdrng_mask(const ChachaKey& key, uint64_t word0, uint32_t count,
                              float update_prob, float* mask, cudaStream_t stream);

// ---- decode (decode.cu) ----
npa_status launch_decode(const npa_gaussian_decode_config& cfg, const float4* positions,
                         const float* states, uint32_t count, int state_dims, float* out,
                         cudaStream_t stream);

inline unsigned grid_for(uint64_t items, unsigned block) {
  uint64_t g = (items + block - 1) / block;
  return static_cast<unsigned>(g > 0 ? g : 1);
}

}  // namespace npa
