/*
 * npa_b200.h -- C ABI of the B200 (sm_100a) implementation of the
 * burn_automata Neural Particle Automata rollout path.
 *
 * The entry points replace the CPU operators of crates/burn_automata_kernels
 * and the step / rollout of crates/burn_automata (mosure/burn_automata); each
 * declaration cites the Rust item it stands in for.  A Rust host binds them
 * with `extern "C"` declarations of the same signatures.
 *
 * Conventions
 *  - Plain pointers and sizes; no framework types.  Lengths are element
 *    counts (positions are counted in [f32; 4] records, like the Rust slices).
 *  - The caller owns every output buffer.  An output whose length does not
 *    match returns NPA_ERR_OUTPUT_SHAPE instead of being reallocated (the Rust
 *    API returns a fresh Vec; KernelError::OutputShape, config.rs:133).
 *  - Index outputs are uint32 (the Rust API uses usize; a binding widens).
 *  - Host-buffer entry points (npa_*) copy in, compute on the current CUDA
 *    device (or the model's device) and copy out before returning.
 *  - Device entry points (npa_dev_*) take device pointers, enqueue on the
 *    given cudaStream_t (passed as void*) and return without synchronising;
 *    they allocate nothing: scratch comes from the caller's workspace, sized by
 *    the matching *_workspace_size query.
 *  - Arithmetic follows the reference's f32 operation order: no FMA
 *    contraction, sequential sums in the reference's loop order, IEEE division
 *    and square root.  f32::ln_1p is the host C library's log1pf, bit for bit
 *    (see npa_prepare_host_tables).
 *  - Every call returns an npa_status; nothing aborts the process.
 */
#ifndef NPA_B200_H
#define NPA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NPA_ABI_VERSION 1

/* Status codes.  1..8 mirror KernelError (crates/burn_automata_kernels/src/
 * config.rs:101-137); 9 mirrors AutomataError::InvalidModel
 * (crates/burn_automata/src/error.rs). */
typedef int32_t npa_status;
enum {
  NPA_OK = 0,
  NPA_ERR_INVALID_DIM = 1,                   /* KernelError::InvalidDim */
  NPA_ERR_INVALID_EPS = 2,                   /* KernelError::InvalidEps */
  NPA_ERR_INVALID_GRID_SIZE = 3,             /* KernelError::InvalidGridSize */
  NPA_ERR_PARTICLE_MODE_REQUIRES_POW2 = 4,   /* KernelError::ParticleModeRequiresPowerOfTwo */
  NPA_ERR_POSITION_SHAPE = 5,                /* KernelError::PositionShape */
  NPA_ERR_STATE_SHAPE = 6,                   /* KernelError::StateShape */
  NPA_ERR_OUTPUT_SHAPE = 7,                  /* KernelError::OutputShape */
  NPA_ERR_INVALID_ARGUMENT = 8,              /* KernelError / AutomataError::InvalidArgument */
  NPA_ERR_INVALID_MODEL = 9,                 /* AutomataError::InvalidModel */
  NPA_ERR_CUDA = 20,                         /* a CUDA runtime call failed */
  NPA_ERR_DEVICE_STATUS = 21,                /* reserved: no entry point returns it */
  NPA_ERR_TIMEOUT = 22,                      /* a bounded device-side wait gave up */
  NPA_ERR_OUT_OF_MEMORY = 23,                /* an allocation failed (or hit the cap) */
  NPA_ERR_UNSUPPORTED = 24,                  /* shape outside what the kernels support */
  NPA_ERR_NO_DEVICE = 25                     /* no CUDA device is usable */
};

/* Boundary (config.rs:6-10) and HashGridMode (config.rs:14-18). */
enum { NPA_BOUNDARY_PERIODIC = 0, NPA_BOUNDARY_CLAMPED = 1 };
enum { NPA_MODE_GRID = 0, NPA_MODE_PARTICLE = 1 };

/* HashGridConfig (crates/burn_automata_kernels/src/config.rs:20-29). */
typedef struct npa_grid_config {
  int32_t dim;                     /* 2 or 3 */
  int32_t boundary;                /* NPA_BOUNDARY_* */
  int32_t mode;                    /* NPA_MODE_* */
  int32_t max_particles_per_block; /* carried for parity; unused by the step */
  int64_t grid_size[3];
  float eps;
  int32_t reserved;
} npa_grid_config;

/* PerceptionOptions (crates/burn_automata_kernels/src/reference/types.rs:4-15). */
typedef struct npa_perception_options {
  uint8_t state_grad;
  uint8_t density_grad;
  uint8_t scale_equivariance;
  uint8_t particle_density_equivariance;
  uint8_t log_norm_grad;
  uint8_t log_norm_density_grad;
  uint8_t hybrid_state_gradient;
  uint8_t position_features;
  float eps0;
  int32_t reserved;
} npa_perception_options;

/* EquivarianceMode (crates/burn_automata/src/config.rs:22-28). */
enum { NPA_EQUIV_NONE = 0, NPA_EQUIV_PARTICLE_DENSITY = 1, NPA_EQUIV_PARTICLE_DENSITY_AND_SCALE = 2 };

/* NpaConfig fields read by NpaModel::step_cpu (crates/burn_automata/src/config.rs:30-53). */
typedef struct npa_model_config {
  int32_t spatial_dims;
  int32_t state_dims;
  int32_t hidden_dims;
  int32_t auxiliary_input_dims;    /* must be 0: step_cpu has no auxiliary inputs */
  float eps0;
  float alpha;
  int32_t equivariance;            /* NPA_EQUIV_* */
  uint8_t density_grad;
  uint8_t state_grad;
  uint8_t log_norm_grad;
  uint8_t log_norm_density_grad;
  uint8_t position_features;
  uint8_t reserved[7];
} npa_model_config;

/* GaussianDecodeMode (crates/burn_automata_kernels/src/gaussian.rs:13-21). */
enum {
  NPA_DECODE_PARTICLE_POINT = 0,
  NPA_DECODE_SH0_FIXED_SCALE = 1,
  NPA_DECODE_SH0_LEARNED_SCALE = 2,
  NPA_DECODE_SH0_ORIENTED = 3
};

/* GaussianDecodeConfig (crates/burn_automata_kernels/src/gaussian.rs:23-35). */
typedef struct npa_gaussian_decode_config {
  int32_t mode;
  int32_t sh_degree;
  float sigma;
  float min_scale;
  float max_scale;
  float max_anisotropy;
  float opacity_scale;
  float min_opacity;
  float max_opacity;
  int32_t reserved;
} npa_gaussian_decode_config;

/* Splat2dConfig (crates/burn_automata_kernels/src/splat.rs:4-28). */
typedef struct npa_splat2d_config {
  int64_t image_size;
  float sigma;
  float lo;
  float hi;
  int32_t normalize_color;
  int32_t y_up;
  float pixel_size;
  int32_t reserved;
} npa_splat2d_config;

/* ------------------------------------------------------------------ */
/* Library                                                             */
/* ------------------------------------------------------------------ */

int32_t npa_abi_version(void);
const char* npa_status_string(npa_status status);
/* Text of the last error on the calling thread (CUDA message, failing shape). */
const char* npa_last_error_message(void);
/* Number of kernels this library has launched in this process (all devices). */
uint64_t npa_kernel_launch_count(void);

/* Diagnostic: feature-tile bulk copies of the MLP step kernel, and feature-tile
 * hand-overs of the warp-specialised step, that did not complete within their
 * bounded wait on the current device (0 in a healthy run; a block that gives
 * up leaves its remaining tiles undone).  The
 * synchronising host calls (npa_model_step, npa_model_run_rollout*,
 * npa_executor_read_state) return NPA_ERR_TIMEOUT when this device's count
 * has grown since the last such check on the device. */
uint64_t npa_bulk_copy_timeouts(void);

/* The payload of the last error on the calling thread, as the reference's
 * KernelError variants carry it (crates/burn_automata_kernels/src/config.rs:
 * 102-137): InvalidDim(dim) -> a = dim; InvalidEps(eps) -> eps;
 * ParticleModeRequiresPowerOfTwo { axis, value } -> a = axis, b = value;
 * PositionShape { positions, expected }, StateShape { states, expected } and
 * OutputShape { actual, expected } -> a = the given length, b = expected;
 * InvalidArgument(String) / AutomataError::InvalidModel(String) -> the text of
 * npa_last_error_message.  status is the code that error returned (NPA_OK
 * before any error); fields a variant does not carry are 0. */
typedef struct npa_error_detail {
  npa_status status;
  float eps;
  int64_t a;
  int64_t b;
} npa_error_detail;
npa_status npa_last_error_detail(npa_error_detail* out);

/* The host C library's log1pf (the reference's f32::ln_1p, which its
 * log-normalisation calls: crates/burn_automata_kernels/src/reference/
 * normalize.rs:60-69) is reproduced bit for bit on the device: ln(1 + x) in
 * f64, rounded once, corrected where the host's log1pf returns the
 * neighbouring float.  Those inputs are found by calling the host's log1pf on
 * every float in [1e-6, inf); the list is cached next to the library file
 * (libnpa_b200.so.log1pf, checked against the running host when read) and
 * turned on each device, on first use, into a 2-bit correction code per input
 * relative to CUDA's log1pf (256 MiB, held until exit).
 *
 * npa_prepare_host_tables builds or loads that list (about 17 CPU-seconds
 * when no valid cache exists) and reports its length.  npa_prepare_device
 * uploads it to `device`; npa_model_create / npa_executor_create do so for
 * models that log-normalise, and the perception entry points on first use.
 * The upload allocates, so a first use inside a stream capture returns
 * NPA_ERR_INVALID_ARGUMENT: call npa_prepare_device before capturing. */
npa_status npa_prepare_host_tables(int64_t* ln_1p_exceptions);
npa_status npa_prepare_device(int32_t device);
/* f32::ln_1p as above on device buffers: d_out[i] = log1pf(d_x[i]) of the host
 * C library, bit for bit for x >= 1e-6 (below, CUDA's log1pf). */
npa_status npa_dev_ln_1p(const float* d_x, int64_t count, float* d_out, void* stream);

/* HashGridConfig::validate (config.rs:65-84). */
npa_status npa_grid_validate(const npa_grid_config* cfg);
/* HashGridConfig::cell_count (config.rs:86-88). */
npa_status npa_grid_cell_count(const npa_grid_config* cfg, int64_t* cell_count);
/* Feature row width, forward.rs:100-103. */
npa_status npa_feature_dims(const npa_grid_config* cfg, const npa_perception_options* options,
                            int64_t state_dims, int64_t* feature_dims);
/* Floats per decoded Gaussian record: [position_visibility 4][rotation 4]
 * [scale_opacity 4][spherical_harmonic 3*k], k = (sh_degree+1)^2 for
 * GaussianSh0Oriented, else 1. */
npa_status npa_gaussian_record_floats(const npa_gaussian_decode_config* cfg, int64_t* floats);

/* ------------------------------------------------------------------ */
/* Host-buffer operators (drop-in for crates/burn_automata_kernels)    */
/* ------------------------------------------------------------------ */

/* build_hashgrid (crates/burn_automata_kernels/src/hashgrid.rs:16-69).
 * positions: positions_len records of [f32; 4]; must equal batch*n.
 * bin_offsets: batch*cell_count+1; permutation / inverse_permutation: batch*n
 * local indices.  Bit-exact with the reference, including the stable
 * ascending order of particles inside a cell. */
npa_status npa_build_hashgrid(const npa_grid_config* cfg, const float* positions,
                              int64_t positions_len, int64_t batch, int64_t n,
                              uint32_t* bin_offsets, int64_t bin_offsets_len,
                              uint32_t* permutation, uint32_t* inverse_permutation,
                              int64_t permutation_len);

/* perceive_with_options (crates/burn_automata_kernels/src/reference/forward.rs:26-143).
 * features: batch*n*feature_dims (required).  density (batch*n), blurred_state
 * (batch*n*c), state_gradient (batch*n*c*dim, only if state_grad) and
 * density_gradient (batch*n*dim, only if density_grad) may be NULL. */
npa_status npa_perceive_with_options(const npa_grid_config* cfg,
                                     const npa_perception_options* options,
                                     const float* positions, int64_t positions_len,
                                     const float* states, int64_t states_len, int64_t batch,
                                     int64_t n, int64_t state_dims, float* features,
                                     int64_t features_len, float* density, float* blurred_state,
                                     float* state_gradient, float* density_gradient);

/* euler_step (crates/burn_automata_kernels/src/reference/step.rs:4-55).
 * dx: [f32; 4] records; update_mask may be NULL (all ones). */
npa_status npa_euler_step(const npa_grid_config* cfg, const float* positions,
                          int64_t positions_len, const float* states, int64_t states_len,
                          const float* dx, int64_t dx_len, const float* ds, int64_t ds_len,
                          int64_t batch, int64_t n, int64_t state_dims, float dt,
                          const float* update_mask, float* next_positions, float* next_states);

/* decode_gaussians_3d (crates/burn_automata_kernels/src/gaussian.rs:53-100).
 * out: count * npa_gaussian_record_floats floats.  A state layout too small for
 * the mode returns NPA_ERR_STATE_SHAPE (the reference panics, gaussian.rs:102-125). */
npa_status npa_decode_gaussians_3d(const npa_gaussian_decode_config* cfg, const float* positions,
                                   int64_t positions_len, const float* states,
                                   int64_t states_len, int64_t state_dims, float* out,
                                   int64_t out_len);

/* ------------------------------------------------------------------ */
/* Model: NpaModel (crates/burn_automata/src/model.rs)                 */
/* ------------------------------------------------------------------ */

typedef struct npa_model npa_model;

/* NpaModel { config, weights } with weights resident on `device`.
 * w1 [hidden, perception_dims] row-major, b1 [hidden], w2 [update_dims, hidden],
 * b2 [update_dims] (NpaWeights, model.rs:11-17; checked like
 * NpaWeights::validate, model.rs:77-107). */
npa_status npa_model_create(const npa_model_config* cfg, const float* w1, int64_t w1_len,
                            const float* b1, int64_t b1_len, const float* w2, int64_t w2_len,
                            const float* b2, int64_t b2_len, int32_t device, npa_model** out);
void npa_model_destroy(npa_model* model);

/* NpaModel::forward_update_from_features (model.rs:900-940); update: rows*update_dims. */
npa_status npa_model_forward_update_from_features(npa_model* model, const float* features,
                                                  int64_t features_len, float* update,
                                                  int64_t update_len);

/* NpaModel::step_cpu (model.rs:768-858).  update_mask, dx ([f32;4] records),
 * ds, features and density may be NULL. */
npa_status npa_model_step(npa_model* model, const npa_grid_config* grid, const float* positions,
                          int64_t positions_len, const float* states, int64_t states_len,
                          int64_t batch, int64_t n, float dt, const float* update_mask,
                          float* next_positions, float* next_states, float* dx, float* ds,
                          float* features, float* density);

/* run_rollout_from_particles (crates/burn_automata/src/rollout/mod.rs:201-283)
 * with update_prob >= 1: `steps` steps, positions / states updated in place. */
npa_status npa_model_run_rollout(npa_model* model, const npa_grid_config* grid, float* positions,
                                 int64_t positions_len, float* states, int64_t states_len,
                                 int64_t batch, int64_t n, int64_t steps, float dt);

/* run_rollout_from_particles with the RolloutTrace's mean_dx
 * (rollout/mod.rs:264-296): as npa_model_run_rollout, plus mean_dx[k] = the
 * mean over particles of |dx| in step k (steps entries).  The per-particle
 * norms follow the reference's f32 arithmetic; their sum is taken in f64
 * (the reference adds them sequentially in f32), so mean_dx agrees to the
 * reference's own summation error. */
npa_status npa_model_run_rollout_trace(npa_model* model, const npa_grid_config* grid,
                                       float* positions, int64_t positions_len, float* states,
                                       int64_t states_len, int64_t batch, int64_t n,
                                       int64_t steps, float dt, float* mean_dx);

/* run_rollout_from_particles (crates/burn_automata/src/rollout/mod.rs:222-238)
 * for any update_prob: the reference seeds StdRng::seed_from_u64(seed ^ 0x5eed)
 * and multiplies every step's update by stochastic_mask (:644-651),
 * random::<f32>() < update_prob per particle in index order (no mask when
 * update_prob >= 1).  StdRng is rand 0.9.4's ChaCha12Rng; the masks are that
 * stream (restated: rand_core 0.9 seed_from_u64, ChaCha12, rand's 24-bit f32),
 * computed on the GPU.  mean_dx (steps entries) may be null. */
npa_status npa_model_run_rollout_seeded(npa_model* model, const npa_grid_config* grid,
                                        float* positions, int64_t positions_len, float* states,
                                        int64_t states_len, int64_t batch, int64_t n,
                                        int64_t steps, float dt, float update_prob,
                                        uint64_t seed, float* mean_dx);

/* The masks npa_model_run_rollout_seeded (run_rollout_from_particles with
 * cfg.seed = seed) applies in steps [first_step, first_step + steps), 0-based:
 * masks[k * count + i] for step first_step + k, particle i < count. */
npa_status npa_rollout_update_masks(uint64_t seed, float update_prob, int64_t count,
                                    int64_t first_step, int64_t steps, float* masks);

/* ---- training rollout (f32 backprop through time) ---- */

/* mlp_backward_from_output_gradients (crates/burn_automata/src/training.rs:558-640):
 * rows = features_len / perception_dims; output_gradients [rows][update_dims].
 * Writes the weight gradients gw1 [hidden][perception_dims], gb1 [hidden],
 * gw2 [update_dims][hidden], gb2 [update_dims] and the feature gradients
 * gfeatures [rows][perception_dims].  Every sum is taken in the reference's
 * order (weight gradients over rows in row order), so the results are its
 * own bit for bit.  Non-finite inputs or results return
 * NPA_ERR_INVALID_ARGUMENT naming the buffer (ensure_finite, :1053-1060). */
npa_status npa_model_mlp_backward(npa_model* model, const float* features, int64_t features_len,
                                  const float* output_gradients, int64_t output_gradients_len,
                                  float* gw1, float* gb1, float* gw2, float* gb2,
                                  float* gfeatures);

/* rollout_for_training (crates/burn_automata/src/target2d.rs:3414-3466):
 * `steps` Euler steps with dt = 1 under stochastic_mask draws of
 * StdRng::seed_from_u64(seed ^ 0x5eed2d) (ones when update_prob >= 1).
 * Step k's input is recorded: snapshot_positions [steps][B*N][4],
 * snapshot_states [steps][B*N*C], snapshot_masks [steps][B*N].  The final
 * particles go to final_positions / final_states and *mean_dx_norm_sum is
 * the f32 running sum over steps of mean_dx_norm.  3D models with position
 * features and C > 3 return NPA_ERR_UNSUPPORTED (the training rollout
 * applies no position gates, the device step does). */
npa_status npa_model_rollout_for_training(npa_model* model, const npa_grid_config* grid,
                                          const float* positions, int64_t positions_len,
                                          const float* states, int64_t states_len, int64_t batch,
                                          int64_t n, int64_t steps, float update_prob,
                                          uint64_t seed, float* snapshot_positions,
                                          float* snapshot_states, float* snapshot_masks,
                                          float* final_positions, float* final_states,
                                          float* mean_dx_norm_sum);

/* bptt_gradients (crates/burn_automata/src/target2d.rs:3550-3722) over the
 * snapshots npa_model_rollout_for_training recorded: starting from the loss
 * adjoints position_gradients [B*N][4] and state_gradients [B*N*C], each
 * step in reverse recomputes the perception and raw update, forms the
 * output adjoint (raw_motion_adjoint, the displacement regularizer with
 * weight / rows, the masked state adjoint), back-propagates the MLP (sums
 * into gw1..gb2) and adds the perception adjoint to the running adjoints
 * unless stopgrad_pos / stopgrad_state.  The Euler step's Jacobian is the
 * identity, as the reference's.  The MLP terms are bit for bit the
 * reference's; the perception adjoint scatters with atomics
 * (npa_perceive_adjoint_with_options), so across steps the results agree to
 * f32 summation error.  initial_position_adjoint [B*N][4] and
 * initial_state_adjoint [B*N*C] (the adjoints at the rollout's input) may
 * be NULL. */
npa_status npa_model_bptt_gradients(npa_model* model, const npa_grid_config* grid,
                                    const float* snapshot_positions, const float* snapshot_states,
                                    const float* snapshot_masks, int64_t batch, int64_t n,
                                    int64_t steps, const float* position_gradients,
                                    const float* state_gradients,
                                    float displacement_regularizer_weight, int32_t stopgrad_pos,
                                    int32_t stopgrad_state, float* gw1, float* gb1, float* gw2,
                                    float* gb2, float* initial_position_adjoint,
                                    float* initial_state_adjoint);

/* perceive_adjoint_with_options
 * (crates/burn_automata_kernels/src/reference/adjoint.rs:28-136): given the
 * adjoint of the perception features [B*N][F] (F as perceive_with_options),
 * writes the state adjoint [B*N*C] and, when position_adjoint is not null,
 * the position adjoint [B*N][4] (w stays 0).  Each term is the reference's;
 * the terms of one entry are added in a different order (one thread per
 * particle scattering with atomics), so results agree to f32 summation error.
 * perceive_state_adjoint_with_options (:4-26) is this call with a null
 * position_adjoint.  A wrong feature_adjoint_len returns NPA_ERR_OUTPUT_SHAPE
 * (KernelError::OutputShape, as the reference). */
npa_status npa_perceive_adjoint_with_options(const npa_grid_config* cfg,
                                             const npa_perception_options* options,
                                             const float* positions, int64_t positions_len,
                                             const float* states, int64_t states_len,
                                             int64_t batch, int64_t n, int64_t state_dims,
                                             const float* feature_adjoint,
                                             int64_t feature_adjoint_len, float* state_adjoint,
                                             float* position_adjoint);

/* splat_particles_2d (crates/burn_automata_kernels/src/splat.rs:30-93):
 * positions [count][4], colors [count][3] -> out [image_size^2][4] (RGB and
 * the weight), row-major from the top row when y_up.  Each pixel's sums are
 * taken in particle order, as the reference's loop; exp is computed in f64
 * and rounded, so pixels agree with the host libm's expf to its own error.
 * The reference asserts positions.len() == colors.len(); here the two share
 * `count`, so a mismatch cannot be expressed.  out_len must be
 * 4 * image_size^2 (NPA_ERR_OUTPUT_SHAPE otherwise). */
npa_status npa_splat_particles_2d(const npa_splat2d_config* cfg, const float* positions,
                                  const float* colors, int64_t count, float* out,
                                  int64_t out_len);

/* ------------------------------------------------------------------ */
/* Device operators (caller-owned device buffers, async on a stream)   */
/* ------------------------------------------------------------------ */

/* Workspace bytes needed by npa_dev_build_hashgrid. */
npa_status npa_dev_hashgrid_workspace_size(const npa_grid_config* cfg, int64_t batch, int64_t n,
                                           size_t* bytes);
/* build_hashgrid on device buffers (hashgrid.rs:16-69). */
npa_status npa_dev_build_hashgrid(const npa_grid_config* cfg, const float* d_positions,
                                  int64_t batch, int64_t n, uint32_t* d_bin_offsets,
                                  uint32_t* d_permutation, uint32_t* d_inverse_permutation,
                                  void* d_workspace, size_t workspace_bytes, void* stream);

/* build_hashgrid on device buffers without allocating anything and without a
 * workspace.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory (they only hold buffers owned by another
 * framework, or must not call cudaMalloc because it synchronises the device).
 * The sort scratch is a fixed device array inside this library (6.5 MiB per
 * device that loads it, held until process exit), so batch * n is limited to
 * 131,072 particles; larger sizes return NPA_ERR_UNSUPPORTED.  The first call
 * on each device looks up the array's device address (make it before any
 * stream capture on that device).  All calls on a device share the one array:
 * calls whose GPU work overlaps (different streams, or different host threads)
 * race on it and must be serialised by the caller.  Results are identical to
 * npa_dev_build_hashgrid. */
npa_status npa_dev_build_hashgrid_noalloc(const npa_grid_config* cfg, const float* d_positions,
                                          int64_t batch, int64_t n, uint32_t* d_bin_offsets,
                                          uint32_t* d_permutation,
                                          uint32_t* d_inverse_permutation, void* stream);

/* Workspace bytes of npa_dev_perceive_adjoint_with_options. */
npa_status npa_dev_perceive_adjoint_workspace_size(const npa_grid_config* cfg, int64_t batch,
                                                   int64_t n, int64_t state_dims,
                                                   size_t* bytes);
/* perceive_adjoint_with_options on device buffers (see the host variant). */
npa_status npa_dev_perceive_adjoint_with_options(
    const npa_grid_config* cfg, const npa_perception_options* options, const float* d_positions,
    const float* d_states, int64_t batch, int64_t n, int64_t state_dims,
    const float* d_feature_adjoint, float* d_state_adjoint, float* d_position_adjoint,
    void* d_workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes of npa_dev_splat_particles_2d for `count` particles. */
npa_status npa_dev_splat_workspace_size(int64_t count, size_t* bytes);
/* splat_particles_2d on device buffers (see npa_splat_particles_2d). */
npa_status npa_dev_splat_particles_2d(const npa_splat2d_config* cfg, const float* d_positions,
                                      const float* d_colors, int64_t count, float* d_out,
                                      void* d_workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes needed by npa_dev_perceive_with_options. */
npa_status npa_dev_perceive_workspace_size(const npa_grid_config* cfg, int64_t batch, int64_t n,
                                           int64_t state_dims, size_t* bytes);
/* perceive_with_options on device buffers (forward.rs:26-143).  Same optional
 * outputs as the host variant. */
npa_status npa_dev_perceive_with_options(const npa_grid_config* cfg,
                                         const npa_perception_options* options,
                                         const float* d_positions, const float* d_states,
                                         int64_t batch, int64_t n, int64_t state_dims,
                                         float* d_features, float* d_density,
                                         float* d_blurred_state, float* d_state_gradient,
                                         float* d_density_gradient, void* d_workspace,
                                         size_t workspace_bytes, void* stream);

/* Benchmark aid, no reference counterpart: `repeats` back-to-back
 * npa_dev_perceive_with_options calls (features and density written) with
 * CUDA events recorded on `stream` between their phases.  phase_ms receives
 * repeats*3 durations (hashgrid build, density, perception) and total_ms the
 * span from the first launch to the last.  Synchronises `stream`. */
npa_status npa_dev_perceive_many_profiled(const npa_grid_config* cfg,
                                          const npa_perception_options* options,
                                          const float* d_positions, const float* d_states,
                                          int64_t batch, int64_t n, int64_t state_dims,
                                          float* d_features, float* d_density,
                                          void* d_workspace, size_t workspace_bytes,
                                          int64_t repeats, void* stream, float* phase_ms,
                                          float* total_ms);

/* forward_update_from_features on device buffers (model.rs:900-940). */
npa_status npa_dev_model_forward_update(npa_model* model, const float* d_features, int64_t rows,
                                        float* d_update, void* stream);

/* euler_step on device buffers (step.rs:4-55). */
npa_status npa_dev_euler_step(const npa_grid_config* cfg, const float* d_positions,
                              const float* d_states, const float* d_dx, const float* d_ds,
                              int64_t batch, int64_t n, int64_t state_dims, float dt,
                              const float* d_update_mask, float* d_next_positions,
                              float* d_next_states, void* stream);

/* decode_gaussians_3d on device buffers (gaussian.rs:53-100). */
npa_status npa_dev_decode_gaussians_3d(const npa_gaussian_decode_config* cfg,
                                       const float* d_positions, const float* d_states,
                                       int64_t count, int64_t state_dims, float* d_out,
                                       void* stream);

/* Workspace bytes needed by npa_dev_model_step. */
npa_status npa_dev_step_workspace_size(npa_model* model, const npa_grid_config* grid,
                                       int64_t batch, int64_t n, size_t* bytes);
/* NpaModel::step_cpu on device buffers (model.rs:768-858): hashgrid, density,
 * perception into feature tiles, then one kernel for MLP + dx/ds + Euler.
 * Optional outputs (d_update_mask, d_dx, d_ds, d_features, d_density) may be
 * NULL.  d_workspace must be 16-byte aligned (cudaMalloc memory is): the MLP
 * kernel bulk-copies feature tiles out of it (NPA_ERR_INVALID_ARGUMENT
 * otherwise). */
npa_status npa_dev_model_step(npa_model* model, const npa_grid_config* grid,
                              const float* d_positions, const float* d_states, int64_t batch,
                              int64_t n, float dt, const float* d_update_mask,
                              float* d_next_positions, float* d_next_states, float* d_dx,
                              float* d_ds, float* d_features, float* d_density,
                              void* d_workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ */
/* Executor: resident rollout state (the CUDA counterpart of            */
/* WgpuAutomataExecutor, crates/burn_automata/src/gpu/executor/*)      */
/* ------------------------------------------------------------------ */

typedef struct npa_executor npa_executor;

/* create_state (executor/state.rs:6-82): device buffers for batch*n particles
 * of the model's state width, on the model's device. */
npa_status npa_executor_create(npa_model* model, const npa_grid_config* grid, int64_t batch,
                               int64_t n, npa_executor** out);
void npa_executor_destroy(npa_executor* exec);
/* Upload host state (blocking). */
npa_status npa_executor_upload_state(npa_executor* exec, const float* positions,
                                     const float* states);
/* Copy state from device buffers of the same shape (async on stream). */
npa_status npa_executor_set_state_device(npa_executor* exec, const float* d_positions,
                                         const float* d_states, void* stream);
/* step_state_many (executor/steps.rs:25): `steps` rollout steps on `stream`.
 * With use_graph != 0 the step sequence is captured once into a CUDA graph
 * and replayed. */
npa_status npa_executor_step_many(npa_executor* exec, int64_t steps, float dt, int32_t use_graph,
                                  void* stream);
/* step_state_many with CUDA events recorded on `stream` around each phase of
 * each step: phase_ms receives steps*4 durations (hashgrid, density,
 * perception, MLP+Euler) and total_ms the whole span.  Synchronises `stream`. */
npa_status npa_executor_step_many_profiled(npa_executor* exec, int64_t steps, float dt,
                                           int32_t use_graph, void* stream, float* phase_ms,
                                           float* total_ms);
/* Stochastic update mask of the resident executor
 * (create_state_with_update_prob, crates/burn_automata/src/gpu/executor/state.rs:29-55,
 * the mask itself crates/burn_automata/src/gpu_step.wgsl:1019-1056).  With
 * update_prob < 1 every later step updates particle i of lane l only when
 * random01(i, step_index, lane_seed[l]) < update_prob (a counter hash of the
 * particle, the step index and the lane seed; update_prob <= 0 freezes all).
 * The 64-bit seed folds to 32 bits as (seed ^ seed >> 32); lane l's seed is
 * that ^ (l * n) (gpu/executor/state.rs:1282-1312), or, when lane_seeds is
 * given (batch entries), the fold of lane_seeds[l].  update_prob >= 1 turns
 * the mask off.  The material / coarse-material extensions of the reference
 * mask are not part of this path. */
npa_status npa_executor_set_update_prob(npa_executor* exec, float update_prob, uint64_t seed,
                                        const uint64_t* lane_seeds);
/* The step index the next step's mask uses (0 after create); each step
 * advances it by one, with or without the mask, as the reference's
 * WgpuAutomataState::step_index. */
npa_status npa_executor_set_step_index(npa_executor* exec, uint32_t step_index);
npa_status npa_executor_step_index(npa_executor* exec, uint32_t* step_index);
/* read_state (executor/readback.rs:85): synchronises and copies to host. */
npa_status npa_executor_read_state(npa_executor* exec, float* positions, float* states);
/* Current resident device buffers ([f32;4] positions, states). */
npa_status npa_executor_state_device(npa_executor* exec, float** d_positions, float** d_states);
/* Kernels launched per rollout step by this executor. */
npa_status npa_executor_launches_per_step(npa_executor* exec, int64_t* launches);

/* Selects the executor's step kernels: fused = 1 runs perception, the MLP
 * and the Euler step as one kernel after the density pass (the feature rows
 * stay in shared memory, the role of the reference's single update pass,
 * crates/burn_automata/src/gpu_step.wgsl:3656-4484), two blocks per SM each
 * alternating perception and MLP; fused = 2 is the warp-specialised form
 * (perception warps and MLP warps of one block per SM handing feature tiles
 * over in shared memory); fused = 0 (the default) runs perception into
 * feature tiles and the MLP stage as two kernels.  All give identical
 * results.  NPA_ERR_UNSUPPORTED outside a fused kernel's range (2D, sparse
 * cells; fused = 1: C > 4, hidden width <= 128; fused = 2: C <= 16, hidden
 * width 128). */
npa_status npa_executor_set_fused_step(npa_executor* exec, int32_t fused);

/* Splits the batch into `groups` (1..min(4, batch)) runs of consecutive
 * rollouts for npa_executor_step_many's graph replay: each run gets its own
 * workspace and its steps form an independent chain of the step graph, so
 * the latency-bound phases of one run (the per-rollout sort, the neighbour
 * walks) overlap the others' work.  Rollouts never interact, so the results
 * are identical for every grouping.  The profiled replay
 * (npa_executor_step_many_profiled) and use_graph = 0 step the whole batch
 * phase by phase. */
npa_status npa_executor_set_step_groups(npa_executor* exec, int32_t groups);
/* The executor's rollout groups: 2 after npa_executor_create for batches of
 * 2 or more rollouts with at most 262,144 particles in all, else 1. */
npa_status npa_executor_step_groups(npa_executor* exec, int32_t* groups);

#ifdef __cplusplus
}
#endif

#endif /* NPA_B200_H */
