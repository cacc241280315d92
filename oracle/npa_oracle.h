/*
 * npa_oracle.h -- CPU restatement of the burn_automata NPA rollout path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * product in burn_automata_b200/.  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline legs of bench.py may load it.  The product never links, calls
 * or falls back to it.
 *
 * It restates, in plain C with the reference's f32 operation order (no FMA
 * contraction, left-to-right sums, binary-exponentiation powi), these files of
 * mosure/burn_automata:
 *   crates/burn_automata_kernels/src/config.rs          (HashGridConfig::validate)
 *   crates/burn_automata_kernels/src/hashgrid.rs        (build_hashgrid, cell math)
 *   crates/burn_automata_kernels/src/reference/{forward,neighbor,kernels,normalize,step}.rs
 *   crates/burn_automata_kernels/src/gaussian.rs        (decode_gaussians_3d)
 *   crates/burn_automata/src/config.rs:133-162          (NpaConfig dims / eps)
 *   crates/burn_automata/src/model.rs:768-940           (step_cpu, MLP)
 *   crates/burn_automata/src/rollout/mod.rs:240-283     (rollout loop)
 *   crates/burn_automata/src/rollout/mod.rs:222-238, :644-651 (StdRng masks;
 *     rand 0.9.4 / rand_chacha 0.9.0 / rand_core 0.9 restated, PARITY UNPINNED)
 * Each function in npa_oracle.c cites the file:line it follows.
 *
 * Index arrays are int64 (the reference uses usize).  Status codes are the
 * same numbers the product's C ABI uses (include/npa_b200.h).
 */
#ifndef NPA_ORACLE_H
#define NPA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORA_OK = 0,
  ORA_ERR_INVALID_DIM = 1,
  ORA_ERR_INVALID_EPS = 2,
  ORA_ERR_INVALID_GRID_SIZE = 3,
  ORA_ERR_PARTICLE_MODE_REQUIRES_POW2 = 4,
  ORA_ERR_POSITION_SHAPE = 5,
  ORA_ERR_STATE_SHAPE = 6,
  ORA_ERR_OUTPUT_SHAPE = 7,
  ORA_ERR_INVALID_ARGUMENT = 8,
  ORA_ERR_INVALID_MODEL = 9,
};

/* Same layout as npa_grid_config in include/npa_b200.h. */
typedef struct ora_grid_config {
  int32_t dim;       /* 2 or 3 */
  int32_t boundary;  /* 0 = Periodic, 1 = Clamped */
  int32_t mode;      /* 0 = Grid, 1 = Particle */
  int32_t max_particles_per_block;
  int64_t grid_size[3];
  float eps;
  int32_t reserved;
} ora_grid_config;

/* Same layout as npa_perception_options. */
typedef struct ora_perception_options {
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
} ora_perception_options;

/* Same layout as npa_model_config. equivariance: 0 None, 1 ParticleDensity,
 * 2 ParticleDensityAndScale. */
typedef struct ora_model_config {
  int32_t spatial_dims;
  int32_t state_dims;
  int32_t hidden_dims;
  int32_t auxiliary_input_dims;
  float eps0;
  float alpha;
  int32_t equivariance;
  uint8_t density_grad;
  uint8_t state_grad;
  uint8_t log_norm_grad;
  uint8_t log_norm_density_grad;
  uint8_t position_features;
  uint8_t reserved[7];
} ora_model_config;

/* Same layout as npa_gaussian_decode_config. mode: 0 ParticlePoint,
 * 1 GaussianSh0FixedScale, 2 GaussianSh0LearnedScale, 3 GaussianSh0Oriented. */
typedef struct ora_decode_config {
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
} ora_decode_config;

int ora_grid_validate(const ora_grid_config* cfg);
int64_t ora_cell_count(const ora_grid_config* cfg);
/* cell index of one position (hashgrid.rs:71 cell_for_position). */
int64_t ora_cell_for_position(const ora_grid_config* cfg, const float* pos4);

int ora_build_hashgrid(const ora_grid_config* cfg, const float* positions,
                       int64_t batch, int64_t n, int64_t* bin_offsets,
                       int64_t* permutation, int64_t* inverse_permutation);

int64_t ora_feature_dims(const ora_grid_config* cfg, const ora_perception_options* opt,
                         int64_t state_dims);

/* perceive_with_options.  Every output pointer may be NULL except features. */
int ora_perceive(const ora_grid_config* cfg, const ora_perception_options* opt,
                 const float* positions, const float* states, int64_t batch,
                 int64_t n, int64_t state_dims, float* features, float* density,
                 float* blurred_state, float* state_gradient,
                 float* density_gradient);

/* Per-particle determinant of the hybrid moment matrix, as
 * safe_inverse_symmetric computes it (test infrastructure). */
int ora_moment_det(const ora_grid_config* cfg, const float* positions, int64_t batch, int64_t n,
                   float* det_out);

int ora_forward_update(const float* features, int64_t rows, int64_t in_dims,
                       int64_t hidden_dims, int64_t out_dims, const float* w1,
                       const float* b1, const float* w2, const float* b2,
                       float* update);

int ora_euler_step(const ora_grid_config* cfg, const float* positions,
                   const float* states, const float* dx, const float* ds,
                   int64_t batch, int64_t n, int64_t state_dims, float dt,
                   const float* update_mask, float* next_positions,
                   float* next_states);

int64_t ora_model_perception_dims(const ora_model_config* m);

/* NpaModel::step_cpu.  features/density/dx/ds outputs may be NULL. */
int ora_step(const ora_model_config* m, const float* w1, const float* b1,
             const float* w2, const float* b2, const ora_grid_config* grid,
             const float* positions, const float* states, int64_t batch,
             int64_t n, float dt, const float* update_mask,
             float* next_positions, float* next_states, float* dx, float* ds,
             float* features, float* density);

/* run_rollout_from_particles with update_prob >= 1 (mask of ones) or a fixed
 * per-step mask callback-free variant: masks == NULL means all ones,
 * otherwise masks holds steps * batch * n values.  positions/states are
 * updated in place; mean_dx (may be NULL) receives one value per step. */
int ora_rollout(const ora_model_config* m, const float* w1, const float* b1,
                const float* w2, const float* b2, const ora_grid_config* grid,
                float* positions, float* states, int64_t batch, int64_t n,
                int64_t steps, float dt, const float* masks, float* mean_dx);

int64_t ora_gaussian_record_floats(const ora_decode_config* cfg);
/* decode_gaussians_3d; record layout per particle:
 * [position_visibility 4][rotation 4][scale_opacity 4][sh 3*k]. */
int ora_decode_gaussians(const ora_decode_config* cfg, const float* positions,
                         const float* states, int64_t count, int64_t state_dims,
                         float* out);

/* The GPU executor's stochastic update mask for one step: out[lane * n + i]
 * (gpu_step.wgsl:1019-1056; tests/gpu_wgpu/common.rs:115-137). */
int ora_gpu_update_mask(int64_t batch, int64_t n, float update_prob, uint32_t step,
                        const uint32_t* lane_seeds, float* out);
/* perceive_adjoint_with_options (reference/adjoint.rs:28-136): feature_adjoint
 * [B*N][F] -> state_adjoint [B*N*C] and position_adjoint [B*N][4]. */
int ora_perceive_adjoint(const ora_grid_config* cfg, const ora_perception_options* opt,
                         const float* positions, const float* states, int64_t batch, int64_t n,
                         int64_t c, const float* feature_adjoint, float* state_adjoint,
                         float* position_adjoint);
/* Splat2dConfig (splat.rs:4-28). */
typedef struct ora_splat2d_config {
  int64_t image_size;
  float sigma, lo, hi;
  int32_t normalize_color, y_up;
  float pixel_size;
} ora_splat2d_config;
/* splat_particles_2d (splat.rs:30-93): out [size * size][4] (RGB + weight). */
int ora_splat_particles_2d(const ora_splat2d_config* cfg, const float* positions,
                           const float* colors, int64_t count, float* out);
/* The CPU rollout's update masks (rollout/mod.rs:222-238 seeds
 * StdRng::seed_from_u64(seed ^ 0x5eed); stochastic_mask :644-651 draws
 * random::<f32>() < update_prob per particle and step).  StdRng is rand 0.9.4's
 * ChaCha12Rng (rand_chacha 0.9.0) seeded by rand_core 0.9's seed_from_u64;
 * see npa_oracle.c for the restated algorithms.  PARITY UNPINNED for the
 * seeding and the 12-round stream (no Rust toolchain, no golden values); the
 * block function is checked at 20 rounds against OpenSSL's ChaCha20. */
void ora_stdrng_key(uint64_t rng_seed, uint32_t key[8]);
void ora_chacha_block(const uint32_t key[8], uint64_t counter, int rounds, uint32_t out[16]);
/* out[k * count + i] for rollout steps first_step + k (0-based), k < steps. */
int ora_rollout_masks(uint64_t rollout_seed, float update_prob, int64_t count,
                      int64_t first_step, int64_t steps, float* out);
/* Training rollout (crates/burn_automata/src/training.rs:558-640,
 * target2d.rs:3414-3722). */
int ora_mlp_backward(const float* features, int64_t rows, int64_t in_dims, int64_t hidden,
                     int64_t out_dims, const float* w1, const float* b1, const float* w2,
                     const float* output_gradients, float* gw1, float* gb1, float* gw2,
                     float* gb2, float* gfeatures);
int ora_rollout_for_training(const ora_model_config* m, const float* w1, const float* b1,
                             const float* w2, const float* b2, const ora_grid_config* grid,
                             const float* positions, const float* states, int64_t batch,
                             int64_t n, int64_t steps, float update_prob, uint64_t seed,
                             float* snap_positions, float* snap_states, float* snap_masks,
                             float* final_positions, float* final_states,
                             float* mean_dx_norm_sum);
int ora_bptt_gradients(const ora_model_config* m, const float* w1, const float* b1,
                       const float* w2, const float* b2, const ora_grid_config* grid,
                       const float* snap_positions, const float* snap_states,
                       const float* snap_masks, int64_t batch, int64_t n, int64_t steps,
                       const float* position_gradients, const float* state_gradients,
                       float regularizer_weight, int stopgrad_pos, int stopgrad_state,
                       float* gw1, float* gb1, float* gw2, float* gb2, float* pos_adj_out,
                       float* state_adj_out);
/* out[i] = log1pf(x[i]) of the host C library (f32::ln_1p of the reference). */
void ora_ln_1p(const float* x, int64_t count, float* out);
/* 0 (default): log1pf as the reference binds it; 1: f64 log1p rounded to f32,
 * the device library's arithmetic (to compare the GPU bit for bit). */
void ora_set_log1p_mode(int mode);
/* Threads used by the OpenMP loops (0 = OpenMP default). */
void ora_set_threads(int threads);
int ora_get_threads(void);

#ifdef __cplusplus
}
#endif

#endif
