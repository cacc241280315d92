// stdrng.cu -- the CPU rollout's stochastic update masks, computed on the GPU.
//
// run_rollout_from_particles (crates/burn_automata/src/rollout/mod.rs:222-238)
// seeds StdRng::seed_from_u64(cfg.seed ^ 0x5eed), and each step's
// stochastic_mask (:644-651) draws random::<f32>() < update_prob for the
// particles in index order (ones, drawing nothing, when update_prob >= 1).
// StdRng is rand 0.9.4's ChaCha12Rng (rand_chacha 0.9.0), seeded by rand_core
// 0.9's seed_from_u64.  Those crates are not in the reference tree; their
// published algorithms, restated:
//   seed_from_u64: a PCG32 generator (O'Neill 2014, XSH-RR 64/32 output) whose
//     64-bit LCG state (multiplier 6364136223846793005, increment
//     11634580027462260723) is stepped before each output; eight outputs,
//     little-endian, form the 32-byte seed;
//   ChaCha12Rng: Bernstein's ChaCha with 12 rounds, words 0-3 the
//     "expand 32-byte k" constants, 4-11 the seed as little-endian words,
//     12-13 a 64-bit block counter from 0, 14-15 the stream (0); the u32
//     outputs are the blocks' words in order;
//   random::<f32>(): (next_u32() >> 8) * 2^-24.
// The stream is counter-based, so step s's value for particle i (stream word
// s * count + i) needs no sequential state: one thread computes one 16-word
// block and writes the mask entries that fall in the requested range.
#include "npa_internal.h"

namespace npa {
namespace {

__device__ __forceinline__ uint32_t rotl(uint32_t x, int r) { return __funnelshift_l(x, x, r); }

__device__ __forceinline__ void quarter_round(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  a += b;
  d = rotl(d ^ a, 16);
  c += d;
  b = rotl(b ^ c, 12);
  a += b;
  d = rotl(d ^ a, 8);
  c += d;
  b = rotl(b ^ c, 7);
}

__global__ void stdrng_mask_kernel(ChachaKey key, uint64_t word0, uint64_t end, float update_prob,
                                   float* __restrict__ mask) {
  const uint64_t block = (word0 >> 4) + uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if ((block << 4) >= end) return;
  uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
#pragma unroll
  for (int k = 0; k < 8; ++k) in[4 + k] = key.k[k];
  in[12] = uint32_t(block);
  in[13] = uint32_t(block >> 32);
  in[14] = 0u;
  in[15] = 0u;
  uint32_t x[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = in[k];
#pragma unroll
  for (int r = 0; r < 12; r += 2) {
    quarter_round(x[0], x[4], x[8], x[12]);
    quarter_round(x[1], x[5], x[9], x[13]);
    quarter_round(x[2], x[6], x[10], x[14]);
    quarter_round(x[3], x[7], x[11], x[15]);
    quarter_round(x[0], x[5], x[10], x[15]);
    quarter_round(x[1], x[6], x[11], x[12]);
    quarter_round(x[2], x[7], x[8], x[13]);
    quarter_round(x[3], x[4], x[9], x[14]);
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const uint64_t word = (block << 4) + k;
    if (word >= word0 && word < end) {
      const float u = float((x[k] + in[k]) >> 8) * (1.0f / 16777216.0f);
      mask[word - word0] = u < update_prob ? 1.0f : 0.0f;
    }
  }
}

}  // namespace

ChachaKey stdrng_key(uint64_t rng_seed) {
  ChachaKey key;
  uint64_t state = rng_seed;
  for (int k = 0; k < 8; ++k) {
    state = state * 6364136223846793005ull + 11634580027462260723ull;
    const uint32_t xorshifted = uint32_t(((state >> 18) ^ state) >> 27);
    const uint32_t rot = uint32_t(state >> 59);
    key.k[k] = (xorshifted >> rot) | (xorshifted << ((32u - rot) & 31u));
  }
  return key;
}

npa_status launch_stdrng_mask(const ChachaKey& key, uint64_t word0, uint32_t count,
                              float update_prob, float* mask, cudaStream_t stream) {
  if (count == 0) return NPA_OK;
  const uint64_t end = word0 + count;
  const uint64_t blocks = ((end + 15) >> 4) - (word0 >> 4);
  stdrng_mask_kernel<<<grid_for(blocks, 256), 256, 0, stream>>>(key, word0, end, update_prob,
                                                                   mask);
  return after_launch("stdrng_mask_kernel");
}

}  // namespace npa
