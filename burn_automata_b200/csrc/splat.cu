// splat.cu -- splat_particles_2d (crates/burn_automata_kernels/src/splat.rs:30-93).
//
// Every particle adds colour * w to the pixels of its (2r+1)^2 footprint; the
// reference loops particles in order, so each pixel's sums run in particle
// order.  On the GPU the image is cut into 16 x 16 pixel tiles, one block per
// tile: the block scans the particles in index order in chunks of 256,
// compacts (order-preserving) the ones whose footprint touches the tile into
// shared memory, and each thread (one pixel) adds their contributions in that
// order.  No atomics, so every pixel receives the reference's sum order.
//   splat_prep_kernel   per particle: pixel coordinates, footprint base and
//                       fraction, and the footprint's weight sum (normaliser),
//                       summed in the reference's (oy, ox) order
//   splat_tile_kernel   per tile: gather and accumulate as above
// exp is evaluated in f64 and rounded once (correctly rounded but for rare
// ties), like the host libm's expf to within its own error.
#include "npa_internal.h"

namespace npa {
namespace {

constexpr int kTile = 16;
constexpr int kTileThreads = kTile * kTile;

struct SplatParams {
  int size;
  float lo, hi, fsize, two_s2, norm_scale;
  long long radius;  // (5 sigma).ceil().max(1) as isize, at most 2^62
  int normalize, y_up;
};

// A particle's footprint: base pixel, fraction, normaliser.
struct SplatPrep {
  long long base_x, base_y;
  float frac_x, frac_y, denom;
  int valid;  // footprint intersects the image
};

__device__ __forceinline__ float gauss(const SplatParams& p, long long ox, long long oy, float fx,
                                       float fy) {
  const float dx = static_cast<float>(ox) - fx;
  const float dy = static_cast<float>(oy) - fy;
  float t = dx * dx;
  t = t + dy * dy;
  return static_cast<float>(exp(static_cast<double>(-t / p.two_s2)));
}

// [lo, hi] of the footprint offsets o in [-r, r] with base + o inside
// [0, size); empty (lo > hi) when the footprint misses the image.  base may be
// any saturated value; r <= 2^62 and size < 2^31 keep every sum in range.
__device__ __forceinline__ void in_image(long long base, long long r, int size, long long& lo,
                                         long long& hi) {
  const long long last_pixel = static_cast<long long>(size) - 1;
  if (base < -r || base > last_pixel + r) {
    lo = 1;
    hi = 0;
    return;
  }
  lo = -base > -r ? -base : -r;
  hi = last_pixel - base < r ? last_pixel - base : r;
}

__global__ void splat_prep_kernel(SplatParams p, const float4* __restrict__ pos,
                                  uint32_t count, SplatPrep* __restrict__ prep) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const float4 q = __ldg(pos + i);
  const float px = (q.x - p.lo) / (p.hi - p.lo) * (p.fsize - 1.0f);
  float py = (q.y - p.lo) / (p.hi - p.lo) * (p.fsize - 1.0f);
  if (p.y_up) py = (p.fsize - 1.0f) - py;
  SplatPrep r;
  r.base_x = f2ll_sat(floorf(px));
  r.base_y = f2ll_sat(floorf(py));
  r.frac_x = px - static_cast<float>(r.base_x);
  r.frac_y = py - static_cast<float>(r.base_y);
  long long xlo, xhi, ylo, yhi;
  in_image(r.base_x, p.radius, p.size, xlo, xhi);
  in_image(r.base_y, p.radius, p.size, ylo, yhi);
  r.valid = (xlo <= xhi && ylo <= yhi) ? 1 : 0;
  float sum = 0.0f;
  if (r.valid)
    for (long long oy = ylo; oy <= yhi; ++oy)
      for (long long ox = xlo; ox <= xhi; ++ox) sum = sum + gauss(p, ox, oy, r.frac_x, r.frac_y);
  r.denom = p.normalize ? fmaxf(sum, 1e-8f) : 1.0f;
  prep[i] = r;
}

__global__ void __launch_bounds__(kTileThreads)
splat_tile_kernel(SplatParams p, const SplatPrep* __restrict__ prep,
                  const float* __restrict__ colors, uint32_t count, float4* __restrict__ out) {
  __shared__ uint32_t list[kTileThreads];
  __shared__ uint32_t warp_count[kTileThreads / 32];
  const int tiles_x = (p.size + kTile - 1) / kTile;
  const int tx0 = (blockIdx.x % tiles_x) * kTile, ty0 = (blockIdx.x / tiles_x) * kTile;
  const int x = tx0 + threadIdx.x % kTile, y = ty0 + threadIdx.x / kTile;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const long long r0 = p.radius;
  for (uint32_t c0 = 0; c0 < count; c0 += kTileThreads) {
    const uint32_t i = c0 + threadIdx.x;
    bool hit = false;
    if (i < count) {
      const SplatPrep& q = prep[i];
      // footprint [base - r, base + r] meets the tile [t0, t0 + kTile)
      hit = q.valid && q.base_x >= tx0 - r0 && q.base_x < tx0 + kTile + r0 &&
            q.base_y >= ty0 - r0 && q.base_y < ty0 + kTile + r0;
    }
    // order-preserving compaction of this chunk's hits
    const uint32_t ballot = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) warp_count[warp] = __popc(ballot);
    __syncthreads();
    uint32_t before = 0, total = 0;
    for (uint32_t w = 0; w < kTileThreads / 32; ++w) {
      if (w < warp) before += warp_count[w];
      total += warp_count[w];
    }
    if (hit) list[before + __popc(ballot & ((1u << lane) - 1u))] = i;
    __syncthreads();
    if (x < p.size && y < p.size) {
      for (uint32_t k = 0; k < total; ++k) {
        const uint32_t j = list[k];
        const SplatPrep q = prep[j];
        const long long ox = x - q.base_x, oy = y - q.base_y;
        if (ox < -r0 || ox > r0 || oy < -r0 || oy > r0) continue;
        const float w = gauss(p, ox, oy, q.frac_x, q.frac_y) / q.denom * p.norm_scale;
        acc.x = acc.x + __ldg(colors + size_t(j) * 3) * w;
        acc.y = acc.y + __ldg(colors + size_t(j) * 3 + 1) * w;
        acc.z = acc.z + __ldg(colors + size_t(j) * 3 + 2) * w;
        acc.w = acc.w + w;
      }
    }
    __syncthreads();
  }
  if (x < p.size && y < p.size) out[size_t(y) * p.size + x] = acc;
}

}  // namespace

size_t splat_workspace_bytes(uint32_t count) { return size_t(count) * sizeof(SplatPrep) + 256; }

npa_status launch_splat_2d(const npa_splat2d_config& cfg, const float4* positions,
                           const float* colors, uint32_t count, float4* out, void* workspace,
                           cudaStream_t stream) {
  SplatParams p;
  p.size = static_cast<int>(cfg.image_size);
  p.lo = cfg.lo;
  p.hi = cfg.hi;
  p.fsize = static_cast<float>(cfg.image_size);
  float sigma = cfg.sigma;
  p.normalize = cfg.normalize_color ? 1 : 0;
  p.y_up = cfg.y_up ? 1 : 0;
  if (p.normalize) sigma = sigma * p.fsize * cfg.pixel_size / (cfg.hi - cfg.lo);
  // (5.0 * sigma).ceil().max(1.0) as isize (NaN -> 0, saturating); any radius
  // of 2^62 or more already covers every pixel from every base.
  const float rf = fmaxf(ceilf(5.0f * sigma), 1.0f);
  p.radius = (rf != rf) ? 0 : (rf >= 4.6e18f ? (1ll << 62) : static_cast<long long>(rf));
  p.two_s2 = 2.0f * sigma * sigma;
  p.norm_scale = 1.0f;
  if (p.normalize) {
    const float r = p.fsize * cfg.pixel_size / (cfg.hi - cfg.lo);
    p.norm_scale = r * r;
  }
  if (p.size == 0) return NPA_OK;
  const int tiles_x = (p.size + kTile - 1) / kTile;
  SplatPrep* prep = static_cast<SplatPrep*>(workspace);
  if (count > 0) {
    splat_prep_kernel<<<grid_for(count, 256), 256, 0, stream>>>(p, positions, count, prep);
    NPA_TRY(after_launch("splat_prep_kernel"));
  }
  splat_tile_kernel<<<tiles_x * tiles_x, kTileThreads, 0, stream>>>(p, prep, colors, count, out);
  return after_launch("splat_tile_kernel");
}

}  // namespace npa
