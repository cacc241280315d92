// hashgrid.cu -- build_hashgrid (crates/burn_automata_kernels/src/hashgrid.rs:16-69)
// as a stable device-wide LSD radix sort.
//
// The reference runs a serial counting sort: count particles per
// (batch, cell) bin, exclusive-prefix the counts into bin_offsets, then scatter
// particles in ascending index order.  The result is the unique ordering by
// key = batch * cell_count + cell with ties broken by particle index.  Any
// stable sort by key produces exactly that ordering, so this file sorts
// (key, index) pairs with 8-bit LSD radix passes whose per-tile ranks are
// stable, and derives bin_offsets from the key boundaries of the sorted
// array.  Output is bit-identical to the reference.
//
// Per pass: a digit histogram per 4096-item tile, one exclusive scan of the
// digit-major [256 x tiles] table, then a scatter that ranks items inside the
// tile in index order (warp match_any + per-warp digit counters + a
// cross-warp prefix).  No kernel waits on another block.  Rollouts of at most
// 16,384 particles instead sort in shared memory, one block per rollout
// (rollout_sort_kernel).
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include <cuda.h>

#include "npa_internal.h"

namespace npa {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kItemsPerLane = 16;
constexpr int kWarpItems = 32 * kItemsPerLane;             // 512
constexpr int kTile = kSortWarps * kWarpItems;              // 4096
constexpr int kDigits = 256;
constexpr uint32_t kOrderCodes = 4096;  // 12-bit Morton codes of the processing order
constexpr int kScanThreads = 1024;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Keys of one tile plus the histogram of digit 0.
__global__ void __launch_bounds__(kSortThreads)
keys_hist_kernel(GridParams g, const float4* __restrict__ pos, uint32_t total, uint32_t n,
                 uint32_t* __restrict__ keys, uint32_t* __restrict__ vals,
                 uint32_t* __restrict__ hist, uint32_t tiles) {
  __shared__ uint32_t h[kDigits];
  for (int i = threadIdx.x; i < kDigits; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t seg = blockIdx.x * kTile + warp * kWarpItems;
#pragma unroll 4
  for (int r = 0; r < kItemsPerLane; ++r) {
    const uint32_t i = seg + r * 32 + lane;
    if (i < total) {
      const uint32_t b = i / n;
      const uint32_t key = b * g.cells + cell_for_position(g, pos[i]);
      keys[i] = key;
      vals[i] = i;
      atomicAdd(&h[key & 0xffu], 1u);
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kDigits; d += blockDim.x) hist[d * tiles + blockIdx.x] = h[d];
}

__global__ void __launch_bounds__(kSortThreads)
hist_kernel(const uint32_t* __restrict__ keys, uint32_t total, uint32_t shift,
            uint32_t* __restrict__ hist, uint32_t tiles) {
  __shared__ uint32_t h[kDigits];
  for (int i = threadIdx.x; i < kDigits; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const uint32_t base = blockIdx.x * kTile;
  for (uint32_t k = threadIdx.x; k < kTile; k += blockDim.x) {
    const uint32_t i = base + k;
    if (i < total) atomicAdd(&h[(keys[i] >> shift) & 0xffu], 1u);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kDigits; d += blockDim.x) hist[d * tiles + blockIdx.x] = h[d];
}

// In-place exclusive scan of `count` (a multiple of 4) uint32 by one block.
__global__ void __launch_bounds__(kScanThreads) scan_kernel(uint32_t* __restrict__ data,
                                                            uint32_t count) {
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t carry_s;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (uint32_t base = 0; base < count; base += kScanThreads * 4) {
    const uint32_t idx = base + tid * 4;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (idx < count) v = *reinterpret_cast<const uint4*>(data + idx);
    const uint32_t s1 = v.x + v.y, s2 = s1 + v.z, s3 = s2 + v.w;
    uint32_t incl = s3;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      uint32_t t = warp_tot[lane];
      uint32_t wi = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t u = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += u;
      }
      warp_tot[lane] = wi - t;  // exclusive warp offsets
    }
    __syncthreads();
    const uint32_t carry = carry_s;
    const uint32_t off = carry + warp_tot[warp] + (incl - s3);
    if (idx < count) {
      uint4 o;
      o.x = off;
      o.y = off + v.x;
      o.z = off + s1;
      o.w = off + s2;
      *reinterpret_cast<uint4*>(data + idx) = o;
    }
    __syncthreads();
    if (tid == kScanThreads - 1) carry_s = off + s3;
    __syncthreads();
  }
}

// One stable radix pass: keys/vals of a tile are ranked in index order and
// scattered to their global slots.
__global__ void __launch_bounds__(kSortThreads)
scatter_kernel(const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
               uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, uint32_t total,
               uint32_t shift, const uint32_t* __restrict__ hist_scanned, uint32_t tiles) {
  __shared__ uint32_t wh[kSortWarps][kDigits];
  for (int i = threadIdx.x; i < kSortWarps * kDigits; i += blockDim.x) (&wh[0][0])[i] = 0;
  __syncthreads();
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t seg = blockIdx.x * kTile + warp * kWarpItems;
  const uint32_t lt = lanemask_lt();
  uint32_t k[kItemsPerLane], v[kItemsPerLane], rank[kItemsPerLane];
#pragma unroll
  for (int r = 0; r < kItemsPerLane; ++r) {
    const uint32_t i = seg + r * 32 + lane;
    const bool valid = i < total;
    k[r] = valid ? keys_in[i] : 0u;
    v[r] = valid ? vals_in[i] : 0u;
    // Invalid lanes get a digit that matches no valid lane.
    const uint32_t d = valid ? ((k[r] >> shift) & 0xffu) : (0x100u + lane);
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const uint32_t before = valid ? wh[warp][d] : 0u;
    __syncwarp();
    if (valid && lane == static_cast<uint32_t>(__ffs(peers) - 1))
      wh[warp][d] = before + __popc(peers);
    __syncwarp();
    rank[r] = before + __popc(peers & lt);
  }
  __syncthreads();
  // Cross-warp exclusive prefix per digit, offset by the tile's global base.
  for (int d = threadIdx.x; d < kDigits; d += blockDim.x) {
    uint32_t run = hist_scanned[d * tiles + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      const uint32_t c = wh[w][d];
      wh[w][d] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kItemsPerLane; ++r) {
    const uint32_t i = seg + r * 32 + lane;
    if (i < total) {
      const uint32_t d = (k[r] >> shift) & 0xffu;
      const uint32_t dst = wh[warp][d] + rank[r];
      if (dst < total) {  // always true for a consistent histogram; keeps writes in bounds
        keys_out[dst] = k[r];
        vals_out[dst] = v[r];
      }
    }
  }
}

// Reference outputs and sorted views from the sorted (key, index) pairs.
__global__ void finalize_kernel(GridParams g, const float4* __restrict__ pos,
                                const uint32_t* __restrict__ keys,
                                const uint32_t* __restrict__ vals, uint32_t total, uint32_t n,
                                uint32_t total_bins, uint32_t* __restrict__ bin_offsets,
                                uint32_t* __restrict__ perm, uint32_t* __restrict__ inv,
                                float4* __restrict__ srec, int2* __restrict__ scyz) {
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= total) return;
  const uint32_t key = keys[q];
  const uint32_t i = vals[q];
  if (i >= total || key >= total_bins) return;  // only reachable if the sort were inconsistent
  const uint32_t b = i / n;
  perm[q] = i - b * n;
  inv[i] = q - b * n;
  const float4 p = pos[i];
  const int3 c = cell_coords(g, p);
  if (g.dim == 2) {
    srec[q] = make_float4(p.x, p.y, __int_as_float(c.x), __int_as_float(c.y));
  } else {
    srec[q] = make_float4(p.x, p.y, p.z, __int_as_float(c.x));
    scyz[q] = make_int2(c.y, c.z);
  }
  // bin_offsets[bin] = first sorted slot whose key >= bin.
  const uint32_t first = q == 0 ? 0u : keys[q - 1] + 1u;
  for (uint32_t bin = first; bin <= key; ++bin) bin_offsets[bin] = q;
  if (q == total - 1)
    for (uint32_t bin = key + 1; bin <= total_bins; ++bin) bin_offsets[bin] = total;
}

// Processing order of the device-wide path: sorted slots keyed by batch and
// the Morton code of their cell block (cell coordinates >> shift, the low
// `bits` bits per axis), so consecutive threads of the neighbour walks handle
// spatially adjacent particles whose neighbours are shared in cache (hash
// order scatters them).  Digit 0 of the keys is histogrammed per tile as in
// keys_hist_kernel; the stable radix passes then sort (key, slot).
__global__ void __launch_bounds__(kSortThreads)
order_keys_kernel(GridParams g, const float4* __restrict__ srec, const int2* __restrict__ scyz,
                  uint32_t total, uint32_t n, int shift, uint32_t* __restrict__ keys,
                  uint32_t* __restrict__ vals, uint32_t* __restrict__ hist, uint32_t tiles) {
  __shared__ uint32_t h[kDigits];
  for (int i = threadIdx.x; i < kDigits; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t seg = blockIdx.x * kTile + warp * kWarpItems;
#pragma unroll 4
  for (int r = 0; r < kItemsPerLane; ++r) {
    const uint32_t i = seg + r * 32 + lane;
    if (i < total) {
      const float4 rec = srec[i];
      uint32_t code = 0;
      if (g.dim == 2) {
        const uint32_t x = uint32_t(__float_as_int(rec.z) >> shift);
        const uint32_t y = uint32_t(__float_as_int(rec.w) >> shift);
#pragma unroll
        for (int b = 0; b < 6; ++b)
          code |= (((x >> b) & 1u) << (2 * b)) | (((y >> b) & 1u) << (2 * b + 1));
      } else {
        const int2 yz = scyz[i];
        const uint32_t x = uint32_t(__float_as_int(rec.w) >> shift);
        const uint32_t y = uint32_t(yz.x >> shift), z = uint32_t(yz.y >> shift);
#pragma unroll
        for (int b = 0; b < 4; ++b)
          code |= (((x >> b) & 1u) << (3 * b)) | (((y >> b) & 1u) << (3 * b + 1)) |
                  (((z >> b) & 1u) << (3 * b + 2));
      }
      const uint32_t key = (i / n) * kOrderCodes + code;
      keys[i] = key;
      vals[i] = i;
      atomicAdd(&h[key & 0xffu], 1u);
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kDigits; d += blockDim.x) hist[d * tiles + blockIdx.x] = h[d];
}

// ---------------------------------------------------------------------------
// Small rollouts: one block per rollout sorts that rollout's particles in
// shared memory and writes the outputs directly (one launch for the batch).
// Same stable (cell, index) order, built as
//   1. per-cell counts (shared atomics) and their exclusive scan = bin starts;
//   2. an unordered scatter of particle indices into their cell's segment
//      (atomic cursor per cell; afterwards cursor[c] = start of cell c + 1);
//   3. each particle's slot = its cell's start + the number of segment
//      members with a smaller index (one read per member: cells hold a few
//      particles, so this is cheaper than a serial stable ranking).
// Used when a rollout's counts and indices fit in shared memory.
// ---------------------------------------------------------------------------
constexpr int kRolloutThreads = 1024;
constexpr uint32_t kRolloutMaxN = 16384;
constexpr uint32_t kRolloutMaxCells = 65535;  // cell ids fit in 16 bits
constexpr size_t kRolloutSmemBudget = 200 * 1024;

// Exclusive scan of cnt[0, count) in place by the whole block.
__device__ __forceinline__ void block_exclusive_scan(uint32_t* cnt, uint32_t count,
                                                     uint32_t* warp_sums) {
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t per = (count + blockDim.x - 1) / blockDim.x;
  const uint32_t lo = min(count, tid * per), hi = min(count, lo + per);
  uint32_t local = 0;
  for (uint32_t c = lo; c < hi; ++c) local += cnt[c];
  uint32_t incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= uint32_t(o)) incl += t;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t nw = blockDim.x >> 5;
    const uint32_t t = lane < nw ? warp_sums[lane] : 0u;
    uint32_t wi = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= uint32_t(o)) wi += u;
    }
    if (lane < nw) warp_sums[lane] = wi - t;
  }
  __syncthreads();
  uint32_t run = warp_sums[warp] + incl - local;
  for (uint32_t c = lo; c < hi; ++c) {
    const uint32_t v = cnt[c];
    cnt[c] = run;
    run += v;
  }
  __syncthreads();
}

// MINB blocks per SM: 2 (32 registers) when there are more rollouts than SMs
// and two blocks' shared memory fits, so all of them run in one wave (cfg2's
// 256 rollouts: 0.031 vs 0.036 ms); else 1 (42 registers; a single rollout
// runs faster: cfg0 0.019 vs 0.020 ms).
template <int MINB>
__global__ void __launch_bounds__(kRolloutThreads, MINB)
rollout_sort_kernel(GridParams g, const float4* __restrict__ pos, uint32_t n, uint32_t batch,
                    uint32_t* __restrict__ bin_offsets, uint32_t* __restrict__ perm,
                    uint32_t* __restrict__ inv, float4* __restrict__ srec,
                    int2* __restrict__ scyz) {
  extern __shared__ uint32_t sm[];
  __shared__ uint32_t warp_sums[32];
  uint32_t* cur = sm;                                          // [cells]
  uint16_t* key = reinterpret_cast<uint16_t*>(sm + g.cells);  // [n]: cell, then slot
  uint16_t* seg = key + n;                                     // [n]: indices by cell
  const uint32_t b = blockIdx.x;
  const uint32_t base = b * n;
  const uint32_t cells = g.cells;
  for (uint32_t c = threadIdx.x; c < cells; c += blockDim.x) cur[c] = 0;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    uint32_t c = cell_for_position(g, pos[base + i]);
    if (c >= cells) c = cells - 1;  // never taken (ids are < cells); keeps indices in bounds
    key[i] = static_cast<uint16_t>(c);
    atomicAdd(&cur[c], 1u);
  }
  __syncthreads();
  block_exclusive_scan(cur, cells, warp_sums);
  uint32_t* offsets = bin_offsets + size_t(b) * cells;
  for (uint32_t c = threadIdx.x; c < cells; c += blockDim.x) offsets[c] = base + cur[c];
  if (b == batch - 1 && threadIdx.x == 0) bin_offsets[size_t(batch) * cells] = batch * n;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t at = atomicAdd(&cur[key[i]], 1u);
    if (at < n) seg[at] = static_cast<uint16_t>(i);
  }
  __syncthreads();
  // cur[c] is now the end of cell c's segment, i.e. the start of cell c + 1.
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t c = key[i];
    const uint32_t lo = c == 0 ? 0u : cur[c - 1];
    const uint32_t hi = min(cur[c], n);
    uint32_t rank = 0;
    for (uint32_t k = lo; k < hi; ++k) rank += seg[k] < i ? 1u : 0u;
    key[i] = static_cast<uint16_t>(lo + rank);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t slot = key[i];
    if (slot >= n) continue;  // only reachable if the counts were inconsistent
    const uint32_t q = base + slot;
    perm[q] = i;
    inv[base + i] = slot;
    const float4 p = pos[base + i];
    const int3 cc = cell_coords(g, p);
    if (g.dim == 2) {
      srec[q] = make_float4(p.x, p.y, __int_as_float(cc.x), __int_as_float(cc.y));
    } else {
      srec[q] = make_float4(p.x, p.y, p.z, __int_as_float(cc.x));
      scyz[q] = make_int2(cc.y, cc.z);
    }
  }
}

size_t rollout_sort_smem(const GridParams& g, uint32_t n) {
  return size_t(g.cells) * sizeof(uint32_t) + size_t(n) * 2 * sizeof(uint16_t);
}

// The shared-memory path needs the rollout to fit, and enough rollouts (or
// small enough ones) that one block per rollout beats the device-wide sort:
// measured on B200, cfg0 (1 x 4,096) 0.019 vs 0.044 ms, cfg2 (256 x 4,096)
// 0.036 vs 0.139 ms, but cfg3 (1 x 16,384, 32,768 cells) 0.123 vs 0.049 ms.
bool rollout_sort_fits(const GridParams& g, uint32_t batch, uint32_t n) {
  return n <= kRolloutMaxN && g.cells <= kRolloutMaxCells &&
         rollout_sort_smem(g, n) <= kRolloutSmemBudget && (batch >= 8 || n <= 8192);
}

__global__ void fill_u32_kernel(uint32_t* p, uint32_t count, uint32_t value) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) p[i] = value;
}

uint32_t key_bits(uint64_t bins) {
  uint32_t bits = 0;
  while (bits < 32 && (uint64_t(1) << bits) < bins) ++bits;
  return bits;
}

}  // namespace

size_t sorted_view_bytes(uint32_t batch, uint32_t n) {
  const size_t total = size_t(batch) * n;
  return ((total * sizeof(float4) + 255) & ~size_t(255)) + total * sizeof(int2) + 256;
}

size_t hashgrid_scratch_bytes(const GridParams& g, uint32_t batch, uint32_t n) {
  const size_t total = size_t(batch) * n;
  const size_t tiles = (total + kTile - 1) / kTile;
  Carve c(nullptr, 0);
  c.take<uint32_t>(total);
  c.take<uint32_t>(total);
  c.take<uint32_t>(total);
  c.take<uint32_t>(total);
  c.take<uint32_t>(tiles * kDigits);
  return c.used + 256;
}

npa_status launch_hashgrid(const GridParams& g, const float4* positions, uint32_t batch,
                           uint32_t n, const HashgridBuffers& out, void* scratch,
                           size_t scratch_bytes, cudaStream_t stream) {
  const uint64_t total64 = uint64_t(batch) * n;
  const uint64_t bins64 = uint64_t(batch) * g.cells;
  const uint32_t total = static_cast<uint32_t>(total64);
  const uint32_t bins = static_cast<uint32_t>(bins64);
  if (total == 0) {
    fill_u32_kernel<<<grid_for(bins + 1, 256), 256, 0, stream>>>(out.bin_offsets, bins + 1, 0u);
    return after_launch("fill_u32_kernel");
  }
  if (rollout_sort_fits(g, batch, n)) {
    const size_t smem = rollout_sort_smem(g, n);
    auto launch = [&](auto kernel) -> npa_status {
      int per_sm = 0, sms = 0;
      NPA_TRY(kernel_occupancy(reinterpret_cast<const void*>(kernel), kRolloutThreads, smem,
                               &per_sm, &sms));
      kernel<<<batch, kRolloutThreads, smem, stream>>>(g, positions, n, batch, out.bin_offsets,
                                                        out.permutation, out.inverse, out.srec,
                                                        out.scyz);
      return after_launch("rollout_sort_kernel");
    };
    if (batch > 148 && smem <= 100 * 1024) return launch(rollout_sort_kernel<2>);
    return launch(rollout_sort_kernel<1>);
  }
  const uint32_t tiles = static_cast<uint32_t>((total64 + kTile - 1) / kTile);
  Carve c(scratch, scratch_bytes);
  uint32_t* ka = c.take<uint32_t>(total);
  uint32_t* va = c.take<uint32_t>(total);
  uint32_t* kb = c.take<uint32_t>(total);
  uint32_t* vb = c.take<uint32_t>(total);
  uint32_t* hist = c.take<uint32_t>(size_t(tiles) * kDigits);
  if (!c.fits()) return fail(NPA_ERR_INVALID_ARGUMENT, "hashgrid workspace too small");

  const uint32_t bits = key_bits(bins64);
  const uint32_t passes = bits == 0 ? 1u : (bits + 7) / 8;
  keys_hist_kernel<<<tiles, kSortThreads, 0, stream>>>(g, positions, total, n, ka, va, hist,
                                                        tiles);
  NPA_TRY(after_launch("keys_hist_kernel"));
  for (uint32_t pass = 0; pass < passes; ++pass) {
    const uint32_t shift = pass * 8;
    if (pass > 0) {
      hist_kernel<<<tiles, kSortThreads, 0, stream>>>(ka, total, shift, hist, tiles);
      NPA_TRY(after_launch("hist_kernel"));
    }
    scan_kernel<<<1, kScanThreads, 0, stream>>>(hist, tiles * kDigits);
    NPA_TRY(after_launch("scan_kernel"));
    scatter_kernel<<<tiles, kSortThreads, 0, stream>>>(ka, va, kb, vb, total, shift, hist, tiles);
    NPA_TRY(after_launch("scatter_kernel"));
    std::swap(ka, kb);
    std::swap(va, vb);
  }
  finalize_kernel<<<grid_for(total, 256), 256, 0, stream>>>(
      g, positions, ka, va, total, n, bins, out.bin_offsets, out.permutation, out.inverse,
      out.srec, out.scyz);
  NPA_TRY(after_launch("finalize_kernel"));
  if (!out.order) return NPA_OK;
  // The processing order: the sorted slots sorted again by (batch, cell-block
  // Morton code), in the same scratch.  The block edge 2^shift cells is chosen
  // from the grid's extent so that 64 blocks span a Particle-mode table's side
  // (or 16 in 3D): cfg1's 512 x 512 table -> blocks of 8 x 8 cells.
  const int axis_bits = g.dim == 2 ? 6 : 4;
  int shift = 0;
  while (shift < 16 && (uint64_t(1) << (axis_bits + shift)) < uint64_t(g.grid_size[0])) ++shift;
  const uint32_t obits = key_bits(uint64_t(batch) * kOrderCodes);
  const uint32_t opasses = (obits + 7) / 8;
  order_keys_kernel<<<tiles, kSortThreads, 0, stream>>>(g, out.srec, out.scyz, total, n, shift, ka,
                                                         va, hist, tiles);
  NPA_TRY(after_launch("order_keys_kernel"));
  for (uint32_t pass = 0; pass < opasses; ++pass) {
    const uint32_t sh = pass * 8;
    if (pass > 0) {
      hist_kernel<<<tiles, kSortThreads, 0, stream>>>(ka, total, sh, hist, tiles);
      NPA_TRY(after_launch("hist_kernel"));
    }
    scan_kernel<<<1, kScanThreads, 0, stream>>>(hist, tiles * kDigits);
    NPA_TRY(after_launch("scan_kernel"));
    scatter_kernel<<<tiles, kSortThreads, 0, stream>>>(ka, va, kb, vb, total, sh, hist, tiles);
    NPA_TRY(after_launch("scatter_kernel"));
    std::swap(ka, kb);
    std::swap(va, vb);
  }
  NPA_CUDA(cudaMemcpyAsync(out.order, va, size_t(total) * sizeof(uint32_t),
                           cudaMemcpyDeviceToDevice, stream),
           "cudaMemcpyAsync order");
  return NPA_OK;
}

// Only dense cells (mean bin occupancy >= 8, the warp-cooperative walks) gain
// more than the extra sort costs: cfg4 (4,194,304 clustered particles)
// perception 3.32 vs 3.70 s per step; cfg1 (1,048,576 uniform, ~4 per bin)
// 1.184 vs 1.262 ms but the order's sort adds 0.081 ms; cfg3 (16,384 on a
// torus) loses 0.02 ms.
bool hashgrid_orders(const GridParams& g, uint32_t batch, uint32_t n) {
  const uint64_t total = uint64_t(batch) * n;
  return total > 0 && !rollout_sort_fits(g, batch, n) && total >= uint64_t(8) * batch * g.cells;
}

// ---------------------------------------------------------------------------
// Hashgrid build that allocates nothing.
//
// Some callers cannot allocate device memory: a host that only holds buffers
// handed to it by another framework's allocator (a Burn / CubeCL tensor, a
// viewer's storage buffer) and owns no allocator of its own, or code that must
// not call cudaMalloc because of its implicit device synchronisation (a
// render or control loop with a latency budget).  For them the sort scratch
// lives in this fixed device array instead of a caller workspace.  The array
// exists once per device that loads the library and is held until exit, so it
// is sized for a modest maximum of kStaticMaxParticles particles (~6.3 MB).
// ---------------------------------------------------------------------------
namespace {

constexpr uint32_t kStaticMaxParticles = 1u << 17;  // batch * n limit (131,072)
constexpr size_t kStaticScratchBytes = size_t(6656) * 1024;  // 6.5 MiB

__device__ __align__(256) unsigned char g_hashgrid_static_scratch[kStaticScratchBytes];

// The array's address belongs to a CUDA context: after cudaDeviceReset, or
// with a caller-created (non-primary) context current, a cached address would
// be stale, so the cache is keyed on the current context, not the ordinal.
struct StaticAddress {
  int device;
  CUcontext ctx;
  void* ptr;
};
std::mutex g_static_mu;
std::vector<StaticAddress> g_static_addresses;

npa_status current_context(CUcontext* out) {
  using GetCurrent = CUresult (*)(CUcontext*);
  static GetCurrent fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    NPA_CUDA(cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q),
             "cudaGetDriverEntryPoint(cuCtxGetCurrent)");
    if (q != cudaDriverEntryPointSuccess || !p)
      return fail(NPA_ERR_CUDA, "cuCtxGetCurrent is not available");
    fn = reinterpret_cast<GetCurrent>(p);
  }
  if (fn(out) != CUDA_SUCCESS) return fail(NPA_ERR_CUDA, "cuCtxGetCurrent failed");
  return NPA_OK;
}

// Device address of the array in the current context, looked up once per
// (device, context) with that device current.  The first call on a device
// makes the CUDA runtime load this library's module there; make it before
// any stream capture on that device.
npa_status static_scratch_address(void** out) {
  int dev = 0;
  NPA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  CUcontext ctx = nullptr;
  NPA_TRY(current_context(&ctx));
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (ctx)
    for (const StaticAddress& a : g_static_addresses)
      if (a.device == dev && a.ctx == ctx) {
        *out = a.ptr;
        return NPA_OK;
      }
  void* p = nullptr;
  // Also makes the device's primary context current when none was.
  NPA_CUDA(cudaGetSymbolAddress(&p, g_hashgrid_static_scratch), "cudaGetSymbolAddress");
  NPA_TRY(current_context(&ctx));
  g_static_addresses.push_back(StaticAddress{dev, ctx, p});
  *out = p;
  return NPA_OK;
}

}  // namespace

// Launch plans: the dynamic shared memory limit is set and the occupancy
// queried once per (device, context, kernel, block size, shared memory); a
// host step makes tens of launches, and these runtime calls cost as much host
// time as the launches themselves.
namespace {
struct PlanKey {
  int device;
  CUcontext ctx;
  const void* kernel;
  int threads;
  size_t smem;
  int per_sm;
  int sms;
};
std::mutex g_plan_mu;
std::vector<PlanKey> g_plans;
}  // namespace

npa_status kernel_occupancy(const void* kernel, int threads, size_t smem, int* per_sm, int* sms) {
  int dev = 0;
  NPA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  CUcontext ctx = nullptr;
  NPA_TRY(current_context(&ctx));
  {
    std::lock_guard<std::mutex> lock(g_plan_mu);
    if (ctx)
      for (const PlanKey& k : g_plans)
        if (k.device == dev && k.ctx == ctx && k.kernel == kernel && k.threads == threads &&
            k.smem == smem) {
          *per_sm = k.per_sm;
          *sms = k.sms;
          return NPA_OK;
        }
  }
  int max_optin = 0, count = 0, blocks = 0;
  NPA_CUDA(cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev),
           "cudaDeviceGetAttribute");
  NPA_CUDA(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev),
           "cudaDeviceGetAttribute");
  if (smem > size_t(max_optin))
    return fail(NPA_ERR_UNSUPPORTED, "kernel needs more shared memory than a block has");
  // The limit only ever rises: launches planned earlier with more shared
  // memory keep theirs.
  size_t limit = smem;
  {
    std::lock_guard<std::mutex> lock(g_plan_mu);
    for (const PlanKey& k : g_plans)
      if (k.device == dev && k.ctx == ctx && k.kernel == kernel) limit = std::max(limit, k.smem);
  }
  NPA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(limit)),
           "cudaFuncSetAttribute");
  NPA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, smem),
           "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  NPA_TRY(current_context(&ctx));
  {
    std::lock_guard<std::mutex> lock(g_plan_mu);
    g_plans.push_back(PlanKey{dev, ctx, kernel, threads, smem, blocks, count});
  }
  *per_sm = blocks;
  *sms = count;
  return NPA_OK;
}

}  // namespace npa

extern "C" npa_status npa_dev_build_hashgrid_noalloc(const npa_grid_config* cfg,
                                                     const float* d_positions, int64_t batch,
                                                     int64_t n, uint32_t* d_bin_offsets,
                                                     uint32_t* d_permutation,
                                                     uint32_t* d_inverse_permutation,
                                                     void* stream) {
  using namespace npa;
  // The same checks, in the same order, as npa_dev_build_hashgrid (through
  // its workspace query); the only added status is NPA_ERR_UNSUPPORTED above
  // the fixed array's particle limit.
  size_t workspace_equivalent = 0;
  NPA_TRY(npa_dev_hashgrid_workspace_size(cfg, batch, n, &workspace_equivalent));
  if (batch > 0 && uint64_t(n) > kStaticMaxParticles / uint64_t(batch))
    return fail(NPA_ERR_UNSUPPORTED,
                "batch * particle_count = " + std::to_string(uint64_t(batch) * uint64_t(n)) +
                    " exceeds the allocation-free hashgrid limit of " +
                    std::to_string(kStaticMaxParticles) + " particles");
  const GridParams g = make_grid_params(*cfg);
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  if (!d_bin_offsets || (total > 0 && (!d_positions || !d_permutation || !d_inverse_permutation)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  void* base = nullptr;
  NPA_TRY(static_scratch_address(&base));
  Carve c(base, kStaticScratchBytes);
  HashgridBuffers hb;
  hb.bin_offsets = d_bin_offsets;
  hb.permutation = d_permutation;
  hb.inverse = d_inverse_permutation;
  hb.srec = c.take<float4>(total);
  hb.scyz = c.take<int2>(total);
  const size_t sb = hashgrid_scratch_bytes(g, B, N);
  char* scratch = c.take<char>(sb);
  if (!c.fits()) return fail(NPA_ERR_UNSUPPORTED, "allocation-free hashgrid scratch is too small");
  return launch_hashgrid(g, reinterpret_cast<const float4*>(d_positions), B, N, hb, scratch, sb,
                         static_cast<cudaStream_t>(stream));
}
