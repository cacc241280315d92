// capi.cu -- the extern "C" boundary (include/npa_b200.h).
//
// Validation mirrors the reference's checks and their order:
//   HashGridConfig::validate       crates/burn_automata_kernels/src/config.rs:65-84
//   check_shapes                   crates/burn_automata_kernels/src/reference/shape.rs:3-25
//   euler_step shape checks        crates/burn_automata_kernels/src/reference/step.rs:16-27
//   NpaModel::validate / weights   crates/burn_automata/src/model.rs:77-107, :757-766
//   step_cpu grid/model dim check  crates/burn_automata/src/model.rs:778-784
// Everything is checked before the first CUDA call, so a bad argument is
// reported the same way with or without a GPU.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "npa_internal.h"

namespace npa {

static thread_local std::string g_last_error;
static thread_local npa_error_detail g_last_detail{};
static std::atomic<uint64_t> g_launches{0};

void set_error(const std::string& msg) { g_last_error = msg; }

npa_status fail(npa_status st, const std::string& msg) {
  set_error(msg);
  g_last_detail = npa_error_detail{st, 0.0f, 0, 0};
  return st;
}

// fail() with the payload the reference's KernelError variant carries.
npa_status fail_with(npa_status st, const std::string& msg, int64_t a, int64_t b = 0,
                     float eps = 0.0f) {
  set_error(msg);
  g_last_detail = npa_error_detail{st, eps, a, b};
  return st;
}

npa_status cuda_fail(cudaError_t err, const char* what) {
  set_error(std::string(what) + ": " + cudaGetErrorString(err));
  if (err == cudaErrorMemoryAllocation) return NPA_ERR_OUT_OF_MEMORY;
  if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver) return NPA_ERR_NO_DEVICE;
  return NPA_ERR_CUDA;
}

npa_status after_launch(const char* kernel, int launches) {
  g_launches.fetch_add(static_cast<uint64_t>(launches), std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, kernel);
  return NPA_OK;
}

static float powi_f32(float x, int n) {
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

npa_status validate_grid(const npa_grid_config* cfg) {
  if (!cfg) return fail(NPA_ERR_INVALID_ARGUMENT, "grid config is null");
  if (!(cfg->dim == 2 || cfg->dim == 3))
    return fail_with(NPA_ERR_INVALID_DIM,
                     "expected spatial dim 2 or 3, got " + std::to_string(cfg->dim), cfg->dim);
  if (!std::isfinite(cfg->eps) || cfg->eps <= 0.0f)
    return fail_with(NPA_ERR_INVALID_EPS,
                     "eps must be finite and positive, got " + std::to_string(cfg->eps), 0, 0,
                     cfg->eps);
  if (!(cfg->mode == NPA_MODE_GRID || cfg->mode == NPA_MODE_PARTICLE))
    return fail(NPA_ERR_INVALID_ARGUMENT, "unknown hashgrid mode");
  if (!(cfg->boundary == NPA_BOUNDARY_PERIODIC || cfg->boundary == NPA_BOUNDARY_CLAMPED))
    return fail(NPA_ERR_INVALID_ARGUMENT, "unknown boundary");
  for (int axis = 0; axis < cfg->dim; ++axis) {
    const int64_t s = cfg->grid_size[axis];
    if (s <= 0) return fail(NPA_ERR_INVALID_GRID_SIZE, "grid sizes must be non-zero for active dimensions");
    if (cfg->mode == NPA_MODE_PARTICLE && (s & (s - 1)) != 0)
      return fail_with(NPA_ERR_PARTICLE_MODE_REQUIRES_POW2,
                       "particle hashgrid mode requires power-of-two grid size at axis " +
                           std::to_string(axis) + ", got " + std::to_string(s),
                       axis, s);
  }
  int64_t cells = 1;
  for (int axis = 0; axis < cfg->dim; ++axis) {
    if (cfg->grid_size[axis] > (int64_t(1) << 30))
      return fail(NPA_ERR_UNSUPPORTED, "grid size above 2^30 on one axis");
    cells *= cfg->grid_size[axis];
    if (cells > (int64_t(1) << 31)) return fail(NPA_ERR_UNSUPPORTED, "cell count above 2^31");
  }
  return NPA_OK;
}

GridParams make_grid_params(const npa_grid_config& cfg) {
  GridParams g{};
  g.dim = cfg.dim;
  g.boundary = cfg.boundary;
  g.mode = cfg.mode;
  uint64_t cells = 1;
  for (int a = 0; a < 3; ++a) {
    g.grid_size[a] = a < cfg.dim ? static_cast<int>(cfg.grid_size[a]) : 1;
    if (a < cfg.dim) cells *= static_cast<uint64_t>(cfg.grid_size[a]);
  }
  g.cells = static_cast<uint32_t>(cells);
  g.cells_mask = (g.cells & (g.cells - 1)) == 0 ? g.cells - 1 : 0u;
  g.eps = cfg.eps;
  g.eps2 = cfg.eps * cfg.eps;
  for (int a = 0; a < 3; ++a) {
    // `grid_size as f32 * eps` (hashgrid.rs:170) == `eps * size as f32` (:80).
    g.extent[a] = static_cast<float>(a < cfg.dim ? cfg.grid_size[a] : 1) * cfg.eps;
    g.half[a] = g.extent[a] * 0.5f;
  }
  const float pi = 3.14159274101257324219f;  // std::f32::consts::PI
  if (cfg.dim == 2) {
    g.poly6_norm = 4.0f / (pi * powi_f32(cfg.eps, 8));
    g.spiky_norm = 10.0f / (pi * powi_f32(cfg.eps, 5));
  } else {
    g.poly6_norm = 315.0f / (64.0f * pi * powi_f32(cfg.eps, 9));
    g.spiky_norm = 15.0f / (pi * powi_f32(cfg.eps, 6));
  }
  return g;
}

}  // namespace npa

using namespace npa;

// ---------------------------------------------------------------------------
// small host helpers
// ---------------------------------------------------------------------------
namespace {

constexpr uint64_t kMaxParticles = (uint64_t(1) << 31);

npa_status check_counts(int64_t batch, int64_t n) {
  if (batch < 0 || n < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "batch and particle count must be >= 0");
  if (batch > 0 && uint64_t(n) > kMaxParticles / uint64_t(batch))
    return fail(NPA_ERR_UNSUPPORTED, "batch * particle_count above 2^31");
  return NPA_OK;
}

npa_status check_bins(const npa_grid_config* cfg, int64_t batch) {
  int64_t cells = 1;
  for (int a = 0; a < cfg->dim; ++a) cells *= cfg->grid_size[a];
  if (batch > 0 && uint64_t(cells) > (uint64_t(0xFFFFFFFEu) / uint64_t(batch)))
    return fail(NPA_ERR_UNSUPPORTED, "batch * cell_count + 1 does not fit in uint32");
  return NPA_OK;
}

// check_shapes (shape.rs:3-25).
npa_status check_shapes(int64_t positions_len, int64_t states_len, int64_t batch, int64_t n,
                        int64_t c) {
  const int64_t expected = batch * n;
  if (positions_len != expected)
    return fail_with(NPA_ERR_POSITION_SHAPE, "positions length " + std::to_string(positions_len) +
                                                 " does not match batch_size * particle_count " +
                                                 std::to_string(expected),
                     positions_len, expected);
  if (states_len != expected * c)
    return fail_with(NPA_ERR_STATE_SHAPE, "state length " + std::to_string(states_len) +
                                              " does not match batch_size * particle_count * state_dims " +
                                              std::to_string(expected * c),
                     states_len, expected * c);
  return NPA_OK;
}

npa_status output_shape(int64_t actual, int64_t expected) {
  if (actual != expected)
    return fail_with(NPA_ERR_OUTPUT_SHAPE, "output buffer length " + std::to_string(actual) +
                                               " does not match expected " + std::to_string(expected),
                     actual, expected);
  return NPA_OK;
}

npa_status ensure_device(int device) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(NPA_ERR_NO_DEVICE, std::string("no CUDA device: ") +
                                       (e != cudaSuccess ? cudaGetErrorString(e) : "count is 0"));
  }
  if (device < 0 || device >= count) return fail(NPA_ERR_INVALID_ARGUMENT, "device ordinal out of range");
  NPA_CUDA(cudaSetDevice(device), "cudaSetDevice");
  return NPA_OK;
}

npa_status current_device(int* device) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(NPA_ERR_NO_DEVICE, "no CUDA device");
  }
  NPA_CUDA(cudaGetDevice(device), "cudaGetDevice");
  return NPA_OK;
}

// Optional test hook: total bytes the host-buffer entry points may allocate
// per call (0 = unlimited).  Exercises the out-of-memory path without
// exhausting a device.
std::atomic<uint64_t> g_alloc_cap{0};

// Device blocks released by host-buffer calls, kept per device (up to
// kCacheBytes) and handed to later calls of a similar size, so a loop of
// host-buffer calls does not pay cudaMalloc / cudaFree every time.
struct BlockCache {
  std::mutex mu;
  std::multimap<size_t, std::pair<int, void*>> blocks;  // size -> (device, pointer)
  size_t bytes = 0;
};
constexpr size_t kCacheBytes = size_t(8) << 30;

BlockCache& block_cache() {
  static BlockCache* c = new BlockCache();  // never destroyed: no frees after the driver unloads
  return *c;
}

// A cached block of at least `bytes` (and at most twice that) on `dev`.
void* cache_take(int dev, size_t bytes, size_t* got) {
  BlockCache& c = block_cache();
  std::lock_guard<std::mutex> lock(c.mu);
  for (auto it = c.blocks.lower_bound(bytes); it != c.blocks.end() && it->first <= 2 * bytes; ++it) {
    if (it->second.first != dev) continue;
    void* p = it->second.second;
    *got = it->first;
    c.bytes -= it->first;
    c.blocks.erase(it);
    return p;
  }
  return nullptr;
}

// Frees every cached block of `dev` (before retrying an allocation that failed).
void cache_release(int dev) {
  BlockCache& c = block_cache();
  std::lock_guard<std::mutex> lock(c.mu);
  for (auto it = c.blocks.begin(); it != c.blocks.end();) {
    if (it->second.first == dev) {
      cudaFree(it->second.second);
      c.bytes -= it->first;
      it = c.blocks.erase(it);
    } else {
      ++it;
    }
  }
}

// cudaMalloc that drops the cached blocks of the device and retries once
// when the device is out of memory.
cudaError_t malloc_or_release(void** p, size_t bytes, int dev) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    cache_release(dev);
    e = cudaMalloc(p, bytes);
  }
  return e;
}

void cache_give(int dev, void* p, size_t bytes) {
  BlockCache& c = block_cache();
  {
    std::lock_guard<std::mutex> lock(c.mu);
    if (c.bytes + bytes <= kCacheBytes) {
      c.blocks.emplace(bytes, std::make_pair(dev, p));
      c.bytes += bytes;
      return;
    }
  }
  cudaFree(p);
}

// Device scratch of one host-buffer call, returned to the block cache on
// scope exit (after the call's stream has drained).
struct Scratch {
  std::vector<std::pair<void*, size_t>> ptrs;
  uint64_t bytes = 0;
  int device = 0;
  cudaStream_t stream = nullptr;
  ~Scratch() {
    if (stream) cudaStreamSynchronize(stream);
    for (auto& b : ptrs) cache_give(device, b.first, b.second);
    if (stream) cudaStreamDestroy(stream);
  }
  npa_status init() {
    NPA_CUDA(cudaGetDevice(&device), "cudaGetDevice");
    NPA_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    return NPA_OK;
  }
  template <class T>
  npa_status alloc(T** out, size_t count) {
    *out = nullptr;
    const size_t b = (std::max<size_t>(count * sizeof(T), 256) + 255) & ~size_t(255);
    const uint64_t cap = g_alloc_cap.load();
    if (cap && bytes + b > cap) return fail(NPA_ERR_OUT_OF_MEMORY, "allocation cap reached");
    size_t got = b;
    void* p = cache_take(device, b, &got);
    if (!p) NPA_CUDA(malloc_or_release(&p, b, device), "cudaMalloc");
    ptrs.emplace_back(p, got);
    bytes += b;
    *out = static_cast<T*>(p);
    return NPA_OK;
  }
  template <class T>
  npa_status upload(T** out, const void* host, size_t count) {
    NPA_TRY(alloc(out, count));
    if (count)
      NPA_CUDA(cudaMemcpyAsync(*out, host, count * sizeof(T), cudaMemcpyHostToDevice, stream),
               "cudaMemcpyAsync H2D");
    return NPA_OK;
  }
  npa_status download(void* host, const void* dev, size_t bytes_) {
    if (bytes_ && host)
      NPA_CUDA(cudaMemcpyAsync(host, dev, bytes_, cudaMemcpyDeviceToHost, stream),
               "cudaMemcpyAsync D2H");
    return NPA_OK;
  }
  npa_status finish() {
    NPA_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    return NPA_OK;
  }
};

// Layout of the workspace behind the device perception / step entry points.
struct PerceiveWorkspace {
  HashgridBuffers hg;
  float* volume;
  void* sort_scratch;
  size_t sort_scratch_bytes;
  float* tiles;  // step path only: feature tiles [tiles][F][tile_rows]
  HitLists hits; // neighbour hits recorded by the density pass
};

// Hits kept per particle by the density pass (a particle with more is walked
// again by the perception kernels).
constexpr int kHitCap = 32;

size_t tiles_floats(uint32_t batch, uint32_t n, int feature_dims, int tile_rows) {
  if (tile_rows <= 0) return 0;
  const size_t total = size_t(batch) * n;
  const size_t padded = (total + tile_rows - 1) / tile_rows * size_t(tile_rows);
  return padded * size_t(feature_dims);
}

// with_order: room for the processing order of the neighbour walks (the
// caller passes hashgrid_orders(g, batch, n)).
size_t perceive_workspace_bytes(const GridParams& g, uint32_t batch, uint32_t n,
                                size_t extra_floats = 0, bool with_order = false) {
  const size_t total = size_t(batch) * n;
  Carve c(nullptr, 0);
  c.take<uint32_t>(size_t(batch) * g.cells + 1);
  c.take<uint32_t>(total);
  c.take<uint32_t>(total);
  c.take<float4>(total);
  c.take<int2>(total);
  c.take<float>(total);
  c.take<uint32_t>(total * kHitCap);
  c.take<uint32_t>(total);
  const size_t sort = hashgrid_scratch_bytes(g, batch, n);
  c.take<char>(sort);
  c.take<float>(extra_floats);
  if (with_order) c.take<uint32_t>(total);
  return c.used + 256;
}

bool carve_perceive(const GridParams& g, uint32_t batch, uint32_t n, void* ws, size_t bytes,
                    PerceiveWorkspace* out, size_t extra_floats = 0, bool with_order = false) {
  const size_t total = size_t(batch) * n;
  Carve c(ws, bytes);
  out->hg.bin_offsets = c.take<uint32_t>(size_t(batch) * g.cells + 1);
  out->hg.permutation = c.take<uint32_t>(total);
  out->hg.inverse = c.take<uint32_t>(total);
  out->hg.srec = c.take<float4>(total);
  out->hg.scyz = c.take<int2>(total);
  out->volume = c.take<float>(total);
  out->hits.slots = c.take<uint32_t>(total * kHitCap);
  out->hits.count = c.take<uint32_t>(total);
  out->hits.cap = kHitCap;
  out->hits.stride = static_cast<uint32_t>(total);
  out->sort_scratch_bytes = hashgrid_scratch_bytes(g, batch, n);
  out->sort_scratch = c.take<char>(out->sort_scratch_bytes);
  out->tiles = extra_floats ? c.take<float>(extra_floats) : nullptr;
  out->hg.order = with_order ? c.take<uint32_t>(total) : nullptr;
  return c.fits();
}

SortedGrid sorted_view(const PerceiveWorkspace& w, uint32_t n, uint32_t batch,
                       const float* positions) {
  SortedGrid s;
  s.bin_offsets = w.hg.bin_offsets;
  s.permutation = w.hg.permutation;
  s.srec = w.hg.srec;
  s.scyz = w.hg.scyz;
  s.positions = reinterpret_cast<const float4*>(positions);
  s.order = w.hg.order;
  s.n = n;
  s.total = n * batch;
  return s;
}

npa_status validate_decode(const npa_gaussian_decode_config* cfg, int64_t c) {
  if (!cfg) return fail(NPA_ERR_INVALID_ARGUMENT, "decode config is null");
  if (cfg->mode < 0 || cfg->mode > 3) return fail(NPA_ERR_INVALID_ARGUMENT, "unknown decode mode");
  if (cfg->sh_degree < 0 || cfg->sh_degree > 8) return fail(NPA_ERR_INVALID_ARGUMENT, "sh_degree out of range");
  const int64_t k = cfg->mode == NPA_DECODE_SH0_ORIENTED ? int64_t(cfg->sh_degree + 1) * (cfg->sh_degree + 1) : 1;
  // validate_decode_layout (gaussian.rs:102-125), an assert! in the reference.
  if ((cfg->mode <= NPA_DECODE_SH0_FIXED_SCALE && c < 3) ||
      (cfg->mode == NPA_DECODE_SH0_LEARNED_SCALE && c < 5) ||
      (cfg->mode == NPA_DECODE_SH0_ORIENTED && c < k * 3 + 8))
    return fail(NPA_ERR_STATE_SHAPE, "state_dims too small for the decode mode's tail channels");
  // f32::clamp asserts min <= max (NaN bounds fail the assert too).
  if (!(cfg->min_scale <= cfg->max_scale) || !(cfg->min_opacity <= cfg->max_opacity))
    return fail(NPA_ERR_INVALID_ARGUMENT, "decode clamp bounds are inverted or NaN");
  return NPA_OK;
}

int64_t record_floats(const npa_gaussian_decode_config* cfg) {
  const int64_t k = cfg->mode == NPA_DECODE_SH0_ORIENTED ? int64_t(cfg->sh_degree + 1) * (cfg->sh_degree + 1) : 1;
  return 12 + 3 * k;
}

}  // namespace

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
// Device buffers and the stream behind a model's host-buffer step calls:
// kept between calls (grown on demand, freed with the model), so a loop of
// host-buffer steps pays for its copies and kernels, not for allocations.
// Device memory and streams of the host-buffer entry points.  `stream` runs
// the kernels; the pipelined step adds a copy-in and a copy-out stream and
// two events per rollout chunk.
struct HostArena {
  void* base = nullptr;
  size_t cap = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t stream2 = nullptr;  // second compute stream of the chunk pipeline
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  std::vector<cudaEvent_t> events;
};

struct npa_model {
  DeviceModel dm{};
  npa_model_config cfg{};
  std::mutex mu;
  HostArena arena;
};

namespace {

int64_t model_perception_dims(const npa_model_config& c) {
  return int64_t(c.state_dims) * 2 + (c.state_grad ? int64_t(c.state_dims) * c.spatial_dims : 0) +
         (c.density_grad ? c.spatial_dims : 0) + (c.position_features ? c.spatial_dims : 0) +
         c.auxiliary_input_dims;
}

npa_perception_options model_options(const npa_model_config& c) {
  npa_perception_options o{};
  o.state_grad = c.state_grad;
  o.density_grad = c.density_grad;
  o.scale_equivariance = c.equivariance == NPA_EQUIV_PARTICLE_DENSITY_AND_SCALE;
  o.particle_density_equivariance = c.equivariance == NPA_EQUIV_PARTICLE_DENSITY ||
                                    c.equivariance == NPA_EQUIV_PARTICLE_DENSITY_AND_SCALE;
  o.log_norm_grad = c.log_norm_grad;
  o.log_norm_density_grad = c.log_norm_density_grad;
  o.hybrid_state_gradient = 1;  // step_cpu always sets it (model.rs:800)
  o.position_features = c.position_features;
  o.eps0 = c.eps0;
  return o;
}

// step_cpu's checks (model.rs:778-784) plus the 3D gate channel requirement.
npa_status check_step(const npa_model* m, const npa_grid_config* grid) {
  NPA_TRY(validate_grid(grid));
  if (grid->dim != m->cfg.spatial_dims)
    return fail(NPA_ERR_INVALID_ARGUMENT, "grid dim does not match model spatial dims");
  if (grid->dim == 3 && m->cfg.position_features && m->cfg.state_dims > 3 &&
      m->cfg.state_dims <= 7)
    return fail(NPA_ERR_INVALID_ARGUMENT,
                "3D position gates read state channel 7; state_dims must exceed 7");
  return NPA_OK;
}

}  // namespace

extern "C" {

int32_t npa_abi_version(void) { return NPA_ABI_VERSION; }

const char* npa_status_string(npa_status status) {
  switch (status) {
    case NPA_OK: return "ok";
    case NPA_ERR_INVALID_DIM: return "invalid dim";
    case NPA_ERR_INVALID_EPS: return "invalid eps";
    case NPA_ERR_INVALID_GRID_SIZE: return "invalid grid size";
    case NPA_ERR_PARTICLE_MODE_REQUIRES_POW2: return "particle mode requires power-of-two grid size";
    case NPA_ERR_POSITION_SHAPE: return "position shape";
    case NPA_ERR_STATE_SHAPE: return "state shape";
    case NPA_ERR_OUTPUT_SHAPE: return "output shape";
    case NPA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NPA_ERR_INVALID_MODEL: return "invalid model";
    case NPA_ERR_CUDA: return "cuda error";
    case NPA_ERR_DEVICE_STATUS: return "device status error";
    case NPA_ERR_TIMEOUT: return "device wait timed out";
    case NPA_ERR_OUT_OF_MEMORY: return "out of memory";
    case NPA_ERR_UNSUPPORTED: return "unsupported";
    case NPA_ERR_NO_DEVICE: return "no device";
    default: return "unknown status";
  }
}

const char* npa_last_error_message(void) { return g_last_error.c_str(); }

npa_status npa_last_error_detail(npa_error_detail* out) {
  if (!out) return NPA_ERR_INVALID_ARGUMENT;
  *out = g_last_detail;
  return NPA_OK;
}

uint64_t npa_kernel_launch_count(void) { return g_launches.load(); }

uint64_t npa_bulk_copy_timeouts(void) { return bulk_copy_timeouts() + ws_step_timeouts(); }

npa_status npa_prepare_host_tables(int64_t* ln_1p_exceptions) {
  NPA_TRY(prepare_host_log1p());
  if (ln_1p_exceptions) *ln_1p_exceptions = int64_t(host_log1p_exceptions());
  return NPA_OK;
}

npa_status npa_prepare_device(int32_t device) {
  NPA_TRY(ensure_device(device));
  Log1pTable l1p;
  return device_log1p_table(&l1p);
}

npa_status npa_dev_ln_1p(const float* d_x, int64_t count, float* d_out, void* stream) {
  if (count < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "count must be >= 0");
  if (count > 0 && (!d_x || !d_out)) return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  return launch_ln_1p(d_x, uint64_t(count), d_out, static_cast<cudaStream_t>(stream));
}

// Test hook for the out-of-memory path of the host-buffer entry points.
void npa_debug_set_allocation_cap(uint64_t bytes) { g_alloc_cap.store(bytes); }

npa_status npa_grid_validate(const npa_grid_config* cfg) { return validate_grid(cfg); }

npa_status npa_grid_cell_count(const npa_grid_config* cfg, int64_t* cell_count) {
  NPA_TRY(validate_grid(cfg));
  if (!cell_count) return fail(NPA_ERR_INVALID_ARGUMENT, "null output");
  int64_t c = 1;
  for (int a = 0; a < cfg->dim; ++a) c *= cfg->grid_size[a];
  *cell_count = c;
  return NPA_OK;
}

npa_status npa_feature_dims(const npa_grid_config* cfg, const npa_perception_options* o,
                            int64_t state_dims, int64_t* feature_dims) {
  NPA_TRY(validate_grid(cfg));
  if (!o || !feature_dims || state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "bad argument");
  *feature_dims = state_dims * 2 + (o->state_grad ? state_dims * cfg->dim : 0) +
                  (o->density_grad ? cfg->dim : 0) + (o->position_features ? cfg->dim : 0);
  return NPA_OK;
}

npa_status npa_gaussian_record_floats(const npa_gaussian_decode_config* cfg, int64_t* floats) {
  if (!cfg || !floats) return fail(NPA_ERR_INVALID_ARGUMENT, "null argument");
  if (cfg->mode < 0 || cfg->mode > 3 || cfg->sh_degree < 0 || cfg->sh_degree > 8)
    return fail(NPA_ERR_INVALID_ARGUMENT, "bad decode config");
  *floats = record_floats(cfg);
  return NPA_OK;
}

// ---- host-buffer operators ----

npa_status npa_build_hashgrid(const npa_grid_config* cfg, const float* positions,
                              int64_t positions_len, int64_t batch, int64_t n,
                              uint32_t* bin_offsets, int64_t bin_offsets_len,
                              uint32_t* permutation, uint32_t* inverse_permutation,
                              int64_t permutation_len) {
  NPA_TRY(validate_grid(cfg));
  NPA_TRY(check_counts(batch, n));
  if (positions_len != batch * n)
    return fail_with(NPA_ERR_POSITION_SHAPE,
                     "positions length " + std::to_string(positions_len) +
                         " does not match batch_size * particle_count " + std::to_string(batch * n),
                     positions_len, batch * n);
  NPA_TRY(check_bins(cfg, batch));
  const GridParams g = make_grid_params(*cfg);
  NPA_TRY(output_shape(bin_offsets_len, batch * int64_t(g.cells) + 1));
  NPA_TRY(output_shape(permutation_len, batch * n));
  if ((batch * n > 0 && (!positions || !permutation || !inverse_permutation)) || !bin_offsets)
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  int dev = 0;
  NPA_TRY(current_device(&dev));
  Scratch s;
  NPA_TRY(s.init());
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  float4* dpos;
  NPA_TRY(s.upload(&dpos, positions, total));
  HashgridBuffers hb;
  NPA_TRY(s.alloc(&hb.bin_offsets, size_t(B) * g.cells + 1));
  NPA_TRY(s.alloc(&hb.permutation, total));
  NPA_TRY(s.alloc(&hb.inverse, total));
  NPA_TRY(s.alloc(&hb.srec, total));
  NPA_TRY(s.alloc(&hb.scyz, total));
  const size_t sb = hashgrid_scratch_bytes(g, B, N);
  char* scratch;
  NPA_TRY(s.alloc(&scratch, sb));
  NPA_TRY(launch_hashgrid(g, dpos, B, N, hb, scratch, sb, s.stream));
  NPA_TRY(s.download(bin_offsets, hb.bin_offsets, (size_t(B) * g.cells + 1) * 4));
  NPA_TRY(s.download(permutation, hb.permutation, size_t(total) * 4));
  NPA_TRY(s.download(inverse_permutation, hb.inverse, size_t(total) * 4));
  return s.finish();
}

npa_status npa_perceive_with_options(const npa_grid_config* cfg, const npa_perception_options* o,
                                     const float* positions, int64_t positions_len,
                                     const float* states, int64_t states_len, int64_t batch,
                                     int64_t n, int64_t state_dims, float* features,
                                     int64_t features_len, float* density, float* blurred_state,
                                     float* state_gradient, float* density_gradient) {
  if (!o) return fail(NPA_ERR_INVALID_ARGUMENT, "options are null");
  NPA_TRY(check_counts(batch, n));
  if (state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "state_dims must be >= 0");
  NPA_TRY(check_shapes(positions_len, states_len, batch, n, state_dims));
  NPA_TRY(validate_grid(cfg));
  NPA_TRY(check_bins(cfg, batch));
  const GridParams g = make_grid_params(*cfg);
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  const PerceptionParams p = make_perception_params(g, *o, N, int(state_dims));
  NPA_TRY(output_shape(features_len, int64_t(total) * p.feature_dims));
  if (total > 0 && (!positions || (state_dims > 0 && !states) || (p.feature_dims > 0 && !features)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  int dev = 0;
  NPA_TRY(current_device(&dev));
  Scratch s;
  NPA_TRY(s.init());
  float4* dpos;
  float* dst;
  NPA_TRY(s.upload(&dpos, positions, total));
  NPA_TRY(s.upload(&dst, states, size_t(total) * state_dims));
  const size_t wsb = perceive_workspace_bytes(g, B, N, 0, hashgrid_orders(g, B, N));
  char* ws;
  NPA_TRY(s.alloc(&ws, wsb));
  float *dfeat, *ddens = nullptr, *dblur = nullptr, *dsg = nullptr, *ddg = nullptr;
  NPA_TRY(s.alloc(&dfeat, size_t(total) * p.feature_dims));
  if (density) NPA_TRY(s.alloc(&ddens, total));
  if (blurred_state) NPA_TRY(s.alloc(&dblur, size_t(total) * state_dims));
  if (state_gradient && p.state_grad) NPA_TRY(s.alloc(&dsg, size_t(total) * state_dims * g.dim));
  if (density_gradient && p.density_grad) NPA_TRY(s.alloc(&ddg, size_t(total) * g.dim));
  NPA_TRY(npa_dev_perceive_with_options(cfg, o, reinterpret_cast<float*>(dpos), dst, batch, n,
                                        state_dims, dfeat, ddens, dblur, dsg, ddg, ws, wsb,
                                        s.stream));
  NPA_TRY(s.download(features, dfeat, size_t(total) * p.feature_dims * 4));
  NPA_TRY(s.download(density, ddens, size_t(total) * 4 * (ddens != nullptr)));
  NPA_TRY(s.download(blurred_state, dblur, size_t(total) * state_dims * 4 * (dblur != nullptr)));
  NPA_TRY(s.download(state_gradient, dsg, size_t(total) * state_dims * g.dim * 4 * (dsg != nullptr)));
  NPA_TRY(s.download(density_gradient, ddg, size_t(total) * g.dim * 4 * (ddg != nullptr)));
  return s.finish();
}

npa_status npa_euler_step(const npa_grid_config* cfg, const float* positions,
                          int64_t positions_len, const float* states, int64_t states_len,
                          const float* dx, int64_t dx_len, const float* ds, int64_t ds_len,
                          int64_t batch, int64_t n, int64_t state_dims, float dt,
                          const float* update_mask, float* next_positions, float* next_states) {
  NPA_TRY(check_counts(batch, n));
  if (state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "state_dims must be >= 0");
  NPA_TRY(check_shapes(positions_len, states_len, batch, n, state_dims));
  NPA_TRY(output_shape(dx_len, positions_len));
  NPA_TRY(output_shape(ds_len, states_len));
  NPA_TRY(validate_grid(cfg));
  const uint32_t total = uint32_t(batch * n);
  if (total > 0 && (!positions || !dx || !next_positions ||
                    (state_dims > 0 && (!states || !ds || !next_states))))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  const GridParams g = make_grid_params(*cfg);
  int dev = 0;
  NPA_TRY(current_device(&dev));
  Scratch s;
  NPA_TRY(s.init());
  float4 *dpos, *ddx, *dnp;
  float *dst, *dds, *dns, *dmask = nullptr;
  NPA_TRY(s.upload(&dpos, positions, total));
  NPA_TRY(s.upload(&dst, states, size_t(total) * state_dims));
  NPA_TRY(s.upload(&ddx, dx, total));
  NPA_TRY(s.upload(&dds, ds, size_t(total) * state_dims));
  if (update_mask) NPA_TRY(s.upload(&dmask, update_mask, total));
  NPA_TRY(s.alloc(&dnp, total));
  NPA_TRY(s.alloc(&dns, size_t(total) * state_dims));
  NPA_TRY(launch_euler(g, dpos, dst, ddx, dds, total, int(state_dims), dt, dmask, dnp, dns,
                       s.stream));
  NPA_TRY(s.download(next_positions, dnp, size_t(total) * 16));
  NPA_TRY(s.download(next_states, dns, size_t(total) * state_dims * 4));
  return s.finish();
}

npa_status npa_decode_gaussians_3d(const npa_gaussian_decode_config* cfg, const float* positions,
                                   int64_t positions_len, const float* states,
                                   int64_t states_len, int64_t state_dims, float* out,
                                   int64_t out_len) {
  if (positions_len < 0 || state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "negative length");
  // assert_eq!(positions.len() * state_dims, states.len()) (gaussian.rs:59)
  if (positions_len * state_dims != states_len)
    return fail_with(NPA_ERR_STATE_SHAPE,
                     "states length " + std::to_string(states_len) +
                         " does not match positions * state_dims " +
                         std::to_string(positions_len * state_dims),
                     states_len, positions_len * state_dims);
  NPA_TRY(validate_decode(cfg, state_dims));
  if (positions_len > int64_t(kMaxParticles)) return fail(NPA_ERR_UNSUPPORTED, "too many particles");
  NPA_TRY(output_shape(out_len, positions_len * record_floats(cfg)));
  const uint32_t count = uint32_t(positions_len);
  if (count > 0 && (!positions || !states || !out)) return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  int dev = 0;
  NPA_TRY(current_device(&dev));
  Scratch s;
  NPA_TRY(s.init());
  float4* dpos;
  float *dst, *dout;
  NPA_TRY(s.upload(&dpos, positions, count));
  NPA_TRY(s.upload(&dst, states, size_t(count) * state_dims));
  NPA_TRY(s.alloc(&dout, size_t(out_len)));
  NPA_TRY(launch_decode(*cfg, dpos, dst, count, int(state_dims), dout, s.stream));
  NPA_TRY(s.download(out, dout, size_t(out_len) * 4));
  return s.finish();
}

// ---- model ----

npa_status npa_model_create(const npa_model_config* cfg, const float* w1, int64_t w1_len,
                            const float* b1, int64_t b1_len, const float* w2, int64_t w2_len,
                            const float* b2, int64_t b2_len, int32_t device, npa_model** out) {
  if (!cfg || !out) return fail(NPA_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  // NpaModel::validate (model.rs:757-766) then NpaWeights::validate (:77-107).
  if (!(cfg->spatial_dims == 2 || cfg->spatial_dims == 3))
    return fail(NPA_ERR_INVALID_MODEL, "spatial_dims must be 2 or 3");
  if (cfg->state_dims < 0 || cfg->hidden_dims <= 0 || cfg->auxiliary_input_dims < 0)
    return fail(NPA_ERR_INVALID_MODEL, "state_dims, hidden_dims and auxiliary_input_dims must be non-negative");
  if (!(cfg->equivariance >= 0 && cfg->equivariance <= 2))
    return fail(NPA_ERR_INVALID_MODEL, "unknown equivariance mode");
  const int64_t F = model_perception_dims(*cfg);
  const int64_t H = cfg->hidden_dims;
  const int64_t O = int64_t(cfg->spatial_dims) + cfg->state_dims;
  if (w1_len != H * F) return fail(NPA_ERR_INVALID_MODEL, "w1 len " + std::to_string(w1_len) + " != " + std::to_string(H * F));
  if (b1_len != H) return fail(NPA_ERR_INVALID_MODEL, "b1 len " + std::to_string(b1_len) + " != " + std::to_string(H));
  if (w2_len != O * H) return fail(NPA_ERR_INVALID_MODEL, "w2 len " + std::to_string(w2_len) + " != " + std::to_string(O * H));
  if (b2_len != O) return fail(NPA_ERR_INVALID_MODEL, "b2 len " + std::to_string(b2_len) + " != " + std::to_string(O));
  if (!w1 || !b1 || !w2 || !b2) return fail(NPA_ERR_INVALID_ARGUMENT, "null weights");
  if (cfg->auxiliary_input_dims != 0)
    return fail(NPA_ERR_UNSUPPORTED, "auxiliary input dims are not part of the rollout step");
  if (H > 256) return fail(NPA_ERR_UNSUPPORTED, "hidden_dims above 256 is not supported");
  {
    DeviceModel probe{};
    probe.state_dims = cfg->state_dims;
    probe.hidden_dims = int(H);
    probe.feature_dims = int(F);
    probe.update_dims = int(O);
    probe.hidden_padded = hidden_padded_for(int(H));
    if (!mlp_step_supported(probe))
      return fail(NPA_ERR_UNSUPPORTED, "update dims too large for the MLP's hidden width");
  }
  NPA_TRY(ensure_device(device));
  if (cfg->log_norm_grad || cfg->log_norm_density_grad) {
    // the log-normalisation's log1pf tables, uploaded now so that later steps
    // (and executor graph captures) find them on the device
    Log1pTable l1p;
    NPA_TRY(device_log1p_table(&l1p));
  }
  const int64_t Hp = hidden_padded_for(int(H));
  std::vector<float> w1t(size_t(F) * Hp, 0.0f);
  for (int64_t h = 0; h < H; ++h)
    for (int64_t f = 0; f < F; ++f) w1t[size_t(f) * Hp + h] = w1[h * F + f];
  npa_model* m = new npa_model();
  m->cfg = *cfg;
  DeviceModel& d = m->dm;
  d.spatial_dims = cfg->spatial_dims;
  d.state_dims = cfg->state_dims;
  d.hidden_dims = int(H);
  d.feature_dims = int(F);
  d.update_dims = int(O);
  d.eps0 = cfg->eps0;
  d.alpha = cfg->alpha;
  d.equivariance = cfg->equivariance;
  d.density_grad = cfg->density_grad;
  d.state_grad = cfg->state_grad;
  d.log_norm_grad = cfg->log_norm_grad;
  d.log_norm_density_grad = cfg->log_norm_density_grad;
  d.position_features = cfg->position_features;
  d.device = device;
  d.hidden_padded = int(Hp);
  auto up = [&](float** dst, const float* src, size_t count) -> npa_status {
    NPA_CUDA(cudaMalloc(dst, std::max<size_t>(count, 4) * sizeof(float)), "cudaMalloc weights");
    NPA_CUDA(cudaMemcpy(*dst, src, count * sizeof(float), cudaMemcpyHostToDevice), "cudaMemcpy weights");
    return NPA_OK;
  };
  npa_status st = up(&d.w1t, w1t.data(), w1t.size());
  if (st == NPA_OK) st = up(&d.b1, b1, size_t(H));
  if (st == NPA_OK) st = up(&d.w2, w2, size_t(O * H));
  if (st == NPA_OK) st = up(&d.b2, b2, size_t(O));
  if (st != NPA_OK) {
    npa_model_destroy(m);
    return st;
  }
  *out = m;
  return NPA_OK;
}

void npa_model_destroy(npa_model* m) {
  if (!m) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m->dm.device);
  cudaFree(m->dm.w1t);
  cudaFree(m->dm.b1);
  cudaFree(m->dm.w2);
  cudaFree(m->dm.b2);
  HostArena& a = m->arena;
  for (cudaStream_t s : {a.stream, a.stream2, a.copy_in, a.copy_out})
    if (s) cudaStreamSynchronize(s);
  cudaFree(a.base);
  for (cudaEvent_t e : a.events) cudaEventDestroy(e);
  for (cudaStream_t s : {a.stream, a.stream2, a.copy_in, a.copy_out})
    if (s) cudaStreamDestroy(s);
  cudaSetDevice(prev);
  delete m;
}

npa_status npa_model_forward_update_from_features(npa_model* m, const float* features,
                                                  int64_t features_len, float* update,
                                                  int64_t update_len) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  const int64_t F = m->dm.feature_dims, O = m->dm.update_dims;
  if (features_len < 0 || features_len % F != 0)
    return fail(NPA_ERR_INVALID_ARGUMENT, "feature len " + std::to_string(features_len) +
                                              " is not divisible by perception dims " + std::to_string(F));
  const int64_t rows = features_len / F;
  if (rows > int64_t(kMaxParticles)) return fail(NPA_ERR_UNSUPPORTED, "too many rows");
  NPA_TRY(output_shape(update_len, rows * O));
  if (rows > 0 && (!features || !update)) return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  NPA_TRY(ensure_device(m->dm.device));
  Scratch s;
  NPA_TRY(s.init());
  float *df, *du;
  NPA_TRY(s.upload(&df, features, size_t(features_len)));
  NPA_TRY(s.alloc(&du, size_t(update_len)));
  NPA_TRY(launch_forward_update(m->dm, df, uint32_t(rows), du, s.stream));
  NPA_TRY(s.download(update, du, size_t(update_len) * 4));
  return s.finish();
}

// After a synchronising call that ran the MLP step kernel on the current
// device: NPA_ERR_TIMEOUT when that device's count of feature-tile copies that
// missed their bounded wait has grown since the last check on that device
// (those blocks left their tiles undone).  One watermark per device ordinal.
static std::mutex g_bulk_mu;
static std::vector<uint64_t> g_bulk_timeouts_seen;
static npa_status check_bulk_copies() {
  int dev = 0;
  NPA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t now = bulk_copy_timeouts() + ws_step_timeouts();
  std::lock_guard<std::mutex> lock(g_bulk_mu);
  if (dev >= int(g_bulk_timeouts_seen.size())) g_bulk_timeouts_seen.resize(dev + 1, 0);
  if (now <= g_bulk_timeouts_seen[dev]) return NPA_OK;
  g_bulk_timeouts_seen[dev] = now;
  return fail(NPA_ERR_TIMEOUT,
              "a bounded wait of the step kernels (an MLP feature-tile copy or a feature-tile "
              "hand-over) gave up");
}

// Reserves `bytes` of the model's host-call arena (caller holds m->mu).
npa_status arena_reserve(npa_model* m, size_t bytes) {
  HostArena& a = m->arena;
  if (!a.stream)
    NPA_CUDA(cudaStreamCreateWithFlags(&a.stream, cudaStreamNonBlocking), "cudaStreamCreate");
  if (bytes <= a.cap) return NPA_OK;
  const uint64_t cap = g_alloc_cap.load();
  if (cap && bytes > cap) return fail(NPA_ERR_OUT_OF_MEMORY, "allocation cap reached");
  NPA_CUDA(cudaStreamSynchronize(a.stream), "cudaStreamSynchronize");
  if (a.stream2) NPA_CUDA(cudaStreamSynchronize(a.stream2), "cudaStreamSynchronize");
  cudaFree(a.base);
  a.base = nullptr;
  a.cap = 0;
  int dev = 0;
  NPA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  NPA_CUDA(malloc_or_release(&a.base, bytes, dev), "cudaMalloc");
  a.cap = bytes;
  return NPA_OK;
}

// True when `p` is page-locked host memory (or null), so that copies from and
// to it run asynchronously on a copy engine.
static bool host_pinned(const void* p) {
  if (!p) return true;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// Rollout chunks of the host step.  Rollouts are independent, so the step of
// a batch is the step of each run of rollouts; with page-locked buffers the
// copy-in of chunk i + 1 and the copy-out of chunk i - 1 overlap the kernels
// of chunk i.  Chunks keep at least 2^17 particles (full kernel grids); at
// most 8.
static uint32_t host_step_chunks(uint32_t B, uint32_t N, bool pinned) {
  if (!pinned || B < 2) return 1;
  const uint64_t by_size = (uint64_t(B) * N) >> 17;
  return uint32_t(std::max<uint64_t>(1, std::min<uint64_t>({8, by_size, B})));
}

static npa_status arena_pipeline(HostArena& a, uint32_t chunks) {
  for (cudaStream_t* s : {&a.copy_in, &a.copy_out, &a.stream2})
    if (!*s) NPA_CUDA(cudaStreamCreateWithFlags(s, cudaStreamNonBlocking), "cudaStreamCreate");
  while (a.events.size() < 2 * size_t(chunks)) {
    cudaEvent_t e;
    NPA_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    a.events.push_back(e);
  }
  return NPA_OK;
}

npa_status npa_model_step(npa_model* m, const npa_grid_config* grid, const float* positions,
                          int64_t positions_len, const float* states, int64_t states_len,
                          int64_t batch, int64_t n, float dt, const float* update_mask,
                          float* next_positions, float* next_states, float* dx, float* ds,
                          float* features, float* density) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  NPA_TRY(check_step(m, grid));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_shapes(positions_len, states_len, batch, n, m->dm.state_dims));
  NPA_TRY(check_bins(grid, batch));
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  const int C = m->dm.state_dims;
  if (total > 0 && (!positions || (C > 0 && (!states || !next_states)) || !next_positions))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  NPA_TRY(ensure_device(m->dm.device));
  bool pinned = true;
  for (const void* h : {static_cast<const void*>(positions), static_cast<const void*>(states),
                        static_cast<const void*>(update_mask), static_cast<const void*>(next_positions),
                        static_cast<const void*>(next_states), static_cast<const void*>(dx),
                        static_cast<const void*>(ds), static_cast<const void*>(features),
                        static_cast<const void*>(density)})
    pinned = pinned && host_pinned(h);
  const uint32_t chunks = host_step_chunks(B, N, pinned);
  // Chunks hold floor(B / chunks) or ceil(B / chunks) rollouts; the workspace
  // serves both (the MLP tile shape, hence the tile padding, may differ).
  size_t wsb = 0;
  NPA_TRY(npa_dev_step_workspace_size(m, grid, chunks > 1 ? (B + chunks - 1) / chunks : batch, n,
                                      &wsb));
  if (chunks > 1 && B / chunks > 0) {
    size_t small = 0;
    NPA_TRY(npa_dev_step_workspace_size(m, grid, B / chunks, n, &small));
    wsb = std::max(wsb, small);
  }
  std::lock_guard<std::mutex> lock(m->mu);
  struct Bufs {
    float4 *pos, *np, *dx;
    float *st, *mask, *ns, *ds, *feat, *dens;
    char* ws;
    char* ws2;  // the second compute stream's workspace (chunked steps)
  } b{};
  const size_t F = size_t(m->dm.feature_dims);
  auto layout = [&](void* base) {
    Carve c(base, ~size_t(0));
    b.pos = c.take<float4>(total);
    b.st = c.take<float>(size_t(total) * C);
    b.mask = update_mask ? c.take<float>(total) : nullptr;
    b.np = c.take<float4>(total);
    b.ns = c.take<float>(size_t(total) * C);
    b.dx = dx ? c.take<float4>(total) : nullptr;
    b.ds = ds ? c.take<float>(size_t(total) * C) : nullptr;
    b.feat = features ? c.take<float>(size_t(total) * F) : nullptr;
    b.dens = density ? c.take<float>(total) : nullptr;
    b.ws = c.take<char>(wsb);
    b.ws2 = chunks > 1 ? c.take<char>(wsb) : nullptr;
    return c.used + 256;
  };
  NPA_TRY(arena_reserve(m, layout(nullptr)));
  layout(m->arena.base);
  HostArena& a = m->arena;
  cudaStream_t st = a.stream, st2 = st, in = st, out = st;
  if (chunks > 1) {
    NPA_TRY(arena_pipeline(a, chunks));
    in = a.copy_in;
    out = a.copy_out;
    st2 = a.stream2;
  }
  auto h2d = [&](void* d, const void* h, size_t bytes) -> npa_status {
    if (bytes) NPA_CUDA(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, in), "cudaMemcpyAsync H2D");
    return NPA_OK;
  };
  auto d2h = [&](void* h, const void* d, size_t bytes) -> npa_status {
    if (bytes && h) NPA_CUDA(cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, out), "cudaMemcpyAsync D2H");
    return NPA_OK;
  };
  // Chunk c holds rollouts [c B / chunks, (c + 1) B / chunks); its particles
  // [p0, p1) are contiguous in every buffer.
  auto span = [&](uint32_t c, size_t* p0, size_t* p1) {
    *p0 = size_t(uint64_t(c) * B / chunks) * N;
    *p1 = size_t(uint64_t(c + 1) * B / chunks) * N;
  };
  const npa_status status = [&]() -> npa_status {
    for (uint32_t c = 0; c < chunks; ++c) {
      size_t p0, p1;
      span(c, &p0, &p1);
      NPA_TRY(h2d(b.pos + p0, positions + 4 * p0, (p1 - p0) * 16));
      NPA_TRY(h2d(b.st + p0 * C, states + p0 * C, (p1 - p0) * C * 4));
      if (update_mask) NPA_TRY(h2d(b.mask + p0, update_mask + p0, (p1 - p0) * 4));
      if (chunks > 1) NPA_CUDA(cudaEventRecord(a.events[2 * c], in), "cudaEventRecord");
    }
    // Consecutive chunks alternate between two compute streams (each with
    // its own workspace), so one chunk's latency-bound phases overlap the
    // next chunk's kernels, as in the executor's rollout groups.
    for (uint32_t c = 0; c < chunks; ++c) {
      size_t p0, p1;
      span(c, &p0, &p1);
      const int64_t rollouts = int64_t((p1 - p0) / std::max<uint32_t>(N, 1));
      cudaStream_t cs = (c & 1) ? st2 : st;
      if (chunks > 1) NPA_CUDA(cudaStreamWaitEvent(cs, a.events[2 * c], 0), "cudaStreamWaitEvent");
      NPA_TRY(npa_dev_model_step(m, grid, reinterpret_cast<float*>(b.pos + p0), b.st + p0 * C,
                                 chunks > 1 ? rollouts : batch, n, dt,
                                 b.mask ? b.mask + p0 : nullptr, reinterpret_cast<float*>(b.np + p0),
                                 b.ns + p0 * C, b.dx ? reinterpret_cast<float*>(b.dx + p0) : nullptr,
                                 b.ds ? b.ds + p0 * C : nullptr, b.feat ? b.feat + p0 * F : nullptr,
                                 b.dens ? b.dens + p0 : nullptr, (c & 1) ? b.ws2 : b.ws, wsb, cs));
      if (chunks > 1) {
        NPA_CUDA(cudaEventRecord(a.events[2 * c + 1], cs), "cudaEventRecord");
        NPA_CUDA(cudaStreamWaitEvent(out, a.events[2 * c + 1], 0), "cudaStreamWaitEvent");
      }
      NPA_TRY(d2h(next_positions + 4 * p0, b.np + p0, (p1 - p0) * 16));
      NPA_TRY(d2h(next_states + p0 * C, b.ns + p0 * C, (p1 - p0) * C * 4));
      if (dx) NPA_TRY(d2h(dx + 4 * p0, b.dx + p0, (p1 - p0) * 16));
      if (ds) NPA_TRY(d2h(ds + p0 * C, b.ds + p0 * C, (p1 - p0) * C * 4));
      if (features) NPA_TRY(d2h(features + p0 * F, b.feat + p0 * F, (p1 - p0) * F * 4));
      if (density) NPA_TRY(d2h(density + p0, b.dens + p0, (p1 - p0) * 4));
    }
    return NPA_OK;
  }();
  // Nothing of this call is in flight on return, on success or failure.
  const cudaError_t e_out = cudaStreamSynchronize(out);
  const cudaError_t e_in = in != out ? cudaStreamSynchronize(in) : cudaSuccess;
  const cudaError_t e_st = st != out ? cudaStreamSynchronize(st) : cudaSuccess;
  const cudaError_t e_st2 = st2 != st ? cudaStreamSynchronize(st2) : cudaSuccess;
  if (status != NPA_OK) return status;
  for (cudaError_t e : {e_out, e_in, e_st, e_st2})
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  return check_bulk_copies();
}

// ---- device operators ----

npa_status npa_dev_hashgrid_workspace_size(const npa_grid_config* cfg, int64_t batch, int64_t n,
                                           size_t* bytes) {
  NPA_TRY(validate_grid(cfg));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_bins(cfg, batch));
  if (!bytes) return fail(NPA_ERR_INVALID_ARGUMENT, "null output");
  const GridParams g = make_grid_params(*cfg);
  *bytes = hashgrid_scratch_bytes(g, uint32_t(batch), uint32_t(n)) +
           sorted_view_bytes(uint32_t(batch), uint32_t(n)) + 256;
  return NPA_OK;
}

npa_status npa_dev_build_hashgrid(const npa_grid_config* cfg, const float* d_positions,
                                  int64_t batch, int64_t n, uint32_t* d_bin_offsets,
                                  uint32_t* d_permutation, uint32_t* d_inverse_permutation,
                                  void* d_workspace, size_t workspace_bytes, void* stream) {
  size_t need = 0;
  NPA_TRY(npa_dev_hashgrid_workspace_size(cfg, batch, n, &need));
  if (workspace_bytes < need) return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  if (!d_bin_offsets || (batch * n > 0 && (!d_positions || !d_permutation || !d_inverse_permutation || !d_workspace)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  const GridParams g = make_grid_params(*cfg);
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  Carve c(d_workspace, workspace_bytes);
  HashgridBuffers hb;
  hb.bin_offsets = d_bin_offsets;
  hb.permutation = d_permutation;
  hb.inverse = d_inverse_permutation;
  hb.srec = c.take<float4>(total);
  hb.scyz = c.take<int2>(total);
  const size_t sb = hashgrid_scratch_bytes(g, B, N);
  char* scratch = c.take<char>(sb);
  if (!c.fits()) return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  return launch_hashgrid(g, reinterpret_cast<const float4*>(d_positions), B, N, hb, scratch, sb,
                         static_cast<cudaStream_t>(stream));
}

npa_status npa_dev_perceive_workspace_size(const npa_grid_config* cfg, int64_t batch, int64_t n,
                                           int64_t state_dims, size_t* bytes) {
  NPA_TRY(validate_grid(cfg));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_bins(cfg, batch));
  if (!bytes || state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "bad argument");
  const GridParams g = make_grid_params(*cfg);
  *bytes = perceive_workspace_bytes(g, uint32_t(batch), uint32_t(n), 0,
                                    hashgrid_orders(g, uint32_t(batch), uint32_t(n)));
  return NPA_OK;
}

namespace {

// The phases of npa_dev_perceive_with_options; `ev` (4 events or null) are
// recorded before the hashgrid, density and perception launches and after.
npa_status perceive_phases(const npa_grid_config* cfg, const npa_perception_options* o,
                           const float* d_positions, const float* d_states, int64_t batch,
                           int64_t n, int64_t state_dims, float* d_features, float* d_density,
                           float* d_blurred_state, float* d_state_gradient,
                           float* d_density_gradient, void* d_workspace, size_t workspace_bytes,
                           cudaStream_t st, cudaEvent_t* ev) {
  if (!o) return fail(NPA_ERR_INVALID_ARGUMENT, "options are null");
  size_t need = 0;
  NPA_TRY(npa_dev_perceive_workspace_size(cfg, batch, n, state_dims, &need));
  if (workspace_bytes < need) return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  const GridParams g = make_grid_params(*cfg);
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  const PerceptionParams p = make_perception_params(g, *o, N, int(state_dims));
  if (total > 0 && (!d_positions || (state_dims > 0 && !d_states) || (p.feature_dims > 0 && !d_features) || !d_workspace))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  PerceiveWorkspace w;
  if (!carve_perceive(g, B, N, d_workspace, workspace_bytes, &w, 0, hashgrid_orders(g, B, N)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  if (ev) NPA_CUDA(cudaEventRecord(ev[0], st), "cudaEventRecord");
  NPA_TRY(launch_hashgrid(g, reinterpret_cast<const float4*>(d_positions), B, N, w.hg,
                          w.sort_scratch, w.sort_scratch_bytes, st));
  if (ev) NPA_CUDA(cudaEventRecord(ev[1], st), "cudaEventRecord");
  const SortedGrid sv = sorted_view(w, N, B, d_positions);
  NPA_TRY(launch_density(g, sv, B, w.volume, d_density, w.hits, st));
  if (ev) NPA_CUDA(cudaEventRecord(ev[2], st), "cudaEventRecord");
  NPA_TRY(launch_perception(g, p, sv, w.hits, B, d_states, int(state_dims), w.volume, d_features,
                            d_blurred_state, p.state_grad ? d_state_gradient : nullptr,
                            p.density_grad ? d_density_gradient : nullptr, st));
  if (ev) NPA_CUDA(cudaEventRecord(ev[3], st), "cudaEventRecord");
  return NPA_OK;
}

}  // namespace

npa_status npa_dev_perceive_with_options(const npa_grid_config* cfg,
                                         const npa_perception_options* o,
                                         const float* d_positions, const float* d_states,
                                         int64_t batch, int64_t n, int64_t state_dims,
                                         float* d_features, float* d_density,
                                         float* d_blurred_state, float* d_state_gradient,
                                         float* d_density_gradient, void* d_workspace,
                                         size_t workspace_bytes, void* stream) {
  return perceive_phases(cfg, o, d_positions, d_states, batch, n, state_dims, d_features,
                         d_density, d_blurred_state, d_state_gradient, d_density_gradient,
                         d_workspace, workspace_bytes, static_cast<cudaStream_t>(stream), nullptr);
}

npa_status npa_dev_perceive_many_profiled(const npa_grid_config* cfg,
                                          const npa_perception_options* o,
                                          const float* d_positions, const float* d_states,
                                          int64_t batch, int64_t n, int64_t state_dims,
                                          float* d_features, float* d_density,
                                          void* d_workspace, size_t workspace_bytes,
                                          int64_t repeats, void* stream, float* phase_ms,
                                          float* total_ms) {
  if (repeats < 0 || (repeats > 0 && (!phase_ms || !total_ms)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "bad repeat count or null timing output");
  if (repeats == 0) return NPA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<cudaEvent_t> ev(size_t(repeats) * 4, nullptr);
  npa_status rc = NPA_OK;
  for (auto& e : ev) {
    if (cudaEventCreate(&e) != cudaSuccess) {
      e = nullptr;
      rc = fail(NPA_ERR_CUDA, "cudaEventCreate");
      break;
    }
  }
  for (int64_t r = 0; rc == NPA_OK && r < repeats; ++r)
    rc = perceive_phases(cfg, o, d_positions, d_states, batch, n, state_dims, d_features,
                         d_density, nullptr, nullptr, nullptr, d_workspace, workspace_bytes, st,
                         &ev[size_t(r) * 4]);
  if (rc == NPA_OK && cudaStreamSynchronize(st) != cudaSuccess)
    rc = fail(NPA_ERR_CUDA, "cudaStreamSynchronize");
  for (int64_t r = 0; rc == NPA_OK && r < repeats; ++r)
    for (int k = 0; k < 3; ++k)
      cudaEventElapsedTime(&phase_ms[r * 3 + k], ev[r * 4 + k], ev[r * 4 + k + 1]);
  if (rc == NPA_OK) cudaEventElapsedTime(total_ms, ev[0], ev[size_t(repeats) * 4 - 1]);
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}

npa_status npa_dev_model_forward_update(npa_model* m, const float* d_features, int64_t rows,
                                        float* d_update, void* stream) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  if (rows < 0 || rows > int64_t(kMaxParticles)) return fail(NPA_ERR_INVALID_ARGUMENT, "bad row count");
  if (rows > 0 && (!d_features || !d_update)) return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  return launch_forward_update(m->dm, d_features, uint32_t(rows), d_update,
                               static_cast<cudaStream_t>(stream));
}

npa_status npa_dev_euler_step(const npa_grid_config* cfg, const float* d_positions,
                              const float* d_states, const float* d_dx, const float* d_ds,
                              int64_t batch, int64_t n, int64_t state_dims, float dt,
                              const float* d_update_mask, float* d_next_positions,
                              float* d_next_states, void* stream) {
  NPA_TRY(validate_grid(cfg));
  NPA_TRY(check_counts(batch, n));
  if (state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "state_dims must be >= 0");
  const GridParams g = make_grid_params(*cfg);
  return launch_euler(g, reinterpret_cast<const float4*>(d_positions), d_states,
                      reinterpret_cast<const float4*>(d_dx), d_ds, uint32_t(batch * n),
                      int(state_dims), dt, d_update_mask, reinterpret_cast<float4*>(d_next_positions),
                      d_next_states, static_cast<cudaStream_t>(stream));
}

npa_status npa_dev_decode_gaussians_3d(const npa_gaussian_decode_config* cfg,
                                       const float* d_positions, const float* d_states,
                                       int64_t count, int64_t state_dims, float* d_out,
                                       void* stream) {
  if (count < 0 || count > int64_t(kMaxParticles)) return fail(NPA_ERR_INVALID_ARGUMENT, "bad count");
  NPA_TRY(validate_decode(cfg, state_dims));
  return launch_decode(*cfg, reinterpret_cast<const float4*>(d_positions), d_states,
                       uint32_t(count), int(state_dims), d_out, static_cast<cudaStream_t>(stream));
}

npa_status npa_dev_step_workspace_size(npa_model* m, const npa_grid_config* grid, int64_t batch,
                                       int64_t n, size_t* bytes) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  NPA_TRY(check_step(m, grid));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_bins(grid, batch));
  if (!bytes) return fail(NPA_ERR_INVALID_ARGUMENT, "null output");
  const GridParams g = make_grid_params(*grid);
  *bytes = perceive_workspace_bytes(g, uint32_t(batch), uint32_t(n),
                                    tiles_floats(uint32_t(batch), uint32_t(n), m->dm.feature_dims,
                                                 step_tile_rows(m->dm, uint64_t(batch) * n)),
                                    hashgrid_orders(g, uint32_t(batch), uint32_t(n)));
  return NPA_OK;
}

npa_status npa_dev_model_step(npa_model* m, const npa_grid_config* grid, const float* d_positions,
                              const float* d_states, int64_t batch, int64_t n, float dt,
                              const float* d_update_mask, float* d_next_positions,
                              float* d_next_states, float* d_dx, float* d_ds, float* d_features,
                              float* d_density, void* d_workspace, size_t workspace_bytes,
                              void* stream) {
  size_t need = 0;
  NPA_TRY(npa_dev_step_workspace_size(m, grid, batch, n, &need));
  if (workspace_bytes < need) return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  const GridParams g = make_grid_params(*grid);
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  if (total > 0 && (!d_positions || !d_next_positions || !d_workspace ||
                    (m->dm.state_dims > 0 && (!d_states || !d_next_states))))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  if (!mlp_step_supported(m->dm))
    return fail(NPA_ERR_UNSUPPORTED, "step shape outside the supported range");
  PerceiveWorkspace w;
  const int tile_rows = step_tile_rows(m->dm, total);
  if (!carve_perceive(g, B, N, d_workspace, workspace_bytes, &w,
                      tiles_floats(B, N, m->dm.feature_dims, tile_rows), hashgrid_orders(g, B, N)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  const PerceptionParams p = make_perception_params(g, model_options(m->cfg), N, m->dm.state_dims);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  NPA_TRY(launch_hashgrid(g, reinterpret_cast<const float4*>(d_positions), B, N, w.hg,
                          w.sort_scratch, w.sort_scratch_bytes, st));
  const SortedGrid sv = sorted_view(w, N, B, d_positions);
  NPA_TRY(launch_density(g, sv, B, w.volume, d_density, w.hits, st));
  NPA_TRY(launch_perception_tiles(g, p, sv, w.hits, B, d_states, m->dm.state_dims, w.volume, tile_rows,
                                  w.tiles, st));
  StepOutputs out;
  out.next_positions = reinterpret_cast<float4*>(d_next_positions);
  out.next_states = d_next_states;
  out.dx = reinterpret_cast<float4*>(d_dx);
  out.ds = d_ds;
  out.features = d_features;
  return launch_mlp_step(m->dm, g, sv, B, w.tiles, d_states, dt, d_update_mask, StochasticMask{},
                         out, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// executor
// ---------------------------------------------------------------------------
// One rollout step is four phases, each captured into its own CUDA graph per
// ping-pong parity: (0) hashgrid, (1) density, (2) perception into feature
// tiles, (3) MLP + dx/ds + Euler.  Replaying the phases as separate graphs
// lets a caller bracket each kernel with CUDA events on the launching stream.
constexpr int kPhases = 4;
constexpr int kMaxStepGroups = 4;
constexpr size_t kGroupedMaxParticles = size_t(1) << 18;  // default grouping up to this batch size

struct npa_executor {
  npa_model* model = nullptr;
  npa_grid_config grid{};
  GridParams g{};
  PerceptionParams p{};
  int64_t batch = 0, n = 0;
  float* pos[2] = {nullptr, nullptr};
  float* st[2] = {nullptr, nullptr};
  int cur = 0;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  PerceiveWorkspace w{};
  cudaGraphExec_t graph[2][kPhases] = {};
  // Whole steps for the unprofiled replay: step_graph[p] is one step from
  // ping-pong parity p, pair_graph[p] two steps (back to parity p); one graph
  // launch instead of one per phase.
  cudaGraphExec_t step_graph[2] = {};
  cudaGraphExec_t pair_graph[2] = {};
  float graph_dt = 0.0f;
  cudaStream_t graph_stream = nullptr;
  int64_t launches[kPhases] = {0, 0, 0, 0};
  int tile_rows = 0;
  // Stochastic update mask (create_state_with_update_prob): active when
  // update_prob < 1; step_index mirrors the device counter d_step.
  int stochastic = 0;
  float update_prob = 1.0f;
  uint32_t* d_lane_seeds = nullptr;  // [batch]
  uint32_t* d_step = nullptr;
  uint32_t step_index = 0;
  // Fused step: phase 2 is empty and phase 3 runs perception + MLP + Euler in
  // one kernel (npa_executor_set_fused_step).
  int fused = 0;
  // Rollout groups of the whole-step replay (npa_executor_set_step_groups):
  // the batch split into `groups` runs of consecutive rollouts, each with its
  // own workspace, step counter and capture stream, whose steps form
  // independent chains in the step graphs (rollouts never interact), so one
  // group's latency-bound phases overlap another's.
  int groups = 1;
  struct Group {
    int64_t first = 0, batch = 0;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    PerceiveWorkspace w{};
    int tile_rows = 0;
    uint32_t* d_step = nullptr;
    cudaStream_t side = nullptr;
    cudaEvent_t joined = nullptr;
  };
  Group grp[kMaxStepGroups];
  cudaEvent_t fork = nullptr;
  int64_t step_launches[2] = {0, 0}, pair_launches[2] = {0, 0};
};

namespace {

// The rollouts [first, first + batch) of the executor with their own
// workspace and step counter: a whole-batch view, or one rollout group.
struct ExecView {
  int64_t first, batch;
  const PerceiveWorkspace* w;
  int tile_rows;
  uint32_t* d_step;
};

ExecView whole_view(const npa_executor* e) {
  return ExecView{0, e->batch, &e->w, e->tile_rows, e->d_step};
}

npa_status exec_enqueue_view_phase(npa_executor* e, const ExecView& v, int from, int phase,
                                   float dt, cudaStream_t s) {
  const uint32_t B = uint32_t(v.batch), N = uint32_t(e->n);
  const int C = e->model->dm.state_dims;
  const size_t row0 = size_t(v.first) * N;
  float* pos = e->pos[from] + row0 * 4;
  float* st = e->st[from] + row0 * C;
  const SortedGrid sv = sorted_view(*v.w, N, B, pos);
  switch (phase) {
    case 0:
      return launch_hashgrid(e->g, reinterpret_cast<const float4*>(pos), B, N, v.w->hg,
                             v.w->sort_scratch, v.w->sort_scratch_bytes, s);
    case 1:
      return launch_density(e->g, sv, B, v.w->volume, nullptr, v.w->hits, s);
    case 2:
      if (e->fused) return NPA_OK;
      return launch_perception_tiles(e->g, e->p, sv, v.w->hits, B, st, C, v.w->volume,
                                     v.tile_rows, v.w->tiles, s);
    default: {
      StepOutputs out;
      out.next_positions = reinterpret_cast<float4*>(e->pos[1 - from] + row0 * 4);
      out.next_states = e->st[1 - from] + row0 * C;
      out.dx = nullptr;
      out.ds = nullptr;
      out.features = nullptr;
      StochasticMask sm;
      if (e->stochastic) {
        sm.update_prob = e->update_prob;
        sm.lane_seeds = e->d_lane_seeds + v.first;
        sm.step_counter = v.d_step;
      }
      if (e->fused == 2)
        NPA_TRY(launch_ws_step(e->model->dm, e->g, e->p, sv, v.w->hits, B, st, v.w->volume, dt,
                               nullptr, sm, out, s));
      else if (e->fused)
        NPA_TRY(launch_fused_step(e->model->dm, e->g, e->p, sv, v.w->hits, B, st, v.w->volume,
                                  dt, nullptr, sm, out, s));
      else
        NPA_TRY(launch_mlp_step(e->model->dm, e->g, sv, B, v.w->tiles, st, dt, nullptr, sm,
                                out, s));
      if (e->stochastic) NPA_TRY(launch_advance_step(v.d_step, s));
      return NPA_OK;
    }
  }
}

npa_status exec_enqueue_phase(npa_executor* e, int from, int phase, float dt, cudaStream_t s) {
  return exec_enqueue_view_phase(e, whole_view(e), from, phase, dt, s);
}

void exec_drop_graphs(npa_executor* e) {
  auto drop = [](cudaGraphExec_t& g) {
    if (g) cudaGraphExecDestroy(g);
    g = nullptr;
  };
  for (auto& row : e->graph)
    for (auto& g : row) drop(g);
  for (auto& g : e->step_graph) drop(g);
  for (auto& g : e->pair_graph) drop(g);
}

// Captures the phases of `steps` consecutive steps from parity `from` into one
// executable graph.
npa_status exec_capture_steps(npa_executor* e, int from, int steps, float dt, cudaStream_t stream,
                              cudaGraphExec_t* out, int64_t* launches) {
  cudaGraph_t graph = nullptr;
  const uint64_t before = npa_kernel_launch_count();
  NPA_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal),
           "cudaStreamBeginCapture");
  npa_status st = NPA_OK;
  if (e->groups <= 1) {
    for (int k = 0; k < steps && st == NPA_OK; ++k)
      for (int phase = 0; phase < kPhases && st == NPA_OK; ++phase)
        st = exec_enqueue_phase(e, (from + k) & 1, phase, dt, stream);
  } else {
    // fork: every group's chain starts after what precedes the graph; join:
    // the capture stream waits for every chain
    if (cudaEventRecord(e->fork, stream) != cudaSuccess) st = fail(NPA_ERR_CUDA, "fork record");
    for (int gi = 0; gi < e->groups && st == NPA_OK; ++gi) {
      npa_executor::Group& gr = e->grp[gi];
      const ExecView v{gr.first, gr.batch, &gr.w, gr.tile_rows, gr.d_step};
      cudaStream_t gs = gi == 0 ? stream : gr.side;
      if (gi > 0 && cudaStreamWaitEvent(gs, e->fork, 0) != cudaSuccess)
        st = fail(NPA_ERR_CUDA, "fork wait");
      for (int k = 0; k < steps && st == NPA_OK; ++k)
        for (int phase = 0; phase < kPhases && st == NPA_OK; ++phase)
          st = exec_enqueue_view_phase(e, v, (from + k) & 1, phase, dt, gs);
      if (st == NPA_OK && gi > 0) {
        if (cudaEventRecord(gr.joined, gs) != cudaSuccess ||
            cudaStreamWaitEvent(stream, gr.joined, 0) != cudaSuccess)
          st = fail(NPA_ERR_CUDA, "join");
      }
    }
  }
  cudaError_t ce = cudaStreamEndCapture(stream, &graph);
  *launches = int64_t(npa_kernel_launch_count() - before);
  if (st != NPA_OK) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
  ce = cudaGraphInstantiate(out, graph, 0);
  cudaGraphDestroy(graph);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
  return NPA_OK;
}

npa_status exec_capture(npa_executor* e, float dt, cudaStream_t stream) {
  exec_drop_graphs(e);
  for (int from = 0; from < 2; ++from) {
    for (int phase = 0; phase < kPhases; ++phase) {
      cudaGraph_t graph = nullptr;
      NPA_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal),
               "cudaStreamBeginCapture");
      const uint64_t before = npa_kernel_launch_count();
      npa_status st = exec_enqueue_phase(e, from, phase, dt, stream);
      cudaError_t ce = cudaStreamEndCapture(stream, &graph);
      if (st != NPA_OK) {
        if (graph) cudaGraphDestroy(graph);
        return st;
      }
      if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
      e->launches[phase] = int64_t(npa_kernel_launch_count() - before);
      ce = cudaGraphInstantiate(&e->graph[from][phase], graph, 0);
      cudaGraphDestroy(graph);
      if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
    }
  }
  for (int from = 0; from < 2; ++from) {
    NPA_TRY(exec_capture_steps(e, from, 1, dt, stream, &e->step_graph[from],
                               &e->step_launches[from]));
    NPA_TRY(exec_capture_steps(e, from, 2, dt, stream, &e->pair_graph[from],
                               &e->pair_launches[from]));
  }
  e->graph_dt = dt;
  e->graph_stream = stream;
  return NPA_OK;
}

npa_status exec_run_phase(npa_executor* e, int phase, float dt, int32_t use_graph,
                          cudaStream_t s) {
  if (use_graph) {
    if (e->launches[phase] == 0) return NPA_OK;  // an empty phase (perception when fused)
    NPA_CUDA(cudaGraphLaunch(e->graph[e->cur][phase], s), "cudaGraphLaunch");
    g_launches.fetch_add(uint64_t(e->launches[phase]), std::memory_order_relaxed);
    return NPA_OK;
  }
  return exec_enqueue_phase(e, e->cur, phase, dt, s);
}

}  // namespace

extern "C" {

npa_status npa_executor_create(npa_model* m, const npa_grid_config* grid, int64_t batch,
                               int64_t n, npa_executor** out) {
  if (!m || !out) return fail(NPA_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  NPA_TRY(check_step(m, grid));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_bins(grid, batch));
  if (!mlp_step_supported(m->dm))
    return fail(NPA_ERR_UNSUPPORTED, "step shape outside the supported range");
  NPA_TRY(ensure_device(m->dm.device));
  if (m->dm.log_norm_grad || m->dm.log_norm_density_grad) {
    Log1pTable l1p;  // uploaded before any step is captured into a graph
    NPA_TRY(device_log1p_table(&l1p));
  }
  npa_executor* e = new npa_executor();
  e->model = m;
  e->grid = *grid;
  e->g = make_grid_params(*grid);
  e->p = make_perception_params(e->g, model_options(m->cfg), uint32_t(n), m->dm.state_dims);
  e->batch = batch;
  e->n = n;
  const size_t total = size_t(batch) * n;
  const size_t C = size_t(m->dm.state_dims);
  e->tile_rows = step_tile_rows(m->dm, total);
  const size_t tf = tiles_floats(uint32_t(batch), uint32_t(n), m->dm.feature_dims, e->tile_rows);
  const bool ordered = hashgrid_orders(e->g, uint32_t(batch), uint32_t(n));
  e->ws_bytes = perceive_workspace_bytes(e->g, uint32_t(batch), uint32_t(n), tf, ordered);
  npa_status st = NPA_OK;
  auto alloc = [&](void** p, size_t b) -> npa_status {
    NPA_CUDA(cudaMalloc(p, std::max<size_t>(b, 256)), "cudaMalloc executor");
    return NPA_OK;
  };
  for (int i = 0; i < 2 && st == NPA_OK; ++i) {
    st = alloc(reinterpret_cast<void**>(&e->pos[i]), total * 16);
    if (st == NPA_OK) st = alloc(reinterpret_cast<void**>(&e->st[i]), total * C * 4);
  }
  if (st == NPA_OK) st = alloc(&e->ws, e->ws_bytes);
  if (st == NPA_OK) st = alloc(reinterpret_cast<void**>(&e->d_lane_seeds), size_t(batch) * 4);
  if (st == NPA_OK) st = alloc(reinterpret_cast<void**>(&e->d_step), 4);
  if (st == NPA_OK && cudaMemset(e->d_step, 0, 4) != cudaSuccess)
    st = fail(NPA_ERR_CUDA, "cudaMemset step counter");
  if (st == NPA_OK &&
      !carve_perceive(e->g, uint32_t(batch), uint32_t(n), e->ws, e->ws_bytes, &e->w, tf, ordered))
    st = fail(NPA_ERR_INVALID_ARGUMENT, "executor workspace layout");
  // Small batches leave most SMs idle in their latency-bound phases: two
  // rollout groups overlap them (cfg2 shards of 32 / 64 rollouts: 0.227 vs
  // 0.243 ms and 0.419 vs 0.441 ms per step); the full 256-rollout batch
  // fills the GPU and runs best as one chain (1.496 vs 1.536 ms).
  if (st == NPA_OK && batch >= 2 && total <= kGroupedMaxParticles)
    st = npa_executor_set_step_groups(e, 2);
  if (st != NPA_OK) {
    npa_executor_destroy(e);
    return st;
  }
  *out = e;
  return NPA_OK;
}

static void exec_free_groups(npa_executor* e) {
  for (auto& gr : e->grp) {
    if (gr.ws) cudaFree(gr.ws);
    if (gr.d_step) cudaFree(gr.d_step);
    if (gr.side) cudaStreamDestroy(gr.side);
    if (gr.joined) cudaEventDestroy(gr.joined);
    gr = npa_executor::Group{};
  }
  if (e->fork) cudaEventDestroy(e->fork);
  e->fork = nullptr;
  e->groups = 1;
}

void npa_executor_destroy(npa_executor* e) {
  if (!e) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(e->model->dm.device);
  exec_drop_graphs(e);
  exec_free_groups(e);
  for (int i = 0; i < 2; ++i) {
    cudaFree(e->pos[i]);
    cudaFree(e->st[i]);
  }
  cudaFree(e->ws);
  cudaFree(e->d_lane_seeds);
  cudaFree(e->d_step);
  cudaSetDevice(prev);
  delete e;
}

npa_status npa_executor_upload_state(npa_executor* e, const float* positions, const float* states) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  NPA_TRY(ensure_device(e->model->dm.device));
  const size_t total = size_t(e->batch) * e->n;
  const size_t C = size_t(e->model->dm.state_dims);
  if (total && (!positions || (C && !states))) return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  NPA_CUDA(cudaMemcpy(e->pos[e->cur], positions, total * 16, cudaMemcpyHostToDevice), "upload positions");
  if (C) NPA_CUDA(cudaMemcpy(e->st[e->cur], states, total * C * 4, cudaMemcpyHostToDevice), "upload states");
  return NPA_OK;
}

npa_status npa_executor_set_state_device(npa_executor* e, const float* d_positions,
                                         const float* d_states, void* stream) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  NPA_TRY(ensure_device(e->model->dm.device));
  const size_t total = size_t(e->batch) * e->n;
  const size_t C = size_t(e->model->dm.state_dims);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  NPA_CUDA(cudaMemcpyAsync(e->pos[e->cur], d_positions, total * 16, cudaMemcpyDeviceToDevice, s), "copy positions");
  if (C) NPA_CUDA(cudaMemcpyAsync(e->st[e->cur], d_states, total * C * 4, cudaMemcpyDeviceToDevice, s), "copy states");
  return NPA_OK;
}

static npa_status exec_prepare(npa_executor* e, int64_t steps, float dt, int32_t use_graph,
                               cudaStream_t s) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  if (steps < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "steps must be >= 0");
  NPA_TRY(ensure_device(e->model->dm.device));
  if (use_graph && s == nullptr) return fail(NPA_ERR_INVALID_ARGUMENT, "graph replay needs a non-default stream");
  if (use_graph && (!e->graph[0][0] || e->graph_dt != dt || e->graph_stream != s))
    NPA_TRY(exec_capture(e, dt, s));
  if (e->stochastic && steps > 0) {  // the device counters start from the host's step index
    NPA_CUDA(cudaMemcpyAsync(e->d_step, &e->step_index, 4, cudaMemcpyHostToDevice, s),
             "upload step index");
    for (int gi = 0; gi < e->groups && e->groups > 1; ++gi)
      NPA_CUDA(cudaMemcpyAsync(e->grp[gi].d_step, &e->step_index, 4, cudaMemcpyHostToDevice, s),
               "upload step index");
  }
  return NPA_OK;
}

npa_status npa_executor_step_many(npa_executor* e, int64_t steps, float dt, int32_t use_graph,
                                  void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  NPA_TRY(exec_prepare(e, steps, dt, use_graph, s));
  int64_t k = 0;
  if (use_graph) {
    for (; k + 2 <= steps; k += 2) {
      NPA_CUDA(cudaGraphLaunch(e->pair_graph[e->cur], s), "cudaGraphLaunch");
      g_launches.fetch_add(uint64_t(e->pair_launches[e->cur]), std::memory_order_relaxed);
      e->step_index += 2u;
    }
    if (k < steps) {
      NPA_CUDA(cudaGraphLaunch(e->step_graph[e->cur], s), "cudaGraphLaunch");
      g_launches.fetch_add(uint64_t(e->step_launches[e->cur]), std::memory_order_relaxed);
      e->cur = 1 - e->cur;
      e->step_index += 1u;
      ++k;
    }
    return NPA_OK;
  }
  for (; k < steps; ++k) {
    for (int phase = 0; phase < kPhases; ++phase) NPA_TRY(exec_run_phase(e, phase, dt, use_graph, s));
    e->cur = 1 - e->cur;
    e->step_index += 1u;
  }
  return NPA_OK;
}

npa_status npa_executor_set_update_prob(npa_executor* e, float update_prob, uint64_t seed,
                                        const uint64_t* lane_seeds) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  NPA_TRY(ensure_device(e->model->dm.device));
  // gpu_random_seed (gpu/helpers/params.rs:186-188) and gpu_lane_seeds
  // (gpu/executor/state.rs:1282-1312): lane l of a shared seed draws with
  // seed ^ (l * particle_count); independent lanes fold their own seeds.
  auto fold = [](uint64_t v) { return uint32_t(v) ^ uint32_t(v >> 32); };
  std::vector<uint32_t> seeds(size_t(e->batch));
  for (int64_t lane = 0; lane < e->batch; ++lane) {
    if (lane_seeds) {
      seeds[size_t(lane)] = fold(lane_seeds[lane]);
    } else {
      const uint64_t offset = uint64_t(lane) * uint64_t(e->n);
      if (offset > 0xffffffffull) return fail(NPA_ERR_INVALID_ARGUMENT, "lane particle offset overflow");
      seeds[size_t(lane)] = fold(seed) ^ uint32_t(offset);
    }
  }
  if (!seeds.empty())
    NPA_CUDA(cudaMemcpy(e->d_lane_seeds, seeds.data(), seeds.size() * 4, cudaMemcpyHostToDevice),
             "upload lane seeds");
  const int stochastic = update_prob >= 1.0f ? 0 : 1;
  if (stochastic != e->stochastic) exec_drop_graphs(e);  // the MLP phase changes shape
  e->stochastic = stochastic;
  e->update_prob = update_prob;
  if (stochastic) exec_drop_graphs(e);  // update_prob is a kernel argument
  return NPA_OK;
}

npa_status npa_executor_set_step_index(npa_executor* e, uint32_t step_index) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  e->step_index = step_index;
  return NPA_OK;
}

npa_status npa_executor_step_index(npa_executor* e, uint32_t* step_index) {
  if (!e || !step_index) return fail(NPA_ERR_INVALID_ARGUMENT, "null argument");
  *step_index = e->step_index;
  return NPA_OK;
}

npa_status npa_executor_step_many_profiled(npa_executor* e, int64_t steps, float dt,
                                           int32_t use_graph, void* stream, float* phase_ms,
                                           float* total_ms) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  NPA_TRY(exec_prepare(e, steps, dt, use_graph, s));
  if (!phase_ms || !total_ms) return fail(NPA_ERR_INVALID_ARGUMENT, "null timing output");
  std::vector<cudaEvent_t> ev(size_t(steps) * (kPhases + 1) + 1, nullptr);
  npa_status st = NPA_OK;
  for (auto& x : ev)
    if (cudaEventCreate(&x) != cudaSuccess) st = fail(NPA_ERR_CUDA, "cudaEventCreate");
  if (st == NPA_OK && steps > 0) {
    for (int64_t k = 0; k < steps && st == NPA_OK; ++k) {
      cudaEventRecord(ev[size_t(k) * (kPhases + 1)], s);
      for (int phase = 0; phase < kPhases && st == NPA_OK; ++phase) {
        st = exec_run_phase(e, phase, dt, use_graph, s);
        cudaEventRecord(ev[size_t(k) * (kPhases + 1) + phase + 1], s);
      }
      e->cur = 1 - e->cur;
      e->step_index += 1u;
    }
    if (st == NPA_OK && cudaStreamSynchronize(s) != cudaSuccess) st = fail(NPA_ERR_CUDA, "sync");
    if (st == NPA_OK) {
      for (int64_t k = 0; k < steps; ++k)
        for (int phase = 0; phase < kPhases; ++phase) {
          float ms = 0.0f;
          cudaEventElapsedTime(&ms, ev[size_t(k) * (kPhases + 1) + phase],
                               ev[size_t(k) * (kPhases + 1) + phase + 1]);
          phase_ms[k * kPhases + phase] = ms;
        }
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, ev[0], ev[size_t(steps - 1) * (kPhases + 1) + kPhases]);
      *total_ms = ms;
    }
  }
  for (auto& x : ev)
    if (x) cudaEventDestroy(x);
  return st;
}

npa_status npa_executor_read_state(npa_executor* e, float* positions, float* states) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  NPA_TRY(ensure_device(e->model->dm.device));
  NPA_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  const size_t total = size_t(e->batch) * e->n;
  const size_t C = size_t(e->model->dm.state_dims);
  if (positions) NPA_CUDA(cudaMemcpy(positions, e->pos[e->cur], total * 16, cudaMemcpyDeviceToHost), "read positions");
  if (states && C) NPA_CUDA(cudaMemcpy(states, e->st[e->cur], total * C * 4, cudaMemcpyDeviceToHost), "read states");
  return check_bulk_copies();
}

npa_status npa_executor_state_device(npa_executor* e, float** d_positions, float** d_states) {
  if (!e || !d_positions || !d_states) return fail(NPA_ERR_INVALID_ARGUMENT, "null argument");
  *d_positions = e->pos[e->cur];
  *d_states = e->st[e->cur];
  return NPA_OK;
}

npa_status npa_executor_set_step_groups(npa_executor* e, int32_t groups) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  if (groups < 1 || groups > kMaxStepGroups || (e->batch > 0 && groups > e->batch))
    return fail(NPA_ERR_INVALID_ARGUMENT,
                "step groups must be between 1 and min(4, batch size), got " +
                    std::to_string(groups));
  if (groups == e->groups) return NPA_OK;
  NPA_TRY(ensure_device(e->model->dm.device));
  NPA_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");  // no replay still uses them
  exec_drop_graphs(e);
  exec_free_groups(e);
  if (groups == 1) return NPA_OK;
  const uint32_t N = uint32_t(e->n);
  const int64_t base = e->batch / groups, extra = e->batch % groups;
  npa_status st = NPA_OK;
  if (cudaEventCreateWithFlags(&e->fork, cudaEventDisableTiming) != cudaSuccess)
    st = fail(NPA_ERR_CUDA, "cudaEventCreate");
  for (int gi = 0; gi < groups && st == NPA_OK; ++gi) {
    npa_executor::Group& gr = e->grp[gi];
    gr.batch = base + (gi < extra ? 1 : 0);
    gr.first = gi * base + std::min<int64_t>(gi, extra);
    const uint64_t rows = uint64_t(gr.batch) * N;
    gr.tile_rows = step_tile_rows(e->model->dm, rows);
    const size_t tf = tiles_floats(uint32_t(gr.batch), N, e->model->dm.feature_dims, gr.tile_rows);
    const bool ordered = hashgrid_orders(e->g, uint32_t(gr.batch), N);
    gr.ws_bytes = perceive_workspace_bytes(e->g, uint32_t(gr.batch), N, tf, ordered);
    if (cudaMalloc(&gr.ws, std::max<size_t>(gr.ws_bytes, 256)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&gr.d_step), 4) != cudaSuccess) {
      cudaGetLastError();
      st = fail(NPA_ERR_OUT_OF_MEMORY, "step group workspace");
      break;
    }
    if (cudaMemset(gr.d_step, 0, 4) != cudaSuccess ||
        cudaStreamCreateWithFlags(&gr.side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&gr.joined, cudaEventDisableTiming) != cudaSuccess)
      st = fail(NPA_ERR_CUDA, "step group set-up");
    else if (!carve_perceive(e->g, uint32_t(gr.batch), N, gr.ws, gr.ws_bytes, &gr.w, tf, ordered))
      st = fail(NPA_ERR_INVALID_ARGUMENT, "step group workspace layout");
  }
  if (st != NPA_OK) {
    exec_free_groups(e);
    return st;
  }
  e->groups = groups;
  return NPA_OK;
}

npa_status npa_executor_step_groups(npa_executor* e, int32_t* groups) {
  if (!e || !groups) return fail(NPA_ERR_INVALID_ARGUMENT, "null argument");
  *groups = e->groups;
  return NPA_OK;
}

npa_status npa_executor_set_fused_step(npa_executor* e, int32_t fused) {
  if (!e) return fail(NPA_ERR_INVALID_ARGUMENT, "null executor");
  if (fused < 0 || fused > 2) return fail(NPA_ERR_INVALID_ARGUMENT, "fused must be 0, 1 or 2");
  const uint32_t B = uint32_t(e->batch), N = uint32_t(e->n);
  if (fused == 1 && !fused_step_supported(e->model->dm, e->g, e->p, B, B * N))
    return fail(NPA_ERR_UNSUPPORTED,
                "the fused step covers 2D models with more than 4 channels, hidden width up to "
                "128 and sparse cells");
  if (fused == 2 && !ws_step_supported(e->model->dm, e->g, e->p, B, B * N))
    return fail(NPA_ERR_UNSUPPORTED,
                "the warp-specialised fused step covers 2D models with at most 16 channels, "
                "hidden width 128 and sparse cells");
  if (fused != e->fused) {
    NPA_TRY(ensure_device(e->model->dm.device));
    exec_drop_graphs(e);
    for (auto& l : e->launches) l = 0;
  }
  e->fused = fused;
  return NPA_OK;
}

npa_status npa_executor_launches_per_step(npa_executor* e, int64_t* launches) {
  if (!e || !launches) return fail(NPA_ERR_INVALID_ARGUMENT, "null argument");
  *launches = e->launches[0] + e->launches[1] + e->launches[2] + e->launches[3];
  return NPA_OK;
}

npa_status npa_model_run_rollout(npa_model* m, const npa_grid_config* grid, float* positions,
                                 int64_t positions_len, float* states, int64_t states_len,
                                 int64_t batch, int64_t n, int64_t steps, float dt) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  NPA_TRY(check_step(m, grid));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_shapes(positions_len, states_len, batch, n, m->dm.state_dims));
  if (steps < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "steps must be >= 0");
  npa_executor* e = nullptr;
  NPA_TRY(npa_executor_create(m, grid, batch, n, &e));
  cudaStream_t s = nullptr;
  npa_status st = NPA_OK;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
    st = fail(NPA_ERR_CUDA, "cudaStreamCreate");
  if (st == NPA_OK) st = npa_executor_upload_state(e, positions, states);
  if (st == NPA_OK) st = npa_executor_step_many(e, steps, dt, steps > 2 ? 1 : 0, s);
  if (st == NPA_OK) st = npa_executor_read_state(e, positions, states);
  if (s) cudaStreamDestroy(s);
  npa_executor_destroy(e);
  return st;
}

// Device scratch of the adjoint beyond the perception workspace (floats):
// caller-order density, density adjoint, per-particle adjoint rows.
static size_t adjoint_extra_floats(const GridParams& g, uint32_t total, int64_t state_dims) {
  return 2 * size_t(total) + 64 + adjoint_scratch_floats(total, int(state_dims), g.dim);
}

static npa_status adjoint_run(const npa_grid_config* cfg, const npa_perception_options* o,
                              const float* d_positions, const float* d_states, int64_t batch,
                              int64_t n, int64_t state_dims, const float* d_fa,
                              float* d_state_adj, float* d_pos_adj, void* ws, size_t ws_bytes,
                              cudaStream_t st) {
  const GridParams g = make_grid_params(*cfg);
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  const PerceptionParams p = make_perception_params(g, *o, N, int(state_dims));
  PerceiveWorkspace w;
  const size_t extra = adjoint_extra_floats(g, total, state_dims);
  if (!carve_perceive(g, B, N, ws, ws_bytes, &w, extra))
    return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  float* density = w.tiles;
  float* dens_adj = density + total + 32;
  float* scratch = dens_adj + total + 32;
  if (total > 0) {
    NPA_TRY(launch_hashgrid(g, reinterpret_cast<const float4*>(d_positions), B, N, w.hg,
                            w.sort_scratch, w.sort_scratch_bytes, st));
    const SortedGrid sv = sorted_view(w, N, B, d_positions);
    NPA_TRY(launch_density(g, sv, B, w.volume, density, w.hits, st));
    return launch_perception_adjoint(g, p, sv, w.hg.inverse, B, d_states, int(state_dims),
                                     density, d_fa, scratch, d_state_adj,
                                     reinterpret_cast<float4*>(d_pos_adj), dens_adj, st);
  }
  return NPA_OK;
}

npa_status npa_perceive_adjoint_with_options(const npa_grid_config* cfg,
                                             const npa_perception_options* o,
                                             const float* positions, int64_t positions_len,
                                             const float* states, int64_t states_len,
                                             int64_t batch, int64_t n, int64_t state_dims,
                                             const float* feature_adjoint,
                                             int64_t feature_adjoint_len, float* state_adjoint,
                                             float* position_adjoint) {
  if (!o) return fail(NPA_ERR_INVALID_ARGUMENT, "options are null");
  NPA_TRY(check_counts(batch, n));
  if (state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "state_dims must be >= 0");
  NPA_TRY(check_shapes(positions_len, states_len, batch, n, state_dims));
  NPA_TRY(validate_grid(cfg));
  NPA_TRY(check_bins(cfg, batch));
  const GridParams g = make_grid_params(*cfg);
  const uint32_t B = uint32_t(batch), N = uint32_t(n), total = B * N;
  const PerceptionParams p = make_perception_params(g, *o, N, int(state_dims));
  NPA_TRY(output_shape(feature_adjoint_len, int64_t(total) * p.feature_dims));
  if (total > 0 && (!positions || (state_dims > 0 && (!states || !state_adjoint)) ||
                    (p.feature_dims > 0 && !feature_adjoint)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  int dev = 0;
  NPA_TRY(current_device(&dev));
  Scratch sc;
  NPA_TRY(sc.init());
  float4* dpos;
  float *dst, *dfa, *dsadj, *dpadj;
  char* ws;
  NPA_TRY(sc.upload(&dpos, positions, total));
  NPA_TRY(sc.upload(&dst, states, size_t(total) * state_dims));
  NPA_TRY(sc.upload(&dfa, feature_adjoint, size_t(total) * p.feature_dims));
  NPA_TRY(sc.alloc(&dsadj, size_t(total) * state_dims + 1));
  NPA_TRY(sc.alloc(&dpadj, size_t(total) * 4 + 4));
  const size_t wsb = perceive_workspace_bytes(g, B, N, adjoint_extra_floats(g, total, state_dims));
  NPA_TRY(sc.alloc(&ws, wsb));
  NPA_TRY(adjoint_run(cfg, o, reinterpret_cast<float*>(dpos), dst, batch, n, state_dims, dfa,
                      dsadj, dpadj, ws, wsb, sc.stream));
  NPA_TRY(sc.download(state_adjoint, dsadj, size_t(total) * state_dims * 4));
  NPA_TRY(sc.download(position_adjoint, dpadj, size_t(total) * 16));
  return sc.finish();
}

npa_status npa_dev_perceive_adjoint_workspace_size(const npa_grid_config* cfg, int64_t batch,
                                                   int64_t n, int64_t state_dims,
                                                   size_t* bytes) {
  NPA_TRY(validate_grid(cfg));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_bins(cfg, batch));
  if (!bytes || state_dims < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "bad argument");
  const GridParams g = make_grid_params(*cfg);
  const uint32_t total = uint32_t(batch * n);
  *bytes = perceive_workspace_bytes(g, uint32_t(batch), uint32_t(n),
                                    adjoint_extra_floats(g, total, state_dims));
  return NPA_OK;
}

npa_status npa_dev_perceive_adjoint_with_options(
    const npa_grid_config* cfg, const npa_perception_options* o, const float* d_positions,
    const float* d_states, int64_t batch, int64_t n, int64_t state_dims,
    const float* d_feature_adjoint, float* d_state_adjoint, float* d_position_adjoint,
    void* d_workspace, size_t workspace_bytes, void* stream) {
  if (!o) return fail(NPA_ERR_INVALID_ARGUMENT, "options are null");
  size_t need = 0;
  NPA_TRY(npa_dev_perceive_adjoint_workspace_size(cfg, batch, n, state_dims, &need));
  if (workspace_bytes < need) return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  if (batch * n > 0 && (!d_positions || !d_feature_adjoint || !d_position_adjoint ||
                        !d_workspace || (state_dims > 0 && (!d_states || !d_state_adjoint))))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  return adjoint_run(cfg, o, d_positions, d_states, batch, n, state_dims, d_feature_adjoint,
                     d_state_adjoint, d_position_adjoint, d_workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream));
}

static npa_status check_splat(const npa_splat2d_config* cfg, int64_t count) {
  if (!cfg) return fail(NPA_ERR_INVALID_ARGUMENT, "null config");
  if (cfg->image_size < 0 || cfg->image_size > 32768)
    return fail(NPA_ERR_INVALID_ARGUMENT, "image_size must be in [0, 32768]");
  if (count < 0 || count > int64_t(kMaxParticles))
    return fail(NPA_ERR_INVALID_ARGUMENT, "bad particle count");
  return NPA_OK;
}

npa_status npa_splat_particles_2d(const npa_splat2d_config* cfg, const float* positions,
                                  const float* colors, int64_t count, float* out,
                                  int64_t out_len) {
  NPA_TRY(check_splat(cfg, count));
  const int64_t pixels = cfg->image_size * cfg->image_size;
  NPA_TRY(output_shape(out_len, pixels * 4));
  if ((count > 0 && (!positions || !colors)) || (pixels > 0 && !out))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  int dev = 0;
  NPA_TRY(current_device(&dev));
  Scratch sc;
  NPA_TRY(sc.init());
  float4* dpos;
  float *dcol, *dout;
  char* ws;
  NPA_TRY(sc.upload(&dpos, positions, size_t(count)));
  NPA_TRY(sc.upload(&dcol, colors, size_t(count) * 3));
  NPA_TRY(sc.alloc(&dout, size_t(pixels) * 4));
  NPA_TRY(sc.alloc(&ws, splat_workspace_bytes(uint32_t(count))));
  NPA_TRY(launch_splat_2d(*cfg, dpos, dcol, uint32_t(count), reinterpret_cast<float4*>(dout), ws,
                          sc.stream));
  NPA_TRY(sc.download(out, dout, size_t(pixels) * 16));
  return sc.finish();
}

npa_status npa_dev_splat_workspace_size(int64_t count, size_t* bytes) {
  if (!bytes || count < 0 || count > int64_t(kMaxParticles))
    return fail(NPA_ERR_INVALID_ARGUMENT, "bad argument");
  *bytes = splat_workspace_bytes(uint32_t(count));
  return NPA_OK;
}

npa_status npa_dev_splat_particles_2d(const npa_splat2d_config* cfg, const float* d_positions,
                                      const float* d_colors, int64_t count, float* d_out,
                                      void* d_workspace, size_t workspace_bytes, void* stream) {
  NPA_TRY(check_splat(cfg, count));
  if (workspace_bytes < splat_workspace_bytes(uint32_t(count)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "workspace too small");
  if ((count > 0 && (!d_positions || !d_colors || !d_workspace)) ||
      (cfg->image_size > 0 && !d_out))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  return launch_splat_2d(*cfg, reinterpret_cast<const float4*>(d_positions), d_colors,
                         uint32_t(count), reinterpret_cast<float4*>(d_out), d_workspace,
                         static_cast<cudaStream_t>(stream));
}

// run_rollout_from_particles with the reference's StdRng masks when
// update_prob < 1 (no mask otherwise) and mean_dx when it is not null.
static npa_status run_rollout_impl(npa_model* m, const npa_grid_config* grid, float* positions,
                                   int64_t positions_len, float* states, int64_t states_len,
                                   int64_t batch, int64_t n, int64_t steps, float dt,
                                   float update_prob, uint64_t seed, float* mean_dx) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  NPA_TRY(check_step(m, grid));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_shapes(positions_len, states_len, batch, n, m->dm.state_dims));
  NPA_TRY(check_bins(grid, batch));
  if (steps < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "steps must be >= 0");
  const uint32_t total = uint32_t(batch * n);
  const int C = m->dm.state_dims;
  if (total > 0 && (!positions || (C > 0 && !states)))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  NPA_TRY(ensure_device(m->dm.device));
  if (total == 0) {
    if (mean_dx)
      for (int64_t k = 0; k < steps; ++k) mean_dx[k] = 0.0f;  // 0 / max(len, 1)
    return NPA_OK;
  }
  // stochastic_mask (rollout/mod.rs:644-651): ones without drawing when
  // update_prob >= 1, so no mask is applied then.
  const bool stochastic = !(update_prob >= 1.0f);
  const ChachaKey key = stdrng_key(seed ^ 0x5eedull);
  size_t wsb = 0;
  NPA_TRY(npa_dev_step_workspace_size(m, grid, batch, n, &wsb));
  Scratch sc;
  NPA_TRY(sc.init());
  float4 *pos[2], *ddx = nullptr;
  float *st[2], *dmean = nullptr, *mask = nullptr;
  double* partials = nullptr;
  char* ws;
  NPA_TRY(sc.upload(&pos[0], positions, total));
  NPA_TRY(sc.upload(&st[0], states, size_t(total) * C));
  NPA_TRY(sc.alloc(&pos[1], total));
  NPA_TRY(sc.alloc(&st[1], size_t(total) * C));
  if (mean_dx) {
    NPA_TRY(sc.alloc(&ddx, total));
    NPA_TRY(sc.alloc(&dmean, size_t(std::max<int64_t>(steps, 1))));
    NPA_TRY(sc.alloc(&partials, mean_norm_scratch_bytes() / sizeof(double)));
  }
  if (stochastic) NPA_TRY(sc.alloc(&mask, total));
  NPA_TRY(sc.alloc(&ws, wsb));
  int cur = 0;
  for (int64_t k = 0; k < steps; ++k) {
    if (stochastic)
      NPA_TRY(launch_stdrng_mask(key, uint64_t(k) * total, total, update_prob, mask, sc.stream));
    NPA_TRY(npa_dev_model_step(m, grid, reinterpret_cast<float*>(pos[cur]), st[cur], batch, n, dt,
                               mask, reinterpret_cast<float*>(pos[1 - cur]), st[1 - cur],
                               reinterpret_cast<float*>(ddx), nullptr, nullptr, nullptr, ws, wsb,
                               sc.stream));
    if (mean_dx) NPA_TRY(launch_mean_norm(ddx, total, partials, dmean + k, sc.stream));
    cur = 1 - cur;
  }
  NPA_TRY(sc.download(positions, pos[cur], size_t(total) * 16));
  NPA_TRY(sc.download(states, st[cur], size_t(total) * C * 4));
  if (mean_dx) NPA_TRY(sc.download(mean_dx, dmean, size_t(steps) * 4));
  NPA_TRY(sc.finish());
  return check_bulk_copies();
}

npa_status npa_model_run_rollout_trace(npa_model* m, const npa_grid_config* grid,
                                       float* positions, int64_t positions_len, float* states,
                                       int64_t states_len, int64_t batch, int64_t n,
                                       int64_t steps, float dt, float* mean_dx) {
  if (steps > 0 && !mean_dx) return fail(NPA_ERR_INVALID_ARGUMENT, "null mean_dx");
  return run_rollout_impl(m, grid, positions, positions_len, states, states_len, batch, n, steps,
                          dt, 1.0f, 0, mean_dx);
}

npa_status npa_model_run_rollout_seeded(npa_model* m, const npa_grid_config* grid,
                                        float* positions, int64_t positions_len, float* states,
                                        int64_t states_len, int64_t batch, int64_t n,
                                        int64_t steps, float dt, float update_prob, uint64_t seed,
                                        float* mean_dx) {
  return run_rollout_impl(m, grid, positions, positions_len, states, states_len, batch, n, steps,
                          dt, update_prob, seed, mean_dx);
}

npa_status npa_rollout_update_masks(uint64_t seed, float update_prob, int64_t count,
                                    int64_t first_step, int64_t steps, float* masks) {
  if (count < 0 || steps < 0 || first_step < 0)
    return fail(NPA_ERR_INVALID_ARGUMENT, "count, first_step and steps must be >= 0");
  if (count > int64_t(kMaxParticles)) return fail(NPA_ERR_UNSUPPORTED, "too many particles");
  const size_t len = size_t(count) * size_t(steps);
  if (len == 0) return NPA_OK;
  if (!masks) return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  if (update_prob >= 1.0f) {
    for (size_t i = 0; i < len; ++i) masks[i] = 1.0f;
    return NPA_OK;
  }
  int dev = 0;
  NPA_TRY(current_device(&dev));
  Scratch sc;
  NPA_TRY(sc.init());
  float* d;
  NPA_TRY(sc.alloc(&d, len));
  const ChachaKey key = stdrng_key(seed ^ 0x5eedull);
  for (int64_t k = 0; k < steps; ++k)
    NPA_TRY(launch_stdrng_mask(key, uint64_t(first_step + k) * uint64_t(count), uint32_t(count),
                               update_prob, d + size_t(k) * count, sc.stream));
  NPA_TRY(sc.download(masks, d, len * 4));
  return sc.finish();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Training rollout (crates/burn_automata/src/target2d.rs:3414-3722,
// crates/burn_automata/src/training.rs:558-640)
// ---------------------------------------------------------------------------
namespace {

// ensure_finite (training.rs:1053-1060).
npa_status ensure_finite_host(const char* name, const float* v, size_t count) {
  for (size_t i = 0; i < count; ++i)
    if (!std::isfinite(v[i])) return fail(NPA_ERR_INVALID_ARGUMENT, std::string(name) + " contain non-finite values");
  return NPA_OK;
}

// The training rollout's forward step is step_cpu's without the 3D position
// gates (rollout_for_training uses update_to_dx_ds + euler_step,
// target2d.rs:3430-3452); the step kernel would apply them.
npa_status check_training_model(const npa_model* m, const npa_grid_config* grid) {
  NPA_TRY(check_step(m, grid));
  if (grid->dim == 3 && m->cfg.position_features && m->dm.state_dims > 3)
    return fail(NPA_ERR_UNSUPPORTED,
                "the training rollout has no 3D position gates; models with 3D position "
                "features are not supported by it");
  return NPA_OK;
}

}  // namespace

extern "C" {

npa_status npa_model_mlp_backward(npa_model* m, const float* features, int64_t features_len,
                                  const float* output_gradients, int64_t output_gradients_len,
                                  float* gw1, float* gb1, float* gw2, float* gb2,
                                  float* gfeatures) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  const int64_t F = m->dm.feature_dims, H = m->dm.hidden_dims, O = m->dm.update_dims;
  const int64_t rows = F > 0 ? features_len / F : 0;
  if (rows == 0 || features_len != rows * F)
    return fail(NPA_ERR_INVALID_ARGUMENT, "features do not form whole perception rows");
  if (output_gradients_len != rows * O)
    return fail(NPA_ERR_INVALID_ARGUMENT, "output_gradients len " + std::to_string(output_gradients_len) +
                                              " != " + std::to_string(rows * O));
  if (rows > int64_t(kMaxParticles)) return fail(NPA_ERR_UNSUPPORTED, "too many rows");
  if (!features || !output_gradients || !gw1 || !gb1 || !gw2 || !gb2 || !gfeatures)
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  NPA_TRY(ensure_finite_host("features", features, size_t(features_len)));
  NPA_TRY(ensure_finite_host("output_gradients", output_gradients, size_t(output_gradients_len)));
  NPA_TRY(ensure_device(m->dm.device));
  const uint32_t R = uint32_t(rows);
  Scratch sc;
  NPA_TRY(sc.init());
  float *df, *dg, *dhid, *dpre, *dgf, *dw;
  NPA_TRY(sc.upload(&df, features, size_t(features_len)));
  NPA_TRY(sc.upload(&dg, output_gradients, size_t(output_gradients_len)));
  NPA_TRY(sc.alloc(&dhid, size_t(R) * H));
  NPA_TRY(sc.alloc(&dpre, size_t(R) * H));
  NPA_TRY(sc.alloc(&dgf, size_t(R) * F));
  const size_t nw = size_t(H * F + H + O * H + O);
  NPA_TRY(sc.alloc(&dw, nw));
  NPA_CUDA(cudaMemsetAsync(dw, 0, nw * 4, sc.stream), "cudaMemsetAsync");
  float* dgw1 = dw;
  float* dgb1 = dgw1 + H * F;
  float* dgw2 = dgb1 + H;
  float* dgb2 = dgw2 + O * H;
  NPA_TRY(launch_mlp_backward(m->dm, df, dg, R, dhid, dpre, dgf, dgw1, dgb1, dgw2, dgb2, sc.stream));
  NPA_TRY(sc.download(gw1, dgw1, size_t(H * F) * 4));
  NPA_TRY(sc.download(gb1, dgb1, size_t(H) * 4));
  NPA_TRY(sc.download(gw2, dgw2, size_t(O * H) * 4));
  NPA_TRY(sc.download(gb2, dgb2, size_t(O) * 4));
  NPA_TRY(sc.download(gfeatures, dgf, size_t(R) * F * 4));
  NPA_TRY(sc.finish());
  // validate_gradients (training.rs:1017-1023)
  NPA_TRY(ensure_finite_host("w1 gradients", gw1, size_t(H * F)));
  NPA_TRY(ensure_finite_host("b1 gradients", gb1, size_t(H)));
  NPA_TRY(ensure_finite_host("w2 gradients", gw2, size_t(O * H)));
  NPA_TRY(ensure_finite_host("b2 gradients", gb2, size_t(O)));
  return ensure_finite_host("feature gradients", gfeatures, size_t(R) * F);
}

npa_status npa_model_rollout_for_training(npa_model* m, const npa_grid_config* grid,
                                          const float* positions, int64_t positions_len,
                                          const float* states, int64_t states_len, int64_t batch,
                                          int64_t n, int64_t steps, float update_prob,
                                          uint64_t seed, float* snapshot_positions,
                                          float* snapshot_states, float* snapshot_masks,
                                          float* final_positions, float* final_states,
                                          float* mean_dx_norm_sum) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  NPA_TRY(check_training_model(m, grid));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_shapes(positions_len, states_len, batch, n, m->dm.state_dims));
  NPA_TRY(check_bins(grid, batch));
  if (steps < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "steps must be >= 0");
  const uint32_t total = uint32_t(batch * n);
  const int C = m->dm.state_dims;
  if (!mean_dx_norm_sum || (total > 0 && (!positions || !final_positions ||
                                          (C > 0 && (!states || !final_states)) ||
                                          (steps > 0 && (!snapshot_positions || !snapshot_masks ||
                                                         (C > 0 && !snapshot_states))))))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  NPA_TRY(ensure_device(m->dm.device));
  *mean_dx_norm_sum = 0.0f;
  if (total == 0) return NPA_OK;
  // stochastic_mask draws of StdRng::seed_from_u64(seed ^ 0x5eed2d), one
  // stream for the whole rollout (target2d.rs:3425-3429); ones without
  // drawing when update_prob >= 1 (rollout/mod.rs:644-651).
  const bool stochastic = !(update_prob >= 1.0f);
  const ChachaKey key = stdrng_key(seed ^ 0x5eed2dull);
  size_t wsb = 0;
  NPA_TRY(npa_dev_step_workspace_size(m, grid, batch, n, &wsb));
  Scratch sc;
  NPA_TRY(sc.init());
  float4 *pos[2], *ddx, *snap_p;
  float *st[2], *dmean, *mask, *snap_s = nullptr, *snap_m;
  double* partials;
  char* ws;
  const int64_t S = std::max<int64_t>(steps, 1);
  NPA_TRY(sc.upload(&pos[0], positions, total));
  NPA_TRY(sc.upload(&st[0], states, size_t(total) * C));
  NPA_TRY(sc.alloc(&pos[1], total));
  NPA_TRY(sc.alloc(&st[1], size_t(total) * C));
  NPA_TRY(sc.alloc(&ddx, total));
  NPA_TRY(sc.alloc(&dmean, size_t(S)));
  NPA_TRY(sc.alloc(&partials, mean_norm_scratch_bytes() / sizeof(double)));
  NPA_TRY(sc.alloc(&mask, total));
  NPA_TRY(sc.alloc(&snap_p, size_t(S) * total));
  if (C > 0) NPA_TRY(sc.alloc(&snap_s, size_t(S) * total * C));
  NPA_TRY(sc.alloc(&snap_m, size_t(S) * total));
  NPA_TRY(sc.alloc(&ws, wsb));
  if (!stochastic) {
    std::vector<float> ones(total, 1.0f);
    NPA_CUDA(cudaMemcpyAsync(mask, ones.data(), size_t(total) * 4, cudaMemcpyHostToDevice, sc.stream),
             "cudaMemcpyAsync");
    NPA_CUDA(cudaStreamSynchronize(sc.stream), "cudaStreamSynchronize");
  }
  int cur = 0;
  for (int64_t k = 0; k < steps; ++k) {
    if (stochastic)
      NPA_TRY(launch_stdrng_mask(key, uint64_t(k) * total, total, update_prob, mask, sc.stream));
    NPA_CUDA(cudaMemcpyAsync(snap_p + size_t(k) * total, pos[cur], size_t(total) * 16,
                             cudaMemcpyDeviceToDevice, sc.stream), "cudaMemcpyAsync");
    if (C > 0)
      NPA_CUDA(cudaMemcpyAsync(snap_s + size_t(k) * total * C, st[cur], size_t(total) * C * 4,
                               cudaMemcpyDeviceToDevice, sc.stream), "cudaMemcpyAsync");
    NPA_CUDA(cudaMemcpyAsync(snap_m + size_t(k) * total, mask, size_t(total) * 4,
                             cudaMemcpyDeviceToDevice, sc.stream), "cudaMemcpyAsync");
    NPA_TRY(npa_dev_model_step(m, grid, reinterpret_cast<float*>(pos[cur]), st[cur], batch, n, 1.0f,
                               mask, reinterpret_cast<float*>(pos[1 - cur]), st[1 - cur],
                               reinterpret_cast<float*>(ddx), nullptr, nullptr, nullptr, ws, wsb,
                               sc.stream));
    NPA_TRY(launch_mean_norm(ddx, total, partials, dmean + k, sc.stream));
    cur = 1 - cur;
  }
  std::vector<float> means(size_t(S), 0.0f);
  NPA_TRY(sc.download(final_positions, pos[cur], size_t(total) * 16));
  if (C > 0) NPA_TRY(sc.download(final_states, st[cur], size_t(total) * C * 4));
  if (steps > 0) {
    NPA_TRY(sc.download(snapshot_positions, snap_p, size_t(steps) * total * 16));
    if (C > 0) NPA_TRY(sc.download(snapshot_states, snap_s, size_t(steps) * total * C * 4));
    NPA_TRY(sc.download(snapshot_masks, snap_m, size_t(steps) * total * 4));
    NPA_TRY(sc.download(means.data(), dmean, size_t(steps) * 4));
  }
  NPA_TRY(sc.finish());
  NPA_TRY(check_bulk_copies());
  // mean_dx_norm_sum += mean_dx_norm(dx) per step, in f32 (target2d.rs:3434)
  float sum = 0.0f;
  for (int64_t k = 0; k < steps; ++k) sum = sum + means[size_t(k)];
  *mean_dx_norm_sum = sum;
  return NPA_OK;
}

npa_status npa_model_bptt_gradients(npa_model* m, const npa_grid_config* grid,
                                    const float* snapshot_positions, const float* snapshot_states,
                                    const float* snapshot_masks, int64_t batch, int64_t n,
                                    int64_t steps, const float* position_gradients,
                                    const float* state_gradients,
                                    float displacement_regularizer_weight, int32_t stopgrad_pos,
                                    int32_t stopgrad_state, float* gw1, float* gb1, float* gw2,
                                    float* gb2, float* initial_position_adjoint,
                                    float* initial_state_adjoint) {
  if (!m) return fail(NPA_ERR_INVALID_ARGUMENT, "null model");
  NPA_TRY(check_training_model(m, grid));
  NPA_TRY(check_counts(batch, n));
  NPA_TRY(check_bins(grid, batch));
  if (steps < 0) return fail(NPA_ERR_INVALID_ARGUMENT, "steps must be >= 0");
  const uint32_t total = uint32_t(batch * n);
  // mlp_backward_from_output_gradients rejects a step with no rows
  if (total == 0 && steps > 0)
    return fail(NPA_ERR_INVALID_ARGUMENT, "features do not form whole perception rows");
  const int C = m->dm.state_dims, D = m->dm.spatial_dims, H = m->dm.hidden_dims;
  const int F = m->dm.feature_dims, O = m->dm.update_dims;
  if (!gw1 || !gb1 || !gw2 || !gb2 ||
      (total > 0 && (!position_gradients || (C > 0 && !state_gradients) ||
                     (steps > 0 && (!snapshot_positions || !snapshot_masks ||
                                    (C > 0 && !snapshot_states))))))
    return fail(NPA_ERR_INVALID_ARGUMENT, "null buffer");
  NPA_TRY(ensure_device(m->dm.device));
  const npa_perception_options opt = model_options(m->cfg);
  const float motion_eps =
      m->dm.equivariance == NPA_EQUIV_PARTICLE_DENSITY_AND_SCALE ? grid->eps : m->dm.eps0;
  const float scale = m->dm.alpha * motion_eps;
  // displacement_scale (target2d.rs:3568-3572)
  const float reg = displacement_regularizer_weight == 0.0f
                        ? 0.0f
                        : displacement_regularizer_weight / float(std::max<uint32_t>(total, 1u));
  size_t pws = 0, aws = 0;
  NPA_TRY(npa_dev_perceive_workspace_size(grid, batch, n, C, &pws));
  NPA_TRY(npa_dev_perceive_adjoint_workspace_size(grid, batch, n, C, &aws));
  Scratch sc;
  NPA_TRY(sc.init());
  const size_t T = std::max<uint32_t>(total, 1u);
  float4 *pos, *padj, *ppos;
  float *stt = nullptr, *sadj = nullptr, *pst = nullptr, *mask, *feat, *upd, *oadj, *hid, *dpre,
        *gfeat, *dw;
  int* flag;
  char *pw, *aw;
  NPA_TRY(sc.alloc(&pos, T));
  NPA_TRY(sc.alloc(&stt, T * std::max(C, 1)));
  NPA_TRY(sc.alloc(&mask, T));
  NPA_TRY(sc.alloc(&padj, T));
  NPA_TRY(sc.alloc(&sadj, T * std::max(C, 1)));
  NPA_TRY(sc.alloc(&ppos, T));
  NPA_TRY(sc.alloc(&pst, T * std::max(C, 1)));
  NPA_TRY(sc.alloc(&feat, T * F));
  NPA_TRY(sc.alloc(&upd, T * O));
  NPA_TRY(sc.alloc(&oadj, T * O));
  NPA_TRY(sc.alloc(&hid, T * H));
  NPA_TRY(sc.alloc(&dpre, T * H));
  NPA_TRY(sc.alloc(&gfeat, T * F));
  const size_t nw = size_t(H) * F + H + size_t(O) * H + O;
  NPA_TRY(sc.alloc(&dw, nw));
  NPA_TRY(sc.alloc(&flag, 1));
  NPA_TRY(sc.alloc(&pw, pws));
  NPA_TRY(sc.alloc(&aw, aws));
  float* dgw1 = dw;
  float* dgb1 = dgw1 + size_t(H) * F;
  float* dgw2 = dgb1 + H;
  float* dgb2 = dgw2 + size_t(O) * H;
  cudaStream_t s = sc.stream;
  NPA_CUDA(cudaMemsetAsync(dw, 0, nw * 4, s), "cudaMemsetAsync");
  NPA_CUDA(cudaMemsetAsync(flag, 0, 4, s), "cudaMemsetAsync");
  if (total > 0) {
    NPA_CUDA(cudaMemcpyAsync(padj, position_gradients, size_t(total) * 16, cudaMemcpyHostToDevice, s),
             "cudaMemcpyAsync");
    if (C > 0)
      NPA_CUDA(cudaMemcpyAsync(sadj, state_gradients, size_t(total) * C * 4, cudaMemcpyHostToDevice, s),
               "cudaMemcpyAsync");
  }
  for (int64_t k = steps - 1; k >= 0 && total > 0; --k) {
    NPA_CUDA(cudaMemcpyAsync(pos, snapshot_positions + size_t(k) * total * 4, size_t(total) * 16,
                             cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
    if (C > 0)
      NPA_CUDA(cudaMemcpyAsync(stt, snapshot_states + size_t(k) * total * C, size_t(total) * C * 4,
                               cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
    NPA_CUDA(cudaMemcpyAsync(mask, snapshot_masks + size_t(k) * total, size_t(total) * 4,
                             cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
    // features and raw update of the recorded step (target2d.rs:3570-3579)
    NPA_TRY(npa_dev_perceive_with_options(grid, &opt, reinterpret_cast<float*>(pos), stt, batch, n,
                                          C, feat, nullptr, nullptr, nullptr, nullptr, pw, pws, s));
    NPA_TRY(launch_forward_update(m->dm, feat, total, upd, s));
    NPA_TRY(launch_output_adjoint(upd, padj, sadj, mask, total, D, C, scale, reg, oadj, s));
    // ensure_finite of mlp_backward_from_output_gradients' inputs (training.rs:577-578)
    NPA_TRY(launch_finite_check(feat, uint64_t(total) * F, flag, 1, s));
    NPA_TRY(launch_finite_check(oadj, uint64_t(total) * O, flag, 2, s));
    NPA_TRY(launch_mlp_backward(m->dm, feat, oadj, total, hid, dpre, gfeat, dgw1, dgb1, dgw2, dgb2, s));
    NPA_TRY(launch_finite_check(gfeat, uint64_t(total) * F, flag, 4, s));
    // perception adjoint of the step, added to the running adjoints
    NPA_TRY(npa_dev_perceive_adjoint_with_options(grid, &opt, reinterpret_cast<float*>(pos), stt,
                                                  batch, n, C, gfeat, pst,
                                                  reinterpret_cast<float*>(ppos), aw, aws, s));
    NPA_TRY(launch_add_adjoint(padj, sadj, ppos, pst, total, D, C, !stopgrad_pos, !stopgrad_state, s));
    // the snapshot buffers are refilled next step: finish this one first
    NPA_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  }
  int fl = 0;
  NPA_TRY(sc.download(&fl, flag, 4));
  NPA_TRY(sc.download(gw1, dgw1, size_t(H) * F * 4));
  NPA_TRY(sc.download(gb1, dgb1, size_t(H) * 4));
  NPA_TRY(sc.download(gw2, dgw2, size_t(O) * H * 4));
  NPA_TRY(sc.download(gb2, dgb2, size_t(O) * 4));
  if (initial_position_adjoint && total > 0)
    NPA_TRY(sc.download(initial_position_adjoint, padj, size_t(total) * 16));
  if (initial_state_adjoint && total > 0 && C > 0)
    NPA_TRY(sc.download(initial_state_adjoint, sadj, size_t(total) * C * 4));
  NPA_TRY(sc.finish());
  if (fl & 1) return fail(NPA_ERR_INVALID_ARGUMENT, "features contain non-finite values");
  if (fl & 2) return fail(NPA_ERR_INVALID_ARGUMENT, "output_gradients contain non-finite values");
  if (fl & 4) return fail(NPA_ERR_INVALID_ARGUMENT, "feature gradients contain non-finite values");
  NPA_TRY(ensure_finite_host("w1 gradients", gw1, size_t(H) * F));
  NPA_TRY(ensure_finite_host("b1 gradients", gb1, size_t(H)));
  NPA_TRY(ensure_finite_host("w2 gradients", gw2, size_t(O) * H));
  return ensure_finite_host("b2 gradients", gb2, size_t(O));
}

}  // extern "C"
