// host_log1p.cu -- the host C library's log1pf, reproduced bit for bit on the device.
//
// The reference's log-normalisation (log_normalize_vector,
// crates/burn_automata_kernels/src/reference/normalize.rs:60-69) calls
// f32::ln_1p, which rustc binds to the host C library's log1pf.  That
// function is not correctly rounded: on Linux x86-64 (glibc 2.39) it returns
// the neighbouring float of the correctly rounded ln(1 + x) for about 9.1 M
// of the 1.06 G floats in [1e-6, inf), always exactly one ulp away.  A rollout
// is chaotic, so one such ulp grows over tens of steps into differences far
// above the 64-step tolerance; to follow the reference's trajectory the device
// must return the host's value itself.
//
// What the host returns is recorded by CALLING the host's log1pf on every
// float in [1e-6, inf) and comparing with the correctly rounded value c (ln(1 +
// x) in f64, rounded once); no part of the C library's implementation is
// restated, only its outputs:
//   differ  the inputs where the host's result is not c.  Except for those of
//           the side list, the host's result is then c's neighbour on the
//           side of the f64 value (the host is off by less than 1.5 ulp);
//   side    the inputs whose host result is stored outright: the differing
//           ones whose result is the neighbour on the far side (one on glibc
//           2.39), and every input whose f64 value lies within 1e-8 of a float
//           gap from a rounding midpoint, where two f64 log1p implementations
//           (each within an ulp or two of f64) may round to different floats.
// On each device a setup kernel turns that into the table the kernels use:
// for every input, the host's result relative to CUDA's f32 log1pf (f) as a
// 2-bit code -- same, one ulp up, one ulp down, or stored in a sorted list --
// so a kernel evaluates ln_1p with one f32 log1pf, one table word (norms of
// similar size share words, which stay resident in L2 / L1) and an add.
//
// Inputs below 1e-6 are not tabulated (the device returns CUDA's log1pf): the
// reference's norm is max(sqrt(|v|^2 + 1e-12), 1e-6) >= 1e-6, so
// log-normalisation never passes a smaller value.
//
// The scan (two libm calls per float, ~17 CPU-seconds) runs once per host
// library: the list of differing inputs is cached next to this library
// (libnpa_b200.so.log1pf) and re-validated against the running host's log1pf
// when loaded; a cache that disagrees is rebuilt.  The device table (2 bits per
// input, 256 MiB, plus the list of stored results) is built on first use on a
// device and kept until process exit.
#include <dlfcn.h>
#include <unistd.h>
#include <gnu/libc-version.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "npa_internal.h"

namespace npa {
namespace {

constexpr double kHostNear = 1e-8;            // host: every input this close is in side
constexpr int kMaxSide = 256;                 // side list capacity
constexpr uint32_t kFileMagic = 0x4650314cu;  // "L1PF"
constexpr uint32_t kFileVersion = 2;

struct HostTables {
  std::vector<uint32_t> differ;     // inputs whose host result is not c, ascending
  std::vector<uint32_t> side_keys;  // inputs of the side list, ascending
  std::vector<uint32_t> side_vals;  // their host log1pf result bits
};

// Distance of v from the f32 rounding midpoint next to c = (float)v, in units
// of the gap between c and that neighbour; the neighbour's bits.
inline double midpoint_distance(double v, float c, float* other) {
  uint32_t cb;
  std::memcpy(&cb, &c, 4);
  const double cd = c;
  const uint32_t ob = cd < v ? cb + 1 : cb - 1;  // c > 0 on the tabulated range
  float o;
  std::memcpy(&o, &ob, 4);
  *other = o;
  const double gap = std::fabs(double(o) - cd);
  return std::fabs(v - 0.5 * (cd + double(o))) / gap;
}

float table_min() { return 1e-6f; }

void scan_range(uint32_t lo, uint32_t hi, HostTables* out) {
  for (uint64_t b = lo; b < hi; ++b) {
    const uint32_t u = static_cast<uint32_t>(b);
    float x;
    std::memcpy(&x, &u, 4);
    const float g = log1pf(x);
    const double v = log1p(static_cast<double>(x));
    const float c = static_cast<float>(v);
    float o;
    const double d = midpoint_distance(v, c, &o);
    uint32_t gb;
    std::memcpy(&gb, &g, 4);
    if (g != c) out->differ.push_back(u);
    if (d < kHostNear || (g != c && g != o)) {
      out->side_keys.push_back(u);
      out->side_vals.push_back(gb);
    }
  }
}

HostTables scan_host() {
  float lo_f = table_min();
  uint32_t lo;
  std::memcpy(&lo, &lo_f, 4);
  const uint32_t hi = 0x7f800000u;  // +inf excluded
  unsigned threads = std::max(1u, std::thread::hardware_concurrency());
  const uint32_t chunks = threads * 8;
  std::vector<HostTables> parts(chunks);
  std::atomic<uint32_t> next{0};
  std::vector<std::thread> pool;
  for (unsigned t = 0; t < threads; ++t)
    pool.emplace_back([&] {
      for (uint32_t k; (k = next.fetch_add(1)) < chunks;) {
        const uint64_t span = uint64_t(hi - lo);
        const uint32_t a = lo + static_cast<uint32_t>(span * k / chunks);
        const uint32_t b = lo + static_cast<uint32_t>(span * (k + 1) / chunks);
        scan_range(a, b, &parts[k]);
      }
    });
  for (auto& th : pool) th.join();
  HostTables all;
  for (auto& p : parts) {
    all.differ.insert(all.differ.end(), p.differ.begin(), p.differ.end());
    all.side_keys.insert(all.side_keys.end(), p.side_keys.begin(), p.side_keys.end());
    all.side_vals.insert(all.side_vals.end(), p.side_vals.begin(), p.side_vals.end());
  }
  return all;
}

std::string cache_path() {
  if (const char* env = std::getenv("NPA_LOG1PF_CACHE")) return env;
  Dl_info info;
  if (dladdr(reinterpret_cast<void*>(&scan_host), &info) && info.dli_fname)
    return std::string(info.dli_fname) + ".log1pf";
  return "libnpa_b200.so.log1pf";
}

// A cache is accepted when it was written for this C library version and
// every recorded entry of a spot-check sample still holds on this host.
bool entries_hold(const HostTables& t) {
  const size_t n = t.differ.size();
  if (n == 0 || t.side_keys.size() > size_t(kMaxSide)) return false;
  for (size_t k = 0; k < 4096; ++k) {
    const uint32_t u = t.differ[(k * 2654435761ull) % n];
    float x;
    std::memcpy(&x, &u, 4);
    if (log1pf(x) == static_cast<float>(log1p(static_cast<double>(x)))) return false;
  }
  for (size_t k = 0; k < t.side_keys.size(); ++k) {
    float x, want;
    std::memcpy(&x, &t.side_keys[k], 4);
    std::memcpy(&want, &t.side_vals[k], 4);
    if (log1pf(x) != want) return false;
  }
  return true;
}

bool read_cache(const std::string& path, HostTables* t) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  uint32_t head[4];
  char ver[32] = {0};
  uint64_t nm = 0, ns = 0;
  bool ok = std::fread(head, 4, 4, f) == 4 && head[0] == kFileMagic && head[1] == kFileVersion &&
            std::fread(ver, 1, 32, f) == 32 && std::fread(&nm, 8, 1, f) == 1 &&
            std::fread(&ns, 8, 1, f) == 1 && nm < (uint64_t(1) << 28) && ns <= uint64_t(kMaxSide);
  ok = ok && std::strncmp(ver, gnu_get_libc_version(), 31) == 0;
  if (ok) {
    // differing inputs: varint of the delta to the previous one
    t->differ.resize(nm);
    uint32_t prev = 0;
    for (uint64_t i = 0; ok && i < nm; ++i) {
      uint64_t v = 0;
      int shift = 0;
      for (;;) {
        const int ch = std::fgetc(f);
        if (ch == EOF || shift > 35) {
          ok = false;
          break;
        }
        v |= uint64_t(ch & 0x7f) << shift;
        shift += 7;
        if (!(ch & 0x80)) break;
      }
      const uint32_t u = prev + static_cast<uint32_t>(v);
      t->differ[i] = u;
      prev = u;
    }
    t->side_keys.resize(ns);
    t->side_vals.resize(ns);
    ok = ok && std::fread(t->side_keys.data(), 4, ns, f) == ns &&
         std::fread(t->side_vals.data(), 4, ns, f) == ns;
  }
  std::fclose(f);
  return ok && entries_hold(*t);
}

void write_cache(const std::string& path, const HostTables& t) {
  const std::string tmp = path + ".tmp" + std::to_string(static_cast<long>(getpid()));
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) return;
  const uint32_t head[4] = {kFileMagic, kFileVersion, 0, 0};
  char ver[32] = {0};
  std::strncpy(ver, gnu_get_libc_version(), 31);
  const uint64_t nm = t.differ.size(), ns = t.side_keys.size();
  bool ok = std::fwrite(head, 4, 4, f) == 4 && std::fwrite(ver, 1, 32, f) == 32 &&
            std::fwrite(&nm, 8, 1, f) == 1 && std::fwrite(&ns, 8, 1, f) == 1;
  uint32_t prev = 0;
  for (uint64_t i = 0; ok && i < nm; ++i) {
    const uint32_t u = t.differ[i];
    uint64_t v = uint64_t(u - prev);
    prev = u;
    do {
      const int ch = int(v & 0x7f) | (v > 0x7f ? 0x80 : 0);
      ok = std::fputc(ch, f) != EOF;
      v >>= 7;
    } while (ok && v);
  }
  ok = ok && std::fwrite(t.side_keys.data(), 4, ns, f) == ns &&
       std::fwrite(t.side_vals.data(), 4, ns, f) == ns;
  ok = (std::fclose(f) == 0) && ok;
  if (ok)
    std::rename(tmp.c_str(), path.c_str());
  else
    std::remove(tmp.c_str());
}

std::mutex g_host_mu;
HostTables* g_host = nullptr;

const HostTables& host_tables() {
  std::lock_guard<std::mutex> lock(g_host_mu);
  if (!g_host) {
    auto* t = new HostTables();
    const std::string path = cache_path();
    if (!read_cache(path, t)) {
      *t = scan_host();
      write_cache(path, *t);
    }
    g_host = t;
  }
  return *g_host;
}

struct DeviceTables {
  uint32_t* codes = nullptr;
  uint2* side = nullptr;
  uint32_t base = 0;
  uint32_t nbits = 0;
  int nside = 0;
};

std::mutex g_dev_mu;
std::vector<DeviceTables> g_dev;  // by device ordinal

uint32_t range_base() {
  const float lo = table_min();
  uint32_t u;
  std::memcpy(&u, &lo, 4);
  return u;
}

constexpr uint32_t kSideCapacity = 1u << 16;  // inputs whose code is 3 (stored outright)

// One thread per 16 inputs (one word of 2-bit codes).  For each input x:
// the host's log1pf g (the correctly rounded value c = f64 log1p rounded once,
// moved to the neighbour on the f64 value's side where the host bitmap says
// the host differs, or taken from the host's side list), CUDA's log1pf f, and
// the code of g relative to f: 0 same, 1 one ulp up, 2 one ulp down, 3 stored
// in the side list (appended, unordered; sorted on the host afterwards).
__global__ void build_codes_kernel(const uint32_t* __restrict__ host_bits,
                                   const uint2* __restrict__ host_side, int host_nside,
                                   uint32_t base, uint32_t nbits, uint32_t* __restrict__ codes,
                                   uint2* __restrict__ side_out, uint32_t* __restrict__ side_count) {
  const uint32_t words = (nbits + 15u) / 16u;
  for (uint32_t w = blockIdx.x * blockDim.x + threadIdx.x; w < words; w += gridDim.x * blockDim.x) {
    uint32_t word = 0;
    for (uint32_t j = 0; j < 16u; ++j) {
      const uint32_t i = w * 16u + j;
      if (i >= nbits) break;
      const uint32_t u = base + i;
      const float x = __uint_as_float(u);
      const double v = log1p(static_cast<double>(x));
      const float c = static_cast<float>(v);
      const uint32_t cb = __float_as_uint(c);
      const double cd = c;
      const float o = __uint_as_float(cd < v ? cb + 1u : cb - 1u);  // c > 0 on the range
      const double gap = fabs(static_cast<double>(o) - cd);
      const bool near = fabs(v - 0.5 * (cd + static_cast<double>(o))) < 5e-9 * gap;
      const bool differs = (__ldg(host_bits + (i >> 5)) >> (i & 31u)) & 1u;
      float g = differs ? o : c;
      if (differs || near)
        for (int k = 0; k < host_nside; ++k) {
          const uint2 e = __ldg(host_side + k);
          if (e.x == u) g = __uint_as_float(e.y);
        }
      const float f = log1pf(x);
      const int diff = static_cast<int>(__float_as_uint(g) - __float_as_uint(f));
      const uint32_t code = diff == 0 ? 0u : diff == 1 ? 1u : diff == -1 ? 2u : 3u;
      if (code == 3u) {
        const uint32_t slot = atomicAdd(side_count, 1u);
        if (slot < kSideCapacity) side_out[slot] = make_uint2(u, __float_as_uint(g));
      }
      word |= code << (2u * j);
    }
    codes[w] = word;
  }
}

npa_status upload(const HostTables& h, DeviceTables* out) {
  if (h.side_keys.size() > size_t(kMaxSide))
    return fail(NPA_ERR_UNSUPPORTED, "log1pf side list larger than its capacity");
  const uint32_t base = range_base();
  const uint32_t nbits = 0x7f800000u - base;
  const size_t bit_words = (size_t(nbits) + 31) / 32;
  const size_t code_words = (size_t(nbits) + 15) / 16;
  std::vector<uint32_t> bits(bit_words, 0u);
  for (uint32_t u : h.differ) {
    const uint32_t i = u - base;
    bits[i >> 5] |= 1u << (i & 31);
  }
  std::vector<uint2> hside(std::max<size_t>(h.side_keys.size(), 1), make_uint2(0xffffffffu, 0));
  for (size_t i = 0; i < h.side_keys.size(); ++i)
    hside[i] = make_uint2(h.side_keys[i], h.side_vals[i]);
  // Temporaries (the host bitmap and side list, the unordered code-3 list and
  // its count) live only while the codes are built.
  uint32_t* d_bits = nullptr;
  uint2* d_hside = nullptr;
  uint2* d_out = nullptr;
  uint32_t* d_count = nullptr;
  DeviceTables d;
  auto release = [&]() {
    cudaFree(d_bits);
    cudaFree(d_hside);
    cudaFree(d_out);
    cudaFree(d_count);
  };
  cudaError_t e = cudaMalloc(&d_bits, bit_words * 4);
  if (e == cudaSuccess) e = cudaMalloc(&d_hside, hside.size() * sizeof(uint2));
  if (e == cudaSuccess) e = cudaMalloc(&d_out, kSideCapacity * sizeof(uint2));
  if (e == cudaSuccess) e = cudaMalloc(&d_count, 4);
  if (e == cudaSuccess) e = cudaMalloc(&d.codes, code_words * 4);
  // synchronous copies followed by a device synchronisation: a pageable-memory
  // cudaMemcpy may return before its DMA ends
  if (e == cudaSuccess) e = cudaMemcpy(d_bits, bits.data(), bit_words * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(d_hside, hside.data(), hside.size() * sizeof(uint2), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(d_count, 0, 4);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) {
    build_codes_kernel<<<148 * 8, 256>>>(d_bits, d_hside, int(h.side_keys.size()), base, nbits,
                                         d.codes, d_out, d_count);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  uint32_t count = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&count, d_count, 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    release();
    cudaFree(d.codes);
    return cuda_fail(e, "building the log1pf code table");
  }
  if (count > kSideCapacity) {
    release();
    cudaFree(d.codes);
    return fail(NPA_ERR_UNSUPPORTED, "log1pf: more stored results than the side list holds");
  }
  std::vector<uint2> side(std::max<uint32_t>(count, 1u), make_uint2(0xffffffffu, 0));
  if (count) e = cudaMemcpy(side.data(), d_out, count * sizeof(uint2), cudaMemcpyDeviceToHost);
  std::sort(side.begin(), side.begin() + count,
            [](const uint2& a, const uint2& b) { return a.x < b.x; });
  if (e == cudaSuccess) e = cudaMalloc(&d.side, side.size() * sizeof(uint2));
  if (e == cudaSuccess)
    e = cudaMemcpy(d.side, side.data(), side.size() * sizeof(uint2), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  release();
  if (e != cudaSuccess) {
    cudaFree(d.codes);
    cudaFree(d.side);
    return cuda_fail(e, "uploading the log1pf side list");
  }
  d.base = base;
  d.nbits = nbits;
  d.nside = int(count);
  *out = d;
  return NPA_OK;
}

Log1pTable as_table(const DeviceTables& d) {
  return Log1pTable{d.codes, d.side, d.base, d.nbits, d.nside, table_min()};
}

}  // namespace

npa_status prepare_host_log1p() {
  host_tables();
  return NPA_OK;
}

npa_status device_log1p_table(Log1pTable* out, cudaStream_t stream) {
  int dev = 0;
  NPA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (dev < int(g_dev.size()) && g_dev[dev].codes) {
      *out = as_table(g_dev[dev]);
      return NPA_OK;
    }
  }
  const HostTables& h = host_tables();
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (dev >= int(g_dev.size())) g_dev.resize(dev + 1);
  if (!g_dev[dev].codes) {
    if (stream) {
      cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
      NPA_CUDA(cudaStreamIsCapturing(stream, &cap), "cudaStreamIsCapturing");
      if (cap != cudaStreamCaptureStatusNone)
        return fail(NPA_ERR_INVALID_ARGUMENT,
                    "the first call on a device uploads its log1pf tables and cannot be captured: "
                    "make it (or npa_prepare_device) before stream capture");
    }
    NPA_TRY(upload(h, &g_dev[dev]));
  }
  *out = as_table(g_dev[dev]);
  return NPA_OK;
}

size_t host_log1p_exceptions() { return host_tables().differ.size(); }

namespace {
__global__ void ln_1p_kernel(const float* __restrict__ x, uint64_t count, Log1pTable t,
                             float* __restrict__ out) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
       i += uint64_t(gridDim.x) * blockDim.x)
    out[i] = log1p_host(__ldg(x + i), t);
}
}  // namespace

npa_status launch_ln_1p(const float* x, uint64_t count, float* out, cudaStream_t stream) {
  if (count == 0) return NPA_OK;
  Log1pTable t;
  NPA_TRY(device_log1p_table(&t, stream));
  const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>((count + 255) / 256, 148u * 16u));
  ln_1p_kernel<<<blocks, 256, 0, stream>>>(x, count, t, out);
  return after_launch("ln_1p_kernel");
}

}  // namespace npa
