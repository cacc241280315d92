// pipe_probe.cu -- the FP32 pipe's practical ceiling for the MLP's inner loop.
//
// The MLP runs in the reference's operation order: every multiply-add is a
// rounded multiply and a separate rounded add, so it is bound by the FP32 pipe
// at two instructions per multiply-add (148 SMs x 128 lanes x clock).  This
// probe runs only the layer-1 register tile of mlp_step_kernel -- per k, two
// 16-byte shared loads of 8 feature rows and two of 8 weights, then 64
// products and 64 sums into an 8 x 8 accumulator tile -- with nothing else
// (no layer 2, epilogue or tile copies), and reports the operations per
// second it sustains: the ceiling the MLP kernel can approach.
#include <algorithm>

#include "npa_internal.h"

namespace npa {
namespace {

constexpr int kProbeThreads = 384;
constexpr int kProbeF = 64, kProbeM = 192, kProbeHp = 128;

__global__ void __launch_bounds__(kProbeThreads)
tile_probe_kernel(const float* __restrict__ seed, float* __restrict__ out, int reps) {
  // power-of-two stand-ins for the feature tile and the weights: the indices
  // below wrap with a mask (16-byte aligned, in bounds) and hit the same
  // shared-memory banks as the kernel's
  constexpr int kFt = 4096, kW = 2048;
  __shared__ float4 ft4[kFt / 4];
  __shared__ float4 w4[kW / 4];
  float* ft = reinterpret_cast<float*>(ft4);
  float* w1 = reinterpret_cast<float*>(w4);
  for (int e = threadIdx.x; e < kFt; e += kProbeThreads) ft[e] = seed[e & 255];
  for (int e = threadIdx.x; e < kW; e += kProbeThreads) w1[e] = seed[(e + 7) & 255];
  __syncthreads();
  const int rg = threadIdx.x / 16, hg = threadIdx.x % 16;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  for (int r = 0; r < reps; ++r) {
#pragma unroll 1
    for (int k = 0; k < kProbeF; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(ft + ((k * kProbeM + rg * 8) & (kFt - 1)));
      const float4 a1 =
          *reinterpret_cast<const float4*>(ft + ((k * kProbeM + rg * 8 + 4) & (kFt - 1)));
      const float4 b0 = *reinterpret_cast<const float4*>(w1 + ((k * kProbeHp + hg * 4) & (kW - 1)));
      const float4 b1 =
          *reinterpret_cast<const float4*>(w1 + ((k * kProbeHp + 64 + hg * 4) & (kW - 1)));
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float p[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) p[i][j] = bv[j] * av[i];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = acc[i][j] + p[i][j];
    }
  }
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) s = s + acc[i][j];
  out[blockIdx.x * kProbeThreads + threadIdx.x] = s;
}

}  // namespace
}  // namespace npa

extern "C" npa_status npa_debug_fp32_tile_rate(int32_t reps, double* ops_per_second,
                                               double* kernel_ms) {
  using namespace npa;
  if (reps < 1 || !ops_per_second || !kernel_ms)
    return fail(NPA_ERR_INVALID_ARGUMENT, "reps must be >= 1 and outputs non-null");
  int dev = 0, sms = 0;
  NPA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  NPA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
           "cudaDeviceGetAttribute");
  const int blocks = sms * 2;  // two 12-warp blocks per SM
  float* seed = nullptr;
  float* out = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  npa_status st = NPA_OK;
  float ms = 0.0f;
  if (cudaMalloc(&seed, 256 * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&out, size_t(blocks) * kProbeThreads * sizeof(float)) != cudaSuccess ||
      cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess ||
      cudaMemsetAsync(seed, 0, 256 * sizeof(float), stream) != cudaSuccess) {
    cudaGetLastError();
    st = fail(NPA_ERR_CUDA, "probe set-up failed");
  }
  for (int pass = 0; pass < 2 && st == NPA_OK; ++pass) {  // the first pass warms up
    cudaEventRecord(e0, stream);
    tile_probe_kernel<<<blocks, kProbeThreads, 0, stream>>>(seed, out, reps);
    st = after_launch("tile_probe_kernel");
    cudaEventRecord(e1, stream);
    if (st == NPA_OK && cudaEventSynchronize(e1) != cudaSuccess)
      st = fail(NPA_ERR_CUDA, "cudaEventSynchronize");
    if (st == NPA_OK) cudaEventElapsedTime(&ms, e0, e1);
  }
  if (stream) cudaStreamSynchronize(stream);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (stream) cudaStreamDestroy(stream);
  cudaFree(seed);
  cudaFree(out);
  NPA_TRY(st);
  // 64 k-steps x 64 multiply-adds x 2 operations per thread and repetition
  const double ops = double(blocks) * kProbeThreads * reps * kProbeF * 64.0 * 2.0;
  *ops_per_second = ops / (double(ms) * 1e-3);
  *kernel_ms = ms;
  return NPA_OK;
}
