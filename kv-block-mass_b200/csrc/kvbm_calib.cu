// MUFU ex2 throughput calibration (kvbm_measure_ex2_rate in include/kvbm.h).
//
// Both block-mass passes issue one ex2.approx.f32 per score element, so their
// binding roofline is the multi-function unit's exp2 rate rather than the
// tensor pipe; this kernel measures that rate on the running device.
#include <cuda_runtime.h>

#include "kvbm_internal.cuh"

namespace kvbm {
namespace {

constexpr int kChains = 8;

__device__ __forceinline__ float ex2_neg(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(-x));
  return y;
}

// Every thread runs kChains independent x <- 2^-x chains (values stay in
// [0.5, 1]), enough independent work per warp to keep the unit saturated.
__global__ void __launch_bounds__(256) ex2_rate_kernel(float* sink, int iters) {
  float x[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) x[c] = 0.001f * (threadIdx.x + c);
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < kChains; ++c) x[c] = ex2_neg(x[c]);
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kChains; ++c) s += x[c];
  if (s == 1234.5f) sink[blockIdx.x] = s;  // keeps the chains live
}

}  // namespace
}  // namespace kvbm

extern "C" int kvbm_measure_ex2_rate(void* stream, double* ex2_per_second) {
  using namespace kvbm;
  if (ex2_per_second == nullptr) return KVBM_ERR_NULL;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KVBM_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = sms * 8, threads = 256, iters = 4096;
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return KVBM_ERR_CUDA;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return KVBM_ERR_CUDA;
  }
  int st = KVBM_OK;
  float ms = 0.f;
  ex2_rate_kernel<<<blocks, threads, 0, s>>>(nullptr, iters);  // warm-up
  cudaEventRecord(e0, s);
  ex2_rate_kernel<<<blocks, threads, 0, s>>>(nullptr, iters);
  cudaEventRecord(e1, s);
  if (cudaGetLastError() != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess ||
      cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess || ms <= 0.f)
    st = KVBM_ERR_CUDA;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st == KVBM_OK)
    *ex2_per_second = (double)blocks * threads * iters * kChains / (ms * 1e-3);
  return st;
}

extern "C" double kvbm_exp2_fma_fraction(void) { return kvbm::exp2_fma_fraction(); }
