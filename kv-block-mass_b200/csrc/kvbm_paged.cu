// Paged-KV input: gathers the key rows of a paged cache into a dense
// [B', H_kv', N, D] block of the workspace, which the block-mass kernels then
// read like any dense k.
//
// The cache is [num_pages, page_size, H_kv, D] with a per-sequence block
// table [B, max_pages] of page ids; logical key n of sequence b lives in page
// block_table[b][n / page_size], slot n % page_size.  This is the layout of
// the paged KV managers that consume block mass (the companion paged-kv block
// manager named in the reference's README.md:7-10 and
// src/kvblockmass/reclaim.py:14-16).  The reference itself takes dense k only.
//
// Why a gather and not paged TMA loads inside the kernels: both passes read
// every key row N/128 times or more out of L2, while the gather reads and
// writes each needed row once (2 * B' * H_kv' * N * D * elem bytes, HBM-bound),
// which on the Llama-3-8B N=32768 shape is about 0.3% of the step (30 us of
// ~10 ms).  The
// kernels keep one 128-row TMA box per key tile instead of one per page.
#include <cuda_runtime.h>

#include "kvbm_internal.cuh"

namespace kvbm {
namespace {

// Set when a block-table entry lies outside [0, num_pages); those rows are
// written as zeros instead of being read.
__device__ unsigned int g_page_error = 0;

constexpr int kGatherThreads = 256;
constexpr int kUnroll = 4;

// One thread moves one V (16 bytes, or one element on the generic path) of
// one dense row; a block covers kGatherThreads / dv whole rows per step.
// Strides are in V units.
template <typename V>
__global__ void __launch_bounds__(kGatherThreads) gather_pages_kernel(
    const V* __restrict__ cache, long long cs0, long long cs1, long long cs2, long long cs3, int num_pages,
    int page_size, const int32_t* __restrict__ table, long long ts, int b0, int g0, int ng, int N, int dv,
    long long rows, const int32_t* __restrict__ lens, const int32_t* __restrict__ cu, long long total,
    V* __restrict__ out) {
  const int rpb = kGatherThreads / dv;  // rows per block step
  const int t = threadIdx.x;
  if (t >= rpb * dv) return;
  const int d = t % dv;
  const long long stride = (long long)gridDim.x * rpb;
  // kUnroll rows per thread per step, all loads issued before the stores
  for (long long r0 = (long long)blockIdx.x * rpb + t / dv; r0 < rows; r0 += kUnroll * stride) {
    V v[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const long long r = r0 + j * stride;
      v[j] = V{};
      if (r < rows) {
        const int n = (int)(r % N);
        const long long bg = r / N;
        const int g = (int)(bg % ng), b = (int)(bg / ng);
        // keys past the sequence's length stay zero: their table entries are not read
        if (n >= seq_view(lens, cu, false, b0 + b, N, total).n) continue;
        const int page = table[(long long)(b0 + b) * ts + n / page_size];
        if (page >= 0 && page < num_pages) {
          v[j] = cache[(long long)page * cs0 + (long long)(n % page_size) * cs1 + (long long)(g0 + g) * cs2 +
                       d * cs3];
        } else if (d == 0) {
          atomicOr(&g_page_error, 1u);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const long long r = r0 + j * stride;
      if (r < rows) out[r * dv + d] = v[j];
    }
  }
}

template <typename V>
int launch_gather(const kvbm_paged_kv* kv, int esize, int b0, int g0, int nb, int ng, int N, int D,
                  const int32_t* lens, const int32_t* cu, long long total, void* out, cudaStream_t s) {
  const int per = (int)sizeof(V) / esize;  // elements per V
  const int dv = D / per;
  const long long rows = (long long)nb * ng * N;
  const int rpb = kGatherThreads / dv;
  long long blocks = (rows + rpb - 1) / rpb;
  if (blocks > 148LL * 8) blocks = 148LL * 8;  // grid-stride beyond 8 blocks per SM
  const int64_t* cs = kv->cache_stride;
  gather_pages_kernel<V><<<(unsigned)blocks, kGatherThreads, 0, s>>>(
      static_cast<const V*>(kv->k_cache), cs[0] / per, cs[1] / per, cs[2] / per, per == 1 ? cs[3] : 1,
      kv->num_pages, kv->page_size, kv->block_table, kv->block_table_stride, b0, g0, ng, N, dv, rows, lens, cu,
      total, static_cast<V*>(out));
  return cudaGetLastError() == cudaSuccess ? KVBM_OK : KVBM_ERR_CUDA;
}

}  // namespace

int launch_page_gather(const kvbm_paged_kv* kv, int dtype, int b0, int g0, int nb, int ng, int N, int D,
                       const int32_t* lens, const int32_t* cu, long long total, void* out, cudaStream_t s) {
  const int esize = dtype == KVBM_F64 ? 8 : (dtype == KVBM_F32 ? 4 : 2);
  const int64_t* cs = kv->cache_stride;
  // 16-byte vectors when every row of D elements starts on a 16-byte boundary
  bool vec = cs[3] == 1 && (D * esize) % 16 == 0 && ((uintptr_t)kv->k_cache % 16) == 0;
  for (int i = 0; i < 3; ++i) vec = vec && (cs[i] * esize) % 16 == 0;
  if (vec) return launch_gather<uint4>(kv, esize, b0, g0, nb, ng, N, D, lens, cu, total, out, s);
  if (esize == 8) return launch_gather<unsigned long long>(kv, esize, b0, g0, nb, ng, N, D, lens, cu, total, out, s);
  if (esize == 4) return launch_gather<unsigned int>(kv, esize, b0, g0, nb, ng, N, D, lens, cu, total, out, s);
  return launch_gather<unsigned short>(kv, esize, b0, g0, nb, ng, N, D, lens, cu, total, out, s);
}

int read_and_clear_page_error(cudaStream_t s, int* err) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_page_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return KVBM_ERR_CUDA;
  *err = v != 0;
  if (v != 0) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_page_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return KVBM_ERR_CUDA;
  }
  return KVBM_OK;
}

}  // namespace kvbm
