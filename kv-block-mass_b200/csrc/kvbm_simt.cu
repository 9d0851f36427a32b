// SIMT block-mass kernels: fp32 FFMA (fp32 / bf16 / fp16 inputs) and fp64 DFMA
// (fp64 inputs), any head dim up to 256, every mask kind.
//
// Pass 1 (row log-sum-exp) restates the online max/denominator loop of the
// reference's Triton kernel (kv-block-mass src/kvblockmass/triton_kernel.py:69-104)
// and the streaming softmax of src/kvblockmass/reference.py:108-119; pass 2
// recomputes each score tile and sums softmax weights per key column
// (triton_kernel.py:106-145, reference.py:121-124), but writes one partial per
// (unit, query chunk, key) into the workspace instead of float atomics, so a
// separate fixed-order reduce makes every result deterministic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "kvbm_internal.cuh"

namespace kvbm {
namespace {

constexpr int BM = kSimtBM;
constexpr int BN = kSimtBN;
constexpr int NT = kSimtThreads;

template <typename Acc>
struct Args {
  const void* q;
  long long qs0, qs1, qs2, qs3;
  const void* k;
  long long ks0, ks1, ks2, ks3;
  int N, D, G, Hkv, ub;
  int rb, hb, hn;  // staged calls: units [rb, ..) of the range, pass-1 q-heads [hb, hb + hn)
  int qt1;         // pass 1: row tiles below qt1, the grid's x covering the last of them
  const uint8_t* kmask;
  long long kmb;
  const uint8_t* qmask;
  long long qmb;
  const uint8_t* pmask;
  long long pmb, pmr;
  Acc C;  // scale * log2(e)
  int causal, skip;
  Acc* lse;   // [U_sel*G, N]
  Acc* part;  // [U_sel, nchunk, N]
  int qchunk, nchunk;
  const int32_t* lens;  // ragged lengths [B] or null
  const int32_t* cu;    // packed row offsets [B+1] or null
  int kpacked;          // k packed like q
  long long total;      // rows of the packed q (and k)
};

template <typename In, typename Acc>
__device__ __forceinline__ Acc load_as(const void* base, long long off);
template <>
__device__ __forceinline__ float load_as<float, float>(const void* b, long long o) {
  return static_cast<const float*>(b)[o];
}
template <>
__device__ __forceinline__ float load_as<__nv_bfloat16, float>(const void* b, long long o) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(b)[o]);
}
template <>
__device__ __forceinline__ float load_as<__half, float>(const void* b, long long o) {
  return __half2float(static_cast<const __half*>(b)[o]);
}
template <>
__device__ __forceinline__ double load_as<double, double>(const void* b, long long o) {
  return static_cast<const double*>(b)[o];
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ double fast_exp2(double x) { return exp2(x); }
__device__ __forceinline__ float acc_log2(float x) { return log2f(x); }
__device__ __forceinline__ double acc_log2(double x) { return log2(x); }

template <typename Acc>
__device__ __forceinline__ Acc neg_inf();
template <>
__device__ __forceinline__ float neg_inf<float>() { return -INFINITY; }
template <>
__device__ __forceinline__ double neg_inf<double>() { return -(double)INFINITY; }

// keep(b, row, col): causal & key mask & query mask & pair mask (reference.py:83-87),
// for positions of a sequence of n <= N positions.
template <typename Acc>
__device__ __forceinline__ bool keep_at(const Args<Acc>& a, int b, int n, int row, int col) {
  if (row >= n || col >= n) return false;
  if (a.causal && col > row) return false;
  if (a.kmask && !a.kmask[b * a.kmb + col]) return false;
  if (a.qmask && !a.qmask[b * a.qmb + row]) return false;
  if (a.pmask && !a.pmask[b * a.pmb + (long long)row * a.pmr + col]) return false;
  return true;
}

// Stage a [rows x D] slab of a [*, N, D] operand into smem as S[d * 64 + r]
// (transposed so that each thread reads 4 consecutive rows with one vector load).
template <typename In, typename Acc>
__device__ __forceinline__ void stage_tile(Acc* S, const void* base, long long off0, long long rs,
                                           long long ds, int r0, int rlim, int D) {
  for (int idx = threadIdx.x; idx < 64 * D; idx += NT) {
    const int r = idx / D;
    const int d = idx - r * D;
    const int row = r0 + r;
    Acc v = Acc(0);
    if (row < rlim) v = load_as<In, Acc>(base, off0 + row * rs + d * ds);
    S[d * 64 + r] = v;
  }
}

template <typename Acc>
__device__ __forceinline__ void load4(const Acc* p, Acc (&v)[4]) {
  if constexpr (sizeof(Acc) == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    const double2 t0 = *reinterpret_cast<const double2*>(p);
    const double2 t1 = *reinterpret_cast<const double2*>(p + 2);
    v[0] = t0.x; v[1] = t0.y; v[2] = t1.x; v[3] = t1.y;
  }
}

// S[4][4] = Qs[rows ty*4.., :] . Ks[cols tx*4.., :]
template <typename Acc>
__device__ __forceinline__ void tile_scores(const Acc* Qs, const Acc* Ks, int D, int tx, int ty,
                                            Acc (&acc)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = Acc(0);
#pragma unroll 4
  for (int d = 0; d < D; ++d) {
    Acc qa[4], kb[4];
    load4(Qs + d * 64 + ty * 4, qa);
    load4(Ks + d * 64 + tx * 4, kb);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fma(qa[i], kb[j], acc[i][j]);
  }
}

// ---------------------------------------------------------------- pass 1: lse2
template <typename In, typename Acc>
__global__ void __launch_bounds__(NT) simt_lse_kernel(Args<Acc> a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Acc* Qs = reinterpret_cast<Acc*>(smem_raw);  // [D][64]
  Acc* Ks = Qs + a.D * 64;                      // [D][64]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int r0 = (a.qt1 - 1 - (int)blockIdx.x) * BM;  // long (late) rows first
  const int hidx = (a.rb + (int)blockIdx.y / a.hn) * a.G + a.hb + (int)blockIdx.y % a.hn;  // (u - ub) * G + hh
  const int u = a.ub + hidx / a.G, hh = hidx % a.G;
  const int b = u / a.Hkv, g = u % a.Hkv, h = g * a.G + hh;
  const SeqView sv = seq_view(a.lens, a.cu, a.kpacked != 0, b, a.N, a.total);
  const int n = sv.n;
  if (r0 >= n) return;  // past the sequence: pass 2 never reads these rows

  stage_tile<In, Acc>(Qs, a.q, sv.q_b * a.qs0 + h * a.qs1 + sv.q_row * a.qs2, a.qs2, a.qs3, r0, n, a.D);

  const int n_end = (a.causal && a.skip) ? min(n, r0 + BM) : n;
  Acc m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { m[i] = neg_inf<Acc>(); l[i] = Acc(0); }

  for (int n0 = 0; n0 < n_end; n0 += BN) {
    __syncthreads();
    stage_tile<In, Acc>(Ks, a.k, sv.k_b * a.ks0 + g * a.ks1 + sv.k_row * a.ks2, a.ks2, a.ks3, n0, n, a.D);
    __syncthreads();
    Acc acc[4][4];
    tile_scores(Qs, Ks, a.D, tx, ty, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = r0 + ty * 4 + i;
      Acc t[4];
      Acc tmax = neg_inf<Acc>();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = n0 + tx * 4 + j;
        t[j] = keep_at(a, b, n, row, col) ? acc[i][j] * a.C : neg_inf<Acc>();
        tmax = t[j] > tmax ? t[j] : tmax;
      }
      // Rescale only when the running max grows: a tile that is fully masked
      // leaves (m, l) bit-identical, which keeps causal_skip on/off identical.
      if (tmax > m[i]) {
        l[i] = l[i] * fast_exp2(m[i] - tmax);
        m[i] = tmax;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (t[j] != neg_inf<Acc>()) l[i] += fast_exp2(t[j] - m[i]);
    }
  }
  // Merge the 16 per-thread partial (m, l) of each row (lanes sharing ty).
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) {
      const Acc mo = __shfl_xor_sync(0xffffffffu, m[i], off);
      const Acc lo = __shfl_xor_sync(0xffffffffu, l[i], off);
      const Acc mn = mo > m[i] ? mo : m[i];
      if (mn != neg_inf<Acc>()) {
        l[i] = l[i] * fast_exp2(m[i] - mn) + lo * fast_exp2(mo - mn);
        m[i] = mn;
      }
    }
  }
  if (tx == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = r0 + ty * 4 + i;
      if (row < n) {
        // Rows that keep no key get +inf: 2^(t - inf) = 0, so they contribute 0.
        a.lse[(long long)hidx * a.N + row] =
            (m[i] == neg_inf<Acc>()) ? -neg_inf<Acc>() : m[i] + acc_log2(l[i]);
      }
    }
  }
}

// ---------------------------------------------------------------- pass 2: mass
template <typename In, typename Acc>
__global__ void __launch_bounds__(NT) simt_mass_kernel(Args<Acc> a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Acc* Ks = reinterpret_cast<Acc*>(smem_raw);  // [D][64]
  Acc* Qs = Ks + a.D * 64;                      // [D][64]
  Acc* Ls = Qs + a.D * 64;                      // [64]
  Acc* red = Ls + 64;                           // [16][64]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int c0 = blockIdx.x * BN;
  const int y = blockIdx.y;
  const int uu = a.rb + (int)blockIdx.z;
  const int u = a.ub + uu;
  const int b = u / a.Hkv, g = u % a.Hkv;
  const SeqView sv = seq_view(a.lens, a.cu, a.kpacked != 0, b, a.N, a.total);
  const int n = sv.n;
  const int qa = y * a.qchunk;
  if (c0 >= n || qa >= n) {
    // nothing of this sequence here: the reduce reads exact zeros
    if (tid < BN && c0 + tid < a.N) a.part[((long long)uu * a.nchunk + y) * a.N + c0 + tid] = Acc(0);
    return;
  }
  const int qb = min(n, qa + a.qchunk);
  // Causal: rows < c0 keep no key of this tile.  With causal_skip the CTA
  // starts at the first row tile that reaches c0 (tile boundaries stay those
  // of the unskipped loop, so the same non-zero terms add in the same order).
  int rs = qa;
  if (a.causal && a.skip) {
    if (qb - 1 < c0) return;  // whole chunk above the diagonal: nothing to add
    if (c0 > qa) rs = qa + ((c0 - qa) / BM) * BM;
  }
  stage_tile<In, Acc>(Ks, a.k, sv.k_b * a.ks0 + g * a.ks1 + sv.k_row * a.ks2, a.ks2, a.ks3, c0, n, a.D);
  Acc cs[4] = {Acc(0), Acc(0), Acc(0), Acc(0)};
  for (int hh = 0; hh < a.G; ++hh) {
    const int h = g * a.G + hh;
    const Acc* lse_h = a.lse + (long long)(uu * a.G + hh) * a.N;
    for (int r0 = rs; r0 < qb; r0 += BM) {
      __syncthreads();
      stage_tile<In, Acc>(Qs, a.q, sv.q_b * a.qs0 + h * a.qs1 + sv.q_row * a.qs2, a.qs2, a.qs3, r0, qb, a.D);
      if (tid < BM) Ls[tid] = (r0 + tid < qb) ? lse_h[r0 + tid] : Acc(0);
      __syncthreads();
      Acc acc[4][4];
      tile_scores(Qs, Ks, a.D, tx, ty, acc);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = r0 + ty * 4 + i;
        if (row >= qb) continue;
        const Acc L = Ls[ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = c0 + tx * 4 + j;
          if (keep_at(a, b, n, row, col)) cs[j] += fast_exp2(acc[i][j] * a.C - L);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 4; ++j) red[ty * 64 + tx * 4 + j] = cs[j];
  __syncthreads();
  if (tid < BN) {
    Acc s = Acc(0);
#pragma unroll
    for (int r = 0; r < 16; ++r) s += red[r * 64 + tid];
    const int col = c0 + tid;
    if (col < a.N) a.part[((long long)uu * a.nchunk + y) * a.N + col] = col < n ? s : Acc(0);
  }
}

template <typename In, typename Acc>
int launch_typed(const kvbm_problem* p, const WsLayout& L, void* ws, cudaStream_t s, const LaunchOpts& o) {
  Args<Acc> a;
  a.q = p->q;
  a.qs0 = p->q_stride[0]; a.qs1 = p->q_stride[1]; a.qs2 = p->q_stride[2]; a.qs3 = p->q_stride[3];
  a.k = p->k;
  a.ks0 = p->k_stride[0]; a.ks1 = p->k_stride[1]; a.ks2 = p->k_stride[2]; a.ks3 = p->k_stride[3];
  a.N = p->N; a.D = p->D; a.G = p->Hq / p->Hkv; a.Hkv = p->Hkv; a.ub = p->unit_begin;
  a.kmask = p->key_mask; a.kmb = p->key_mask_bstride;
  a.qmask = p->query_mask; a.qmb = p->query_mask_bstride;
  a.pmask = p->pair_mask; a.pmb = p->pair_mask_bstride; a.pmr = p->pair_mask_rstride;
  a.C = static_cast<Acc>(p->scale * kLog2e);
  a.causal = p->causal != 0;
  a.skip = p->causal_skip != 0;
  a.lse = reinterpret_cast<Acc*>(static_cast<char*>(ws) + L.lse_off);
  a.part = reinterpret_cast<Acc*>(static_cast<char*>(ws) + L.part_off);
  a.qchunk = L.qchunk;
  a.nchunk = L.nchunk;
  a.lens = o.rg.lens;
  a.cu = o.rg.cu;
  a.kpacked = o.rg.k_packed ? 1 : 0;
  a.total = o.rg.total;

  const RunRange rr = run_range(p, o);
  a.rb = rr.rb;
  a.hb = rr.hb;
  a.hn = rr.nh;
  a.qt1 = (rr.qe + BM - 1) / BM;
  const int U = rr.nu;  // units this launch runs
  const size_t smem1 = size_t(2) * p->D * 64 * sizeof(Acc);
  const size_t smem2 = smem1 + (64 + 16 * 64) * sizeof(Acc);
  auto k1 = simt_lse_kernel<In, Acc>;
  auto k2 = simt_mass_kernel<In, Acc>;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1) != cudaSuccess ||
      cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2) != cudaSuccess)
    return KVBM_ERR_CUDA;
  dim3 g1(a.qt1 - rr.qb / BM, U * a.hn);
  if (o.run_pass1) {
    k1<<<g1, NT, smem1, s>>>(a);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  }
  if (o.mid_event != nullptr && cudaEventRecord(static_cast<cudaEvent_t>(o.mid_event), s) != cudaSuccess)
    return KVBM_ERR_CUDA;
  if (o.run_pass2) {
    dim3 g2((p->N + BN - 1) / BN, L.nchunk, U);
    k2<<<g2, NT, smem2, s>>>(a);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  }
  return KVBM_OK;
}

// ---------------------------------------------------------------- bucket reduce
// mass[j] = sum over (unit, query chunk, key c in bucket j) of the partials,
// accumulated in fp64 in a fixed order (deterministic).  With causal, a chunk
// whose last row lies before the key tile start holds no kept pair and is not
// read (its CTA either returned early or wrote exact zeros).
//
// Thread t adds the flattened (unit, chunk, key) entries t, t + 256, ... of
// its bucket in that order; the warp and block sums then follow a fixed tree.
// The (unit, chunk, key) of the next entry is stepped forward with carries
// instead of being divided out of the flat index each time (two 64-bit
// divisions per entry), and loads are issued in batches (one load in flight
// per thread left the reduce bound by memory latency).  key_tile is a power
// of two (64 or 128).
template <typename Acc>
__device__ __forceinline__ double bucket_partial_sum(const Acc* part, int N, int cb, int nk, long long u0,
                                                     long long nu, int nchunk, int qchunk, int key_tile,
                                                     int causal) {
  constexpr int T = 256;
  const long long total = nu * nchunk * nk;
  double s = 0.0;
  if (threadIdx.x >= total) return s;
  const int dc = T % nk, dr = T / nk;
  const int dy = dr % nchunk, du = dr / nchunk;
  int co = (int)threadIdx.x % nk;
  const int r0 = (int)threadIdx.x / nk;
  int y = r0 % nchunk;
  long long uu = u0 + r0 / nchunk;
  // kBatch entries are loaded before any of them is added, so each thread has
  // kBatch loads in flight; the adds then run in entry order (same bits).
  constexpr int kBatch = 8;
  for (long long idx = threadIdx.x; idx < total; idx += (long long)T * kBatch) {
    Acc v[kBatch];
    unsigned kept = 0u;
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int c = cb + co;
      const bool keep = idx + (long long)i * T < total &&
                        (!causal || (long long)(y + 1) * qchunk - 1 >= (long long)(c & ~(key_tile - 1)));
      v[i] = keep ? part[(uu * nchunk + y) * N + c] : Acc(0);
      kept |= keep ? (1u << i) : 0u;
      co += dc;
      y += dy;
      uu += du;
      if (co >= nk) {
        co -= nk;
        ++y;
      }
      if (y >= nchunk) {
        y -= nchunk;
        ++uu;
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
      if (kept & (1u << i)) s += (double)v[i];
  }
  return s;
}

__device__ __forceinline__ double block_sum_256(double s, double* warp_sums) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = s;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < 8; ++w) t += warp_sums[w];
  return t;
}

template <typename Acc, typename Out>
__global__ void __launch_bounds__(256) reduce_kernel(const Acc* part, Out* mass, int N, int bs,
                                                     int U, int nchunk, int qchunk, int key_tile,
                                                     int causal) {
  __shared__ double warp_sums[8];
  const int j = blockIdx.x;
  const int cb = j * bs;
  const int nk = min(N, cb + bs) - cb;
  const double s = bucket_partial_sum(part, N, cb, nk, 0, U, nchunk, qchunk, key_tile, causal);
  const double t = block_sum_256(s, warp_sums);
  if (threadIdx.x == 0) mass[j] = static_cast<Out>(t);
}

// Per-sequence variant: mass[b][j] sums the units of batch b inside
// [ub, ub + U) (none: 0), same order and skips as reduce_kernel.
template <typename Acc, typename Out>
__global__ void __launch_bounds__(256) reduce_seq_kernel(const Acc* part, Out* mass, int N, int bs, int nb,
                                                         int ub, int U, int Hkv, int nchunk, int qchunk,
                                                         int key_tile, int causal) {
  __shared__ double warp_sums[8];
  const int j = blockIdx.x, b = blockIdx.y;
  const int cb = j * bs;
  const int nk = min(N, cb + bs) - cb;
  const int u0 = max(ub, b * Hkv), u1 = min(ub + U, (b + 1) * Hkv);
  const double s = u1 > u0 ? bucket_partial_sum(part, N, cb, nk, u0 - ub, u1 - u0, nchunk, qchunk, key_tile, causal)
                           : 0.0;
  const double t = block_sum_256(s, warp_sums);
  if (threadIdx.x == 0) mass[(long long)b * nb + j] = static_cast<Out>(t);
}

// ---------------------------------------------------------------- one-pass reduce
// The one-pass method leaves one partial per (head, query tile, bucket):
// part1[item][j], item = hidx * ntiles + qt over the problem's (unit, q-head)
// pairs hidx.  Step 1: CTA (bucket group, split, batch) sums the items of its
// split for 32 consecutive buckets (a lane per bucket, coalesced rows); warp
// w takes items i0 + w, i0 + w + 8, ... in order, kBatch loads in flight per
// thread, and the 8 warps' sums add in warp order.  Under causal an item
// whose last query row lies before the bucket's first key is not read (qt <
// floor(j * bs / 128)): its pass-1 CTA wrote nothing there.  Step 2 adds the
// splits in order.  Both steps accumulate in fp64: deterministic.
__global__ void __launch_bounds__(256) tile_reduce_kernel(const float* part1, double* red, int nb, int bs,
                                                          int ntiles, int G, int Hkv, int ub, int U, int causal,
                                                          int splits, int per_seq) {
  __shared__ double wsum[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  const int split = blockIdx.y, b = blockIdx.z;
  long long h0 = 0, h1 = (long long)U * G;  // (unit, q-head) pairs of this output row
  if (per_seq) {
    const int u0 = max(ub, b * Hkv), u1 = min(ub + U, (b + 1) * Hkv);
    h0 = (long long)(u0 - ub) * G;
    h1 = u1 > u0 ? (long long)(u1 - ub) * G : h0;
  }
  const long long items = (h1 - h0) * ntiles;
  const long long i0 = items * split / splits, i1 = items * (split + 1) / splits;
  const int qmin = causal ? (int)(((long long)j * bs) / kTcTile) : 0;
  double acc = 0.0;
  if (i0 + w < i1) {
    long long hid = h0 + (i0 + w) / ntiles;
    int qt = (int)((i0 + w) % ntiles);
    constexpr int kBatch = 8;
    for (long long i = i0 + w; i < i1; i += 8 * kBatch) {
      float v[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const bool keep = i + 8LL * k < i1 && j < nb && qt >= qmin;
        v[k] = keep ? part1[(hid * ntiles + qt) * nb + j] : 0.f;
        qt += 8;
        while (qt >= ntiles) {
          qt -= ntiles;
          ++hid;
        }
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) acc += (double)v[k];
    }
  }
  wsum[w][lane] = acc;
  __syncthreads();
  if (w == 0 && j < nb) {
    double t = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += wsum[k][lane];
    red[((long long)split * gridDim.z + b) * nb + j] = t;
  }
}

__global__ void tile_reduce_final_kernel(const double* red, float* mass, int nb, int splits, int b_out) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= (long long)b_out * nb) return;
  double t = 0.0;
  for (int sp = 0; sp < splits; ++sp) t += red[(long long)sp * b_out * nb + idx];
  mass[idx] = (float)t;
}

}  // namespace

int launch_simt(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws,
                cudaStream_t s, const LaunchOpts& o) {
  (void)mass_out;
  switch (p->dtype) {
    case KVBM_F32: return launch_typed<float, float>(p, L, ws, s, o);
    case KVBM_BF16: return launch_typed<__nv_bfloat16, float>(p, L, ws, s, o);
    case KVBM_F16: return launch_typed<__half, float>(p, L, ws, s, o);
    case KVBM_F64: return launch_typed<double, double>(p, L, ws, s, o);
    default: return KVBM_ERR_DTYPE;
  }
}

// Caller-provided row LSE (natural log of sum_c exp(scale * q.k_c) over kept
// keys, as an attention forward returns it) -> the lse2 layout of the path:
// SIMT keeps +lse2 in the accumulation type with +inf for rows that keep no
// key; the tensor-core path keeps -lse2 (fp32) over whole 128-row tiles with
// -inf for rows that keep no key and for padding rows.  A non-finite input or
// a dropped query_mask row counts as a row that keeps no key.
template <typename Acc, bool kNegated>
__global__ void lse_import_kernel(const float* lse, long long s0, long long s1, long long s2, Acc* out, int N,
                                  int Nrow, int G, int Hkv, int ub, RunRange rr, long long rows_total,
                                  const uint8_t* qmask, long long qmb, const int32_t* lens, const int32_t* cu,
                                  long long total) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= rows_total) return;
  const int i = (int)(idx % Nrow);
  const long long pr = idx / Nrow;  // (unit, head) pair of the run
  const long long hidx = (rr.rb + pr / rr.nh) * (long long)G + rr.hb + pr % rr.nh;  // (u - ub) * G + hh
  const int u = ub + (int)(hidx / G), hh = (int)(hidx % G);
  const int b = u / Hkv, h = (u % Hkv) * G + hh;
  // a packed batch indexes its LSE like q: row cu[b] + i of [H_q, total_tokens]
  const SeqView sv = seq_view(lens, cu, false, b, N, total);
  bool dead = i >= sv.n;
  double v = 0.0;
  if (!dead) {
    v = (double)lse[sv.q_b * s0 + h * s1 + ((long long)sv.q_row + i) * s2];
    dead = !isfinite(v) || (qmask != nullptr && qmask[b * qmb + i] == 0);
  }
  const double l2 = v * kLog2e;
  Acc r;
  if (kNegated) r = dead ? (Acc)(-INFINITY) : (Acc)(-l2);
  else r = dead ? (Acc)INFINITY : (Acc)l2;
  out[hidx * Nrow + (kNegated ? lse_tile_slot(i) : i)] = r;  // the tensor-core paths' row order
}

int launch_lse_import(const kvbm_problem* p, const WsLayout& L, const float* lse, const int64_t* st, void* ws,
                      cudaStream_t s, const Ragged& rg, const RunRange& rr) {
  const int G = p->Hq / p->Hkv;
  const int Nrow = L.path >= 1 ? (p->N + kTcTile - 1) / kTcTile * kTcTile : p->N;
  const long long rows = (long long)rr.nu * rr.nh * Nrow;
  const int threads = 256;
  const long long blocks = (rows + threads - 1) / threads;
  char* base = static_cast<char*>(ws) + L.lse_off;
  if (L.path >= 1) {
    lse_import_kernel<float, true><<<(unsigned)blocks, threads, 0, s>>>(
        lse, st[0], st[1], st[2], reinterpret_cast<float*>(base), p->N, Nrow, G, p->Hkv, p->unit_begin, rr, rows,
        p->query_mask, p->query_mask_bstride, rg.lens, rg.cu, rg.total);
  } else if (p->dtype == KVBM_F64) {
    lse_import_kernel<double, false><<<(unsigned)blocks, threads, 0, s>>>(
        lse, st[0], st[1], st[2], reinterpret_cast<double*>(base), p->N, Nrow, G, p->Hkv, p->unit_begin, rr, rows,
        p->query_mask, p->query_mask_bstride, rg.lens, rg.cu, rg.total);
  } else {
    lse_import_kernel<float, false><<<(unsigned)blocks, threads, 0, s>>>(
        lse, st[0], st[1], st[2], reinterpret_cast<float*>(base), p->N, Nrow, G, p->Hkv, p->unit_begin, rr, rows,
        p->query_mask, p->query_mask_bstride, rg.lens, rg.cu, rg.total);
  }
  return cudaGetLastError() == cudaSuccess ? KVBM_OK : KVBM_ERR_CUDA;
}

int launch_reduce(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws,
                  cudaStream_t s, bool per_sequence) {
  if (L.key_tile <= 0 || (L.key_tile & (L.key_tile - 1)) != 0) return KVBM_ERR_SHAPE;  // power of two
  const int nb = (int)kvbm_num_blocks(p->N, p->block_size);
  const int U = p->unit_end - p->unit_begin;
  const char* base = static_cast<const char*>(ws) + L.part_off;
  if (L.one_pass) {
    const int b_out = per_sequence ? p->B : 1;
    const int ntiles = (p->N + kTcTile - 1) / kTcTile;
    double* red = reinterpret_cast<double*>(static_cast<char*>(ws) + L.red_off);
    const dim3 grid((nb + 31) / 32, L.red_splits, b_out);
    tile_reduce_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float*>(base), red, nb, p->block_size, ntiles,
                                            p->Hq / p->Hkv, p->Hkv, p->unit_begin, U, p->causal != 0,
                                            L.red_splits, per_sequence ? 1 : 0);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
    const long long n = (long long)b_out * nb;
    tile_reduce_final_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(red, static_cast<float*>(mass_out), nb,
                                                                       L.red_splits, b_out);
    return cudaGetLastError() == cudaSuccess ? KVBM_OK : KVBM_ERR_CUDA;
  }
  if (per_sequence) {
    const dim3 grid(nb, p->B);
    if (p->dtype == KVBM_F64)
      reduce_seq_kernel<double, double><<<grid, 256, 0, s>>>(
          reinterpret_cast<const double*>(base), static_cast<double*>(mass_out), p->N, p->block_size, nb,
          p->unit_begin, U, p->Hkv, L.nchunk, L.qchunk, L.key_tile, p->causal != 0);
    else
      reduce_seq_kernel<float, float><<<grid, 256, 0, s>>>(
          reinterpret_cast<const float*>(base), static_cast<float*>(mass_out), p->N, p->block_size, nb,
          p->unit_begin, U, p->Hkv, L.nchunk, L.qchunk, L.key_tile, p->causal != 0);
    return cudaGetLastError() == cudaSuccess ? KVBM_OK : KVBM_ERR_CUDA;
  }
  if (p->dtype == KVBM_F64) {
    reduce_kernel<double, double><<<nb, 256, 0, s>>>(reinterpret_cast<const double*>(base),
                                                     static_cast<double*>(mass_out), p->N,
                                                     p->block_size, U, L.nchunk, L.qchunk,
                                                     L.key_tile, p->causal != 0);
  } else {
    reduce_kernel<float, float><<<nb, 256, 0, s>>>(reinterpret_cast<const float*>(base),
                                                   static_cast<float*>(mass_out), p->N,
                                                   p->block_size, U, L.nchunk, L.qchunk,
                                                   L.key_tile, p->causal != 0);
  }
  return cudaGetLastError() == cudaSuccess ? KVBM_OK : KVBM_ERR_CUDA;
}

}  // namespace kvbm
