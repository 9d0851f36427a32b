// Device-side consumers of the mass vector: the eviction design of
// kv-block-mass (src/kvblockmass/evict.py) computed where the mass already
// is, so a serving step never copies the mass to the host.
//
//   expand_block_scores (evict.py:64-83)   score of token i = mass[i / block_size]
//   design_from_scores  (evict.py:95-171)  certainty set = sinks + recency +
//                                          top slice; tail pi = clip(m w / sum w,
//                                          eps, 1); keep = certainty | u < pi
//   hajek_log_offsets   (evict.py:174-187) -log(pi)
//   block retention     (reclaim.py:46-55) blocks with a kept token
//
// Scores are constant inside a block, so nothing here sorts tokens.  One CTA
// per sequence (row) works on the blocks: a radix select over the blocks'
// float64 score bits, weighted by their token counts, finds the top slice's
// threshold; within a block the certain tokens are then a prefix (sinks,
// top slice: ties go to the lower index, as the reference's _top_slice
// docstring states, evict.py:86-87) plus a suffix (recency window), which
// fixed-order scans over blocks turn into per-block counts and prefixes.  A
// grid kernel then writes every token's pi / keep / certainty from its
// block's numbers alone.
//
// Tail draws: the caller's uniforms (uniforms[t] for the t-th tail token in
// ascending index order: what the reference's torch.rand(n_tail, float64,
// generator) yields, for bit parity), or Philox4x32-10 (Salmon et al.,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by the seed,
// counter = (token, row).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "kvbm_internal.cuh"

namespace kvbm {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kWarps = kSelThreads / 32;

// Per-row results of the select kernel (in the workspace).
struct RowPlan {
  double total;          // sum of tail weights (after the uniform fallback)
  long long n_tail;      // tail tokens
  long long n_certain;   // certainty-set tokens
  int uniform_w;         // 1: tail weights are all 1 (uniform_tail, or zero-sum fallback)
  int flags;             // 1: a used block's mass is negative or NaN
};

struct DesignArgs {
  const void* mass;      // [B, mass_stride] float32 or float64
  int mass_f64;
  long long mass_stride; // elements between rows
  int B, N, bs, nb;      // nb = ceil(N / bs) used blocks
  long long m;           // tail budget
  int n_sinks, recency, top;  // top = min(top_slice, N)
  double eps;
  int uniform_tail;
  const double* uniforms;     // [B, ustride] or null
  long long ustride;
  unsigned long long seed;
  // outputs (any may be null except counts)
  double* pi;                 // [B, N]
  uint8_t* keep;              // [B, N]
  uint8_t* certainty;         // [B, N]
  double* scores;             // [B, N] expanded scores
  double* log_offsets;        // [B, N] -log(pi)
  int64_t* counts;            // [B, 5]: kept, certain, tail, blocks kept, flags
  // scratch
  RowPlan* plan;              // [B]
  int* prefix;                // [B, nb]: certain prefix length of each block (sinks / top slice)
  long long* cert_before;     // [B, nb]: certain tokens before each block
};

__device__ __forceinline__ double mass_at(const DesignArgs& a, int row, int b) {
  const long long o = (long long)row * a.mass_stride + b;
  return a.mass_f64 ? static_cast<const double*>(a.mass)[o] : (double)static_cast<const float*>(a.mass)[o];
}

// Order-preserving key of a non-negative double (+0 and -0 both map to 0).
__device__ __forceinline__ unsigned long long score_key(double s) {
  return s > 0.0 ? (unsigned long long)__double_as_longlong(s) : 0ull;
}

__global__ void __launch_bounds__(kSelThreads) design_select_kernel(DesignArgs a) {
  __shared__ unsigned int hist[256];
  __shared__ long long sh_ll[kWarps];
  __shared__ double sh_d[kWarps];
  __shared__ unsigned long long s_prefix;
  __shared__ long long s_remaining;
  __shared__ int s_flags;
  const int row = blockIdx.x;
  const int t = threadIdx.x;
  const int nb = a.nb, N = a.N, bs = a.bs;
  if (t == 0) {
    s_flags = 0;
    s_prefix = 0;
    s_remaining = a.top;
  }
  __syncthreads();
  for (int b = t; b < nb; b += kSelThreads) {
    const double s = mass_at(a, row, b);
    if (!(s >= 0.0)) atomicOr(&s_flags, 1);
  }

  // 1. radix select, MSB first, 8-bit digits: threshold key T of the top
  //    slice; s_remaining ends as the tokens taken from the blocks whose key
  //    equals T (lowest indices first).
  if (a.top > 0) {
    for (int digit = 7; digit >= 0; --digit) {
      for (int i = t; i < 256; i += kSelThreads) hist[i] = 0;
      __syncthreads();
      const int shift = digit * 8;
      const unsigned long long pre = s_prefix;
      const unsigned long long hi_mask = digit == 7 ? 0ull : (~0ull << (shift + 8));
      for (int b = t; b < nb; b += kSelThreads) {
        const unsigned long long key = score_key(mass_at(a, row, b));
        if ((key & hi_mask) == (pre & hi_mask)) {
          const int len = min(bs, N - b * bs);
          atomicAdd(&hist[(key >> shift) & 255u], (unsigned int)len);
        }
      }
      __syncthreads();
      if (t < 32) {
        // warp 0: lane l owns bins [248 - 8l, 256 - 8l); counts accumulate
        // from the top bin down, and the bin where they reach `rem` is the
        // digit of T.
        const long long rem = s_remaining;
        long long mine = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) mine += hist[255 - 8 * t - j];
        long long incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const long long y = __shfl_up_sync(0xffffffffu, incl, o);
          if (t >= o) incl += y;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, incl >= rem);
        const int lane = hit ? __ffs(hit) - 1 : 31;  // counts always reach rem by bin 0
        if (t == lane) {
          long long above = incl - mine;
          int v = 255 - 8 * t;
          for (int j = 0; j < 7; ++j, --v) {
            if (above + hist[v] >= rem) break;
            above += hist[v];
          }
          s_remaining = rem - above;
          s_prefix = pre | ((unsigned long long)v << shift);
        }
      }
      __syncthreads();
    }
  }
  const unsigned long long T = s_prefix;
  const long long take_eq = s_remaining;
  const long long R = a.recency > 0 ? max(0, N - a.recency) : N;  // first recency token

  // 2. per block, in index order (chunks of kSelThreads blocks with carries):
  //    tied tokens before the block, certain prefix / suffix, union, and the
  //    certain tokens before the block.
  long long eq_carry = 0, cert_carry = 0;
  double w_sum = 0.0;  // this thread's tail weights, accumulated in a fixed order
  for (int base = 0; base < nb; base += kSelThreads) {
    const int b = base + t;
    const bool valid = b < nb;
    const long long start = (long long)b * bs;
    const int len = valid ? (int)min((long long)bs, N - start) : 0;
    const double s = valid ? mass_at(a, row, b) : 0.0;
    const unsigned long long key = score_key(s);
    long long eq_tot;
    const long long eq_before = eq_carry + block_exclusive_scan<long long, kSelThreads>(
                                               (valid && a.top > 0 && key == T) ? len : 0, sh_ll, &eq_tot);
    eq_carry += eq_tot;
    long long top_b = 0;
    if (valid && a.top > 0) {
      if (key > T) top_b = len;
      else if (key == T) top_b = min((long long)len, max(0ll, take_eq - eq_before));
    }
    const long long sinks_b = valid ? min((long long)len, max(0ll, (long long)a.n_sinks - start)) : 0;
    const long long pref = max(sinks_b, top_b);
    const long long suf = valid ? max(0ll, start + len - max(R, start)) : 0;
    const long long uni = min((long long)len, pref + suf);
    long long cert_tot;
    const long long cb = cert_carry + block_exclusive_scan<long long, kSelThreads>(uni, sh_ll, &cert_tot);
    cert_carry += cert_tot;
    if (valid) {
      a.prefix[(long long)row * nb + b] = (int)pref;
      a.cert_before[(long long)row * nb + b] = cb;
      const double w = a.uniform_tail ? 1.0 : s;
      w_sum += w * (double)(len - uni);
    }
  }
  // 3. tail total: fixed-order tree over the threads' partial sums
  double tot = w_sum;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_down_sync(0xffffffffu, tot, o);
  if ((t & 31) == 0) sh_d[t >> 5] = tot;
  __syncthreads();
  if (t == 0) {
    double total = 0.0;
    for (int w = 0; w < kWarps; ++w) total += sh_d[w];
    RowPlan p;
    p.n_certain = cert_carry;
    p.n_tail = (long long)N - cert_carry;
    p.uniform_w = a.uniform_tail;
    if (p.n_tail > 0 && a.m > 0 && !(total > 0.0)) {  // no signal: uniform design (evict.py:147-152)
      p.uniform_w = 1;
      total = (double)p.n_tail;
    }
    p.total = total;
    p.flags = s_flags;
    a.plan[row] = p;
    int64_t* c = a.counts + (long long)row * 5;
    c[1] = p.n_certain;
    c[2] = p.n_tail;
    c[4] = p.flags;
  }
}

// Philox4x32-10 (Salmon et al. 2011): 10 rounds of the 4x32 bijection.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// Uniform double in [0, 1) with 53 random bits.
__device__ __forceinline__ double philox_uniform(unsigned long long seed, long long token, int row) {
  const uint4 r = philox4x32_10(make_uint4((uint32_t)token, (uint32_t)((unsigned long long)token >> 32),
                                           (uint32_t)row, 0u),
                                make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
  const unsigned long long bits = ((unsigned long long)r.x << 21) | (r.y >> 11);
  return (double)bits * 0x1.0p-53;
}

__global__ void __launch_bounds__(256) design_tokens_kernel(DesignArgs a) {
  __shared__ unsigned long long s_kept;
  const int row = blockIdx.y;
  if (threadIdx.x == 0) s_kept = 0;
  __syncthreads();
  const RowPlan p = a.plan[row];
  const long long R = a.recency > 0 ? max(0, a.N - a.recency) : a.N;
  unsigned long long kept = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < a.N;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / a.bs);
    const long long start = (long long)b * a.bs;
    const long long pref = a.prefix[(long long)row * a.nb + b];
    const bool certain = (i - start) < pref || i >= R;
    const double s = mass_at(a, row, b);
    double pi = 1.0;
    if (!certain) {
      if (p.n_tail > 0 && a.m > 0) {
        const double w = p.uniform_w ? 1.0 : s;
        pi = fmin(fmax((double)a.m * w / p.total, a.eps), 1.0);
      } else {
        pi = a.eps;
      }
    }
    bool keep = certain;
    if (!certain) {
      double u;
      if (a.uniforms != nullptr) {
        // t = index of this token among the tail tokens (ascending)
        const long long in_blk = i - start;
        const long long suf0 = max(R, start + pref) - start;  // suffix start inside the block
        const long long before = a.cert_before[(long long)row * a.nb + b] + min(in_blk, pref) +
                                 max(0ll, in_blk - suf0);
        u = a.uniforms[(long long)row * a.ustride + (i - before)];
      } else {
        u = philox_uniform(a.seed, i, row);
      }
      keep = u < pi;
    }
    const long long o = (long long)row * a.N + i;
    if (a.pi) a.pi[o] = pi;
    if (a.keep) a.keep[o] = keep ? 1 : 0;
    if (a.certainty) a.certainty[o] = certain ? 1 : 0;
    if (a.scores) a.scores[o] = s;
    if (a.log_offsets) a.log_offsets[o] = -log(pi);
    kept += keep ? 1 : 0;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) kept += __shfl_down_sync(0xffffffffu, kept, off);
  if ((threadIdx.x & 31) == 0) atomicAdd(&s_kept, kept);
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(reinterpret_cast<unsigned long long*>(&a.counts[(long long)row * 5]), s_kept);
}

// Blocks with at least one kept token (reclaim.py:46-55), from the keep bytes.
__global__ void __launch_bounds__(256) design_blocks_kernel(DesignArgs a, const uint8_t* keep) {
  const int row = blockIdx.y;
  unsigned long long n = 0;
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < a.nb; b += gridDim.x * blockDim.x) {
    const long long start = (long long)b * a.bs;
    const long long end = min((long long)a.N, start + a.bs);
    bool any = false;
    for (long long i = start; i < end && !any; ++i) any = keep[(long long)row * a.N + i] != 0;
    n += any ? 1 : 0;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) n += __shfl_down_sync(0xffffffffu, n, off);
  if ((threadIdx.x & 31) == 0 && n)
    atomicAdd(reinterpret_cast<unsigned long long*>(&a.counts[(long long)row * 5 + 3]), n);
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

int check_design(const kvbm_design_args* d) {
  if (d == nullptr) return KVBM_ERR_NULL;
  if (d->mass == nullptr) return KVBM_ERR_NULL;
  if (d->mass_dtype != KVBM_F32 && d->mass_dtype != KVBM_F64) return KVBM_ERR_DTYPE;
  if (d->rows < 1 || d->seq_len < 1 || d->block_size < 1 || d->num_blocks < 1) return KVBM_ERR_SHAPE;
  if ((long long)d->num_blocks * d->block_size < d->seq_len) return KVBM_ERR_SHAPE;
  if (d->mass_row_stride < d->num_blocks && d->rows > 1) return KVBM_ERR_SHAPE;
  if (!(d->eps > 0.0) || d->tail_budget < 0 || d->n_sinks < 0 || d->recency < 0 || d->top_slice < 0)
    return KVBM_ERR_SHAPE;
  if (d->uniforms != nullptr && d->uniforms_row_stride < d->seq_len && d->rows > 1) return KVBM_ERR_SHAPE;
  if (d->rows > 65535) return KVBM_ERR_SHAPE;
  if (d->seq_len > kMaxN) return KVBM_ERR_SHAPE;  // the mass passes' bound on N
  return KVBM_OK;
}

size_t design_scratch_bytes(const kvbm_design_args* d) {
  const size_t nb = (size_t)(((long long)d->seq_len + d->block_size - 1) / d->block_size);
  return align256(sizeof(RowPlan) * d->rows) + align256(sizeof(int) * nb * d->rows) +
         align256(sizeof(long long) * nb * d->rows);
}

}  // namespace
}  // namespace kvbm

using namespace kvbm;

extern "C" size_t kvbm_design_workspace_bytes(const kvbm_design_args* d) {
  if (check_design(d) != KVBM_OK) return 0;
  return design_scratch_bytes(d);
}

extern "C" int kvbm_design(const kvbm_design_args* d, const kvbm_design_out* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int st = check_design(d);
  if (st != KVBM_OK) return st;
  if (out == nullptr || out->counts == nullptr) return KVBM_ERR_NULL;
  const size_t need = design_scratch_bytes(d);
  if (workspace == nullptr || workspace_bytes < need || ((uintptr_t)workspace % 256) != 0)
    return KVBM_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DesignArgs a;
  a.mass = d->mass;
  a.mass_f64 = d->mass_dtype == KVBM_F64;
  a.mass_stride = d->rows > 1 ? d->mass_row_stride : 0;
  a.B = d->rows;
  a.N = d->seq_len;
  a.bs = d->block_size;
  a.nb = (int)(((long long)d->seq_len + d->block_size - 1) / d->block_size);
  a.m = d->tail_budget;
  a.n_sinks = d->n_sinks;
  a.recency = d->recency;
  a.top = d->top_slice < d->seq_len ? d->top_slice : d->seq_len;
  a.eps = d->eps;
  a.uniform_tail = d->uniform_tail != 0;
  a.uniforms = d->uniforms;
  a.ustride = d->rows > 1 ? d->uniforms_row_stride : 0;
  a.seed = d->seed;
  a.pi = out->pi;
  a.keep = out->keep;
  a.certainty = out->certainty;
  a.scores = out->scores;
  a.log_offsets = out->log_offsets;
  a.counts = out->counts;
  char* w = static_cast<char*>(workspace);
  a.plan = reinterpret_cast<RowPlan*>(w);
  w += align256(sizeof(RowPlan) * d->rows);
  a.prefix = reinterpret_cast<int*>(w);
  w += align256(sizeof(int) * (size_t)a.nb * d->rows);
  a.cert_before = reinterpret_cast<long long*>(w);
  if (cudaMemsetAsync(out->counts, 0, sizeof(int64_t) * 5 * d->rows, s) != cudaSuccess) return KVBM_ERR_CUDA;
  design_select_kernel<<<d->rows, kSelThreads, 0, s>>>(a);
  if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  const long long tok_blocks = ((long long)d->seq_len + 255) / 256;
  const unsigned gx = (unsigned)(tok_blocks < 148 * 8 ? tok_blocks : 148 * 8);
  design_tokens_kernel<<<dim3(gx, d->rows), 256, 0, s>>>(a);
  if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  if (out->keep != nullptr) {
    const unsigned bx = (unsigned)((a.nb + 255) / 256 < 148 ? (a.nb + 255) / 256 : 148);
    design_blocks_kernel<<<dim3(bx, d->rows), 256, 0, s>>>(a, out->keep);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  }
  return KVBM_OK;
}
