// Internal declarations shared by the block-mass kernels and the C ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kvbm.h"

namespace kvbm {

// log2(e): scores are kept in the base-2 domain, t = (q.k) * scale * log2(e),
// so softmax(s)_c = 2^(t_c - lse2) with lse2 = log2(sum_c 2^t_c).
constexpr double kLog2e = 1.4426950408889634073599246810018921;

// ---- SIMT tiles (fp32 FFMA / fp64 DFMA path) ----
constexpr int kSimtBM = 64;        // query rows per tile
constexpr int kSimtBN = 64;        // key columns per tile
constexpr int kSimtThreads = 256;  // 16 x 16 threads, 4 x 4 scores each
constexpr int kSimtQChunk = 512;   // query rows per mass-pass CTA

// ---- tcgen05 tiles (bf16 / fp16 path) ----
constexpr int kTcTile = 128;       // rows of an MMA tile (M) and key/query tile (N)
#ifndef KVBM_TC_QCHUNK
#define KVBM_TC_QCHUNK 2048
#endif
constexpr int kTcQChunk = KVBM_TC_QCHUNK;  // query rows per mass-pass CTA
// Upper bound on query chunks (partial rows per unit) on both paths; above
// N = 64 * chunk the chunks grow (Llama-3-70B N=131072 keeps 2048-row chunks
// on the tensor-core path).
constexpr int kMaxQueryChunks = 64;
// Largest sequence length accepted (2^28 positions): 128-row tiles then stay
// below 2^21, the width of a work-item field, and padded lengths fit int.
constexpr int kMaxN = 1 << 28;

// Exp/sum warpgroups of the tensor-core kernels (kvbm_tc.cu) and the columns
// of a 128-column accumulator tile each exp thread covers.
#ifndef KVBM_EXP_WG
#define KVBM_EXP_WG 2
#endif
constexpr int kTcExpCols = kTcTile / KVBM_EXP_WG;

// Stored position of row r in the tensor-core paths' lse2 array: inside each
// kTcExpCols-row group of a 128-row tile, row 8m + 2p + e goes to
// p * (kTcExpCols / 4) + 2m + e, so that the query rows one pass-2 thread
// reads (p = lane % 4) are consecutive (kvbm_tc.cu).
__host__ __device__ inline int lse_tile_slot(int r) {
  const int i = r & (kTcExpCols - 1);
  return (r & ~(kTcExpCols - 1)) | (((i >> 1) & 3) * (kTcExpCols / 4)) | ((i >> 3) << 1) | (i & 1);
}

// Where each array lives inside the caller's workspace.
struct WsLayout {
  size_t lse_off = 0, lse_bytes = 0;     // [U_sel * G * N] lse2 (Acc)
  size_t part_off = 0, part_bytes = 0;   // [U_sel * nchunk * N] per-key partials (Acc)
  size_t split_off = 0, split_bytes = 0; // path 2: tf32 hi/lo copies of q and k (fp32)
  size_t bits_off = 0, bits_bytes = 0;   // tensor-core paths with a pair mask: packed bits
  int bits_batches = 0;                  // batch entries of the packed bits (1 or B)
  // tensor-core paths with ragged lengths: the CTA work lists and their plan
  size_t plan_off = 0, plan_bytes = 0;
  size_t flag_off = 0;                   // tensor-core paths: a word of the key-mask pre-pass
  long long work1_cap = 0;               // pass-1 items: U * G * ceil(N / 128)
  long long work2_cap = 0;               // pass-2 items: U * (pass-2 CTAs of a full-length unit)
  // One-pass method (tensor-core paths): pass 1 also turns its row sums into
  // per-(head, query tile, bucket) partials, so there is no pass 2.
  //   part region: [U_sel * G, ntiles, nb] fp32 partials (in place of the per-key ones)
  //   slot region: [slot_count, slot_cols, 128] fp32 segment log-sums, one
  //                slot per CTA resident at a time (2 per SM)
  //   red region:  [red_splits, B_out, nb] fp64 sums of the first reduce step
  bool one_pass = false;
  size_t slot_off = 0, slot_bytes = 0;
  size_t red_off = 0, red_bytes = 0;
  int slot_count = 0;  // slots: 2 per SM of the device
  int slot_cols = 0;   // segment sums per row of one slot
  int seg_tiles = 1;   // key tiles one segment sum covers (F)
  int seg_per_bucket = 0;
  int red_splits = 0;  // item ranges of the first reduce step
  size_t total = 0;
  int path = 0;        // 0 SIMT, 1 tcgen05 (bf16/fp16), 2 tcgen05 3xTF32 (fp32)
  int qchunk = 0;      // query rows per mass-pass CTA
  int key_tile = 0;    // keys per mass-pass CTA
  int nchunk = 0;      // ceil(N / qchunk)
  int acc_bytes = 4;   // 4 (float) or 8 (double)
};

// Ragged batches (kvbm_options.seq_lens / cu_seqlens) as the kernels see them.
// With neither, every sequence has the problem's N positions.
struct Ragged {
  const int32_t* lens = nullptr;  // [B] lengths (padded layout), or null
  const int32_t* cu = nullptr;    // [B + 1] row offsets (packed layout of q), or null
  long long total = 0;            // rows of the packed q (and k when k_packed)
  bool k_packed = false;          // k packed like q (false: k is [B, H_kv, N, D])
};

// Where sequence b lives: its length n (<= N) and, per operand, the first row
// and the batch coordinate of its rows (packed: row cu[b], batch 0; padded:
// row 0, batch b).  A packed sequence's rows are clamped into
// [0, total): offsets that a caller got wrong never reach memory past the
// packed tensors.
struct SeqView {
  int n;
  int q_row, q_b;
  int k_row, k_b;
};

__host__ __device__ inline SeqView seq_view(const int32_t* lens, const int32_t* cu, bool k_packed, int b, int N,
                                            long long total) {
  SeqView v{N, 0, b, 0, b};
  if (cu != nullptr) {
    long long s0 = cu[b], s1 = cu[b + 1];
    s0 = s0 < 0 ? 0 : (s0 > total ? total : s0);
    s1 = s1 < s0 ? s0 : (s1 > total ? total : s1);
    const long long len = s1 - s0;
    v.n = (int)(len < N ? len : N);
    v.q_row = s0;
    v.q_b = 0;
    if (k_packed) {
      v.k_row = s0;
      v.k_b = 0;
    }
  } else if (lens != nullptr) {
    const int len = lens[b];
    v.n = len < 0 ? 0 : (len < N ? len : N);
  }
  return v;
}

// Exclusive prefix sum over a CTA of kThreads threads (one value per thread,
// in thread order); *total receives the CTA's sum.  Every thread must call it;
// warp_buf holds kThreads / 32 values in shared memory.  Fixed order:
// deterministic.
template <typename T, int kThreads>
__device__ T block_exclusive_scan(T v, T* warp_buf, T* total) {
  constexpr int kWarps = kThreads / 32;
  static_assert(kWarps >= 1 && kWarps <= 32, "one warp scans the warp sums");
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_buf[w] = x;
  __syncthreads();
  if (w == 0) {
    T s = lane < kWarps ? warp_buf[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < kWarps) warp_buf[lane] = s;  // inclusive warp prefix
  }
  __syncthreads();
  const T before = (w > 0 ? warp_buf[w - 1] : T(0)) + x - v;
  *total = warp_buf[kWarps - 1];
  __syncthreads();
  return before;
}

// Byte offsets, inside the workspace's plan region, of the arrays that the
// ragged plan kernel (kvbm_tc.cu) builds and the tensor-core passes read.
struct RaggedPlanLayout {
  size_t work1 = 0, work2 = 0;  // u64 items: pass 1 (unit, head, query tile), pass 2 (unit, chunk, key tile)
  size_t counts = 0;            // long long[2]: items in work1, work2
  size_t nt = 0, rank = 0;      // int[U]: query tiles of each unit, its place in the longest-first order
  size_t hist = 0, start = 0, fill = 0;  // int[ntmax + 1]: units per tile count, suffix sums, cursors
  size_t lvl_off = 0;           // long long[ntmax]: first pass-1 item of each query tile level
  size_t unit_off = 0;          // long long[U + 1]: first pass-2 item of each unit
  size_t total = 0;
};

inline RaggedPlanLayout ragged_plan_layout(long long U, long long ntmax, long long cap1, long long cap2) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  RaggedPlanLayout r;
  size_t o = 0;
  r.work1 = o; o = up(o + 8 * (size_t)cap1);
  r.work2 = o; o = up(o + 8 * (size_t)cap2);
  r.counts = o; o = up(o + 2 * sizeof(long long));
  r.nt = o; o = up(o + 4 * (size_t)U);
  r.rank = o; o = up(o + 4 * (size_t)U);
  r.hist = o; o = up(o + 4 * (size_t)(ntmax + 1));
  r.start = o; o = up(o + 4 * (size_t)(ntmax + 1));
  r.fill = o; o = up(o + 4 * (size_t)(ntmax + 1));
  r.lvl_off = o; o = up(o + 8 * (size_t)ntmax);
  r.unit_off = o; o = up(o + 8 * (size_t)(U + 1));
  r.total = o;
  return r;
}

// Host helpers (kvbm_api.cu).
bool tc_path_enabled();  // kvbm_tc.cu
double exp2_fma_fraction();  // kvbm_tc.cu: share of exp2 evaluated on the FMA pipe
int validate(const kvbm_problem* p);
int select_path(const kvbm_problem* p, int device);
// `rg` sizes the tf32 split copies of a packed q/k (path 2) by their rows.
// `method` is a KVBM_METHOD_*; `sms` the device's SM count (0: unknown, the
// largest supported count).
WsLayout layout_for(const kvbm_problem* p, int path, const Ragged* rg = nullptr, int method = KVBM_METHOD_TWO_PASS,
                    int sms = 0, bool lse_input = false, bool per_sequence = false);
// Whether `p` can run the one-pass method on kernel path `path`.
bool one_pass_eligible(const kvbm_problem* p, int path, bool lse_input);
// Workspace bytes kvbm_block_mass needs for `p` on the current device (the
// problem narrowed to the batches x kv-heads of its unit range).
int planned_workspace_bytes(const kvbm_problem* p, size_t* bytes, const kvbm_options* o = nullptr);

// Launchers (return a kvbm_status).
struct LaunchOpts {
  void* mid_event = nullptr;  // cudaEvent_t recorded between pass 1 and pass 2 (or null)
  bool run_pass1 = true;      // false: lse2 is already in the workspace (LSE input, two passes), or not this stage
  bool lse_known = false;     // one pass with the caller's LSE in the workspace (pass 1 forms the masses directly)
  bool run_pass2 = true;
  bool run_split = true;      // fp32 on path 2: convert the run's q/k rows to tf32 pairs
  bool run_masks = true;      // pack a pair mask into bits (tensor-core paths)
  Ragged rg;                  // ragged batch lengths / packed layout
  // Staged execution: the passes cover units [rb, re) of the problem's range
  // (relative to unit_begin) and pass 1 the q-heads [hb, he) of each group
  // and the query rows [qb, qe) of each head.
  int rb = 0, re = 0;         // re <= rb: every unit
  int hb = 0, he = 0;         // he <= hb: every head
  int qb = 0, qe = 0;         // qe <= qb: every row
};

// The units and heads a launch covers (LaunchOpts' run ranges resolved).
struct RunRange {
  int rb, nu;  // units [rb, rb + nu) of the problem's range
  int hb, nh;  // pass-1 q-heads [hb, hb + nh) of each group
  int qb, qe;  // pass-1 query rows [qb, qe)
};
inline RunRange run_range(const kvbm_problem* p, const LaunchOpts& o) {
  const int U = p->unit_end - p->unit_begin, G = p->Hq / p->Hkv;
  RunRange r;
  r.rb = o.re > o.rb ? o.rb : 0;
  r.nu = o.re > o.rb ? o.re - o.rb : U;
  r.hb = o.he > o.hb ? o.hb : 0;
  r.nh = o.he > o.hb ? o.he - o.hb : G;
  r.qb = o.qe > o.qb ? o.qb : 0;
  r.qe = o.qe > o.qb ? o.qe : p->N;
  return r;
}
int launch_simt(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws, cudaStream_t s,
                const LaunchOpts& o);
int launch_tc(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws, cudaStream_t s,
              const LaunchOpts& o);
// Writes a caller's natural-log row LSE into the workspace's lse2 layout of `L.path`.
int launch_lse_import(const kvbm_problem* p, const WsLayout& L, const float* lse, const int64_t* lse_stride,
                      void* ws, cudaStream_t s, const Ragged& rg, const RunRange& rr);
// per_sequence: mass_out is [B, num_blocks] (row b: the units of batch b in the range).
int launch_reduce(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws,
                  cudaStream_t s, bool per_sequence);

// Device error word: set when a bounded wait in a tcgen05 kernel gives up.
int read_and_clear_device_error(cudaStream_t s, int* err);
// kvbm_tc.cu: a bounded wait that nothing satisfies (kvbm_selftest_wait_timeout).
int selftest_wait_timeout(cudaStream_t s, unsigned long long limit_ns, int* waited);

// Paged-KV input (kvbm_paged.cu): copies the key rows of batches
// [b0, b0 + nb) x kv-heads [g0, g0 + ng) out of the paged cache into a dense
// contiguous [nb, ng, N, D] array `out`.
// Rows n >= the sequence's length (lens / cu, batch index b0 + b) are written
// as zeros without reading the block table.
int launch_page_gather(const kvbm_paged_kv* kv, int dtype, int b0, int g0, int nb, int ng, int N, int D,
                       const int32_t* lens, const int32_t* cu, long long total, void* out, cudaStream_t s);
// Page error word: set when a block-table entry was outside [0, num_pages).
int read_and_clear_page_error(cudaStream_t s, int* err);

}  // namespace kvbm
