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

// Where each array lives inside the caller's workspace.
struct WsLayout {
  size_t lse_off = 0, lse_bytes = 0;     // [U_sel * G * N] lse2 (Acc)
  size_t part_off = 0, part_bytes = 0;   // [U_sel * nchunk * N] per-key partials (Acc)
  size_t split_off = 0, split_bytes = 0; // path 2: tf32 hi/lo copies of q and k (fp32)
  size_t bits_off = 0, bits_bytes = 0;   // tensor-core paths with a pair mask: packed bits
  int bits_batches = 0;                  // batch entries of the packed bits (1 or B)
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

// Host helpers (kvbm_api.cu).
bool tc_path_enabled();  // kvbm_tc.cu
double exp2_fma_fraction();  // kvbm_tc.cu: share of exp2 evaluated on the FMA pipe
int validate(const kvbm_problem* p);
int select_path(const kvbm_problem* p, int device);
// `rg` sizes the tf32 split copies of a packed q/k (path 2) by their rows.
WsLayout layout_for(const kvbm_problem* p, int path, const Ragged* rg = nullptr);

// Launchers (return a kvbm_status).
struct LaunchOpts {
  void* mid_event = nullptr;  // cudaEvent_t recorded between pass 1 and pass 2 (or null)
  bool run_pass1 = true;      // false: lse2 is already in the workspace (kvbm_block_mass_lse)
  Ragged rg;                  // ragged batch lengths / packed layout
};
int launch_simt(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws, cudaStream_t s,
                const LaunchOpts& o);
int launch_tc(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws, cudaStream_t s,
              const LaunchOpts& o);
// Writes a caller's natural-log row LSE into the workspace's lse2 layout of `L.path`.
int launch_lse_import(const kvbm_problem* p, const WsLayout& L, const float* lse, const int64_t* lse_stride,
                      void* ws, cudaStream_t s, const Ragged& rg);
// per_sequence: mass_out is [B, num_blocks] (row b: the units of batch b in the range).
int launch_reduce(const kvbm_problem* p, const WsLayout& L, void* mass_out, const void* ws,
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
