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

// Host helpers (kvbm_api.cu).
bool tc_path_enabled();  // kvbm_tc.cu
int validate(const kvbm_problem* p);
int select_path(const kvbm_problem* p, int device);
WsLayout layout_for(const kvbm_problem* p, int path);

// Launchers (return a kvbm_status).
struct LaunchOpts {
  void* mid_event = nullptr;  // cudaEvent_t recorded between pass 1 and pass 2 (or null)
  bool run_pass1 = true;      // false: lse2 is already in the workspace (kvbm_block_mass_lse)
};
int launch_simt(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws, cudaStream_t s,
                const LaunchOpts& o);
int launch_tc(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws, cudaStream_t s,
              const LaunchOpts& o);
// Writes a caller's natural-log row LSE into the workspace's lse2 layout of `L.path`.
int launch_lse_import(const kvbm_problem* p, const WsLayout& L, const float* lse, const int64_t* lse_stride,
                      void* ws, cudaStream_t s);
int launch_reduce(const kvbm_problem* p, const WsLayout& L, void* mass_out, const void* ws,
                  cudaStream_t s);

// Device error word: set when a bounded wait in a tcgen05 kernel gives up.
int read_and_clear_device_error(cudaStream_t s, int* err);

// Paged-KV input (kvbm_paged.cu): copies the key rows of batches
// [b0, b0 + nb) x kv-heads [g0, g0 + ng) out of the paged cache into a dense
// contiguous [nb, ng, N, D] array `out`.
int launch_page_gather(const kvbm_paged_kv* kv, int dtype, int b0, int g0, int nb, int ng, int N, int D,
                       void* out, cudaStream_t s);
// Page error word: set when a block-table entry was outside [0, num_pages).
int read_and_clear_page_error(cudaStream_t s, int* err);

}  // namespace kvbm
