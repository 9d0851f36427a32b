// C ABI entry points (include/kvbm.h): validation, kernel-path choice,
// workspace layout and the two-pass + reduce launch sequence.
#include <cuda_runtime.h>
#include <stdio.h>

#include <atomic>

#include "kvbm_internal.cuh"

namespace kvbm {

namespace {

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr int kMaxDevices = 64;
// Lazily filled per-device attribute cache: 0 unknown, 1 sm_100, 2 other.
// Threads that race on a first lookup compute and store the same value.
std::atomic<int> g_dev_kind[kMaxDevices] = {};

int device_kind(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 2;
  int kind = g_dev_kind[dev].load(std::memory_order_acquire);
  if (kind == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      cudaGetLastError();
      return 2;
    }
    kind = (major == 10 && minor == 0) ? 1 : 2;
    g_dev_kind[dev].store(kind, std::memory_order_release);
  }
  return kind;
}

}  // namespace

int validate(const kvbm_problem* p) {
  if (p == nullptr) return KVBM_ERR_NULL;
  if (p->dtype < KVBM_F32 || p->dtype > KVBM_F64) return KVBM_ERR_DTYPE;
  if (p->B < 1 || p->Hq < 1 || p->Hkv < 1 || p->N < 1 || p->D < 1) return KVBM_ERR_SHAPE;
  if (p->Hq % p->Hkv != 0) return KVBM_ERR_GQA;
  if (p->block_size < 1) return KVBM_ERR_BLOCK_SIZE;
  const int dmax = (p->dtype == KVBM_F64) ? 128 : 256;
  if (p->D > dmax) return KVBM_ERR_HEAD_DIM;
  const long long units = (long long)p->B * p->Hkv;
  if (p->unit_begin < 0 || p->unit_end > units || p->unit_begin >= p->unit_end)
    return KVBM_ERR_UNITS;
  if ((long long)p->B * p->Hq > 65535) return KVBM_ERR_SHAPE;  // grid.y of pass 1
  if (p->q == nullptr || p->k == nullptr) return KVBM_ERR_NULL;
  for (int i = 0; i < 4; ++i)
    if (p->q_stride[i] < 0 || p->k_stride[i] < 0) return KVBM_ERR_SHAPE;
  if (p->pair_mask && p->pair_mask_rstride < 0) return KVBM_ERR_SHAPE;
  if (!(p->scale == p->scale)) return KVBM_ERR_SHAPE;  // NaN scale
  return KVBM_OK;
}

// Path 1 (tcgen05, bf16/fp16) needs D in {64, 128}, a unit-stride head dim,
// 16-byte aligned base pointers and row/head/batch strides (TMA rules).
// Path 2 (tcgen05 3xTF32 for fp32 inputs) needs D in {32, 64}; it reads q/k
// with a split kernel, so any strides work.  Both need a positive scale;
// pair masks are packed to bits for them.  Everything else runs the SIMT
// kernels.
int select_path(const kvbm_problem* p, int device) {
  if (device >= 0 && device_kind(device) != 1) return 0;
  if (!(p->scale > 0.0)) return 0;  // the exp/sum warps assume a positive scale
  if (!tc_path_enabled()) return 0;
  if (p->dtype == KVBM_F32) return (p->D == 32 || p->D == 64) ? 2 : 0;
  if (p->dtype != KVBM_BF16 && p->dtype != KVBM_F16) return 0;
  if (p->D != 64 && p->D != 128) return 0;
  const int64_t* qs = p->q_stride;
  const int64_t* ks = p->k_stride;
  if (qs[3] != 1 || ks[3] != 1) return 0;
  for (int i = 0; i < 3; ++i)
    if ((qs[i] * 2) % 16 != 0 || (ks[i] * 2) % 16 != 0) return 0;
  if (((uintptr_t)p->q % 16) != 0 || ((uintptr_t)p->k % 16) != 0) return 0;
  return 1;
}

WsLayout layout_for(const kvbm_problem* p, int path) {
  WsLayout L;
  L.path = path;
  L.acc_bytes = (p->dtype == KVBM_F64) ? 8 : 4;
  const bool tc = path >= 1;
  L.qchunk = tc ? kTcQChunk : kSimtQChunk;
  L.key_tile = tc ? kTcTile : kSimtBN;
  L.nchunk = (p->N + L.qchunk - 1) / L.qchunk;
  const size_t U = (size_t)(p->unit_end - p->unit_begin);
  const size_t G = (size_t)(p->Hq / p->Hkv);
  // The tensor-core path pads each head's lse2 row to whole 128-row tiles
  // (padding rows hold +inf) so that pass 2 can bulk-copy full tiles.
  const size_t n_lse = tc ? (size_t)(p->N + kTcTile - 1) / kTcTile * kTcTile : (size_t)p->N;
  L.lse_off = 0;
  L.lse_bytes = U * G * n_lse * L.acc_bytes;
  L.part_off = align_up(L.lse_off + L.lse_bytes, 256);
  L.part_bytes = U * (size_t)L.nchunk * (size_t)p->N * L.acc_bytes;
  L.split_off = align_up(L.part_off + L.part_bytes, 256);
  L.split_bytes = path == 2 ? (size_t)2 * 4 * p->N * p->D * ((size_t)p->B * p->Hq + (size_t)p->B * p->Hkv) : 0;
  L.bits_off = align_up(L.split_off + L.split_bytes, 256);
  if (tc && p->pair_mask != nullptr) {
    const bool per_b = p->pair_mask_bstride != 0 || (p->key_mask && p->key_mask_bstride != 0) ||
                       (p->query_mask && p->query_mask_bstride != 0);
    L.bits_batches = per_b ? p->B : 1;
    const size_t npad = n_lse;  // whole 128-row tiles
    L.bits_bytes = (size_t)2 * L.bits_batches * npad * (npad / 32) * 4;  // row bits + column bits
  }
  L.total = align_up(L.bits_off + L.bits_bytes, 256);
  return L;
}

// Largest workspace over the kernel paths `p`'s dtype can take: SIMT, plus
// tcgen05 for bf16/fp16 (path 1) or 3xTF32 for fp32 (path 2).
size_t max_layout_bytes(const kvbm_problem* p) {
  size_t m = layout_for(p, 0).total;
  const int tc = p->dtype == KVBM_F32 ? 2 : (p->dtype == KVBM_F64 ? 0 : 1);
  if (tc != 0) {
    const size_t t = layout_for(p, tc).total;
    m = t > m ? t : m;
  }
  return m;
}

// Launch sequence shared by the entry points: (pass 1 | lse import), pass 2,
// bucket reduce, with optional events around them.
int run_passes(const kvbm_problem* p, const WsLayout& L, int path, void* mass_out, void* ws, cudaStream_t s,
               void* const* events, const float* lse, const int64_t* lse_stride) {
  auto mark = [&](int i) {
    if (events != nullptr && events[i] != nullptr)
      return cudaEventRecord(static_cast<cudaEvent_t>(events[i]), s) == cudaSuccess;
    return true;
  };
  if (!mark(0)) return KVBM_ERR_CUDA;
  LaunchOpts o;
  o.mid_event = events != nullptr ? events[1] : nullptr;
  o.run_pass1 = lse == nullptr;
  int st = KVBM_OK;
  if (lse != nullptr) st = launch_lse_import(p, L, lse, lse_stride, ws, s);
  if (st != KVBM_OK) return st;
  st = (path >= 1) ? launch_tc(p, L, mass_out, ws, s, o) : launch_simt(p, L, mass_out, ws, s, o);
  if (st != KVBM_OK) return st;
  if (!mark(2)) return KVBM_ERR_CUDA;
  st = launch_reduce(p, L, mass_out, ws, s);
  if (st != KVBM_OK) return st;
  return mark(3) ? KVBM_OK : KVBM_ERR_CUDA;
}

// A paged call: the dense sub-problem over the smallest box of batches x
// kv-heads that holds the requested units, and where its gathered keys go.
struct PagedPlan {
  kvbm_problem sub;        // batch/head origin shifted to (b0, g0); k set at launch
  int b0 = 0, g0 = 0;
  size_t gather_off = 0;   // gathered [B', H_kv', N, D] keys, after the dense workspace
  size_t gather_bytes = 0;
};

int plan_paged(const kvbm_problem* p, const kvbm_paged_kv* kv, PagedPlan* out) {
  if (p == nullptr || kv == nullptr) return KVBM_ERR_NULL;
  if (kv->k_cache == nullptr || kv->block_table == nullptr) return KVBM_ERR_NULL;
  if (kv->num_pages < 1 || kv->page_size < 1 || kv->max_pages < 1 || kv->block_table_stride < 0)
    return KVBM_ERR_SHAPE;
  for (int i = 0; i < 4; ++i)
    if (kv->cache_stride[i] < 0) return KVBM_ERR_SHAPE;
  kvbm_problem sub = *p;
  sub.k = kv->k_cache;  // stands in for validate(); replaced by the gathered rows
  for (int i = 0; i < 4; ++i) sub.k_stride[i] = 0;
  int st = validate(&sub);
  if (st != KVBM_OK) return st;
  if ((int64_t)kv->max_pages * kv->page_size < p->N) return KVBM_ERR_SHAPE;
  // unit u = b*H_kv + g: a range inside one batch keeps only its heads,
  // otherwise whole batches
  const int G = p->Hq / p->Hkv;
  const int b0 = p->unit_begin / p->Hkv, b1 = (p->unit_end - 1) / p->Hkv;
  int g0 = 0, ng = p->Hkv;
  if (b0 == b1) {
    g0 = p->unit_begin % p->Hkv;
    ng = (p->unit_end - 1) % p->Hkv - g0 + 1;
  }
  const int esize = p->dtype == KVBM_F64 ? 8 : (p->dtype == KVBM_F32 ? 4 : 2);
  sub.B = b1 - b0 + 1;
  sub.Hkv = ng;
  sub.Hq = ng * G;
  sub.q = static_cast<const char*>(p->q) + (b0 * p->q_stride[0] + (int64_t)g0 * G * p->q_stride[1]) * esize;
  sub.k_stride[0] = (int64_t)ng * p->N * p->D;
  sub.k_stride[1] = (int64_t)p->N * p->D;
  sub.k_stride[2] = p->D;
  sub.k_stride[3] = 1;
  if (sub.key_mask != nullptr) sub.key_mask += b0 * p->key_mask_bstride;
  if (sub.query_mask != nullptr) sub.query_mask += b0 * p->query_mask_bstride;
  if (sub.pair_mask != nullptr) sub.pair_mask += b0 * p->pair_mask_bstride;
  sub.unit_begin = p->unit_begin - b0 * p->Hkv - g0;
  sub.unit_end = p->unit_end - b0 * p->Hkv - g0;
  st = validate(&sub);
  if (st != KVBM_OK) return st;
  // The dense workspace must fit whichever kernel path runs: size it for the
  // largest layout (the gathered base address decides nothing but TMA
  // alignment, which the 256-byte offset satisfies).
  const size_t dense = max_layout_bytes(&sub);
  out->sub = sub;
  out->b0 = b0;
  out->g0 = g0;
  out->gather_off = align_up(dense, 256);
  out->gather_bytes = align_up((size_t)sub.B * ng * p->N * p->D * esize, 256);
  return KVBM_OK;
}

}  // namespace kvbm

using namespace kvbm;

extern "C" {

int kvbm_abi_version(void) { return KVBM_ABI_VERSION; }

const char* kvbm_status_string(int status) {
  switch (status) {
    case KVBM_OK: return "ok";
    case KVBM_ERR_GQA: return "GQA requires H_q % H_kv == 0";
    case KVBM_ERR_SHAPE: return "invalid or inconsistent sizes/strides";
    case KVBM_ERR_DTYPE: return "unsupported dtype (expected float32, bfloat16, float16 or float64)";
    case KVBM_ERR_HEAD_DIM: return "head dim D not supported (D <= 256; D <= 128 for float64)";
    case KVBM_ERR_BLOCK_SIZE: return "block_size must be >= 1";
    case KVBM_ERR_UNITS: return "unit range must satisfy 0 <= unit_begin < unit_end <= B*H_kv";
    case KVBM_ERR_NULL: return "required pointer is NULL";
    case KVBM_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
    case KVBM_ERR_CUDA: return "CUDA runtime error";
    case KVBM_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case KVBM_ERR_TIMEOUT: return "a device-side wait exceeded its iteration limit";
    case KVBM_ERR_SCRATCH:
      return "problem needs more scratch than the fixed area of kvbm_block_mass_static "
             "(see kvbm_static_scratch_bytes); split it into unit ranges";
    case KVBM_ERR_PAGE:
      return "a block-table entry was outside [0, num_pages); its keys were read as zeros";
    default: return "unknown status";
  }
}

int kvbm_validate(const kvbm_problem* p) { return validate(p); }

int64_t kvbm_num_blocks(int32_t N, int32_t block_size) {
  if (N < 0 || block_size < 1) return 0;
  return ((int64_t)N + block_size - 1) / block_size;
}

size_t kvbm_workspace_bytes(const kvbm_problem* p) {
  if (validate(p) != KVBM_OK) return 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  const int path = select_path(p, dev);
  // Size for the largest layout the dtype can select when the device is
  // unknown, so a workspace sized on the host is valid for whichever path runs.
  if (dev < 0) return max_layout_bytes(p);
  return layout_for(p, path).total;
}

int kvbm_kernel_path(const kvbm_problem* p) {
  const int st = validate(p);
  if (st != KVBM_OK) return -st;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  return select_path(p, dev);
}

int kvbm_launches_per_call(const kvbm_problem* p) {
  if (validate(p) != KVBM_OK) return 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  // pass 1 (lse2) or the lse import, pass 2 (per-key partials), bucket reduce,
  // for 3xTF32 the split of q/k into tf32 pairs, for a pair mask its packing
  const int path = select_path(p, dev);
  return 3 + (path == 2 ? 1 : 0) + (path >= 1 && p->pair_mask != nullptr ? 1 : 0);
}

int kvbm_block_mass(const kvbm_problem* p, void* mass_out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return kvbm_block_mass_events(p, mass_out, workspace, workspace_bytes, stream, nullptr);
}

int kvbm_block_mass_events(const kvbm_problem* p, void* mass_out, void* workspace,
                           size_t workspace_bytes, void* stream, void* const* events) {
  int st = validate(p);
  if (st != KVBM_OK) return st;
  if (mass_out == nullptr) return KVBM_ERR_NULL;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return KVBM_ERR_CUDA;
  }
  if (device_kind(dev) != 1) return KVBM_ERR_DEVICE;
  const int path = select_path(p, dev);
  const WsLayout L = layout_for(p, path);
  if (workspace == nullptr || workspace_bytes < L.total || ((uintptr_t)workspace % 256) != 0)
    return KVBM_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return run_passes(p, L, path, mass_out, workspace, s, events, nullptr, nullptr);
}

int kvbm_block_mass_lse(const kvbm_problem* p, const float* lse, const int64_t* lse_stride, void* mass_out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  int st = validate(p);
  if (st != KVBM_OK) return st;
  if (mass_out == nullptr || lse == nullptr || lse_stride == nullptr) return KVBM_ERR_NULL;
  for (int i = 0; i < 3; ++i)
    if (lse_stride[i] < 0) return KVBM_ERR_SHAPE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return KVBM_ERR_CUDA;
  }
  if (device_kind(dev) != 1) return KVBM_ERR_DEVICE;
  const int path = select_path(p, dev);
  const WsLayout L = layout_for(p, path);
  if (workspace == nullptr || workspace_bytes < L.total || ((uintptr_t)workspace % 256) != 0)
    return KVBM_ERR_WORKSPACE;
  return run_passes(p, L, path, mass_out, workspace, static_cast<cudaStream_t>(stream), nullptr, lse,
                    lse_stride);
}

int kvbm_validate_paged(const kvbm_problem* p, const kvbm_paged_kv* kv) {
  PagedPlan plan;
  return plan_paged(p, kv, &plan);
}

size_t kvbm_paged_workspace_bytes(const kvbm_problem* p, const kvbm_paged_kv* kv) {
  PagedPlan plan;
  if (plan_paged(p, kv, &plan) != KVBM_OK) return 0;
  return plan.gather_off + plan.gather_bytes;
}

int kvbm_block_mass_paged(const kvbm_problem* p, const kvbm_paged_kv* kv, const float* lse,
                          const int64_t* lse_stride, void* mass_out, void* workspace, size_t workspace_bytes,
                          void* stream) {
  PagedPlan plan;
  int st = plan_paged(p, kv, &plan);
  if (st != KVBM_OK) return st;
  if (mass_out == nullptr) return KVBM_ERR_NULL;
  if (lse != nullptr) {
    if (lse_stride == nullptr) return KVBM_ERR_NULL;
    for (int i = 0; i < 3; ++i)
      if (lse_stride[i] < 0) return KVBM_ERR_SHAPE;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return KVBM_ERR_CUDA;
  }
  if (device_kind(dev) != 1) return KVBM_ERR_DEVICE;
  if (workspace == nullptr || workspace_bytes < plan.gather_off + plan.gather_bytes ||
      ((uintptr_t)workspace % 256) != 0)
    return KVBM_ERR_WORKSPACE;
  // the dense sub-problem reads k from the gathered rows
  kvbm_problem sub = plan.sub;
  sub.k = static_cast<char*>(workspace) + plan.gather_off;
  const int path = select_path(&sub, dev);
  const WsLayout L = layout_for(&sub, path);
  if (L.total > plan.gather_off) return KVBM_ERR_WORKSPACE;  // cannot happen: plan sized the larger layout
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = launch_page_gather(kv, p->dtype, plan.b0, plan.g0, sub.B, sub.Hkv, p->N, p->D, const_cast<void*>(sub.k), s);
  if (st != KVBM_OK) return st;
  const float* sub_lse = nullptr;
  if (lse != nullptr) sub_lse = lse + plan.b0 * lse_stride[0] + (int64_t)plan.g0 * (p->Hq / p->Hkv) * lse_stride[1];
  return run_passes(&sub, L, path, mass_out, workspace, s, nullptr, sub_lse, lse_stride);
}

int kvbm_check_device_errors(void* stream) {
  int err = 0, perr = 0;
  int st = read_and_clear_device_error(static_cast<cudaStream_t>(stream), &err);
  if (st != KVBM_OK) return st;
  st = read_and_clear_page_error(static_cast<cudaStream_t>(stream), &perr);
  if (st != KVBM_OK) return st;
  return err ? KVBM_ERR_TIMEOUT : (perr ? KVBM_ERR_PAGE : KVBM_OK);
}

}  // extern "C"
