// C ABI entry points (include/kvbm.h): validation, kernel-path choice,
// workspace layout and the two-pass + reduce launch sequence.
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
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
  if ((long long)p->B * p->Hq > 65535) return KVBM_ERR_SHAPE;  // grid.y of the SIMT pass 1
  if (p->N > kMaxN) return KVBM_ERR_SHAPE;  // tile indexes fit the 21-bit work-item fields
  if (p->q == nullptr || p->k == nullptr) return KVBM_ERR_NULL;
  for (int i = 0; i < 4; ++i)
    if (p->q_stride[i] < 0 || p->k_stride[i] < 0) return KVBM_ERR_SHAPE;
  if (p->pair_mask && p->pair_mask_rstride < 0) return KVBM_ERR_SHAPE;
  if (!(p->scale == p->scale)) return KVBM_ERR_SHAPE;  // NaN scale
  return KVBM_OK;
}

// Path 1 (tcgen05, bf16/fp16) needs D <= 256 with 16-byte rows (D % 8 == 0),
// a unit-stride head dim, 16-byte aligned base pointers and row/head/batch
// strides (TMA rules); D is padded to 64/128/192/256 by the TMA's zero fill.
// Path 2 (tcgen05 3xTF32 for fp32 inputs) needs D <= 128 with D % 4 == 0; it
// reads q/k with a split kernel, so any strides work.  Both need a positive
// scale; pair masks are packed to bits for them.  Everything else runs the
// SIMT kernels.
int select_path(const kvbm_problem* p, int device) {
  if (device >= 0 && device_kind(device) != 1) return 0;
  if (!(p->scale > 0.0)) return 0;  // the exp/sum warps assume a positive scale
  if (!tc_path_enabled()) return 0;
  if (p->dtype == KVBM_F32) return (p->D <= 128 && p->D % 4 == 0) ? 2 : 0;
  if (p->dtype != KVBM_BF16 && p->dtype != KVBM_F16) return 0;
  if (p->D > 256 || p->D % 8 != 0) return 0;
  const int64_t* qs = p->q_stride;
  const int64_t* ks = p->k_stride;
  if (qs[3] != 1 || ks[3] != 1) return 0;
  for (int i = 0; i < 3; ++i)
    if ((qs[i] * 2) % 16 != 0 || (ks[i] * 2) % 16 != 0) return 0;
  if (((uintptr_t)p->q % 16) != 0 || ((uintptr_t)p->k % 16) != 0) return 0;
  return 1;
}

// SM count of a device, cached like device_kind (0 when unknown).
std::atomic<int> g_dev_sms[kMaxDevices] = {};

int device_sms(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 0;
  int n = g_dev_sms[dev].load(std::memory_order_acquire);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) {
      cudaGetLastError();
      return 0;
    }
    g_dev_sms[dev].store(n, std::memory_order_release);
  }
  return n;
}

// SM count assumed when the device is unknown (sizes a workspace that fits
// any sm_100 part).
constexpr int kMaxSms = 160;

bool one_pass_eligible(const kvbm_problem* p, int path, bool lse_input) {
  (void)lse_input;  // with the caller's LSE pass 1 forms the masses directly
  return (path == 1 || path == 2) && p->block_size % kTcExpCols == 0;
}

WsLayout layout_for(const kvbm_problem* p, int path, const Ragged* rg, int method, int sms, bool lse_input,
                    bool per_sequence) {
  if (method == KVBM_METHOD_AUTO) {
    if (!one_pass_eligible(p, path, lse_input)) return layout_for(p, path, rg, KVBM_METHOD_TWO_PASS, sms);
    const WsLayout two = layout_for(p, path, rg, KVBM_METHOD_TWO_PASS, sms);
    const WsLayout one = layout_for(p, path, rg, KVBM_METHOD_ONE_PASS, sms, false, per_sequence);
    return one.total <= 2 * two.total + (size_t(256) << 20) ? one : two;
  }
  WsLayout L;
  L.path = path;
  L.acc_bytes = (p->dtype == KVBM_F64) ? 8 : 4;
  const bool tc = path >= 1;
  // The per-key partials hold one row per query chunk: with at most
  // kMaxQueryChunks chunks they stay O(N) per unit, so long sequences widen
  // the chunks (multiples of 128 rows) instead of multiplying the rows.
  L.qchunk = tc ? kTcQChunk : kSimtQChunk;
  const int min_chunk = (p->N + kMaxQueryChunks - 1) / kMaxQueryChunks;
  if (L.qchunk < min_chunk) L.qchunk = (min_chunk + kTcTile - 1) / kTcTile * kTcTile;
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
  L.one_pass = method == KVBM_METHOD_ONE_PASS && one_pass_eligible(p, path, lse_input);
  if (L.one_pass) {
    // partials per (head, query tile, bucket); segment sums per resident CTA
    const size_t ntiles = n_lse / kTcTile;
    const size_t nb = (size_t)kvbm_num_blocks(p->N, p->block_size);
    L.part_bytes = U * G * ntiles * nb * 4;
    L.seg_tiles = p->block_size % kTcTile == 0 ? p->block_size / kTcTile : 1;
    L.seg_per_bucket = L.seg_tiles > 1 ? kTcTile / kTcExpCols : p->block_size / kTcExpCols;
    L.slot_cols = (int)((ntiles + L.seg_tiles - 1) / L.seg_tiles) * (kTcTile / kTcExpCols);
    L.slot_count = 2 * (sms > 0 ? sms : kMaxSms);
    L.slot_off = align_up(L.part_off + L.part_bytes, 256);
    L.slot_bytes = (size_t)L.slot_count * L.slot_cols * kTcTile * 4;
    // first reduce step: enough (bucket group, split) CTAs to cover the SMs
    const size_t b_out = per_sequence ? (size_t)p->B : 1;
    const size_t groups = (nb + 31) / 32 * b_out;
    const size_t items = U * G * ntiles;
    size_t splits = (296 + groups - 1) / groups;
    splits = splits < 1 ? 1 : (splits > 64 ? 64 : splits);
    if (splits > items) splits = items;
    L.red_splits = (int)splits;
    L.red_off = align_up(L.slot_off + L.slot_bytes, 256);
    L.red_bytes = splits * b_out * nb * 8;
  }
  L.split_off = align_up((L.one_pass ? L.red_off + L.red_bytes : L.part_off + L.part_bytes), 256);
  // path 2: tf32 hi/lo copies of every q and k row (packed operands: total_tokens rows per head)
  const bool q_packed = rg != nullptr && rg->cu != nullptr, k_packed = rg != nullptr && rg->k_packed;
  const size_t q_rows = q_packed ? (size_t)rg->total : (size_t)p->B * p->N;
  const size_t k_rows = k_packed ? (size_t)rg->total : (size_t)p->B * p->N;
  L.split_bytes = path == 2 ? (size_t)2 * 4 * p->D * (q_rows * p->Hq + k_rows * p->Hkv) : 0;
  L.bits_off = align_up(L.split_off + L.split_bytes, 256);
  if (tc && p->pair_mask != nullptr) {
    const bool per_b = p->pair_mask_bstride != 0 || (p->key_mask && p->key_mask_bstride != 0) ||
                       (p->query_mask && p->query_mask_bstride != 0);
    L.bits_batches = per_b ? p->B : 1;
    const size_t npad = n_lse;  // whole 128-row tiles
    L.bits_bytes = (size_t)2 * L.bits_batches * npad * (npad / 32) * 4;  // row bits + column bits
  }
  L.plan_off = align_up(L.bits_off + L.bits_bytes, 256);
  if (tc && rg != nullptr && (rg->lens != nullptr || rg->cu != nullptr)) {
    // work lists of the ragged tensor-core passes, sized for every sequence at full length
    const long long ntmax = (p->N + kTcTile - 1) / kTcTile;
    long long per_unit = 0;
    for (int y = 0; y < L.nchunk; ++y) {
      const long long lim = (long long)(y + 1) * (L.qchunk / kTcTile);
      per_unit += (p->causal && p->causal_skip) ? (lim < ntmax ? lim : ntmax) : ntmax;
    }
    L.work1_cap = (long long)U * G * ntmax;
    L.work2_cap = (long long)U * per_unit;
    L.plan_bytes = ragged_plan_layout((long long)U, ntmax, L.work1_cap, L.work2_cap).total;
  }
  L.flag_off = align_up(L.plan_off + L.plan_bytes, 256);
  L.total = L.flag_off + (tc ? 256 : 0);
  return L;
}

// Largest workspace over the kernel paths `p`'s dtype can take: SIMT, plus
// tcgen05 for bf16/fp16 (path 1) or 3xTF32 for fp32 (path 2).
size_t max_layout_bytes(const kvbm_problem* p, const Ragged* rg, int method, bool lse_input, bool per_sequence) {
  size_t m = layout_for(p, 0, rg).total;
  const int tc = p->dtype == KVBM_F32 ? 2 : (p->dtype == KVBM_F64 ? 0 : 1);
  if (tc != 0) {
    const size_t t = layout_for(p, tc, rg, method, 0, lse_input, per_sequence).total;
    m = t > m ? t : m;
  }
  return m;
}

// Launch sequence shared by the entry points: (pass 1 | lse import), pass 2,
// bucket reduce, with optional events around them.
// Stages and run ranges of a call (kvbm_options); all stages when not staged.
struct Staging {
  int stages = KVBM_STAGE_MASKS | KVBM_STAGE_PASS1 | KVBM_STAGE_PASS2 | KVBM_STAGE_REDUCE;
  int rb = 0, re = 0, hb = 0, he = 0, qb = 0, qe = 0;
};

int run_passes(const kvbm_problem* p, const WsLayout& L, int path, void* mass_out, void* ws, cudaStream_t s,
               void* const* events, const float* lse, const int64_t* lse_stride, const Ragged& rg = Ragged(),
               bool per_sequence = false, bool marked = false, const Staging& sg = Staging()) {
  auto mark = [&](int i) {
    if (events != nullptr && events[i] != nullptr)
      return cudaEventRecord(static_cast<cudaEvent_t>(events[i]), s) == cudaSuccess;
    return true;
  };
  if (!marked && !mark(0)) return KVBM_ERR_CUDA;
  const bool s1 = (sg.stages & KVBM_STAGE_PASS1) != 0, s2 = (sg.stages & KVBM_STAGE_PASS2) != 0;
  const bool sm = (sg.stages & KVBM_STAGE_MASKS) != 0, sr = (sg.stages & KVBM_STAGE_REDUCE) != 0;
  LaunchOpts o;
  o.mid_event = events != nullptr ? events[1] : nullptr;
  o.run_pass1 = s1 && (lse == nullptr || L.one_pass);
  o.lse_known = lse != nullptr && L.one_pass;
  o.run_pass2 = s2;
  o.run_split = s1;
  o.run_masks = sm;
  o.rg = rg;
  o.rb = sg.rb;
  o.re = sg.re;
  o.hb = sg.hb;
  o.he = sg.he;
  o.qb = sg.qb;
  o.qe = sg.qe;
  int st = KVBM_OK;
  if (lse != nullptr && s1) {
    nvtxRangePushA("kvbm lse import");
    st = launch_lse_import(p, L, lse, lse_stride, ws, s, rg, run_range(p, o));
    nvtxRangePop();
  }
  if (st != KVBM_OK) return st;
  if (s1 || s2 || sm) {
    // NVTX ranges mark the host-side enqueue of each pass (a profiler pairs
    // them with the kernels they launch)
    nvtxRangePushA(L.one_pass ? "kvbm pass 1 (lse + mass)"
                              : (o.run_pass1 ? "kvbm pass 1 (lse) + pass 2 (mass)" : "kvbm pass 2 (mass)"));
    st = (path >= 1) ? launch_tc(p, L, mass_out, ws, s, o) : launch_simt(p, L, mass_out, ws, s, o);
    nvtxRangePop();
    if (st != KVBM_OK) return st;
  }
  if (!mark(2)) return KVBM_ERR_CUDA;
  if (sr) {
    nvtxRangePushA("kvbm bucket reduce");
    st = launch_reduce(p, L, mass_out, ws, s, per_sequence);
    nvtxRangePop();
    if (st != KVBM_OK) return st;
  }
  return mark(3) ? KVBM_OK : KVBM_ERR_CUDA;
}

// One kvbm_block_mass_ex call resolved into what the kernels see: the
// sub-problem over the smallest box of batches x kv-heads that holds the
// requested units (a range inside one batch keeps only its heads, otherwise
// whole batches).  q, k, the masks, the LSE, the ragged arrays and a
// per-sequence output are shifted to that box's origin, so the workspace
// (the tf32 copies of fp32 inputs, per-batch pair-mask bits) covers the box
// and not the whole tensors.  A paged k is gathered into a dense array of the
// box after the dense workspace.
struct Plan {
  kvbm_problem sub;                  // the problem the kernels see (paged: k set at launch)
  Ragged rg;                         // ragged arrays, shifted to the box
  const int32_t* lens0 = nullptr;    // the caller's ragged arrays (page gather indexes b0 + b)
  const int32_t* cu0 = nullptr;
  const float* lse = nullptr;
  int64_t lse_stride[3] = {0, 0, 0};
  const kvbm_paged_kv* paged = nullptr;
  bool per_sequence = false;
  Staging staging;
  int B = 0;                         // the caller's batch (rows of a per-sequence output)
  int b0 = 0, g0 = 0;                // origin of the box
  int path = -1;                     // kernel path (-1: unknown device)
  WsLayout L;
  size_t gather_off = 0, gather_bytes = 0;
  size_t total = 0;                  // workspace bytes
};

int esize_of(int dtype) { return dtype == KVBM_F64 ? 8 : (dtype == KVBM_F32 ? 4 : 2); }

// dev < 0: the device is unknown; the workspace is sized for the largest
// layout the dtype can select.
int make_plan(const kvbm_problem* p, const kvbm_options* o, int dev, Plan* out) {
  if (p == nullptr) return KVBM_ERR_NULL;
  kvbm_options opt{};
  if (o != nullptr) opt = *o;
  if (opt.seq_lens != nullptr && opt.cu_seqlens != nullptr) return KVBM_ERR_SHAPE;
  if (opt.cu_seqlens != nullptr && (opt.total_tokens < 1 || opt.total_tokens > INT32_MAX)) return KVBM_ERR_SHAPE;
  Plan pl;
  pl.sub = *p;
  kvbm_problem& sub = pl.sub;
  const bool packed = opt.cu_seqlens != nullptr;
  if (packed) sub.q_stride[0] = 0;  // rows are addressed through cu_seqlens
  if (opt.lse != nullptr) {
    for (int i = 0; i < 3; ++i) {
      if (opt.lse_stride[i] < 0) return KVBM_ERR_SHAPE;
      pl.lse_stride[i] = opt.lse_stride[i];
    }
    if (packed) pl.lse_stride[0] = 0;
    pl.lse = opt.lse;
  }
  int st = KVBM_OK;
  const kvbm_paged_kv* kv = opt.paged;
  if (kv != nullptr) {
    if (kv->k_cache == nullptr || kv->block_table == nullptr) return KVBM_ERR_NULL;
    if (kv->num_pages < 1 || kv->page_size < 1 || kv->max_pages < 1 || kv->block_table_stride < 0)
      return KVBM_ERR_SHAPE;
    for (int i = 0; i < 4; ++i)
      if (kv->cache_stride[i] < 0) return KVBM_ERR_SHAPE;
    sub.k = kv->k_cache;  // stands in for validate(); replaced by the gathered rows
    for (int i = 0; i < 4; ++i) sub.k_stride[i] = 0;
  } else if (packed) {
    sub.k_stride[0] = 0;
  }
  st = validate(&sub);
  if (st != KVBM_OK) return st;
  if (kv != nullptr && (int64_t)kv->max_pages * kv->page_size < p->N) return KVBM_ERR_SHAPE;
  // staged execution: run ranges relative to the unit range, checked before narrowing
  const bool staged = opt.stages != 0 || opt.run_unit_end > opt.run_unit_begin ||
                      opt.run_head_end > opt.run_head_begin || opt.run_row_end > opt.run_row_begin;
  if (staged) {
    const int U = p->unit_end - p->unit_begin, G = p->Hq / p->Hkv;
    if (opt.stages < 0 || opt.stages > 15) return KVBM_ERR_SHAPE;
    if (kv != nullptr || opt.seq_lens != nullptr || opt.cu_seqlens != nullptr) return KVBM_ERR_SHAPE;
    Staging& sg = pl.staging;
    if (opt.stages != 0) sg.stages = opt.stages;
    if (opt.run_unit_end > opt.run_unit_begin) {
      if (opt.run_unit_begin < 0 || opt.run_unit_end > U) return KVBM_ERR_UNITS;
      sg.rb = opt.run_unit_begin;
      sg.re = opt.run_unit_end;
    }
    if (opt.run_head_end > opt.run_head_begin) {
      if (opt.run_head_begin < 0 || opt.run_head_end > G) return KVBM_ERR_SHAPE;
      const int nu = sg.re > sg.rb ? sg.re - sg.rb : U;
      if (opt.run_head_end - opt.run_head_begin < G && nu != 1) return KVBM_ERR_SHAPE;
      sg.hb = opt.run_head_begin;
      sg.he = opt.run_head_end;
    }
    if (opt.run_row_end > opt.run_row_begin) {
      if (opt.run_row_begin < 0 || opt.run_row_end > p->N || opt.run_row_begin % 128 != 0 ||
          (opt.run_row_end % 128 != 0 && opt.run_row_end != p->N) || opt.lse != nullptr)
        return KVBM_ERR_SHAPE;
      sg.qb = opt.run_row_begin;
      sg.qe = opt.run_row_end;
    }
  }
  {
    const int G = p->Hq / p->Hkv;
    const int b0 = p->unit_begin / p->Hkv, b1 = (p->unit_end - 1) / p->Hkv;
    int g0 = 0, ng = p->Hkv;
    if (b0 == b1) {
      g0 = p->unit_begin % p->Hkv;
      ng = (p->unit_end - 1) % p->Hkv - g0 + 1;
    }
    const int es = esize_of(p->dtype);
    sub.B = b1 - b0 + 1;
    sub.Hkv = ng;
    sub.Hq = ng * G;
    sub.q = static_cast<const char*>(p->q) + (b0 * sub.q_stride[0] + (int64_t)g0 * G * sub.q_stride[1]) * es;
    if (sub.key_mask != nullptr) sub.key_mask += b0 * p->key_mask_bstride;
    if (sub.query_mask != nullptr) sub.query_mask += b0 * p->query_mask_bstride;
    if (sub.pair_mask != nullptr) sub.pair_mask += b0 * p->pair_mask_bstride;
    sub.unit_begin = p->unit_begin - b0 * p->Hkv - g0;
    sub.unit_end = p->unit_end - b0 * p->Hkv - g0;
    if (pl.lse != nullptr) pl.lse += b0 * pl.lse_stride[0] + (int64_t)g0 * G * pl.lse_stride[1];
    pl.b0 = b0;
    pl.g0 = g0;
    if (kv != nullptr) {
      sub.k_stride[0] = (int64_t)ng * p->N * p->D;
      sub.k_stride[1] = (int64_t)p->N * p->D;
      sub.k_stride[2] = p->D;
      sub.k_stride[3] = 1;
      pl.paged = kv;
      pl.gather_bytes = align_up((size_t)sub.B * ng * p->N * p->D * es, 256);
      // the gathered rows start on a 256-byte boundary: path selection sees an aligned k
      sub.k = reinterpret_cast<const void*>(uintptr_t(256));
    } else {
      sub.k = static_cast<const char*>(p->k) + (b0 * sub.k_stride[0] + (int64_t)g0 * sub.k_stride[1]) * es;
    }
  }
  st = validate(&sub);
  if (st != KVBM_OK) return st;
  pl.lens0 = opt.seq_lens;
  pl.cu0 = opt.cu_seqlens;
  pl.rg.lens = opt.seq_lens ? opt.seq_lens + pl.b0 : nullptr;
  pl.rg.cu = packed ? opt.cu_seqlens + pl.b0 : nullptr;
  pl.rg.total = packed ? opt.total_tokens : 0;
  pl.rg.k_packed = packed && kv == nullptr;
  pl.per_sequence = opt.per_sequence != 0;
  pl.B = p->B;
  if (opt.method < KVBM_METHOD_AUTO || opt.method > KVBM_METHOD_ONE_PASS) return KVBM_ERR_SHAPE;
  const bool lse_in = pl.lse != nullptr;
  size_t dense = 0;
  if (dev >= 0) {
    pl.path = select_path(&sub, dev);
    // a pass-1 row range on the 3xTF32 path would leave the tf32 copies of
    // the other rows unconverted
    if (pl.path == 2 && pl.staging.qe > pl.staging.qb) return KVBM_ERR_SHAPE;
    if (opt.method == KVBM_METHOD_ONE_PASS && !one_pass_eligible(&sub, pl.path, lse_in)) return KVBM_ERR_SHAPE;
    pl.L = layout_for(&sub, pl.path, &pl.rg, opt.method, device_sms(dev), lse_in, pl.per_sequence);
    dense = pl.L.total;
  } else {
    if (opt.method == KVBM_METHOD_ONE_PASS && !one_pass_eligible(&sub, sub.dtype == KVBM_F32 ? 2 : 1, lse_in))
      return KVBM_ERR_SHAPE;
    if (opt.method == KVBM_METHOD_ONE_PASS && sub.dtype == KVBM_F64) return KVBM_ERR_SHAPE;
    dense = max_layout_bytes(&sub, &pl.rg, opt.method, lse_in, pl.per_sequence);
  }
  pl.gather_off = align_up(dense, 256);
  pl.total = pl.gather_off + pl.gather_bytes;
  *out = pl;
  return KVBM_OK;
}

int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess) {
    cudaGetLastError();
    *dev = -1;
    return KVBM_ERR_CUDA;
  }
  return KVBM_OK;
}

int run_plan(Plan& pl, void* mass_out, void* workspace, size_t workspace_bytes, cudaStream_t s,
             void* const* events) {
  if (mass_out == nullptr && (pl.staging.stages & KVBM_STAGE_REDUCE) != 0) return KVBM_ERR_NULL;
  if (workspace == nullptr || workspace_bytes < pl.total || ((uintptr_t)workspace % 256) != 0)
    return KVBM_ERR_WORKSPACE;
  kvbm_problem& sub = pl.sub;
  if (events != nullptr && events[0] != nullptr &&
      cudaEventRecord(static_cast<cudaEvent_t>(events[0]), s) != cudaSuccess)
    return KVBM_ERR_CUDA;
  if (pl.paged != nullptr) {
    void* gathered = static_cast<char*>(workspace) + pl.gather_off;
    sub.k = gathered;
    nvtxRangePushA("kvbm page gather");
    const int st = launch_page_gather(pl.paged, sub.dtype, pl.b0, pl.g0, sub.B, sub.Hkv, sub.N, sub.D, pl.lens0,
                                      pl.cu0, pl.rg.total, gathered, s);
    nvtxRangePop();
    if (st != KVBM_OK) return st;
  }
  void* out = mass_out;
  if (pl.per_sequence && (sub.B != pl.B) && (pl.staging.stages & KVBM_STAGE_REDUCE) != 0) {
    // rows of sequences outside the box are zeros; the box writes its own rows
    const size_t row = (size_t)kvbm_num_blocks(sub.N, sub.block_size) * (sub.dtype == KVBM_F64 ? 8 : 4);
    char* base = static_cast<char*>(mass_out);
    if (pl.b0 > 0 && cudaMemsetAsync(base, 0, row * pl.b0, s) != cudaSuccess) return KVBM_ERR_CUDA;
    const int tail = pl.B - pl.b0 - sub.B;
    if (tail > 0 && cudaMemsetAsync(base + row * (pl.b0 + sub.B), 0, row * tail, s) != cudaSuccess)
      return KVBM_ERR_CUDA;
    out = base + row * pl.b0;
  }
  return run_passes(&sub, pl.L, pl.path, out, workspace, s, events, pl.lse, pl.lse_stride, pl.rg,
                    pl.per_sequence, true, pl.staging);
}

int plan_on_device(const kvbm_problem* p, const kvbm_options* o, Plan* pl) {
  int dev = -1;
  if (current_device(&dev) != KVBM_OK) return KVBM_ERR_CUDA;
  if (device_kind(dev) != 1) {
    const int st = make_plan(p, o, -1, pl);  // argument errors first
    return st != KVBM_OK ? st : KVBM_ERR_DEVICE;
  }
  return make_plan(p, o, dev, pl);
}

int planned_workspace_bytes(const kvbm_problem* p, size_t* bytes, const kvbm_options* o) {
  Plan pl;
  const int st = plan_on_device(p, o, &pl);
  if (st != KVBM_OK) return st;
  *bytes = pl.total;
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
  // When the device is unknown (or not an sm_100), the size covers the
  // largest layout the dtype can select, so a workspace sized on the host is
  // valid for whichever path runs.
  return kvbm_workspace_bytes_ex(p, nullptr);
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
  // for 3xTF32 the split of q/k into tf32 pairs, for a pair mask its packing,
  // for a key mask on path 1 its pre-pass over the masked keys' rows; the
  // one-pass method has no pass 2 but reduces in two steps (same count)
  const int path = select_path(p, dev);
  return 3 + (path == 2 ? 1 : 0) + (path >= 1 && p->pair_mask != nullptr ? 1 : 0) +
         (path == 1 && p->key_mask != nullptr && p->pair_mask == nullptr ? 1 : 0);
}

int kvbm_block_mass(const kvbm_problem* p, void* mass_out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return kvbm_block_mass_events(p, mass_out, workspace, workspace_bytes, stream, nullptr);
}

int kvbm_block_mass_events(const kvbm_problem* p, void* mass_out, void* workspace,
                           size_t workspace_bytes, void* stream, void* const* events) {
  Plan pl;
  const int st = plan_on_device(p, nullptr, &pl);
  if (st != KVBM_OK) return st;
  return run_plan(pl, mass_out, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), events);
}

int kvbm_block_mass_lse(const kvbm_problem* p, const float* lse, const int64_t* lse_stride, void* mass_out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (lse == nullptr || lse_stride == nullptr) return KVBM_ERR_NULL;
  kvbm_options o{};
  o.lse = lse;
  for (int i = 0; i < 3; ++i) o.lse_stride[i] = lse_stride[i];
  return kvbm_block_mass_ex(p, &o, mass_out, workspace, workspace_bytes, stream);
}

int kvbm_validate_paged(const kvbm_problem* p, const kvbm_paged_kv* kv) {
  if (kv == nullptr) return KVBM_ERR_NULL;
  kvbm_options o{};
  o.paged = kv;
  return kvbm_validate_ex(p, &o);
}

size_t kvbm_paged_workspace_bytes(const kvbm_problem* p, const kvbm_paged_kv* kv) {
  if (kv == nullptr) return 0;
  kvbm_options o{};
  o.paged = kv;
  return kvbm_workspace_bytes_ex(p, &o);
}

int kvbm_block_mass_paged(const kvbm_problem* p, const kvbm_paged_kv* kv, const float* lse,
                          const int64_t* lse_stride, void* mass_out, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (kv == nullptr) return KVBM_ERR_NULL;
  kvbm_options o{};
  o.paged = kv;
  if (lse != nullptr) {
    if (lse_stride == nullptr) return KVBM_ERR_NULL;
    o.lse = lse;
    for (int i = 0; i < 3; ++i) o.lse_stride[i] = lse_stride[i];
  }
  return kvbm_block_mass_ex(p, &o, mass_out, workspace, workspace_bytes, stream);
}

int kvbm_validate_ex(const kvbm_problem* p, const kvbm_options* o) {
  Plan pl;
  return make_plan(p, o, -1, &pl);
}

size_t kvbm_workspace_bytes_ex(const kvbm_problem* p, const kvbm_options* o) {
  int dev = -1;
  current_device(&dev);
  if (dev >= 0 && device_kind(dev) != 1) dev = -1;
  Plan pl;
  if (make_plan(p, o, dev, &pl) != KVBM_OK) return 0;
  return pl.total;
}

int kvbm_method(const kvbm_problem* p, const kvbm_options* o) {
  Plan pl;
  const int st = plan_on_device(p, o, &pl);
  if (st != KVBM_OK) return -st;
  return pl.L.one_pass ? KVBM_METHOD_ONE_PASS : KVBM_METHOD_TWO_PASS;
}

int kvbm_block_mass_ex(const kvbm_problem* p, const kvbm_options* o, void* mass_out, void* workspace,
                       size_t workspace_bytes, void* stream) {
  Plan pl;
  const int st = plan_on_device(p, o, &pl);
  if (st != KVBM_OK) return st;
  return run_plan(pl, mass_out, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                  o != nullptr ? o->events : nullptr);
}

int kvbm_selftest_wait_timeout(void* stream, uint64_t limit_ns, int* waited) {
  if (waited == nullptr) return KVBM_ERR_NULL;
  if (limit_ns < 1000 || limit_ns > 2000000000ull) return KVBM_ERR_SHAPE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return KVBM_ERR_CUDA;
  }
  if (device_kind(dev) != 1) return KVBM_ERR_DEVICE;
  return selftest_wait_timeout(static_cast<cudaStream_t>(stream), limit_ns, waited);
}

int kvbm_copy_2d_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width,
                       int64_t height, void* stream) {
  if (dst == nullptr || src == nullptr) return KVBM_ERR_NULL;
  if (width < 0 || height < 0 || (height > 1 && (dst_pitch < width || src_pitch < width))) return KVBM_ERR_SHAPE;
  if (width == 0 || height == 0) return KVBM_OK;
  if (height == 1)
    return cudaMemcpyAsync(dst, src, (size_t)width, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? KVBM_OK
               : KVBM_ERR_CUDA;
  return cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch, (size_t)width, (size_t)height,
                           cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? KVBM_OK
             : KVBM_ERR_CUDA;
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
