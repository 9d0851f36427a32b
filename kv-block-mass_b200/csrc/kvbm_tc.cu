// tcgen05 (sm_100a tensor core) block-mass kernels for bf16 / fp16 inputs
// with head dim 64 or 128.
//
// Both passes stream 128 x 128 score tiles through TMEM:
//   warp 0     TMA producer (one elected lane): Q/K tiles -> 128B-swizzled smem
//   warp 1     MMA issuer (one lane) + TMEM owner: tcgen05.mma kind::f16, fp32
//              accumulators in two 128-column TMEM buffers
//   warps 2-9  exp/sum: two warpgroups, each reading one 64-column half of
//              every accumulator row with tcgen05.ld (one thread per row
//              and half), so four exp warps share each SM sub-partition
//
// Pass 1 (row log-sum-exp) follows the reference Triton kernel's pass 1
// (kv-block-mass src/kvblockmass/triton_kernel.py:69-104): S = Q K^T with
// query rows as the MMA's M.  Each thread keeps an online max / denominator
// over its column half of every key tile in registers; the two halves of a
// row merge once, at the end.  Causal tiles stop at the query tile's last
// row (triton_kernel.py:57-60).
//
// Pass 2 (mass) recomputes the scores transposed, S^T = K Q^T with key rows as
// M, so each thread owns one key (and one half of the query columns) and
// sums 2^(t - lse2) over every query of every head of its GQA group
// (triton_kernel.py:106-145, reference.py:121-124) in registers.  One partial
// per (unit, query chunk, key) goes to the workspace; the SIMT reduce
// (kvbm_simt.cu) adds them in a fixed order.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "kvbm_internal.cuh"
#include "kvbm_sm100.cuh"

namespace kvbm {

namespace {
using namespace sm100;

constexpr int TILE = kTcTile;       // 128
// The exp/sum warps form kExpWG warpgroups; warpgroup w covers the columns
// [w * COLS, (w + 1) * COLS) of every accumulator tile.
constexpr int kExpWG = KVBM_EXP_WG;
constexpr int COLS = kTcExpCols;    // columns per exp thread and tile
constexpr int kExpThreads = 128 * kExpWG;
constexpr int kThreads = 64 + kExpThreads;  // + TMA warp + MMA warp
static_assert(COLS == TILE / kExpWG && COLS % 32 == 0, "exp warpgroups split a tile's columns evenly");
#ifndef KVBM_STAGES
#define KVBM_STAGES 2
#endif
constexpr int kStages = KVBM_STAGES;  // K (pass 1) / Q (pass 2) ring depth
// lse2 ring depth (pass 2).  The ring has no release barrier of its own: the
// producer refills the slot of tile j - kLStages only after the MMA of tile
// j - kStages completed (its Q-slot wait), that MMA waited until every exp
// thread released the TMEM buffer of tile j - kStages - 2, and an exp thread
// releases a buffer only after it finished computing the tile before it.  So
// every exp thread is done with tiles <= j - kStages - 3, which covers the
// slot's previous tile when kLStages >= kStages + 3.
constexpr int kLStages = 8;
static_assert(kLStages >= kStages + 3, "lse2 ring too shallow to be reused without a release barrier");
// Pass 2 folds -lse2 into the accumulator (KVBM_P2_BIAS, bf16/fp16 inputs):
// after a tile's K steps, one more 16-element K step adds ones (key side) x
// the bf16 split hi + mid + lo of -lse2 / C (query side), so the exp threads
// compute 2^(C * D) with no per-column lse2 load.
#ifndef KVBM_P2_BIAS
#define KVBM_P2_BIAS 1
#endif
constexpr int kBiasBytes = TILE * 32;  // a 128-row x 16-element bf16 operand
constexpr int kTmemCols = 256;      // two 128-column fp32 accumulators
constexpr int kMinSmem = 100 * 1024;  // caps residency at 2 CTAs/SM (TMEM: 2 x 256 columns)
// k bytes that the units of one pass-1 CTA group may hold together (L2 is 126 MB).
#ifndef KVBM_P1_GROUP_MIB
#define KVBM_P1_GROUP_MIB 32
#endif
constexpr long long kPass1GroupBytes = (long long)KVBM_P1_GROUP_MIB << 20;
constexpr int kExpBarrier = 1;      // named barrier of the exp threads
#ifndef KVBM_P1_KEY_BIAS
#define KVBM_P1_KEY_BIAS 1
#endif
#ifndef KVBM_L2_HINTS
#define KVBM_L2_HINTS 1
#endif

struct TcArgs {
  int N, Npad, G, Hkv, ub;
  float C;                 // scale * log2(e), > 0
  int causal, skip;
  const uint8_t* kmask;    // [B|1, N] or null
  long long kmb;
  const uint8_t* qmask;    // [B|1, N] or null
  long long qmb;
  float* lse;              // [U_sel * G, Npad], stored negated (-lse2)
  float* part;             // [U_sel, nchunk, N]
  const uint32_t* prow;    // pair mask bits, [Bm, Npad, W]: row = query, bit = key (or null)
  const uint32_t* pcol;    // the same bits transposed: row = key, bit = query
  long long pb;            // batch stride of prow/pcol in words (0: shared by all batch entries)
  int W;                   // words per bit row (Npad / 32)
  int qchunk, nchunk;
  int per_unit;            // pass-2 CTAs per unit (sum of keys_in_chunk over chunks)
  int usel, ugroup;        // pass 1 (uniform grid): units run, units per CTA group
  int rb;                  // first unit run (relative to ub; staged calls run a sub-range)
  int hb, hn;              // pass 1 runs q-heads [hb, hb + hn) of each group
  int qt0, nqts;           // and query tiles [qt0, qt0 + nqts) of each head (uniform grid)
  const int32_t* lens;     // ragged lengths [B] or null
  const int32_t* cu;       // packed row offsets [B+1] or null
  int kpacked;             // k packed like q
  long long total;         // rows of the packed q (and k)
  // kRagged: the CTA work lists built by ragged_plan_kernel
  const unsigned long long* work1;  // pass 1: (unit, head, query tile), longest tiles first
  const unsigned long long* work2;  // pass 2: (unit, chunk, key tile), unit-major
  const long long* work_count;      // items in work1, work2
  // One-pass method: pass 1 keeps, per row, the log2-sum of 2^(s*C) over each
  // segment of seg_tiles key tiles x one exp thread's COLS columns in a slot
  // of `slots`, and at the end turns them into the bucket partials `part1`.
  int one_pass;
  int lse_known;           // one pass with the caller's row LSE (already in `lse`): no running max
  int nb, bs;              // buckets of the mass vector, block size
  int seg_tiles;           // key tiles one segment covers (block_size / 128, or 1)
  int seg_per_bucket;      // segments of one bucket
  int slot_cols;           // segments per row of one slot
  int slot_count;          // slots: 2 per SM (index 2 * %smid + TMEM half)
  float* slots;            // [slot_count][slot_cols][128]
  float* part1;            // [U_sel * G][Npad / 128][nb]
  const unsigned* keys_finite;  // kKeysFiniteMark: every key the key mask drops has a finite k row
};

// Written over the key-mask check word (byte-wise 0x5A) before the pre-pass;
// the pre-pass clears it on a non-finite element, and pass 1 trusts the bias
// alone only on this exact value (an unset workspace takes the select).
constexpr unsigned kKeysFiniteMark = 0x5A5A5A5Au;

// A work item: three fields of 21 bits (units, heads, chunks and tiles all
// stay below 2^21).
__host__ __device__ constexpr unsigned long long pack_item(int hi, int mid, int lo) {
  return ((unsigned long long)hi << 42) | ((unsigned long long)mid << 21) | (unsigned long long)lo;
}
__host__ __device__ constexpr int item_hi(unsigned long long it) { return (int)(it >> 42); }
__host__ __device__ constexpr int item_mid(unsigned long long it) { return (int)((it >> 21) & 0x1FFFFFull); }
__host__ __device__ constexpr int item_lo(unsigned long long it) { return (int)(it & 0x1FFFFFull); }

// Key tiles of query chunk y that hold a kept pair: with causal_skip only
// those up to the chunk's last row, otherwise all of them.
__host__ __device__ inline int keys_in_chunk(const TcArgs& a, int y) {
  const int ntiles = a.Npad / TILE;
  if (!(a.causal && a.skip)) return ntiles;
  const int lim = (y + 1) * (a.qchunk / TILE);
  return lim < ntiles ? lim : ntiles;
}

// Mask handled inside the tensor-core kernels (causality is always index math).
constexpr int kMaskNone = 0;   // no mask
constexpr int kMaskKeys = 1;   // [B|1, N] key mask
constexpr int kMaskPairs = 2;  // [B|1, N, N] pair mask, packed to bits (key/query masks folded in)

// Operand type of the MMAs.  TF32X3 carries an fp32 operand as a tf32 pair
// hi + lo (hi = tf32(x), lo = x - hi, both stored as fp32) and multiplies
// A.B ~= A_hi.B_lo + A_lo.B_hi + A_hi.B_hi, about 2^-22 relative error (the
// A_lo.B_lo term is below that), i.e. fp32-grade scores from tf32 MMAs.
enum class Op { F16, BF16, TF32X3 };

template <int D, Op kOp>
struct Cfg {
  static constexpr int kElem = kOp == Op::TF32X3 ? 4 : 2;    // bytes per element in smem
  static constexpr int kBlockElems = 128 / kElem;            // elements per 128-byte row block
  static constexpr int kBlocks = D * kElem / 128;            // 128-byte K-blocks per row
  static constexpr int kBlockBytes = TILE * 128;             // 16 KB
  static constexpr int kTileBytes = TILE * D * kElem;        // one component tile
  static constexpr int kParts = kOp == Op::TF32X3 ? 2 : 1;   // tiles per operand (hi, lo)
  static constexpr int kOperandBytes = kTileBytes * kParts;  // one ring slot
  static constexpr int kSteps = kBlocks * 4;                 // 32-byte (K=16 f16 / K=8 tf32) MMA steps
  static constexpr uint32_t kFmt = kOp == Op::F16 ? 0u : kOp == Op::BF16 ? 1u : 2u;
  static_assert(kBlocks >= 1 && D * kElem % 128 == 0, "row must be whole 128-byte blocks");
  // The streamed operand (K in pass 1, Q in pass 2) goes through ring slots of
  // kSlotBlocks K-blocks: a whole tile per slot, except for fp32 at D = 128 on
  // the 3xTF32 path, whose tile (hi + lo: 128 KB) streams one 128-byte K-block
  // (32 KB) per slot, so that the resident operand and two slots fit in
  // shared memory.  The MMAs of a tile then run block by block as they land.
  static constexpr int kSlotBlocks = (kOp == Op::TF32X3 && kBlocks > 2) ? 1 : kBlocks;
  static constexpr int kSlotsPerTile = kBlocks / kSlotBlocks;
  static constexpr int kSlotPartBytes = kSlotBlocks * kBlockBytes;  // one component of a slot
  static constexpr int kSlotBytes = kSlotPartBytes * kParts;
  static_assert(kBlocks % kSlotBlocks == 0, "slots hold whole K-blocks");
};

__device__ __forceinline__ uint8_t* align1k(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

__device__ __forceinline__ void exp_bar_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kExpBarrier), "n"(kExpThreads) : "memory");
}

// Issue the MMAs of the K-blocks of one ring slot of a 128 x 128 tile,
// D[tmem] (+)= A * B^T: A is the resident operand (every K-block, component
// tiles kTileBytes apart), B the slot holding K-blocks [kb0, kb0 + kSlotBlocks)
// (components kSlotPartBytes apart).  The tile's first K-step overwrites D.
template <int D, Op kOp>
__device__ __forceinline__ void issue_slot_mma(uint32_t d_tmem, uint32_t a_smem, uint32_t b_smem, int kb0,
                                               uint32_t idesc) {
  using C = Cfg<D, kOp>;
#pragma unroll
  for (int i = 0; i < C::kSlotBlocks; ++i) {
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
      const uint32_t aoff = (kb0 + i) * C::kBlockBytes + k4 * 32;
      const uint32_t boff = i * C::kBlockBytes + k4 * 32;
      const uint32_t acc = (kb0 + i > 0 || k4 > 0) ? 1u : 0u;
      if constexpr (kOp == Op::TF32X3) {
        // the small cross terms first, then hi.hi
        mma_tf32(d_tmem, sw128_desc(a_smem + C::kTileBytes + aoff), sw128_desc(b_smem + boff), idesc, acc);
        mma_tf32(d_tmem, sw128_desc(a_smem + aoff), sw128_desc(b_smem + C::kSlotPartBytes + boff), idesc, 1u);
        mma_tf32(d_tmem, sw128_desc(a_smem + aoff), sw128_desc(b_smem + boff), idesc, 1u);
      } else {
        mma_f16(d_tmem, sw128_desc(a_smem + aoff), sw128_desc(b_smem + boff), idesc, acc);
      }
    }
  }
}

// TMA-load the resident operand (every K-block of all its component tiles)
// of rows [row, row + 128) of head h of batch b into `dst`, completing on `bar`.
template <int D, Op kOp>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* m0, const CUtensorMap* m1,
                                             uint64_t* bar, int row, int h, int b) {
  using C = Cfg<D, kOp>;
#pragma unroll
  for (int part = 0; part < C::kParts; ++part)
#pragma unroll
    for (int kb = 0; kb < C::kBlocks; ++kb)
      tma_load_4d(dst + part * C::kTileBytes + kb * C::kBlockBytes, part == 0 ? m0 : m1, bar,
                  kb * C::kBlockElems, row, h, b);
}

// load_operand with an L2 eviction policy on every copy.
template <int D, Op kOp>
__device__ __forceinline__ void load_operand_hint(uint8_t* dst, const CUtensorMap* m0, const CUtensorMap* m1,
                                                  uint64_t* bar, int row, int h, int b, uint64_t policy) {
  using C = Cfg<D, kOp>;
#pragma unroll
  for (int part = 0; part < C::kParts; ++part)
#pragma unroll
    for (int kb = 0; kb < C::kBlocks; ++kb)
      tma_load_4d_hint(dst + part * C::kTileBytes + kb * C::kBlockBytes, part == 0 ? m0 : m1, bar,
                       kb * C::kBlockElems, row, h, b, policy);
}

// TMA-load ring slot `sb` of a streamed tile: K-blocks [sb * kSlotBlocks, ..)
// of every component, kSlotBytes in all, completing on `bar`.
template <int D, Op kOp>
__device__ __forceinline__ void load_slot(uint8_t* dst, const CUtensorMap* m0, const CUtensorMap* m1,
                                          uint64_t* bar, int sb, int row, int h, int b) {
  using C = Cfg<D, kOp>;
#pragma unroll
  for (int part = 0; part < C::kParts; ++part)
#pragma unroll
    for (int i = 0; i < C::kSlotBlocks; ++i)
      tma_load_4d(dst + part * C::kSlotPartBytes + i * C::kBlockBytes, part == 0 ? m0 : m1, bar,
                  (sb * C::kSlotBlocks + i) * C::kBlockElems, row, h, b);
}

// One exp thread's COLS consecutive accumulator columns of its TMEM lane.
__device__ __forceinline__ void load_cols(uint32_t taddr, float (&v)[COLS]) {
#pragma unroll
  for (int i = 0; i < COLS / 32; ++i) tmem_ld32(taddr + 32 * i, *reinterpret_cast<float(*)[32]>(&v[32 * i]));
  tmem_ld_wait();
}

// Of every 16 four-column groups of a row, KVBM_EMU_GROUPS take their exp2
// from the FMA-pipe polynomial (exp2_fma2) and the rest from MUFU
// ex2.approx: one ex2 per score element is the binding unit of both passes,
// and the FMA pipe has room to absorb part of it.  The groups are spread
// evenly so that the scheduler can interleave both kinds.
// 4 of 16 groups, degree-4 polynomial: on the Llama-3-8B N=32768 step a
// sweep of 2-6 groups x degree 3/4 gave 10.05 ms for this choice against
// 10.1-10.2 ms for 2 groups.  Degree 3 (max relative error 7.5e-5) was about
// 1% faster still, but its bias does not cancel between the two passes: the
// sum rule of the Llama-3-70B N=131072 shape came out 1.15e-5 off, over the
// 1e-5 that the sum rule must hold to.
#ifndef KVBM_EMU_GROUPS
#define KVBM_EMU_GROUPS 4
#endif
// Degree of the FMA-pipe polynomial for bf16/fp16 inputs (4: max relative
// error 2.7e-6; fp32 inputs on the 3xTF32 path always use degree 4).
#ifndef KVBM_EXP2_DEGREE
#define KVBM_EXP2_DEGREE 4
#endif
// The same for the one-pass kernel.  There each row's bucket masses and its
// normaliser are sums of the same exponentials (segment sums over sum of all
// of them), so a polynomial's bias cancels in the sum rule, and degree 3
// (max relative error 7.5e-5 per emulated element, one FFMA2 fewer) stays
// far inside the 1e-3 of bf16/fp16 inputs: on the Llama-3-8B N=32768 step it
// measured 4.82-4.90 ms against 4.95-5.01 ms for degree 4 (three interleaved
// rounds of 20 steps; 5.235 against 5.299 ms sustained).
#ifndef KVBM_EXP2_DEGREE_ONE_PASS
#define KVBM_EXP2_DEGREE_ONE_PASS 3
#endif
constexpr int kEmuPer16 = KVBM_EMU_GROUPS;
constexpr int kGroups = COLS / 4;                     // four-column groups of one thread's row
constexpr int kEmuGroups = kEmuPer16 * kGroups / 16;  // of them on the FMA pipe
static_assert(kEmuPer16 >= 0 && kEmuPer16 <= 16 && kEmuPer16 * kGroups % 16 == 0,
              "the emulated share must be whole groups of a thread's columns");

__host__ __device__ constexpr bool emu_group(int g) {
  return ((g + 1) * kEmuGroups) / kGroups != (g * kEmuGroups) / kGroups;  // Bresenham spread
}

template <Op kOp>
constexpr int exp2_degree() {
  return kOp == Op::TF32X3 ? 4 : KVBM_EXP2_DEGREE;
}
template <Op kOp>
constexpr int exp2_degree_one_pass() {
  return kOp == Op::TF32X3 ? 4 : KVBM_EXP2_DEGREE_ONE_PASS;
}

// Sum over the thread's columns of 2^(v*C + nm), nm = -(running max); masked entries hold -inf.
template <int kDeg>
__device__ __forceinline__ float row_sum_exp2(const float (&v)[COLS], float C, float nm) {
  const float2 C2 = make_float2(C, C), N2 = make_float2(nm, nm);
  float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll
  for (int g = 0; g < kGroups; ++g) {
    const int c = 4 * g;
    const float2 x0 = ffma2(make_float2(v[c], v[c + 1]), C2, N2);
    const float2 x1 = ffma2(make_float2(v[c + 2], v[c + 3]), C2, N2);
    if (emu_group(g)) {
      a0 = fadd2_ftz(a0, exp2_fma2<kDeg>(x0));
      a1 = fadd2_ftz(a1, exp2_fma2<kDeg>(x1));
    } else {
      a0 = fadd2_ftz(a0, make_float2(ex2(x0.x), ex2(x0.y)));
      a1 = fadd2_ftz(a1, make_float2(ex2(x1.x), ex2(x1.y)));
    }
  }
  a0 = fadd2(a0, a1);
  return a0.x + a0.y;
}

// ---- pass 2: thread layout and the lse2 order ----
// A pass-2 exp thread reads its warp's 32 TMEM lanes (keys) x its
// warpgroup's COLS query columns with two tcgen05.ld.16x256b loads (lanes +0
// and +16), each covering kBlk = COLS / 8 blocks of 8 columns.  Lane l then
// holds the keys l/4 + {0, 8, 16, 24} of the warp's 32 and, in each block m,
// the query columns 8m + 2(l%4) + {0, 1}: 4 keys x 2*kBlk columns, in
//   v[(COLS/2)*ld + 4m + 2*rr + e] = (key l/4 + 16*ld + 8*rr, column 8m + 2(l%4) + e).
// The 2*kBlk columns of lane l need as many lse2 values, which are stored
// consecutively (lse_tile_slot), so a thread reads them with kBlk/2 shared
// loads per tile (a full row of COLS columns per thread would need COLS/4).
constexpr int kBlk = COLS / 8;

// Of the kBlk column blocks of a pass-2 thread, KVBM_EMU_GROUPS_P2/16 of them
// take their exp2 from the FMA-pipe polynomial (by default the same share as
// pass 1).
#ifndef KVBM_EMU_GROUPS_P2
#define KVBM_EMU_GROUPS_P2 KVBM_EMU_GROUPS
#endif
constexpr int kEmuPer16P2 = KVBM_EMU_GROUPS_P2;
constexpr int kEmuBlocks = kEmuPer16P2 * kBlk / 16;
static_assert(kEmuPer16P2 >= 0 && kEmuPer16P2 <= 16 && kEmuPer16P2 * kBlk % 16 == 0,
              "pass 2 emulates whole 8-column blocks");
__host__ __device__ constexpr bool emu_block(int m) {
  return ((m + 1) * kEmuBlocks) / kBlk != (m * kEmuBlocks) / kBlk;
}

// acc[i] += 2^(v*C + nL) over one thread's 4 keys (i: key l/4 + 8i) x 2*kBlk
// query columns, nL = -lse2 of the columns (lse_tile_slot order, this
// thread's 2*kBlk values at nL[2*kBlk * (l%4) ..]).  Masks (a masked element
// adds 0): kDiag keeps column col >= keep_from + 8i of key i (the causal
// diagonal tile); kBits keeps column col of key i iff bit col of bits[i] is
// set (the thread's COLS columns); kTail keeps columns col < keep_to (a
// ragged sequence's end).
// kBias: the accumulator already holds s - lse2 / C (no nL reads).
template <int kDeg, bool kDiag, bool kBits, bool kTail, bool kBias = false>
__device__ __forceinline__ void col_sum4(const float (&v)[COLS], float C, const float* nL, int pc, int keep_from,
                                         const uint2 (&bits)[4], int keep_to, float2 (&acc)[4]) {
  const float2 C2 = make_float2(C, C);
  const float4* l4p = reinterpret_cast<const float4*>(nL + pc * 2 * kBlk);
#pragma unroll
  for (int mp = 0; mp < kBlk / 2; ++mp) {
    const float4 l4 = kBias ? make_float4(0.f, 0.f, 0.f, 0.f) : l4p[mp];  // -lse2 of blocks 2mp, 2mp + 1
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = 2 * mp + h;
      const float2 L = h ? make_float2(l4.z, l4.w) : make_float2(l4.x, l4.y);
      const int col = 8 * m + 2 * pc;  // this thread's first column in block m (warpgroup-local)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int o = (COLS / 2) * (i >> 1) + 4 * m + 2 * (i & 1);
        float2 x = make_float2(v[o], v[o + 1]);
        if (kDiag) {
          x.x = col - 8 * i >= keep_from ? x.x : -INFINITY;
          x.y = col + 1 - 8 * i >= keep_from ? x.y : -INFINITY;
        }
        if (kBits) {
          const uint32_t w = m < 4 ? bits[i].x : bits[i].y;
          x.x = ((w >> (col & 31)) & 1u) ? x.x : -INFINITY;
          x.y = ((w >> ((col + 1) & 31)) & 1u) ? x.y : -INFINITY;
        }
        if (kTail) {
          x.x = col < keep_to ? x.x : -INFINITY;
          x.y = col + 1 < keep_to ? x.y : -INFINITY;
        }
        x = ffma2(x, C2, L);
        acc[i] = fadd2_ftz(acc[i], emu_block(m) ? exp2_fma2<kDeg>(x) : make_float2(ex2(x.x), ex2(x.y)));
      }
    }
  }
}

// A pass-2 thread's 4 keys x 2*kBlk columns: lanes +0..15, then +16..31.
__device__ __forceinline__ void load_keys16(uint32_t taddr, float (&v)[COLS]) {
#pragma unroll
  for (int ld = 0; ld < 2; ++ld) {
    const uint32_t t = taddr + ((uint32_t)(16 * ld) << 16);
    if constexpr (COLS == 64)
      tmem_ld16x256_x8(t, *reinterpret_cast<float(*)[32]>(&v[32 * ld]));
    else
      tmem_ld16x256_x4(t, *reinterpret_cast<float(*)[16]>(&v[16 * ld]));
  }
  tmem_ld_wait();
}
static_assert(COLS == 64 || COLS == 32, "pass-2 loads cover 32 or 64 columns");

// Max of a thread's COLS columns (3-input max tree).
__device__ __forceinline__ float row_max(const float (&v)[COLS]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(v[i], v[i + 8]);
#pragma unroll
  for (int c = 16; c < COLS; c += 16)
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      m[i] = fmax3(m[i], v[c + i], v[c + i + 8]);
      m[i + 1] = fmax3(m[i + 1], v[c + i + 1], v[c + i + 9]);
    }
  return fmax3(fmax3(m[0], m[1], m[2]), fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// Merge two online-softmax states (m, l) in the base-2 domain.
__device__ __forceinline__ void merge_ml(float& m, float& l, float mo, float lo) {
  const float mn = fmaxf(m, mo);
  if (mn == -INFINITY) return;  // both halves saw only masked entries
  l = l * ex2(m - mn) + lo * ex2(mo - mn);
  m = mn;
}

// ============================================================ pass 1: lse2
// 1-D grid of U_sel * G * ceil(N / 128) CTAs.  The units are cut into groups
// of a.ugroup (the last may be smaller) whose k fits in L2 together; the grid
// runs the groups one after another, and inside a group the query tiles from
// the last (longest under causal_skip) to the first, every (unit, head) of the
// group per tile.
template <int D, Op kOp, int kMask, bool kRagged>
__global__ void __launch_bounds__(kThreads, 2)
    tc_lse_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tq2,
                  const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tk2, TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  using CF = Cfg<D, kOp>;
  // A key mask is folded into the accumulator: after a tile's K steps, one
  // more bf16 MMA adds ones (query side) x [0 or -inf, 0, ...] (key side:
  // -inf for a masked key or one past the sequence), which the producer warp
  // writes per K slot from the mask bytes.  Kept scores gain exact zeros, so
  // the bits are those of a select; the exp threads then mask only the
  // causal diagonal.  (fp32 on the 3xTF32 path has no shared memory left for
  // the operand and keeps the select.)
  constexpr bool kKeyBias = KVBM_P1_KEY_BIAS != 0 && kMask == kMaskKeys && kOp != Op::TF32X3;
  static_assert(!kKeyBias || CF::kSlotsPerTile == 1, "the key bias step follows a whole K tile per slot");
  constexpr int TB = CF::kOperandBytes, SB = CF::kSlotBytes;
  constexpr int KS = SB + (kKeyBias ? kBiasBytes : 0);  // K ring slot: the K operand, then its key-bias operand
  static_assert(KS % 1024 == 0, "K slots stay on 1024-byte swizzle atoms");
  uint8_t* q_tile = smem;
  uint8_t* k_ring = smem + TB;
  uint8_t* ones = k_ring + KS * kStages;  // kKeyBias: the query-side operand of the bias step
  float2* merge = reinterpret_cast<float2*>(ones + (kKeyBias ? kBiasBytes : 0));  // [kExpWG - 1][128] (m, l) of parts 1..
  float* lse_s = reinterpret_cast<float*>(merge + (kExpWG - 1) * TILE);  // [128] -lse2 (one pass)
  uint64_t* bars = reinterpret_cast<uint64_t*>(lse_s + TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kStages;
  uint64_t* s_full = k_empty + kStages;
  uint64_t* s_empty = s_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Uniform lengths: grid (unit x head, query tile from the last).  kRagged:
  // a 1-D grid over the plan's work list, which holds only tiles that exist
  // (longest first); the CTAs past its end return at once, at the tail.
  int hidx, qt;
  if constexpr (kRagged) {
    if ((long long)blockIdx.x >= a.work_count[0]) return;
    const unsigned long long it = a.work1[blockIdx.x];
    hidx = item_hi(it) * a.G + item_mid(it);
    qt = item_lo(it);
  } else {
    const long long per_group = (long long)a.ugroup * a.hn * a.nqts;
    const int grp = (int)(blockIdx.x / per_group);
    const int r = (int)(blockIdx.x - grp * per_group);
    const int width = min(a.ugroup, a.usel - grp * a.ugroup) * a.hn;  // (unit, head) pairs of this group
    const int pr = r % width;
    hidx = (a.rb + grp * a.ugroup + pr / a.hn) * a.G + a.hb + pr % a.hn;
    qt = a.qt0 + a.nqts - 1 - r / width;
  }
  const int u = a.ub + hidx / a.G, hh = hidx % a.G;
  const int b = u / a.Hkv, g = u % a.Hkv, h = g * a.G + hh;
  // kRagged: per-sequence lengths / packed rows (kvbm_options); otherwise
  // every sequence has a.N positions at rows [0, a.N) of batch entry b
  const SeqView sv = kRagged ? seq_view(a.lens, a.cu, a.kpacked != 0, b, a.N, a.total) : SeqView{a.N, 0, b, 0, b};
  const int N = sv.n;  // positions of this sequence
  const int ntiles = (N + TILE - 1) / TILE;
  if (qt >= ntiles) return;  // past the sequence: pass 2 never reads these rows
  const int r0 = qt * TILE;
  const int nkt = (a.causal && a.skip) ? min(ntiles, qt + 1) : ntiles;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], kKeyBias ? 2 : 1);  // kKeyBias: + the producer warp's bias rows
      mbar_init(&k_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kExpThreads);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (kKeyBias) {
    // The bias operands' constant parts (16-byte chunks): the query-side tile
    // of ones ([1, 0, ...] in the first K half of every row, zeros in the
    // second), and the zero second K half of every slot's key-side tile.
    if (threadIdx.x >= 64) {
      constexpr int kOnesChunks = kBiasBytes / 16, kZeroChunks = kBiasBytes / 32;  // per tile, per slot
      for (int c = threadIdx.x - 64; c < kOnesChunks + kStages * kZeroChunks; c += kExpThreads) {
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        uint8_t* dst;
        if (c < kOnesChunks) {
          dst = ones + 16 * c;
          if (((16 * c) & 128) == 0) val = make_uint4(0x00003F80u, 0u, 0u, 0u);  // bf16 1, 0, ...
        } else {
          const int e = c - kOnesChunks, sl = e / kZeroChunks, r = e % kZeroChunks;  // slot, 16-byte row of its K half 2
          dst = k_ring + sl * KS + SB + (r >> 3) * 256 + 128 + (r & 7) * 16;
        }
        *reinterpret_cast<uint4*>(dst) = val;
      }
      fence_proxy_async_smem();
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // One pass: this CTA's slot of segment sums.  At most two pass-1 CTAs are
  // resident on an SM (each holds 256 of the 512 TMEM columns), and two
  // disjoint 256-column allocations are exactly the two halves, so
  // (SM, TMEM half) names one resident CTA.  A CTA reuses a slot only after
  // the previous holder freed its TMEM, i.e. after its last read of the slot.
  static_assert(2 * kTmemCols == 512, "two pass-1 CTAs per SM take the two TMEM halves");
  static_assert(2 * kTmemCols == 512, "two pass-1 CTAs per SM take the two TMEM halves");
  int slot = 0;
  if (a.one_pass) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    slot = 2 * (int)smid + ((tmem & 0xFFFFu) >= 256u ? 1 : 0);
    if (slot >= a.slot_count) {  // an SM id past the device's SM count: no slot (recorded, no work)
      if (threadIdx.x == 0) atomicOr(&g_kvbm_device_error, 1u);
      goto done;
    }
  }

  if (kKeyBias && warp == 0) {
    // Producer warp: lane 0 issues the copies; every lane then writes the
    // key-bias rows of 4 keys of the slot's tile.
    const uint8_t* km = a.kmask + b * a.kmb;
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      mbar_arrive_expect_tx(q_full, TB);
      // the Q tile is read once: first out of L2, so that k and the slots stay
      if (KVBM_L2_HINTS)
        load_operand_hint<D, kOp>(q_tile, &tq, &tq2, q_full, sv.q_row + r0, h, sv.q_b, l2_policy_evict_first());
      else
        load_operand<D, kOp>(q_tile, &tq, &tq2, q_full, sv.q_row + r0, h, sv.q_b);
    }
    int issued = 0;
    for (int j = 0; j < nkt; ++j) {
      const int s = j % kStages, n = j / kStages;
      // this lane's keys, read before the slot wait so that the loads overlap it
      bool keep[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = j * TILE + lane * 4 + e;
        keep[e] = c < N && km[c] != 0;
      }
      const bool ok = n == 0 || mbar_wait(&k_empty[s], (n - 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&k_full[s], SB);
        load_slot<D, kOp>(k_ring + s * KS, &tk, &tk2, &k_full[s], 0, sv.k_row + j * TILE, g, sv.k_b);
      }
      issued = j + 1;
      uint8_t* bt = k_ring + s * KS + SB;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = lane * 4 + e;
        const uint4 w = make_uint4(keep[e] ? 0u : 0x0000FF80u, 0u, 0u, 0u);  // bf16 0 or -inf, then zeros
        *reinterpret_cast<uint4*>(bt + (rl >> 3) * 256 + (rl & 7) * 16) = w;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&k_full[s]);
    }
    // Do not leave while our copies are in flight.
    if (lane == 0) {
      mbar_wait(q_full, 0, abort_flag);
      for (int qn = max(0, issued - kStages); qn < issued; ++qn)
        mbar_wait(&k_full[qn % kStages], (qn / kStages) & 1, abort_flag);
    }
  } else if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      mbar_arrive_expect_tx(q_full, TB);
      // the Q tile is read once: first out of L2, so that k and the slots stay
      if (KVBM_L2_HINTS)
        load_operand_hint<D, kOp>(q_tile, &tq, &tq2, q_full, sv.q_row + r0, h, sv.q_b, l2_policy_evict_first());
      else
        load_operand<D, kOp>(q_tile, &tq, &tq2, q_full, sv.q_row + r0, h, sv.q_b);
      int issued = 0;  // ring slots (kSlotsPerTile per key tile)
      for (int j = 0; j < nkt; ++j) {
        bool ok = true;
        for (int sb = 0; sb < CF::kSlotsPerTile; ++sb) {
          const int qn = j * CF::kSlotsPerTile + sb;
          const int s = qn % kStages, n = qn / kStages;
          if (n > 0 && !mbar_wait(&k_empty[s], (n - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[s], SB);
          load_slot<D, kOp>(k_ring + s * KS, &tk, &tk2, &k_full[s], sb, sv.k_row + j * TILE, g, sv.k_b);
          issued = qn + 1;
        }
        if (!ok) break;
      }
      // Do not leave while our copies are in flight.
      mbar_wait(q_full, 0, abort_flag);
      for (int qn = max(0, issued - kStages); qn < issued; ++qn)
        mbar_wait(&k_full[qn % kStages], (qn / kStages) & 1, abort_flag);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_mma(TILE, TILE, Cfg<D, kOp>::kFmt);
      const uint32_t qs = smem_u32(q_tile), ks = smem_u32(k_ring), os = smem_u32(ones);
      const uint32_t idesc_b = idesc_mma(TILE, TILE, 1u);  // the key bias step: bf16 operands
      int issued = 0;
      if (mbar_wait(q_full, 0, abort_flag)) {
        for (int j = 0; j < nkt; ++j) {
          const int buf = j & 1;
          if (j >= 2 && !mbar_wait(&s_empty[buf], ((j >> 1) - 1) & 1, abort_flag)) break;
          int done = 0;  // slots of this tile whose MMAs were issued
          for (; done < CF::kSlotsPerTile; ++done) {
            const int qn = j * CF::kSlotsPerTile + done, s = qn % kStages;
            if (!mbar_wait(&k_full[s], (qn / kStages) & 1, abort_flag)) break;
            tc_fence_after();
            issue_slot_mma<D, kOp>(tmem + buf * TILE, qs, ks + s * KS, done * CF::kSlotBlocks, idesc);
            if constexpr (kKeyBias)  // D += ones x (0 or -inf per key)
              mma_f16(tmem + buf * TILE, k16_interleaved_desc(os), k16_interleaved_desc(ks + s * KS + SB), idesc_b,
                      1u);
            mma_commit(&k_empty[s]);
          }
          if (done > 0) {  // (a partial tile only after an abort: committed so that the drain waits for it)
            mma_commit(&s_full[buf]);
            issued = j + 1;
          }
          if (done < CF::kSlotsPerTile) break;
        }
      }
      if (issued > 0) mbar_wait(&s_full[(issued - 1) & 1], ((issued - 1) >> 1) & 1, abort_flag);
    }
  } else {
    // exp/sum warps: thread owns query row r0 + rl, columns [wg*COLS, (wg + 1)*COLS) of each tile.
    const int sub = warp & 3;
    const int wg = (warp - 2) >> 2;
    const int rl = sub * 32 + lane;
    const int row = r0 + rl;
    const uint32_t trow = tmem + ((uint32_t)(sub * 32) << 16) + wg * COLS;
    const uint8_t* kmask = kMask == kMaskKeys ? a.kmask + b * a.kmb : nullptr;
    // With the key bias, the mask is also applied as a select unless the
    // pre-pass found every masked key's k row finite (a NaN or an infinity
    // there scores NaN despite the -inf bias; the reference's masked_fill
    // drops any value).
    const bool key_select = kMask == kMaskKeys && (!kKeyBias || *a.keys_finite != kKeysFiniteMark);
    const uint32_t* prow = kMask == kMaskPairs ? a.prow + b * a.pb + (long long)row * a.W : nullptr;
    float m = -INFINITY, l = 0.f;
    // one pass: the current segment's sum (relative to m), its index and the
    // tile that starts the next segment
    float* seg = a.one_pass ? a.slots + (size_t)slot * a.slot_cols * TILE + rl : nullptr;
    const uint64_t keep_pol = l2_policy_evict_last();  // segment sums: kept in L2 for the epilogue
    float bacc = 0.f;
    // With the caller's LSE (imported as -lse2, -inf for rows that keep no
    // key and rows past the sequence) each score's share is 2^(s*C - lse2)
    // at once: the segment sums are the masses themselves, with no running
    // max, no rescale and no lg2.
    const float nlk = a.lse_known ? a.lse[(long long)hidx * a.Npad + lse_tile_slot(row)] : 0.f;
    int cur = wg, seg_end = a.seg_tiles;
    for (int j = 0; j < nkt; ++j) {
      const int buf = j & 1;
      uint32_t kw[COLS / 32];
#pragma unroll
      for (int w = 0; w < COLS / 32; ++w) kw[w] = 0xffffffffu;
      if (kMask == kMaskPairs) {  // issued before the wait so the load overlaps it
#pragma unroll
        for (int w = 0; w < COLS / 32; ++w) kw[w] = prow[((j * TILE + wg * COLS) >> 5) + w];
      }
      bool kkeep[COLS / 32];  // key mask bytes of this lane's columns, also loaded before the wait
      if (key_select) {
#pragma unroll
        for (int w = 0; w < COLS / 32; ++w) {
          const int col = j * TILE + wg * COLS + w * 32 + lane;
          kkeep[w] = col < N && kmask[col] != 0;
        }
      }
      const bool ok = mbar_wait(&s_full[buf], (j >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      float v[COLS];
      load_cols(trow + buf * TILE, v);
      tc_fence_before();
      mbar_arrive(&s_empty[buf]);

      const int c0 = j * TILE + wg * COLS;  // first key of this thread's columns
      if (key_select) {
#pragma unroll
        for (int w = 0; w < COLS / 32; ++w) kw[w] = __ballot_sync(0xffffffffu, kkeep[w]);
      }
      // (with the key bias alone, masked keys already hold -inf; the keys
      // past N are still selected away, since their rows may hold any value)
      const bool need_mask = (kMask != kMaskNone && (kMask != kMaskKeys || key_select)) || (c0 + COLS > N) ||
                             (a.causal && c0 + COLS - 1 > r0);
      if (need_mask) {
        const int lim_causal = a.causal ? row - c0 : COLS - 1;  // keep col_local <= row - c0
        const int lim = min(lim_causal, N - 1 - c0);            // and col < N
#pragma unroll
        for (int c = 0; c < COLS; ++c) {
          const bool keep = (c <= lim) && ((kw[c >> 5] >> (c & 31)) & 1u);
          v[c] = keep ? v[c] : -INFINITY;
        }
      }
      if (seg != nullptr && j == seg_end) {  // a new segment: store the finished one
        const float sv_ = a.lse_known ? bacc : m + lg2(bacc);
        if (KVBM_L2_HINTS)
          st_cg_hint(seg + (size_t)cur * TILE, sv_, keep_pol);
        else
          __stcg(seg + (size_t)cur * TILE, sv_);
        cur += kExpWG;
        seg_end += a.seg_tiles;
        bacc = 0.f;
      }
      if (a.lse_known) {
        bacc += row_sum_exp2<exp2_degree<kOp>()>(v, a.C, nlk);
        continue;
      }
      const float tmax = row_max(v);
      if (tmax != -INFINITY) {
        const float mt = tmax * a.C;
        // Rescale only when the running max grows: a fully masked tile leaves
        // (m, l) bit-identical, which keeps causal_skip on/off identical.
        if (mt > m) {
          const float al = ex2(m - mt);
          l = l * al;
          bacc = bacc * al;
          m = mt;
        }
        // (pass 1 of the two-pass method keeps the degree of pass 2)
        const float t = a.one_pass ? row_sum_exp2<exp2_degree_one_pass<kOp>()>(v, a.C, -m)
                                   : row_sum_exp2<exp2_degree<kOp>()>(v, a.C, -m);
        l += t;
        bacc += t;
      }
    }
    // log2 of the segment's sum of 2^(s*C): -inf when it kept no key (with
    // the caller's LSE: the segment's mass itself)
    if (seg != nullptr) {
      const float sv_ = a.lse_known ? bacc : m + lg2(bacc);
      if (KVBM_L2_HINTS)
        st_cg_hint(seg + (size_t)cur * TILE, sv_, keep_pol);
      else
        __stcg(seg + (size_t)cur * TILE, sv_);
    }
    if (a.lse_known) {
      if (wg == 0) lse_s[rl] = nlk;
    } else {
    // Merge the column parts of each row (fixed order: part 0, then 1, 2, ...).
    if (wg > 0) merge[(wg - 1) * TILE + rl] = make_float2(m, l);
    exp_bar_sync();
    if (wg == 0) {
#pragma unroll
      for (int w = 1; w < kExpWG; ++w) {
        const float2 o = merge[(w - 1) * TILE + rl];
        merge_ml(m, l, o.x, o.y);
      }
      bool dead = (m == -INFINITY) || row >= N;
      if (!dead && a.qmask != nullptr) dead = a.qmask[b * a.qmb + row] == 0;
      // Stored negated (pass 2 adds it): rows that keep no key, and padding
      // rows, get -inf, so 2^(t - lse2) = 0 for them.
      const float nl = dead ? -INFINITY : -(m + log2f(l));
      a.lse[(long long)(hidx) * a.Npad + lse_tile_slot(row)] = nl;
      lse_s[rl] = nl;
    }
    }
    if (a.one_pass) {
      // Bucket partials of this query tile: part1[j] = sum over the 128 rows r
      // and the segments sg of bucket j of 2^(seg[sg][r] - lse2[r]).  Warp w
      // takes buckets w, w + 8, ...; lane l rows 4l .. 4l + 3 (one float4 of
      // each segment), then a fixed xor tree over the lanes.  The buckets are
      // those the reduce reads: under causal, every bucket whose first key is
      // at most the tile's last row; a segment this CTA did not visit (past
      // its causal bound) adds nothing, as a visited one past the diagonal
      // adds exact zeros.
      __threadfence_block();
      exp_bar_sync();
      const int ew = (warp - 2);
      const float4 nl4 = reinterpret_cast<const float4*>(lse_s)[lane];
      // rows that keep no key, and rows past the sequence (whose scores may
      // come from padding of any value, NaN included), add exact zeros
      const bool d0 = nl4.x == -INFINITY, d1 = nl4.y == -INFINITY, d2 = nl4.z == -INFINITY,
                 d3 = nl4.w == -INFINITY;
      const int nseg = ((nkt - 1) / a.seg_tiles + 1) * kExpWG;
      const int nbw = a.causal ? min(a.nb, (r0 + TILE - 1) / a.bs + 1) : a.nb;
      const float4* sbase = reinterpret_cast<const float4*>(a.slots + (size_t)slot * a.slot_cols * TILE) + lane;
      float* dst = a.part1 + ((long long)hidx * (a.Npad / TILE) + qt) * a.nb;
      // kEpiU buckets per warp at a time, their loads issued together (one
      // L2 round trip per group instead of per bucket); a segment past the
      // CTA's last adds +0, as if it had not been read
      constexpr int kEpiU = 8, kEw = kExpThreads / 32;
      const uint64_t drop_pol = l2_policy_evict_first();  // read once: first out of L2
      for (int base = ew; base < nbw; base += kEw * kEpiU) {
        float acc[kEpiU];
#pragma unroll
        for (int u = 0; u < kEpiU; ++u) acc[u] = 0.f;
        for (int so = 0; so < a.seg_per_bucket; ++so) {
          float4 L[kEpiU];
#pragma unroll
          for (int u = 0; u < kEpiU; ++u) {
            const int jb = base + kEw * u, sg = jb * a.seg_per_bucket + so;
            L[u] = (jb < nbw && sg < nseg)
                       ? (KVBM_L2_HINTS ? ld_cg_hint(sbase + (size_t)sg * (TILE / 4), drop_pol)
                                        : __ldcg(sbase + (size_t)sg * (TILE / 4)))
                       : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
          }
#pragma unroll
          for (int u = 0; u < kEpiU; ++u) {
            float4 e = L[u];  // with the caller's LSE: the masses themselves
            if (!a.lse_known)
              e = make_float4(ex2(L[u].x + nl4.x), ex2(L[u].y + nl4.y), ex2(L[u].z + nl4.z), ex2(L[u].w + nl4.w));
            const float e0 = d0 ? 0.f : e.x, e1 = d1 ? 0.f : e.y;
            const float e2 = d2 ? 0.f : e.z, e3 = d3 ? 0.f : e.w;
            acc[u] += (e0 + e1) + (e2 + e3);
          }
        }
#pragma unroll
        for (int u = 0; u < kEpiU; ++u) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
          const int jb = base + kEw * u;
          if (lane == 0 && jb < nbw) dst[jb] = acc[u];
        }
      }
    }
  }

done:
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================ pass 2: mass
// One CTA owns 128 keys of one (batch, kv-head) unit and one chunk of query
// rows, for every head of the GQA group.  The 1-D grid enumerates only the
// (unit, chunk, key tile) triples that keep a pair: per unit, chunks run from
// the last (most key tiles under causal_skip) to the first, and all key tiles
// of a chunk are adjacent, so the CTAs resident at one time share that
// chunk's query tiles in L2.
template <int D, Op kOp, int kMask, bool kRagged>
__global__ void __launch_bounds__(kThreads, 2)
    tc_mass_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tq2,
                   const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tk2, TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  using CF = Cfg<D, kOp>;
  constexpr bool kBias = KVBM_P2_BIAS != 0 && kOp != Op::TF32X3;
  static_assert(!kBias || CF::kSlotsPerTile == 1, "the bias step follows a whole Q tile per slot");
  constexpr int TB = CF::kOperandBytes, SB = CF::kSlotBytes;
  constexpr int QS = SB + (kBias ? kBiasBytes : 0);  // Q ring slot: the Q operand, then its bias operand
  static_assert(QS % 1024 == 0, "Q slots stay on 1024-byte swizzle atoms");
  constexpr int LB = TILE * 4;  // lse2 bytes of one query tile
  constexpr int LR = kBias ? 0 : LB * kLStages;
  uint8_t* k_tile = smem;
  uint8_t* q_ring = smem + TB;
  uint8_t* ones = q_ring + QS * kStages;  // kBias: the key-side operand of the bias step
  float* l_ring = reinterpret_cast<float*>(ones + (kBias ? kBiasBytes : 0));
  float* merge = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(l_ring) + LR);  // [kExpWG - 1][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(merge + (kExpWG - 1) * TILE);
  uint64_t* k_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = q_full + kStages;
  uint64_t* s_full = q_empty + kStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* l_full = s_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(l_full + kLStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int uu, y, kt;
  if constexpr (kRagged) {  // the plan's work list: only (chunk, key tile) pairs inside the sequence
    if ((long long)blockIdx.x >= a.work_count[1]) return;
    const unsigned long long it = a.work2[blockIdx.x];
    uu = item_hi(it);
    y = item_mid(it);
    kt = item_lo(it);
  } else {
    const int ul = (int)blockIdx.x / a.per_unit;
    uu = a.rb + ul;
    y = a.nchunk - 1;
    kt = (int)blockIdx.x - ul * a.per_unit;
    while (kt >= keys_in_chunk(a, y)) {
      kt -= keys_in_chunk(a, y);
      --y;
    }
  }
  const int u = a.ub + uu;
  const int b = u / a.Hkv, g = u % a.Hkv;
  const SeqView sv = kRagged ? seq_view(a.lens, a.cu, a.kpacked != 0, b, a.N, a.total) : SeqView{a.N, 0, b, 0, b};
  const int N = sv.n;  // positions of this sequence
  const int c0 = kt * TILE;
  const int qa = y * a.qchunk;
  // (the plan lists no chunk or key tile past the sequence; the partials they
  // would own were zeroed before the pass)
  if (kRagged && (c0 >= N || qa >= N)) return;
  const int qb = min(N, qa + a.qchunk);
  int rs = qa;
  if (a.causal && a.skip) {
    if (qb - 1 < c0) return;  // chunk entirely above the diagonal: nothing kept
    rs = max(qa, c0);
  }
  const int nqt = (qb - rs + TILE - 1) / TILE;
  const int J = a.G * nqt;

  if (threadIdx.x == 0) {
    mbar_init(k_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&q_full[s], kBias ? 2 : 1);  // kBias: + the producer warp's bias rows
      mbar_init(&q_empty[s], 1);  // MMA commit: the Q tile is no longer read
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kExpThreads);
    }
    for (int t = 0; t < kLStages; ++t) {
      mbar_init(&l_full[t], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (kBias) {
    // The bias operands' constant parts (16-byte chunks): the key-side tile
    // of ones ([1, 1, 1, 0, ...] in the first K half of every row, zeros in
    // the second), and the zero second K half of every slot's query-side tile.
    if (threadIdx.x >= 64) {
      constexpr int kOnesChunks = kBiasBytes / 16, kZeroChunks = kBiasBytes / 32;  // per tile, per slot
      for (int c = threadIdx.x - 64; c < kOnesChunks + kStages * kZeroChunks; c += kExpThreads) {
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        uint8_t* dst;
        if (c < kOnesChunks) {
          dst = ones + 16 * c;
          if (((16 * c) & 128) == 0) val = make_uint4(0x3F803F80u, 0x00003F80u, 0u, 0u);  // bf16 1, 1, 1, 0
        } else {
          const int e = c - kOnesChunks, sl = e / kZeroChunks, r = e % kZeroChunks;  // slot, 16-byte row of its K half 2
          dst = q_ring + sl * QS + SB + (r >> 3) * 256 + 128 + (r & 7) * 16;
        }
        *reinterpret_cast<uint4*>(dst) = val;
      }
      fence_proxy_async_smem();
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (kBias && warp == 0) {
    // Producer warp: lane 0 issues the copies; every lane then writes the
    // bias rows of 4 query rows of the slot's tile.
    const float invC = 1.0f / a.C;
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      mbar_arrive_expect_tx(k_full, TB);
      load_operand<D, kOp>(k_tile, &tk, &tk2, k_full, sv.k_row + c0, g, sv.k_b);
    }
    int issued = 0;
    for (int j = 0; j < J; ++j) {
      const int hh = j / nqt;
      const int r = rs + (j - hh * nqt) * TILE;
      const int h = g * a.G + hh;
      const int s = j % kStages, n = j / kStages;
      // The lse2 rows of the tile, loaded before the slot wait so that their
      // latency overlaps it (pass 1 wrote them; nothing writes them now).
      const float* lrow = a.lse + (long long)(uu * a.G + hh) * a.Npad + r;
      float nls[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) nls[e] = lrow[lse_tile_slot(lane * 4 + e)];
      const bool ok = n == 0 || mbar_wait(&q_empty[s], (n - 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&q_full[s], SB);
        load_slot<D, kOp>(q_ring + s * QS, &tq, &tq2, &q_full[s], 0, sv.q_row + r, h, sv.q_b);
      }
      issued = j + 1;
      uint8_t* bt = q_ring + s * QS + SB;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = lane * 4 + e;
        const float nl = nls[e];  // -lse2 (-inf: the row keeps no key)
        const float v = nl == -INFINITY ? -60000.f : nl * invC;
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const float r1 = v - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
        const uint4 w = make_uint4((uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(mid) << 16),
                                   (uint32_t)__bfloat16_as_ushort(lo), 0u, 0u);
        *reinterpret_cast<uint4*>(bt + (rl >> 3) * 256 + (rl & 7) * 16) = w;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_full[s]);
    }
    // Do not leave while our copies are in flight.
    if (lane == 0) {
      mbar_wait(k_full, 0, abort_flag);
      for (int qn = max(0, issued - kStages); qn < issued; ++qn)
        mbar_wait(&q_full[qn % kStages], (qn / kStages) & 1, abort_flag);
    }
  } else if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      mbar_arrive_expect_tx(k_full, TB);
      load_operand<D, kOp>(k_tile, &tk, &tk2, k_full, sv.k_row + c0, g, sv.k_b);
      int issued = 0, issued_l = 0;  // Q ring slots (kSlotsPerTile per query tile), lse2 tiles
      for (int j = 0; j < J; ++j) {
        const int t = j % kLStages;
        const int hh = j / nqt;
        const int r = rs + (j - hh * nqt) * TILE;
        const int h = g * a.G + hh;
        bool ok = true;
        for (int sb = 0; sb < CF::kSlotsPerTile; ++sb) {
          const int qn = j * CF::kSlotsPerTile + sb;
          const int s = qn % kStages, n = qn / kStages;
          if (n > 0 && !mbar_wait(&q_empty[s], (n - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&q_full[s], SB);
          load_slot<D, kOp>(q_ring + s * QS, &tq, &tq2, &q_full[s], sb, sv.q_row + r, h, sv.q_b);
          issued = qn + 1;
          if (sb == 0) {
            mbar_arrive_expect_tx(&l_full[t], LB);
            bulk_load(l_ring + t * TILE, a.lse + (long long)(uu * a.G + hh) * a.Npad + r, LB, &l_full[t]);
            issued_l = j + 1;
          }
        }
        if (!ok) break;
      }
      // Do not leave while our copies are in flight.
      mbar_wait(k_full, 0, abort_flag);
      for (int qn = max(0, issued - kStages); qn < issued; ++qn)
        mbar_wait(&q_full[qn % kStages], (qn / kStages) & 1, abort_flag);
      for (int j = max(0, issued_l - kLStages); j < issued_l; ++j)
        mbar_wait(&l_full[j % kLStages], (j / kLStages) & 1, abort_flag);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_mma(TILE, TILE, Cfg<D, kOp>::kFmt);
      const uint32_t ks = smem_u32(k_tile), qs = smem_u32(q_ring), os = smem_u32(ones);
      const uint32_t idesc_b = idesc_mma(TILE, TILE, 1u);  // the bias step: bf16 operands
      int issued = 0;
      if (mbar_wait(k_full, 0, abort_flag)) {
        for (int j = 0; j < J; ++j) {
          const int buf = j & 1;
          if (j >= 2 && !mbar_wait(&s_empty[buf], ((j >> 1) - 1) & 1, abort_flag)) break;
          int done = 0;  // slots of this tile whose MMAs were issued
          for (; done < CF::kSlotsPerTile; ++done) {
            const int qn = j * CF::kSlotsPerTile + done, s = qn % kStages;
            if (!mbar_wait(&q_full[s], (qn / kStages) & 1, abort_flag)) break;
            tc_fence_after();
            issue_slot_mma<D, kOp>(tmem + buf * TILE, ks, qs + s * QS, done * CF::kSlotBlocks, idesc);
            if constexpr (kBias)  // D += ones x (hi + mid + lo of -lse2 / C)
              mma_f16(tmem + buf * TILE, k16_interleaved_desc(os), k16_interleaved_desc(qs + s * QS + SB), idesc_b,
                      1u);
            mma_commit(&q_empty[s]);  // the Q slot is free once these MMAs complete
          }
          if (done > 0) {  // (a partial tile only after an abort: committed so that the drain waits for it)
            mma_commit(&s_full[buf]);
            issued = j + 1;
          }
          if (done < CF::kSlotsPerTile) break;
        }
      }
      if (issued > 0) mbar_wait(&s_full[(issued - 1) & 1], ((issued - 1) >> 1) & 1, abort_flag);
    }
  } else {
    // exp/sum warps: warp w covers keys c0 + 32*(w%4) + [0, 32) and warpgroup wg
    // the query columns [wg*COLS, (wg + 1)*COLS) of each tile; lane l holds keys
    // kr[i] = 32*(w%4) + l/4 + 8i (i < 4) and 2*kBlk of the columns (col_sum4).
    const int sub = warp & 3;
    const int wg = (warp - 2) >> 2;
    const int pc = lane & 3;
    const int kr0 = sub * 32 + (lane >> 2);  // local key of row i: kr0 + 8i
    const uint32_t trow = tmem + ((uint32_t)(sub * 32) << 16) + wg * COLS;
    const float C = a.C;
    // kRagged: the sequence length is re-read from shared memory per tile
    // rather than held in a register across the loop (register budget).
    __shared__ int s_len;
    if (kRagged && threadIdx.x == 64) s_len = N;
    if (kRagged) exp_bar_sync();
    const volatile int* len_v = &s_len;
    float2 acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);
    for (int j = 0; j < J; ++j) {
      const int buf = j & 1, t = j % kLStages;
      const int hh = j / nqt;
      const int r = rs + (j - hh * nqt) * TILE;
      uint2 pw[4];
      if (kMask == kMaskPairs) {  // issued before the waits so the loads overlap them
        const uint32_t* pcol = a.pcol + b * a.pb + ((r + wg * COLS) >> 5);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t* w = pcol + (long long)(c0 + kr0 + 8 * i) * a.W;
          pw[i] = COLS == 64 ? *reinterpret_cast<const uint2*>(w) : make_uint2(w[0], 0xffffffffu);
        }
      }
      bool ok = mbar_wait(&s_full[buf], (j >> 1) & 1, abort_flag);
      if (!kBias) ok = ok && mbar_wait(&l_full[t], (j / kLStages) & 1, abort_flag);  // lse2 bytes landed
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      float v[COLS];
      load_keys16(trow + buf * TILE, v);
      tc_fence_before();
      mbar_arrive(&s_empty[buf]);

      const float* nL = l_ring + t * TILE + wg * COLS;  // -lse2 of this warpgroup's query rows (lse_tile_slot order)
      constexpr bool kB = kMask == kMaskPairs;
      constexpr int kDeg = exp2_degree<kOp>();
      // On the diagonal, query r + wg*COLS + col keeps key c0 + kr iff wg*COLS + col >= kr.
      // r < c0 (only without causal_skip): every pair is above the diagonal, adds 0.
      // kRagged: query columns at or past the sequence's end contribute 0
      // whatever their scores (their rows may hold another sequence's, or
      // undefined, values).  Otherwise those rows are the TMA's zero fill
      // past N, whose lse2 is -inf.
      if (!a.causal || r >= c0) {
        const int keep_from = kr0 - wg * COLS;  // key i keeps columns >= keep_from + 8i
        const int keep_to = kRagged ? *len_v - r - wg * COLS : COLS;
        const bool diag = a.causal && r == c0;
        if (kRagged && keep_to < COLS) {
          if (diag)
            col_sum4<kDeg, true, kB, true, kBias>(v, C, nL, pc, keep_from, pw, keep_to, acc);
          else
            col_sum4<kDeg, false, kB, true, kBias>(v, C, nL, pc, keep_from, pw, keep_to, acc);
        } else if (diag) {
          col_sum4<kDeg, true, kB, false, kBias>(v, C, nL, pc, keep_from, pw, keep_to, acc);
        } else {
          col_sum4<kDeg, false, kB, false, kBias>(v, C, nL, pc, keep_from, pw, keep_to, acc);  // every pair kept
        }
      }
    }
    // Per key: the thread's columns, then the 4 lanes holding the key's other
    // columns (xor 1, 2), then the warpgroups' column parts (part 0 first).
    float tot[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      tot[i] = acc[i].x + acc[i].y;
      tot[i] += __shfl_xor_sync(0xffffffffu, tot[i], 1);
      tot[i] += __shfl_xor_sync(0xffffffffu, tot[i], 2);
    }
    if (wg > 0 && pc == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) merge[(wg - 1) * TILE + kr0 + 8 * i] = tot[i];
    }
    exp_bar_sync();
    if (wg == 0 && pc == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = c0 + kr0 + 8 * i;
        if (key < a.N) {
          float total = tot[i];
#pragma unroll
          for (int w = 1; w < kExpWG; ++w) total += merge[(w - 1) * TILE + kr0 + 8 * i];
          if (kRagged && key >= *len_v) total = 0.f;  // past the sequence's end
          else if (kMask == kMaskKeys && a.kmask[b * a.kmb + key] == 0) total = 0.f;
          a.part[((long long)uu * a.nchunk + y) * a.N + key] = total;
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================ ragged plan
// One CTA turns the device-side sequence lengths into the two work lists of a
// ragged call, so that the passes launch only CTAs that have work (a grid
// sized for the longest sequence would otherwise hold mostly CTAs that return
// at once, and their dispatch cost time: ~19 % of pass 1 on a serving batch).
//   pass 1: (unit, head, query tile qt), levels of qt from the last tile down
//           (longest rows first); inside a level the units run longest first
//           (a counting sort by tile count).
//   pass 2: (unit, chunk, key tile), unit-major, chunks from the last: the
//           order of the uniform grid without its empty entries.
constexpr int kPlanThreads = 1024;

struct PlanArgs {
  const int32_t* lens;
  const int32_t* cu;
  long long total;
  int N, ub, U, Hkv, G, ntmax, tiles_per_chunk, skip;  // skip: causal && causal_skip
  unsigned long long* work1;
  unsigned long long* work2;
  long long* counts;
  int* nt;
  int* rank;
  int* hist;
  int* start;
  int* fill;
  long long* lvl_off;
  long long* unit_off;
  long long grid1;  // CTAs of the pass-1 launch (the items past it would not run)
};

// pass-2 key tiles of chunk y for a unit of nt tiles (keys_in_chunk, per unit)
__device__ __forceinline__ int plan_keys_in_chunk(const PlanArgs& p, int nt, int y) {
  if (!p.skip) return nt;
  const int lim = (y + 1) * p.tiles_per_chunk;
  return lim < nt ? lim : nt;
}

__global__ void __launch_bounds__(kPlanThreads) ragged_plan_kernel(PlanArgs p) {
  __shared__ long long sh[kPlanThreads / 32];
  const int t = threadIdx.x;
  // 1. query tiles of each unit, and how many units have each tile count
  for (int i = t; i <= p.ntmax; i += kPlanThreads) p.hist[i] = 0;
  __syncthreads();
  for (int uu = t; uu < p.U; uu += kPlanThreads) {
    const int n = seq_view(p.lens, p.cu, false, (p.ub + uu) / p.Hkv, p.N, p.total).n;
    const int nt = (n + TILE - 1) / TILE;
    p.nt[uu] = nt;
    atomicAdd(&p.hist[nt], 1);
  }
  __syncthreads();
  // 2. start[c] = units with more than c tiles (suffix sums), fill = cursors
  long long carry = 0;
  for (int base = 0; base <= p.ntmax; base += kPlanThreads) {
    const int i = base + t, c = p.ntmax - i;
    long long tot;
    const long long before =
        carry + block_exclusive_scan<long long, kPlanThreads>(i <= p.ntmax ? p.hist[c] : 0, sh, &tot);
    carry += tot;
    if (i <= p.ntmax) p.start[c] = p.fill[c] = (int)before;
  }
  __syncthreads();
  // 3. units longest first (equal counts in any order: the order of CTAs
  //    changes no result, each one's work is the same wherever it runs)
  for (int uu = t; uu < p.U; uu += kPlanThreads) p.rank[uu] = atomicAdd(&p.fill[p.nt[uu]], 1);
  // 4. pass-1 levels: level qt holds G items for each unit of more than qt tiles
  carry = 0;
  for (int base = 0; base < p.ntmax; base += kPlanThreads) {
    const int i = base + t, qt = p.ntmax - 1 - i;
    long long tot;
    const long long before = carry + block_exclusive_scan<long long, kPlanThreads>(
                                         i < p.ntmax ? (long long)p.G * p.start[qt] : 0, sh, &tot);
    carry += tot;
    if (i < p.ntmax) p.lvl_off[qt] = before;
  }
  const long long total1 = carry;
  // 5. pass-2 items of each unit: chunks that start inside the sequence
  carry = 0;
  for (int base = 0; base < p.U; base += kPlanThreads) {
    const int uu = base + t;
    long long v = 0;
    if (uu < p.U) {
      const int nt = p.nt[uu];
      const int nch = (nt + p.tiles_per_chunk - 1) / p.tiles_per_chunk;
      for (int y = 0; y < nch; ++y) v += plan_keys_in_chunk(p, nt, y);
    }
    long long tot;
    const long long before = carry + block_exclusive_scan<long long, kPlanThreads>(v, sh, &tot);
    carry += tot;
    if (uu < p.U) p.unit_off[uu] = before;
  }
  const long long total2 = carry;
  __syncthreads();
  // 6. write the lists, one warp per unit
  const int warp = t >> 5, lane = t & 31;
  for (int uu = warp; uu < p.U; uu += kPlanThreads / 32) {
    const int nt = p.nt[uu], j = p.rank[uu];
    for (int k = lane; k < nt * p.G; k += 32) {
      const int qt = k / p.G, h = k - qt * p.G;
      p.work1[p.lvl_off[qt] + (long long)j * p.G + h] = pack_item(uu, h, qt);
    }
    long long o = p.unit_off[uu];
    const int nch = (nt + p.tiles_per_chunk - 1) / p.tiles_per_chunk;
    for (int y = nch - 1; y >= 0; --y) {
      const int kc = plan_keys_in_chunk(p, nt, y);
      for (int kt = lane; kt < kc; kt += 32) p.work2[o + kt] = pack_item(uu, y, kt);
      o += kc;
    }
  }
  if (t == 0) {
    p.counts[0] = total1;
    p.counts[1] = total2;
    // more pass-1 items than the launch has CTAs: only cu_seqlens that
    // decrease somewhere give more tiles than total_tokens allows
    if (total1 > p.grid1) atomicOr(&g_kvbm_device_error, 1u);
  }
}

// ============================================================ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// 4-D map over a [B, H, N, D] operand with unit-stride D: box (128 bytes of
// D) x 128 rows x 1 x 1, 128-byte swizzle, zero fill outside [N) so ragged
// tiles read zeros.
bool make_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int esize, int B, int H, int N,
              int D, const int64_t* st) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
  // Size-1 dims get a harmless nonzero stride (TMA wants multiples of 16 bytes).
  const uint64_t row = (uint64_t)st[2] * esize;
  uint64_t hs = (uint64_t)st[1] * esize, bs = (uint64_t)st[0] * esize;
  if (H == 1) hs = row * (uint64_t)N;
  if (B == 1) bs = hs * (uint64_t)H;
  const cuuint64_t strides[3] = {row, hs, bs};
  const cuuint32_t box[4] = {(cuuint32_t)(128 / esize), (cuuint32_t)TILE, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, type, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp32 operand -> contiguous [B, H, N, D] tf32 pairs: hi = tf32(x), lo = x - hi
// (exact in fp32).  One launch converts the rows of a box of batch entries
// [b0, b0 + nb): q-heads [qh0, qh0 + nqh) (rows Nq per head) and kv-heads
// [kh0, kh0 + nkh) (rows Nk), written at their places in the full
// [B, Hq, Nq, D] / [B, Hkv, Nk, D] copies; a packed operand is one batch
// entry of total_tokens rows.
struct SplitBox {
  int qb0, qnb, qh0, nqh;  // q: batch entries, heads
  int kb0, knb, kh0, nkh;  // k: batch entries, heads
};

__global__ void split_tf32_kernel(const float* q, long long q0, long long q1, long long q2, long long q3,
                                  int Hq, const float* k, long long k0, long long k1, long long k2,
                                  long long k3, int Hkv, int Nq, int Nk, int D, SplitBox box, long long q_elems,
                                  long long k_elems, float* q_hi, float* q_lo, float* k_hi, float* k_lo) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= q_elems + k_elems) return;
  const bool is_q = idx < q_elems;
  const long long e = is_q ? idx : idx - q_elems;
  const int d = (int)(e % D);
  const long long r = e / D;
  const int N = is_q ? Nq : Nk;
  const int n = (int)(r % N);
  const long long bh = r / N;
  const int nh = is_q ? box.nqh : box.nkh;
  const int h = (is_q ? box.qh0 : box.kh0) + (int)(bh % nh);
  const int b = (is_q ? box.qb0 : box.kb0) + (int)(bh / nh);
  const float x = is_q ? q[b * q0 + h * q1 + n * q2 + d * q3] : k[b * k0 + h * k1 + n * k2 + d * k3];
  const float hi = to_tf32(x);
  const long long o = (((long long)b * (is_q ? Hq : Hkv) + h) * N + n) * D + d;
  (is_q ? q_hi : k_hi)[o] = hi;
  (is_q ? q_lo : k_lo)[o] = x - hi;
}

// Pair mask (bytes, nonzero = keep) ANDed with the key and query masks ->
// bit rows for pass 1 (row = query i, bit c of word c/32 = key c) and the
// transposed bits for pass 2 (row = key c, bit i = query i), over [Npad]^2
// with zero padding.  One warp packs one 32 x 32 block: 32 ballots give the
// row words; the column words are their bit transpose, built in registers.
__global__ void pack_pair_mask_kernel(const uint8_t* pm, long long pbs, long long prs, const uint8_t* km,
                                      long long kbs, const uint8_t* qm, long long qbs, int N, int Npad,
                                      long long nblk, uint32_t* prow, uint32_t* pcol) {
  const long long wid = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= nblk) return;  // whole warps exit together
  const int nb = Npad / 32;
  const long long per_b = (long long)nb * nb;
  const int bm = (int)(wid / per_b);
  const long long rem = wid - bm * per_b;
  const int ib = (int)(rem / nb), cb = (int)(rem % nb);
  const int i0 = ib * 32, c = cb * 32 + lane;
  const bool col_ok = c < N && (km == nullptr || km[bm * kbs + c] != 0);
  uint32_t myrow = 0, mycol = 0;
#pragma unroll 4
  for (int r = 0; r < 32; ++r) {
    const int i = i0 + r;
    bool v = col_ok && i < N && pm[bm * pbs + (long long)i * prs + c] != 0;
    if (qm != nullptr && i < N) v = v && qm[bm * qbs + i] != 0;
    const uint32_t R = __ballot_sync(0xffffffffu, v);
    if (lane == r) myrow = R;
    mycol |= ((R >> lane) & 1u) << r;
  }
  const long long Wl = nb;
  prow[((long long)bm * Npad + i0 + lane) * Wl + cb] = myrow;
  pcol[((long long)bm * Npad + cb * 32 + lane) * Wl + ib] = mycol;
}

// Key-mask pre-pass of the tensor-core pass 1 (bf16/fp16): clears *finite
// when a key the mask drops holds a NaN or an infinity in any head's k row.
// One thread per (batch, key, kv-head); rows the mask keeps, and keys past the
// sequence (selected away in pass 1), are not read.  16-bit elements, 16-byte
// rows chunks (path 1 guarantees 16-byte aligned rows).
__global__ void masked_keys_finite_kernel(const uint16_t* k, long long s0, long long s1, long long s2, int B,
                                          int Hkv, int N, int D, const uint8_t* km, long long kmb,
                                          const int32_t* lens, const int32_t* cu, int kpacked, long long total,
                                          uint32_t exp_mask, unsigned* finite) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= (long long)B * N * Hkv) return;
  const int g = (int)(idx % Hkv);
  const long long bc = idx / Hkv;
  const int c = (int)(bc % N), b = (int)(bc / N);
  const SeqView sv = seq_view(lens, cu, kpacked != 0, b, N, total);
  if (c >= sv.n || km[b * kmb + c] != 0) return;
  const uint4* row = reinterpret_cast<const uint4*>(k + sv.k_b * s0 + g * s1 + (long long)(sv.k_row + c) * s2);
  bool bad = false;
  for (int i = 0; i < D / 8; ++i) {
    const uint4 w = row[i];
    const uint32_t x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      bad |= ((x[e] & exp_mask) == exp_mask) || ((x[e] & (exp_mask << 16)) == (exp_mask << 16));
  }
  if (bad) *finite = 0u;
}

constexpr size_t kBarBytes = 8 * (1 + 2 * kStages + 4) + 16;  // mbarriers + TMEM slot + abort flag

template <int D, Op kOp, int kMask>
constexpr size_t smem_lse() {
  constexpr bool kKeyBias = KVBM_P1_KEY_BIAS != 0 && kMask == kMaskKeys && kOp != Op::TF32X3;
  return 1024 + (size_t)Cfg<D, kOp>::kOperandBytes +
         (size_t)(Cfg<D, kOp>::kSlotBytes + (kKeyBias ? kBiasBytes : 0)) * kStages + (kKeyBias ? kBiasBytes : 0) +
         (kExpWG - 1) * TILE * 8 + TILE * 4 + kBarBytes;
}
template <int D, Op kOp>
constexpr size_t smem_mass() {
  constexpr bool kBias = KVBM_P2_BIAS != 0 && kOp != Op::TF32X3;
  return 1024 + (size_t)Cfg<D, kOp>::kOperandBytes +
         (size_t)(Cfg<D, kOp>::kSlotBytes + (kBias ? kBiasBytes : 0)) * kStages + (kBias ? kBiasBytes : 0) +
         (kBias ? 0 : TILE * 4 * kLStages) + (kExpWG - 1) * TILE * 4 + kBarBytes + 8 * kLStages;
}

template <int D, Op kOp, int kMask, bool kRagged>
int launch_variant(const kvbm_problem* p, const WsLayout& L, void* ws, cudaStream_t s, const LaunchOpts& o) {
  CUtensorMap tq, tq2, tk, tk2;
  // The kernels work on D-element rows (whole 128-byte blocks); a head dim
  // Dr < D is mapped with its real extent, and the TMA's zero fill past it
  // makes the extra columns add exact zeros to every dot product.
  const int Dr = p->D;
  // A packed operand is one batch entry of total_tokens rows; sequence b
  // starts at row cu[b] (TMA coordinates from seq_view).
  const Ragged& rg = o.rg;
  const int Bq = rg.cu ? 1 : p->B, Nq = rg.cu ? (int)rg.total : p->N;
  const int Bk = rg.k_packed ? 1 : p->B, Nk = rg.k_packed ? (int)rg.total : p->N;
  const RunRange rr = run_range(p, o);
  if constexpr (kOp == Op::TF32X3) {
    // split q/k into tf32 hi/lo pairs in the workspace, then map those
    float* base = reinterpret_cast<float*>(static_cast<char*>(ws) + L.split_off);
    const long long qe = (long long)Bq * p->Hq * Nq * Dr, ke = (long long)Bk * p->Hkv * Nk * Dr;
    float *q_hi = base, *q_lo = base + qe, *k_hi = base + 2 * qe, *k_lo = base + 2 * qe + ke;
    if (o.run_split) {
      SplitBox bx;
      if (rg.cu != nullptr || rg.lens != nullptr) {
        // ragged calls (never staged) convert every row of q and k
        bx = SplitBox{0, Bq, 0, p->Hq, 0, Bk, 0, p->Hkv};
      } else {
        // the rows passes 1 and 2 of the run units read: their batch entries x
        // their kv-heads (whole batch entries when the run crosses one), the
        // run's q-heads, and k unless the head range starts past 0
        const int G = p->Hq / p->Hkv;
        const int u0 = p->unit_begin + rr.rb, u1 = u0 + rr.nu - 1;
        const int b0 = u0 / p->Hkv, nb = u1 / p->Hkv - b0 + 1;
        const int g0 = nb == 1 ? u0 % p->Hkv : 0, ng = nb == 1 ? u1 % p->Hkv - g0 + 1 : p->Hkv;
        const bool one = nb == 1 && ng == 1;
        bx = SplitBox{b0, nb, g0 * G + (one ? rr.hb : 0), one ? rr.nh : ng * G, b0, nb, g0, rr.hb == 0 ? ng : 0};
      }
      const long long qn = (long long)bx.qnb * bx.nqh * Nq * Dr, kn = (long long)bx.knb * bx.nkh * Nk * Dr;
      const long long total = qn + kn;
      split_tf32_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
          static_cast<const float*>(p->q), p->q_stride[0], p->q_stride[1], p->q_stride[2], p->q_stride[3], p->Hq,
          static_cast<const float*>(p->k), p->k_stride[0], p->k_stride[1], p->k_stride[2], p->k_stride[3],
          p->Hkv, Nq, Nk, Dr, bx, qn, kn, q_hi, q_lo, k_hi, k_lo);
      if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
    }
    const int64_t qs[4] = {(int64_t)p->Hq * Nq * Dr, (int64_t)Nq * Dr, Dr, 1};
    const int64_t ks[4] = {(int64_t)p->Hkv * Nk * Dr, (int64_t)Nk * Dr, Dr, 1};
    const CUtensorMapDataType t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    if (!make_map(&tq, q_hi, t, 4, Bq, p->Hq, Nq, Dr, qs) || !make_map(&tq2, q_lo, t, 4, Bq, p->Hq, Nq, Dr, qs) ||
        !make_map(&tk, k_hi, t, 4, Bk, p->Hkv, Nk, Dr, ks) || !make_map(&tk2, k_lo, t, 4, Bk, p->Hkv, Nk, Dr, ks))
      return KVBM_ERR_CUDA;
  } else {
    const CUtensorMapDataType t =
        kOp == Op::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (!make_map(&tq, p->q, t, 2, Bq, p->Hq, Nq, Dr, p->q_stride) ||
        !make_map(&tk, p->k, t, 2, Bk, p->Hkv, Nk, Dr, p->k_stride))
      return KVBM_ERR_CUDA;
    tq2 = tq;
    tk2 = tk;
  }
  TcArgs a;
  a.N = p->N;
  a.Npad = (p->N + TILE - 1) / TILE * TILE;
  a.G = p->Hq / p->Hkv;
  a.Hkv = p->Hkv;
  a.ub = p->unit_begin;
  a.C = (float)(p->scale * kLog2e);
  a.causal = p->causal != 0;
  a.skip = p->causal_skip != 0;
  a.kmask = p->key_mask;
  a.kmb = p->key_mask_bstride;
  a.qmask = p->query_mask;
  a.qmb = p->query_mask_bstride;
  a.lse = reinterpret_cast<float*>(static_cast<char*>(ws) + L.lse_off);
  a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + L.part_off);
  a.qchunk = L.qchunk;
  a.nchunk = L.nchunk;
  a.per_unit = 0;
  for (int y = 0; y < a.nchunk; ++y) a.per_unit += keys_in_chunk(a, y);
  a.prow = a.pcol = nullptr;
  a.pb = 0;
  a.W = a.Npad / 32;
  a.lens = rg.lens;
  a.cu = rg.cu;
  a.kpacked = rg.k_packed ? 1 : 0;
  a.total = rg.total;
  a.work1 = a.work2 = nullptr;
  a.work_count = nullptr;
  a.one_pass = L.one_pass ? 1 : 0;
  a.lse_known = (L.one_pass && o.lse_known) ? 1 : 0;
  a.nb = (int)kvbm_num_blocks(p->N, p->block_size);
  a.bs = p->block_size;
  a.seg_tiles = L.seg_tiles;
  a.seg_per_bucket = L.seg_per_bucket;
  a.slot_cols = L.slot_cols;
  a.slot_count = L.slot_count;
  a.slots = L.one_pass ? reinterpret_cast<float*>(static_cast<char*>(ws) + L.slot_off) : nullptr;
  a.part1 = L.one_pass ? a.part : nullptr;
  unsigned* finite_word = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + L.flag_off);
  a.keys_finite = finite_word;
  constexpr bool kKeyBias = KVBM_P1_KEY_BIAS != 0 && kMask == kMaskKeys && kOp != Op::TF32X3;
  if (kKeyBias && o.run_masks) {
    if (cudaMemsetAsync(finite_word, 0x5A, sizeof(unsigned), s) != cudaSuccess) return KVBM_ERR_CUDA;
    const long long n = (long long)p->B * p->N * p->Hkv;
    if ((n + 255) / 256 > 0x7fffffffLL) return KVBM_ERR_SHAPE;
    masked_keys_finite_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        static_cast<const uint16_t*>(p->k), p->k_stride[0], p->k_stride[1], p->k_stride[2], p->B, p->Hkv, p->N,
        Dr, p->key_mask, p->key_mask_bstride, rg.lens, rg.cu, rg.k_packed ? 1 : 0, rg.total,
        kOp == Op::BF16 ? 0x7F80u : 0x7C00u, finite_word);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  }
  if (kMask == kMaskPairs) {
    uint32_t* bits = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + L.bits_off);
    const long long words = (long long)L.bits_batches * a.Npad * a.W;
    a.prow = bits;
    a.pcol = bits + words;
    a.pb = L.bits_batches > 1 ? (long long)a.Npad * a.W : 0;
    if (o.run_masks) {
      const long long nblk = (long long)L.bits_batches * (a.Npad / 32) * (a.Npad / 32);
      const bool per_b = L.bits_batches > 1;
      pack_pair_mask_kernel<<<(unsigned)((nblk * 32 + 255) / 256), 256, 0, s>>>(
          p->pair_mask, per_b ? p->pair_mask_bstride : 0, p->pair_mask_rstride, p->key_mask,
          per_b ? p->key_mask_bstride : 0, p->query_mask, per_b ? p->query_mask_bstride : 0, p->N, a.Npad, nblk,
          bits, bits + words);
      if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
    }
  }
  const int U = rr.nu;  // units this launch runs
  a.rb = rr.rb;
  a.hb = rr.hb;
  a.hn = rr.nh;
  const int ntiles = a.Npad / TILE;
  a.qt0 = rr.qb / TILE;
  a.nqts = std::min(ntiles, (rr.qe + TILE - 1) / TILE) - a.qt0;
  // Pass-1 CTAs of a unit all stream its whole k (under causal_skip, from the
  // first tile up); running the units in groups whose k fits in L2 reads each
  // k from DRAM about once.  On the Llama-3-8B N=32768 shape (8 MiB of k per
  // unit) one group of all 8 units read 597 MB per launch against 335 MB of
  // q + k.
  const long long k_unit_bytes = (long long)Nk * Dr * (kOp == Op::TF32X3 ? 8 : 2);
  a.usel = U;
  a.ugroup = (int)std::max(1LL, std::min<long long>(U, kPass1GroupBytes / std::max(1LL, k_unit_bytes)));
  const long long n1 = (long long)U * a.hn * a.nqts, n2 = (long long)U * a.per_unit;
  if (n1 > 0x7fffffffLL || n2 > 0x7fffffffLL) return KVBM_ERR_SHAPE;
  dim3 grid1((unsigned)n1), grid2((unsigned)n2);
  if constexpr (kRagged) {
    // plan the work lists on the device, and zero the partials no CTA will write
    if (L.work1_cap > 0x7fffffffLL || L.work2_cap > 0x7fffffffLL) return KVBM_ERR_SHAPE;
    const RaggedPlanLayout pl = ragged_plan_layout(U, ntiles, L.work1_cap, L.work2_cap);
    char* plan = static_cast<char*>(ws) + L.plan_off;
    PlanArgs pa;
    pa.lens = rg.lens;
    pa.cu = rg.cu;
    pa.total = rg.total;
    pa.N = p->N;
    pa.ub = p->unit_begin;
    pa.U = U;
    pa.Hkv = p->Hkv;
    pa.G = a.G;
    pa.ntmax = ntiles;
    pa.tiles_per_chunk = L.qchunk / TILE;
    pa.skip = (p->causal && p->causal_skip) ? 1 : 0;
    pa.work1 = reinterpret_cast<unsigned long long*>(plan + pl.work1);
    pa.work2 = reinterpret_cast<unsigned long long*>(plan + pl.work2);
    pa.counts = reinterpret_cast<long long*>(plan + pl.counts);
    pa.nt = reinterpret_cast<int*>(plan + pl.nt);
    pa.rank = reinterpret_cast<int*>(plan + pl.rank);
    pa.hist = reinterpret_cast<int*>(plan + pl.hist);
    pa.start = reinterpret_cast<int*>(plan + pl.start);
    pa.fill = reinterpret_cast<int*>(plan + pl.fill);
    pa.lvl_off = reinterpret_cast<long long*>(plan + pl.lvl_off);
    pa.unit_off = reinterpret_cast<long long*>(plan + pl.unit_off);
    // Pass 1 launches one CTA per item, and the CTAs past the item count
    // return at once; they still cost a launch each.  A packed batch of
    // total_tokens rows has at most ceil(T / 128) + B query tiles per
    // kv-head, far fewer than B * ceil(N / 128) when the lengths are uneven.
    pa.grid1 = L.work1_cap;
    if (rg.cu != nullptr) {
      const long long tiles = (rg.total + TILE - 1) / TILE + p->B;
      pa.grid1 = std::min(pa.grid1, (long long)a.G * p->Hkv * tiles);
    }
    ragged_plan_kernel<<<1, kPlanThreads, 0, s>>>(pa);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
    if (cudaMemsetAsync(static_cast<char*>(ws) + L.part_off, 0, L.part_bytes, s) != cudaSuccess)
      return KVBM_ERR_CUDA;
    a.work1 = pa.work1;
    a.work2 = pa.work2;
    a.work_count = pa.counts;
    grid1 = dim3((unsigned)pa.grid1);
    grid2 = dim3((unsigned)L.work2_cap);
  }

  const size_t sm1 = smem_lse<D, kOp, kMask>() > (size_t)kMinSmem ? smem_lse<D, kOp, kMask>() : (size_t)kMinSmem;
  const size_t sm2 = smem_mass<D, kOp>() > (size_t)kMinSmem ? smem_mass<D, kOp>() : (size_t)kMinSmem;
  auto k1 = tc_lse_kernel<D, kOp, kMask, kRagged>;
  auto k2 = tc_mass_kernel<D, kOp, kMask, kRagged>;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1) != cudaSuccess ||
      cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2) != cudaSuccess)
    return KVBM_ERR_CUDA;
  if (o.run_pass1) {
    k1<<<grid1, kThreads, sm1, s>>>(tq, tq2, tk, tk2, a);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  }
  if (o.mid_event != nullptr && cudaEventRecord(static_cast<cudaEvent_t>(o.mid_event), s) != cudaSuccess)
    return KVBM_ERR_CUDA;
  if (o.run_pass2 && !L.one_pass) {
    k2<<<grid2, kThreads, sm2, s>>>(tq, tq2, tk, tk2, a);
    if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  }
  return KVBM_OK;
}

template <int D, Op kOp>
int launch_km(const kvbm_problem* p, const WsLayout& L, void* ws, cudaStream_t s, const LaunchOpts& o) {
  if (o.rg.lens != nullptr || o.rg.cu != nullptr) {
    if (p->pair_mask != nullptr) return launch_variant<D, kOp, kMaskPairs, true>(p, L, ws, s, o);
    return p->key_mask != nullptr ? launch_variant<D, kOp, kMaskKeys, true>(p, L, ws, s, o)
                                  : launch_variant<D, kOp, kMaskNone, true>(p, L, ws, s, o);
  }
  if (p->pair_mask != nullptr) return launch_variant<D, kOp, kMaskPairs, false>(p, L, ws, s, o);
  return p->key_mask != nullptr ? launch_variant<D, kOp, kMaskKeys, false>(p, L, ws, s, o)
                                : launch_variant<D, kOp, kMaskNone, false>(p, L, ws, s, o);
}

}  // namespace

bool tc_path_enabled() { return encode_fn() != nullptr; }

namespace {
__device__ int g_selftest_result = -1;

// One thread waits on an mbarrier that nothing arrives at, through the same
// bounded wait as the pipeline kernels: it gives up after limit_ns, sets the
// device error word and the kernel returns (no async copy targets the
// barrier, so leaving it pending is harmless).
__global__ void selftest_wait_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) g_selftest_result = mbar_wait(&bar, 0, &abort_flag, limit_ns) ? 1 : 0;
}
}  // namespace

int selftest_wait_timeout(cudaStream_t s, unsigned long long limit_ns, int* waited) {
  selftest_wait_kernel<<<1, 32, 0, s>>>(limit_ns);
  if (cudaGetLastError() != cudaSuccess) return KVBM_ERR_CUDA;
  if (cudaMemcpyFromSymbolAsync(waited, g_selftest_result, sizeof(int), 0, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return KVBM_ERR_CUDA;
  return KVBM_OK;
}

double exp2_fma_fraction() { return (double)kEmuPer16 / 16; }

int launch_tc(const kvbm_problem* p, const WsLayout& L, void* mass_out, void* ws, cudaStream_t s,
              const LaunchOpts& o) {
  (void)mass_out;
  if (L.path == 2) {  // fp32 inputs on tf32 tensor cores (3 MMAs per step)
    if (p->D <= 32) return launch_km<32, Op::TF32X3>(p, L, ws, s, o);
    if (p->D <= 64) return launch_km<64, Op::TF32X3>(p, L, ws, s, o);
    if (p->D <= 128) return launch_km<128, Op::TF32X3>(p, L, ws, s, o);  // K-block slots (Cfg::kSlotBlocks)
    return KVBM_ERR_HEAD_DIM;
  }
  // Head dims run on the next whole number of 128-byte blocks (64 bf16/fp16
  // elements); 192 and 256 take one CTA per SM (operand tiles of 48 / 64 KB)
  // and are bound by the tensor pipe, not the exp unit.
  const bool bf16 = p->dtype == KVBM_BF16;
  if (p->D <= 64) return bf16 ? launch_km<64, Op::BF16>(p, L, ws, s, o) : launch_km<64, Op::F16>(p, L, ws, s, o);
  if (p->D <= 128) return bf16 ? launch_km<128, Op::BF16>(p, L, ws, s, o) : launch_km<128, Op::F16>(p, L, ws, s, o);
  if (p->D <= 192) return bf16 ? launch_km<192, Op::BF16>(p, L, ws, s, o) : launch_km<192, Op::F16>(p, L, ws, s, o);
  if (p->D <= 256) return bf16 ? launch_km<256, Op::BF16>(p, L, ws, s, o) : launch_km<256, Op::F16>(p, L, ws, s, o);
  return KVBM_ERR_HEAD_DIM;
}

int read_and_clear_device_error(cudaStream_t s, int* err) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, sm100::g_kvbm_device_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return KVBM_ERR_CUDA;
  *err = v != 0;
  if (v != 0) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbolAsync(sm100::g_kvbm_device_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s) !=
            cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return KVBM_ERR_CUDA;
  }
  return KVBM_OK;
}

}  // namespace kvbm
