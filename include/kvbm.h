/*
 * kvbm.h - C ABI of the B200 (sm_100a) block-granular attention-mass kernels.
 *
 *   mass[j] = sum over (b, h_q, query i, key c in block j) of
 *             softmax_c(q[b,h_q,i] . k[b,h_q/G,c] * scale),   G = H_q / H_kv
 *
 * computed in two passes (row log-sum-exp, then column sums of the softmax)
 * without materialising the [B, H, N, N] matrix.
 *
 * Every entry point takes plain pointers and sizes; no C++ or torch types
 * cross this boundary.  All device pointers must belong to the CUDA device
 * that is current on the calling thread, and `stream` is a cudaStream_t of
 * that device (NULL = legacy default stream).  Launches are asynchronous on
 * `stream`; nothing here synchronises the host.  The caller owns every
 * buffer, including the workspace.  Status codes are returned, nothing is
 * thrown across the ABI.
 *
 * Reference interfaces replaced (kv-block-mass, file:line):
 *   kvbm_block_mass      <- block_mass_triton(q, k, attn_mask, causal, block_size,
 *                           scale, BLOCK_M, BLOCK_N, causal_skip)
 *                           src/kvblockmass/triton_kernel.py:148-196, whose
 *                           kernel launch is at :183-195; and the CUDA branch of
 *                           the dispatcher block_mass, src/kvblockmass/reference.py:129-135
 *   kvbm_validate        <- the wrapper's argument checks, triton_kernel.py:159-164
 *                           (GQA ValueError, reference.py:29-30)
 *   kvbm_workspace_bytes <- the wrapper's device allocations, triton_kernel.py:166-180
 *   kvbm_num_blocks      <- num_blocks = ceil(N / block_size), reference.py:89
 */
#ifndef KVBM_H
#define KVBM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVBM_ABI_VERSION 4

/* Only the entry points below are exported from libkvbm.so (it is built with
 * hidden default visibility). */
#if defined(__GNUC__)
#define KVBM_API __attribute__((visibility("default")))
#else
#define KVBM_API
#endif

/* Element type of q and k.  The mass output is float32, or float64 for
 * KVBM_F64 inputs (reference.py:77: fp64 stays fp64, everything else
 * accumulates in fp32). */
enum kvbm_dtype {
  KVBM_F32 = 0,
  KVBM_BF16 = 1,
  KVBM_F16 = 2,
  KVBM_F64 = 3
};

enum kvbm_status {
  KVBM_OK = 0,
  KVBM_ERR_GQA = 1,         /* H_q % H_kv != 0 (reference raises ValueError) */
  KVBM_ERR_SHAPE = 2,       /* a size is out of range or inconsistent        */
  KVBM_ERR_DTYPE = 3,       /* unknown dtype                                  */
  KVBM_ERR_HEAD_DIM = 4,    /* head dim D not supported for this dtype        */
  KVBM_ERR_BLOCK_SIZE = 5,  /* block_size < 1                                  */
  KVBM_ERR_UNITS = 6,       /* unit range not inside [0, B*H_kv]              */
  KVBM_ERR_NULL = 7,        /* a required pointer is NULL                     */
  KVBM_ERR_WORKSPACE = 8,   /* workspace missing, too small or misaligned     */
  KVBM_ERR_CUDA = 9,        /* a CUDA runtime call or launch failed           */
  KVBM_ERR_DEVICE = 10,     /* current device is not an sm_100 GPU            */
  KVBM_ERR_TIMEOUT = 11,    /* a device-side wait ran out its iteration limit */
  KVBM_ERR_SCRATCH = 12,    /* problem needs more scratch than the fixed area  */
  KVBM_ERR_PAGE = 13        /* a block-table entry was outside [0, num_pages) */
};

/* Attention-mass problem.  Strides are in ELEMENTS for the dims [B, H, N, D]
 * of q ([B, H_q, N, D]) and k ([B, H_kv, N, D]); any strides are accepted.
 *
 * Masks are byte arrays, nonzero = keep, NULL = absent; they combine with
 * `causal` by logical AND (reference.py:83-87):
 *   key_mask   [B|1, N]     column mask: key_mask[b*key_mask_bstride + c]
 *                           (an [N] attn_mask of the reference is bstride 0)
 *   query_mask [B|1, N]     row mask: a row whose entry is 0 keeps no key
 *                           and contributes exactly 0 (extension)
 *   pair_mask  [B|1, N, N]  pair mask: pair_mask[b*bstride + i*rstride + c]
 *                           (an [N, N] attn_mask of the reference is bstride 0)
 *
 * Sizes: B, H_q, H_kv, D >= 1 with B*H_q <= 65535, and 1 <= N <= 2^28
 * (268,435,456 positions, a bound that keeps every tile and work-list index
 * in range); larger values return KVBM_ERR_SHAPE.
 *
 * `units`: the problem splits into B*H_kv independent (batch, kv-head) units,
 * u = b*H_kv + g, each owning q-heads [g*G, (g+1)*G).  One call computes the
 * mass of units [unit_begin, unit_end); the full problem is [0, B*H_kv).
 * Mass is a sum over units, so shards of one problem add up exactly.
 */
typedef struct kvbm_problem {
  const void* q;
  int64_t q_stride[4];
  const void* k;
  int64_t k_stride[4];
  int32_t dtype;
  int32_t B, Hq, Hkv, N, D;
  const uint8_t* key_mask;
  int64_t key_mask_bstride;
  const uint8_t* query_mask;
  int64_t query_mask_bstride;
  const uint8_t* pair_mask;
  int64_t pair_mask_bstride;
  int64_t pair_mask_rstride;
  double scale;          /* score scale; the reference's default is 1/sqrt(D) */
  int32_t block_size;    /* KV block (bucket) size; the last bucket may be ragged */
  int32_t causal;        /* keep key c for query i only if c <= i           */
  int32_t causal_skip;   /* 1: never visit tiles above the causal diagonal  */
  int32_t unit_begin;
  int32_t unit_end;
} kvbm_problem;

/* ABI version of the loaded library (KVBM_ABI_VERSION it was built with). */
KVBM_API int kvbm_abi_version(void);

/* Static description of a status code. */
KVBM_API const char* kvbm_status_string(int status);

/* Host-only argument validation; touches no GPU.  Returns KVBM_OK or the
 * first failing check. */
KVBM_API int kvbm_validate(const kvbm_problem* p);

/* ceil(N / block_size), the length of the mass vector. */
KVBM_API int64_t kvbm_num_blocks(int32_t N, int32_t block_size);

/* Bytes of device workspace kvbm_block_mass needs for `p` (0 on invalid
 * input).  Host-only; the size depends on the device's kernel path but not
 * on pointer values. */
KVBM_API size_t kvbm_workspace_bytes(const kvbm_problem* p);

/* Which kernel family will run `p` on the current device:
 * 0 = SIMT (fp32 FFMA / fp64 DFMA, any mask, D <= 256),
 * 1 = tcgen05 tensor cores with TMA and TMEM (bf16/fp16, D <= 256 with
 *     D % 8 == 0, padded to 64/128/192/256 by the TMA's zero fill; 192 and
 *     256 run one CTA per SM and are bound by the tensor pipe),
 * 2 = tcgen05 3xTF32 for fp32 inputs (D <= 128 with D % 4 == 0): tf32 hi/lo
 *     split, three MMAs per step, fp32-grade scores (D > 64: one CTA per SM,
 *     the streamed operand in 128-byte K-blocks),
 * (paths 1 and 2 take pair masks as packed bits: 2 * Npad^2 / 8 bytes of
 * workspace per mask batch entry, Npad = N rounded up to 128),
 * negative = a kvbm_status error code, negated. */
KVBM_API int kvbm_kernel_path(const kvbm_problem* p);

/* Kernel launches one kvbm_block_mass call of `p` makes (host-only). */
KVBM_API int kvbm_launches_per_call(const kvbm_problem* p);

/* Compute the mass of units [p->unit_begin, p->unit_end) into
 * `mass_out` (device, num_blocks elements of float32, or float64 for
 * KVBM_F64 inputs; overwritten, not accumulated).  `workspace` is device
 * memory of at least kvbm_workspace_bytes(p) bytes, 256-byte aligned; its
 * contents on entry do not matter.  Results are deterministic: the same
 * inputs give the same bits, and causal_skip on/off give the same bits. */
KVBM_API int kvbm_block_mass(const kvbm_problem* p, void* mass_out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* kvbm_block_mass for callers that already hold each query row's
 * log-sum-exp, as an attention forward pass returns it (for example the
 * softmax LSE of a FlashAttention forward): lse[b*s0 + h*s1 + i*s2] =
 * log(sum over kept keys c of exp(scale * q[b,h,i] . k[b,h/G,c])), natural
 * log, fp32, with the same scale and masks as `p`.  The row statistics are
 * not recomputed: the LSE is copied into the workspace, and then (one-pass
 * method, the default where it applies) pass 1 sums 2^(s - lse2) per segment
 * with no running max, rescale or lg2 (measured 7 % under the call without
 * an LSE), or (two-pass method) only pass 2 and the bucket reduce run, about
 * half the two-pass work.  A non-finite LSE marks a row that keeps no key (it
 * contributes 0).  lse_stride = {s0, s1, s2} in elements.  It extends the
 * reference's entry points (there the row statistics are always recomputed,
 * triton_kernel.py:69-104); workspace and output as kvbm_block_mass. */
KVBM_API int kvbm_block_mass_lse(const kvbm_problem* p, const float* lse, const int64_t* lse_stride, void* mass_out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* kvbm_block_mass that also records up to four CUDA events (cudaEvent_t,
 * each may be NULL) on `stream`: events[0] before pass 1, events[1] between
 * pass 1 and pass 2, events[2] between pass 2 and the bucket reduce,
 * events[3] after the reduce (with the one-pass method events[1] and [2] mark
 * the same point).  Per-kernel timing for benchmarks; it replaces
 * the CUDA-event timing of the reference's bench (bench/bench_block_mass.py:37-54)
 * at kernel rather than call granularity. */
KVBM_API int kvbm_block_mass_events(const kvbm_problem* p, void* mass_out, void* workspace,
                           size_t workspace_bytes, void* stream, void* const* events);

/* Measures the current device's MUFU ex2.approx.f32 throughput (results per
 * second, all SMs) with a calibration kernel, timed with CUDA events on
 * `stream`; synchronises `stream`.  The exp/sum warps of both passes are
 * bound by this rate, so benchmarks report it as the roofline denominator.
 * No counterpart in the reference. */
KVBM_API int kvbm_measure_ex2_rate(void* stream, double* ex2_per_second);

/* Share of the tensor-core kernels' exp2 evaluations done on the FMA pipe
 * (a minimax polynomial) instead of MUFU ex2.approx: the MUFU unit sees
 * (1 - this) of the exponentials.  No counterpart in the reference. */
KVBM_API double kvbm_exp2_fma_fraction(void);

/* kvbm_block_mass for callers that cannot allocate device memory.  It has
 * no counterpart in the reference.
 *
 * Who needs it: a serving engine that reserves all free device memory for its
 * own KV-cache pool at start-up has none left for a cudaMalloc, and cannot
 * afford cudaMalloc/cudaFree in its step loop because they synchronise the
 * device and stall its other streams.  A C/FFI host may hold only the input and
 * output pointers another framework gave it.  Such callers still pass q, k, the
 * masks and `mass_out`; the scratch the passes need (the per-row lse2 values
 * and the partial sums) comes from a fixed device array inside this library
 * instead of a caller workspace.  The call takes the two-pass method
 * (KVBM_METHOD_TWO_PASS) when the one-pass method's scratch does not fit.
 *
 * Limit: the array holds kvbm_static_scratch_bytes() bytes (64 MiB).  Every
 * GPU that loads the library holds it until the process exits.  A problem
 * whose workspace (kvbm_workspace_bytes) is larger is rejected with
 * KVBM_ERR_SCRATCH before anything is launched.  Split such a problem into
 * unit ranges (unit_begin/unit_end) that fit: a range inside one batch entry
 * needs scratch for its own units only (their lse2 rows and partials, and for
 * fp32 inputs on kernel path 2 the tf32 copies of their q/k rows), and the
 * mass vectors of the ranges add up to the whole.  A pair mask needs
 * Npad^2 / 4 bytes of packed bits per mask batch entry whatever the range
 * (Npad = N rounded up to 128), so pair-masked problems longer than about
 * N = 16000 cannot use this entry point.
 *
 * No allocation: the call makes no cudaMalloc, cudaFree or other allocating
 * call.  The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.
 *
 * Sharing: every call on a device uses the same array.  The array keeps the
 * last call's contents, and each call overwrites what it reads, so nothing has
 * to be cleared between calls.  Calls that can overlap on the GPU (different
 * streams without ordering between them) race on the array and give wrong
 * results; order them on one stream or with events. */
KVBM_API int kvbm_block_mass_static(const kvbm_problem* p, void* mass_out, void* stream);

/* Size in bytes of the fixed scratch array used by kvbm_block_mass_static.
 * No counterpart in the reference. */
KVBM_API size_t kvbm_static_scratch_bytes(void);

/* Paged key cache (extension; the reference takes dense k only).
 *
 *   k_cache      [num_pages, page_size, H_kv, D] of the problem's dtype, on
 *                the device; cache_stride = element strides of those dims
 *   block_table  [B, max_pages] int32 page ids on the device: logical key n
 *                of sequence b is slot n % page_size of page
 *                block_table[b * block_table_stride + n / page_size]
 *
 * This is the layout of the paged KV-cache managers that consume block mass
 * (the companion paged-kv block manager, README.md:7-10 and
 * src/kvblockmass/reclaim.py:14-16 of kv-block-mass).  Every sequence has
 * the problem's N keys; max_pages * page_size must be >= N.  Table entries
 * past ceil(N / page_size) are not read.  block_size == page_size gives one
 * mass bucket per page. */
typedef struct kvbm_paged_kv {
  const void* k_cache;
  int64_t cache_stride[4];
  int32_t num_pages;
  int32_t page_size;
  const int32_t* block_table;
  int64_t block_table_stride;
  int32_t max_pages;
} kvbm_paged_kv;

/* Host-only checks of a paged problem (p->k and p->k_stride are ignored). */
KVBM_API int kvbm_validate_paged(const kvbm_problem* p, const kvbm_paged_kv* kv);

/* Workspace bytes kvbm_block_mass_paged needs (0 on invalid input): the
 * kvbm_workspace_bytes of the dense problem plus a dense copy of the key
 * rows of the units [unit_begin, unit_end) touch. */
KVBM_API size_t kvbm_paged_workspace_bytes(const kvbm_problem* p, const kvbm_paged_kv* kv);

/* kvbm_block_mass (lse == NULL) or kvbm_block_mass_lse (lse != NULL) with k
 * read from a paged cache.  A first kernel copies the key rows of the
 * requested units, page by page, into a dense array in the workspace; the
 * dense kernels then run on it, so the result has the same bits as the dense
 * call on the same key values.  A block-table entry outside [0, num_pages)
 * is not read: its rows count as zero vectors and kvbm_check_device_errors
 * reports KVBM_ERR_PAGE.  Workspace: kvbm_paged_workspace_bytes(p, kv). */
KVBM_API int kvbm_block_mass_paged(const kvbm_problem* p, const kvbm_paged_kv* kv, const float* lse,
                          const int64_t* lse_stride, void* mass_out, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Options of kvbm_block_mass_ex (extensions; the reference has one dense
 * [B, H, N, D] layout, one length N and a mass summed over the batch).
 * Zero-initialise and set what is used; every pointer may be NULL.
 *
 *   lse, lse_stride   row LSE input as kvbm_block_mass_lse (skips pass 1);
 *                     with cu_seqlens the LSE is packed like q: row i of
 *                     sequence b, head h is lse[h*s1 + (cu_seqlens[b] + i)*s2]
 *                     (s0 unused; [H_q, total_tokens] as FlashAttention's
 *                     varlen forward returns it)
 *   paged             k from a paged cache as kvbm_block_mass_paged
 *   seq_lens          [B] int32 on the device: sequence b has seq_lens[b] <= N
 *                     keys and queries (padded layout: q/k as in kvbm_problem,
 *                     positions >= seq_lens[b] are never part of any pair)
 *   cu_seqlens        [B + 1] int32 on the device: packed (varlen) layout.
 *                     Sequence b is rows [cu_seqlens[b], cu_seqlens[b+1]) of
 *                     q [total_tokens, H_q, D] (and of k [total_tokens, H_kv, D]
 *                     unless `paged`); its length must be <= N (p->N is the
 *                     longest sequence, longer ones are cut at N).  q_stride /
 *                     k_stride give {unused, head, row, d} in elements.
 *                     Offsets outside [0, total_tokens] are clamped into it
 *                     on the device: no row past the packed tensors is read.
 *                     seq_lens and cu_seqlens are exclusive.
 *   total_tokens      rows of the packed q/k (required with cu_seqlens)
 *   per_sequence      0: mass_out is [num_blocks], summed over the batch (the
 *                     reference's output); 1: mass_out is [B, num_blocks],
 *                     row b the mass of sequence b alone (rows of sequences
 *                     outside the unit range are written as zeros)
 *   events            4 cudaEvent_t as kvbm_block_mass_events (or NULL)
 *   method            KVBM_METHOD_* (0: automatic), how the mass is formed:
 *                     TWO_PASS: pass 1 writes each row's lse2, pass 2
 *                     recomputes the scores and sums 2^(s - lse2) per key
 *                     (the reference's scheme, triton_kernel.py:69-145);
 *                     ONE_PASS (tensor-core paths 1 and 2, block_size a
 *                     multiple of 64): pass 1 also keeps, for
 *                     each row, the log2-sum of 2^s over every 64-key segment
 *                     it visits, and once the row's lse2 is final turns them
 *                     into bucket partials, sum_i 2^(segment sum - lse2_i):
 *                     the same mass from half the MMAs and exponentials.
 *                     With an LSE input pass 1 takes the caller's lse2 and
 *                     sums 2^(s - lse2) per segment directly (no running
 *                     max, no lg2, no exponentials in the epilogue).
 *                     AUTO takes ONE_PASS where it applies and its workspace
 *                     stays within 2x the two-pass one + 256 MiB, else
 *                     TWO_PASS.  ONE_PASS on a problem it does not apply to
 *                     is KVBM_ERR_SHAPE.  One pass keeps its segment sums
 *                     in 2 slots per SM indexed by %smid; on a device whose
 *                     SM ids reach past its SM count (not so on a whole
 *                     B200) a CTA there finds no slot, does no work and
 *                     kvbm_check_device_errors reports KVBM_ERR_TIMEOUT:
 *                     use TWO_PASS there.
 *   stages, run_unit_begin/end, run_head_begin/end
 *                     staged execution (all zero: the whole call).  A caller
 *                     that receives a problem in pieces, e.g. copying it from
 *                     host memory one unit at a time, runs the passes piece by
 *                     piece into ONE workspace sized for the whole problem
 *                     (kvbm_workspace_bytes_ex of the same p and o), on any
 *                     streams, and the bucket reduce once at the end; the
 *                     result then has the bits of one whole call.
 *                     stages: KVBM_STAGE_* bits (0 = all of them);
 *                     run_unit_begin/end: passes 1 and 2 cover units
 *                     [unit_begin + run_unit_begin, unit_begin + run_unit_end)
 *                     only (end <= begin: every unit of the problem); the
 *                     reduce always sums every unit;
 *                     run_head_begin/end: pass 1 covers q-heads [begin, end)
 *                     of each GQA group, 0 <= begin < end <= H_q/H_kv (end <=
 *                     begin: all); a head range narrower than the group needs
 *                     a run range of one unit;
 *                     run_row_begin/end: pass 1 covers query rows
 *                     [begin, end) of each head it runs (end <= begin: all
 *                     rows); begin a multiple of 128, end a multiple of 128
 *                     or N; it reads the k rows [0, end) under causal_skip,
 *                     all k rows otherwise.  Kernel paths 0 and 1 only, and
 *                     not with the LSE input (KVBM_ERR_SHAPE).  Pass 2 of a
 *                     unit reads pass 1 of all its heads and rows, and (fp32
 *                     inputs on path 2) the unit's k rows as converted by the
 *                     pass-1 piece whose head range starts at 0.  mass_out
 *                     may be NULL without KVBM_STAGE_REDUCE.  Pieces that
 *                     write disjoint units, heads or rows may run
 *                     concurrently.  Not combined with seq_lens, cu_seqlens
 *                     or paged (KVBM_ERR_SHAPE).
 *
 * Every ragged/per-sequence result equals the sum over sequences of the
 * reference run on each sequence alone (its first seq_lens[b] positions);
 * buckets j >= ceil(len / block_size) of a sequence get 0 from it. */
#define KVBM_STAGE_MASKS 1   /* pack a pair mask into bits; check a key mask's dropped keys
                                (tensor-core paths; run it before any pass-1 piece)      */
#define KVBM_STAGE_PASS1 2   /* row lse2, or the LSE import; fp32 path 2: tf32 split first;
                                one pass: also the bucket partials                       */
#define KVBM_STAGE_PASS2 4   /* per-key partials (two passes; launches nothing with one)   */
#define KVBM_STAGE_REDUCE 8  /* bucket reduce into mass_out                                */
#define KVBM_METHOD_AUTO 0
#define KVBM_METHOD_TWO_PASS 1
#define KVBM_METHOD_ONE_PASS 2
typedef struct kvbm_options {
  const float* lse;
  int64_t lse_stride[3];
  const kvbm_paged_kv* paged;
  const int32_t* seq_lens;
  const int32_t* cu_seqlens;
  int64_t total_tokens;
  int32_t per_sequence;
  void* const* events;
  int32_t stages;
  int32_t run_unit_begin;
  int32_t run_unit_end;
  int32_t run_head_begin;
  int32_t run_head_end;
  int32_t run_row_begin;
  int32_t run_row_end;
  int32_t method;
} kvbm_options;

/* Host-only checks of `p` with options `o` (o may be NULL). */
KVBM_API int kvbm_validate_ex(const kvbm_problem* p, const kvbm_options* o);

/* Workspace bytes kvbm_block_mass_ex needs (0 on invalid input). */
KVBM_API size_t kvbm_workspace_bytes_ex(const kvbm_problem* p, const kvbm_options* o);

/* The method (KVBM_METHOD_TWO_PASS or KVBM_METHOD_ONE_PASS) a
 * kvbm_block_mass_ex call of `p` with options `o` (may be NULL) takes on the
 * current device, or a kvbm_status error code, negated.  Host-only.  No
 * counterpart in the reference (it has only the two-pass scheme). */
KVBM_API int kvbm_method(const kvbm_problem* p, const kvbm_options* o);

/* Every option combined: dense, paged, padded-ragged or packed-varlen k/q,
 * optional LSE input, summed or per-sequence output.  `o` may be NULL (then
 * this is kvbm_block_mass).  Deterministic; the dense entry points above are
 * this call with the matching options. */
KVBM_API int kvbm_block_mass_ex(const kvbm_problem* p, const kvbm_options* o, void* mass_out, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Device-side consumers of the mass vector: the eviction design of
 * kv-block-mass (src/kvblockmass/evict.py), for `rows` sequences at once.
 *
 *   expand_block_scores  evict.py:64-83    scores[i] = mass[i / block_size] (float64)
 *   design_from_scores   evict.py:95-171   certainty = first n_sinks tokens, last
 *                                          recency tokens, the top_slice highest
 *                                          scores (ties: lower index first, the
 *                                          rule _top_slice's docstring states,
 *                                          evict.py:86-87); tail pi =
 *                                          clip(tail_budget * w / sum_tail w, eps, 1),
 *                                          w = scores (1 with uniform_tail, and a
 *                                          uniform design when the tail's scores
 *                                          sum to 0), eps for every tail token when
 *                                          tail_budget = 0; keep = certainty | u < pi
 *   hajek_log_offsets    evict.py:174-187  log_offsets = -log(pi)
 *   block retention      reclaim.py:46-55  blocks with at least one kept token
 *
 * Tail draws u: uniforms[row * uniforms_row_stride + t] for the t-th tail token
 * (ascending index) when `uniforms` is not NULL: the reference's
 * torch.rand(n_tail, dtype=float64, generator) gives bit parity; otherwise
 * Philox4x32-10 keyed by `seed`, counter = (token, row).
 * Row r's block mass is mass[r * mass_row_stride + b], b < num_blocks
 * (float32 or float64); blocks past ceil(seq_len / block_size) are ignored.
 * 1 <= rows <= 65535 and 1 <= seq_len <= 2^28, else KVBM_ERR_SHAPE. */
typedef struct kvbm_design_args {
  const void* mass;
  int32_t mass_dtype;            /* KVBM_F32 or KVBM_F64 */
  int32_t rows;
  int64_t mass_row_stride;
  int32_t num_blocks;
  int32_t seq_len;
  int32_t block_size;
  int32_t n_sinks;
  int32_t recency;
  int32_t top_slice;
  int64_t tail_budget;
  double eps;                    /* > 0 */
  int32_t uniform_tail;
  const double* uniforms;        /* or NULL */
  int64_t uniforms_row_stride;
  uint64_t seed;
} kvbm_design_args;

/* Outputs, [rows, seq_len] each, on the device; any may be NULL except
 * counts.  counts [rows, 5] int64: kept tokens, certainty tokens, tail tokens,
 * blocks kept (0 when keep is NULL), flags (1: a block mass is negative or
 * NaN, where the reference raises ValueError). */
typedef struct kvbm_design_out {
  double* pi;
  uint8_t* keep;
  uint8_t* certainty;
  double* scores;
  double* log_offsets;
  int64_t* counts;
} kvbm_design_out;

/* Workspace bytes of kvbm_design (0 on invalid arguments). */
KVBM_API size_t kvbm_design_workspace_bytes(const kvbm_design_args* d);

/* The design on the device, asynchronous on `stream` (three kernels: a
 * per-row select/scan CTA, a token kernel, a block-retention kernel).
 * No counterpart in the reference's GPU path: there the design runs in torch
 * on the host after mass.cpu(). */
KVBM_API int kvbm_design(const kvbm_design_args* d, const kvbm_design_out* out, void* workspace,
                size_t workspace_bytes, void* stream);

/* Queue `height` copies of `width` bytes on `stream`: row i goes from
 * src + i * src_pitch to dst + i * dst_pitch (cudaMemcpy2DAsync, direction
 * from the pointers).  The host-input path of the Python binding moves a
 * piece of q (the same rows of several q-heads) with one call; it stands in
 * for the host-to-device move of reference.py:74-76 (`q.to(device)`).  The
 * source must stay valid until the copy completes (pinned host memory:
 * asynchronous; pageable: the call returns after staging).  KVBM_ERR_NULL for
 * NULL pointers, KVBM_ERR_SHAPE for negative sizes or a pitch below `width`;
 * zero sizes queue nothing. */
KVBM_API int kvbm_copy_2d_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width,
                       int64_t height, void* stream);

/* Self-test of the failure path of the tcgen05 kernels' pipeline waits: one
 * thread waits on an mbarrier that nothing arrives at, through the same
 * bounded wait the kernels use, with a limit of limit_ns (1 us .. 2 s).  The
 * wait gives up, sets the device error word (kvbm_check_device_errors then
 * returns KVBM_ERR_TIMEOUT) and the kernel returns; *waited = 1 if the wait
 * was satisfied (it never is), 0 if it gave up.  Synchronises `stream`.
 * Nothing faults or hangs, and the context stays usable.  No counterpart in
 * the reference. */
KVBM_API int kvbm_selftest_wait_timeout(void* stream, uint64_t limit_ns, int* waited);

/* Reads and clears the device-side error words of the current device (set
 * when a bounded wait inside a tcgen05 kernel gave up, when a tcgen05 kernel
 * found no work slot or more work items than its launch covers (cu_seqlens
 * that decrease), or when a page gather met a block-table entry out of
 * range).  Synchronises `stream`.  Returns KVBM_OK, KVBM_ERR_TIMEOUT (the
 * first three; takes precedence), KVBM_ERR_PAGE or KVBM_ERR_CUDA. */
KVBM_API int kvbm_check_device_errors(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVBM_H */
