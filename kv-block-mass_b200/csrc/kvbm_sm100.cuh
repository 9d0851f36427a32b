// Thin inline-PTX wrappers for the sm_100a features the tensor-core kernels use:
// mbarriers (with bounded waits), TMA tensor/bulk copies, tcgen05 MMA, commit,
// TMEM alloc/ld and the tcgen05 ordering fences.  Instruction forms follow the
// PTX ISA 8.6+ (tcgen05.*, cp.async.bulk.tensor.*, mbarrier.*).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace kvbm {
namespace sm100 {

// Device-wide error word: nonzero once a bounded wait gave up (see kvbm.h,
// kvbm_check_device_errors).  Only kvbm_tc.cu includes this header, so the
// library holds exactly one copy.
__device__ unsigned int g_kvbm_device_error = 0;

// A wait on an mbarrier gives up after this many nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with `parity` to complete.  Returns false (and records
// the failure in the device error word and in *abort) if it does not within
// kWaitLimitNs, or if another role of this CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      *abort = 1;
      atomicOr(&g_kvbm_device_error, 1u);
      return false;
    }
  }
}

// ---- TMA ----
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// The same load with an L2 eviction policy (createpolicy).
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

// L2 eviction policies for a whole access (fraction 1.0).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2-only (.cg) global store / 16-byte load with an L2 eviction policy.
__device__ __forceinline__ void st_cg_hint(float* a, float v, uint64_t policy) {
  asm volatile("st.global.cg.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(a), "f"(v), "l"(policy) : "memory");
}
__device__ __forceinline__ float4 ld_cg_hint(const float4* a, uint64_t policy) {
  float4 v;
  asm volatile("ld.global.cg.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(a), "l"(policy)
               : "memory");
  return v;
}

// 1-D bulk copy global -> shared; both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads of them (an MMA operand written by threads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 ----
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/fp16 in, fp32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::tf32 (fp32 storage read as tf32, fp32 accumulate).
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when all tcgen05.mma previously issued by this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane
// (32 * (warp % 4) + t) of the accumulator, columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 lanes x 256 bits, repeated over 8 blocks of 8 columns starting at
// `taddr`'s column: thread t of the warp gets, for block m, lanes
// (lane(taddr) + t/4) and (+ 8) and the columns 8m + 2(t%4) + {0, 1}, in
// v[4m .. 4m+3] = (row t/4, c), (t/4, c+1), (t/4+8, c), (t/4+8, c+1).
__device__ __forceinline__ void tmem_ld16x256_x8(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tmem_ld16x256_x8 over 4 blocks of 8 columns: v[4m .. 4m+3], m < 4.
__device__ __forceinline__ void tmem_ld16x256_x4(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte-swizzle layout TMA writes (8-row x 128-byte swizzle atoms, atoms
// of consecutive rows 1024 bytes apart).  `addr` is the shared address of
// the first element this MMA reads (atom-aligned base + K offset in bytes).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4)   // start address
         | ((uint64_t)1 << 16)                  // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)        // stride byte offset: next 8-row group
         | ((uint64_t)1 << 46)                  // descriptor version (sm_100)
         | ((uint64_t)2 << 61);                 // swizzle mode: 128-byte
}

// Shared-memory matrix descriptor for a K-major operand of one 16-element
// (32-byte) K step stored without swizzle: 8-row x 16-byte core matrices,
// the two K halves 128 bytes apart, 8-row groups 256 bytes apart.
__device__ __forceinline__ uint64_t k16_interleaved_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4)  // start address
         | ((uint64_t)(128 >> 4) << 16)        // leading byte offset: the second K half
         | ((uint64_t)(256 >> 4) << 32)        // stride byte offset: next 8-row group
         | ((uint64_t)1 << 46);                // descriptor version (sm_100); swizzle: none
}

// Instruction descriptor, kind::f16 / kind::tf32: fp32 accumulate, A and B of
// the same input format (0 = fp16, 1 = bf16, 2 = tf32), both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_mma(int M, int N, uint32_t fmt) {
  return (1u << 4)                               // D format: f32
         | (fmt << 7)                            // A format
         | (fmt << 10)                           // B format
         | ((uint32_t)(N >> 3) << 17)            // N / 8
         | ((uint32_t)(M >> 4) << 24);           // M / 16
}

// Round fp32 to the nearest tf32 (10 explicit mantissa bits, low 13 bits zero).
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// MUFU log2 (lg2.approx: 0 -> -inf; subnormal inputs flush to zero)
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions) ----
__device__ __forceinline__ unsigned long long pk(float2 v) { return *reinterpret_cast<unsigned long long*>(&v); }
__device__ __forceinline__ float2 upk(unsigned long long u) { return *reinterpret_cast<float2*>(&u); }

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
  return upk(d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
  return upk(d);
}
// Flush-to-zero add: denormal inputs count as 0 (matches ex2.approx.ftz).
__device__ __forceinline__ float2 fadd2_ftz(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
  return upk(d);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for two arguments on the FMA pipe (no MUFU): x = j + f with
// j = rint(x) (the 1.5 * 2^23 shift rounds to nearest), f in [-1/2, 1/2];
// p(f) ~= 2^f is the degree-kDeg minimax polynomial for relative error on
// that interval (degree 4: max 2.7e-6; degree 3: 7.5e-5;
// kv-block-mass_b200/csrc/gen_exp2_poly.py), and 2^j is
// added into the exponent field.  x is clamped at -126.75 so that every
// result below 2^-126 is a positive denormal (never a wrapped exponent); a
// flush-to-zero accumulate adds those as exact zeros, like ex2.approx.ftz.
template <int kDeg = 4>
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  static_assert(kDeg == 3 || kDeg == 4, "minimax degree 3 or 4");
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.75f);
  x.y = fmaxf(x.y, -126.75f);
  const float2 t = fadd2(x, make_float2(kShift, kShift));
  const float2 j = fadd2(t, make_float2(-kShift, -kShift));
  const float2 f = ffma2(j, make_float2(-1.f, -1.f), x);
  float2 p;
  if constexpr (kDeg == 4) {  // max relative error 2.7e-6
    p = ffma2(f, make_float2(0.009570102207362652f, 0.009570102207362652f),
              make_float2(0.05591785907745361f, 0.05591785907745361f));
    p = ffma2(p, f, make_float2(0.240247443318367f, 0.240247443318367f));
    p = ffma2(p, f, make_float2(0.6931217908859253f, 0.6931217908859253f));
    p = ffma2(p, f, make_float2(0.9999992847442627f, 0.9999992847442627f));
  } else {  // max relative error 7.5e-5
    p = ffma2(f, make_float2(0.0551716685295105f, 0.0551716685295105f),
              make_float2(0.2426111251115799f, 0.2426111251115799f));
    p = ffma2(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
    p = ffma2(p, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
  }
  // bits(t) = bits(1.5 * 2^23) + j and 0x4B400000 << 23 == 0 (mod 2^32), so
  // (bits(t) << 23) is j << 23: the exponent increment of 2^j.
  const uint32_t rx = __float_as_uint(p.x) + (__float_as_uint(t.x) << 23);
  const uint32_t ry = __float_as_uint(p.y) + (__float_as_uint(t.y) << 23);
  return make_float2(__uint_as_float(rx), __uint_as_float(ry));
}

}  // namespace sm100
}  // namespace kvbm
