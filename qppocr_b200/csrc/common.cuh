// Shared device helpers for the qppocr B200 backend (sm_100a only).
//
//  * Epilogue arithmetic that restates the reference CPU path element by
//    element (qppocr-kernels activation.rs), so fused epilogues reproduce the
//    reference's separate passes bit for bit given the same pre-activation.
//  * Thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor) and the
//    5th-generation tensor core (tcgen05.*).  Every spin-wait is bounded: on
//    timeout the kernel records an error code in a device error word that the
//    host checks, and the kernel unwinds instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qpc {

// ------------------------------------------------------------ error flag
// Kernels with bounded waits receive a pointer to a per-device error word
// (allocated once by the runtime).  A wait that runs out sets a bit there;
// the host reads and clears it after synchronising.

enum KernelError : unsigned int {
  KERR_MBAR_TIMEOUT = 1u,   // an mbarrier wait exceeded its iteration limit
  KERR_BAD_CONFIG = 2u,     // a kernel was launched with an impossible shape
};

// Time limit for one mbarrier wait (global timer, ns).  Legitimate waits in
// these kernels last microseconds; 200 ms means the pipeline is broken.
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;

// ----------------------------------------------------- epilogue semantics
// Activation codes used by fused epilogues.  They name the reference's graph
// patterns that the planner folds into a producer kernel:
//   ACT_NONE        -
//   ACT_RELU        Relu / Conv act=2            (activation.rs:157-162)
//   ACT_HARDSWISH   x * HardSigmoid(x)           (activation.rs:170-189, then Mul)
//   ACT_SIGMOID     Sigmoid                      (activation.rs:197-201)
//   ACT_GELU        Conv act=1 / FusedGelu       (activation.rs:208-217)
//   ACT_HARDSIGMOID HardSigmoid alone            (activation.rs:170-189)
//   ACT_SWISH       x * Sigmoid(x)               (Sigmoid then Mul)
enum ActKind : int {
  ACT_NONE = 0,
  ACT_RELU = 1,
  ACT_HARDSWISH = 2,
  ACT_SIGMOID = 3,
  ACT_GELU = 4,
  ACT_HARDSIGMOID = 5,
  ACT_SWISH = 6,
};

struct ActParams {
  int kind;
  float alpha, beta;      // HardSigmoid alpha / beta
  float c1, c2, c3;       // GELU constants
  // depthwise conv only: round the final output to tf32 (nearest), set when
  // every consumer is a TF32 GEMM that rounds its A operand the same way, so
  // the GEMM can skip that pass and the results do not change
  int round_tf32;
};

// exp1: the reference's polynomial exp (activation.rs:28-47): clamp to
// [-88, 88], k = round-ties-even(x / ln2), two-part ln2 reduction, 7-term
// Horner with fused multiply-adds, scale by 2^k through the exponent field.
__device__ __forceinline__ float exp1(float x) {
  const float LN2_HI = 0.6931472f;
  const float LN2_LO = -2.9802322e-8f;
  const float INV_LN2 = 1.442695f;
  x = fmaxf(fminf(x, 88.0f), -88.0f);
  const float kf = rintf(__fmul_rn(x, INV_LN2));
  float r = __fmaf_rn(-kf, LN2_HI, x);
  r = __fmaf_rn(-kf, LN2_LO, r);
  float p = 1.0f / 720.0f;
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ki = (int)kf + 127;
  return __fmul_rn(__int_as_float(ki << 23), p);
}

// erf1: Abramowitz & Stegun 7.1.26 as the reference writes it (activation.rs:53-66).
__device__ __forceinline__ float erf1(float x) {
  const float ax = fabsf(x);
  const float t = __fdiv_rn(1.0f, __fmaf_rn(0.3275911f, ax, 1.0f));
  float p = 1.0614054f;
  p = __fmaf_rn(p, t, -1.453152027f);
  p = __fmaf_rn(p, t, 1.421413741f);
  p = __fmaf_rn(p, t, -0.284496736f);
  p = __fmaf_rn(p, t, 0.2548296f);
  p = __fmul_rn(p, t);
  const float e = exp1(__fmul_rn(ax, __fsub_rn(0.0f, ax)));
  const float r = __fmaf_rn(-p, e, 1.0f);
  return __uint_as_float(__float_as_uint(r) | (__float_as_uint(x) & 0x80000000u));
}

__device__ __forceinline__ float hardsigmoid(float v, float alpha, float beta) {
  const float t = __fmaf_rn(v, alpha, beta);
  return t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
}

__device__ __forceinline__ float sigmoid1(float v) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp1(-v)));
}

// Apply a fused activation to an already bias-added value v.
__device__ __forceinline__ float apply_act(float v, const ActParams& a) {
  switch (a.kind) {
    case ACT_RELU: return v > 0.0f ? v : 0.0f;
    case ACT_HARDSWISH: return __fmul_rn(v, hardsigmoid(v, a.alpha, a.beta));
    case ACT_SIGMOID: return sigmoid1(v);
    case ACT_GELU: {
      const float inv_c1 = __fdiv_rn(1.0f, a.c1);
      return __fmul_rn(__fmul_rn(a.c3, v), __fadd_rn(erf1(__fmul_rn(v, inv_c1)), a.c2));
    }
    case ACT_HARDSIGMOID: return hardsigmoid(v, a.alpha, a.beta);
    case ACT_SWISH: return __fmul_rn(v, sigmoid1(v));
    default: return v;
  }
}

// Activation over a register array: one (uniform) switch per array, not per
// element, so the epilogue's inner loops stay branch-free.
template <int N>
__device__ __forceinline__ void apply_act_n(float (&v)[N], const ActParams& a) {
  switch (a.kind) {
    case ACT_NONE: return;
    case ACT_RELU:
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = v[j] > 0.0f ? v[j] : 0.0f;
      return;
    case ACT_HARDSWISH:
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = __fmul_rn(v[j], hardsigmoid(v[j], a.alpha, a.beta));
      return;
    case ACT_HARDSIGMOID:
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = hardsigmoid(v[j], a.alpha, a.beta);
      return;
    case ACT_SIGMOID:
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = sigmoid1(v[j]);
      return;
    case ACT_SWISH:
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = __fmul_rn(v[j], sigmoid1(v[j]));
      return;
    default:
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = apply_act(v[j], a);
      return;
  }
}

// ------------------------------------------------------------- smem / PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false when the time limit passes (raising the error flag) or when another
// CTA has already raised it (so a broken launch drains in one timeout, not
// one per CTA).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, unsigned int* err,
                                              uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 127u) == 0) {
      if (err && *reinterpret_cast<volatile unsigned int*>(err)) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        if (err) atomicOr(err, (unsigned)KERR_MBAR_TIMEOUT);
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
  return mbar_wait_for(bar, parity, err, kWaitNs);
}

// TMA tiled loads (no multicast).  Coordinates are element indices, innermost first.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// TMA tiled stores from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          (uint64_t)map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          (uint64_t)map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Named barrier among `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Brings the 128-byte line holding p into L2 (no register result).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Brings the 128-byte line holding p into this SM's L1 (no register result).
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor core / TMA) before signalling.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: 8-row x 128-byte swizzle atoms stacked along M/N
// (stride byte offset 1024), start address in 16-byte units, descriptor
// version 1 (bits 46-47), layout type SWIZZLE_128B (= 2, bits 61-63).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(1u) << 16;                 // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;  // stride byte offset
  d |= (uint64_t)1u << 46;                   // version
  d |= (uint64_t)2u << 61;                   // SWIZZLE_128B
  return d;
}

// fp32 -> tf32 with round-to-nearest (ties away), as a 32-bit container with
// the low 13 mantissa bits zero.  The tensor core would otherwise truncate,
// which biases every product toward zero.
// Integer form: add half an ulp of tf32 to the magnitude bits, clear the low
// 13 bits (ties away from zero; identical to cvt.rna.tf32.f32 for finite
// values) -- two full-rate integer ops instead of a conversion instruction.
__device__ __forceinline__ float tf32_rna(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// Issue one 32x32b x16 TMEM load without waiting (pair with tmem_ld_wait).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Instruction descriptor, kind::tf32: D f32, A/B tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

}  // namespace qpc
