// hb_common.cuh -- device helpers shared by the sm_100a kernels: bf16 bit
// conversions, the reference's exp polynomial, mbarrier / bulk-copy PTX
// wrappers and bounded waits.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define HB_DEV __device__ __forceinline__

namespace hb {

// A bounded wait gives up after this many SM clock cycles (~1 s at 2 GHz).
constexpr long long kSpinCycles = 2000000000LL;

// ------------------------------------------------------------- bf16 bits

HB_DEV float bf16_to_f32(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }
HB_DEV float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
HB_DEV float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Round to nearest even with the vcvtneps2bf16 special cases the reference's
// epilogues use: zero and denormal inputs give a signed zero, NaN stays NaN.
// Written with selects, no branches, so that many elements interleave.
HB_DEV uint16_t f32_to_bf16_cvtne(float x) {
  const uint32_t u = __float_as_uint(x);
  const uint32_t ex = u & 0x7F800000u;
  const uint32_t rounded = (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
  const uint32_t special = (u & 0x7FFFFFu) ? ((u >> 16) | 0x40u) : (u >> 16);
  uint32_t r = ex == 0x7F800000u ? special : rounded;
  r = ex == 0u ? ((u >> 16) & 0x8000u) : r;
  return uint16_t(r);
}

// The emitted exp polynomial of the reference (src/jit/exp_constants.rs:14-23,
// src/jit/target/x86/emit_sdpa/x86/base.rs:189-212): clamp at -87.33654,
// split x*log2(e) into integer and fraction, degree-4 polynomial in the
// fraction, scale by 2^r built in the exponent field.  Every step rounds as
// the x86 sequence does.
HB_DEV float exp_poly(float x) {
  x = fmaxf(x, -87.33654f);  // vmaxps(x, c): c also when x is NaN, as fmaxf
  float t1 = __fmul_rn(x, 1.442695f);
  // round t1 to an integer, nearest even (vrndscaleps imm 0), by adding and
  // removing 1.5 * 2^23; the low bits of the sum hold that integer
  const float big = __fadd_rn(t1, 12582912.0f);
  const float t2 = __fsub_rn(big, 12582912.0f);
  t1 = __fsub_rn(t1, t2);
  float p = __fmaf_rn(0.00967248f, t1, 0.05550411f);
  p = __fmaf_rn(p, t1, 0.2402265f);
  p = __fmaf_rn(p, t1, 0.6931472f);
  p = __fmaf_rn(p, t1, 1.0f);
  const uint32_t r = uint32_t(__float_as_int(big) - 0x4B400000);
  return __fmul_rn(p, __uint_as_float((r << 23) + 0x3F800000u));
}

// The output gate of one element, y = bf16(a / (1 + exp(-b))), with the
// SigmoidMul arm's steps (src/jit/target/x86/emit_elem.rs:333-420).
HB_DEV uint16_t gate_bf16(uint16_t a_bits, uint16_t g_bits) {
  float a = bf16_to_f32(a_bits), u = bf16_to_f32(g_bits);
  float e = fminf(__fsub_rn(0.0f, u), 88.0f);  // vminps(e, 88): 88 also for NaN
  e = exp_poly(e);
  e = __fadd_rn(e, 1.0f);
  return f32_to_bf16_cvtne(__fdiv_rn(a, e));
}

// ------------------------------------------------ paired f32 arithmetic
// sm_100 add/sub/mul/fma on two f32 lanes at once, each lane rounded to
// nearest as the scalar instruction is: same bits, half the instructions.
// A paired multiply whose result feeds a paired add or subtract may be
// fused into one rounding by the assembler (measured: it was), so products
// that must round on their own stay on the scalar __fmul_rn.
HB_DEV uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
HB_DEV float f2lo(uint64_t v) { return __uint_as_float(uint32_t(v)); }
HB_DEV float f2hi(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }
HB_DEV uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
HB_DEV uint64_t f2sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
HB_DEV uint64_t f2mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
HB_DEV uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// f32_to_bf16_cvtne on two values, packed (lo in the low half): the
// hardware round-to-nearest-even conversion, then the reference's special
// cases (zero/denormal inputs give a signed zero, NaN keeps its payload).
HB_DEV uint32_t bf16x2_cvtne(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  const uint32_t ul = __float_as_uint(lo), uh = __float_as_uint(hi);
  const uint32_t el = ul & 0x7F800000u, eh = uh & 0x7F800000u;
  uint32_t rl = r & 0xFFFFu, rh = r >> 16;
  rl = el == 0u ? (ul >> 16) & 0x8000u : rl;
  rh = eh == 0u ? (uh >> 16) & 0x8000u : rh;
  rl = (el == 0x7F800000u && (ul & 0x7FFFFFu)) ? (ul >> 16) | 0x40u : rl;
  rh = (eh == 0x7F800000u && (uh & 0x7FFFFFu)) ? (uh >> 16) | 0x40u : rh;
  return rl | (rh << 16);
}

// exp_poly on two lanes: the additions, subtractions and polynomial FMAs
// paired, the products (which feed paired additions) on the scalar
// instruction so that none is fused.  Same bits as exp_poly per lane.
HB_DEV uint64_t exp_poly2(uint64_t x) {
  const float x0 = fmaxf(f2lo(x), -87.33654f), x1 = fmaxf(f2hi(x), -87.33654f);
  uint64_t t1 = f2(__fmul_rn(x0, 1.442695f), __fmul_rn(x1, 1.442695f));
  const uint64_t big = f2add(t1, f2(12582912.0f, 12582912.0f));
  const uint64_t t2 = f2sub(big, f2(12582912.0f, 12582912.0f));
  t1 = f2sub(t1, t2);
  uint64_t p = f2fma(f2(0.00967248f, 0.00967248f), t1, f2(0.05550411f, 0.05550411f));
  p = f2fma(p, t1, f2(0.2402265f, 0.2402265f));
  p = f2fma(p, t1, f2(0.6931472f, 0.6931472f));
  p = f2fma(p, t1, f2(1.0f, 1.0f));
  const uint32_t r0 = uint32_t(int32_t(uint32_t(big)) - 0x4B400000);
  const uint32_t r1 = uint32_t(int32_t(uint32_t(big >> 32)) - 0x4B400000);
  return f2(__fmul_rn(f2lo(p), __uint_as_float((r0 << 23) + 0x3F800000u)),
            __fmul_rn(f2hi(p), __uint_as_float((r1 << 23) + 0x3F800000u)));
}

// gate_divisor of the two bf16 gate values in `gw` (lo, hi), with the
// polynomial steps on paired lanes.
HB_DEV uint64_t gate_divisor2(uint32_t gw) {
  const uint64_t u = f2(__uint_as_float(gw << 16), __uint_as_float(gw & 0xFFFF0000u));
  const uint64_t neg = f2sub(f2(0.0f, 0.0f), u);
  float x0 = fminf(f2lo(neg), 88.0f), x1 = fminf(f2hi(neg), 88.0f);
  x0 = fmaxf(x0, -87.33654f);
  x1 = fmaxf(x1, -87.33654f);
  uint64_t t1 = f2(__fmul_rn(x0, 1.442695f), __fmul_rn(x1, 1.442695f));
  const uint64_t big = f2add(t1, f2(12582912.0f, 12582912.0f));
  const uint64_t t2 = f2sub(big, f2(12582912.0f, 12582912.0f));
  t1 = f2sub(t1, t2);
  uint64_t p = f2fma(f2(0.00967248f, 0.00967248f), t1, f2(0.05550411f, 0.05550411f));
  p = f2fma(p, t1, f2(0.2402265f, 0.2402265f));
  p = f2fma(p, t1, f2(0.6931472f, 0.6931472f));
  p = f2fma(p, t1, f2(1.0f, 1.0f));
  const uint32_t r0 = uint32_t(int32_t(uint32_t(big)) - 0x4B400000);
  const uint32_t r1 = uint32_t(int32_t(uint32_t(big >> 32)) - 0x4B400000);
  const float e0 = __fmul_rn(f2lo(p), __uint_as_float((r0 << 23) + 0x3F800000u));
  const float e1 = __fmul_rn(f2hi(p), __uint_as_float((r1 << 23) + 0x3F800000u));
  return f2(__fadd_rn(e0, 1.0f), __fadd_rn(e1, 1.0f));
}

// The gate's divisor 1 + exp(-b) with the SigmoidMul arm's steps.
HB_DEV float gate_divisor(uint16_t g_bits) {
  const float e = fminf(__fsub_rn(0.0f, bf16_to_f32(g_bits)), 88.0f);  // 88 also for NaN
  return __fadd_rn(exp_poly(e), 1.0f);
}

// a / d for d >= 1 through the SFU reciprocal, and whether that quotient
// may round to a different bf16 than the correctly rounded one: the
// reciprocal is off by a few f32 ulps at most, so the bf16 rounding can
// only differ when the quotient's low 16 bits lie within 32 ulps of the
// half-way point 0x8000, or when the quotient is near the smallest normal
// (denormals flush to zero in the conversion).  Callers recompute those
// rare quotients with the correctly rounded division.
HB_DEV float gate_quotient_fast(float a, float d, bool& risky) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  const float q = __fmul_rn(a, r);
  const uint32_t qb = __float_as_uint(q);
  risky = ((qb & 0xFFFFu) - 0x7FE0u) <= 0x40u || (qb & 0x7F000000u) == 0u;
  return q;
}

// 2^x with the SFU (ex2.approx.ftz): -inf -> +0.
HB_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------ shared memory PTX

HB_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

HB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

HB_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

HB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar))
               : "memory");
}

HB_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

HB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete; false after `limit` SM
// cycles (kSpinCycles, about a second, in every product kernel).
HB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, long long limit = kSpinCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

// One-dimensional bulk copy global -> this CTA's shared memory, completing
// `bytes` of transaction count on `bar`.  Both addresses 16-byte aligned,
// bytes a multiple of 16.  No multicast.
HB_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// bulk_g2s under an L2 policy (l2_evict_first below).
HB_DEV void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// An L2 policy that marks the lines an access brings in as the first to
// evict: for a stream read once (a KV cache swept by a decode step), so that
// it does not push out data that later launches read again.
HB_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Hint: bring `bytes` (a multiple of 16) from 16-byte-aligned global memory
// into L2.  A prefetch has no effect on the values any load returns (L2 is
// the point of coherence), so it may run before griddep_wait().
HB_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch.  griddep_wait() returns once the grids this
// one depends on have completed and their memory is visible (at once when
// the launch had no programmatic dependency); griddep_launch_dependents()
// lets the next grid on the stream be scheduled before this one ends.
HB_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
HB_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

HB_DEV void record_status(int* status, int code) {
  if (status) atomicMax(status, code);
}

// Named barriers: bar.sync waits for `n` threads to arrive (itself
// included), bar.arrive counts the calling warp without waiting.
HB_DEV void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
HB_DEV void named_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Warp 0's ordered sum of one pass's terms for column `lane`, kd ascending:
// group g (rows [GR g, GR (g + 1)), published by named barrier 1 + g of
// `nt` threads) read from shared memory while group g - 1 is summed.
template <int NG, int GR>
HB_DEV float sum_terms(const float4 (*terms)[32], int lane, int nt) {
  float acc = 0.f;
  float4 cur[GR / 4], nxt[GR / 4];
  named_sync(1, nt);
#pragma unroll
  for (int j = 0; j < GR / 4; ++j) cur[j] = terms[j][lane];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    if (g + 1 < NG) {
      named_sync(2 + g, nt);
#pragma unroll
      for (int j = 0; j < GR / 4; ++j) nxt[j] = terms[(g + 1) * (GR / 4) + j][lane];
    }
#pragma unroll
    for (int j = 0; j < GR / 4; ++j) {
      acc = __fadd_rn(acc, cur[j].x);
      acc = __fadd_rn(acc, cur[j].y);
      acc = __fadd_rn(acc, cur[j].z);
      acc = __fadd_rn(acc, cur[j].w);
    }
#pragma unroll
    for (int j = 0; j < GR / 4; ++j) cur[j] = nxt[j];
  }
  return acc;
}

// Sequential L2 of one head held in shared memory: sum of squares left to
// right, + eps, sqrt, 1/x (the L2 step of delta-l2-gates,
// src/jit/target/x86/execution/delta.rs:28-62).
template <int N>
HB_DEV float l2_inverse(const float* x, float eps) {
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    const float4 v = x4[i];
    sum = __fadd_rn(sum, __fmul_rn(v.x, v.x));
    sum = __fadd_rn(sum, __fmul_rn(v.y, v.y));
    sum = __fadd_rn(sum, __fmul_rn(v.z, v.z));
    sum = __fadd_rn(sum, __fmul_rn(v.w, v.w));
  }
  sum = __fadd_rn(sum, eps);
  return __fdiv_rn(1.0f, __fsqrt_rn(sum));
}

// One position of the delta rule on the state column s[0..HKD) a thread
// owns (delta-causal-recurrence, src/jit/target/x86/emit_recurrence.rs:108-217):
// pass 1 decays the column and reads kv = S^T k, pass 2 adds k delta and
// reads out = S^T q, each sum over kd in increasing order with separate
// multiply and add.  kn and qn are the normalised k and the scaled q in
// shared memory.
template <int HKD>
HB_DEV float gdn_step_column(float (&s)[HKD], const float* kn, const float* qn, float v, float beta,
                             float decay) {
  const float4* k4 = reinterpret_cast<const float4*>(kn);
  const float4* q4 = reinterpret_cast<const float4*>(qn);
  float kv = 0.f;
#pragma unroll
  for (int k = 0; k < HKD / 4; ++k) {
    const float4 kk = k4[k];
    const float kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float r = __fmul_rn(s[4 * k + e], decay);
      s[4 * k + e] = r;
      kv = __fadd_rn(kv, __fmul_rn(r, kw[e]));
    }
  }
  const float delta = __fmul_rn(__fsub_rn(v, kv), beta);
  float o = 0.f;
#pragma unroll
  for (int k = 0; k < HKD / 4; ++k) {
    const float4 kk = k4[k], qq = q4[k];
    const float kw[4] = {kk.x, kk.y, kk.z, kk.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float r = __fadd_rn(s[4 * k + e], __fmul_rn(kw[e], delta));
      s[4 * k + e] = r;
      o = __fadd_rn(o, __fmul_rn(r, qw[e]));
    }
  }
  return o;
}

}  // namespace hb
