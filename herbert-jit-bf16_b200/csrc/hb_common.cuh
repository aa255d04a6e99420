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

// Waits for phase `parity` of `bar` to complete; false after kSpinCycles.
HB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kSpinCycles) return false;
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

HB_DEV void record_status(int* status, int code) {
  if (status) atomicMax(status, code);
}

}  // namespace hb
