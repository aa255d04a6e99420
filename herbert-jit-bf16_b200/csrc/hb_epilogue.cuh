// hb_epilogue.cuh -- the prefill epilogue's arithmetic for a block of W
// consecutive columns of one output row (W = kEpilogueWidth in the kernel):
// a = bf16(O / l), then, with the output gate, y = bf16(a / (1 + exp(-g))).
// Element by element the result is the bits of f32_to_bf16_cvtne(O * inv)
// followed by gate_bf16(a, g), the reference's conversion and SigmoidMul
// steps (src/jit/target/x86/emit_elem.rs:333-420).
//
// Fast path, for all W columns at once:
//  * conversions by cvt.rn.bf16x2, which give bf16x2_cvtne's bits unless an
//    input is denormal or NaN;
//  * the divisor 1 + exp(-g) on paired lanes (gate_divisor2, the reference's
//    polynomial and rounding steps);
//  * the quotient from the SFU reciprocal r ~ 1/d (relative error below
//    2^-22) refined by one Newton correction, q1 = q0 + (a - q0 d) r with
//    q0 = a r and the residual by FMA (Markstein, "Computation of elementary
//    functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34,
//    1990).  q1 lies within 1e-5 of an f32 ulp of a / d, so it is the
//    correctly rounded quotient unless a / d sits that close to an f32
//    rounding boundary, and even then it is one ulp off, which changes the
//    bf16 rounding only when q1's low 16 bits are 0x7FFF, 0x8000 or 0x8001.
// A pair of columns whose quotient has such low bits, or lies below 2^-100
// in magnitude (zero, a reciprocal flushed to zero, an `a` rounded from a
// denormal), or is infinite or NaN, is recomputed with the exact
// per-element steps; without the gate the same goes for a pair of O / l
// values that is zero, denormal, infinite or NaN.  The self-test
// hb_selftest_prefill_epilogue runs this code over every (a, g) pair of
// bf16 values and every f32 O / l against the exact steps.
#pragma once

#include "hb_common.cuh"

namespace hb {

// cvt.rn.bf16x2.f32 alone (lo in the low half).
HB_DEV uint32_t bf16x2_cvt_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// |lo| and |hi| both at least `lim` and finite (zero, NaN and infinity fail).
HB_DEV bool pair_in_range(float lo, float hi, float lim) {
  const float a = fabsf(lo), b = fabsf(hi);
  return fminf(a, b) >= lim && a + b < INFINITY;
}

// Low 16 bits of q in 0x7FFF .. 0x8001.
HB_DEV bool near_bf16_tie(float q) { return ((__float_as_uint(q) & 0xFFFFu) - 0x7FFFu) <= 2u; }

// a / d for d >= 1: SFU reciprocal, then one Newton correction.
HB_DEV float gate_quotient_newton(float a, float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  const float q0 = __fmul_rn(a, r);
  const float e = __fmaf_rn(-q0, d, a);
  return __fmaf_rn(e, r, q0);
}

// Columns per block in the prefill kernel's epilogue (and its self-test).
constexpr int kEpilogueWidth = 16;

// One block of W columns: o = f32 bits of O, inv = 1 / l, gw = the gate's
// bf16 values two per word (GATE only), w = output bf16 two per word.
// Returns the number of column pairs that took the exact steps.
template <int W, bool GATE>
HB_DEV int epilogue_block(const uint32_t (&o)[W], float inv, const uint32_t (&gw)[W / 2],
                          uint32_t (&w)[W / 2]) {
  constexpr int H = W / 2;
  const uint64_t inv2 = f2(inv, inv);
  int slow = 0;
  if constexpr (!GATE) {
    bool fast = true;
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const uint64_t ov = f2mul(f2(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2);
      w[i] = bf16x2_cvt_rn(f2lo(ov), f2hi(ov));
      fast = fast && pair_in_range(f2lo(ov), f2hi(ov), 0x1p-126f);
    }
    if (!fast) {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const uint64_t ov =
            f2mul(f2(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2);
        if (!pair_in_range(f2lo(ov), f2hi(ov), 0x1p-126f)) {
          w[i] = bf16x2_cvtne(f2lo(ov), f2hi(ov));
          ++slow;
        }
      }
    }
  } else {
    float q[W];
    bool fast = true;
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const uint64_t ov = f2mul(f2(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2);
      const uint32_t a2 = bf16x2_cvt_rn(f2lo(ov), f2hi(ov));
      const uint64_t d2 = gate_divisor2(gw[i]);
      q[2 * i] = gate_quotient_newton(bf16lo(a2), f2lo(d2));
      q[2 * i + 1] = gate_quotient_newton(bf16hi(a2), f2hi(d2));
      w[i] = bf16x2_cvt_rn(q[2 * i], q[2 * i + 1]);
      fast = fast && !near_bf16_tie(q[2 * i]) && !near_bf16_tie(q[2 * i + 1]) &&
             pair_in_range(q[2 * i], q[2 * i + 1], 0x1p-100f);
    }
    if (!fast) {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        if (near_bf16_tie(q[2 * i]) || near_bf16_tie(q[2 * i + 1]) ||
            !pair_in_range(q[2 * i], q[2 * i + 1], 0x1p-100f)) {
          const uint64_t ov =
              f2mul(f2(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2);
          const uint32_t ab = bf16x2_cvtne(f2lo(ov), f2hi(ov));
          w[i] = uint32_t(gate_bf16(uint16_t(ab & 0xFFFFu), uint16_t(gw[i] & 0xFFFFu))) |
                 (uint32_t(gate_bf16(uint16_t(ab >> 16), uint16_t(gw[i] >> 16))) << 16);
          ++slow;
        }
      }
    }
  }
  return slow;
}

}  // namespace hb
