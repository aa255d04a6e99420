// hb_front.cuh -- the arithmetic of the head-norm-rope node for one head
// held by a warp: the reference's GemmaRMSNorm (or RMSNorm) and RoPE steps,
// shared by the front-end kernel (attn_front.cu) and the decode kernel that
// runs the front end of its own query row (attn_decode_mma.cu).
//
// Norm (src/jit/target/x86/emit_elem.rs:242-330): sum of squares as
// vdpbf16ps lanes -- lane i of block c (32 elements) accumulates
// x[32c+2i+1]^2 then x[32c+2i]^2 by FMA, with denormal operands and results
// flushed -- into chain c % min(4, blocks); chains added in order; the hsum
// tree (emit_elem.rs:177-186); then x (1/dim), + eps, sqrt, 1/x, each
// rounded; per element y = bf16((x inv) w'), w' = w (+ 1 in f32).  RoPE
// (emit_elem.rs:479-514): a' = fma(-b, s, a c), b' = fma(b, c, a s), rounded
// to bf16 (vcvtneps2bf16 special cases).  Paired f32 operations where each
// lane is the scalar operation, the hardware bf16x2 conversion for zero and
// normal values, and the flushes skipped when no element of the head can
// produce a denormal, give the same bits.  Finite inputs are assumed (NaN
// payloads are not reproduced).
#pragma once

#include "hb_common.cuh"

namespace hb {
namespace front {

constexpr uint32_t kFull = 0xFFFFFFFFu;

// W packed words (two bf16 each) from / to global memory (W = 2 or 4).
template <int W>
HB_DEV void load_words(uint32_t (&w)[W], const uint16_t* p) {
  if constexpr (W == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  }
}
template <int W>
HB_DEV void store_words(uint16_t* p, const uint32_t (&w)[W]) {
  if constexpr (W == 4)
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  else
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
}

// vdpbf16ps operand and result modes: denormals are zero / flushed to zero.
HB_DEV float daz_bf16(uint16_t h) {
  return (h & 0x7F80u) == 0 ? __uint_as_float(uint32_t(h & 0x8000u) << 16) : bf16_to_f32(h);
}
HB_DEV float ftz(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x7F800000u) == 0 ? __uint_as_float(u & 0x80000000u) : x;
}

// zero, or a normal finite value: cvt.rn.bf16x2 then gives vcvtneps2bf16's bits
HB_DEV bool plain_for_cvt(float x) {
  const uint32_t u = __float_as_uint(x), e = u & 0x7F800000u;
  return (u & 0x7FFFFFFFu) == 0 || (e != 0 && e != 0x7F800000u);
}
// f32_to_bf16_cvtne of (lo, hi), packed: the hardware conversion, and the
// reference's special cases (denormal -> signed zero, NaN payload) only for
// the rare pairs that need them
HB_DEV uint32_t cvt_pair(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  if (!(plain_for_cvt(lo) && plain_for_cvt(hi))) r = bf16x2_cvtne(lo, hi);
  return r;
}

// Norm and RoPE of one head held by a warp: lane `lane` enters with the
// head's elements [lane E, lane E + E) as packed words xw (E = HD / 32), the
// norm weights ww, and -- for lanes below rotary -- the cos / sin table
// words cw, sw of the row's position (pair index j0 = element - half in the
// second rotated half); returns the bf16 results as packed words yw.  xs is
// HD / 2 words of shared memory for the warp.
template <int HD>
HB_DEV void norm_rope(const uint32_t (&xw)[HD / 64], const uint32_t (&ww)[HD / 64],
                      const uint32_t (&cw)[HD / 64], const uint32_t (&sw)[HD / 64], int rotary,
                      float eps, float inv_dim, bool gemma, uint32_t* xs, int lane,
                      uint32_t (&yw)[HD / 64]) {
  constexpr int E = HD / 32;   // elements per lane
  constexpr int W = E / 2;     // packed words per lane
  constexpr int NB = HD / 32;  // 32-element blocks (vdpbf16ps operands)
  constexpr int NA = 4;        // sum-of-squares chains (min(4, NB), NB >= 4 here)
  static_assert(NB >= NA, "head_dim 128 or 256");
  const int half = rotary / 2;
  const bool rot = lane * E < rotary, first = lane * E < half;
  // ---- sum of squares: the vdpbf16ps chains.  Lane L is accumulator lane
  // L % 16 of chains 2 (L / 16) and 2 (L / 16) + 1; chain k takes blocks k,
  // k + 4, ...; each block step accumulates the odd element of the pair,
  // then the even one.  When every element is zero or at least 2^-63 in
  // magnitude no operand or partial sum can be denormal, and the flushes
  // are no-ops (one decision for the warp).
  __syncwarp();  // the previous unit's reads of xs are done
  bool fast_l = true;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const uint32_t m = xw[i] & 0x7FFF7FFFu, lo = m & 0xFFFFu, hi = m >> 16;
    fast_l = fast_l && (lo == 0 || lo >= 0x2000u) && (hi == 0 || hi >= 0x2000u);
    xs[lane * W + i] = xw[i];
  }
  const bool fast = __all_sync(kFull, fast_l);
  __syncwarp();
  const int ai = lane & 15, cb = (lane >> 4) * 2;
  float acc[2];
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    float a = 0.f;
#pragma unroll
    for (int c = cb + kk; c < NB; c += NA) {
      const uint32_t pw = xs[16 * c + ai];  // elements 32c + 2ai (low), + 1 (high)
      if (fast) {
        const float xo = bf16hi(pw), xe = bf16lo(pw);
        a = __fmaf_rn(xo, xo, a);
        a = __fmaf_rn(xe, xe, a);
      } else {
        const float xo = daz_bf16(uint16_t(pw >> 16)), xe = daz_bf16(uint16_t(pw & 0xFFFFu));
        a = ftz(__fmaf_rn(xo, xo, a));
        a = ftz(__fmaf_rn(xe, xe, a));
      }
    }
    acc[kk] = a;
  }
  // chains added in order: ((c0 + c1) + c2) + c3, lane i < 16 takes c2, c3
  // from lane i + 16
  const float c2 = __shfl_sync(kFull, acc[0], ai + 16), c3 = __shfl_sync(kFull, acc[1], ai + 16);
  const float a0 = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), c2), c3);
  // hsum: (l, l + 8), then (l, l + 4), then (e1 + e0) and (e3 + e2), summed
  const float d = __fadd_rn(a0, __shfl_down_sync(kFull, a0, 8));
  const float e = __fadd_rn(d, __shfl_down_sync(kFull, d, 4));
  const float e0 = __shfl_sync(kFull, e, 0), e1 = __shfl_sync(kFull, e, 1);
  const float e2 = __shfl_sync(kFull, e, 2), e3 = __shfl_sync(kFull, e, 3);
  float s = __fadd_rn(__fadd_rn(e3, e2), __fadd_rn(e1, e0));
  s = __fmul_rn(s, inv_dim);
  s = __fadd_rn(s, eps);
  s = __fsqrt_rn(s);
  const float inv = __fdiv_rn(1.0f, s);

  // ---- y = bf16((x inv) w'), two elements per paired operation
  {
    const uint64_t inv2 = f2(inv, inv), one2 = f2(1.0f, 1.0f);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      uint64_t w2 = f2(bf16lo(ww[i]), bf16hi(ww[i]));
      if (gemma) w2 = f2add(w2, one2);
      const uint64_t y2 = f2mul(f2mul(f2(bf16lo(xw[i]), bf16hi(xw[i])), inv2), w2);
      yw[i] = cvt_pair(f2lo(y2), f2hi(y2));
    }
  }

  // ---- RoPE on elements [0, rotary): the partner of element j < half is
  // j + half, half / E lanes away.  a' = fma(b, -s, a c), b' = fma(b, c, a s)
  // (the products a c and a s rounded on their own).
  {
    const int step = half / E;
    const int src = !rot ? lane : first ? lane + step : lane - step;
    uint32_t pw[W];
#pragma unroll
    for (int i = 0; i < W; ++i) pw[i] = __shfl_sync(kFull, yw[i], src);
    if (rot) {
#pragma unroll
      for (int i = 0; i < W; ++i) {
        const float c_lo = bf16lo(cw[i]), c_hi = bf16hi(cw[i]);
        const float s_lo = bf16lo(sw[i]), s_hi = bf16hi(sw[i]);
        // (a, b) of the pair: own value and partner's, by half
        const uint32_t aw = first ? yw[i] : pw[i], bw = first ? pw[i] : yw[i];
        const float a_lo = bf16lo(aw), a_hi = bf16hi(aw);
        const float m_lo = first ? c_lo : s_lo, m_hi = first ? c_hi : s_hi;  // a's factor
        const float n_lo = first ? -s_lo : c_lo, n_hi = first ? -s_hi : c_hi;  // b's factor
        const uint64_t o2 = f2fma(f2(bf16lo(bw), bf16hi(bw)), f2(n_lo, n_hi),
                                  f2(__fmul_rn(a_lo, m_lo), __fmul_rn(a_hi, m_hi)));
        yw[i] = cvt_pair(f2lo(o2), f2hi(o2));
      }
    }
  }

}

}  // namespace front
}  // namespace hb
