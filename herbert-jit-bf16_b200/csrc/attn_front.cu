// attn_front.cu -- the attention front end of one layer on sm_100a: the
// head-norm-rope nodes of q and of k and the kv-append node, in one launch.
//
// Replaces (src/jit/schedule/lowering.rs:549-592): for every row r and every
// q head, then every k head, ElemOp::RmsNormGemma (or RmsNorm) in place
// followed by ElemOp::Rope on the first `rotary` elements with the cos/sin
// table row of position past + r (src/jit/target/x86/execution/transforms.rs:30-81);
// then K[h][past + r][:] <- k[r][h][:] and V likewise
// (src/jit/target/x86/execution/kv.rs:17-69).
//
// Arithmetic: the reference's emitted instructions, step for step, so the
// results are its bits.  Norm (src/jit/target/x86/emit_elem.rs:242-330):
// sum of squares as vdpbf16ps lanes -- lane i of block c (32 elements)
// accumulates x[32c+2i+1]^2 then x[32c+2i]^2 by FMA, with denormal operands
// and results flushed -- into chain c % min(4, blocks); chains added in
// order; the hsum tree (emit_elem.rs:177-186); then x (1/dim), + eps, sqrt,
// 1/x, each rounded; per element y = bf16((x inv) w'), w' = w (+ 1 in f32).
// RoPE (emit_elem.rs:479-514): a' = fma(-b, s, a c), b' = fma(b, c, a s),
// rounded to bf16 (vcvtneps2bf16 special cases).  The same bits come
// cheaper where that is provable: paired f32 operations where each lane is
// the scalar operation, the hardware bf16x2 conversion for zero and normal
// values (the special cases only for the pairs that need them), and the
// flushes of the sum of squares skipped when no element of the head can
// produce a denormal (all zero or at least 2^-63 in magnitude).  Finite
// inputs are assumed (NaN payloads are not reproduced).
//
// Work decomposition: one warp per (row, head), q heads then k heads; a
// lane holds head_dim / 32 consecutive elements (one 16-byte load at
// head_dim 256).  The warp of k head h also moves v head h into the cache.
// HBM-bound: every element is read once and written once (k twice: in place
// and into the cache).
#include <cstdint>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_internal.h"

namespace hb {
namespace {

constexpr int kWarps = 4;
constexpr uint32_t kFull = 0xFFFFFFFFu;

struct FrontParams {
  uint16_t* q;
  uint16_t* k;
  const uint16_t* v;
  const uint16_t* qn;
  const uint16_t* kn;
  const uint16_t* cos;
  const uint16_t* sin;
  uint16_t* keys;
  uint16_t* values;
  int64_t q_row, kv_row, kv_stride, past;
  int rows, heads, kv_heads, rotary;
  float eps, inv_dim;
  int gemma;
};

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

// One (row, head) unit of the front end: where it lives and its loaded words.
template <int W>
struct Unit {
  uint16_t* x;  // the head's elements (q or k row)
  int r, h;
  bool isq, valid;
  uint32_t xw[W], ww[W], vw[W], cw[W], sw[W];
};

template <int HD>
HB_DEV void load_unit(Unit<HD / 64>& U, const FrontParams& p, int64_t u, int lane) {
  constexpr int E = HD / 32, W = E / 2;
  const int units = p.heads + p.kv_heads;
  U.valid = u < int64_t(p.rows) * units;
  if (!U.valid) return;
  U.r = int(u / units);
  const int hu = int(u % units);
  U.isq = hu < p.heads;
  U.h = U.isq ? hu : hu - p.heads;
  U.x = U.isq ? p.q + int64_t(U.r) * p.q_row + int64_t(U.h) * HD
              : p.k + int64_t(U.r) * p.kv_row + int64_t(U.h) * HD;
  load_words<W>(U.xw, U.x + lane * E);
  load_words<W>(U.ww, (U.isq ? p.qn : p.kn) + lane * E);
  if (!U.isq) load_words<W>(U.vw, p.v + int64_t(U.r) * p.kv_row + int64_t(U.h) * HD + lane * E);
  // the table row of this position; lanes of the second rotated half use
  // pair index j0 = element - half
  const int half = p.rotary / 2;
  if (lane * E < p.rotary) {
    const int j0 = lane * E < half ? lane * E : lane * E - half;
    const int64_t t = (p.past + U.r) * int64_t(half) + j0;
    load_words<W>(U.cw, p.cos + t);
    load_words<W>(U.sw, p.sin + t);
  }
}

template <int HD>
HB_DEV void process_unit(Unit<HD / 64>& U, const FrontParams& p, uint32_t* xs, int lane) {
  constexpr int E = HD / 32;   // elements per lane
  constexpr int W = E / 2;     // packed words per lane
  constexpr int NB = HD / 32;  // 32-element blocks (vdpbf16ps operands)
  constexpr int NA = 4;        // sum-of-squares chains (min(4, NB), NB >= 4 here)
  static_assert(NB >= NA, "head_dim 128 or 256");
  const int half = p.rotary / 2;
  const bool rot = lane * E < p.rotary, first = lane * E < half;
  uint32_t* xw = U.xw;

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
  s = __fmul_rn(s, p.inv_dim);
  s = __fadd_rn(s, p.eps);
  s = __fsqrt_rn(s);
  const float inv = __fdiv_rn(1.0f, s);

  // ---- y = bf16((x inv) w'), two elements per paired operation
  uint32_t yw[W];
  {
    const uint64_t inv2 = f2(inv, inv), one2 = f2(1.0f, 1.0f);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      uint64_t w2 = f2(bf16lo(U.ww[i]), bf16hi(U.ww[i]));
      if (p.gemma) w2 = f2add(w2, one2);
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
        const float c_lo = bf16lo(U.cw[i]), c_hi = bf16hi(U.cw[i]);
        const float s_lo = bf16lo(U.sw[i]), s_hi = bf16hi(U.sw[i]);
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

  // ---- results: in place, and a k head (with its v head) into the cache
  store_words<W>(U.x + lane * E, yw);
  if (!U.isq && p.keys) {
    const int64_t dst = int64_t(U.h) * p.kv_stride + (p.past + U.r) * int64_t(HD) + lane * E;
    store_words<W>(p.keys + dst, yw);
    store_words<W>(p.values + dst, U.vw);
  }
}

// Units per warp.  Two units per warp, both loaded before the first is
// transformed, ran slower on B200 (64 registers halve the resident warps;
// 56.0 against 44.4 us for a 4096-row block), so each warp takes one.
constexpr int kUnitsPerWarp = 1;

template <int HD>
__global__ void __launch_bounds__(kWarps * 32) attn_front_kernel(const FrontParams p) {
  __shared__ __align__(16) uint32_t xs[kWarps][HD / 2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = (int64_t(blockIdx.x) * kWarps + warp) * kUnitsPerWarp;
  Unit<HD / 64> U[kUnitsPerWarp];
#pragma unroll
  for (int j = 0; j < kUnitsPerWarp; ++j) load_unit<HD>(U[j], p, u0 + j, lane);
#pragma unroll
  for (int j = 0; j < kUnitsPerWarp; ++j)
    if (U[j].valid) process_unit<HD>(U[j], p, xs[warp], lane);  // warp-uniform
}

}  // namespace

bool front_serves(int64_t head_dim, int64_t rotary) {
  return (head_dim == 128 || head_dim == 256) && rotary >= 0 && rotary % 32 == 0 &&
         rotary <= head_dim;
}

cudaError_t launch_attn_front(const FrontLaunch& L, cudaStream_t st) {
  FrontParams p;
  p.q = L.q;
  p.k = L.k;
  p.v = L.v;
  p.qn = L.q_norm;
  p.kn = L.k_norm;
  p.cos = L.cos;
  p.sin = L.sin;
  p.keys = L.keys;
  p.values = L.values;
  p.q_row = L.q_row;
  p.kv_row = L.kv_row;
  p.kv_stride = L.kv_stride;
  p.past = L.past;
  p.rows = int(L.rows);
  p.heads = int(L.heads);
  p.kv_heads = int(L.kv_heads);
  p.rotary = int(L.rotary);
  p.eps = L.eps;
  p.inv_dim = 1.0f / float(L.head_dim);
  p.gemma = L.gemma ? 1 : 0;
  const int64_t warps = (L.rows * (L.heads + L.kv_heads) + kUnitsPerWarp - 1) / kUnitsPerWarp;
  const unsigned grid = unsigned((warps + kWarps - 1) / kWarps);
  if (L.head_dim == 256)
    attn_front_kernel<256><<<grid, kWarps * 32, 0, st>>>(p);
  else if (L.head_dim == 128)
    attn_front_kernel<128><<<grid, kWarps * 32, 0, st>>>(p);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace hb
