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
#include "hb_front.cuh"
#include "hb_internal.h"

namespace hb {
namespace {

constexpr int kWarps = 4;
using front::load_words;
using front::store_words;

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
  uint32_t yw[W];
  front::norm_rope<HD>(U.xw, U.ww, U.cw, U.sw, p.rotary, p.eps, p.inv_dim, p.gemma != 0, xs, lane, yw);
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
