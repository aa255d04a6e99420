// gdn_front.cu -- the DeltaNet front and back ends of one layer on sm_100a:
// the causal depthwise conv + SiLU over the qkv projection and the beta /
// decay gates (one launch), and the gated RMS norm of the recurrence output.
//
// Replaces, for the x86 AVX-512 path of the reference:
//  * delta-causal-convolution (src/jit/target/x86/execution/delta.rs:609-705):
//    per channel, state[0..ck) <- state[1..ck) ++ x, y = silu(sum_j state_j w_j).
//    Channels of full 16-channel blocks at ck = 4 take the vector kernel
//    (src/jit/target/x86/emit_conv.rs:141-211): products summed as
//    (p0 + p1) + (p2 + p3), SiLU g / (1 + exp(min(0 - g, 88))) with the emitted
//    exp polynomial.  The other channels (a ragged last block, or every channel
//    when ck != 4) take the scalar body (delta_scalar.rs:85-155): products
//    added in tap order from +0, SiLU with the scalar exp of -g.
//  * the gate part of delta-l2-gates (delta.rs:290-389), task row*nv + h:
//    beta = 1 / (exp(-b) + 1); dt = a + bf16(dt_bias); dt = log(exp(dt) + 1)
//    unless dt > 20; decay = exp((-exp(a_log)) dt).
//  * delta-gated-norm (delta.rs:706-774): per (row, V head) of width dim,
//    inv = 1 / sqrt(sum x^2 / dim + eps); y = ((x inv) w) silu(z).  dim a
//    multiple of 16 up to 128 takes the vector kernel
//    (src/jit/target/x86/emit_gated_norm.rs:112-169: sum of squares in
//    min(4, dim/16) FMA chains of 16 lanes, chains added in order, the hsum
//    tree; SiLU with the exp polynomial; bf16 by vcvtneps2bf16); other widths
//    the scalar body (delta_scalar.rs:159-239: sum in order from +0, scalar
//    exp, bf16 by the wrapping integer rounding).
//
// The scalar exp and log are the reference's emitted routines
// (src/jit/target/x86/execution/math.rs, FMA form): the published Arm
// optimized-routines expf / logf, evaluated in double.  Every step below is
// one IEEE operation of the reference's sequence, so results are its bits
// (NaN payloads excepted).
//
// Layout in HBM (the reference's): qkv [rows][conv] f32 (conv = 2 nk hkd +
// nv hvd), conv state [conv][ck] f32, conv weights [conv][ck] bf16, ab
// [rows][2 nv] f32 (a then b), beta / decay [rows][nv] f32; gated norm x, z
// [rows][nv hvd] f32, weight [hvd] bf16, out [rows][nv hvd] bf16.
//
// Conv decomposition: one CTA per strip of 32 channels walks every row of
// the strip, so the in-place update needs no ordering between CTAs.  TMA
// brings boxes of 128 rows x 32 channels (16 KB) into a five-slot ring; a
// box stays resident while the next one is computed (its last rows are that
// box's first taps), so three boxes are in flight while one is computed.
// Warp w of 16 owns rows [8w, 8w + 8) of a box, lane l channel l: a thread
// reads its 11-row tap window from shared memory once and stores 8 outputs
// straight to HBM (a warp writes one 128-byte row segment per row).
// HBM-bound: every element is read once and written once.  The gate tasks
// are spread over the same CTAs, computed while their first boxes arrive.
// Gated norm: a warp per (row, V head), striding over the rows.

#include <cuda.h>

#include <algorithm>

#include "hb_internal.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

// ----------------------------------------------------- scalar exp and log

// Table data of the published expf / logf algorithm (Arm optimized-routines,
// the reference's src/jit/execution/math_data.rs).  kExpT[i] is
// bits(2^(i/32)) - (i << 47); kLogT[i] = {invc_i, log(1/invc_i)}.
//
// The two tables are data of Arm optimized-routines (math/exp2f_data.c,
// math/logf_data.c at revision 22bc70e01a192aaeac161143353315f051f3e647),
// used under the MIT option of its "MIT OR Apache-2.0 WITH LLVM-exception"
// licence:
//
//   Copyright (c) 1999-2022, Arm Limited.  SPDX-License-Identifier: MIT
//
//   Permission is hereby granted, free of charge, to any person obtaining a
//   copy of this software and associated documentation files (the
//   "Software"), to deal in the Software without restriction, including
//   without limitation the rights to use, copy, modify, merge, publish,
//   distribute, sublicense, and/or sell copies of the Software, and to permit
//   persons to whom the Software is furnished to do so, subject to the
//   following conditions:
//
//   The above copyright notice and this permission notice shall be included
//   in all copies or substantial portions of the Software.
//
//   THE SOFTWARE IS PROVIDED "AS IS", WITHOUT WARRANTY OF ANY KIND, EXPRESS
//   OR IMPLIED, INCLUDING BUT NOT LIMITED TO THE WARRANTIES OF
//   MERCHANTABILITY, FITNESS FOR A PARTICULAR PURPOSE AND NONINFRINGEMENT. IN
//   NO EVENT SHALL THE AUTHORS OR COPYRIGHT HOLDERS BE LIABLE FOR ANY CLAIM,
//   DAMAGES OR OTHER LIABILITY, WHETHER IN AN ACTION OF CONTRACT, TORT OR
//   OTHERWISE, ARISING FROM, OUT OF OR IN CONNECTION WITH THE SOFTWARE OR THE
//   USE OR OTHER DEALINGS IN THE SOFTWARE.
__device__ const uint64_t kExpT[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};
__device__ const uint64_t kLogT[16][2] = {
    {0x3ff661ec79f8f3beull, 0xbfd57bf7808caadeull}, {0x3ff571ed4aaf883dull, 0xbfd2bef0a7c06ddbull},
    {0x3ff49539f0f010b0ull, 0xbfd01eae7f513a67ull}, {0x3ff3c995b0b80385ull, 0xbfcb31d8a68224e9ull},
    {0x3ff30d190c8864a5ull, 0xbfc6574f0ac07758ull}, {0x3ff25e227b0b8ea0ull, 0xbfc1aa2bc79c8100ull},
    {0x3ff1bb4a4a1a343full, 0xbfba4e76ce8c0e5eull}, {0x3ff12358f08ae5baull, 0xbfb1973c5a611cccull},
    {0x3ff0953f419900a7ull, 0xbfa252f438e10c1eull}, {0x3ff0000000000000ull, 0x0000000000000000ull},
    {0x3fee608cfd9a47acull, 0x3faaa5aa5df25984ull}, {0x3feca4b31f026aa0ull, 0x3fbc5e53aa362eb4ull},
    {0x3feb2036576afce6ull, 0x3fc526e57720db08ull}, {0x3fe9c2d163a1aa2dull, 0x3fcbc2860d224770ull},
    {0x3fe886e6037841edull, 0x3fd1058bc8a07ee1ull}, {0x3fe767dcf5534862ull, 0x3fd4043057b6ee09ull}};

HB_DEV double dbits(uint64_t b) { return __longlong_as_double(static_cast<long long>(b)); }

// exp (math.rs:23-104).  |x| >= 88: -inf -> 0, NaN / +inf -> x + x,
// x > 88.72284 -> +inf, x < -103.972084 -> 0, else the core.  Core:
// z = (32/ln2) x + 1.5*2^52 fused, k = low bits of z, r = (32/ln2) x - (z -
// 1.5*2^52) fused, s = table[k % 32] with k/32 added to the exponent,
// y = ((E0 r + E1) r^2 + (E2 r + 1)) s, rounded to f32.
HB_DEV float expf_ref(float x) {
  const uint32_t ux = __float_as_uint(x), ax = ux & 0x7FFFFFFFu;
  if (ax >= 0x42B00000u) {
    if (ux == 0xFF800000u) return 0.0f;
    if (ax >= 0x7F800000u) return __fadd_rn(x, x);
    if (x > 88.72284f) return __uint_as_float(0x7F800000u);
    if (x < -103.972084f) return 0.0f;
  }
  const double inv = dbits(0x40471547652b82feull), shift = dbits(0x4338000000000000ull);
  const double xd = static_cast<double>(x);
  const double z = __fma_rn(inv, xd, shift);
  const uint64_t ki = static_cast<uint64_t>(__double_as_longlong(z));
  const double kd = __dsub_rn(z, shift);
  const double r = __fma_rn(inv, xd, -kd);
  const double s = dbits(kExpT[ki & 31] + (ki << 47));
  const double p = __fma_rn(r, dbits(0x3ebc6af84b912394ull), dbits(0x3f2ebfce50fac4f3ull));
  const double r2 = __dmul_rn(r, r);
  const double q = __fma_rn(r, dbits(0x3f962e42ff0c52d6ull), 1.0);
  return __double2float_rn(__dmul_rn(__fma_rn(p, r2, q), s));
}

// log (math.rs:114-199).  1 -> +0; outside the positive normal range:
// +-0 -> -inf, +inf -> +inf, NaN / negative -> NaN, subnormals scaled by
// 2^23.  Core: tmp = ix - 0x3f330000 gives subinterval i (bits 19..22) and
// exponent k (tmp >> 23, arithmetic); z = x 2^-k; r = z invc - 1 fused,
// y0 = k ln2 + logc fused, y = (L0 r^2 + (L1 r + L2)) r^2 + (r + y0).
HB_DEV float logf_ref(float x) {
  uint32_t ix = __float_as_uint(x);
  if (ix == 0x3F800000u) return 0.0f;
  if (ix - 0x00800000u > 0x7EFFFFFFu) {
    if (ix * 2u == 0u) return __uint_as_float(0xFF800000u);
    if (ix == 0x7F800000u) return x;
    if (ix * 2u >= 0xFF000000u || (ix & 0x80000000u)) return __uint_as_float(0x7FC00000u);
    ix = __float_as_uint(__fmul_rn(x, 8388608.0f)) - (23u << 23);
  }
  const uint32_t tmp = ix - 0x3F330000u;
  const int i = static_cast<int>((tmp >> 19) & 15u);
  const int k = static_cast<int32_t>(tmp) >> 23;
  const double z = static_cast<double>(__uint_as_float(ix - (tmp & 0xFF800000u)));
  const double r = __fma_rn(z, dbits(kLogT[i][0]), -1.0);
  const double y0 = __fma_rn(static_cast<double>(k), dbits(0x3fe62e42fefa39efull), dbits(kLogT[i][1]));
  double y = __fma_rn(r, dbits(0x3fd5575b0be00b6aull), dbits(0xbfdffffef20a4123ull));
  const double r2 = __dmul_rn(r, r);
  const double yr = __dadd_rn(r, y0);
  y = __fma_rn(r2, dbits(0xbfd00ea348b88334ull), y);
  return __double2float_rn(__fma_rn(r2, y, yr));
}

HB_DEV float neg(float x) { return __uint_as_float(__float_as_uint(x) ^ 0x80000000u); }

// SiLU of the vector kernels, g / (1 + exp(min(0 - g, 88))) with the
// polynomial exp (vminps gives 88 for NaN, as fminf), on two lanes (g0, g1),
// paired where the bits allow.
HB_DEV void silu_poly2(float g0, float g1, float& y0, float& y1) {
  const uint64_t ng = f2sub(f2(0.0f, 0.0f), f2(g0, g1));
  const uint64_t e = f2add(exp_poly2(f2(fminf(f2lo(ng), 88.0f), fminf(f2hi(ng), 88.0f))),
                           f2(1.0f, 1.0f));
  y0 = __fdiv_rn(g0, f2lo(e));
  y1 = __fdiv_rn(g1, f2hi(e));
}

// SiLU of the scalar bodies: g / (exp(-g) + 1) with the scalar exp.
HB_DEV float silu_scalar(float g) { return __fdiv_rn(g, __fadd_rn(expf_ref(neg(g)), 1.0f)); }

// --------------------------------------------------------- conv + gates

constexpr int kStrip = 32;                      // channels per CTA: one 128-byte row segment
constexpr int kRun = 8;                         // consecutive rows per thread
constexpr int kBox = 128;                       // rows per TMA box (16 KB)
constexpr int kStages = 5;                      // ring slots: computed, resident, three in flight
constexpr int kFrontThreads = kBox / kRun * 32; // 512: warp w owns rows [8w, 8w + 8) of a box
constexpr int kMaxCk = 8;

struct FrontParams {
  float* qkv;
  float* state;
  const uint16_t* weight;
  int conv, rows, ck, vec_channels, nbox, box_rows;
  const float* ab;
  const uint16_t* dt_bias;
  const float* a_log;
  float* beta;
  float* decay;
  int nv, n_tasks;
  int* status;
};

struct __align__(128) FrontSmem {
  float ring[kStages][kBox][kStrip];
  float old_state[kStrip][kMaxCk];
  uint64_t full[kStages];
  int abort;
};

// The gates of one (row, V head) from its a, b, dt_bias and a_log
// (delta.rs:290-389).
HB_DEV void gate_values(float a, float b, uint16_t dt_bias, float a_log, float& beta, float& decay) {
  beta = __fdiv_rn(1.0f, __fadd_rn(expf_ref(neg(b)), 1.0f));
  float dt = __fadd_rn(a, bf16_to_f32(dt_bias));
  if (!(dt > 20.0f)) dt = logf_ref(__fadd_rn(expf_ref(dt), 1.0f));
  decay = expf_ref(__fmul_rn(neg(expf_ref(a_log)), dt));
}

// One gate task: row task / nv, V head task % nv.
__device__ void gate_task(const FrontParams& p, int task) {
  const int row = task / p.nv, h = task - row * p.nv;
  const float* r = p.ab + static_cast<size_t>(row) * 2 * p.nv;
  gate_values(r[h], r[p.nv + h], p.dt_bias[h], p.a_log[h], p.beta[task], p.decay[task]);
}

__global__ void __launch_bounds__(kFrontThreads)
    gdn_front_kernel(const __grid_constant__ CUtensorMap tmX, const FrontParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  FrontSmem& S = *reinterpret_cast<FrontSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, l = tid % kStrip, w = tid / kStrip;
  const int c0 = blockIdx.x * kStrip, c = c0 + l;
  const bool active = c < p.conv;
  const int ck = p.ck;
  const uint32_t box_bytes = uint32_t(p.box_rows) * kStrip * 4u;

  if (tid == 0) {
    sm100::prefetch_tmap(&tmX);
    for (int s = 0; s < kStages; s++) mbar_init(&S.full[s], 1);
    fence_mbar_init();
    S.abort = 0;
    for (int j = 0; j < kStages - 1 && j < p.nbox; j++) {
      mbar_arrive_expect_tx(&S.full[j], box_bytes);
      sm100::tma_load_2d(&S.ring[j][0][0], &tmX, &S.full[j], c0, j * kBox);
    }
  }
  if (w == 0 && active)
    for (int m = 0; m < ck; m++) S.old_state[l][m] = p.state[static_cast<size_t>(c) * ck + m];
  // the gates while the first boxes arrive: task blockIdx.x * 512 + tid, strided
  for (int t = blockIdx.x * kFrontThreads + tid; t < p.n_tasks; t += gridDim.x * kFrontThreads)
    gate_task(p, t);
  __syncthreads();

  const bool vec = c < p.vec_channels;
  const uint16_t* wc = p.weight + static_cast<size_t>(active ? c : 0) * ck;
  float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f;
  if (vec) {
    w0 = bf16_to_f32(wc[0]);
    w1 = bf16_to_f32(wc[1]);
    w2 = bf16_to_f32(wc[2]);
    w3 = bf16_to_f32(wc[3]);
  }

  for (int j = 0; j < p.nbox; j++) {
    const int s = j % kStages, sp = (j + kStages - 1) % kStages;
    if (!mbar_wait(&S.full[s], (j / kStages) & 1)) S.abort = 1;
    // input x of row r of the block, r >= j*kBox - 7: this box, the
    // previous one, or the state before the block
    auto tap = [&](int r) -> float {
      if (r >= j * kBox) return S.ring[s][r - j * kBox][l];
      if (r >= 0) return S.ring[sp][r - (j - 1) * kBox][l];
      return S.old_state[l][ck + r];
    };
    const int r0 = j * kBox + w * kRun;
    const int n = min(kRun, p.rows - r0);  // rows of this run (<= 0: none)
    if (active && n > 0) {
      float* out = p.qkv + static_cast<size_t>(r0) * p.conv + c;
      if (vec) {
        // window x[r0 - 3 .. r0 + 7]: only warp 0 reaches into the previous
        // box or the state
        float x[kRun + 3];
        if (w == 0) {
#pragma unroll
          for (int t = 0; t < 3; t++) x[t] = tap(r0 - 3 + t);
        } else {
#pragma unroll
          for (int t = 0; t < 3; t++) x[t] = S.ring[s][w * kRun - 3 + t][l];
        }
#pragma unroll
        for (int t = 0; t < kRun; t++) x[3 + t] = S.ring[s][w * kRun + t][l];
        // rows t and t + 1 on paired lanes: g = (p0 + p1) + (p2 + p3)
#pragma unroll
        for (int t = 0; t < kRun; t += 2) {
          const uint64_t a = f2add(f2(__fmul_rn(x[t], w0), __fmul_rn(x[t + 1], w0)),
                                   f2(__fmul_rn(x[t + 1], w1), __fmul_rn(x[t + 2], w1)));
          const uint64_t b = f2add(f2(__fmul_rn(x[t + 2], w2), __fmul_rn(x[t + 3], w2)),
                                   f2(__fmul_rn(x[t + 3], w3), __fmul_rn(x[t + 4], w3)));
          const uint64_t g = f2add(a, b);
          float y0, y1;
          silu_poly2(f2lo(g), f2hi(g), y0, y1);
          if (t < n) out[static_cast<size_t>(t) * p.conv] = y0;
          if (t + 1 < n) out[static_cast<size_t>(t + 1) * p.conv] = y1;
        }
      } else {
        for (int t = 0; t < n; t++) {
          float acc = 0.0f;
          for (int m = 0; m < ck; m++)
            acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(wc[m]), tap(r0 + t - ck + 1 + m)));
          out[static_cast<size_t>(t) * p.conv] = silu_scalar(acc);
        }
      }
    }
    __syncthreads();
    if (S.abort) {
      if (tid == 0) {
        // leave no copy in flight into this CTA's shared memory: boxes j ..
        // j + kStages - 2 have been issued (bounded waits)
        record_status(p.status, kStatusTimeout);
        const int issued = min(p.nbox - 1, j + kStages - 2);
        for (int b = j; b <= issued; b++) mbar_wait(&S.full[b % kStages], (b / kStages) & 1);
      }
      return;
    }
    // box j - 1 is no longer needed: its slot takes box j + kStages - 1
    if (tid == 0 && j + kStages - 1 < p.nbox) {
      const int jn = j + kStages - 1;
      mbar_arrive_expect_tx(&S.full[sp], box_bytes);
      sm100::tma_load_2d(&S.ring[sp][0][0], &tmX, &S.full[sp], c0, jn * kBox);
    }
    if (j == p.nbox - 1 && w == 0 && active) {
      // the state after the block: the last ck inputs (boxes j and j - 1
      // are still resident: nothing is loaded after the last box)
      for (int m = 0; m < ck; m++) p.state[static_cast<size_t>(c) * ck + m] = tap(p.rows - ck + m);
    }
  }
}

// ------------------------------------------------------------ gated norm

constexpr int kNormThreads = 256;

struct NormParams {
  const float* x;
  const float* z;
  const uint16_t* weight;
  uint16_t* out;
  float* out_f32;
  long long n_rows;
  int dim;
  float eps;
};

// bf16x2_cvtne with the special-case fix-ups only when a value needs them
// (zero, denormal, infinite or NaN): the hardware conversion alone is the
// reference's rounding for every other value.
HB_DEV uint32_t bf16x2_cvtne_fast(float lo, float hi) {
  const uint32_t el = __float_as_uint(lo) & 0x7F800000u, eh = __float_as_uint(hi) & 0x7F800000u;
  const bool plain = el != 0u && el != 0x7F800000u && eh != 0u && eh != 0x7F800000u;
  if (__builtin_expect(plain, 1)) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  return bf16x2_cvtne(lo, hi);
}

// 1 / sqrt(sum x^2 / dim + eps) of one row in the vector kernel's order,
// dim = 16 NB (NB <= 8), every lane of the warp taking part.  Lane (l, h) =
// (lane % 16, lane / 16) enters with xv[k] = x[16 b + l], b = 2h + (k & 1) +
// 4 (k >> 1) (0 where b >= NB): zmm lane l of blocks 2h, 2h + 1, 2h + 4,
// 2h + 5, chains 2h and 2h + 1 of the sum of squares (block b feeds chain
// b % 4; absent chains stay +0, which adds exactly).  Every lane returns the
// same value.
template <int NB>
HB_DEV float norm_inverse_vec(const float (&xv)[4], float eps) {
  const int h = (threadIdx.x & 31) >> 4;
  float acc[2] = {0.0f, 0.0f};
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int b = 2 * h + (k & 1) + 4 * (k >> 1);
    if (b < NB) acc[k & 1] = __fmaf_rn(xv[k], xv[k], acc[k & 1]);
  }
  // chains added in order: ((c0 + c1) + c2) + c3, on the lanes l < 16
  const float c2 = __shfl_down_sync(0xFFFFFFFFu, acc[0], 16);
  const float c3 = __shfl_down_sync(0xFFFFFFFFu, acc[1], 16);
  float s = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), c2), c3);
  // hsum: (l, l+8), (l, l+4), then the two hadds
  s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, 8));
  s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, 4));
  s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, 1));
  s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, 2));
  s = __shfl_sync(0xFFFFFFFFu, s, 0);
  s = __fadd_rn(__fdiv_rn(s, static_cast<float>(16 * NB)), eps);
  return __fdiv_rn(1.0f, __fsqrt_rn(s));
}

// The vector kernel's form at dim = 16 NB (NB <= 8).  A warp walks rows
// (row, V head) with a stride of the grid's warps, the weights held in
// registers.  Lane (l, h) = (lane % 16, lane / 16) holds zmm lane l of
// blocks 2h, 2h + 1, 2h + 4, 2h + 5: chains 2h and 2h + 1 of the sum of
// squares (block b feeds chain b % 4; absent chains stay +0, which adds
// exactly).
template <int NB>
__global__ void __launch_bounds__(kNormThreads) gdn_gated_norm_vec(const NormParams p) {
  constexpr int dim = 16 * NB;
  const int lane = threadIdx.x & 31, l = lane & 15, h = lane >> 4;
  const long long warps = static_cast<long long>(gridDim.x) * (kNormThreads / 32);
  float wv[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int b = 2 * h + (k & 1) + 4 * (k >> 1);
    wv[k] = b < NB ? bf16_to_f32(p.weight[16 * b + l]) : 0.0f;
  }
  for (long long row = static_cast<long long>(blockIdx.x) * (kNormThreads / 32) + (threadIdx.x >> 5);
       row < p.n_rows; row += warps) {
    const size_t base = static_cast<size_t>(row) * dim;
    const float* x = p.x + base;
    const float* z = p.z + base;
    float xv[4], zv[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int b = 2 * h + (k & 1) + 4 * (k >> 1);
      xv[k] = b < NB ? x[16 * b + l] : 0.0f;
      zv[k] = b < NB ? z[16 * b + l] : 0.0f;
    }
    const float inv = norm_inverse_vec<NB>(xv, p.eps);
    // elements k and k + 1 on paired lanes (absent blocks compute on zeros
    // and are not stored)
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
      const int b0 = 2 * h + 4 * (k >> 1), b1 = b0 + 1;
      if (b0 >= NB) continue;
      float s0, s1;
      silu_poly2(zv[k], zv[k + 1], s0, s1);
      const float y0 = __fmul_rn(__fmul_rn(__fmul_rn(xv[k], inv), wv[k]), s0);
      const float y1 = __fmul_rn(__fmul_rn(__fmul_rn(xv[k + 1], inv), wv[k + 1]), s1);
      const uint32_t o = bf16x2_cvtne_fast(y0, y1);
      const int d0 = 16 * b0 + l, d1 = 16 * b1 + l;
      if (p.out_f32) p.out_f32[base + d0] = y0;
      p.out[base + d0] = static_cast<uint16_t>(o & 0xFFFFu);
      if (b1 < NB) {
        if (p.out_f32) p.out_f32[base + d1] = y1;
        p.out[base + d1] = static_cast<uint16_t>(o >> 16);
      }
    }
  }
}

// The scalar body's form (other widths), one warp per row: the sum in
// order from +0 (every lane, same bits), the scalar exp, the integer
// rounding to bf16.
__global__ void __launch_bounds__(kNormThreads) gdn_gated_norm_scalar(const NormParams p) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= p.n_rows) return;
  const int dim = p.dim;
  const size_t base = static_cast<size_t>(row) * dim;
  const float* x = p.x + base;
  const float* z = p.z + base;
  float s = 0.0f;
  for (int d = 0; d < dim; d++) s = __fadd_rn(s, __fmul_rn(x[d], x[d]));
  s = __fadd_rn(__fdiv_rn(s, static_cast<float>(dim)), p.eps);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(s));
  __syncwarp();  // every lane has read x before any lane writes y over it
  for (int d = lane; d < dim; d += 32) {
    const float silu = silu_scalar(z[d]);
    const float y = __fmul_rn(__fmul_rn(__fmul_rn(x[d], inv), bf16_to_f32(p.weight[d])), silu);
    if (p.out_f32) p.out_f32[base + d] = y;
    const uint32_t u = __float_as_uint(y);
    p.out[base + d] = static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
  }
}

// ------------------------------------------------ one-row DeltaNet layer
//
// A decode step of a whole DeltaNet layer in one launch: conv + SiLU of the
// row, the gates, the L2 step, the recurrence and the gated norm, each in
// the operation order of its own kernel above (and of the reference), so
// the results are the three-launch path's bits.  CTA h = V head h, 4 hvd
// threads: thread t < hkd owns q / k channel t of the head's key head,
// thread t < hvd v channel t.  The recurrence gives state column c to four
// threads, one per quarter of the kd rows (thread q hvd + c holds rows
// [q hkd/4, (q + 1) hkd/4) in registers): all four form their products at
// once, then the sums over kd run quarter after quarter in increasing kd,
// each continuing the previous quarter's value through shared memory -- the
// reference's order, with 32-step code (not 128) to fetch and run.
//
// The V heads of one key head read the same q / k inputs and conv state and
// compute the same conv results; the last of them to finish reading writes
// those back in place.  After its reads each CTA counts itself on the key
// head's counter (an acquire-release atomic add): the CTA that sees the count
// complete resets it and writes, when every other CTA of the key head is
// past its reads -- no CTA waits for another.  Launched with programmatic
// stream serialization: before griddepcontrol.wait only L2 prefetches (the
// state tile and the row's lines).

constexpr int kRowSubs = 4;       // threads per state column
constexpr int kRowMaxHvd = 128;

struct RowParams {
  float* qkv;                   // [conv] conv + SiLU in place
  float* conv_state;            // [conv][4]
  const uint16_t* conv_weight;  // [conv][4] bf16
  const float* ab;              // [2 nv]
  const uint16_t* dt_bias;      // [nv] bf16
  const float* a_log;           // [nv]
  const float* z;               // [nv hvd]
  const uint16_t* norm_weight;  // [hvd] bf16
  uint16_t* out;                // [nv hvd] bf16
  float* out_f32;               // [nv hvd] or nullptr
  float* state;                 // [nv][hkd][hvd] (read by the tensor map, written by bulk copies)
  unsigned* counters;           // [nk] readers of each key head's inputs (zero between calls)
  int nk, nv;
  float l2_eps, scale, norm_eps;
  int* status;
};


// (s1 w0 + s2 w1) + (s3 w2 + x w3): the vector kernel's sum at ck = 4 for a
// row whose taps are the state's last three inputs and x.
HB_DEV float conv4_sum(const float4& st, uint2 w, float x) {
  const float a = __fadd_rn(__fmul_rn(st.y, bf16lo(w.x)), __fmul_rn(st.z, bf16hi(w.x)));
  const float b = __fadd_rn(__fmul_rn(st.w, bf16lo(w.y)), __fmul_rn(x, bf16hi(w.y)));
  return __fadd_rn(a, b);
}

template <int HKD, int NB>
__global__ void __launch_bounds__(kRowSubs * 16 * NB, 1)
    gdn_row_kernel(const __grid_constant__ CUtensorMap tmS, const RowParams p) {
  constexpr int HVD = 16 * NB;
  constexpr int KS = HKD / kRowSubs;  // kd rows per thread in the recurrence
  static_assert(HKD <= kRowSubs * HVD && HVD <= kRowMaxHvd && HVD % 32 == 0 && KS % 4 == 0,
                "thread roles");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  float* st = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* qn = st + HKD * HVD;  // [HKD] q, then q inv_q scale
  float* kn = qn + HKD;        // [HKD] k, then k inv_k
  float* os = kn + HKD;        // [HVD] recurrence output
  float* vb = os + HVD;        // [HVD] v after the conv
  float* cb = vb + HVD;        // [HVD] a column's sum handed to the next quarter
  float* db = cb + HVD;        // [HVD] delta
  float* yb = db + HVD;        // [2 HKD] the conv results of q, k (written back by the last reader)
  float4* sb = reinterpret_cast<float4*>(yb + 2 * HKD);  // [2 HKD] their new conv states
  float* misc = reinterpret_cast<float*>(sb + 2 * HKD);  // inv_q, inv_k, beta, decay
  uint64_t* bar = reinterpret_cast<uint64_t*>(misc + 8);  // misc[4]: the last-reader flag

  const int tid = threadIdx.x, lane = tid & 31;
  const int h = blockIdx.x, ratio = p.nv / p.nk, kh = h / ratio;
  const int64_t key = int64_t(p.nk) * HKD;
  const int64_t cq = int64_t(kh) * HKD + tid, ck = key + cq, cv = 2 * key + int64_t(h) * HVD + tid;
  const bool has_qk = tid < HKD, has_v = tid < HVD;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    sm100::prefetch_tmap(&tmS);
    sm100::tma_prefetch_l2_2d(&tmS, 0, h * HKD);
  }
  if (has_qk && lane % 8 == 0) {  // conv state: 8 channels per line; q, k, weights a line per warp
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_state + cq * 4));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_state + ck * 4));
    if (lane == 0) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.qkv + cq));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.qkv + ck));
    }
    if (lane % 16 == 0) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_weight + cq * 4));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_weight + ck * 4));
    }
  }
  if (has_v && lane % 8 == 0) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_state + cv * 4));
    if (lane == 0) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.qkv + cv));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.z + int64_t(h) * HVD + tid));
    }
    if (lane % 16 == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_weight + cv * 4));
  }
  __syncthreads();  // the barrier's initialisation is visible
  griddep_wait();
  griddep_launch_dependents();
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, HKD * HVD * 4);
    sm100::tma_load_2d(st, &tmS, bar, 0, h * HKD);
  }

  // every load of the row
  float4 sq = make_float4(0.f, 0.f, 0.f, 0.f), sk = sq, sv = sq;
  uint2 wq = make_uint2(0u, 0u), wk = wq, wv = wq;
  float xq = 0.f, xk = 0.f, xv = 0.f, zz = 0.f, nw = 0.f;
  if (has_qk) {
    sq = *reinterpret_cast<const float4*>(p.conv_state + cq * 4);
    sk = *reinterpret_cast<const float4*>(p.conv_state + ck * 4);
    wq = *reinterpret_cast<const uint2*>(p.conv_weight + cq * 4);
    wk = *reinterpret_cast<const uint2*>(p.conv_weight + ck * 4);
    xq = p.qkv[cq];
    xk = p.qkv[ck];
  }
  if (has_v) {
    sv = *reinterpret_cast<const float4*>(p.conv_state + cv * 4);
    wv = *reinterpret_cast<const uint2*>(p.conv_weight + cv * 4);
    xv = p.qkv[cv];
    zz = p.z[int64_t(h) * HVD + tid];
    nw = bf16_to_f32(p.norm_weight[tid]);
  }
  float ga = 0.f, gb = 0.f, a_log = 0.f;
  uint16_t dtb = 0;
  if (tid == 64) {
    ga = p.ab[h];
    gb = p.ab[p.nv + h];
    dtb = p.dt_bias[h];
    a_log = p.a_log[h];
  }

  float yq = 0.f, yk = 0.f, yv = 0.f;
  if (has_qk) {
    silu_poly2(conv4_sum(sq, wq, xq), conv4_sum(sk, wk, xk), yq, yk);
    qn[tid] = yq;
    kn[tid] = yk;
    yb[tid] = yq;
    yb[HKD + tid] = yk;
    sb[tid] = make_float4(sq.y, sq.z, sq.w, xq);
    sb[HKD + tid] = make_float4(sk.y, sk.z, sk.w, xk);
  }
  if (has_v) {
    float unused;
    const float g = conv4_sum(sv, wv, xv);
    silu_poly2(g, g, yv, unused);
    vb[tid] = yv;
  }
  __syncthreads();  // every thread has consumed its loads
  // this CTA is past its reads of the key head's inputs (the answer is
  // used at the end, so nothing waits on the atomic here)
  unsigned readers_before = 0;
  if (tid == 96)  // release: the CTA's reads (ordered by the barrier) come before it
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(readers_before) : "l"(p.counters + kh) : "memory");
  if (tid == 0 || tid == 32) misc[tid >> 5] = l2_inverse<HKD>(tid == 0 ? qn : kn, p.l2_eps);
  if (tid == 64) gate_values(ga, gb, dtb, a_log, misc[2], misc[3]);
  __syncthreads();
  if (has_qk) {
    qn[tid] = __fmul_rn(__fmul_rn(qn[tid], misc[0]), p.scale);
    kn[tid] = __fmul_rn(kn[tid], misc[1]);
  }
  if (has_v) {  // this head's own v channel back in place
    p.qkv[cv] = yv;
    *reinterpret_cast<float4*>(p.conv_state + cv * 4) = make_float4(sv.y, sv.z, sv.w, xv);
  }
  const bool late = __syncthreads_or(!mbar_wait(bar, 0));  // the state tile

  if (!late) {
    const int sub = tid / HVD, col = tid % HVD;  // uniform per warp: HVD is a multiple of 32
    float sr[KS], pr[KS];
    const float4* k4 = reinterpret_cast<const float4*>(kn + sub * KS);
    const float4* q4 = reinterpret_cast<const float4*>(qn + sub * KS);
    const float decay = misc[3], beta = misc[2];
#pragma unroll
    for (int j = 0; j < KS; ++j) sr[j] = st[(sub * KS + j) * HVD + col];
    // pass 1: decay the rows, the products r k
#pragma unroll
    for (int j4 = 0; j4 < KS / 4; ++j4) {
      const float4 kk = k4[j4];
      const float kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float r = __fmul_rn(sr[4 * j4 + e], decay);
        sr[4 * j4 + e] = r;
        pr[4 * j4 + e] = __fmul_rn(r, kw[e]);
      }
    }
    // kv = S^T k, kd in increasing order across the quarters; the last one
    // forms delta
#pragma unroll 1
    for (int i = 0; i < kRowSubs; ++i) {
      if (sub == i) {
        float acc = i == 0 ? 0.f : cb[col];
#pragma unroll
        for (int j = 0; j < KS; ++j) acc = __fadd_rn(acc, pr[j]);
        if (i < kRowSubs - 1) cb[col] = acc;
        else db[col] = __fmul_rn(__fsub_rn(vb[col], acc), beta);
      }
      __syncthreads();
    }
    // pass 2: S += k delta, the products r (q scale)
    const float delta = db[col];
#pragma unroll
    for (int j4 = 0; j4 < KS / 4; ++j4) {
      const float4 kk = k4[j4], qq = q4[j4];
      const float kw[4] = {kk.x, kk.y, kk.z, kk.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float r = __fadd_rn(sr[4 * j4 + e], __fmul_rn(kw[e], delta));
        sr[4 * j4 + e] = r;
        pr[4 * j4 + e] = __fmul_rn(r, qw[e]);
      }
    }
    // this quarter's new state rows back into the tile and out by one bulk
    // copy (its KS rows are contiguous in both), in flight during the sums
#pragma unroll
    for (int j = 0; j < KS; ++j) st[(sub * KS + j) * HVD + col] = sr[j];
    sm100::fence_proxy_async_smem();
    asm volatile("bar.sync %0, %1;" ::"r"(1 + sub), "r"(HVD) : "memory");  // the quarter's warps
    if (col == 0) {
      sm100::bulk_s2g(p.state + (int64_t(h) * HKD + sub * KS) * HVD, st + sub * KS * HVD,
                      uint32_t(KS * HVD * 4));
      sm100::tma_store_commit();
    }
    // out = S^T (q scale), in the same order
#pragma unroll 1
    for (int i = 0; i < kRowSubs; ++i) {
      if (sub == i) {
        float acc = i == 0 ? 0.f : cb[col];
#pragma unroll
        for (int j = 0; j < KS; ++j) acc = __fadd_rn(acc, pr[j]);
        if (i < kRowSubs - 1) cb[col] = acc;
        else os[col] = acc;
      }
      __syncthreads();
    }
    // the gated norm: every warp forms the row's inverse (the same bits)
    // and finishes its own columns
    float xs[4];
    const int l = lane & 15, hh = lane >> 4;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int b = 2 * hh + (k & 1) + 4 * (k >> 1);
      xs[k] = b < NB ? os[16 * b + l] : 0.0f;
    }
    const float inv = norm_inverse_vec<NB>(xs, p.norm_eps);
    if (has_v) {
      float s0, s1;
      silu_poly2(zz, zz, s0, s1);
      const float y = __fmul_rn(__fmul_rn(__fmul_rn(os[tid], inv), nw), s0);
      const int64_t o = int64_t(h) * HVD + tid;
      if (p.out_f32) p.out_f32[o] = y;
      p.out[o] = static_cast<uint16_t>(bf16x2_cvtne_fast(y, y) & 0xFFFFu);
    }
    if (col == 0) sm100::tma_store_wait_read();  // the tile stays until the copy has read it
  } else if (tid == 0) {
    // the state and the outputs are not written (the conv results are, as
    // the three-launch path's front end would have written them)
    record_status(p.status, kStatusTimeout);
    mbar_wait(bar, 0);  // a second bounded wait for the copy in flight
  }
  // the last reader of the key head's inputs writes the conv results back
  // and leaves the counter at zero for the next call
  int* last = reinterpret_cast<int*>(misc + 4);
  if (tid == 96) {
    const bool is_last = readers_before == unsigned(ratio - 1);
    if (is_last) p.counters[kh] = 0u;
    *last = is_last;
  }
  __syncthreads();
  if (*last && has_qk) {
    p.qkv[cq] = yb[tid];
    p.qkv[ck] = yb[HKD + tid];
    *reinterpret_cast<float4*>(p.conv_state + cq * 4) = sb[tid];
    *reinterpret_cast<float4*>(p.conv_state + ck * 4) = sb[HKD + tid];
  }
}

}  // namespace

bool gdn_front_serves(int64_t conv, int64_t ck) {
  return ck >= 1 && ck <= kMaxCk && conv > 0 && conv % 4 == 0;
}

cudaError_t launch_gdn_front(const GdnFrontLaunch& L, cudaStream_t st) {
  FrontParams p;
  p.qkv = L.qkv;
  p.state = L.state;
  p.weight = L.weight;
  p.conv = static_cast<int>(L.conv);
  p.rows = static_cast<int>(L.rows);
  p.ck = static_cast<int>(L.ck);
  p.vec_channels = L.ck == 4 ? static_cast<int>(L.conv / 16 * 16) : 0;
  p.box_rows = static_cast<int>(L.rows < kBox ? L.rows : kBox);
  p.nbox = static_cast<int>((L.rows + kBox - 1) / kBox);
  const int n_strips = static_cast<int>((L.conv + kStrip - 1) / kStrip);
  p.ab = L.ab;
  p.dt_bias = L.dt_bias;
  p.a_log = L.a_log;
  p.beta = L.beta;
  p.decay = L.decay;
  p.nv = static_cast<int>(L.nv);
  p.n_tasks = static_cast<int>(L.rows * L.nv);
  p.status = L.status;
  CUtensorMap tm;
  if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.qkv, uint64_t(L.rows), uint64_t(L.conv),
                 uint64_t(L.conv), uint32_t(p.box_rows), kStrip, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const size_t smem = sizeof(FrontSmem) + 1024;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(gdn_front_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr = true;
  }
  gdn_front_kernel<<<n_strips, kFrontThreads, smem, st>>>(tm, p);
  return cudaGetLastError();
}

bool gdn_row_serves(const hb_gdn_shape& s, int64_t ck) {
  return ck == 4 && (s.hkd == 64 || s.hkd == 128) && s.hvd % 32 == 0 && s.hvd >= 32 &&
         s.hvd <= kRowMaxHvd && s.nk > 0 && s.nk <= kRowMaxKeyHeads && s.nv % s.nk == 0;
}

namespace {
template <int HKD, int NB>
cudaError_t launch_row(const CUtensorMap& tm, const RowParams& p, cudaLaunchConfig_t cfg) {
  constexpr int HVD = 16 * NB;
  const size_t smem = 1024 + size_t(HKD) * HVD * 4 + (2 * HKD + 4 * HVD + 2 * HKD + 8 * HKD + 8) * 4 + 8;
  static bool attr = false;  // one flag per instantiation
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(gdn_row_kernel<HKD, NB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attr = true;
  }
  cfg.blockDim = dim3(kRowSubs * HVD);
  cfg.dynamicSmemBytes = smem;
  return cudaLaunchKernelEx(&cfg, gdn_row_kernel<HKD, NB>, tm, p);
}
}  // namespace

cudaError_t launch_gdn_row(const GdnRowLaunch& L, cudaStream_t st) {
  RowParams p;
  p.qkv = L.qkv;
  p.conv_state = L.conv_state;
  p.conv_weight = L.conv_weight;
  p.ab = L.ab;
  p.dt_bias = L.dt_bias;
  p.a_log = L.a_log;
  p.z = L.z;
  p.norm_weight = L.norm_weight;
  p.out = L.out;
  p.out_f32 = L.out_f32;
  p.state = L.state;
  p.counters = L.counters;
  p.nk = int(L.shape.nk);
  p.nv = int(L.shape.nv);
  p.l2_eps = L.l2_eps;
  p.scale = L.scale;
  p.norm_eps = L.norm_eps;
  p.status = L.status;
  // the state as [nv*hkd rows][hvd columns] f32, one [hkd][hvd] tile per V head
  CUtensorMap tm;
  if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.state, uint64_t(L.shape.nv) * L.shape.hkd,
                 uint64_t(L.shape.hvd), uint64_t(L.shape.hvd), uint32_t(L.shape.hkd),
                 uint32_t(L.shape.hvd), CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(L.shape.nv));
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int nb = int(L.shape.hvd / 16);
  if (L.shape.hkd == 128) {
    switch (nb) {
      case 2: return launch_row<128, 2>(tm, p, cfg);
      case 4: return launch_row<128, 4>(tm, p, cfg);
      case 6: return launch_row<128, 6>(tm, p, cfg);
      case 8: return launch_row<128, 8>(tm, p, cfg);
    }
  } else if (L.shape.hkd == 64) {
    switch (nb) {
      case 2: return launch_row<64, 2>(tm, p, cfg);
      case 4: return launch_row<64, 4>(tm, p, cfg);
      case 6: return launch_row<64, 6>(tm, p, cfg);
      case 8: return launch_row<64, 8>(tm, p, cfg);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gdn_gated_norm(const GdnNormLaunch& L, cudaStream_t st) {
  NormParams p;
  p.x = L.x;
  p.z = L.z;
  p.weight = L.weight;
  p.out = L.out;
  p.out_f32 = L.out_f32;
  p.n_rows = L.rows * L.nv;
  p.dim = static_cast<int>(L.hvd);
  p.eps = L.eps;
  const long long warps = kNormThreads / 32;
  long long ctas = (p.n_rows + warps - 1) / warps;
  if (p.dim % 16 == 0 && p.dim <= 128) {
    // a resident grid (eight CTAs per SM) whose warps stride over the rows
    static int sms = 0;
    if (!sms) {
      int dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (sms <= 0) sms = 148;
    }
    ctas = std::min<long long>(ctas, 8LL * sms);
    switch (p.dim / 16) {
      case 1: gdn_gated_norm_vec<1><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
      case 2: gdn_gated_norm_vec<2><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
      case 3: gdn_gated_norm_vec<3><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
      case 4: gdn_gated_norm_vec<4><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
      case 5: gdn_gated_norm_vec<5><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
      case 6: gdn_gated_norm_vec<6><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
      case 7: gdn_gated_norm_vec<7><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
      default: gdn_gated_norm_vec<8><<<unsigned(ctas), kNormThreads, 0, st>>>(p); break;
    }
  } else {
    gdn_gated_norm_scalar<<<static_cast<unsigned>(ctas), kNormThreads, 0, st>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace hb
