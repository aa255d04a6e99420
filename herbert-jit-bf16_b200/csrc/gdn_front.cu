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
// the results are the three-launch path's bits.
//
// A step is a chain of latencies: the row's inputs, the two L2 sums, pass 1
// (kv) and pass 2 (out) of the recurrence, each a sequential sum of hkd
// terms, then the gated norm over the head's hvd outputs.  So each V head is
// a cluster of hvd / 32 CTAs, CTA c owning the state columns [32 c, 32 c +
// 32), and every CTA runs the head's front end itself.  A warp that only
// adds issues about four cycles per term of such a sum, one that also forms
// the terms (two or three multiplies, a store in pass 2) about ten, so the
// terms are formed by other warps:
//   warp 0        the v channels of its columns (conv + SiLU), then only
//                 sums: the q / k L2 sums (lanes 0 / 1, over the squares the
//                 row warps wrote), kv and out of its 32 columns, reading
//                 each group of terms while the previous group is summed;
//   row warps     warp 1 + w: q / k channel 32 w + lane of the key head (conv
//                 + SiLU, the squares), and the state rows 8 (NR g + w) ..
//                 + 8 (g = 0 .. 3) of the CTA's 32 columns, loaded straight
//                 into registers; for each pass and group g, the terms of
//                 those 8 rows (pass 2: also the new rows, stored once the
//                 terms are out), published by named barrier 1 + g;
//   the last warp the gates, then the key head's reader count.
// The gated norm needs the head's whole output row: each CTA stores its 32
// outputs into every CTA of the cluster with st.async, counted on the
// receiver's mbarrier (no cluster barrier on the path), and every CTA forms
// the same norm and finishes its own columns.
//
// The CTAs of one key head read the same q / k inputs and conv state and
// compute the same conv results; the last of them to finish reading writes
// those back in place.  The last warp counts the CTA on the key head's
// counter once the row warps are past their reads (an acquire-release atomic
// add, off the recurrence's path); the CTA that sees the count complete
// resets it, and its row warps write, when every other CTA of the key head
// is past its reads -- no CTA waits for another.  Launched with
// programmatic stream serialization: before griddepcontrol.wait only L2
// prefetches.

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
  float* state;                 // [nv][hkd][hvd]
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

// Named barriers of the row kernel (0 is __syncthreads):
//   1 .. 4     a group of rows' terms published (row warps arrive, warp 0 waits)
//   kRowFront  q, k and their squares written (row warps arrive, warp 0 waits)
//   kRowInv    the L2 inverses (warp 0) and the gates (the last warp) in misc
//              (they arrive, the row warps wait)
//   kRowDelta  delta in ds (warp 0 arrives, the row warps wait)
//   kRowRead   the row warps are past their reads (they arrive, the last warp waits)
//   kRowLast   the count's answer is in `last` (the last warp arrives, the row warps wait)
constexpr int kRowFront = 5, kRowInv = 6, kRowDelta = 7, kRowRead = 8, kRowLast = 9;
// The address of `local`'s counterpart in cluster CTA `rank`.
HB_DEV uint32_t peer_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
// A store into a cluster CTA's shared memory whose 4 bytes count on that
// CTA's mbarrier (complete_tx).
HB_DEV void st_peer_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(addr),
               "f"(v), "r"(bar)
               : "memory");
}

template <int HKD, int NB>
__global__ void __launch_bounds__(HKD + 64, 1) gdn_row_kernel(const RowParams p) {
  constexpr int HVD = 16 * NB;
  constexpr int QC = HVD / 32;        // CTAs of a V head's cluster
  constexpr int NR = HKD / 32;        // q / k warps, which also hold the state rows
  constexpr int LAST = NR + 1;        // the gates / counting warp
  constexpr int NG = 4;               // groups of rows (named barriers 1 .. 4)
  constexpr int GR = HKD / NG;        // rows per group: an 8-row block of every row warp
  constexpr int NT = HKD + 32;        // row warps and warp 0 (or the last warp)
  static_assert(HVD <= kRowMaxHvd && HVD % 32 == 0 && HKD % 32 == 0 && HKD >= 64 && GR == 8 * NR,
                "thread roles");
  __shared__ __align__(16) float qraw[HKD];       // q, k after the conv
  __shared__ __align__(16) float kraw[HKD];
  __shared__ __align__(16) float sqs[2][HKD];     // their squares
  __shared__ __align__(16) float4 terms[HKD / 4][32];
  __shared__ float os[HVD];                       // the head's recurrence outputs (every CTA's columns)
  __shared__ float misc[4];                       // inv_q, inv_k, decay, beta
  __shared__ float ds[32];                        // delta per column
  __shared__ __align__(8) uint64_t os_bar;        // the cluster's outputs have landed in os
  __shared__ int last;                            // this CTA is the key head's last reader

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t crank;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  const int h = blockIdx.x / QC, col = int(crank) * 32 + lane;
  const int ratio = p.nv / p.nk, kh = h / ratio;
  const int64_t key = int64_t(p.nk) * HKD;
  const int ch = tid - 32;  // q / k channel of the row warps
  const int64_t cq = int64_t(kh) * HKD + ch, ck = key + cq, cv = 2 * key + int64_t(h) * HVD + col;
  float* scol = p.state + int64_t(h) * HKD * HVD + col;  // state column col: row kd at kd * HVD

  if (tid == 0) {
    mbar_init(&os_bar, 1);
    mbar_arrive_expect_tx(&os_bar, (QC - 1) * 32 * 4);  // the other CTAs' outputs
    fence_mbar_init();
  }
  __syncthreads();
  // this CTA's barrier is set: warp 0 waits for the whole cluster before its
  // first store into a peer
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  if (warp == 0) {  // ---------------------------------- v channels, the sums
    if (lane % 8 == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_state + cv * 4));
    if (lane % 16 == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_weight + cv * 4));
    if (lane == 0) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.qkv + cv));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.z + int64_t(h) * HVD + col));
    }
    griddep_wait();
    griddep_launch_dependents();
    const float4 sv = *reinterpret_cast<const float4*>(p.conv_state + cv * 4);
    const uint2 wv = *reinterpret_cast<const uint2*>(p.conv_weight + cv * 4);
    const float xv = p.qkv[cv];
    const float zz = p.z[int64_t(h) * HVD + col];
    const float nw = bf16_to_f32(p.norm_weight[col]);
    float v, sz;
    silu_poly2(conv4_sum(sv, wv, xv), zz, v, sz);  // the v channel; SiLU(z) of the norm's gate
    // this CTA's own v channel back in place
    p.qkv[cv] = v;
    *reinterpret_cast<float4*>(p.conv_state + cv * 4) = make_float4(sv.y, sv.z, sv.w, xv);
    named_sync(kRowFront, NT);  // q, k and their squares in shared memory
    if (lane < 2) {  // lanes 0 / 1: the squares of q / k summed in order, 32 at a time
      const float4* x4 = reinterpret_cast<const float4*>(sqs[lane]);
      float sum = 0.f;
#pragma unroll
      for (int b = 0; b < HKD / 32; ++b) {
        float4 r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = x4[8 * b + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          sum = __fadd_rn(sum, r[j].x);
          sum = __fadd_rn(sum, r[j].y);
          sum = __fadd_rn(sum, r[j].z);
          sum = __fadd_rn(sum, r[j].w);
        }
      }
      sum = __fadd_rn(sum, p.l2_eps);
      misc[lane] = __fdiv_rn(1.0f, __fsqrt_rn(sum));
    }
    __syncwarp();
    named_arrive(kRowInv, NT + 32);
    // kv = S^T k; delta; out = S^T (q scale): kd ascending, the row warps'
    // terms a group at a time
    const float kv = sum_terms<NG, GR>(terms, lane, NT);
    ds[lane] = __fmul_rn(__fsub_rn(v, kv), misc[3]);
    named_arrive(kRowDelta, NT);
    const float o = sum_terms<NG, GR>(terms, lane, NT);
    // the 32 outputs into os of this CTA and of every other CTA of the cluster
    os[col] = o;
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
#pragma unroll
    for (int r = 0; r < QC; ++r)
      if (r != int(crank))
        st_peer_f32(peer_addr(&os[col], uint32_t(r)), o, peer_addr(&os_bar, uint32_t(r)));
    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&os_bar, 0))) {  // the outputs are not written
      if (lane == 0) record_status(p.status, kStatusTimeout);
      return;
    }
    __syncwarp();  // the warp's own os entries
    // the gated norm: the row's inverse (every CTA forms the same bits),
    // then this CTA's columns
    float xs[4];
    const int l = lane & 15, hh = lane >> 4;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int b = 2 * hh + (k & 1) + 4 * (k >> 1);
      xs[k] = b < NB ? os[16 * b + l] : 0.0f;
    }
    const float inv = norm_inverse_vec<NB>(xs, p.norm_eps);
    const float y = __fmul_rn(__fmul_rn(__fmul_rn(o, inv), nw), sz);
    const int64_t oi = int64_t(h) * HVD + col;
    if (p.out_f32) p.out_f32[oi] = y;
    p.out[oi] = static_cast<uint16_t>(bf16x2_cvtne_fast(y, y) & 0xFFFFu);
    return;
  }

  if (warp == LAST) {  // ------------------------------ gates, reader count
    if (lane == 0) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.ab + h));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.ab + p.nv + h));
    }
    griddep_wait();
    griddep_launch_dependents();
    if (lane == 0) gate_values(p.ab[h], p.ab[p.nv + h], p.dt_bias[h], p.a_log[h], misc[3], misc[2]);
    __syncwarp();
    named_arrive(kRowInv, NT + 32);
    named_sync(kRowRead, NT);  // the row warps are past their reads of the key head's inputs
    if (lane == 0) {
      unsigned before;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                   : "=r"(before) : "l"(p.counters + kh) : "memory");
      const bool is_last = before == unsigned(ratio * QC - 1);
      if (is_last) p.counters[kh] = 0u;  // zero for the next call
      last = is_last;
    }
    named_arrive(kRowLast, NT);
    return;
  }

  // ----------------------------------------------------------- row warps
  const int w = warp - 1;
#pragma unroll
  for (int g = 0; g < NG; ++g)  // the state rows' lines (lanes 0..7: the 8 rows of block g)
    if (lane < 8) asm volatile("prefetch.global.L2 [%0];" ::"l"(scol - lane + (8 * (NR * g + w) + lane) * HVD));
  if (lane % 8 == 0) {  // conv state: 8 channels per line; q, k, weights a line per warp
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
  griddep_wait();
  griddep_launch_dependents();
  const float4 sq = *reinterpret_cast<const float4*>(p.conv_state + cq * 4);
  const float4 sk = *reinterpret_cast<const float4*>(p.conv_state + ck * 4);
  const uint2 wq = *reinterpret_cast<const uint2*>(p.conv_weight + cq * 4);
  const uint2 wk = *reinterpret_cast<const uint2*>(p.conv_weight + ck * 4);
  const float xq = p.qkv[cq], xk = p.qkv[ck];
  float s[NG * 8];  // state rows 8 (NR g + w) + e of column col
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) s[8 * g + e] = scol[(8 * (NR * g + w) + e) * HVD];
  float yq, yk;
  silu_poly2(conv4_sum(sq, wq, xq), conv4_sum(sk, wk, xk), yq, yk);
  qraw[ch] = yq;
  kraw[ch] = yk;
  sqs[0][ch] = __fmul_rn(yq, yq);
  sqs[1][ch] = __fmul_rn(yk, yk);
  named_arrive(kRowRead, NT);   // past the reads of the key head's inputs
  named_arrive(kRowFront, NT);  // q, k, squares written
  named_sync(kRowInv, NT + 32); // the inverses (warp 0) and the gates (the last warp)
  const float iq = misc[0], ik = misc[1], decay = misc[2];
  float kn[NG * 8], qn[NG * 8];  // this warp's rows of k inv_k and q inv_q scale
  // pass 1: the decayed rows and their terms r k
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int kd0 = 8 * (NR * g + w);
    float tm[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      kn[8 * g + e] = __fmul_rn(kraw[kd0 + e], ik);
      const float r = __fmul_rn(s[8 * g + e], decay);
      s[8 * g + e] = r;
      tm[e] = __fmul_rn(r, kn[8 * g + e]);
    }
    terms[kd0 / 4][lane] = make_float4(tm[0], tm[1], tm[2], tm[3]);
    terms[kd0 / 4 + 1][lane] = make_float4(tm[4], tm[5], tm[6], tm[7]);
    named_arrive(1 + g, NT);
  }
#pragma unroll
  for (int g = 0; g < NG; ++g)  // q inv_q scale (two roundings) while warp 0 sums
#pragma unroll
    for (int e = 0; e < 8; ++e)
      qn[8 * g + e] = __fmul_rn(__fmul_rn(qraw[8 * (NR * g + w) + e], iq), p.scale);
  named_sync(kRowDelta, NT);  // warp 0 has summed pass 1's terms
  const float delta = ds[lane];
  // pass 2: the new rows S + k delta and their terms r (q scale); the
  // group's rows stored once its terms are out
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int kd0 = 8 * (NR * g + w);
    float tm[8], rn[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      rn[e] = __fadd_rn(s[8 * g + e], __fmul_rn(kn[8 * g + e], delta));
      tm[e] = __fmul_rn(rn[e], qn[8 * g + e]);
    }
    terms[kd0 / 4][lane] = make_float4(tm[0], tm[1], tm[2], tm[3]);
    terms[kd0 / 4 + 1][lane] = make_float4(tm[4], tm[5], tm[6], tm[7]);
    named_arrive(1 + g, NT);
#pragma unroll
    for (int e = 0; e < 8; ++e) scol[(kd0 + e) * HVD] = rn[e];
  }
  // the last reader of the key head's inputs writes the conv results back
  named_sync(kRowLast, NT);
  if (last) {
    p.qkv[cq] = yq;
    p.qkv[ck] = yk;
    *reinterpret_cast<float4*>(p.conv_state + cq * 4) = make_float4(sq.y, sq.z, sq.w, xq);
    *reinterpret_cast<float4*>(p.conv_state + ck * 4) = make_float4(sk.y, sk.z, sk.w, xk);
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
cudaError_t launch_row(const RowParams& p, cudaLaunchConfig_t cfg) {
  constexpr int QC = NB / 2;  // hvd / 32 CTAs per V head
  cfg.gridDim = dim3(unsigned(p.nv * QC));
  cfg.blockDim = dim3(HKD + 64);
  cfg.dynamicSmemBytes = 0;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = QC;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gdn_row_kernel<HKD, NB>, p);
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
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  const int nb = int(L.shape.hvd / 16);
  if (L.shape.hkd == 128) {
    switch (nb) {
      case 2: return launch_row<128, 2>(p, cfg);
      case 4: return launch_row<128, 4>(p, cfg);
      case 6: return launch_row<128, 6>(p, cfg);
      case 8: return launch_row<128, 8>(p, cfg);
    }
  } else if (L.shape.hkd == 64) {
    switch (nb) {
      case 2: return launch_row<64, 2>(p, cfg);
      case 4: return launch_row<64, 4>(p, cfg);
      case 6: return launch_row<64, 6>(p, cfg);
      case 8: return launch_row<64, 8>(p, cfg);
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
    ctas = std::min<long long>(ctas, 8LL * device_sms());
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
