// gdn_decode.cu -- the GatedDeltaNet recurrence on sm_100a, position by
// position, with the reference's non-FMA rounding order.
//
// Replaces the delta-causal-recurrence node (RecurrenceFn,
// src/jit/emit_recurrence.rs:63-73; x86 src/jit/target/x86/emit_recurrence.rs:108-217;
// traversal src/jit/target/x86/execution/delta.rs:519-607) and the L2 step of
// delta-l2-gates (delta.rs:28-62, 442-515).
//
// Column vd of a head's state only ever meets column vd: kv[vd], delta[vd]
// and out[vd] are sums over kd of one column.  So one thread owns one state
// column for the whole call, holds its hkd values in registers, and runs the
// kd sums in increasing order with separate multiply and add (__fmul_rn /
// __fadd_rn): the outputs and the state are the reference's bits.  Grid =
// (value heads, hvd/32), one warp per CTA; the state crosses HBM once per
// call however many positions the call carries.
#include <cstdint>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_internal.h"

namespace hb {
namespace {

struct GdnParams {
  float* state;
  float* out;
  const float* qkv;
  const float* beta;
  const float* decay;
  int64_t rows;
  int nk, nv, hvd;
  int l2;
  float eps, scale;
};

// Sequential L2 of one head held in shared memory: sum of squares left to
// right, + eps, sqrt, 1/x (delta.rs:28-62).
template <int N>
HB_DEV float l2_inverse(const float* x, float eps) {
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) sum = __fadd_rn(sum, __fmul_rn(x[i], x[i]));
  sum = __fadd_rn(sum, eps);
  return __fdiv_rn(1.0f, __fsqrt_rn(sum));
}

template <int HKD>
__global__ void __launch_bounds__(32) gdn_decode_kernel(const GdnParams p) {
  __shared__ __align__(16) float qn[HKD];
  __shared__ __align__(16) float kn[HKD];
  __shared__ float inv[2];
  const int h = blockIdx.x, lane = threadIdx.x;
  const int col = blockIdx.y * 32 + lane;
  const int kh = h / (p.nv / p.nk);
  const int64_t key = int64_t(p.nk) * HKD, value = int64_t(p.nv) * p.hvd;
  const int64_t conv = 2 * key + value;

  float* sp = p.state + int64_t(h) * HKD * p.hvd + col;
  float s[HKD];
#pragma unroll
  for (int kd = 0; kd < HKD; ++kd) s[kd] = sp[int64_t(kd) * p.hvd];

  for (int64_t t = 0; t < p.rows; ++t) {
    const float* row = p.qkv + t * conv;
#pragma unroll
    for (int i = lane; i < HKD; i += 32) {
      qn[i] = row[int64_t(kh) * HKD + i];
      kn[i] = row[key + int64_t(kh) * HKD + i];
    }
    __syncwarp();
    if (p.l2) {
      if (lane < 2) inv[lane] = l2_inverse<HKD>(lane == 0 ? qn : kn, p.eps);
      __syncwarp();
      const float iq = inv[0], ik = inv[1];
#pragma unroll
      for (int i = lane; i < HKD; i += 32) {
        qn[i] = __fmul_rn(qn[i], iq);
        kn[i] = __fmul_rn(kn[i], ik);
      }
      __syncwarp();
    }
    const float beta = p.beta[t * p.nv + h];
    const float decay = p.decay[t * p.nv + h];
    const float v = row[2 * key + int64_t(h) * p.hvd + col];

    // pass 1: decay, then read kv = S^T k
    float kv = 0.f;
#pragma unroll
    for (int kd = 0; kd < HKD; ++kd) {
      const float r = __fmul_rn(s[kd], decay);
      s[kd] = r;
      kv = __fadd_rn(kv, __fmul_rn(r, kn[kd]));
    }
    const float delta = __fmul_rn(__fsub_rn(v, kv), beta);
    // pass 2: write S += k delta, read out = S^T (q scale)
    float o = 0.f;
#pragma unroll
    for (int kd = 0; kd < HKD; ++kd) {
      const float qs = __fmul_rn(qn[kd], p.scale);
      const float r = __fadd_rn(s[kd], __fmul_rn(kn[kd], delta));
      s[kd] = r;
      o = __fadd_rn(o, __fmul_rn(r, qs));
    }
    p.out[t * value + int64_t(h) * p.hvd + col] = o;
    __syncwarp();
  }
#pragma unroll
  for (int kd = 0; kd < HKD; ++kd) sp[int64_t(kd) * p.hvd] = s[kd];
}

}  // namespace

bool gdn_decode_serves(const hb_gdn_shape& s) {
  return (s.hkd == 64 || s.hkd == 128) && s.hvd > 0 && s.hvd % 32 == 0 && s.hvd <= 512;
}

cudaError_t launch_gdn_decode(const GdnLaunch& L, cudaStream_t st) {
  GdnParams p;
  p.state = L.call.state;
  p.out = L.call.output;
  p.qkv = L.call.qkv;
  p.beta = L.call.beta;
  p.decay = L.call.decay;
  p.rows = L.call.rows;
  p.nk = int(L.shape.nk);
  p.nv = int(L.shape.nv);
  p.hvd = int(L.shape.hvd);
  p.l2 = L.call.l2;
  p.eps = L.call.eps;
  p.scale = L.scale;
  dim3 grid(unsigned(L.shape.nv), unsigned(L.shape.hvd / 32));
  if (L.shape.hkd == 128) gdn_decode_kernel<128><<<grid, 32, 0, st>>>(p);
  else if (L.shape.hkd == 64) gdn_decode_kernel<64><<<grid, 32, 0, st>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace hb
