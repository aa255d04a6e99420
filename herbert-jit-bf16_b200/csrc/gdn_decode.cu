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
//
// The CTA's state slice [hkd rows][32 columns] f32 moves as one TMA tile
// each way (shared memory in between): with one warp per SM, per-thread
// loads of 128 strided rows left the step latency-bound on memory
// parallelism (a loads-and-stores-only kernel took 9 us per step, the TMA
// tile takes one request).  The first position's L2 norms run while the
// tile is in flight.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_internal.h"
#include "hb_sm100.cuh"

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
  int* status;  // device status word: the caller's workspace or the per-device word
};

template <int HKD>
__global__ void __launch_bounds__(32)
    gdn_decode_kernel(const __grid_constant__ CUtensorMap tmS, const GdnParams p) {
  __shared__ __align__(128) float st[HKD * 32];  // state rows kd, columns col0..col0+31
  __shared__ __align__(16) float qn[HKD];
  __shared__ __align__(16) float kn[HKD];
  __shared__ float inv[2];
  __shared__ __align__(8) uint64_t bar;
  const int h = blockIdx.x, lane = threadIdx.x;
  const int col0 = blockIdx.y * 32, col = col0 + lane;
  const int kh = h / (p.nv / p.nk);
  const int64_t key = int64_t(p.nk) * HKD, value = int64_t(p.nv) * p.hvd;
  const int64_t conv = 2 * key + value;

  if (lane == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    sm100::prefetch_tmap(&tmS);
  }
  // Launched with programmatic stream serialization: the CTAs are made
  // resident while the previous kernel finishes, and until
  // griddepcontrol.wait they only prefetch into L2 (the state tile and the
  // first position's lines; a prefetch cannot change what a later load
  // returns).  Every load follows the wait: the previous kernel may be the
  // front end that writes qkv, beta and decay.
  {
    const float* row = p.qkv;
    if (lane == 0) sm100::tma_prefetch_l2_2d(&tmS, col0, h * HKD);
    if (lane < HKD / 32) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(row + int64_t(kh) * HKD + lane * 32));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(row + key + int64_t(kh) * HKD + lane * 32));
    }
    if (lane == 4) asm volatile("prefetch.global.L2 [%0];" ::"l"(row + 2 * key + int64_t(h) * p.hvd + col0));
    if (lane == 5) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.beta + h));
    if (lane == 6) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.decay + h));
  }
  __syncwarp();
  griddep_wait();
  griddep_launch_dependents();
  if (lane == 0) {  // the state tile, in flight while the first position's norms run
    mbar_arrive_expect_tx(&bar, HKD * 32 * 4);
    sm100::tma_load_2d(st, &tmS, &bar, col0, h * HKD);
  }
  bool loaded = false;
  float s[HKD];

  for (int64_t t = 0; t < p.rows; ++t) {
    const float* row = p.qkv + t * conv;
    // every load of the position first, so their latencies overlap
    const float beta = p.beta[t * p.nv + h];
    const float decay = p.decay[t * p.nv + h];
    const float v = row[2 * key + int64_t(h) * p.hvd + col];
#pragma unroll
    for (int i = lane; i < HKD; i += 32) {
      qn[i] = row[int64_t(kh) * HKD + i];
      kn[i] = row[key + int64_t(kh) * HKD + i];
    }
    __syncwarp();
    // qn <- q * inv_q * scale (the reference scales q inside pass 2, per
    // element, after the L2 step: the same two roundings), kn <- k * inv_k
    float iq = 1.f, ik = 1.f;
    if (p.l2) {
      if (lane < 2) inv[lane] = l2_inverse<HKD>(lane == 0 ? qn : kn, p.eps);
      __syncwarp();
      iq = inv[0];
      ik = inv[1];
    }
#pragma unroll
    for (int i = lane; i < HKD; i += 32) {
      const float qv = p.l2 ? __fmul_rn(qn[i], iq) : qn[i];
      qn[i] = __fmul_rn(qv, p.scale);
      if (p.l2) kn[i] = __fmul_rn(kn[i], ik);
    }
    __syncwarp();
    if (!loaded) {  // the state tile (first position only)
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bar, 0))) {
        // the call's outputs are not written; the status word tells the caller
        if (lane == 0) record_status(p.status, kStatusTimeout);
        mbar_wait(&bar, 0);  // a second bounded wait for the copy in flight
        return;
      }
#pragma unroll
      for (int kd = 0; kd < HKD; ++kd) s[kd] = st[kd * 32 + lane];
      loaded = true;
    }

    const float o = gdn_step_column<HKD>(s, kn, qn, v, beta, decay);
    p.out[t * value + int64_t(h) * p.hvd + col] = o;
    __syncwarp();
  }
  if (!loaded) {  // no position (the host refuses empty calls): state untouched
    mbar_wait(&bar, 0);  // the copy in flight lands before the CTA ends (bounded)
    return;
  }
#pragma unroll
  for (int kd = 0; kd < HKD; ++kd) st[kd * 32 + lane] = s[kd];
  sm100::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    sm100::tma_store_2d(&tmS, st, col0, h * HKD);
    sm100::tma_store_commit();
    sm100::tma_store_wait_read();
  }
  __syncwarp();
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
  p.status = L.status;
  // the state as [nv*hkd rows][hvd columns] f32, tiles [hkd rows][32 columns]
  CUtensorMap tm;
  if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.call.state,
                 uint64_t(L.shape.nv) * L.shape.hkd, uint64_t(L.shape.hvd), uint64_t(L.shape.hvd),
                 uint32_t(L.shape.hkd), 32, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  // programmatic dependent launch: the CTAs of consecutive steps are made
  // resident while the previous step finishes (griddepcontrol.wait in the
  // kernel orders every memory access after it)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(L.shape.nv), unsigned(L.shape.hvd / 32));
  cfg.blockDim = dim3(32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (L.shape.hkd == 128) return cudaLaunchKernelEx(&cfg, gdn_decode_kernel<128>, tm, p);
  if (L.shape.hkd == 64) return cudaLaunchKernelEx(&cfg, gdn_decode_kernel<64>, tm, p);
  return cudaErrorInvalidValue;
}

}  // namespace hb
