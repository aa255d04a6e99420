// hb_selftest.cu -- exhaustive self-test of the prefill epilogue's fast
// arithmetic (hb_epilogue.cuh): every (a, g) pair of bf16 values through the
// gated block and every f32 value of O / l through the plain block, each
// result compared with the exact per-element steps (f32_to_bf16_cvtne and
// gate_bf16).  Random parity inputs cannot reach the rare cases the fast
// path must send to the exact steps; this covers the whole input domain.
//
// Test-only: built into libherbert_b200_selftest.so (hb_selftest.h), never
// into the product library.
#include <cuda_runtime.h>

#include <cstdio>

#include "../hb_common.cuh"
#include "../hb_epilogue.cuh"
#include "hb_selftest.h"

namespace hb {
namespace {

// [0] gate mismatches, [1] gate pairs on the exact steps, [2] first gate
// mismatch (a | g << 16) + 1, [3] its result | expected << 16; [4..7] the
// same for the O / l conversion (element = f32 bits)
__device__ unsigned long long g_selftest[8];

HB_DEV bool same_bf16(uint16_t x, uint16_t y) {
  const bool nx = (x & 0x7F80u) == 0x7F80u && (x & 0x7Fu);
  const bool ny = (y & 0x7F80u) == 0x7F80u && (y & 0x7Fu);
  return x == y || (nx && ny);  // NaN payloads are not compared
}

HB_DEV uint16_t half_of(const uint32_t (&w)[kEpilogueWidth / 2], int i) {
  return uint16_t(i & 1 ? w[i >> 1] >> 16 : w[i >> 1] & 0xFFFFu);
}

HB_DEV void record(unsigned long long* slot, uint64_t element, uint16_t got, uint16_t want) {
  if (atomicCAS(slot, 0ull, (unsigned long long)element + 1ull) == 0ull)
    slot[1] = (unsigned long long)got | ((unsigned long long)want << 16);
}

constexpr int W = kEpilogueWidth;

// element e = a | g << 16; one block = W consecutive a for one g
__global__ void __launch_bounds__(256) selftest_gate_kernel() {
  unsigned long long bad = 0, slow = 0;
  const uint64_t nblocks = (uint64_t(1) << 32) / W;
  for (uint64_t b = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < nblocks;
       b += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t e0 = uint32_t(b * W);
    const uint32_t g = e0 >> 16;
    uint32_t o[W], gw[W / 2], w[W / 2];
#pragma unroll
    for (int i = 0; i < W; ++i) o[i] = ((e0 + uint32_t(i)) & 0xFFFFu) << 16;
#pragma unroll
    for (int i = 0; i < W / 2; ++i) gw[i] = g | (g << 16);
    slow += epilogue_block<W, true>(o, 1.0f, gw, w);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const uint16_t a = f32_to_bf16_cvtne(__fmul_rn(__uint_as_float(o[i]), 1.0f));
      const uint16_t want = gate_bf16(a, uint16_t(g));
      const uint16_t got = half_of(w, i);
      if (!same_bf16(got, want)) {
        ++bad;
        record(&g_selftest[2], e0 + uint32_t(i), got, want);
      }
    }
  }
  if (bad) atomicAdd(&g_selftest[0], bad);
  if (slow) atomicAdd(&g_selftest[1], slow);
}

// element = f32 bits of O (with 1 / l = 1); one block = W consecutive values
__global__ void __launch_bounds__(256) selftest_plain_kernel() {
  unsigned long long bad = 0, slow = 0;
  const uint64_t nblocks = (uint64_t(1) << 32) / W;
  for (uint64_t b = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < nblocks;
       b += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t e0 = uint32_t(b * W);
    uint32_t o[W], gw[W / 2], w[W / 2];
#pragma unroll
    for (int i = 0; i < W; ++i) o[i] = e0 + uint32_t(i);
#pragma unroll
    for (int i = 0; i < W / 2; ++i) gw[i] = 0;
    slow += epilogue_block<W, false>(o, 1.0f, gw, w);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const uint16_t want = f32_to_bf16_cvtne(__fmul_rn(__uint_as_float(o[i]), 1.0f));
      const uint16_t got = half_of(w, i);
      if (!same_bf16(got, want)) {
        ++bad;
        record(&g_selftest[6], e0 + uint32_t(i), got, want);
      }
    }
  }
  if (bad) atomicAdd(&g_selftest[4], bad);
  if (slow) atomicAdd(&g_selftest[5], slow);
}

}  // namespace
}  // namespace hb

namespace {
thread_local char g_msg[256] = "";
int selftest_fail(int code, const char* what, cudaError_t e) {
  snprintf(g_msg, sizeof g_msg, "%s: %s", what, e == cudaSuccess ? "" : cudaGetErrorString(e));
  return code;
}
}  // namespace

extern "C" const char* hbt_last_error(void) { return g_msg; }

extern "C" int hbt_prefill_epilogue(uint64_t* out, hb_stream_t stream) {
  using namespace hb;
  if (!out) return selftest_fail(HB_ERR_ARG, "hbt_prefill_epilogue: out is null", cudaSuccess);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void* slots = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&slots, g_selftest);
  if (e == cudaSuccess) e = cudaMemsetAsync(slots, 0, sizeof(unsigned long long) * 8, st);
  int sms = 148;
  if (e == cudaSuccess) {
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  if (e != cudaSuccess) return selftest_fail(HB_ERR_CUDA, "hbt_prefill_epilogue set-up", e);
  selftest_gate_kernel<<<unsigned(sms * 4), 256, 0, st>>>();
  selftest_plain_kernel<<<unsigned(sms * 4), 256, 0, st>>>();
  e = cudaGetLastError();
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(out, slots, sizeof(unsigned long long) * 8, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return selftest_fail(HB_ERR_CUDA, "hbt_prefill_epilogue", e);
  return HB_OK;
}
