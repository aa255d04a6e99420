// kv_append.cu -- the KV append of the reference on sm_100a:
// K[h][past + r][:] <- input_keys[r][h][:] (and V), token-major block into
// the head-major cache (src/jit/target/x86/execution/kv.rs:17-69).
// One CTA per (row, KV head); 16-byte vector copies when every address is
// 16-byte aligned, element copies otherwise.
#include <cstdint>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_internal.h"

namespace hb {
namespace {

struct AppendParams {
  uint16_t* keys;
  uint16_t* values;
  const uint16_t* ik;
  const uint16_t* iv;
  int64_t past, stride;
  int heads, head_dim;
  int vec;  // 1: 16-byte copies
};

__global__ void kv_append_kernel(const AppendParams p) {
  const int r = blockIdx.x, h = blockIdx.y;
  const int64_t src = (int64_t(r) * p.heads + h) * p.head_dim;
  const int64_t dst = int64_t(h) * p.stride + (p.past + r) * p.head_dim;
  if (p.vec) {
    const int nv = p.head_dim / 8;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      reinterpret_cast<uint4*>(p.keys + dst)[i] = reinterpret_cast<const uint4*>(p.ik + src)[i];
      reinterpret_cast<uint4*>(p.values + dst)[i] = reinterpret_cast<const uint4*>(p.iv + src)[i];
    }
  } else {
    for (int i = threadIdx.x; i < p.head_dim; i += blockDim.x) {
      p.keys[dst + i] = p.ik[src + i];
      p.values[dst + i] = p.iv[src + i];
    }
  }
}

}  // namespace

cudaError_t launch_kv_append(const hb_kv_spec& s, const hb_kv_call& c, cudaStream_t st) {
  AppendParams p;
  p.keys = c.keys;
  p.values = c.values;
  p.ik = c.input_keys;
  p.iv = c.input_values;
  p.past = c.past;
  p.stride = s.stride;
  p.heads = int(s.heads);
  p.head_dim = int(s.head_dim);
  const uintptr_t mis = reinterpret_cast<uintptr_t>(c.keys) | reinterpret_cast<uintptr_t>(c.values) |
                        reinterpret_cast<uintptr_t>(c.input_keys) |
                        reinterpret_cast<uintptr_t>(c.input_values);
  p.vec = (mis % 16 == 0) && (s.head_dim % 8 == 0) && (s.stride % 8 == 0);
  dim3 grid(unsigned(c.rows), unsigned(s.heads));
  kv_append_kernel<<<grid, 128, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace hb
