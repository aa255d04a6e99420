// hb_selftest_wait.cu -- a bounded device wait that is made to run out, so
// that the path every product kernel takes when a wait gives up (mbar_wait
// returns false, record_status writes the workspace status word, the kernel
// returns, hb_workspace_status reports HB_ERR_TIMEOUT) runs end to end on a
// GPU without a fault or a hang: nothing is in flight when the CTA returns
// (no bulk copy, no MMA, no TMEM), and the wait ends by its own limit.
//
// Test-only: built into libherbert_b200_selftest.so (hb_selftest.h).
#include <cuda_runtime.h>

#include <cstdio>

#include "../hb_common.cuh"
#include "../hb_internal.h"
#include "hb_selftest.h"

namespace hb {
namespace {

__global__ void __launch_bounds__(64) selftest_wait_kernel(int* status, long long spin,
                                                           int complete) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 2);  // two arrivals complete phase 0
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive(&bar);
    if (complete) mbar_arrive(&bar);
  }
  __syncthreads();
  if (threadIdx.x == 32) {
    if (!mbar_wait(&bar, 0, spin)) record_status(status, kStatusTimeout);
  }
  __syncthreads();
}

}  // namespace
}  // namespace hb

extern "C" int hbt_wait_timeout(void* ws, size_t bytes, long long spin, int complete,
                                hb_stream_t stream) {
  using namespace hb;
  if (!ws || bytes < kWsHeader || (reinterpret_cast<uintptr_t>(ws) & 255)) return HB_ERR_WORKSPACE;
  if (spin < 1000 || spin > 2000000000LL) return HB_ERR_ARG;
  selftest_wait_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<int*>(ws), spin, complete ? 1 : 0);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_CUDA;
}
