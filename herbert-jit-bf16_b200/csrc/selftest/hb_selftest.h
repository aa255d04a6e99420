/*
 * hb_selftest.h -- C ABI of libherbert_b200_selftest.so, the test-only
 * companion of libherbert_b200.so.  Nothing here is part of the product
 * interface (include/herbert_b200.h); the tests load this library beside the
 * product library to check device code paths that random parity inputs do
 * not reach.  Status codes are the product's hb_status values.
 */
#ifndef HB_SELFTEST_H
#define HB_SELFTEST_H

#include <stddef.h>
#include <stdint.h>

#include "../../../include/herbert_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Message of the last failing self-test call on this thread. */
HB_API const char *hbt_last_error(void);

/*
 * Runs the arithmetic of hb_attn_prefill's epilogue (O / l rounded to bf16,
 * then the output gate) over every pair of bf16 values (a, g) and over every
 * f32 value of O / l, and compares each result with the exact per-element
 * steps.  Synchronous on `stream`; tens of milliseconds on a B200.  out[8]:
 * [0] gate mismatches, [1] column pairs the fast path sent to the exact
 * steps, [2] first mismatching element + 1 (a | g << 16; 0 = none), [3] its
 * result | expected << 16; [4..7] the same for the O / l rounding (element =
 * the f32 bits).
 */
HB_API int hbt_prefill_epilogue(uint64_t *out, hb_stream_t stream);

/*
 * A bounded device wait made to run out.  One CTA of 64 threads: warp 0
 * initialises an mbarrier that expects two arrivals and arrives once; no
 * copy and no other thread ever completes the phase.  Warp 1 waits on it
 * with the product kernels' bounded wait (mbar_wait) and a limit of
 * `spin_cycles` SM cycles, then records the timeout in the workspace's status
 * word exactly as the product kernels do, and every thread returns.  The
 * product's hb_workspace_status then reports HB_ERR_TIMEOUT.  With
 * `complete` = 1 the second arrival is made before the wait and the wait
 * succeeds (the status word stays clear).  spin_cycles must lie in
 * [1000, 2e9]; the workspace must be at least 256 bytes and zeroed.
 */
HB_API int hbt_wait_timeout(void *workspace, size_t workspace_bytes, long long spin_cycles,
                            int complete, hb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HB_SELFTEST_H */
