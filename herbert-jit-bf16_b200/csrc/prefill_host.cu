// prefill_host.cu -- hb_attn_prefill_host and hb_gdn_prefill_host: the
// prefill of rows whose inputs and output are in host memory, with the
// host <-> device copies overlapped with the computation.
//
// An engine that keeps its buffers on the host -- the reference's own
// arrangement, Runner-owned buffers handed to the prefill node
// (src/jit/model.rs:570-611; node src/jit/target/x86/execution/attention.rs:56-224)
// -- would otherwise copy the inputs in, run hb_attn_prefill and copy the
// output back, one after the other.  Here the rows are cut into blocks of a
// multiple of 128 rows.  Block j's q rows and the K/V positions it adds go
// in on a copy stream (one cudaMemcpyAsync for the q rows and one per KV
// head for K and for V); its prefill (the block's rows over every position
// copied so far) runs on the caller's stream once they have landed; its
// output rows go back on a second copy stream.  Causal prefill makes later
// blocks longer (block j of B is (2j+1)/B^2 of the work), so the later
// blocks' copies hide under the earlier blocks' computation: only the first
// block's inputs and the last block's output stand outside it.  The blocks
// run one after the other: blocks spread over several compute streams ran
// 9 % slower at 131072 rows (their CTAs interleave), and a block's tail
// costs less than that.
//
// Block boundaries are query-tile boundaries, so every row is computed by
// the same products in the same order as in one hb_attn_prefill call over
// all the rows: the result is bit-identical.
//
// hb_gdn_prefill_host does the same for the chunked DeltaNet prefill: block
// j's qkv, beta and decay rows in, hb_gdn_prefill over the block (the state
// carried in place from block to block), its output rows out.  The chunked
// kernels carry the state between chunks only through its bf16 rounding
// (each chunk's products read the bf16 state; the f32 state is formed by
// them), and a call starts by rounding the f32 state it reads, so blocks
// that start on chunk boundaries and all take the chunked kernels (128 rows
// or more each) give one call's bits.  DeltaNet rows are copy-bound (32 KB
// of f32 inputs per row at Qwen3.5 geometry against ≈ 50 ns of computation),
// so the blocks are small enough that the first block's copy, the only one
// not hidden, stays short.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "hb_internal.h"

namespace hb {

int64_t prefill_host_block(int64_t rows, int64_t block_rows) {
  if (block_rows > 0) return block_rows;
  // about sixteen blocks, at least 1024 rows each (the copies of smaller
  // blocks cost more per byte than their overlap gains: 4096 rows took
  // 1.94 ms from host to host in blocks of 1024, 2.05 in blocks of 512)
  const int64_t b = ((rows + 15) / 16 + 127) / 128 * 128;
  return std::max<int64_t>(1024, b);
}

int64_t prefill_host_blocks(int64_t rows, int64_t block) {
  int64_t n = (rows + block - 1) / block;
  // a remainder of fewer rows than the tensor-core kernel takes joins the
  // block before it, so that every block runs the kernel one call would
  if (n > 1 && rows - (n - 1) * block < kPrefillMinRows) --n;
  return n;
}

namespace {

// The copy-in and copy-out streams of a device, made once,
// and its pool of events.  A call holds the device's lock while it queues
// its work: each event it uses is recorded and then waited on inside the
// call (a wait takes the event's latest record at the time it is queued),
// so the next call may record the same events again.  Nothing is created
// or destroyed while a caller's stream may be capturing a graph, except on
// a device's first calls.
struct HostStreams {
  cudaStream_t in = nullptr, out = nullptr;
  std::vector<cudaEvent_t> events;
  std::mutex mu;
};
HostStreams g_streams[64];
DeviceFlags g_streams_made;

cudaError_t host_streams(HostStreams** hs) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  e = g_streams_made.once([&] {
    HostStreams& s = g_streams[dev];
    cudaError_t r = cudaStreamCreateWithFlags(&s.in, cudaStreamNonBlocking);
    if (r == cudaSuccess) r = cudaStreamCreateWithFlags(&s.out, cudaStreamNonBlocking);
    return r;
  });
  if (e != cudaSuccess) return e;
  *hs = &g_streams[dev];
  return cudaSuccess;
}

// The pool's events [0, n), made on first need (under the device's lock).
cudaError_t pool_events(HostStreams* hs, size_t n) {
  while (hs->events.size() < n) {
    cudaEvent_t e;
    const cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (r != cudaSuccess) return r;
    hs->events.push_back(e);
  }
  return cudaSuccess;
}

hb_status check_host_call(const hb_attn_spec* s, const hb_attn_host_call* h) {
  hb_status r = check_spec(s);
  if (r != HB_OK) return r;
  if (!h) return fail(HB_ERR_ARG, "host call is null");
  if ((r = check_call(s, &h->dev)) != HB_OK) return r;
  if (!h->q_host || !h->keys_host || !h->values_host || !h->out_host)
    return fail(HB_ERR_ARG, "host q/keys/values/output pointers must not be null");
  if (h->block_rows < 0 || h->block_rows % 128)
    return fail(HB_ERR_ARG, "block_rows %lld must be 0 or a positive multiple of 128",
                (long long)h->block_rows);
  return HB_OK;
}

// Call of block [r0, r0 + nb) of the rows.
hb_attn_call block_call(const hb_attn_spec* s, const hb_attn_call& c, int64_t r0, int64_t nb) {
  hb_attn_call b = c;
  b.q = c.q + r0 * s->q_row;
  b.output = c.output + r0 * s->out_row;
  b.rows = nb;
  b.past = c.past + r0;
  return b;
}

int64_t gdn_host_block(int64_t rows, int64_t block_rows) {
  if (block_rows > 0) return block_rows;
  // about sixteen blocks, at least 256 rows each
  const int64_t b = ((rows + 15) / 16 + 63) / 64 * 64;
  return std::max<int64_t>(256, b);
}

int64_t gdn_host_blocks(int64_t rows, int64_t block) {
  int64_t n = (rows + block - 1) / block;
  // a remainder below the chunked kernels' minimum joins the block before it
  if (n > 1 && rows - (n - 1) * block < 128) --n;
  return n;
}

hb_status check_gdn_host_call(const hb_gdn_shape* s, const hb_gdn_host_call* h) {
  if (!s || !h) return fail(HB_ERR_ARG, "DeltaNet shape or host call is null");
  if (!h->qkv_host || !h->beta_host || !h->decay_host || !h->output_host)
    return fail(HB_ERR_ARG, "host qkv/beta/decay/output pointers must not be null");
  if (h->block_rows < 0 || h->block_rows % 64)
    return fail(HB_ERR_ARG, "block_rows %lld must be 0 or a positive multiple of 64",
                (long long)h->block_rows);
  if (h->dev.rows <= 0) return fail(HB_DECLINE_EMPTY, "empty DeltaNet block");
  if (h->dev.rows >= (int64_t(1) << 31))
    return fail(HB_ERR_ARG, "rows %lld beyond the host prefill's range", (long long)h->dev.rows);
  return HB_OK;
}

hb_gdn_call gdn_block_call(const hb_gdn_shape* s, const hb_gdn_call& c, int64_t r0, int64_t nb) {
  const int64_t conv = 2 * s->nk * s->hkd + s->nv * s->hvd;
  hb_gdn_call b = c;
  b.qkv = c.qkv + r0 * conv;
  b.beta = c.beta + r0 * s->nv;
  b.decay = c.decay + r0 * s->nv;
  b.output = c.output + r0 * s->nv * s->hvd;
  b.rows = nb;
  return b;
}

}  // namespace
}  // namespace hb

using namespace hb;

size_t hb_attn_prefill_host_workspace_bytes(const hb_attn_spec* s, const hb_attn_host_call* h) {
  if (check_host_call(s, h) != HB_OK) return 0;
  const int64_t rows = h->dev.rows, block = prefill_host_block(rows, h->block_rows);
  const int64_t nblocks = prefill_host_blocks(rows, block);
  // a block's need grows with its rows and its first position: the first
  // block, the last full one and the last one cover every block
  size_t need = 0;
  for (const int64_t j : {int64_t(0), std::max<int64_t>(0, nblocks - 2), nblocks - 1}) {
    const int64_t r0 = j * block, nb = j + 1 < nblocks ? block : rows - r0;
    const hb_attn_call b = block_call(s, h->dev, r0, nb);
    need = std::max(need, hb_attn_prefill_workspace_bytes(s, &b));
  }
  return need;
}

hb_status hb_attn_prefill_host(const hb_attn_spec* s, const hb_attn_host_call* h, void* ws,
                               size_t ws_bytes, hb_stream_t stream) {
  hb_status r = check_host_call(s, h);
  if (r != HB_OK) return r;
  if ((r = check_ws(ws, ws_bytes, hb_attn_prefill_host_workspace_bytes(s, h))) != HB_OK) return r;
  HostStreams* hs = nullptr;
  cudaError_t e = host_streams(&hs);
  if (e != cudaSuccess) return cuda_fail(e, "hb_attn_prefill_host streams");
  const cudaStream_t main = reinterpret_cast<cudaStream_t>(stream);
  const hb_attn_call& c = h->dev;
  const int64_t rows = c.rows, block = prefill_host_block(rows, h->block_rows);
  const int64_t nblocks = prefill_host_blocks(rows, block);
  const int64_t hkv = s->heads / s->gqa, hd = s->head_dim;
  std::lock_guard<std::mutex> lock(hs->mu);
  // fork, then per block "landed" and "done", then the join
  if ((e = pool_events(hs, size_t(2 * nblocks + 2))) != cudaSuccess)
    return cuda_fail(e, "hb_attn_prefill_host events");
  cudaEvent_t* ev = hs->events.data();
  // every stream starts after the work already queued on `stream`
  if ((e = cudaEventRecord(ev[0], main)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(hs->in, ev[0], 0)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(hs->out, ev[0], 0)) != cudaSuccess)
    return cuda_fail(e, "hb_attn_prefill_host fork");
  for (int64_t j = 0; j < nblocks; ++j) {
    const int64_t r0 = j * block, nb = j + 1 < nblocks ? block : rows - r0;
    const int64_t pos = c.past + r0;  // first K/V position the block adds
    // its q rows and K/V positions in
    e = cudaMemcpyAsync(const_cast<uint16_t*>(c.q) + r0 * s->q_row, h->q_host + r0 * s->q_row,
                        size_t(nb * s->q_row) * 2, cudaMemcpyHostToDevice, hs->in);
    for (int64_t kh = 0; e == cudaSuccess && kh < hkv; ++kh) {
      const int64_t off = kh * c.kv_stride + pos * hd;
      e = cudaMemcpyAsync(const_cast<uint16_t*>(c.keys) + off, h->keys_host + off,
                          size_t(nb * hd) * 2, cudaMemcpyHostToDevice, hs->in);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(const_cast<uint16_t*>(c.values) + off, h->values_host + off,
                            size_t(nb * hd) * 2, cudaMemcpyHostToDevice, hs->in);
    }
    cudaEvent_t landed = ev[1 + 2 * j], done = ev[2 + 2 * j];
    if (e == cudaSuccess) e = cudaEventRecord(landed, hs->in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(main, landed, 0);
    if (e != cudaSuccess) return cuda_fail(e, "hb_attn_prefill_host copy-in");
    // the block's rows over every position copied so far
    const hb_attn_call b = block_call(s, c, r0, nb);
    if ((r = hb_attn_prefill(s, &b, ws, ws_bytes, stream)) != HB_OK)
      return r;
    // its output rows back
    if ((e = cudaEventRecord(done, main)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(hs->out, done, 0)) != cudaSuccess ||
        (e = cudaMemcpyAsync(h->out_host + r0 * s->out_row, c.output + r0 * s->out_row,
                             size_t(nb * s->out_row) * 2, cudaMemcpyDeviceToHost, hs->out)) !=
            cudaSuccess)
      return cuda_fail(e, "hb_attn_prefill_host copy-out");
  }
  // `stream` continues after the last copy out
  cudaEvent_t join = ev[1 + 2 * nblocks];
  if ((e = cudaEventRecord(join, hs->out)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(main, join, 0)) != cudaSuccess)
    return cuda_fail(e, "hb_attn_prefill_host join");
  return HB_OK;
}

size_t hb_gdn_prefill_host_workspace_bytes(const hb_gdn_shape* s, const hb_gdn_host_call* h) {
  if (check_gdn_host_call(s, h) != HB_OK) return 0;
  const int64_t rows = h->dev.rows, block = gdn_host_block(rows, h->block_rows);
  const int64_t nblocks = gdn_host_blocks(rows, block);
  // every block but the last has `block` rows
  const int64_t last = rows - (nblocks - 1) * block;
  return std::max(hb_gdn_prefill_workspace_bytes(s, std::min(rows, block)),
                  hb_gdn_prefill_workspace_bytes(s, last));
}

hb_status hb_gdn_prefill_host(const hb_gdn_shape* s, const hb_gdn_host_call* h, void* ws,
                              size_t ws_bytes, hb_stream_t stream) {
  hb_status r = check_gdn_host_call(s, h);
  if (r != HB_OK) return r;
  const hb_gdn_call& c = h->dev;
  const int64_t rows = c.rows, block = gdn_host_block(rows, h->block_rows);
  const int64_t nblocks = gdn_host_blocks(rows, block);
  // the blocks' own checks before any copy is queued
  if ((r = check_ws(ws, ws_bytes, hb_gdn_prefill_host_workspace_bytes(s, h))) != HB_OK) return r;
  const hb_gdn_call first = gdn_block_call(s, c, 0, std::min(rows, block));
  if ((r = hb_gdn_check(s, &first)) != HB_OK) return r;
  HostStreams* hs = nullptr;
  cudaError_t e = host_streams(&hs);
  if (e != cudaSuccess) return cuda_fail(e, "hb_gdn_prefill_host streams");
  const cudaStream_t main = reinterpret_cast<cudaStream_t>(stream);
  const int64_t conv = 2 * s->nk * s->hkd + s->nv * s->hvd, value = s->nv * s->hvd;
  std::lock_guard<std::mutex> lock(hs->mu);
  if ((e = pool_events(hs, size_t(2 * nblocks + 2))) != cudaSuccess)
    return cuda_fail(e, "hb_gdn_prefill_host events");
  cudaEvent_t* ev = hs->events.data();
  if ((e = cudaEventRecord(ev[0], main)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(hs->in, ev[0], 0)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(hs->out, ev[0], 0)) != cudaSuccess)
    return cuda_fail(e, "hb_gdn_prefill_host fork");
  for (int64_t j = 0; j < nblocks; ++j) {
    const int64_t r0 = j * block, nb = j + 1 < nblocks ? block : rows - r0;
    const hb_gdn_call b = gdn_block_call(s, c, r0, nb);
    e = cudaMemcpyAsync(const_cast<float*>(b.qkv), h->qkv_host + r0 * conv, size_t(nb * conv) * 4,
                        cudaMemcpyHostToDevice, hs->in);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(const_cast<float*>(b.beta), h->beta_host + r0 * s->nv,
                          size_t(nb * s->nv) * 4, cudaMemcpyHostToDevice, hs->in);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(const_cast<float*>(b.decay), h->decay_host + r0 * s->nv,
                          size_t(nb * s->nv) * 4, cudaMemcpyHostToDevice, hs->in);
    cudaEvent_t landed = ev[1 + 2 * j], done = ev[2 + 2 * j];
    if (e == cudaSuccess) e = cudaEventRecord(landed, hs->in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(main, landed, 0);
    if (e != cudaSuccess) return cuda_fail(e, "hb_gdn_prefill_host copy-in");
    if ((r = hb_gdn_prefill(s, &b, ws, ws_bytes, stream)) != HB_OK) return r;
    if ((e = cudaEventRecord(done, main)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(hs->out, done, 0)) != cudaSuccess ||
        (e = cudaMemcpyAsync(h->output_host + r0 * value, b.output, size_t(nb * value) * 4,
                             cudaMemcpyDeviceToHost, hs->out)) != cudaSuccess)
      return cuda_fail(e, "hb_gdn_prefill_host copy-out");
  }
  cudaEvent_t join = ev[1 + 2 * nblocks];
  if ((e = cudaEventRecord(join, hs->out)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(main, join, 0)) != cudaSuccess)
    return cuda_fail(e, "hb_gdn_prefill_host join");
  return HB_OK;
}
