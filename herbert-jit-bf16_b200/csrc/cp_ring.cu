// cp_ring.cu -- context-parallel causal prefill: a zig-zag sharded sequence,
// K/V shards rotated around a ring of GPUs by NCCL send/recv, the partial
// attention of every hop merged by log-sum-exp (the hop kernel is the
// tcgen05 prefill kernel of attn_prefill.cu in its CP form).
//
// No counterpart in the reference: its prefill runs on the cores of one
// machine (src/jit/target/x86/execution/attention.rs:56-224).  The rows of a
// shard are the reference's q rows and its K/V the reference's cache layout
// ([kv_head][capacity][head_dim], src/jit/model.rs:545-559).
//
// Zig-zag sharding: the 2*P*chunk positions are 2P chunks; rank r holds
// chunks r and 2P-1-r, so every rank does the same causal work.  At hop i
// rank r computes against the shard of rank (r - i) mod P:
//   hop 0        chunk r vs r (diagonal), chunk 2P-1-r vs r (full) and vs
//                2P-1-r (diagonal);
//   source j < r both local chunks vs chunk j (full);
//   source j > r chunk 2P-1-r vs chunks j and 2P-1-j (full).
// The kernel derives all of this from absolute positions; a q tile that
// sees none of a shard's keys exits at once.
//
// Streams: hop i runs on `stream` while the shard of hop i+1 arrives on
// `comm_stream` (one grouped send/recv per hop); events order each receive
// after the hop that last read its buffer.  NCCL is loaded with dlopen so
// the library carries no link-time dependency on it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "hb_host.h"
#include "hb_internal.h"

namespace hb {
namespace {

constexpr int64_t kCpTile = 128;  // query rows per CTA of the hop kernel

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  const char* (*error_string)(ncclResult_t);
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*comm_abort)(ncclComm_t);
};

// The NCCL already loaded in the process (torch's, for instance) if there is
// one, else libnccl.so.2 from the loader path.
const NcclApi* nccl_api() {
  static NcclApi api;
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    bool all = true;
    auto sym = [&](const char* name) {
      void* f = dlsym(h, name);
      all = all && f != nullptr;
      return f;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
    api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.comm_get_async_error =
        reinterpret_cast<decltype(api.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    ok = all;
  });
  return ok ? &api : nullptr;
}

hb_status nccl_fail(const NcclApi* n, ncclResult_t r, const char* what) {
  return fail(HB_ERR_NCCL, "%s: %s", what, n->error_string(r));
}

bool valid_cp(const hb_cp_spec* cp) {
  return cp && cp->ranks >= 1 && cp->rank >= 0 && cp->rank < cp->ranks && cp->chunk > 0;
}

// The whole sequence, 2 x ranks x chunk positions, stays below 2^31 (written
// as a division: the product itself could overflow on a hostile record).
bool cp_sequence_ok(const hb_cp_spec* cp) {
  return cp->chunk < (int64_t(1) << 31) / (int64_t(2) * cp->ranks);
}

int64_t chunk_position(const hb_cp_spec* cp, int32_t rank, int second) {
  return (second ? int64_t(2) * cp->ranks - 1 - rank : int64_t(rank)) * cp->chunk;
}

// K and V of one shard: [kv_head][2*chunk][head_dim] bf16 each.
size_t shard_bytes(const hb_attn_spec* s, const hb_cp_spec* cp) {
  return size_t(mul_sat(mul_sat(s->heads / s->gqa, 2 * cp->chunk), s->head_dim * 2));
}

struct CpPlan {
  size_t acc_off, ring_off, bytes;
};

CpPlan plan_cp(const hb_attn_spec* s, const hb_cp_spec* cp) {
  CpPlan p;
  p.acc_off = kWsHeader;
  p.ring_off = p.acc_off + cp_acc_bytes(s->heads, 2 * cp->chunk);
  p.bytes = p.ring_off + (cp->ranks > 1 ? 4 * align256(shard_bytes(s, cp)) : 0);
  return p;
}

hb_status check_cp(const hb_attn_spec* s, const hb_cp_spec* cp, const hb_attn_call* c) {
  hb_status r = check_spec(s);
  if (r != HB_OK) return r;
  if (!valid_cp(cp)) return fail(HB_ERR_ARG, "invalid ring (ranks >= 1, 0 <= rank < ranks, chunk > 0)");
  if (!prefill_serves(s->head_dim))
    return fail(HB_DECLINE_HEAD_DIM, "context-parallel prefill serves head_dim 256; got %lld",
                (long long)s->head_dim);
  if (cp->chunk % kCpTile)
    return fail(HB_DECLINE_GEOMETRY, "chunk %lld is not a multiple of %lld", (long long)cp->chunk,
                (long long)kCpTile);
  if (!cp_sequence_ok(cp))
    return fail(HB_DECLINE_GEOMETRY, "sequence of 2 x %d ranks x %lld positions is above 2^31",
                int(cp->ranks), (long long)cp->chunk);
  if ((r = check_call(s, c)) != HB_OK) return r;
  if (c->rows != 2 * cp->chunk || c->past != 0)
    return fail(HB_ERR_ARG, "a shard has rows = 2*chunk = %lld and past = 0 (got rows %lld, past %lld)",
                (long long)(2 * cp->chunk), (long long)c->rows, (long long)c->past);
  return HB_OK;
}

// The launch of one hop over the shard in (keys, values, kv_stride).
PrefillLaunch hop_launch(const hb_attn_spec* s, const hb_cp_spec* cp, const hb_attn_call* c,
                         int32_t hop, const uint16_t* keys, const uint16_t* values,
                         int64_t kv_stride, void* ws, const CpPlan& pl) {
  const int32_t src = hb_cp_hop_source(cp, hop);
  PrefillLaunch L;
  L.q = c->q;
  L.keys = keys;
  L.values = values;
  L.out = c->output;
  L.q_row = s->q_row;
  L.out_row = s->out_row;
  L.gate_offset = s->gate_offset;
  L.kv_stride = kv_stride;
  L.rows = c->rows;
  L.past = 0;
  L.heads = s->heads;
  L.gqa = s->gqa;
  L.hkv = s->heads / s->gqa;
  L.scale = c->scale;
  char* base = static_cast<char*>(ws);
  L.status = reinterpret_cast<int*>(base);
  L.cp = true;
  L.merge = hop > 0;
  L.chunk = cp->chunk;
  L.q_pos0 = chunk_position(cp, cp->rank, 0);
  L.q_pos1 = chunk_position(cp, cp->rank, 1);
  L.kpos[0] = chunk_position(cp, src, 0);
  L.kpos[1] = chunk_position(cp, src, 1);
  L.kv_rows = 2 * cp->chunk;
  L.acc = reinterpret_cast<float*>(base + pl.acc_off);
  return L;
}

// Events of one ring call, released when the call returns (their pending
// records complete on their own).
struct EventSet {
  std::vector<cudaEvent_t> ev;
  ~EventSet() {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
  }
  cudaError_t make(size_t n) {
    ev.reserve(n);
    for (size_t i = 0; i < n; ++i) {
      cudaEvent_t e;
      cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
      if (r != cudaSuccess) return r;
      ev.push_back(e);
    }
    return cudaSuccess;
  }
};

}  // namespace
}  // namespace hb

using namespace hb;

extern "C" {

int32_t hb_cp_hop_source(const hb_cp_spec* cp, int32_t hop) {
  if (!valid_cp(cp) || hop < 0 || hop >= cp->ranks) return -1;
  return int32_t((int64_t(cp->rank) - hop + cp->ranks) % cp->ranks);
}

int64_t hb_cp_row_position(const hb_cp_spec* cp, int32_t rank, int64_t row) {
  if (!valid_cp(cp) || !cp_sequence_ok(cp) || rank < 0 || rank >= cp->ranks || row < 0 ||
      row >= 2 * cp->chunk)
    return -1;
  return row < cp->chunk ? chunk_position(cp, rank, 0) + row
                         : chunk_position(cp, rank, 1) + (row - cp->chunk);
}

size_t hb_attn_prefill_cp_workspace_bytes(const hb_attn_spec* s, const hb_cp_spec* cp) {
  if (check_spec(s) != HB_OK || !valid_cp(cp) || !cp_sequence_ok(cp) || !prefill_serves(s->head_dim))
    return 0;
  return plan_cp(s, cp).bytes;
}

hb_status hb_attn_prefill_cp_hop(const hb_attn_spec* s, const hb_cp_spec* cp,
                                 const hb_attn_call* c, int32_t hop, void* ws, size_t ws_bytes,
                                 hb_stream_t stream) {
  hb_status r = check_cp(s, cp, c);
  if (r != HB_OK) return r;
  if (hop < 0 || hop >= cp->ranks)
    return fail(HB_ERR_ARG, "hop %d outside [0, %d)", int(hop), int(cp->ranks));
  const CpPlan pl = plan_cp(s, cp);
  if ((r = check_ws(ws, ws_bytes, pl.ring_off)) != HB_OK) return r;
  const PrefillLaunch L = hop_launch(s, cp, c, hop, c->keys, c->values, c->kv_stride, ws, pl);
  cudaError_t e = launch_attn_prefill(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attn_prefill_cp hop launch");
  return HB_OK;
}

hb_status hb_attn_prefill_cp_finish(const hb_attn_spec* s, const hb_cp_spec* cp,
                                    const hb_attn_call* c, void* ws, size_t ws_bytes,
                                    hb_stream_t stream) {
  hb_status r = check_cp(s, cp, c);
  if (r != HB_OK) return r;
  const CpPlan pl = plan_cp(s, cp);
  if ((r = check_ws(ws, ws_bytes, pl.ring_off)) != HB_OK) return r;
  const PrefillLaunch L = hop_launch(s, cp, c, 0, c->keys, c->values, c->kv_stride, ws, pl);
  cudaError_t e = launch_attn_cp_finish(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attn_prefill_cp finish launch");
  return HB_OK;
}

hb_status hb_cp_comm_unique_id(void* id) {
  if (!id) return fail(HB_ERR_ARG, "id is null");
  const NcclApi* n = nccl_api();
  if (!n) return fail(HB_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  ncclResult_t r = n->get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(n, r, "ncclGetUniqueId");
  static_assert(sizeof(u) == HB_CP_ID_BYTES, "ncclUniqueId size");
  memcpy(id, &u, sizeof u);
  return HB_OK;
}

hb_status hb_cp_comm_init(void** comm, int32_t ranks, const void* id, int32_t rank) {
  if (!comm || !id || ranks < 1 || rank < 0 || rank >= ranks)
    return fail(HB_ERR_ARG, "invalid communicator arguments");
  const NcclApi* n = nccl_api();
  if (!n) return fail(HB_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  ncclComm_t c = nullptr;
  ncclResult_t r = n->comm_init_rank(&c, ranks, u, rank);
  if (r != ncclSuccess) return nccl_fail(n, r, "ncclCommInitRank");
  *comm = c;
  return HB_OK;
}

hb_status hb_cp_comm_destroy(void* comm) {
  if (!comm) return HB_OK;
  const NcclApi* n = nccl_api();
  if (!n) return fail(HB_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclResult_t r = n->comm_destroy(static_cast<ncclComm_t>(comm));
  if (r != ncclSuccess) return nccl_fail(n, r, "ncclCommDestroy");
  return HB_OK;
}

hb_status hb_cp_wait(void* comm, hb_stream_t stream, double timeout_s) {
  if (!(timeout_s >= 0.0)) return fail(HB_ERR_ARG, "timeout is negative or NaN");
  const NcclApi* n = comm ? nccl_api() : nullptr;
  if (comm && !n) return fail(HB_ERR_NCCL, "libnccl.so.2 could not be loaded");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ncclComm_t nc = static_cast<ncclComm_t>(comm);
  ncclResult_t async = ncclSuccess;
  cudaError_t qerr = cudaSuccess;
  const WaitResult w = wait_with_deadline(
      [&] {
        qerr = cudaStreamQuery(st);
        return qerr == cudaSuccess ? 0 : qerr == cudaErrorNotReady ? 1 : 2;
      },
      [&] {
        if (!nc) return false;
        ncclResult_t r = ncclSuccess;
        if (n->comm_get_async_error(nc, &r) != ncclSuccess) r = ncclInternalError;
        if (r != ncclSuccess && r != ncclInProgress) async = r;
        return async != ncclSuccess;
      },
      monotonic_seconds, sleep_poll_interval, timeout_s);
  if (w == WaitResult::kDone) return HB_OK;
  // abort, so that the peers' transfers that wait on this rank end too
  if (nc) n->comm_abort(nc);
  switch (w) {
    case WaitResult::kTimeout:
      return fail(HB_ERR_TIMEOUT, "the ring did not complete within %.3f s; communicator aborted",
                  timeout_s);
    case WaitResult::kCommError:
      return fail(HB_ERR_NCCL, "the communicator reported %s; communicator aborted",
                  n->error_string(async));
    default:
      return fail(HB_ERR_CUDA, "stream query failed: %s%s", cudaGetErrorString(qerr),
                  nc ? "; communicator aborted" : "");
  }
}

hb_status hb_attn_prefill_cp(const hb_attn_spec* s, const hb_cp_spec* cp, const hb_attn_call* c,
                             void* comm, void* ws, size_t ws_bytes, hb_stream_t stream,
                             hb_stream_t comm_stream) {
  hb_status r = check_cp(s, cp, c);
  if (r != HB_OK) return r;
  const CpPlan pl = plan_cp(s, cp);
  if ((r = check_ws(ws, ws_bytes, pl.bytes)) != HB_OK) return r;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(comm_stream);
  const int P = cp->ranks;
  if (P == 1) {  // the whole sequence is local: the single-GPU prefill kernel
    PrefillLaunch L = hop_launch(s, cp, c, 0, c->keys, c->values, c->kv_stride, ws, pl);
    L.cp = false;
    L.merge = false;
    cudaError_t e = launch_attn_prefill(L, st);
    if (e != cudaSuccess) return cuda_fail(e, "attn_prefill launch");
    return HB_OK;
  }
  if (!comm) return fail(HB_ERR_ARG, "a ring of %d ranks needs a communicator", P);
  if (cs == st) return fail(HB_ERR_ARG, "comm_stream must differ from stream");
  const NcclApi* n = nccl_api();
  if (!n) return fail(HB_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclComm_t nc = static_cast<ncclComm_t>(comm);

  const int64_t hkv = s->heads / s->gqa;
  const int64_t ring_stride = 2 * cp->chunk * s->head_dim;    // elements per head
  const size_t head_bytes = size_t(ring_stride) * 2;           // bytes per head of K or V
  const size_t ring_half = align256(shard_bytes(s, cp));       // K or V of one buffer
  char* ring = static_cast<char*>(ws) + pl.ring_off;
  auto ring_k = [&](int b) { return reinterpret_cast<uint16_t*>(ring + (2 * b) * ring_half); };
  auto ring_v = [&](int b) { return reinterpret_cast<uint16_t*>(ring + (2 * b + 1) * ring_half); };
  const int next = (cp->rank + 1) % P, prev = (cp->rank - 1 + P) % P;

  EventSet ev;  // [0] inputs ready, [1 + i] shard i+1 received, [1 + P + i] hop i computed
  cudaError_t e = ev.make(1 + 2 * size_t(P));
  if (e != cudaSuccess) return cuda_fail(e, "attn_prefill_cp events");
  cudaEvent_t ev_in = ev.ev[0];
  auto ev_recv = [&](int i) { return ev.ev[1 + i]; };
  auto ev_hop = [&](int i) { return ev.ev[1 + P + i]; };
  if ((e = cudaEventRecord(ev_in, st)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(cs, ev_in, 0)) != cudaSuccess)
    return cuda_fail(e, "attn_prefill_cp ordering");

  for (int i = 0; i < P; ++i) {
    const uint16_t* k = i == 0 ? c->keys : ring_k((i - 1) & 1);
    const uint16_t* v = i == 0 ? c->values : ring_v((i - 1) & 1);
    const int64_t kvs = i == 0 ? c->kv_stride : ring_stride;
    if (i + 1 < P) {
      // the buffer receiving shard i+1 was last read by hop i-1
      const int b = i & 1;
      if (i >= 2 && (e = cudaStreamWaitEvent(cs, ev_hop(i - 1), 0)) != cudaSuccess)
        return cuda_fail(e, "attn_prefill_cp ordering");
      ncclResult_t nr = n->group_start();
      for (int64_t h = 0; nr == ncclSuccess && h < hkv; ++h) {
        nr = n->send(k + h * kvs, head_bytes, ncclUint8, next, nc, cs);
        if (nr == ncclSuccess) nr = n->send(v + h * kvs, head_bytes, ncclUint8, next, nc, cs);
        if (nr == ncclSuccess) nr = n->recv(ring_k(b) + h * ring_stride, head_bytes, ncclUint8, prev, nc, cs);
        if (nr == ncclSuccess) nr = n->recv(ring_v(b) + h * ring_stride, head_bytes, ncclUint8, prev, nc, cs);
      }
      const ncclResult_t ne = n->group_end();
      if (nr != ncclSuccess) return nccl_fail(n, nr, "ncclSend/ncclRecv");
      if (ne != ncclSuccess) return nccl_fail(n, ne, "ncclGroupEnd");
      if ((e = cudaEventRecord(ev_recv(i), cs)) != cudaSuccess)
        return cuda_fail(e, "attn_prefill_cp ordering");
    }
    if (i >= 1 && (e = cudaStreamWaitEvent(st, ev_recv(i - 1), 0)) != cudaSuccess)
      return cuda_fail(e, "attn_prefill_cp ordering");
    const PrefillLaunch L = hop_launch(s, cp, c, i, k, v, kvs, ws, pl);
    if ((e = launch_attn_prefill(L, st)) != cudaSuccess) return cuda_fail(e, "attn_prefill_cp hop launch");
    if ((e = cudaEventRecord(ev_hop(i), st)) != cudaSuccess)
      return cuda_fail(e, "attn_prefill_cp ordering");
  }
  const PrefillLaunch L = hop_launch(s, cp, c, 0, c->keys, c->values, c->kv_stride, ws, pl);
  if ((e = launch_attn_cp_finish(L, st)) != cudaSuccess)
    return cuda_fail(e, "attn_prefill_cp finish launch");
  return HB_OK;
}

}  // extern "C"
