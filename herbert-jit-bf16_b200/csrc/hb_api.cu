// hb_api.cu -- the C ABI of libherbert_b200: argument validation that
// mirrors the reference's own refusals, workspace layout, and dispatch to
// the sm_100a kernels.  No allocation, no CPU compute path: a shape no
// kernel serves is refused with a named status.
//
// Validation follows the reference:
//  - attention geometry: tile_selector (src/jit/target/x86/execution/attention.rs:56-89)
//  - SDPA shape:         SdpaShape::check (src/jit/ir.rs:140-160), Decline (:177-230)
//  - KV geometry:        KvSpec::validate (src/jit/execution/abi.rs:75-103)
//  - DeltaNet geometry:  Shape::check (src/jit/execution/abi.rs:283-306)
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <numeric>
#include <queue>
#include <vector>

#include "hb_host.h"
#include "hb_internal.h"

namespace hb {
namespace {

thread_local char g_err[512] = "";

}  // namespace

hb_status fail(hb_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return s;
}

hb_status cuda_fail(cudaError_t e, const char* what) {
  return fail(HB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

constexpr int64_t kI32Half = 0x3FFFFFFF;  // i32::MAX / 2, the reference's bound
// Ranges far beyond any model, chosen so that every product the checks and
// the planner form fits in 64 bits: rows x past < 2^62, positions x head_dim
// < 2^48.
constexpr int64_t kMaxRows = int64_t(1) << 24;
constexpr int64_t kMaxPositions = int64_t(1) << 38;
inline bool call_in_range(int64_t rows, int64_t past) {
  return rows >= 0 && rows <= kMaxRows && past >= 0 && past <= kMaxPositions;
}

// AttentionSpec checks of the tile selector, plus the head_dim domain.
hb_status check_spec(const hb_attn_spec* s) {
  if (!s) return fail(HB_ERR_ARG, "attention spec is null");
  if (s->sink) return fail(HB_DECLINE_SINK, "attention sink is not served (Qwen3.5 has none)");
  if (s->heads <= 0 || s->gqa <= 0 || s->head_dim <= 0)
    return fail(HB_DECLINE_EMPTY, "empty shape (heads=%lld gqa=%lld head_dim=%lld)",
                (long long)s->heads, (long long)s->gqa, (long long)s->head_dim);
  // each field bounded before it enters a product (no check overflows)
  if (s->heads > kI32Half || s->gqa > kI32Half || s->head_dim > kI32Half || s->q_row > kI32Half ||
      s->q_head > kI32Half || s->out_row > kI32Half || s->gate_offset > kI32Half ||
      s->heads % s->gqa || s->q_head < s->head_dim || s->heads * s->q_head > s->q_row ||
      s->heads * s->head_dim > s->out_row)
    return fail(HB_DECLINE_GEOMETRY, "invalid generated attention geometry");
  if (s->gate_offset >= 0 && s->gate_offset + s->heads * s->head_dim > s->q_row)
    return fail(HB_DECLINE_GEOMETRY, "gate_offset %lld + heads*head_dim exceeds q_row %lld",
                (long long)s->gate_offset, (long long)s->q_row);
  if (!decode_serves(s->head_dim, s->gqa))
    return fail(HB_DECLINE_HEAD_DIM,
                "head_dim out of domain (served: 128, 256 with gqa 1/2/4/8); got head_dim=%lld gqa=%lld",
                (long long)s->head_dim, (long long)s->gqa);
  if (s->q_row % 8 || s->q_head % 8 || s->out_row % 8 || (s->gate_offset > 0 && s->gate_offset % 8))
    return fail(HB_ERR_ARG,
                "q_row, q_head, out_row and gate_offset must be multiples of 8 elements (16 bytes)");
  return HB_OK;
}

hb_status check_call(const hb_attn_spec* s, const hb_attn_call* c) {
  if (!c) return fail(HB_ERR_ARG, "attention call is null");
  if (c->rows <= 0) return fail(HB_DECLINE_EMPTY, "empty shape (rows=%lld)", (long long)c->rows);
  if (!c->q || !c->keys || !c->values || !c->output)
    return fail(HB_ERR_ARG, "null q/keys/values/output pointer");
  if (!aligned16(c->q) || !aligned16(c->keys) || !aligned16(c->values) || !aligned16(c->output))
    return fail(HB_ERR_ARG, "q/keys/values/output must be 16-byte aligned");
  if (c->past < 0) return fail(HB_ERR_ARG, "negative past");
  if (!call_in_range(c->rows, c->past) || c->capacity > kMaxPositions)
    return fail(HB_ERR_ARG, "rows %lld / past %lld / capacity %lld beyond the served range",
                (long long)c->rows, (long long)c->past, (long long)c->capacity);
  const int64_t n_max = c->past + c->rows;
  if (c->kv_stride % 8) return fail(HB_ERR_ARG, "kv_stride must be a multiple of 8 elements");
  if (c->kv_stride < n_max * s->head_dim)
    return fail(HB_ERR_ARG, "kv_stride %lld cannot hold past+rows=%lld positions",
                (long long)c->kv_stride, (long long)n_max);
  if (c->capacity > 0 && (n_max > c->capacity || c->kv_stride < c->capacity * s->head_dim))
    return fail(HB_ERR_ARG, "past+rows=%lld exceeds the KV reserve (capacity %lld)",
                (long long)n_max, (long long)c->capacity);
  if (!(c->scale == c->scale)) return fail(HB_ERR_ARG, "scale is NaN");
  return HB_OK;
}

namespace {

struct DecodePlan {
  int64_t units;
  int chunk, nsplit, ranges;
  size_t counters_off, partials_off, bytes;
};

DecodePlan plan_decode(const hb_attn_spec* s, int64_t nseq, int64_t rows, int64_t max_n,
                       int64_t total_positions) {
  DecodePlan p;
  const int64_t hkv = s->heads / s->gqa;
  p.units = mul_sat(mul_sat(nseq, rows), hkv);
  p.chunk = decode_chunk(mul_sat(total_positions, hkv), p.units, max_n, device_sms());
  p.nsplit = int((max_n + p.chunk - 1) / p.chunk);
  p.ranges = decode_ranges(mul_sat(total_positions, hkv), s->gqa, device_sms());
  p.counters_off = kWsHeader;
  p.partials_off = p.counters_off + align256(size_t(mul_sat(p.units, sizeof(unsigned))));
  // partial slots: [unit][split] for the split forms, [range + unit] for
  // the balanced ranges
  const int64_t split_slots = mul_sat(p.units, p.nsplit);
  const int64_t range_slots = p.units + p.ranges;
  const int64_t partial_bytes =
      mul_sat(split_slots > range_slots ? split_slots : range_slots,
              mul_sat(int64_t(decode_partial_floats(s->gqa, s->head_dim)), sizeof(float)));
  p.bytes = p.partials_off + align256(size_t(partial_bytes));
  return p;
}

// Positions summed over the rows of one sequence: row r sees past + r + 1.
// (rows and past within call_in_range: the sum fits in 64 bits)
int64_t row_positions(int64_t past, int64_t rows) { return rows * past + rows * (rows + 1) / 2; }

}  // namespace

hb_status check_ws(void* ws, size_t have, size_t need) {
  if (!ws) return fail(HB_ERR_WORKSPACE, "workspace is null (need %zu bytes)", need);
  if (reinterpret_cast<uintptr_t>(ws) & 255)
    return fail(HB_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if (have < need) return fail(HB_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", have, need);
  return HB_OK;
}

// Status word of the entry points that take no workspace (hb_gdn_decode,
// hb_attn_decode_noalloc): zero when the module loads, raised by a kernel
// whose bounded wait ran out, read and cleared by hb_device_status.
static __device__ int g_device_status;

namespace {

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// A driver function reached through the runtime's entry point, so that the
// library keeps no link-time libcuda dependency (it loads on machines
// without a driver, where only the host-side checks run).
template <class Fn>
Fn driver_fn(const char* name) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(ptr);
}

// Unique id of the current context (0 on success), non-zero without one.
int current_context_id(unsigned long long* id) {
  static const CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  if (!get_current || !get_id) return 1;
  CUcontext c = nullptr;
  if (get_current(&c) != CUDA_SUCCESS || !c) return 1;
  return get_id(c, id) == CUDA_SUCCESS ? 0 : 1;
}

}  // namespace

cudaError_t symbol_address(SymbolCache& cache, const void* symbol, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int r = cache.get(dev, current_context_id,
                          [symbol](void** p) { return int(cudaGetSymbolAddress(p, symbol)); }, out);
  if (r < 0) return cudaErrorInvalidDevice;
  return cudaError_t(r);
}

cudaError_t device_status_word(int** out) {
  static SymbolCache cache;
  void* p = nullptr;
  cudaError_t e = symbol_address(cache, reinterpret_cast<const void*>(&g_device_status), &p);
  *out = static_cast<int*>(p);
  return e;
}

int device_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::atomic<int>& v = cache[dev & 63];
  int n = v.load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    v.store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace hb

using namespace hb;

extern "C" {

int hb_version(void) { return (0 << 16) | 1; }

const char* hb_last_error(void) { return g_err; }

const char* hb_status_name(int status) {
  switch (status) {
    case HB_OK: return "HB_OK";
    case HB_DECLINE_EMPTY: return "HB_DECLINE_EMPTY";
    case HB_DECLINE_HEAD_DIM: return "HB_DECLINE_HEAD_DIM";
    case HB_DECLINE_GEOMETRY: return "HB_DECLINE_GEOMETRY";
    case HB_DECLINE_SINK: return "HB_DECLINE_SINK";
    case HB_ERR_ARG: return "HB_ERR_ARG";
    case HB_ERR_WORKSPACE: return "HB_ERR_WORKSPACE";
    case HB_ERR_CUDA: return "HB_ERR_CUDA";
    case HB_ERR_TIMEOUT: return "HB_ERR_TIMEOUT";
    case HB_ERR_NCCL: return "HB_ERR_NCCL";
    default: return "HB_UNKNOWN";
  }
}

hb_status hb_workspace_init(void* ws, size_t bytes, hb_stream_t stream) {
  if (!ws || bytes < kWsHeader) return fail(HB_ERR_WORKSPACE, "workspace null or under 256 bytes");
  cudaError_t e = cudaMemsetAsync(ws, 0, bytes, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hb_workspace_init");
  return HB_OK;
}

// Reads the device status word at `word` on `stream`, clears it when set,
// and turns its code into a status.
static hb_status read_status_word(int* word, hb_stream_t stream, const char* what) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int code = 0;
  cudaError_t e = cudaMemcpyAsync(&code, word, sizeof code, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, what);
  if (code == 0) return HB_OK;
  e = cudaMemsetAsync(word, 0, sizeof code, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, what);
  if (code == kStatusTimeout) return fail(HB_ERR_TIMEOUT, "a bounded device wait ran out");
  return fail(HB_ERR_ARG, "a kernel met a misaligned or invalid table entry (code %d)", code);
}

hb_status hb_workspace_status(void* ws, size_t bytes, hb_stream_t stream) {
  if (!ws || bytes < kWsHeader) return fail(HB_ERR_WORKSPACE, "workspace null or under 256 bytes");
  return read_status_word(static_cast<int*>(ws), stream, "hb_workspace_status");
}

hb_status hb_device_status(hb_stream_t stream) {
  int* word = nullptr;
  cudaError_t e = device_status_word(&word);
  if (e != cudaSuccess) return cuda_fail(e, "hb_device_status set-up");
  return read_status_word(word, stream, "hb_device_status");
}

size_t hb_attn_decode_workspace_bytes(const hb_attn_spec* s, const hb_attn_call* c) {
  if (check_spec(s) != HB_OK || !c || c->rows <= 0 || !call_in_range(c->rows, c->past)) return 0;
  return plan_decode(s, 1, c->rows, c->past + c->rows, row_positions(c->past, c->rows)).bytes;
}

// Launches the decode kernel of one sequence on a validated call with the
// workspace `ws` laid out by plan `pl`.
static DecodeLaunch decode_launch_of(const hb_attn_spec* s, const hb_attn_call* c, const DecodePlan& pl,
                                     void* ws, int* status) {
  DecodeLaunch L;
  L.seqs = nullptr;
  L.one.q = c->q;
  L.one.keys = c->keys;
  L.one.values = c->values;
  L.one.output = c->output;
  L.one.past = c->past;
  L.one.kv_stride = c->kv_stride;
  L.nseq = 1;
  L.rows = c->rows;
  L.hkv = s->heads / s->gqa;
  L.gqa = s->gqa;
  L.head_dim = s->head_dim;
  L.q_row = s->q_row;
  L.q_head = s->q_head;
  L.out_row = s->out_row;
  L.gate_offset = s->gate_offset;
  L.scale = c->scale;
  L.chunk = pl.chunk;
  L.nsplit = pl.nsplit;
  L.ranges = pl.ranges;
  char* base = static_cast<char*>(ws);
  L.status = status ? status : reinterpret_cast<int*>(base);
  L.counters = reinterpret_cast<unsigned*>(base + pl.counters_off);
  L.partials = reinterpret_cast<float*>(base + pl.partials_off);
  return L;
}

static hb_status decode_launch(const hb_attn_spec* s, const hb_attn_call* c, const DecodePlan& pl,
                               void* ws, hb_stream_t stream, int* status = nullptr) {
  const DecodeLaunch L = decode_launch_of(s, c, pl, ws, status);
  cudaError_t e = launch_attn_decode(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attn_decode launch");
  return HB_OK;
}

static hb_status decode_common(const hb_attn_spec* s, const hb_attn_call* c, void* ws,
                               size_t ws_bytes, hb_stream_t stream) {
  hb_status r = check_spec(s);
  if (r != HB_OK) return r;
  if ((r = check_call(s, c)) != HB_OK) return r;
  const DecodePlan pl = plan_decode(s, 1, c->rows, c->past + c->rows, row_positions(c->past, c->rows));
  if ((r = check_ws(ws, ws_bytes, pl.bytes)) != HB_OK) return r;
  return decode_launch(s, c, pl, ws, stream);
}

// The allocation-free variant: the same kernel and plan, with the static
// scratch of attn_decode.cu as its workspace.  Its split counters must start
// at zero, and the array keeps whatever the previous call left, so they are
// cleared (one cudaMemsetAsync, no allocation) on `stream` before the
// launch.  A bounded wait that runs out is recorded in the per-device status
// word (hb_device_status), which no later call clears.
hb_status hb_attn_decode_noalloc(const hb_attn_spec* s, const hb_attn_call* c,
                                 hb_stream_t stream) {
  hb_status r = check_spec(s);
  if (r != HB_OK) return r;
  if ((r = check_call(s, c)) != HB_OK) return r;
  const DecodePlan pl = plan_decode(s, 1, c->rows, c->past + c->rows, row_positions(c->past, c->rows));
  if (pl.bytes > size_t(HB_NOALLOC_SCRATCH_BYTES))
    return fail(HB_ERR_WORKSPACE,
                "hb_attn_decode_noalloc: this call needs %zu bytes of scratch, above the static "
                "maximum HB_NOALLOC_SCRATCH_BYTES = %zu; use hb_attn_decode with a workspace",
                pl.bytes, size_t(HB_NOALLOC_SCRATCH_BYTES));
  void* scratch = nullptr;
  cudaError_t e = noalloc_scratch(&scratch);
  if (e != cudaSuccess) return cuda_fail(e, "hb_attn_decode_noalloc scratch set-up");
  int* status = nullptr;
  if ((e = device_status_word(&status)) != cudaSuccess)
    return cuda_fail(e, "hb_attn_decode_noalloc status set-up");
  // the split counters start at zero; the status word is the per-device
  // one, kept until hb_device_status reads it
  char* base = static_cast<char*>(scratch);
  e = cudaMemsetAsync(base + pl.counters_off, 0, pl.partials_off - pl.counters_off,
                      reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hb_attn_decode_noalloc scratch clear");
  return decode_launch(s, c, pl, scratch, stream, status);
}

hb_status hb_attn_decode(const hb_attn_spec* s, const hb_attn_call* c, void* ws, size_t ws_bytes,
                         hb_stream_t stream) {
  return decode_common(s, c, ws, ws_bytes, stream);
}

size_t hb_attn_decode_batch_workspace_bytes(const hb_attn_spec* s, int64_t nseq, int64_t max_past,
                                            int64_t sum_past) {
  if (check_spec(s) != HB_OK || nseq <= 0 || nseq > 65535 || max_past < 0 ||
      max_past > kMaxPositions || sum_past > kMaxPositions * 65535)
    return 0;
  const int64_t total = sum_past > 0 ? sum_past + nseq : nseq * (max_past + 1);
  return plan_decode(s, nseq, 1, max_past + 1, total).bytes;
}

hb_status hb_attn_decode_batch(const hb_attn_spec* s, const hb_decode_seq* seqs, int64_t nseq,
                               int64_t max_past, int64_t sum_past, void* ws, size_t ws_bytes,
                               hb_stream_t stream) {
  hb_status r = check_spec(s);
  if (r != HB_OK) return r;
  if (nseq <= 0) return fail(HB_DECLINE_EMPTY, "empty batch");
  if (!seqs) return fail(HB_ERR_ARG, "sequence table is null");
  if (max_past < 0) return fail(HB_ERR_ARG, "negative max_past");
  if (nseq > 65535) return fail(HB_DECLINE_GEOMETRY, "at most 65535 sequences per call");
  if (max_past > kMaxPositions || sum_past > kMaxPositions * 65535)
    return fail(HB_ERR_ARG, "max_past / sum_past beyond the served range");
  const int64_t total = sum_past > 0 ? sum_past + nseq : nseq * (max_past + 1);
  const DecodePlan pl = plan_decode(s, nseq, 1, max_past + 1, total);
  if ((r = check_ws(ws, ws_bytes, pl.bytes)) != HB_OK) return r;
  DecodeLaunch L;
  memset(&L.one, 0, sizeof L.one);
  L.seqs = seqs;
  L.nseq = nseq;
  L.rows = 1;
  L.hkv = s->heads / s->gqa;
  L.gqa = s->gqa;
  L.head_dim = s->head_dim;
  L.q_row = s->q_row;
  L.q_head = s->q_head;
  L.out_row = s->out_row;
  L.gate_offset = s->gate_offset;
  // the scale of a batch: 1/sqrt(head_dim), as ModelShape::scale without attn_scale
  L.scale = 1.0f / std::sqrt(float(s->head_dim));
  L.chunk = pl.chunk;
  L.nsplit = pl.nsplit;
  L.ranges = pl.ranges;
  char* base = static_cast<char*>(ws);
  L.status = reinterpret_cast<int*>(base);
  L.counters = reinterpret_cast<unsigned*>(base + pl.counters_off);
  L.partials = reinterpret_cast<float*>(base + pl.partials_off);
  cudaError_t e = launch_attn_decode(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attn_decode_batch launch");
  return HB_OK;
}

hb_status hb_decode_shard_plan(const int64_t* cost, int64_t nseq, int32_t parts, int32_t* part,
                               int64_t* load) {
  if (nseq <= 0) return fail(HB_DECLINE_EMPTY, "empty batch");
  if (!cost || !part) return fail(HB_ERR_ARG, "cost or part is null");
  if (nseq > (int64_t(1) << 24) || parts < 1 || parts > 4096)
    return fail(HB_ERR_ARG, "nseq %lld / parts %d out of range (nseq <= 2^24, parts 1..4096)",
                (long long)nseq, int(parts));
  int64_t total = 0;
  for (int64_t i = 0; i < nseq; ++i) {
    if (cost[i] < 0 || cost[i] >= (int64_t(1) << 62) - total)
      return fail(HB_ERR_ARG, "cost[%lld] negative or the costs' sum at or above 2^62",
                  (long long)i);
    total += cost[i];
  }
  std::vector<int64_t> order(static_cast<size_t>(nseq));
  std::iota(order.begin(), order.end(), int64_t(0));
  std::stable_sort(order.begin(), order.end(),
                   [cost](int64_t a, int64_t b) { return cost[a] > cost[b]; });
  // least-loaded GPU first, the lowest index on a tie
  typedef std::pair<int64_t, int32_t> Bin;
  std::priority_queue<Bin, std::vector<Bin>, std::greater<Bin>> bins;
  for (int32_t g = 0; g < parts; ++g) bins.push(Bin(0, g));
  std::vector<int64_t> sums(static_cast<size_t>(parts), 0);
  for (int64_t i : order) {
    Bin b = bins.top();
    bins.pop();
    part[i] = b.second;
    b.first += cost[i];
    sums[size_t(b.second)] = b.first;
    bins.push(b);
  }
  if (load) std::copy(sums.begin(), sums.end(), load);
  return HB_OK;
}

// Rows from which the tensor-core kernel takes a prefill block; shorter
// blocks go to the decode kernel, as the reference serves the rows a block
// kernel does not cover with its decode kernel.

static bool prefill_on_tensor_cores(const hb_attn_spec* s, const hb_attn_call* c) {
  return prefill_serves(s->head_dim) && c->rows >= kPrefillMinRows &&
         c->past + c->rows < (int64_t(1) << 31) &&
         (s->gate_offset < 0 || s->gate_offset % 8 == 0);
}

size_t hb_attn_prefill_workspace_bytes(const hb_attn_spec* s, const hb_attn_call* c) {
  if (check_spec(s) != HB_OK || !c || c->rows <= 0 || !call_in_range(c->rows, c->past)) return 0;
  if (prefill_on_tensor_cores(s, c)) return kWsHeader;
  return hb_attn_decode_workspace_bytes(s, c);
}

hb_status hb_attn_prefill(const hb_attn_spec* s, const hb_attn_call* c, void* ws, size_t ws_bytes,
                          hb_stream_t stream) {
  hb_status r = check_spec(s);
  if (r != HB_OK) return r;
  if ((r = check_call(s, c)) != HB_OK) return r;
  if (!prefill_on_tensor_cores(s, c)) return decode_common(s, c, ws, ws_bytes, stream);
  if ((r = check_ws(ws, ws_bytes, kWsHeader)) != HB_OK) return r;
  PrefillLaunch L;
  L.q = c->q;
  L.keys = c->keys;
  L.values = c->values;
  L.out = c->output;
  L.q_row = s->q_row;
  L.out_row = s->out_row;
  L.gate_offset = s->gate_offset;
  L.kv_stride = c->kv_stride;
  L.rows = c->rows;
  L.past = c->past;
  L.heads = s->heads;
  L.gqa = s->gqa;
  L.hkv = s->heads / s->gqa;
  L.scale = c->scale;
  L.status = static_cast<int*>(ws);
  cudaError_t e = launch_attn_prefill(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attn_prefill launch");
  return HB_OK;
}

hb_status hb_kv_append(const hb_kv_spec* s, const hb_kv_call* c, hb_stream_t stream) {
  if (!s || !c) return fail(HB_ERR_ARG, "kv spec or call is null");
  // bounds before products: no check may overflow on a hostile record
  const bool valid = s->heads > 0 && s->head_dim > 0 && s->max_batch > 0 && s->stride > 0 &&
                     s->stride <= 0x3FFFFFFF && s->head_dim <= s->stride &&
                     s->heads <= 0x7FFFFFFF / (2 * s->head_dim) && s->capacity >= s->max_batch &&
                     s->capacity <= s->stride / s->head_dim;
  if (!valid) return fail(HB_DECLINE_GEOMETRY, "invalid generated KV reserve geometry");
  if (c->rows <= 0) return fail(HB_DECLINE_EMPTY, "empty KV append");
  if (!c->keys || !c->values || !c->input_keys || !c->input_values)
    return fail(HB_ERR_ARG, "null KV append pointer");
  if (c->rows > s->max_batch || c->past < 0 || c->past > s->capacity - c->rows)
    return fail(HB_ERR_ARG, "append of %lld rows at %lld exceeds the reserve (capacity %lld, batch %lld)",
                (long long)c->rows, (long long)c->past, (long long)s->capacity,
                (long long)s->max_batch);
  cudaError_t e = launch_kv_append(*s, *c, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  return HB_OK;
}

static hb_status check_front(const hb_attn_spec* s, const hb_kv_spec* kv, const hb_front_spec* f,
                             const hb_front_call* c) {
  hb_status r = check_spec(s);
  if (r != HB_OK) return r;
  if (!kv || !f || !c) return fail(HB_ERR_ARG, "kv spec, front spec or call is null");
  const int64_t hkv = s->heads / s->gqa;
  if (kv->heads != hkv || kv->head_dim != s->head_dim)
    return fail(HB_DECLINE_GEOMETRY, "KV spec (heads %lld, head_dim %lld) does not match the "
                "attention spec (%lld KV heads, head_dim %lld)",
                (long long)kv->heads, (long long)kv->head_dim, (long long)hkv,
                (long long)s->head_dim);
  if (!front_serves(s->head_dim, f->rotary))
    return fail(HB_DECLINE_HEAD_DIM, "head_dim %lld / rotary %lld out of domain (served: head_dim "
                "128 or 256, rotary a multiple of 32 up to head_dim)",
                (long long)s->head_dim, (long long)f->rotary);
  if (!(f->eps == f->eps) || f->eps < 0.f) return fail(HB_ERR_ARG, "eps is NaN or negative");
  if (c->rows <= 0) return fail(HB_DECLINE_EMPTY, "empty shape (rows=%lld)", (long long)c->rows);
  if (c->past < 0) return fail(HB_ERR_ARG, "negative past");
  if (!c->q || !c->k || !c->v || !c->q_norm || !c->k_norm ||
      (f->rotary > 0 && (!c->cos || !c->sin)) || (!c->keys != !c->values))
    return fail(HB_ERR_ARG, "null front-end pointer");
  const void* ptrs[] = {c->q, c->k, c->v, c->q_norm, c->k_norm, c->cos, c->sin, c->keys, c->values};
  for (const void* ptr : ptrs)
    if (ptr && !aligned16(ptr)) return fail(HB_ERR_ARG, "front-end pointers must be 16-byte aligned");
  if (c->rows > 0x3FFFFFFF / (s->heads + hkv) || c->past > kI32Half)
    return fail(HB_ERR_ARG, "rows or past out of range");
  if (c->keys) {
    const bool valid = kv->max_batch > 0 && kv->capacity >= kv->max_batch &&
                       kv->capacity * kv->head_dim <= kv->stride && kv->stride <= 0x3FFFFFFF &&
                       kv->stride % 8 == 0;
    if (!valid) return fail(HB_DECLINE_GEOMETRY, "invalid generated KV reserve geometry");
    if (c->rows > kv->max_batch || c->past + c->rows > kv->capacity)
      return fail(HB_ERR_ARG, "append of %lld rows at %lld exceeds the reserve (capacity %lld, batch %lld)",
                  (long long)c->rows, (long long)c->past, (long long)kv->capacity,
                  (long long)kv->max_batch);
  }
  return HB_OK;
}

hb_status hb_attn_front(const hb_attn_spec* s, const hb_kv_spec* kv, const hb_front_spec* f,
                        const hb_front_call* c, hb_stream_t stream) {
  hb_status r = check_front(s, kv, f, c);
  if (r != HB_OK) return r;
  const int64_t hkv = s->heads / s->gqa;
  FrontLaunch L;
  L.q = c->q;
  L.k = c->k;
  L.v = c->v;
  L.q_norm = c->q_norm;
  L.k_norm = c->k_norm;
  L.cos = c->cos;
  L.sin = c->sin;
  L.keys = c->keys;
  L.values = c->values;
  L.q_row = s->q_row;
  L.kv_row = hkv * s->head_dim;
  L.kv_stride = kv->stride;
  L.past = c->past;
  L.rows = c->rows;
  L.heads = s->heads;
  L.kv_heads = hkv;
  L.head_dim = s->head_dim;
  L.rotary = f->rotary;
  L.eps = f->eps;
  L.gemma = f->gemma != 0;
  cudaError_t e = launch_attn_front(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attn_front launch");
  return HB_OK;
}

static hb_status check_gdn(const hb_gdn_shape* s, const hb_gdn_call* c) {
  if (!s || !c) return fail(HB_ERR_ARG, "DeltaNet shape or call is null");
  const int64_t lim = int64_t(1) << 16;
  if (s->nk <= 0 || s->nv <= 0 || s->nv % s->nk || s->hkd <= 0 || s->hvd <= 0 || s->nk > lim ||
      s->nv > lim || s->hkd > lim || s->hvd > lim ||
      (2 * s->nk * s->hkd + s->nv * s->hvd) > 0x7FFFFFFF / 16 ||
      s->nv * s->hkd * s->hvd > 0x7FFFFFFF / 4)
    return fail(HB_DECLINE_GEOMETRY, "invalid generated DeltaNet geometry");
  if (!gdn_decode_serves(*s))
    return fail(HB_DECLINE_HEAD_DIM, "DeltaNet head dims not served (hkd 64/128, hvd multiple of 32)");
  if (c->rows <= 0) return fail(HB_DECLINE_EMPTY, "empty DeltaNet block");
  if (!c->state || !c->output || !c->qkv || !c->beta || !c->decay)
    return fail(HB_ERR_ARG, "null DeltaNet pointer");
  if (c->l2 && !(c->eps >= 0.f)) return fail(HB_ERR_ARG, "invalid L2 eps");
  return HB_OK;
}

// The recurrence on a validated call; its status word is `status`.
static hb_status gdn_decode_launch(const hb_gdn_shape* s, const hb_gdn_call* c, int* status,
                                   hb_stream_t stream) {
  GdnLaunch L;
  L.shape = *s;
  L.call = *c;
  L.scale = 1.0f / std::sqrt(float(s->hkd));
  L.status = status;
  cudaError_t e = launch_gdn_decode(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_decode launch");
  return HB_OK;
}

hb_status hb_gdn_decode(const hb_gdn_shape* s, const hb_gdn_call* c, hb_stream_t stream) {
  hb_status r = check_gdn(s, c);
  if (r != HB_OK) return r;
  int* status = nullptr;
  cudaError_t e = device_status_word(&status);
  if (e != cudaSuccess) return cuda_fail(e, "gdn_decode status set-up");
  return gdn_decode_launch(s, c, status, stream);
}

// Positions from which the chunked tensor-core kernels take a block; shorter
// blocks run the recurrence in order.
static constexpr int64_t kGdnChunkMinRows = 128;

static bool gdn_chunked(const hb_gdn_shape* s, const hb_gdn_call* c) {
  const uintptr_t mis = reinterpret_cast<uintptr_t>(c->qkv) | reinterpret_cast<uintptr_t>(c->state) |
                        reinterpret_cast<uintptr_t>(c->output);
  return gdn_prefill_serves(*s) && c->rows >= kGdnChunkMinRows && (mis & 15) == 0 &&
         c->rows < (int64_t(1) << 31);
}

static hb_status check_gdn_shape(const hb_gdn_shape* s) {
  const int64_t lim = int64_t(1) << 16;
  if (s->nk <= 0 || s->nv <= 0 || s->nv % s->nk || s->hkd <= 0 || s->hvd <= 0 || s->nk > lim ||
      s->nv > lim || s->hkd > lim || s->hvd > lim ||
      (2 * s->nk * s->hkd + s->nv * s->hvd) > 0x7FFFFFFF / 16)
    return fail(HB_DECLINE_GEOMETRY, "invalid generated DeltaNet geometry");
  return HB_OK;
}

static hb_status check_gdn_front(const hb_gdn_shape* s, const hb_gdn_front_call* c, void* ws,
                                 size_t ws_bytes) {
  if (!s || !c) return fail(HB_ERR_ARG, "DeltaNet shape or front call is null");
  hb_status r = check_gdn_shape(s);
  if (r != HB_OK) return r;
  const int64_t conv = 2 * s->nk * s->hkd + s->nv * s->hvd;
  if (!gdn_front_serves(conv, c->ck))
    return fail(HB_DECLINE_GEOMETRY, "DeltaNet conv not served (ck 1..8, conv width a multiple of 4)");
  if (c->rows <= 0) return fail(HB_DECLINE_EMPTY, "empty DeltaNet block");
  if (c->rows >= (int64_t(1) << 31) / s->nv || c->rows * conv >= (int64_t(1) << 40))
    return fail(HB_ERR_ARG, "DeltaNet block too long");
  if (!c->qkv || !c->conv_state || !c->conv_weight || !c->ab || !c->dt_bias || !c->a_log ||
      !c->beta || !c->decay)
    return fail(HB_ERR_ARG, "null DeltaNet front pointer");
  if (!aligned16(c->qkv)) return fail(HB_ERR_ARG, "qkv must be 16-byte aligned");
  return check_ws(ws, ws_bytes, kWsHeader);
}

static hb_status check_gdn_norm(const hb_gdn_shape* s, const hb_gdn_norm_call* c) {
  if (!s || !c) return fail(HB_ERR_ARG, "DeltaNet shape or norm call is null");
  hb_status r = check_gdn_shape(s);
  if (r != HB_OK) return r;
  if (c->rows <= 0) return fail(HB_DECLINE_EMPTY, "empty DeltaNet block");
  if (c->rows >= (int64_t(1) << 40) / (s->nv * s->hvd)) return fail(HB_ERR_ARG, "DeltaNet block too long");
  if (!c->x || !c->z || !c->weight || !c->out) return fail(HB_ERR_ARG, "null DeltaNet norm pointer");
  if (!(c->eps >= 0.f) || c->eps == INFINITY) return fail(HB_ERR_ARG, "invalid gated-norm eps");
  return HB_OK;
}

hb_status hb_gdn_front(const hb_gdn_shape* s, const hb_gdn_front_call* c, void* ws, size_t ws_bytes,
                       hb_stream_t stream) {
  hb_status r = check_gdn_front(s, c, ws, ws_bytes);
  if (r != HB_OK) return r;
  const int64_t conv = 2 * s->nk * s->hkd + s->nv * s->hvd;
  GdnFrontLaunch L;
  L.qkv = c->qkv;
  L.state = c->conv_state;
  L.weight = c->conv_weight;
  L.ab = c->ab;
  L.dt_bias = c->dt_bias;
  L.a_log = c->a_log;
  L.beta = c->beta;
  L.decay = c->decay;
  L.rows = c->rows;
  L.conv = conv;
  L.ck = c->ck;
  L.nv = s->nv;
  L.status = static_cast<int*>(ws);
  cudaError_t e = launch_gdn_front(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_front launch");
  return HB_OK;
}

hb_status hb_gdn_gated_norm(const hb_gdn_shape* s, const hb_gdn_norm_call* c, hb_stream_t stream) {
  hb_status r = check_gdn_norm(s, c);
  if (r != HB_OK) return r;
  GdnNormLaunch L;
  L.x = c->x;
  L.z = c->z;
  L.weight = c->weight;
  L.out = c->out;
  L.out_f32 = c->out_f32;
  L.rows = c->rows;
  L.nv = s->nv;
  L.hvd = s->hvd;
  L.eps = c->eps;
  cudaError_t e = launch_gdn_gated_norm(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_gated_norm launch");
  return HB_OK;
}

size_t hb_gdn_prefill_workspace_bytes(const hb_gdn_shape* s, int64_t rows) {
  // blocks the chunked kernels never take (rows >= 2^31, heads beyond the
  // geometry's limit) need only the header
  if (!s || rows <= 0 || rows >= (int64_t(1) << 31) || s->nk > (int64_t(1) << 16) ||
      s->nv > (int64_t(1) << 16))
    return kWsHeader;
  if (!gdn_prefill_serves(*s)) return kWsHeader;
  return gdn_prefill_plan(*s, rows).bytes;
}

hb_status hb_gdn_prefill(const hb_gdn_shape* s, const hb_gdn_call* c, void* ws, size_t ws_bytes,
                         hb_stream_t stream) {
  hb_status r = check_gdn(s, c);
  if (r != HB_OK) return r;
  if (!gdn_chunked(s, c)) {  // the recurrence in order, its status in the workspace
    if ((r = check_ws(ws, ws_bytes, kWsHeader)) != HB_OK) return r;
    return gdn_decode_launch(s, c, static_cast<int*>(ws), stream);
  }
  const GdnPrefillPlan pl = gdn_prefill_plan(*s, c->rows);
  if ((r = check_ws(ws, ws_bytes, pl.bytes)) != HB_OK) return r;
  GdnLaunch L;
  L.shape = *s;
  L.call = *c;
  L.scale = 1.0f / std::sqrt(float(s->hkd));
  L.status = static_cast<int*>(ws);
  cudaError_t e = launch_gdn_prefill(L, pl, ws, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_prefill launch");
  return HB_OK;
}

}  // extern "C"

namespace hb {

hb_status hb_gdn_check(const hb_gdn_shape* s, const hb_gdn_call* c) { return check_gdn(s, c); }

hb_status attn_layer_row(const hb_attn_spec* s, const hb_kv_spec* kv, const hb_front_spec* f,
                         const hb_front_call* fc, const hb_attn_call* ac, void* ws, size_t ws_bytes,
                         hb_stream_t stream, bool* served) {
  *served = false;
  if (!s || !kv || !f || !fc || !ac || fc->rows != 1 || ac->rows != 1 || fc->past != ac->past ||
      fc->q != ac->q || !fc->keys || fc->keys != ac->keys || fc->values != ac->values ||
      kv->stride != ac->kv_stride)
    return HB_OK;
  // both nodes' checks; a call either refuses goes the two-launch way,
  // which reports it as before
  if (check_front(s, kv, f, fc) != HB_OK || check_spec(s) != HB_OK || check_call(s, ac) != HB_OK)
    return HB_OK;
  const DecodePlan pl = plan_decode(s, 1, ac->rows, ac->past + ac->rows, row_positions(ac->past, ac->rows));
  if (check_ws(ws, ws_bytes, pl.bytes) != HB_OK) return HB_OK;
  const DecodeLaunch L = decode_launch_of(s, ac, pl, ws, nullptr);
  DecodeFront F;
  F.k = fc->k;
  F.v = fc->v;
  F.q_norm = fc->q_norm;
  F.k_norm = fc->k_norm;
  F.cos = fc->cos;
  F.sin = fc->sin;
  F.rotary = f->rotary;
  F.eps = f->eps;
  F.gemma = f->gemma != 0;
  cudaError_t e = cudaSuccess;
  if (!launch_attn_decode_long(L, reinterpret_cast<cudaStream_t>(stream), &e, &F)) return HB_OK;
  *served = true;
  if (e != cudaSuccess) return cuda_fail(e, "attn_decode launch (with the front end)");
  return HB_OK;
}

hb_status gdn_layer_row(const hb_gdn_shape* s, const hb_gdn_front_call* fc, const hb_gdn_call* gc,
                        const hb_gdn_norm_call* nc, void* front_ws, size_t front_ws_bytes,
                        int* status, hb_stream_t stream, bool* served) {
  *served = false;
  if (!s || !fc || !gc || !nc || fc->rows != 1 || gc->rows != 1 || nc->rows != 1 ||
      !gdn_row_serves(*s, fc->ck) || gc->l2 != 1 || gc->qkv != fc->qkv || nc->x != gc->output ||
      !front_ws || front_ws_bytes < kWsHeader + kRowCounterBytes)
    return HB_OK;
  // the three nodes' own checks, all before anything launches
  hb_status r = check_gdn_front(s, fc, front_ws, front_ws_bytes);
  if (r == HB_OK) r = check_gdn(s, gc);
  if (r == HB_OK) r = check_gdn_norm(s, nc);
  if (r != HB_OK) {
    *served = true;
    return r;
  }
  const uintptr_t mis16 = reinterpret_cast<uintptr_t>(fc->conv_state) | reinterpret_cast<uintptr_t>(gc->state);
  if ((mis16 & 15) != 0 || (reinterpret_cast<uintptr_t>(fc->conv_weight) & 7) != 0) return HB_OK;
  *served = true;
  GdnRowLaunch L;
  L.shape = *s;
  L.qkv = fc->qkv;
  L.conv_state = fc->conv_state;
  L.conv_weight = fc->conv_weight;
  L.ab = fc->ab;
  L.dt_bias = fc->dt_bias;
  L.a_log = fc->a_log;
  L.state = gc->state;
  L.z = nc->z;
  L.norm_weight = nc->weight;
  L.out = nc->out;
  L.out_f32 = nc->out_f32;
  L.l2_eps = gc->eps;
  L.scale = 1.0f / std::sqrt(float(s->hkd));
  L.norm_eps = nc->eps;
  L.status = status;
  L.counters = reinterpret_cast<unsigned*>(static_cast<char*>(front_ws) + kWsHeader);
  cudaError_t e = launch_gdn_row(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_row launch");
  return HB_OK;
}

}  // namespace hb

