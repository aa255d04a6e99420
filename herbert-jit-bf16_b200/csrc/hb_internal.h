// hb_internal.h -- declarations shared between the host API layer
// (hb_api.cu) and the kernel translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>

#include "../../include/herbert_b200.h"

namespace hb {

// Once-per-device initialisation flag (function attributes are per device).
struct DeviceFlags {
  std::atomic<uint64_t> done{0};
  template <class F>
  cudaError_t once(F&& f) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = f();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
  }
};

// Codes of the device-side status word kept at the head of every workspace.
enum : int { kStatusOk = 0, kStatusTimeout = 1, kStatusArg = 2 };

// Layout of every workspace: a 256-byte header whose first int is the
// device-side status word, then the kernel's own sections (256-aligned).
constexpr size_t kWsHeader = 256;
inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// ----------------------------------------------------------- attn decode
struct DecodeLaunch {
  const hb_decode_seq* seqs;  // device table or nullptr
  hb_decode_seq one;          // the single sequence when seqs == nullptr
  int64_t nseq, rows, hkv, gqa, head_dim;
  int64_t q_row, q_head, out_row, gate_offset;
  float scale;
  int chunk, nsplit;  // splits of the cluster and tensor-core forms
  int ranges;         // CTAs of the balanced-range form
  int* status;
  unsigned* counters;
  float* partials;
};
bool decode_serves(int64_t head_dim, int64_t gqa);
// Device address of the static scratch of hb_attn_decode_noalloc on the
// current device (looked up on the first call per device and context).
cudaError_t noalloc_scratch(void** ptr);
// Positions per split of the decode kernel: `total_positions` summed over
// the `units` (row, KV head) pairs, each at most max_n long.
int decode_chunk(int64_t total_positions, int64_t units, int64_t max_n, int num_sms);
// CTAs of the balanced-range decode: `unit_positions` summed over the
// (row, KV head) units.
int decode_ranges(int64_t unit_positions, int64_t gqa, int num_sms);
size_t decode_partial_floats(int64_t gqa, int64_t head_dim);
cudaError_t launch_attn_decode(const DecodeLaunch& L, cudaStream_t st);
// The tensor-core form for one sequence of at most 16 x 128 positions at
// head_dim 256: returns false (nothing launched) when the call is not in
// its domain, else launches and sets *err.
bool launch_attn_decode_mma(const DecodeLaunch& L, cudaStream_t st, cudaError_t* err);
// The front end of a one-row call (head-norm-rope of q and k, kv-append of
// the row's position) for the long decode kernel to run itself.
struct DecodeFront {
  uint16_t* k;              // the row's k [hkv][head_dim]: normed and rotated in place
  const uint16_t* v;        // the row's v
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const uint16_t* cos;
  const uint16_t* sin;
  int64_t rotary;
  float eps;
  bool gemma;
};
// one sequence longer than 16 x 256 positions: split-KV on the tensor cores
// (false: not served, the CUDA-core kernel runs); with `front`, a one-row
// call that also runs its front end (q normed in place through L.one.q,
// k and v into L.one.keys / values at position L.one.past)
bool launch_attn_decode_long(const DecodeLaunch& L, cudaStream_t st, cudaError_t* err,
                             const DecodeFront* front = nullptr);

// ---------------------------------------------------------- attn prefill
struct PrefillLaunch {
  const uint16_t* q;
  const uint16_t* keys;
  const uint16_t* values;
  uint16_t* out;
  int64_t q_row, out_row, gate_offset, kv_stride;
  int64_t rows, past, heads, gqa, hkv;
  float scale;
  int* status;
  // context-parallel hop (cp): query rows [0, chunk) at positions q_pos0..,
  // rows [chunk, 2 chunk) at q_pos1..; the hop's K/V rows [0, chunk) hold
  // positions kpos[0].., rows [chunk, 2 chunk) kpos[1]..; kv_rows =
  // positions the K/V buffers hold.  The hop merges into the accumulators
  // at acc (cp_acc_bytes; merge = false on the first hop, which writes them).
  bool cp = false, merge = false;
  int64_t chunk = 0, q_pos0 = 0, q_pos1 = 0;
  int64_t kpos[2] = {0, 0};
  int64_t kv_rows = 0;
  float* acc = nullptr;
};
bool prefill_serves(int64_t head_dim);
cudaError_t launch_attn_prefill(const PrefillLaunch& L, cudaStream_t st);
// Bytes of the O and (m, l) accumulators of a context-parallel prefill over
// `rows` local query rows (O first, then (m, l)).
size_t cp_acc_bytes(int64_t heads, int64_t rows);
cudaError_t launch_attn_cp_finish(const PrefillLaunch& L, cudaStream_t st);

// ------------------------------------------------------------ kv append
cudaError_t launch_kv_append(const hb_kv_spec& s, const hb_kv_call& c, cudaStream_t st);

// ------------------------------------------- attention front end (norm, RoPE)
struct FrontLaunch {
  uint16_t* q;
  uint16_t* k;
  const uint16_t* v;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const uint16_t* cos;
  const uint16_t* sin;
  uint16_t* keys;    // nullptr: no append
  uint16_t* values;
  int64_t q_row, kv_row, kv_stride, past, rows;
  int64_t heads, kv_heads, head_dim, rotary;
  float eps;
  bool gemma;
};
bool front_serves(int64_t head_dim, int64_t rotary);
cudaError_t launch_attn_front(const FrontLaunch& L, cudaStream_t st);

// ------------------------------------------------- gdn front / gated norm
struct GdnFrontLaunch {
  float* qkv;               // [rows][conv], conv + SiLU in place
  float* state;             // [conv][ck]
  const uint16_t* weight;   // [conv][ck] bf16
  const float* ab;          // [rows][2 nv]
  const uint16_t* dt_bias;  // [nv] bf16
  const float* a_log;       // [nv]
  float* beta;              // [rows][nv]
  float* decay;             // [rows][nv]
  int64_t rows, conv, ck, nv;
  int* status;
};
struct GdnNormLaunch {
  const float* x;
  const float* z;
  const uint16_t* weight;
  uint16_t* out;
  float* out_f32;  // nullptr: not written
  int64_t rows, nv, hvd;
  float eps;
};
bool gdn_front_serves(int64_t conv, int64_t ck);
// one decode row of a whole DeltaNet layer (conv + gates + L2 + recurrence
// + gated norm) in one launch; beta, decay and the recurrence output are
// not materialised
struct GdnRowLaunch {
  hb_gdn_shape shape;
  float* qkv;                   // [conv] conv + SiLU in place
  float* conv_state;            // [conv][4], 16-byte aligned
  const uint16_t* conv_weight;  // [conv][4] bf16, 8-byte aligned
  const float* ab;
  const uint16_t* dt_bias;
  const float* a_log;
  float* state;                 // [nv][hkd][hvd], 16-byte aligned
  const float* z;
  const uint16_t* norm_weight;
  uint16_t* out;
  float* out_f32;
  float l2_eps, scale, norm_eps;
  int* status;
  unsigned* counters;           // [nk], zero between calls
};
// key heads whose write-back counters the one-row launch keeps (after the
// 256-byte header of the caller's front-end workspace)
constexpr int kRowMaxKeyHeads = 1024;
constexpr size_t kRowCounterBytes = kRowMaxKeyHeads * sizeof(unsigned);
bool gdn_row_serves(const hb_gdn_shape& s, int64_t ck);
cudaError_t launch_gdn_row(const GdnRowLaunch& L, cudaStream_t st);
// A one-row DeltaNet layer given as its three nodes' calls (front, L2 +
// recurrence, gated norm): when the fused kernel serves it (*served), the
// three calls' checks run first and then the one launch; otherwise nothing
// happens and the caller runs the nodes.
// A one-row attention layer given as its two nodes' calls (front end,
// decode): when both pass their checks and the long decode kernel serves
// the call (*served), that kernel runs the front end too, in one launch;
// otherwise nothing happens and the caller runs the nodes.
hb_status attn_layer_row(const hb_attn_spec* s, const hb_kv_spec* kv, const hb_front_spec* f,
                         const hb_front_call* fc, const hb_attn_call* ac, void* ws, size_t ws_bytes,
                         hb_stream_t stream, bool* served);
// front_ws holds the header, then the key heads' counters (kRowCounterBytes,
// zero between calls) when front_ws_bytes covers them.
hb_status gdn_layer_row(const hb_gdn_shape* s, const hb_gdn_front_call* fc, const hb_gdn_call* gc,
                        const hb_gdn_norm_call* nc, void* front_ws, size_t front_ws_bytes,
                        int* status, hb_stream_t stream, bool* served);

cudaError_t launch_gdn_front(const GdnFrontLaunch& L, cudaStream_t st);
cudaError_t launch_gdn_gated_norm(const GdnNormLaunch& L, cudaStream_t st);

// ------------------------------------------------------------ gdn decode
struct GdnLaunch {
  hb_gdn_shape shape;
  hb_gdn_call call;
  float scale;  // 1/sqrt(hkd), f32 as the reference computes it
  int* status;  // device status word (workspace header or device_status_word)
};
bool gdn_decode_serves(const hb_gdn_shape& s);
cudaError_t launch_gdn_decode(const GdnLaunch& L, cudaStream_t st);

// chunked prefill: workspace sections (bytes from the workspace start)
struct GdnPrefillPlan {
  int64_t nchunks;
  size_t off_Ac, off_Pc, off_Kt, off_M, off_U, bytes;
};
bool gdn_prefill_serves(const hb_gdn_shape& s);
GdnPrefillPlan gdn_prefill_plan(const hb_gdn_shape& s, int64_t rows);
cudaError_t launch_gdn_prefill(const GdnLaunch& L, const GdnPrefillPlan& pl, void* ws,
                               cudaStream_t st);

// Number of SMs of the current device (cached per device).
int device_sms();

// Device address, in the current context, of a file-scope __device__
// variable (`symbol` is the variable's address in host code, i.e. its
// host-side stand-in), cached per device and context (hb_host.h).
class SymbolCache;
cudaError_t symbol_address(SymbolCache& cache, const void* symbol, void** out);

// Device address of the status word of the entry points that take no
// workspace (hb_gdn_decode, hb_attn_decode_noalloc) on the current device;
// hb_device_status reads and clears it.
cudaError_t device_status_word(int** out);

// TMA tensor maps (hb_tma.cu): a rank-`rank` tiled map, element strides in
// bytes for dimensions 1.., no interleave, zero fill out of bounds; and the
// 2-D row-major case [rows][cols] with a row stride in elements.
bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                  const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
                  CUtensorMapSwizzle swizzle);
bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base,
               uint64_t rows, uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows,
               uint32_t box_cols, CUtensorMapSwizzle swizzle);

// A state geometry (hb_state_geometry) that the snapshot and mount entry
// points accept: layer offsets multiples of 2 x kv_heads x kv_reserve.
hb_status check_state_geometry(const hb_state_geometry* g);

// a x b for non-negative a, b, saturated at 2^62: a size no check accepts,
// so a hostile request is refused instead of wrapping around.
inline int64_t mul_sat(int64_t a, int64_t b) {
  int64_t r;
  if (__builtin_mul_overflow(a, b, &r) || r > (int64_t(1) << 62)) return int64_t(1) << 62;
  return r;
}

// Host-side checks and error reporting shared by the API translation units
// (hb_api.cu): a failure sets the thread-local message of hb_last_error.
hb_status fail(hb_status s, const char* fmt, ...);
hb_status cuda_fail(cudaError_t e, const char* what);
bool aligned16(const void* p);
hb_status check_spec(const hb_attn_spec* s);
hb_status check_call(const hb_attn_spec* s, const hb_attn_call* c);
hb_status check_ws(void* ws, size_t have, size_t need);
// hb_gdn_decode / hb_gdn_prefill's checks of a call (hb_api.cu).
hb_status hb_gdn_check(const hb_gdn_shape* s, const hb_gdn_call* c);
// Fewest rows hb_attn_prefill takes to the tensor-core kernel (fewer go to
// the decode kernel).
constexpr int64_t kPrefillMinRows = 64;
// hb_attn_prefill_host's blocks: rows per block (block_rows, or the
// library's choice when 0) and the number of blocks, the last one taking
// the rest.
int64_t prefill_host_block(int64_t rows, int64_t block_rows);
int64_t prefill_host_blocks(int64_t rows, int64_t block);

}  // namespace hb
