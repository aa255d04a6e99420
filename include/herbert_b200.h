/*
 * herbert_b200.h -- C ABI of the B200 (sm_100a) attention hot path of the
 * herbert-jit-bf16 Qwen3.5 engine: full-attention SDPA (GQA over a bf16 KV
 * cache, f32 softmax/accumulators, bf16 out, sigmoid output gate) in the
 * prefill and decode regimes, and the GatedDeltaNet mixer core (recurrent
 * decode over an f32 per-head state, chunked prefill).
 *
 * Conventions
 *  - Every pointer in a *_call record is DEVICE memory (except the *_host
 *    fields of hb_attn_host_call); records themselves are read on the host
 *    during the call (they may live on the stack).
 *  - Strides are in ELEMENTS (bf16 for attention, f32 for DeltaNet), as in
 *    the reference's call records.
 *  - Layouts are the reference's:
 *      KV cache  [kv_head][capacity][head_dim] bf16, head h at h*kv_stride
 *                (src/jit/model.rs:545-559; src/jit/execution/abi.rs:57-130)
 *      q row     [Q_0 .. Q_{H-1} | g_0 .. g_{H-1}] (src/jit/schedule.rs:109-133)
 *      DeltaNet  qkv [rows][2*nk*hkd + nv*hvd] f32, beta/decay [rows][nv] f32,
 *                state [nv][hkd][hvd] f32, out [rows][nv*hvd] f32
 *                (src/jit/target/x86/execution/delta.rs:519-607)
 *  - Calls are stream-ordered and never allocate.  Scratch ("workspace") is
 *    owned by the caller and sized by the *_workspace_bytes queries; a
 *    workspace must be zeroed once after allocation (hb_workspace_init) and
 *    every completed call leaves it reusable without re-zeroing.  Calls that
 *    share one workspace must be ordered on the GPU (same stream or events).
 *  - A shape the kernels do not serve is refused with an HB_DECLINE_* status,
 *    as the reference's emitters refuse with a named Decline
 *    (src/jit/ir.rs:177-230); the caller falls back.  Failures return
 *    HB_ERR_*; hb_last_error() gives a thread-local message.
 */
#ifndef HERBERT_B200_H
#define HERBERT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HB_API __attribute__((visibility("default")))
#else
#define HB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without including the CUDA headers; 0 = the legacy stream. */
typedef struct CUstream_st *hb_stream_t;

typedef enum hb_status {
    HB_OK = 0,
    /* Refusals (src/jit/ir.rs:177-230 Decline, abi.rs validate/check). */
    HB_DECLINE_EMPTY = 1,     /* Decline::Empty: zero rows / heads / length   */
    HB_DECLINE_HEAD_DIM = 2,  /* Decline::HeadDim: head_dim not served        */
    HB_DECLINE_GEOMETRY = 3,  /* "invalid generated ... geometry"             */
    HB_DECLINE_SINK = 4,      /* attention sink (not used by Qwen3.5)         */
    /* Errors. */
    HB_ERR_ARG = 10,          /* null / misaligned pointer, capacity exceeded */
    HB_ERR_WORKSPACE = 11,    /* workspace too small or misaligned            */
    HB_ERR_CUDA = 12,         /* a CUDA runtime call failed                   */
    HB_ERR_TIMEOUT = 13,      /* a bounded device wait ran out                */
    HB_ERR_NCCL = 14          /* the ring's communicator reported an error    */
} hb_status;

/* Library version, (major << 16) | minor. */
HB_API int hb_version(void);
/* Message of the last non-OK status on this thread ("" if none). */
HB_API const char *hb_last_error(void);
/* Static name of a status code. */
HB_API const char *hb_status_name(int status);
/* Zero a freshly allocated workspace (one cudaMemsetAsync on `stream`). */
HB_API hb_status hb_workspace_init(void *workspace, size_t bytes, hb_stream_t stream);
/* Read (and clear) the device-side status word of a workspace: HB_OK,
 * HB_ERR_TIMEOUT if a kernel's bounded wait ran out, HB_ERR_ARG if a kernel
 * met a misaligned table entry.  Synchronises `stream`. */
HB_API hb_status hb_workspace_status(void *workspace, size_t bytes, hb_stream_t stream);
/* The same for the entry points that take no workspace (hb_gdn_decode,
 * hb_attn_decode_noalloc): one status word per device, in static device
 * memory, raised by any of their calls on the current device and kept until
 * this call reads and clears it.  Synchronises `stream`.  No counterpart in
 * the reference, whose calls fail synchronously (src/jit/execution/plan.rs:6). */
HB_API hb_status hb_device_status(hb_stream_t stream);

/* ------------------------------------------------------------------ SDPA */

/* Per-layer attention geometry: AttentionSpec (src/jit/execution/abi.rs:136-151)
 * plus the gate position of the output-gate node (src/jit/schedule/lowering.rs:642-666). */
typedef struct hb_attn_spec {
    int64_t heads;       /* query heads (Qwen3.5: 16)                          */
    int64_t gqa;         /* query heads per KV head (4)                        */
    int64_t head_dim;    /* elements per head (256)                            */
    int64_t q_row;       /* elements between query rows (2*heads*head_dim)     */
    int64_t q_head;      /* elements between query heads (head_dim)            */
    int64_t out_row;     /* elements between output rows (heads*head_dim)      */
    int64_t gate_offset; /* elements from a q row to its gate (heads*head_dim);
                            < 0: no gate node, the output is the SDPA alone    */
    int32_t grouped;     /* AttentionSpec::grouped task order (no effect on results) */
    int32_t sink;        /* SdpaShape::sink: must be 0 (declined otherwise)    */
} hb_attn_spec;

/* One attention operation: AttentionCall (src/jit/execution/abi.rs:156-180).
 * Row r (0 <= r < rows) is the query at absolute position past + r; it sees
 * past + r + 1 keys, which must already be in the cache. */
typedef struct hb_attn_call {
    const uint16_t *q;       /* query rows (bf16), row stride spec.q_row       */
    const uint16_t *keys;    /* head-major K cache (bf16)                      */
    const uint16_t *values;  /* head-major V cache (bf16)                      */
    uint16_t *output;        /* token-major output (bf16), row stride out_row  */
    int64_t rows;            /* query rows in this block (>= 1)                */
    int64_t past;            /* absolute position of row 0                     */
    int64_t kv_stride;       /* elements between KV heads (capacity*head_dim)  */
    int64_t capacity;        /* positions reserved per KV head; 0 = unchecked  */
    float scale;             /* softmax scale (1/sqrt(head_dim))               */
    float sink;              /* ignored unless spec.sink                       */
} hb_attn_call;

/* One sequence of a batched decode step (device memory, one row each). */
typedef struct hb_decode_seq {
    const uint16_t *q;       /* the sequence's query row                       */
    const uint16_t *keys;    /* its K cache                                    */
    const uint16_t *values;  /* its V cache                                    */
    uint16_t *output;        /* its output row                                 */
    int64_t past;            /* positions already cached (sees past + 1 keys)  */
    int64_t kv_stride;       /* elements between its KV heads                  */
} hb_decode_seq;

/*
 * Decode SDPA (split-KV flash decoding) for `rows` query rows of one
 * sequence.  Replaces the attention node in the decode regime:
 * SdpaHeadFn (src/jit/emit_sdpa.rs:131-140) driven by the tile selector
 * (src/jit/target/x86/execution/attention.rs:56-224), followed by the
 * output-gate node ElemOp::SigmoidMul (src/jit/target/x86/emit_elem.rs:333-420).
 * Beyond 4096 positions the splits' merge is spread over the last CTAs of
 * each KV head, which wait (a bounded wait, about a second) for the others
 * to finish; that needs every CTA of the launch resident at once (one per
 * SM), so a kernel on another stream that holds SMs for that long makes the
 * call report HB_ERR_TIMEOUT through hb_workspace_status.
 */
HB_API size_t hb_attn_decode_workspace_bytes(const hb_attn_spec *spec, const hb_attn_call *call);
HB_API hb_status hb_attn_decode(const hb_attn_spec *spec, const hb_attn_call *call,
                         void *workspace, size_t workspace_bytes, hb_stream_t stream);

/*
 * Decode SDPA that allocates nothing and takes no workspace.  No counterpart
 * in the reference: it exists for callers that cannot hand this library any
 * device memory -- an engine whose device memory is planned once at start-up
 * with nothing allocated during a pass, a host that exposes no workspace to
 * its plugins, or code that must not trigger cudaMalloc's implicit device
 * synchronisation in a latency-bound decode loop.
 *
 * Same arguments, kernel and results as hb_attn_decode.  Its scratch is one
 * file-scope device array of HB_NOALLOC_SCRATCH_BYTES that every GPU loading
 * the library holds until exit; a call needing more (see
 * hb_attn_decode_workspace_bytes) is refused with HB_ERR_WORKSPACE before
 * anything is launched.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) -- make that first call before any
 * stream capture; the address is looked up again only when the device's
 * context changes (after cudaDeviceReset, for instance).  Each call clears
 * the part of the array that must start at zero (one cudaMemsetAsync on
 * `stream`) and then launches; the array is shared by all calls on a device,
 * so calls whose executions overlap on the GPU (different streams without
 * ordering) race and give wrong results.  A bounded device wait that runs
 * out (the output is then incomplete) is reported by hb_device_status, not
 * by the return value, which only covers the host-side checks and launch.
 */
#define HB_NOALLOC_SCRATCH_BYTES (4u << 20)
HB_API hb_status hb_attn_decode_noalloc(const hb_attn_spec *spec, const hb_attn_call *call,
                                        hb_stream_t stream);

/*
 * Batched decode: `nseq` independent sequences (table in device memory),
 * one query row each; max_past bounds every seqs[i].past and sum_past is
 * their sum (0 = unknown), used only to size the splits.  No counterpart in
 * the reference (one Runner = one sequence, src/jit/model.rs:329-396); it is
 * the single-sequence node above applied per sequence.  Pointers in the
 * table must be 16-byte aligned (a misaligned entry is skipped and reported
 * through hb_workspace_status as HB_ERR_ARG).
 */
HB_API size_t hb_attn_decode_batch_workspace_bytes(const hb_attn_spec *spec, int64_t nseq,
                                            int64_t max_past, int64_t sum_past);
HB_API hb_status hb_attn_decode_batch(const hb_attn_spec *spec, const hb_decode_seq *seqs,
                               int64_t nseq, int64_t max_past, int64_t sum_past,
                               void *workspace, size_t workspace_bytes, hb_stream_t stream);

/*
 * Batched decode over several GPUs, one process per GPU with no collective:
 * the plan of which GPU serves which sequence.  Sequences are taken in
 * decreasing order of `cost` (their KV positions, or bytes: the decode step
 * streams each cache once) and each goes to the GPU with the least cost so
 * far, the lowest index on a tie -- the longest-processing-time rule, whose
 * busiest GPU carries at most 4/3 - 1/(3 parts) of the optimal maximum.
 * part[i] receives the GPU of sequence i, and load[g] (optional, `parts`
 * entries) the cost assigned to GPU g.  Every rank computes the same plan
 * from the same costs.  Host only; nseq <= 2^24, parts 1 .. 4096, costs >= 0
 * with a sum below 2^62.  No counterpart in the reference, where one Runner
 * serves one sequence (src/jit/model.rs:329-396).
 */
HB_API hb_status hb_decode_shard_plan(const int64_t *cost, int64_t nseq, int32_t parts,
                                      int32_t *part, int64_t *load);

/*
 * Prefill SDPA: causal flash attention over `rows` query rows (tcgen05 MMA,
 * TMEM accumulators).  Replaces the attention node in the prefill regime:
 * SdpaPrefillFn blocks (src/jit/emit_sdpa.rs:173-304;
 * src/jit/target/x86/emit_sdpa/x86/prefill.rs:733-912) plus the decode
 * kernel for remainder rows, then the output-gate node.
 */
HB_API size_t hb_attn_prefill_workspace_bytes(const hb_attn_spec *spec, const hb_attn_call *call);
HB_API hb_status hb_attn_prefill(const hb_attn_spec *spec, const hb_attn_call *call,
                          void *workspace, size_t workspace_bytes, hb_stream_t stream);

/*
 * Prefill from host memory: hb_attn_prefill for rows whose q rows, new K/V
 * positions and output live in host memory (the reference hands its prefill
 * node host buffers owned by the Runner, src/jit/model.rs:570-611), with the
 * transfers overlapped with the computation.  `dev` is the device call
 * (device buffers with the same row strides and KV layout, rows, past,
 * kv_stride, capacity, scale); positions [0, past) must already be in the
 * device cache.  The host buffers mirror the device layouts: q_host
 * [rows][q_row], keys_host/values_host [kv_head][kv_stride] of which
 * positions past .. past+rows-1 are copied, out_host [rows][out_row].  The
 * rows are cut into blocks of `block_rows` (a multiple of 128; 0 = about
 * sixteen blocks of at least 1024 rows; a remainder under 64 rows joins the
 * last block): block j's inputs are copied on the
 * library's copy stream, its prefill runs on `stream` once they have
 * landed, and its output is copied back on another copy stream, so that
 * copies and computation overlap.
 * Every row is computed exactly as by hb_attn_prefill over all the rows.
 * On return the work, copies included, is ordered on `stream`; pinned host
 * memory lets the copies run asynchronously.  The calls on one device queue
 * their work one at a time (a lock) on the library's two copy streams of
 * that device, and may be captured in a graph; a captured call keeps those
 * streams in its capture until the capture ends, so no other call on the
 * device may run meanwhile (it would fail with HB_ERR_CUDA).
 */
typedef struct hb_attn_host_call {
    hb_attn_call dev;           /* device buffers and the call                 */
    const uint16_t *q_host;     /* [rows][q_row] bf16                          */
    const uint16_t *keys_host;  /* [kv_head][kv_stride] bf16                   */
    const uint16_t *values_host;
    uint16_t *out_host;         /* [rows][out_row] bf16                        */
    int64_t block_rows;         /* rows per block, a multiple of 128; 0: auto */
} hb_attn_host_call;
HB_API size_t hb_attn_prefill_host_workspace_bytes(const hb_attn_spec *spec,
                                                   const hb_attn_host_call *call);
HB_API hb_status hb_attn_prefill_host(const hb_attn_spec *spec, const hb_attn_host_call *call,
                                      void *workspace, size_t workspace_bytes, hb_stream_t stream);

/*
 * Context-parallel causal prefill over a ring of P GPUs.  No counterpart in
 * the reference (its prefill runs on one machine's cores through the same
 * tile selector, src/jit/target/x86/execution/attention.rs:56-224); it
 * extends hb_attn_prefill (past = 0) to a sequence of 2*P*chunk tokens
 * sharded zig-zag: rank r holds the query rows, keys and values of chunks r
 * and 2P-1-r (absolute positions r*chunk.. and (2P-1-r)*chunk..) as its
 * local rows [0, chunk) and [chunk, 2*chunk), in the reference's layouts
 * (call->rows = 2*chunk, call->past = 0, K/V [kv_head][kv_stride]).  K/V
 * shards travel the ring (rank r sends to r+1 and receives from r-1) by
 * NCCL send/recv on `comm_stream` while the previous shard is computed on
 * `stream`; the partial results of each hop are merged by log-sum-exp into
 * an f32 accumulator in the workspace, and the last step divides, rounds to
 * bf16 and applies the output gate as hb_attn_prefill does.
 */
typedef struct hb_cp_spec {
    int32_t ranks;  /* P >= 1                                     */
    int32_t rank;   /* this GPU's place on the ring, 0 <= rank < P */
    int64_t chunk;  /* positions per chunk, a multiple of 128     */
} hb_cp_spec;

/* Ring schedule (host only): the rank whose K/V shard `cp->rank` computes
 * at hop `hop` (hop 0 = its own), or -1; the absolute position of local row
 * `row` of rank `rank`, or -1. */
HB_API int32_t hb_cp_hop_source(const hb_cp_spec *cp, int32_t hop);
HB_API int64_t hb_cp_row_position(const hb_cp_spec *cp, int32_t rank, int64_t row);

/* Workspace of hb_attn_prefill_cp and of the hop/finish pair below: header,
 * (m, l) and O accumulators of the 2*chunk local rows, and for P > 1 two
 * K/V receive buffers. */
HB_API size_t hb_attn_prefill_cp_workspace_bytes(const hb_attn_spec *spec, const hb_cp_spec *cp);

/* One hop without transport, for callers that move the shards themselves:
 * call->keys/values hold the shard of rank hb_cp_hop_source(cp, hop) in the
 * shard layout above; hop 0 must run first on a workspace (it writes the
 * accumulators, later hops merge into them).  hb_attn_prefill_cp_finish
 * then writes call->output. */
HB_API hb_status hb_attn_prefill_cp_hop(const hb_attn_spec *spec, const hb_cp_spec *cp,
                                 const hb_attn_call *call, int32_t hop, void *workspace,
                                 size_t workspace_bytes, hb_stream_t stream);
HB_API hb_status hb_attn_prefill_cp_finish(const hb_attn_spec *spec, const hb_cp_spec *cp,
                                    const hb_attn_call *call, void *workspace,
                                    size_t workspace_bytes, hb_stream_t stream);

/* NCCL communicator of the ring.  NCCL is loaded on first use (the copy
 * already in the process if there is one, else libnccl.so.2); the library
 * itself does not depend on it.  `id` is HB_CP_ID_BYTES bytes made by one
 * rank with hb_cp_comm_unique_id and given to every rank; hb_cp_comm_init is
 * collective over the P ranks, each with its own GPU current. */
#define HB_CP_ID_BYTES 128
HB_API hb_status hb_cp_comm_unique_id(void *id);
HB_API hb_status hb_cp_comm_init(void **comm, int32_t ranks, const void *id, int32_t rank);
HB_API hb_status hb_cp_comm_destroy(void *comm);

/* The whole ring: P hops and the finishing step.  Every rank calls it with
 * the same chunk; `comm` comes from hb_cp_comm_init (unused when P = 1).
 * On return all work, transfers included, is ordered on `stream`. */
HB_API hb_status hb_attn_prefill_cp(const hb_attn_spec *spec, const hb_cp_spec *cp,
                             const hb_attn_call *call, void *comm, void *workspace,
                             size_t workspace_bytes, hb_stream_t stream, hb_stream_t comm_stream);

/* Host wait with a deadline on a ring call: polls `stream` (the ring's
 * compute stream; its completion implies every transfer's) and the
 * communicator's asynchronous error until the work completes or `timeout_s`
 * seconds pass.  HB_OK when complete.  On a timeout (HB_ERR_TIMEOUT), an
 * error the communicator reports (HB_ERR_NCCL) or a failed stream query
 * (HB_ERR_CUDA) the communicator is aborted (ncclCommAbort), which ends the
 * transfers of the peers that wait on this rank: it is then released and
 * must not be used or destroyed again; the ranks make a new one.  `comm`
 * NULL waits on the stream alone.  No counterpart in the reference, whose
 * pool waits without a deadline (src/pool/thread_pool.rs:261-290). */
HB_API hb_status hb_cp_wait(void *comm, hb_stream_t stream, double timeout_s);

/* KV cache geometry: KvSpec (src/jit/execution/abi.rs:57-104). */
typedef struct hb_kv_spec {
    int64_t heads;      /* KV heads                        */
    int64_t head_dim;   /* bf16 elements per head          */
    int64_t stride;     /* bf16 elements reserved per head */
    int64_t capacity;   /* positions reserved per head     */
    int64_t max_batch;  /* maximum rows in one block       */
} hb_kv_spec;

/* KV append: KvCall (abi.rs:108-130) and append (src/jit/target/x86/execution/kv.rs:17-69):
 * K[h][past + r][:] <- input_keys[r][h][:] (same for V), token-major inputs
 * with row stride heads*head_dim. */
typedef struct hb_kv_call {
    uint16_t *keys;
    uint16_t *values;
    const uint16_t *input_keys;
    const uint16_t *input_values;
    int64_t rows;
    int64_t past;
} hb_kv_call;
HB_API hb_status hb_kv_append(const hb_kv_spec *spec, const hb_kv_call *call, hb_stream_t stream);

/*
 * Attention front end of one layer: the head-norm-rope nodes of q and of k
 * and the kv-append node, in one launch (src/jit/schedule/lowering.rs:549-592;
 * per head src/jit/target/x86/execution/transforms.rs:30-81).  For each row
 * r (position past + r) and each q head, then each k head, in place:
 *   y = bf16((x * rsqrt(sum x^2 / head_dim + eps)) * w')   ElemOp::RmsNormGemma
 *       (w' = 1 + w in f32) or ElemOp::RmsNorm (w' = w)   (emit_elem.rs:242-330)
 *   then ElemOp::Rope on elements [0, rotary): pairs (j, j + rotary/2) rotated
 *   by table row past + r of cos/sin                        (emit_elem.rs:479-514)
 * then K[h][past + r][:] <- k[r][h][:] and V[h][past + r][:] <- v[r][h][:]
 * (as hb_kv_append).  Results are the reference's bits.
 */
typedef struct hb_front_spec {
    int64_t rotary;   /* rotated elements per head (Qwen3.5: 64), multiple of 32, <= head_dim */
    float eps;        /* RMSNorm epsilon (Qwen3.5: 1e-6)                                   */
    int32_t gemma;    /* 1: w' = 1 + w (GemmaRMSNorm, Qwen3.5), 0: w' = w                   */
} hb_front_spec;
typedef struct hb_front_call {
    uint16_t *q;              /* query rows, stride spec.q_row; heads*head_dim elements per row
                                 transformed in place (the gate after them is not touched) */
    uint16_t *k;              /* key rows [rows][kv_heads*head_dim], transformed in place   */
    const uint16_t *v;        /* value rows [rows][kv_heads*head_dim]                       */
    const uint16_t *q_norm;   /* [head_dim] bf16 weight of the q head norm                  */
    const uint16_t *k_norm;   /* [head_dim] bf16 weight of the k head norm                  */
    const uint16_t *cos;      /* [positions][rotary/2] bf16, row past + r used by row r      */
    const uint16_t *sin;
    uint16_t *keys;           /* the layer's K cache (hb_kv_spec layout); NULL: no append  */
    uint16_t *values;         /* the layer's V cache                                        */
    int64_t rows;
    int64_t past;             /* position of row 0                                          */
} hb_front_call;
HB_API hb_status hb_attn_front(const hb_attn_spec *spec, const hb_kv_spec *kv,
                               const hb_front_spec *front, const hb_front_call *call,
                               hb_stream_t stream);

/* ------------------------------------------------------------- DeltaNet */

/* DeltaNet geometry: Shape (src/jit/execution/abi.rs:266-307) without the conv width. */
typedef struct hb_gdn_shape {
    int64_t nk;   /* key heads (16)    */
    int64_t nv;   /* value heads (32)  */
    int64_t hkd;  /* key head dim (128)*/
    int64_t hvd;  /* value head dim (128) */
} hb_gdn_shape;

/* RecurrenceCall (src/jit/execution/abi.rs:310-317) plus the L2 step of the
 * delta-l2-gates node (src/jit/target/x86/execution/delta.rs:442-515). */
typedef struct hb_gdn_call {
    float *state;        /* [nv][hkd][hvd], read and updated in place      */
    float *output;       /* [rows][nv*hvd]                                 */
    const float *qkv;    /* [rows][2*nk*hkd + nv*hvd] (not modified)       */
    const float *beta;   /* [rows][nv]                                     */
    const float *decay;  /* [rows][nv]                                     */
    int64_t rows;        /* positions in this block (>= 1)                 */
    int32_t l2;          /* 1: L2-normalise q and k heads on load (eps)    */
    float eps;           /* DN_L2_EPS = 1e-6 (src/jit/schedule/deltanet.rs:69) */
} hb_gdn_call;

/*
 * Recurrent DeltaNet: the positions in order, one step each.  Replaces the
 * delta-causal-recurrence node (RecurrenceFn, src/jit/emit_recurrence.rs:63-73;
 * x86 src/jit/target/x86/emit_recurrence.rs:108-217; traversal
 * src/jit/target/x86/execution/delta.rs:519-607) with the default non-FMA
 * order, so the state and outputs are the reference's bits.  It takes no
 * workspace, as RecurrenceFn takes no scratch: a bounded device wait that
 * runs out (state and outputs then unwritten) is reported by
 * hb_device_status.
 */
HB_API hb_status hb_gdn_decode(const hb_gdn_shape *shape, const hb_gdn_call *call, hb_stream_t stream);

/*
 * Chunked DeltaNet prefill (chunk 64, WY/UT form, intra-chunk products on
 * tcgen05).  Same inputs and outputs as hb_gdn_decode; sums are
 * reassociated (the reference's own chunked form,
 * src/jit/target/aarch64/deltanet_chunk.rs:6-15, is also not the bits of
 * the sequential recurrence).
 */
HB_API size_t hb_gdn_prefill_workspace_bytes(const hb_gdn_shape *shape, int64_t rows);
HB_API hb_status hb_gdn_prefill(const hb_gdn_shape *shape, const hb_gdn_call *call, void *workspace,
                         size_t workspace_bytes, hb_stream_t stream);

/*
 * hb_gdn_prefill for rows whose inputs (qkv, beta, decay) and output live in
 * host memory, with the copies overlapped with the computation.  `dev`
 * names the device buffers the rows go through (state, output, qkv, beta,
 * decay; rows, l2, eps as in hb_gdn_prefill); the *_host arrays hold the
 * same rows in the same layouts.  The rows run in blocks of `block_rows`
 * (0: the library's choice; else a positive multiple of 64): block j's
 * inputs go in on a copy stream, hb_gdn_prefill runs the block on `stream`
 * (the state carried from block to block), its output rows come back on a
 * second copy stream.  Blocks start on chunk boundaries and every block
 * takes the same kernels one call over all the rows would (a remainder of
 * fewer than 128 rows joins the block before it), so the output and the
 * final state are that call's bits.  Pin the host arrays: pageable memory
 * makes the copies synchronous.  Not for stream capture on a device's first
 * call (the copy streams and events are created then).
 */
typedef struct hb_gdn_host_call {
    hb_gdn_call dev;
    const float *qkv_host;     /* [rows][2*nk*hkd + nv*hvd] */
    const float *beta_host;    /* [rows][nv]                */
    const float *decay_host;   /* [rows][nv]                */
    float *output_host;        /* [rows][nv*hvd]            */
    int64_t block_rows;
} hb_gdn_host_call;
HB_API size_t hb_gdn_prefill_host_workspace_bytes(const hb_gdn_shape *shape,
                                                  const hb_gdn_host_call *call);
HB_API hb_status hb_gdn_prefill_host(const hb_gdn_shape *shape, const hb_gdn_host_call *call,
                                     void *workspace, size_t workspace_bytes, hb_stream_t stream);

/*
 * DeltaNet front end of one layer, in one launch: the delta-causal-convolution
 * node (src/jit/target/x86/execution/delta.rs:609-705) and the gate part of
 * delta-l2-gates (delta.rs:290-389; its L2 part is hb_gdn_call.l2).  Per
 * channel c of qkv, positions in order:
 *   state[c][0..ck) <- state[c][1..ck) ++ qkv[r][c];  qkv[r][c] <- silu(sum_j state[c][j] w[c][j])
 * in the vector kernel's form (src/jit/target/x86/emit_conv.rs) for the
 * channels of full 16-channel blocks at ck = 4, the scalar body's
 * (delta_scalar.rs:85-155) for the others; per (row, V head) h:
 *   beta = 1 / (exp(-b) + 1); dt = a + dt_bias[h]; dt = log(exp(dt) + 1) unless dt > 20;
 *   decay = exp(-exp(a_log[h]) * dt)
 * with the reference's scalar exp / log (execution/math.rs).  Results are
 * the reference's bits.  The workspace holds only the status word
 * (hb_workspace_status reports a bounded wait that ran out).
 */
typedef struct hb_gdn_front_call {
    float *qkv;                   /* [rows][2*nk*hkd + nv*hvd] f32 (conv width a multiple of 4,
                                     16-byte aligned): conv + SiLU in place                    */
    float *conv_state;            /* [conv][ck] f32: the last ck inputs; read and updated       */
    const uint16_t *conv_weight;  /* [conv][ck] bf16                                            */
    const float *ab;              /* [rows][2*nv] f32: a (dt) then b (beta) projections         */
    const uint16_t *dt_bias;      /* [nv] bf16                                                  */
    const float *a_log;           /* [nv] f32                                                   */
    float *beta;                  /* [rows][nv] f32 out                                         */
    float *decay;                 /* [rows][nv] f32 out                                         */
    int64_t rows;                 /* positions (>= 1)                                           */
    int64_t ck;                   /* conv kernel length, 1..8 (Qwen3.5: 4)                      */
} hb_gdn_front_call;
HB_API hb_status hb_gdn_front(const hb_gdn_shape *shape, const hb_gdn_front_call *call,
                              void *workspace, size_t workspace_bytes, hb_stream_t stream);

/*
 * Gated RMS norm of the recurrence output, the delta-gated-norm node
 * (src/jit/target/x86/execution/delta.rs:706-774): per (row, V head) of
 * width hvd, y = ((x * 1/sqrt(sum x^2 / hvd + eps)) * w) * silu(z), in the
 * vector kernel's form (src/jit/target/x86/emit_gated_norm.rs) at hvd a
 * multiple of 16 up to 128, the scalar body's (delta_scalar.rs:159-239)
 * otherwise.  Results are the reference's bits.
 */
typedef struct hb_gdn_norm_call {
    const float *x;           /* [rows][nv*hvd] f32 recurrence output                          */
    const float *z;           /* [rows][nv*hvd] f32 gate projection                            */
    const uint16_t *weight;   /* [hvd] bf16 norm weight                                        */
    uint16_t *out;            /* [rows][nv*hvd] bf16: the out-projection input                 */
    float *out_f32;           /* y in f32 (the reference writes it over x); NULL: not written  */
    int64_t rows;
    float eps;                /* the config's rms_norm_eps (Qwen3.5: 1e-6)                     */
} hb_gdn_norm_call;
HB_API hb_status hb_gdn_gated_norm(const hb_gdn_shape *shape, const hb_gdn_norm_call *call,
                                   hb_stream_t stream);

/* ------------------------------------------------------------- snapshot */

/*
 * Snapshot / restore of a sequence's device state in the reference's
 * serialized `Instantaneous` format, version 1 (src/jit/model.rs:100-326;
 * take src/jit/model.rs:732-774, restore :786-857).  The image, all
 * little-endian, is
 *   u32 1 | u64 n, u64 kv_offsets[n] | u64 n, u64 snap_offsets[n] |
 *   u64 n, u64 snap_positions[n] | u64 n, u16 kv[n] | u64 n, u16 logits[n] |
 *   u64 n, f32 dn_conv[n] | u64 n, f32 dn_recurrent[n] | u64 pos
 * with snap_positions[l] = min(kv_reserve, max_positions) on a layer with a
 * cache (0 without), the snapshot KV of layer l at snap_offsets[l] laid out as
 * the device cache [K|V][kv_heads][snap_positions[l]][head_dim].  Written
 * once to disk, an image is the reference's file (Instantaneous::write_to,
 * :270-287); a file it wrote restores here.
 *
 * The slot is the image itself, in host memory (pinned for full DMA speed):
 * a take moves the first `pos` positions of every head with one 2-D copy
 * per (layer, K|V), and the states and logits with one copy each, straight
 * to their place in the image; a restore copies the first `p` positions
 * back.  Positions of the slot beyond `pos` are written as zeros (the bytes
 * of a freshly reserved slot).  Copies are stream-ordered: the image is
 * complete, and the device state restored, when `stream` reaches them.
 */
typedef struct hb_state_geometry {
    const int64_t *kv_offsets;  /* [n_layers + 1] offsets (bf16 elements) of each layer's cache in
                                   the device KV buffer: Runner::kv_offsets (model.rs:545-559)  */
    int64_t n_layers;
    int64_t kv_heads;           /* n_kv_heads                                                    */
    int64_t kv_reserve;         /* positions reserved per head (kv_reserve_tokens)               */
    int64_t conv_len;           /* f32 elements of the DeltaNet conv states, all layers          */
    int64_t recurrent_len;      /* f32 elements of the DeltaNet recurrent states, all layers     */
    int64_t logits_len;         /* bf16 logits of the last token (vocab rounded up to 16)        */
} hb_state_geometry;
typedef struct hb_state_buffers {  /* device memory */
    uint16_t *kv;
    float *dn_conv;
    float *dn_recurrent;
    uint16_t *logits;
} hb_state_buffers;

/* Bytes of the image of a slot reserved for `max_positions` (snapshot_reserve,
 * model.rs:675-699); 0 for an invalid geometry. */
HB_API size_t hb_snapshot_bytes(const hb_state_geometry *geometry, int64_t max_positions);
/* snapshot_take: the state at position `pos` into `image` (hb_snapshot_bytes
 * bytes).  Refused (HB_ERR_ARG, nothing copied) when a layer holds more
 * positions than the slot (pos > min(kv_reserve, max_positions)). */
HB_API hb_status hb_snapshot_take(const hb_state_geometry *geometry, const hb_state_buffers *state,
                                  int64_t pos, int64_t max_positions, void *image,
                                  size_t image_bytes, hb_stream_t stream);
/* Instantaneous::read + restore_from: validates the image (format version,
 * every length bounded by 64 GiB and by image_bytes, self-consistent
 * offsets) and the request, then restores the state truncated to `p`
 * positions.  Refusals, before any copy: HB_ERR_ARG for another format
 * version, a corrupted image, p > pos, or p < pos when the model has a
 * recurrent state; HB_DECLINE_GEOMETRY for an image of another geometry
 * (kv_offsets or state lengths differ). */
HB_API hb_status hb_snapshot_restore(const hb_state_geometry *geometry, const hb_state_buffers *state,
                                     const void *image, size_t image_bytes, int64_t p,
                                     hb_stream_t stream);
/* The position an image holds and Instantaneous::restorable_at(p) for each
 * p: *restorable_below = 1 when positions below *pos restore too (no
 * recurrent state).  Validates as hb_snapshot_restore. */
HB_API hb_status hb_snapshot_info(const void *image, size_t image_bytes, int64_t *pos,
                                  int32_t *restorable_below);

/* --------------------------------------------------------------- mount */

/*
 * Routing of a model pass to the kernels: what the reference's lowering does
 * per layer when it mounts a regime (src/jit/model/mounted.rs:237-380) --
 * bind each layer to its slice of the sequence's state (the KV cache of an
 * attention layer at kv_offsets[layer], keys then values; the conv and
 * recurrent slots of the d-th DeltaNet layer at d * conv_stride and
 * d * recurrent_stride) and run the layer's mixer nodes for a block of rows:
 *   attention layer: head-norm-rope of q and k + kv-append (hb_attn_front),
 *     then the attention and gate nodes (hb_attn_decode for one row,
 *     hb_attn_prefill otherwise)     (src/jit/schedule/lowering.rs:549-666)
 *   DeltaNet layer: conv + gates (hb_gdn_front), L2 + recurrence
 *     (hb_gdn_prefill: the reference's order below 128 rows, chunked above),
 *     gated norm (hb_gdn_gated_norm)  (src/jit/schedule/lowering.rs:897-1010)
 * The projections around the mixers stay with the caller.  A mount owns
 * every workspace and scratch buffer its calls need, allocated once by
 * hb_mount_create: nothing allocates during a pass, and a pass may be
 * captured in a CUDA graph.  Calls on one mount share that scratch: order
 * them on one stream (or with events).
 */
typedef struct hb_mount hb_mount;  /* opaque */
enum { HB_LAYER_ATTENTION = 1, HB_LAYER_DELTA = 2 };
typedef struct hb_mount_desc {
    const hb_state_geometry *geometry;  /* the sequence's state (as for the snapshot)            */
    const hb_state_buffers *state;      /* its device buffers                                    */
    const int32_t *layer_kinds;         /* [geometry->n_layers]: HB_LAYER_ATTENTION / _DELTA      */
    hb_attn_spec attn;                  /* attention layers (heads / gqa = geometry kv_heads)    */
    float attn_scale;                   /* softmax scale                                         */
    int64_t rotary;                     /* rotated elements per head                             */
    const uint16_t *cos;                /* RoPE tables [kv_reserve][rotary/2] bf16, device        */
    const uint16_t *sin;
    float norm_eps;                     /* head-norm and gated-norm epsilon (config rms_norm_eps) */
    int32_t gemma;                      /* head-norm weight form (1: 1 + w, Qwen3.5)              */
    hb_gdn_shape delta;                 /* DeltaNet layers                                       */
    int64_t conv_kernel;                /* conv kernel length (4)                                */
    int64_t conv_stride;                /* f32 elements of one layer's conv slot (>= conv x ck)   */
    int64_t recurrent_stride;           /* f32 elements of one recurrent slot (>= nv hkd hvd)     */
    int64_t max_rows;                   /* the largest block a pass feeds (<= kv_reserve, 2^20)   */
} hb_mount_desc;
/* Where a layer's mixer reads and writes its state. */
typedef struct hb_layer_route {
    int32_t kind;              /* HB_LAYER_ATTENTION or HB_LAYER_DELTA                           */
    int32_t delta_index;       /* DeltaNet layers: index among them; -1 otherwise                */
    uint16_t *keys;            /* attention: the layer's K cache, [kv_heads][kv_reserve][d]       */
    uint16_t *values;          /* its V cache                                                    */
    int64_t kv_stride;         /* elements between KV heads                                      */
    float *conv_state;         /* DeltaNet: the layer's conv slot                                */
    float *recurrent_state;    /* its recurrent slot                                             */
} hb_layer_route;
/* Validates the description as the lowering does (a DeltaNet layer has no
 * KV and fits its slots; an attention layer's KV is heads x kv_reserve x
 * head_dim) and gives layer `layer`'s route; host only, no allocation.
 * HB_DECLINE_GEOMETRY for a plan mismatch. */
HB_API hb_status hb_mount_route(const hb_mount_desc *desc, int64_t layer, hb_layer_route *route);
/* hb_mount_route's checks for every layer, then the workspaces and scratch.
 * The mount copies the description's records but keeps its device pointers
 * (state buffers, RoPE tables): those must outlive the mount. */
HB_API hb_status hb_mount_create(const hb_mount_desc *desc, hb_mount **mount);
HB_API void hb_mount_destroy(hb_mount *mount);
/* The status word of the mount's workspaces (as hb_workspace_status).  A
 * device-side failure it finds poisons the mount (below); on a poisoned
 * mount it returns the first failure's status. */
HB_API hb_status hb_mount_status(hb_mount *mount, hb_stream_t stream);
/* A mixer call that fails after it entered execution (a node launched, so
 * state may be half updated), or a failure hb_mount_status finds, poisons the
 * mount: every later hb_mount_attention / hb_mount_delta is refused with the
 * first failure's status until hb_mount_reset, as a failed call poisons the
 * reference's execution session until its owner resets or restores the model
 * (src/jit/execution/runtime.rs:144-151, 310-327; program.rs:289).  Refusals
 * before any launch (declines, bad arguments) do not poison.  Reset after the
 * caller has restored (hb_snapshot_restore) or cleared every state buffer the
 * failed call may have touched; it clears the workspaces' status words and
 * the one-row DeltaNet launches' write-back counters. */
HB_API int hb_mount_needs_reset(const hb_mount *mount);
HB_API hb_status hb_mount_reset(hb_mount *mount, hb_stream_t stream);

typedef struct hb_mount_attention_call {
    uint16_t *q;               /* [rows][attn.q_row]: heads (normed and rotated in place), gates  */
    uint16_t *k;               /* [rows][kv_heads*d]: normed and rotated in place, then cached     */
    const uint16_t *v;         /* [rows][kv_heads*d]: cached                                       */
    const uint16_t *q_norm;    /* [d] bf16 head-norm weights of the layer                          */
    const uint16_t *k_norm;
    uint16_t *out;             /* [rows][attn.out_row] bf16                                        */
    int64_t rows;              /* 1 .. max_rows                                                     */
    int64_t pos;               /* position of row 0 (pos + rows <= kv_reserve)                      */
} hb_mount_attention_call;
/* One attention layer's block: head-norm-rope of q and k, kv-append, then the
 * attention and gate (decode for one row, prefill otherwise).  A one-row
 * block over more than 4096 cached positions (head_dim 256) runs as one
 * launch -- the split-KV decode does the front end itself -- with the same
 * bits as the node-by-node path; a block either node refuses takes that path
 * and is reported as before. */
HB_API hb_status hb_mount_attention(hb_mount *mount, int64_t layer, const hb_mount_attention_call *call,
                                    hb_stream_t stream);

typedef struct hb_mount_delta_call {
    float *qkv;                   /* [rows][2 nk hkd + nv hvd]: conv + SiLU in place             */
    const float *ab;              /* [rows][2 nv]                                                */
    const float *z;               /* [rows][nv hvd] gate projection                              */
    const uint16_t *conv_weight;  /* [conv][ck] bf16                                             */
    const uint16_t *dt_bias;      /* [nv] bf16                                                   */
    const float *a_log;           /* [nv]                                                        */
    const uint16_t *norm_weight;  /* [hvd] bf16                                                  */
    uint16_t *out;                /* [rows][nv hvd] bf16: the out-projection's input             */
    float *out_f32;               /* optional f32 copy of out (NULL: not written)                */
    int64_t rows;                 /* 1 .. max_rows                                               */
} hb_mount_delta_call;
/* One DeltaNet layer's block: conv + gates, L2 + recurrence, gated norm.  A
 * one-row block (conv kernel 4, hkd 64 or 128, hvd a multiple of 32 up to
 * 128) runs as one launch with the node-by-node path's bits; every node's
 * checks run before it, so a refused one-row call launches nothing and does
 * not poison the mount. */
HB_API hb_status hb_mount_delta(hb_mount *mount, int64_t layer, const hb_mount_delta_call *call,
                                hb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HERBERT_B200_H */
