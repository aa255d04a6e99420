/*
 * herbert_oracle.h -- CPU restatement of the reference's attention-path
 * kernels (xigh/herbert-jit-bf16, x86 AVX-512 BF16 emitters).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links this
 * file; only the tests, the smoke check and the CPU-baseline leg of
 * bench.py load it, as the checker.
 *
 * Parity status: the reference is Rust and cannot be built here (no
 * cargo/rustc, crates not vendored), and it ships no tests or golden
 * vectors.  The restatement is therefore pinned in two ways instead:
 *   (1) every primitive the reference emits (vdpbf16ps, vcvtneps2bf16,
 *       the inline exp polynomial, the hsum/hmax trees) is emulated in
 *       portable C and checked bit for bit against the same x86
 *       instruction sequence transcribed with intrinsics, run on a CPU
 *       with AVX512-BF16;
 *   (2) the reference's own stated invariants (prefill block == repeated
 *       decode, bit for bit; qk_group changes at most one bf16 step;
 *       non-FMA recurrence == scalar order) are tests.
 * There is no reference output to compare against: parity is "unpinned"
 * by reference golden vectors.
 *
 * Layouts follow the reference:
 *   K/V cache   : [kv_head][capacity][head_dim] bf16, head h at h*kv_stride
 *                 (src/jit/model.rs:545-559, src/jit/execution/abi.rs:57-104)
 *   q row       : [Q_0 .. Q_{H-1} | g_0 .. g_{H-1}], row stride q_row
 *                 (src/jit/schedule.rs:109-133,172-186)
 *   DeltaNet qkv: [rows][2*nk*hkd + nv*hvd] f32, state [nv][hkd][hvd] f32
 *                 (src/jit/target/x86/execution/delta.rs:519-607)
 */
#ifndef HERBERT_ORACLE_H
#define HERBERT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 1 when the AVX512-BF16 transcription can run on this CPU. */
int orc_has_avx512bf16(void);

/* Conversions (src/core/tensor.rs:8-24 and vcvtneps2bf16). */
float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16_cvtne(float x);
void orc_f32_to_bf16_array(const float *x, uint16_t *y, size_t n);
void orc_bf16_to_f32_array(const uint16_t *x, float *y, size_t n);

/* Primitive checks: one vdpbf16ps over 16 lanes (acc[16] updated in place),
 * scalar emulation and hardware instruction. */
void orc_dpbf16_scalar(float *acc, const uint16_t *a, const uint16_t *b);
int orc_dpbf16_hw(float *acc, const uint16_t *a, const uint16_t *b);
/* The emitted exp polynomial (src/jit/target/x86/emit_sdpa/x86/base.rs:189-212). */
float orc_exp_poly(float x);
int orc_exp_poly_hw16(const float *x, float *y);

/*
 * Decode SDPA for one query head (SdpaHeadFn, src/jit/emit_sdpa.rs:131-140;
 * Chained form, qk_group 8 = one accumulation chain per position).
 * q[head_dim], k/v: [n][head_dim] rows of this KV head, out[head_dim].
 * scores: caller scratch of align16(n) floats (may be NULL: internal).
 * impl: 0 = portable emulation, 1 = AVX512-BF16 transcription (returns -1
 * if unavailable).  qk_chains: 1 (qk_group 8/16, the default) or 4 (the
 * historical row-by-row kernel, qk_group 0).
 */
int orc_sdpa_head(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                  float *scores, uint16_t *out, size_t n, size_t head_dim,
                  float scale, int impl, int qk_chains);

/*
 * Prefill block of `rows` consecutive queries of one head against the same
 * K/V (SdpaPrefillFn, src/jit/emit_sdpa.rs:173-304; assemble_prefill,
 * src/jit/target/x86/emit_sdpa/x86/prefill.rs:733-912): the QK rectangle
 * rows x (past+rows), -inf pad per row, softmax per row, masked columns set
 * to +0, SV over the block.  q rows at q_row_stride, out rows at
 * out_row_stride (elements).  Portable emulation only.
 */
int orc_sdpa_prefill_block(const uint16_t *q, const uint16_t *k,
                           const uint16_t *v, uint16_t *out, size_t past,
                           size_t rows, size_t head_dim, size_t q_row_stride,
                           size_t out_row_stride, float scale);

/* Output gate y = bf16(a / (1 + exp(-b))) over n elements
 * (ElemOp::SigmoidMul, src/jit/target/x86/emit_elem.rs:333-420). */
int orc_sigmoid_mul(const uint16_t *a, const uint16_t *b, uint16_t *y,
                    size_t n, int impl);

/*
 * The attention node (src/jit/target/x86/execution/attention.rs:56-224)
 * followed by the output-gate node (src/jit/schedule/lowering.rs:642-666):
 * for every row r < rows and query head h < heads, n = past + r + 1 keys of
 * KV head h / gqa.  q + r*q_row + h*q_head; out + r*out_row + h*head_dim;
 * gate (if gate_offset >= 0) at q + r*q_row + gate_offset + h*head_dim.
 * threads: OpenMP threads (0 = runtime default).  use_block: 1 = 8-row
 * prefill blocks for full chunks (the reference's x86 path), 0 = decode
 * kernel row by row (same bits).
 */
int orc_attention(const uint16_t *q, const uint16_t *keys,
                  const uint16_t *values, uint16_t *out, size_t rows,
                  size_t past, size_t heads, size_t gqa, size_t head_dim,
                  size_t q_row, size_t q_head, size_t out_row,
                  ptrdiff_t gate_offset, size_t kv_stride, float scale,
                  int impl, int use_block, int threads);

/* DeltaNet L2 norm of one head in place (src/jit/target/x86/execution/delta.rs:28-62). */
void orc_l2norm(float *x, size_t dim, float eps);

/* One recurrence step for one V head (RecurrenceFn,
 * src/jit/target/x86/emit_recurrence.rs:108-217).  fma = 0 is the default
 * (the bits of the scalar order), 1 the Knobs::deltanet_fma form. */
void orc_gdn_recurrence(float *s, float *out, const float *q, const float *k,
                        const float *v, size_t hkd, size_t hvd, float beta,
                        float decay, float scale, int fma);

/*
 * The delta-l2-gates L2 part and the delta-causal-recurrence node over
 * `rows` positions (src/jit/target/x86/execution/delta.rs:442-607):
 * qkv [rows][2*nk*hkd + nv*hvd] f32 (L2-normalised in place when l2 != 0),
 * beta/decay [rows][nv], state [nv][hkd][hvd] (updated), out [rows][nv*hvd].
 */
int orc_gdn_layer(float *qkv, float *state, float *out, const float *beta,
                  const float *decay, size_t rows, size_t nk, size_t nv,
                  size_t hkd, size_t hvd, int l2, float eps, int fma,
                  int threads);

/* Deterministic inputs: splitmix64 stream, Box-Muller N(0,1) in double,
 * rounded to bf16 (RNE) -- the generator the fixtures use. */
/* Attention front end of one layer: head-norm-rope of the q heads and of the
 * k heads, then kv-append (src/jit/schedule/lowering.rs:549-592).  q rows
 * [rows][q_row] (the first heads*head_dim elements are transformed), k and
 * v rows [rows][kv_row]; tables [positions][rotary/2]; keys/values may be
 * NULL (no append).  impl 0: scalar restatement, 1: AVX-512 BF16
 * transcription (-1 when the CPU lacks it). */
int orc_attn_front(uint16_t *q, size_t q_row, size_t heads, uint16_t *k, const uint16_t *v,
                   size_t kv_row, size_t kv_heads, size_t head_dim, const uint16_t *q_norm,
                   const uint16_t *k_norm, const uint16_t *cos_tab, const uint16_t *sin_tab,
                   size_t rotary, float eps, int gemma, uint16_t *keys, uint16_t *values,
                   size_t kv_stride, size_t rows, size_t past, int impl);

/* DeltaNet front end (src/jit/target/x86/execution/delta.rs:290-389, 609-774).
 * The reference's scalar exp / log (math.rs, FMA form: Arm optimized-routines
 * expf / logf) and their tables (32 exp entries, 16 {invc, logc} pairs). */
float orc_expf_arm(float x);
float orc_logf_arm(float x);
void orc_mathf_tables(uint64_t *exp_tab, uint64_t *log_tab);
void orc_expf_arm_array(const float *x, float *y, size_t n);
void orc_logf_arm_array(const float *x, float *y, size_t n);
void orc_expf_libm_array(const float *x, float *y, size_t n);
void orc_logf_libm_array(const float *x, float *y, size_t n);
uint64_t orc_mathf_sweep(uint32_t stride, int which);
/* Causal depthwise conv + SiLU over rows, in place on data [rows][conv];
 * state [conv][ck] and weights [conv][ck] (bf16).  impl 0: restatement,
 * 1: AVX-512 transcription of the K = 4 vector kernel (-1 without it). */
int orc_gdn_conv(float *data, size_t rows, size_t conv, const uint16_t *w, float *state,
                 size_t ck, int impl);
/* beta / decay of rows x nv tasks from ab [rows][2*nv] (a then b). */
void orc_gdn_gates(const float *ab, const uint16_t *dt_bias, const float *a_log, float *beta,
                   float *decay, size_t rows, size_t nv);
/* Gated RMS norm of n_rows rows of width dim: out (f32, in place) and
 * out_bf16.  impl as orc_gdn_conv. */
int orc_gdn_gated_norm(float *out, const float *z, const uint16_t *w, uint16_t *out_bf16,
                       size_t n_rows, size_t dim, float eps, int impl);

/* The snapshot image of the state at `pos` in a slot reserved for
 * max_positions (src/jit/model.rs:270-287, 675-774); out NULL asks the size;
 * -1 when pos does not fit the slot. */
long long orc_snapshot_image(const uint16_t *kv, const int64_t *kv_offsets, size_t n_layers,
                             size_t kv_heads, size_t kv_reserve, size_t max_positions, size_t pos,
                             const float *conv, size_t conv_len, const float *rec, size_t rec_len,
                             const uint16_t *logits, size_t logits_len, uint8_t *out);

void orc_fill_normal_bf16(uint16_t *x, size_t n, uint64_t seed);
void orc_fill_normal_f64(double *x, size_t n, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
