// gdn_decode.cu -- the GatedDeltaNet recurrence on sm_100a, position by
// position, with the reference's non-FMA rounding order.
//
// Replaces the delta-causal-recurrence node (RecurrenceFn,
// src/jit/emit_recurrence.rs:63-73; x86 src/jit/target/x86/emit_recurrence.rs:108-217;
// traversal src/jit/target/x86/execution/delta.rs:519-607) and the L2 step of
// delta-l2-gates (delta.rs:28-62, 442-515).
//
// Column vd of a head's state only ever meets column vd: kv[vd], delta[vd]
// and out[vd] are sums over kd of one column.  So one thread owns one state
// column for the whole call, holds its hkd values in registers, and runs the
// kd sums in increasing order with separate multiply and add (__fmul_rn /
// __fadd_rn): the outputs and the state are the reference's bits.  Grid =
// (value heads, hvd/32); the state crosses HBM once per call however many
// positions the call carries.
//
// CTA = one state warp and two producer warps.  The producers (even and odd
// positions) stage each position's inputs in an 8-slot shared-memory ring
// ahead of use: the key head's q and k, L2-normalised (sequential sums, as
// the reference) with q scaled, the CTA's 32 v values, beta and decay.  The
// state warp then only runs the recurrence, and runs two positions' sums at
// once: for each kd, pass 2 of position t (S += k_t delta_t, out_t += S q_t)
// and then pass 1 of position t + 1 (S *= decay_{t+1}, kv_{t+1} += S k_{t+1})
// -- per element the same operations in the same order as one position
// after the other, with the two dependent sums interleaved.
//
// The CTA's state slice [hkd rows][32 columns] f32 moves as one TMA tile
// each way (shared memory in between): per-thread loads of 128 strided rows
// left a step latency-bound on memory parallelism, the TMA tile takes one
// request.
//
// A call of one position (every decode step of a model) takes a second
// form, gdn_step_split_kernel, built for latency, and a short block of up to
// kRowsSplitMax positions a third, gdn_rows_split_kernel: see their comments.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_internal.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

struct GdnParams {
  float* state;
  float* out;
  const float* qkv;
  const float* beta;
  const float* decay;
  int64_t rows;
  int nk, nv, hvd;
  int l2;
  float eps, scale;
  int* status;  // device status word: the caller's workspace or the per-device word
};

constexpr int kRing = 8;       // positions staged ahead of the state warp
constexpr int kProducers = 2;  // warps 1 .. kProducers: positions w - 1, w - 1 + kProducers, ...

// One staged position: normalised (and for q scaled) q and k of the key
// head, the CTA's 32 v values, beta, decay.
template <int HKD>
struct __align__(16) Stage {
  float q[HKD];
  float k[HKD];
  float v[32];
  float beta, decay, pad[2];
};

// Pass 2 of position t fused with pass 1 of position t + 1 on the column s:
// per kd, r = s + k_t delta_t; out += r q_t; r' = r decay_{t+1};
// kv += r' k_{t+1}; s = r'.  NEXT false: pass 2 alone (the last position).
template <int HKD, bool NEXT>
HB_DEV void sweep(float (&s)[HKD], const float* kt, const float* qt, float delta, const float* kn,
                  float decay_n, float& out, float& kv) {
  const float4* k4 = reinterpret_cast<const float4*>(kt);
  const float4* q4 = reinterpret_cast<const float4*>(qt);
  const float4* n4 = reinterpret_cast<const float4*>(kn);
  float o = 0.f, a = 0.f;
#pragma unroll
  for (int k = 0; k < HKD / 4; ++k) {
    const float4 kk = k4[k], qq = q4[k];
    const float kw[4] = {kk.x, kk.y, kk.z, kk.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
    float nw[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (NEXT) {
      const float4 nn = n4[k];
      nw[0] = nn.x; nw[1] = nn.y; nw[2] = nn.z; nw[3] = nn.w;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float r = __fadd_rn(s[4 * k + e], __fmul_rn(kw[e], delta));
      o = __fadd_rn(o, __fmul_rn(r, qw[e]));
      if constexpr (NEXT) {
        r = __fmul_rn(r, decay_n);
        a = __fadd_rn(a, __fmul_rn(r, nw[e]));
      }
      s[4 * k + e] = r;
    }
  }
  out = o;
  kv = a;
}

template <int HKD>
__global__ void __launch_bounds__(32 * (1 + kProducers), 1)
    gdn_decode_kernel(const __grid_constant__ CUtensorMap tmS, const GdnParams p) {
  __shared__ __align__(128) float st[HKD * 32];  // state rows kd, columns col0..col0+31
  __shared__ Stage<HKD> ring[kRing];
  __shared__ float inv[kProducers][2];
  __shared__ __align__(8) uint64_t bar, full[kRing], empty[kRing];
  __shared__ int abort_flag;
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col0 = blockIdx.y * 32, col = col0 + lane;
  const int kh = h / (p.nv / p.nk);
  const int64_t key = int64_t(p.nk) * HKD, value = int64_t(p.nv) * p.hvd;
  const int64_t conv = 2 * key + value;

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    abort_flag = 0;
    fence_mbar_init();
    sm100::prefetch_tmap(&tmS);
  }
  // Launched with programmatic stream serialization: the CTAs are made
  // resident while the previous kernel finishes, and until
  // griddepcontrol.wait they only prefetch into L2 (the state tile and the
  // first position's lines; a prefetch cannot change what a later load
  // returns).  Every load follows the wait: the previous kernel may be the
  // front end that writes qkv, beta and decay.
  if (warp == 0) {
    if (lane == 0) sm100::tma_prefetch_l2_2d(&tmS, col0, h * HKD);
    if (lane < HKD / 32) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.qkv + int64_t(kh) * HKD + lane * 32));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.qkv + key + int64_t(kh) * HKD + lane * 32));
    }
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  auto wait = [&](uint64_t* b, uint32_t parity) -> bool {
    if (*reinterpret_cast<volatile int*>(&abort_flag)) return false;
    if (__all_sync(0xFFFFFFFFu, mbar_wait(b, parity))) return true;
    if (lane == 0) record_status(p.status, kStatusTimeout);
    *reinterpret_cast<volatile int*>(&abort_flag) = 1;
    return false;
  };

  if (warp > 0) {  // ------------------------------------------- producers
    const int w = warp - 1;
    for (int64_t t = w; t < p.rows; t += kProducers) {
      const int slot = int(t % kRing);
      const int64_t use = t / kRing;
      if (use > 0 && !wait(&empty[slot], uint32_t((use - 1) & 1))) break;
      Stage<HKD>& S = ring[slot];
      const float* row = p.qkv + t * conv;
#pragma unroll
      for (int i = lane; i < HKD; i += 32) {
        S.q[i] = row[int64_t(kh) * HKD + i];
        S.k[i] = row[key + int64_t(kh) * HKD + i];
      }
      S.v[lane] = row[2 * key + int64_t(h) * p.hvd + col];
      if (lane == 0) {
        S.beta = p.beta[t * p.nv + h];
        S.decay = p.decay[t * p.nv + h];
      }
      __syncwarp();
      // q <- q * inv_q * scale (the reference scales q inside pass 2, per
      // element, after the L2 step: the same two roundings), k <- k * inv_k
      float iq = 1.f, ik = 1.f;
      if (p.l2) {
        if (lane < 2) inv[w][lane] = l2_inverse<HKD>(lane == 0 ? S.q : S.k, p.eps);
        __syncwarp();
        iq = inv[w][0];
        ik = inv[w][1];
      }
#pragma unroll
      for (int i = lane; i < HKD; i += 32) {
        const float qv = p.l2 ? __fmul_rn(S.q[i], iq) : S.q[i];
        S.q[i] = __fmul_rn(qv, p.scale);
        if (p.l2) S.k[i] = __fmul_rn(S.k[i], ik);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[slot]);
    }
    return;
  }

  // ----------------------------------------------------------- state warp
  if (lane == 0) {
    mbar_arrive_expect_tx(&bar, HKD * 32 * 4);
    sm100::tma_load_2d(st, &tmS, &bar, col0, h * HKD);
  }
  float s[HKD];
  const bool have = wait(&bar, 0);
  if (!have) {
    mbar_wait(&bar, 0);  // a second bounded wait for the copy in flight
    return;
  }
#pragma unroll
  for (int kd = 0; kd < HKD; ++kd) s[kd] = st[kd * 32 + lane];
  bool ok = p.rows > 0 && wait(&full[0], 0);
  float delta = 0.f;
  if (ok) {  // pass 1 of position 0: decay, then kv = S^T k
    const Stage<HKD>& A = ring[0];
    const float4* k4 = reinterpret_cast<const float4*>(A.k);
    float kv = 0.f;
#pragma unroll
    for (int k = 0; k < HKD / 4; ++k) {
      const float4 kk = k4[k];
      const float kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float r = __fmul_rn(s[4 * k + e], A.decay);
        s[4 * k + e] = r;
        kv = __fadd_rn(kv, __fmul_rn(r, kw[e]));
      }
    }
    delta = __fmul_rn(__fsub_rn(A.v[lane], kv), A.beta);
  }
  for (int64_t t = 0; ok && t < p.rows; ++t) {
    const int slot = int(t % kRing), nslot = int((t + 1) % kRing);
    const Stage<HKD>& A = ring[slot];
    const bool next = t + 1 < p.rows;
    if (next && !wait(&full[nslot], uint32_t(((t + 1) / kRing) & 1))) {
      ok = false;
      break;
    }
    const Stage<HKD>& B = ring[nslot];
    float o, kv;
    if (next)
      sweep<HKD, true>(s, A.k, A.q, delta, B.k, B.decay, o, kv);
    else
      sweep<HKD, false>(s, A.k, A.q, delta, nullptr, 0.f, o, kv);
    p.out[t * value + int64_t(h) * p.hvd + col] = o;
    if (next) delta = __fmul_rn(__fsub_rn(B.v[lane], kv), B.beta);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // slot t is read
  }
  if (!ok) return;  // the status word tells the caller; the state is not written
#pragma unroll
  for (int kd = 0; kd < HKD; ++kd) st[kd * 32 + lane] = s[kd];
  sm100::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    sm100::tma_store_2d(&tmS, st, col0, h * HKD);
    sm100::tma_store_commit();
    sm100::tma_store_wait_read();
  }
  __syncwarp();
}

// ------------------------------------------------------------- one row
// A call of one position (every decode step) is a chain of latencies: the
// inputs, the two L2 sums, pass 1 (kv) and pass 2 (out), each a sequential
// sum of HKD terms.  A warp that only adds issues about four cycles per
// term; one that also forms the terms (two or three multiplies each, a
// store in pass 2) about ten.  So warp 0 only sums: the q / k L2 sums (lanes
// 0 / 1, over the squares the row warps wrote), then kv and out for its 32
// columns, each term read from shared memory.
// The HKD / 32 row warps hold the state rows, 8-row blocks dealt round-robin
// (warp w: rows 8 (NR g + w) .. + 8 for g = 0, 1, ...), and form each pass's
// terms for a group of rows at a time: group g, rows [8 NR g, 8 NR (g + 1)),
// is one block from every row warp, published by named barrier 1 + g.  Pass
// 2's row warps also store the new state rows.  Terms are laid out
// [kd / 4][column][4] so that a row warp writes four rows of its column with
// one 16-byte store and warp 0 reads four terms with one.  Same operations,
// same order, same bits as gdn_step_column.  HVD (the state's row length) is
// a constant, so that the state rows are one base address and immediate
// offsets.
template <int HKD, int HVD>
__global__ void __launch_bounds__(HKD + 32, 1) gdn_step_split_kernel(const GdnParams p) {
  constexpr int NR = HKD / 32;      // row warps
  constexpr int NG = 4;             // groups of rows (barriers 1 .. 4)
  constexpr int GR = HKD / NG;      // rows per group = 8 NR
  static_assert(GR == 8 * NR, "one 8-row block per row warp and group");
  constexpr int kFront = 5, kInv = 6, kDelta = 7;  // named barriers, HKD + 32 threads each
  __shared__ __align__(16) float qraw[HKD];
  __shared__ __align__(16) float kraw[HKD];
  __shared__ __align__(16) float4 terms[HKD / 4][32];
  __shared__ __align__(16) float sqs[2][HKD];  // the squares of q and of k
  __shared__ float misc[4];  // inv_q, inv_k, decay
  __shared__ float ds[32];   // delta per column
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.y * 32 + lane;
  const int kh = h / (p.nv / p.nk);
  const int64_t key = int64_t(p.nk) * HKD;
  const float* qrow = p.qkv + int64_t(kh) * HKD;
  const float* krow = p.qkv + key + int64_t(kh) * HKD;
  float* srow = p.state + int64_t(h) * HKD * HVD + col;  // column col, row kd at kd * HVD
  constexpr int NT = HKD + 32;

  if (warp > 0) {  // ------------------------------------------------ row warps
    const int w = warp - 1, t = threadIdx.x - 32;
#pragma unroll
    for (int g = 0; g < NG; ++g)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(srow - lane + (8 * (NR * g + w) + (lane & 7)) * HVD));
    if (lane == 0) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(qrow + 32 * w));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(krow + 32 * w));
    }
    griddep_wait();
    griddep_launch_dependents();
    const float qv = qrow[t], kv = krow[t];
    qraw[t] = qv;
    kraw[t] = kv;
    sqs[0][t] = __fmul_rn(qv, qv);
    sqs[1][t] = __fmul_rn(kv, kv);
    float s[NG * 8];
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int e = 0; e < 8; ++e) s[8 * g + e] = srow[(8 * (NR * g + w) + e) * HVD];
    named_arrive(kFront, NT);
    named_sync(kInv, NT);  // the inverses and the decay
    const float ik = misc[1], decay = misc[2];
    float kn[NG * 8], qn[NG * 8];  // this warp's rows of k inv_k and q inv_q scale
    // pass 1: the decayed rows and their terms r k
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const int kd0 = 8 * (NR * g + w);
      float tm[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        kn[8 * g + e] = p.l2 ? __fmul_rn(kraw[kd0 + e], ik) : kraw[kd0 + e];
        const float r = __fmul_rn(s[8 * g + e], decay);
        s[8 * g + e] = r;
        tm[e] = __fmul_rn(r, kn[8 * g + e]);
      }
      terms[kd0 / 4][lane] = make_float4(tm[0], tm[1], tm[2], tm[3]);
      terms[kd0 / 4 + 1][lane] = make_float4(tm[4], tm[5], tm[6], tm[7]);
      named_arrive(1 + g, NT);
    }
    {  // q inv_q scale (two roundings) while warp 0 sums
      const float iq = misc[0];
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float qq = qraw[8 * (NR * g + w) + e];
          qn[8 * g + e] = __fmul_rn(p.l2 ? __fmul_rn(qq, iq) : qq, p.scale);
        }
    }
    named_sync(kDelta, NT);  // warp 0 has summed pass 1's terms
    const float delta = ds[lane];
    // pass 2: the new rows S + k delta, stored, and their terms r (q scale)
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const int kd0 = 8 * (NR * g + w);
      float tm[8];
      float rn[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        rn[e] = __fadd_rn(s[8 * g + e], __fmul_rn(kn[8 * g + e], delta));
        tm[e] = __fmul_rn(rn[e], qn[8 * g + e]);
      }
      terms[kd0 / 4][lane] = make_float4(tm[0], tm[1], tm[2], tm[3]);
      terms[kd0 / 4 + 1][lane] = make_float4(tm[4], tm[5], tm[6], tm[7]);
      named_arrive(1 + g, NT);
#pragma unroll
      for (int e = 0; e < 8; ++e) srow[(kd0 + e) * HVD] = rn[e];
    }
    return;
  }

  // ------------------------------------------------------------- warp 0
  griddep_wait();
  griddep_launch_dependents();
  const float v = p.qkv[2 * key + int64_t(h) * HVD + col];
  const float beta = p.beta[h], decay = p.decay[h];
  named_sync(kFront, NT);  // q, k in shared memory
  if (p.l2 && lane < 2) {  // lanes 0 / 1: the squares of q / k summed in order, 32 at a time
    const float4* x4 = reinterpret_cast<const float4*>(sqs[lane]);
    float sum = 0.f;
#pragma unroll
    for (int b = 0; b < HKD / 32; ++b) {
      float4 r[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = x4[8 * b + j];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sum = __fadd_rn(sum, r[j].x);
        sum = __fadd_rn(sum, r[j].y);
        sum = __fadd_rn(sum, r[j].z);
        sum = __fadd_rn(sum, r[j].w);
      }
    }
    sum = __fadd_rn(sum, p.eps);
    misc[lane] = __fdiv_rn(1.0f, __fsqrt_rn(sum));
  }
  if (lane == 2) misc[2] = decay;
  __syncwarp();
  named_arrive(kInv, NT);
  // kv = S^T k, then out = S^T (q scale): kd ascending, a group at a time
  const float kv = sum_terms<NG, GR>(terms, lane, NT);
  ds[lane] = __fmul_rn(__fsub_rn(v, kv), beta);
  named_arrive(kDelta, NT);
  p.out[int64_t(h) * HVD + col] = sum_terms<NG, GR>(terms, lane, NT);
}


// ---------------------------------------------------- rows, split passes
// A block of positions in order (hb_gdn_decode with rows > 1, hb_gdn_prefill
// below the chunked kernels' minimum), the one-row form's division of work
// carried over the positions.  Per position t the row warps, once delta_t is
// known, form for each of their state rows r = S + k_t delta_t (pass 2 of
// t), its output term r (q_t scale), and -- when t + 1 exists -- r' = r
// decay_{t+1} and its term r' k_{t+1} (pass 1 of t + 1), keeping r' as the
// row; warp 0 sums both term arrays a group of rows at a time, the two
// ordered chains interleaved, writes out_t and forms delta_{t+1}.  The
// producer warps stage each position's normalised q and k (their sequential
// L2 sums), the CTA's v values, beta and decay in the ring ahead of use.
// Same operations in the same order as gdn_step_column, position after
// position.
constexpr int kRowsProducers = 4;
constexpr int64_t kRowsSplitMax = 16;  // blocks the split form takes (more: the pipelined form)

template <int HKD, int HVD>
__global__ void __launch_bounds__(32 * (1 + HKD / 32 + kRowsProducers), 1)
    gdn_rows_split_kernel(const GdnParams p) {
  constexpr int NR = HKD / 32;      // row warps
  constexpr int NG = 4;             // groups of rows (barriers 1 .. 4)
  constexpr int GR = HKD / NG;      // rows per group = 8 NR
  constexpr int NP = kRowsProducers;
  static_assert(GR == 8 * NR, "one 8-row block per row warp and group");
  constexpr int kDelta = 5;         // delta in ds (warp 0 arrives, the row warps wait)
  constexpr int NT = HKD + 32;      // threads of the group and delta barriers
  __shared__ __align__(16) float4 ta[HKD / 4][32];  // pass-2 terms of t
  __shared__ __align__(16) float4 tb[HKD / 4][32];  // pass-1 terms of t + 1
  __shared__ Stage<HKD> ring[kRing];
  __shared__ float inv[NP][2];
  __shared__ float ds[32];
  __shared__ __align__(8) uint64_t full[kRing], empty[kRing];
  __shared__ int abort_flag;
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.y * 32 + lane;
  const int kh = h / (p.nv / p.nk);
  const int64_t key = int64_t(p.nk) * HKD, value = int64_t(p.nv) * HVD;
  const int64_t conv = 2 * key + value;
  float* scol = p.state + int64_t(h) * HKD * HVD + col;  // column col, row kd at kd * HVD

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NR + 1);  // the row warps and warp 0 release a slot
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp >= 1 && warp <= NR) {  // the row warps' state lines into L2
    const int w = warp - 1;
#pragma unroll
    for (int g = 0; g < NG; ++g)
      if (lane < 8) asm volatile("prefetch.global.L2 [%0];" ::"l"(scol - lane + (8 * (NR * g + w) + lane) * HVD));
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  // a bounded wait of the whole warp; false (and the abort flag) on timeout
  auto wait = [&](uint64_t* b, uint32_t parity) -> bool {
    if (*reinterpret_cast<volatile int*>(&abort_flag)) return false;
    if (__all_sync(0xFFFFFFFFu, mbar_wait(b, parity))) return true;
    if (lane == 0) record_status(p.status, kStatusTimeout);
    *reinterpret_cast<volatile int*>(&abort_flag) = 1;
    return false;
  };
  const int64_t rows = p.rows;

  if (warp > NR) {  // ------------------------------------------- producers
    const int w = warp - 1 - NR;
    for (int64_t t = w; t < rows; t += NP) {
      const int slot = int(t % kRing);
      const int64_t use = t / kRing;
      if (use > 0 && !wait(&empty[slot], uint32_t((use - 1) & 1))) break;
      Stage<HKD>& S = ring[slot];
      const float* row = p.qkv + t * conv;
#pragma unroll
      for (int i = lane; i < HKD; i += 32) {
        S.q[i] = row[int64_t(kh) * HKD + i];
        S.k[i] = row[key + int64_t(kh) * HKD + i];
      }
      S.v[lane] = row[2 * key + int64_t(h) * HVD + col];
      if (lane == 0) {
        S.beta = p.beta[t * p.nv + h];
        S.decay = p.decay[t * p.nv + h];
      }
      __syncwarp();
      // q <- q inv_q scale (two roundings), k <- k inv_k
      float iq = 1.f, ik = 1.f;
      if (p.l2) {
        if (lane < 2) inv[w][lane] = l2_inverse<HKD>(lane == 0 ? S.q : S.k, p.eps);
        __syncwarp();
        iq = inv[w][0];
        ik = inv[w][1];
      }
#pragma unroll
      for (int i = lane; i < HKD; i += 32) {
        const float qv = p.l2 ? __fmul_rn(S.q[i], iq) : S.q[i];
        S.q[i] = __fmul_rn(qv, p.scale);
        if (p.l2) S.k[i] = __fmul_rn(S.k[i], ik);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[slot]);
    }
    return;
  }

  if (warp >= 1) {  // -------------------------------------------- row warps
    const int w = warp - 1;
    float s[NG * 8];  // state rows 8 (NR g + w) + e of column col
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int e = 0; e < 8; ++e) s[8 * g + e] = scol[(8 * (NR * g + w) + e) * HVD];
    // pass 1 of position 0: the decayed rows and their terms r k_0
    wait(&full[0], 0);
    {
      const Stage<HKD>& A = ring[0];
      const float decay = A.decay;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const int kd0 = 8 * (NR * g + w);
        float tm[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float r = __fmul_rn(s[8 * g + e], decay);
          s[8 * g + e] = r;
          tm[e] = __fmul_rn(r, A.k[kd0 + e]);
        }
        tb[kd0 / 4][lane] = make_float4(tm[0], tm[1], tm[2], tm[3]);
        tb[kd0 / 4 + 1][lane] = make_float4(tm[4], tm[5], tm[6], tm[7]);
        named_arrive(1 + g, NT);
      }
    }
    // position t: pass 2 of t and pass 1 of t + 1 on every row
    for (int64_t t = 0; t < rows; ++t) {
      named_sync(kDelta, NT);  // delta_t in ds
      const float delta = ds[lane];
      const bool next = t + 1 < rows;
      const Stage<HKD>& A = ring[t % kRing];
      if (next) wait(&full[(t + 1) % kRing], uint32_t(((t + 1) / kRing) & 1));
      const Stage<HKD>& B = ring[(t + 1) % kRing];
      const float dn = next ? B.decay : 0.f;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const int kd0 = 8 * (NR * g + w);
        // the block's k_t, q_t, k_{t+1} in 16-byte reads
        float ak[8], aq[8], bk[8];
#pragma unroll
        for (int h4 = 0; h4 < 2; ++h4) {
          const float4 x = *reinterpret_cast<const float4*>(A.k + kd0 + 4 * h4);
          const float4 y = *reinterpret_cast<const float4*>(A.q + kd0 + 4 * h4);
          const float4 z = next ? *reinterpret_cast<const float4*>(B.k + kd0 + 4 * h4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
          ak[4 * h4] = x.x; ak[4 * h4 + 1] = x.y; ak[4 * h4 + 2] = x.z; ak[4 * h4 + 3] = x.w;
          aq[4 * h4] = y.x; aq[4 * h4 + 1] = y.y; aq[4 * h4 + 2] = y.z; aq[4 * h4 + 3] = y.w;
          bk[4 * h4] = z.x; bk[4 * h4 + 1] = z.y; bk[4 * h4 + 2] = z.z; bk[4 * h4 + 3] = z.w;
        }
        float ua[8], ub[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float r = __fadd_rn(s[8 * g + e], __fmul_rn(ak[e], delta));
          ua[e] = __fmul_rn(r, aq[e]);
          if (next) {
            const float r2 = __fmul_rn(r, dn);
            ub[e] = __fmul_rn(r2, bk[e]);
            s[8 * g + e] = r2;
          } else {
            ub[e] = 0.f;
            s[8 * g + e] = r;
          }
        }
        ta[kd0 / 4][lane] = make_float4(ua[0], ua[1], ua[2], ua[3]);
        ta[kd0 / 4 + 1][lane] = make_float4(ua[4], ua[5], ua[6], ua[7]);
        if (next) {
          tb[kd0 / 4][lane] = make_float4(ub[0], ub[1], ub[2], ub[3]);
          tb[kd0 / 4 + 1][lane] = make_float4(ub[4], ub[5], ub[6], ub[7]);
        }
        named_arrive(1 + g, NT);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[t % kRing]);  // slot t's k and q are read
    }
    if (!*reinterpret_cast<volatile int*>(&abort_flag)) {  // the state after the last position
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) scol[(8 * (NR * g + w) + e) * HVD] = s[8 * g + e];
    }
    return;
  }

  // --------------------------------------------------------------- warp 0
  // the two ordered sums of one position: out over ta and (when `next`) kv
  // over tb, kd ascending, group after group, both chains interleaved and
  // the next group's terms read while this group is summed
  auto sums = [&](bool with_a, bool with_b, float& oa, float& ob) {
    float a = 0.f, b = 0.f;
    float4 ca[GR / 4], cb[GR / 4], na[GR / 4], nb[GR / 4];
    named_sync(1, NT);
#pragma unroll
    for (int j = 0; j < GR / 4; ++j) {
      ca[j] = with_a ? ta[j][lane] : make_float4(0.f, 0.f, 0.f, 0.f);
      cb[j] = with_b ? tb[j][lane] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      if (g + 1 < NG) {
        named_sync(2 + g, NT);
#pragma unroll
        for (int j = 0; j < GR / 4; ++j) {
          na[j] = with_a ? ta[(g + 1) * (GR / 4) + j][lane] : make_float4(0.f, 0.f, 0.f, 0.f);
          nb[j] = with_b ? tb[(g + 1) * (GR / 4) + j][lane] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < GR / 4; ++j) {
        a = __fadd_rn(a, ca[j].x);
        b = __fadd_rn(b, cb[j].x);
        a = __fadd_rn(a, ca[j].y);
        b = __fadd_rn(b, cb[j].y);
        a = __fadd_rn(a, ca[j].z);
        b = __fadd_rn(b, cb[j].z);
        a = __fadd_rn(a, ca[j].w);
        b = __fadd_rn(b, cb[j].w);
      }
#pragma unroll
      for (int j = 0; j < GR / 4; ++j) {
        ca[j] = na[j];
        cb[j] = nb[j];
      }
    }
    oa = a;
    ob = b;
  };
  wait(&full[0], 0);
  {
    float unused, kv;
    sums(false, true, unused, kv);
    const Stage<HKD>& A = ring[0];
    ds[lane] = __fmul_rn(__fsub_rn(A.v[lane], kv), A.beta);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[0]);  // slot 0's v and beta are read
    named_arrive(kDelta, NT);
  }
  for (int64_t t = 0; t < rows; ++t) {
    const bool next = t + 1 < rows;
    if (next) wait(&full[(t + 1) % kRing], uint32_t(((t + 1) / kRing) & 1));
    float o, kv;
    sums(true, next, o, kv);
    if (!*reinterpret_cast<volatile int*>(&abort_flag)) p.out[t * value + int64_t(h) * HVD + col] = o;
    if (next) {
      const Stage<HKD>& B = ring[(t + 1) % kRing];
      ds[lane] = __fmul_rn(__fsub_rn(B.v[lane], kv), B.beta);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[(t + 1) % kRing]);  // slot t + 1's v and beta are read
      named_arrive(kDelta, NT);
    }
  }
}

}  // namespace

bool gdn_decode_serves(const hb_gdn_shape& s) {
  return (s.hkd == 64 || s.hkd == 128) && s.hvd > 0 && s.hvd % 32 == 0 && s.hvd <= 512;
}

cudaError_t launch_gdn_decode(const GdnLaunch& L, cudaStream_t st) {
  GdnParams p;
  p.state = L.call.state;
  p.out = L.call.output;
  p.qkv = L.call.qkv;
  p.beta = L.call.beta;
  p.decay = L.call.decay;
  p.rows = L.call.rows;
  p.nk = int(L.shape.nk);
  p.nv = int(L.shape.nv);
  p.hvd = int(L.shape.hvd);
  p.l2 = L.call.l2;
  p.eps = L.call.eps;
  p.scale = L.scale;
  p.status = L.status;
  // the state as [nv*hkd rows][hvd columns] f32, tiles [hkd rows][32 columns]
  CUtensorMap tm;
  if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.call.state,
                 uint64_t(L.shape.nv) * L.shape.hkd, uint64_t(L.shape.hvd), uint64_t(L.shape.hvd),
                 uint32_t(L.shape.hkd), 32, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  // programmatic dependent launch: the CTAs of consecutive steps are made
  // resident while the previous step finishes (griddepcontrol.wait in the
  // kernel orders every memory access after it)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(L.shape.nv), unsigned(L.shape.hvd / 32));
  cfg.blockDim = dim3(32 * (1 + kProducers));
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // a short block of positions: split passes (2 rows 7.2 -> 4.6 µs, 16 rows
  // 18.2 -> 17.6 µs); longer blocks run at ≈ 0.86 µs per position in the
  // pipelined form against ≈ 0.93 in this one
  if (L.call.rows > 1 && L.call.rows <= kRowsSplitMax && L.shape.hvd == 128) {
    cfg.blockDim = dim3(unsigned(32 * (1 + L.shape.hkd / 32 + kRowsProducers)));
    if (L.shape.hkd == 128) return cudaLaunchKernelEx(&cfg, gdn_rows_split_kernel<128, 128>, p);
    if (L.shape.hkd == 64) return cudaLaunchKernelEx(&cfg, gdn_rows_split_kernel<64, 128>, p);
    return cudaErrorInvalidValue;
  }
  if (L.call.rows == 1 && L.shape.hvd == 128) {  // one position: the latency-first form
    cfg.blockDim = dim3(unsigned(L.shape.hkd + 32));
    if (L.shape.hkd == 128) return cudaLaunchKernelEx(&cfg, gdn_step_split_kernel<128, 128>, p);
    if (L.shape.hkd == 64) return cudaLaunchKernelEx(&cfg, gdn_step_split_kernel<64, 128>, p);
    return cudaErrorInvalidValue;
  }
  if (L.shape.hkd == 128) return cudaLaunchKernelEx(&cfg, gdn_decode_kernel<128>, tm, p);
  if (L.shape.hkd == 64) return cudaLaunchKernelEx(&cfg, gdn_decode_kernel<64>, tm, p);
  return cudaErrorInvalidValue;
}

}  // namespace hb
