// gdn_prefill.cu -- chunked GatedDeltaNet prefill on sm_100a tensor cores.
//
// Replaces, for long blocks, the delta-causal-recurrence node
// (RecurrenceFn, src/jit/emit_recurrence.rs:63-73; traversal
// src/jit/target/x86/execution/delta.rs:519-607) with the chunked WY form the
// reference writes for its matrix engine (src/jit/target/aarch64/deltanet_chunk.rs:6-15),
// in the same "decay before read" order.  For a value head and a chunk of C =
// 64 positions starting from state S0 (dk x dv), with G_t = sum_{s<=t} log a_s,
// gamma_t = e^{G_t}, r_tj = e^{G_t - G_j}:
//
//   A_tj = beta_t r_tj (k_t . k_j)  (j < t)       T = (I + A)^-1
//   W    = T diag(beta gamma) K                   U = T diag(beta) V
//   D    = U - W S0                               (the corrected values)
//   O    = diag(gamma scale) Q S0 + M D,   M_tj = scale r_tj (q_t . k_j)  (j <= t)
//   S_C  = gamma_{C-1} S0 + (diag(r_{C-1,.}) K)^T D
//
// Two kernels:
//  * gdn_prep, one CTA per (chunk, key head): both value heads of the key head
//    at once so that every product is an M=128 tcgen05 MMA -- [K;Q] K^T gives
//    K K^T and Q K^T; [T0'; T1'] K gives W for both heads; a block-diagonal
//    [T0'' 0; 0 T1''] times [V0; V1] gives U for both.  T comes from forward
//    substitution on the CUDA cores (one thread per column).  It writes W, U,
//    M, Qg = diag(gamma scale) Q, Kt = diag(r_{C-1,.}) K and gamma_{C-1}.
//  * gdn_scan, one CTA per (value head, half of dv), sequential over chunks:
//    [W; Qg] S0 in one MMA (rows 0-63 W S0, rows 64-127 Q S0), D on the CUDA
//    cores, then [0; M] D accumulated onto the Q S0 rows (= O) and Kt^T D
//    accumulated onto the state, which lives in TMEM in f32 (scaled by
//    gamma_{C-1} first); its bf16 copy in shared memory is the next chunk's
//    operand.  Chunk inputs stream in by TMA two chunks ahead.
// MMA operands are bf16, accumulators and the state f32; the result is not
// the bits of the sequential recurrence (as for the reference's own chunked
// kernel) and is held to a relative Frobenius tolerance.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_internal.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

using namespace sm100;

constexpr int C = 64;    // positions per chunk
constexpr int DK = 128;  // key head dim
constexpr int DV = 128;  // value head dim

// ------------------------------------------------------------------ prep

constexpr int P_SA = 0;             // [K; Q] bf16, 2 blocks of [128 rows x 128 B]
constexpr int P_SV = 32768;         // [V0; V1] bf16, 2 blocks of [128 rows x 128 B]
constexpr int P_S2 = 65536;         // [T0 bg0; T1 bg1] bf16, 1 block [128 x 128 B]
constexpr int P_S3 = 81920;         // blockdiag(T0 b0, T1 b1) bf16, 2 blocks
constexpr int P_AF = 114688;        // A f32 [2][64][65] (row stride 65: no bank conflicts)
constexpr int P_VEC = 149504;       // beta[2][64], G[2][64]
constexpr int P_BAR = P_VEC + 1024;
constexpr int P_SMEM = P_BAR + 64 + 1024;

struct PrepParams {
  const float* qkv;
  const float* beta;
  const float* decay;
  int64_t rows;
  int nk, nv, nchunks, l2;
  float eps, scale;
  uint16_t* W;   // [nv][nchunks][64][128]
  uint16_t* Qg;  // same
  uint16_t* Kt;  // same
  uint16_t* M;   // [nv][nchunks][64][64]
  float* U;      // [nv][nchunks][64][128]
  float* gl;     // [nv][nchunks]
  int* status;
};

// byte offset of element (row, col) of a K-major bf16 tile whose column
// blocks of 64 are `block_bytes` apart, 128B-swizzled
HB_DEV uint32_t sw_off(int row, int col, int block_bytes) {
  return uint32_t((col >> 6) * block_bytes + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                  (col & 7) * 2);
}

__global__ void __launch_bounds__(128, 1) gdn_prep_kernel(const PrepParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + P_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 2);
  float* beta_s = reinterpret_cast<float*>(smem + P_VEC);  // [2][64]
  float* G_s = beta_s + 128;                               // [2][64]

  const int c = blockIdx.x, kh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t key = int64_t(p.nk) * DK, conv = 2 * key + int64_t(p.nv) * DV;
  const int64_t t0 = int64_t(c) * C;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 256);
  // zero the block-diagonal operand (its off-diagonal halves stay zero)
  for (int i = tid; i < 32768 / 16; i += 128)
    reinterpret_cast<uint4*>(smem + P_S3)[i] = make_uint4(0, 0, 0, 0);

  // ---- rows: k (tid < 64) or q (tid >= 64) of position t0 + (tid & 63), L2 normalised
  {
    const int r = tid & 63, which = tid >> 6;
    const int64_t t = t0 + r;
    float x[DK];
    if (t < p.rows) {
      const float4* src = reinterpret_cast<const float4*>(
          p.qkv + t * conv + (which ? int64_t(kh) * DK : key + int64_t(kh) * DK));
#pragma unroll
      for (int i = 0; i < DK / 4; ++i) {
        const float4 v = src[i];
        x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DK; ++i) x[i] = 0.f;
    }
    float inv = 1.f;
    if (p.l2) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < DK; ++i) ss = fmaf(x[i], x[i], ss);
      inv = 1.f / sqrtf(ss + p.eps);
    }
    const int row = which * 64 + r;  // stacked [K; Q]
#pragma unroll
    for (int ch = 0; ch < DK / 8; ++ch) {
      uint4 w;
      w.x = pack_bf16x2(x[8 * ch] * inv, x[8 * ch + 1] * inv);
      w.y = pack_bf16x2(x[8 * ch + 2] * inv, x[8 * ch + 3] * inv);
      w.z = pack_bf16x2(x[8 * ch + 4] * inv, x[8 * ch + 5] * inv);
      w.w = pack_bf16x2(x[8 * ch + 6] * inv, x[8 * ch + 7] * inv);
      *reinterpret_cast<uint4*>(smem + P_SA + sw_off(row, ch * 8, 16384)) = w;
    }
  }
  // ---- values of both heads (row = head * 64 + j), gates
  {
    const int r = tid & 63, hh = tid >> 6, h = kh * 2 + hh;
    const int64_t t = t0 + r;
    float x[DV];
    if (t < p.rows) {
      const float4* src =
          reinterpret_cast<const float4*>(p.qkv + t * conv + 2 * key + int64_t(h) * DV);
#pragma unroll
      for (int i = 0; i < DV / 4; ++i) {
        const float4 v = src[i];
        x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DV; ++i) x[i] = 0.f;
    }
#pragma unroll
    for (int ch = 0; ch < DV / 8; ++ch) {
      uint4 w;
      w.x = pack_bf16x2(x[8 * ch], x[8 * ch + 1]);
      w.y = pack_bf16x2(x[8 * ch + 2], x[8 * ch + 3]);
      w.z = pack_bf16x2(x[8 * ch + 4], x[8 * ch + 5]);
      w.w = pack_bf16x2(x[8 * ch + 6], x[8 * ch + 7]);
      *reinterpret_cast<uint4*>(smem + P_SV + sw_off(hh * 64 + r, ch * 8, 16384)) = w;
    }
    const bool in = t < p.rows;
    beta_s[hh * 64 + r] = in ? p.beta[t * p.nv + h] : 0.f;
    G_s[hh * 64 + r] = in ? logf(p.decay[t * p.nv + h]) : 0.f;  // padded rows: decay 1
  }
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t sa = smem_u32(smem + P_SA);

  // ---- MMA 1: [K; Q] K^T -> TMEM cols [0, 64)
  if (tid == 0) {
    constexpr uint32_t id = idesc_bf16(128, 64, false, false);
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
      mma_bf16_ss(tmem, sw128_desc(sa + off, 16, 1024), sw128_desc(sa + off, 16, 1024), id, kk > 0);
    }
    mma_commit(&bar[0]);
  }
  // ---- prefix sums of log decay per head (warp hh, 2 values per lane)
  if (warp < 2) {
    float a0 = G_s[warp * 64 + 2 * lane], a1 = G_s[warp * 64 + 2 * lane + 1];
    float s = a0 + a1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= o) s += n;
    }
    const float before = s - (a0 + a1);
    G_s[warp * 64 + 2 * lane] = before + a0;
    G_s[warp * 64 + 2 * lane + 1] = s;
  }
  __syncthreads();
  if (!mbar_wait(&bar[0], 0)) record_status(p.status, kStatusTimeout);
  fence_after_sync();

  // ---- read K K^T (rows 0-63) and Q K^T (rows 64-127)
  float* Af = reinterpret_cast<float*>(smem + P_AF);
  {
    const uint32_t tq = tmem + (uint32_t(warp * 32) << 16);
    uint32_t ra[32], rb[32];
    tmem_ld32(tq, ra);
    tmem_ld32(tq + 32, rb);
    tmem_wait_ld();
    const int t = tid & 63;
    if (tid < 64) {  // A_h[t][j] = beta_t r_tj (k_t . k_j), j < t
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float bt = beta_s[hh * 64 + t], Gt = G_s[hh * 64 + t];
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float kk = __uint_as_float(j < 32 ? ra[j] : rb[j - 32]);
          Af[(hh * 64 + t) * 65 + j] = j < t ? bt * __expf(Gt - G_s[hh * 64 + j]) * kk : 0.f;
        }
      }
    } else {  // M_h[t][j] = scale r_tj (q_t . k_j), j <= t
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int h = kh * 2 + hh;
        const float Gt = G_s[hh * 64 + t];
        uint16_t* mrow = p.M + ((int64_t(h) * p.nchunks + c) * C + t) * C;
#pragma unroll
        for (int j8 = 0; j8 < 8; ++j8) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j0 = j8 * 8 + 2 * i, j1 = j0 + 1;
            const float q0 = __uint_as_float(j0 < 32 ? ra[j0] : rb[j0 - 32]);
            const float q1 = __uint_as_float(j1 < 32 ? ra[j1] : rb[j1 - 32]);
            const float m0 = j0 <= t ? p.scale * __expf(Gt - G_s[hh * 64 + j0]) * q0 : 0.f;
            const float m1 = j1 <= t ? p.scale * __expf(Gt - G_s[hh * 64 + j1]) * q1 : 0.f;
            w[i] = pack_bf16x2(m0, m1);
          }
          reinterpret_cast<uint4*>(mrow)[j8] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
  // ---- Qg = diag(gamma scale) Q and Kt = diag(r_{63,.}) K for both heads
  {
    const int hh = tid >> 6, t = tid & 63, h = kh * 2 + hh;
    const float G = G_s[hh * 64 + t];
    const float gq = __expf(G) * p.scale, gk = __expf(G_s[hh * 64 + 63] - G);
    const int64_t base = ((int64_t(h) * p.nchunks + c) * C + t) * DK;
#pragma unroll 4
    for (int ch = 0; ch < DK / 8; ++ch) {
      const uint4 kv = *reinterpret_cast<const uint4*>(smem + P_SA + sw_off(t, ch * 8, 16384));
      const uint4 qv = *reinterpret_cast<const uint4*>(smem + P_SA + sw_off(64 + t, ch * 8, 16384));
      const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w}, qw[4] = {qv.x, qv.y, qv.z, qv.w};
      uint32_t ko[4], qo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ko[i] = pack_bf16x2(bf16lo(kw[i]) * gk, bf16hi(kw[i]) * gk);
        qo[i] = pack_bf16x2(bf16lo(qw[i]) * gq, bf16hi(qw[i]) * gq);
      }
      reinterpret_cast<uint4*>(p.Kt + base)[ch] = make_uint4(ko[0], ko[1], ko[2], ko[3]);
      reinterpret_cast<uint4*>(p.Qg + base)[ch] = make_uint4(qo[0], qo[1], qo[2], qo[3]);
    }
    if (t == 63) p.gl[int64_t(h) * p.nchunks + c] = __expf(G);
  }
  fence_before_sync();
  __syncthreads();

  // ---- T = (I + A)^-1 by forward substitution: thread (head hh, column j)
  {
    const int hh = tid >> 6, j = tid & 63;
    const float* A = Af + hh * 64 * 65;
    float tc[64];
#pragma unroll
    for (int t = 0; t < 64; ++t) {
      float acc = 0.f;
#pragma unroll
      for (int s = 0; s < t; ++s) acc = fmaf(A[t * 65 + s], tc[s], acc);
      tc[t] = t == j ? 1.f : (t < j ? 0.f : -acc);
    }
    const float bj = beta_s[hh * 64 + j], gj = __expf(G_s[hh * 64 + j]);
    const float wbg = bj * gj;
    // S2 row (hh*64 + t), column j: T[t][j] beta_j gamma_j
    // S3 row (hh*64 + t), column hh*64 + j: T[t][j] beta_j
#pragma unroll
    for (int t = 0; t < 64; ++t) {
      const int row = hh * 64 + t;
      *reinterpret_cast<uint16_t*>(smem + P_S2 + sw_off(row, j, 16384)) =
          f32_to_bf16_cvtne(tc[t] * wbg);
      *reinterpret_cast<uint16_t*>(smem + P_S3 + sw_off(row, hh * 64 + j, 16384)) =
          f32_to_bf16_cvtne(tc[t] * bj);
    }
  }
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();

  // ---- MMA 2: W = [T0 bg0; T1 bg1] K -> cols [0,128); MMA 3: U -> cols [128,256)
  if (tid == 0) {
    constexpr uint32_t id = idesc_bf16(128, 128, false, true);
    const uint32_t s2 = smem_u32(smem + P_S2), s3 = smem_u32(smem + P_S3),
                   sv = smem_u32(smem + P_SV);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      mma_bf16_ss(tmem, sw128_desc(s2 + kk * 32, 16, 1024), sw128_desc(sa + kk * 2048, 16384, 1024),
                  id, kk > 0);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      mma_bf16_ss(tmem + 128, sw128_desc(s3 + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                  sw128_desc(sv + kk * 2048, 16384, 1024), id, kk > 0);
    mma_commit(&bar[1]);
  }
  __syncwarp();
  if (!mbar_wait(&bar[1], 0)) record_status(p.status, kStatusTimeout);
  fence_after_sync();
  {
    const int hh = tid >> 6, t = tid & 63, h = kh * 2 + hh;
    const uint32_t tq = tmem + (uint32_t(warp * 32) << 16);
    const int64_t base = ((int64_t(h) * p.nchunks + c) * C + t) * DK;
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t w[32], u[32];
      tmem_ld32(tq + cb * 32, w);
      tmem_ld32(tq + 128 + cb * 32, u);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<uint4*>(p.W + base + cb * 32)[i] =
            make_uint4(pack_bf16x2(__uint_as_float(w[8 * i]), __uint_as_float(w[8 * i + 1])),
                       pack_bf16x2(__uint_as_float(w[8 * i + 2]), __uint_as_float(w[8 * i + 3])),
                       pack_bf16x2(__uint_as_float(w[8 * i + 4]), __uint_as_float(w[8 * i + 5])),
                       pack_bf16x2(__uint_as_float(w[8 * i + 6]), __uint_as_float(w[8 * i + 7])));
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(p.U + base + cb * 32)[i] =
            make_float4(__uint_as_float(u[4 * i]), __uint_as_float(u[4 * i + 1]),
                        __uint_as_float(u[4 * i + 2]), __uint_as_float(u[4 * i + 3]));
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------------------------ scan

constexpr int BV = 64;                    // value columns per CTA
constexpr int S_A1 = 0;                   // per stage: [W; Qg] 2 blocks x 16 KB
constexpr int S_A2 = 32768;               //            [0; M] 1 block 16 KB
constexpr int S_KT = 49152;               //            Kt 2 blocks of [64 x 128 B]
constexpr int S_U = 65536;                //            U f32 [64][64]
constexpr int STAGE = 81920;
constexpr int S_D = 2 * STAGE;            // D bf16 [64 rows x 128 B]
constexpr int S_SB = S_D + 8192;          // S bf16 [128 rows x 128 B]
constexpr int S_BAR = S_SB + 16384;
constexpr int NSBAR = 10;
constexpr int S_SMEM = S_BAR + NSBAR * 8 + 16 + 1024;

enum ScanBar { FULL = 0, EMPTY = 2, D0_FULL = 4, DELTA_FULL = 5, S_SCALED = 6, STEP_DONE = 7,
               SBF_READY = 8 };

struct ScanParams {
  float* state;     // [nv][DK][DV]
  float* out;       // [rows][nv*DV]
  const float* gl;  // [nv][nchunks]
  int64_t rows;
  int nv, nchunks;
  int* status;
};

__global__ void __launch_bounds__(192, 1)
    gdn_scan_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmQg,
                    const __grid_constant__ CUtensorMap tmKt, const __grid_constant__ CUtensorMap tmM,
                    const __grid_constant__ CUtensorMap tmU, const ScanParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + NSBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int h = blockIdx.x, vb = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nc = p.nchunks;

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[FULL + s], 1);
      mbar_init(&bar[EMPTY + s], 1);
    }
    mbar_init(&bar[D0_FULL], 1);
    mbar_init(&bar[DELTA_FULL], 64);
    mbar_init(&bar[S_SCALED], 128);
    mbar_init(&bar[STEP_DONE], 1);
    mbar_init(&bar[SBF_READY], 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // rows 0-63 of both [0; M] buffers stay zero
  for (int i = tid; i < 8192 / 16; i += 192) {
    reinterpret_cast<uint4*>(smem + S_A2)[i] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(smem + STAGE + S_A2)[i] = make_uint4(0, 0, 0, 0);
  }
  if (warp == 5) tmem_alloc(tslot, 128);
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;  // D0 cols [0,64), state cols [64,128)

  auto wait = [&](int b, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait(&bar[b], parity)) return true;
    record_status(p.status, kStatusTimeout);
    *abort_flag = 1;
    return false;
  };

  if (warp == 4) {  // -------------------------------------------------- TMA
    if (lane == 0) {
      for (int c = 0; c < nc; ++c) {
        const int s = c & 1;
        if (c >= 2 && !wait(EMPTY + s, ((c >> 1) - 1) & 1)) break;
        uint8_t* st = smem + s * STAGE;
        const int row = (h * nc + c) * C;
        mbar_arrive_expect_tx(&bar[FULL + s], 16384 * 2 + 8192 + 16384 + 16384);
        for (int b = 0; b < 2; ++b) {
          tma_load_2d(st + S_A1 + b * 16384, &tmW, &bar[FULL + s], b * 64, row);
          tma_load_2d(st + S_A1 + b * 16384 + 8192, &tmQg, &bar[FULL + s], b * 64, row);
          tma_load_2d(st + S_KT + b * 8192, &tmKt, &bar[FULL + s], b * 64, row);
        }
        tma_load_2d(st + S_A2 + 8192, &tmM, &bar[FULL + s], 0, row);
        tma_load_2d(st + S_U, &tmU, &bar[FULL + s], vb * BV, row);
      }
    }
  } else if (warp == 5) {  // -------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t id1 = idesc_bf16(128, BV, false, true);
      constexpr uint32_t id3 = idesc_bf16(128, BV, true, true);
      const uint32_t sb = smem_u32(smem + S_SB), dl = smem_u32(smem + S_D);
      for (int c = 0; c < nc; ++c) {
        const int s = c & 1;
        const uint32_t st = smem_u32(smem + s * STAGE);
        if (!wait(FULL + s, (c >> 1) & 1) || !wait(SBF_READY, c & 1)) break;
        fence_after_sync();
        // D0 = [W; Qg] S0  (M128 N64 K128)
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)
          mma_bf16_ss(tmem, sw128_desc(st + S_A1 + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      sw128_desc(sb + kk * 2048, 8192, 1024), id1, kk > 0);
        mma_commit(&bar[D0_FULL]);
        if (!wait(DELTA_FULL, c & 1) || !wait(S_SCALED, c & 1)) break;
        fence_after_sync();
        // D0 += [0; M] D  (rows 64-127 become O);  S += Kt^T D
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {
          mma_bf16_ss(tmem, sw128_desc(st + S_A2 + kk * 32, 16, 1024),
                      sw128_desc(dl + kk * 2048, 8192, 1024), id1, true);
          mma_bf16_ss(tmem + 64, sw128_desc(st + S_KT + kk * 2048, 8192, 1024),
                      sw128_desc(dl + kk * 2048, 8192, 1024), id3, true);
        }
        mma_commit(&bar[STEP_DONE]);
        mma_commit(&bar[EMPTY + s]);
      }
    }
    __syncwarp();
  } else {  // ---------------------------------------------- warps 0-3 (rows)
    const int row = tid;  // TMEM lane: rows 0-63 = t (W S0 / O), state rows = dk
    const uint32_t tq = tmem + (uint32_t(warp * 32) << 16);
    float* sp = p.state + (int64_t(h) * DK + row) * DV + vb * BV;
    // initial state: TMEM f32 and the bf16 operand copy
    {
      uint32_t a[32], b[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 x = reinterpret_cast<const float4*>(sp)[i];
        const float4 y = reinterpret_cast<const float4*>(sp + 32)[i];
        a[4 * i] = __float_as_uint(x.x); a[4 * i + 1] = __float_as_uint(x.y);
        a[4 * i + 2] = __float_as_uint(x.z); a[4 * i + 3] = __float_as_uint(x.w);
        b[4 * i] = __float_as_uint(y.x); b[4 * i + 1] = __float_as_uint(y.y);
        b[4 * i + 2] = __float_as_uint(y.z); b[4 * i + 3] = __float_as_uint(y.w);
      }
      tmem_st32(tq + 64, a);
      tmem_st32(tq + 96, b);
      tmem_wait_st();
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const uint32_t* v = ch < 4 ? a : b;
        const int o = (ch & 3) * 8;
        *reinterpret_cast<uint4*>(smem + S_SB + sw_off(row, ch * 8, 16384)) =
            make_uint4(pack_bf16x2(__uint_as_float(v[o]), __uint_as_float(v[o + 1])),
                       pack_bf16x2(__uint_as_float(v[o + 2]), __uint_as_float(v[o + 3])),
                       pack_bf16x2(__uint_as_float(v[o + 4]), __uint_as_float(v[o + 5])),
                       pack_bf16x2(__uint_as_float(v[o + 6]), __uint_as_float(v[o + 7])));
      }
      fence_proxy_async_smem();
      fence_before_sync();
      mbar_arrive(&bar[SBF_READY]);
    }
    bool ok = true;
    for (int c = 0; c < nc && ok; ++c) {
      const int s = c & 1;
      ok = __all_sync(0xFFFFFFFFu, wait(D0_FULL, c & 1));
      fence_after_sync();
      if (warp < 2) {  // D = U - W S0 for row t
        uint32_t a[32], b[32];
        tmem_ld32(tq, a);
        tmem_ld32(tq + 32, b);
        tmem_wait_ld();
        const float* u = reinterpret_cast<const float*>(smem + s * STAGE + S_U) + row * BV;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint32_t* v = ch < 4 ? a : b;
          const int o = (ch & 3) * 8;
          const float4 u0 = reinterpret_cast<const float4*>(u + ch * 8)[0];
          const float4 u1 = reinterpret_cast<const float4*>(u + ch * 8)[1];
          *reinterpret_cast<uint4*>(smem + S_D + sw_off(row, ch * 8, 8192)) =
              make_uint4(pack_bf16x2(u0.x - __uint_as_float(v[o]), u0.y - __uint_as_float(v[o + 1])),
                         pack_bf16x2(u0.z - __uint_as_float(v[o + 2]), u0.w - __uint_as_float(v[o + 3])),
                         pack_bf16x2(u1.x - __uint_as_float(v[o + 4]), u1.y - __uint_as_float(v[o + 5])),
                         pack_bf16x2(u1.z - __uint_as_float(v[o + 6]), u1.w - __uint_as_float(v[o + 7])));
        }
        fence_proxy_async_smem();
        mbar_arrive(&bar[DELTA_FULL]);
      }
      {  // S <- gamma_{C-1} S
        const float g = p.gl[int64_t(h) * nc + c];
        uint32_t a[32], b[32];
        tmem_ld32(tq + 64, a);
        tmem_ld32(tq + 96, b);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          a[i] = __float_as_uint(__uint_as_float(a[i]) * g);
          b[i] = __float_as_uint(__uint_as_float(b[i]) * g);
        }
        tmem_st32(tq + 64, a);
        tmem_st32(tq + 96, b);
        tmem_wait_st();
        fence_before_sync();
        mbar_arrive(&bar[S_SCALED]);
      }
      ok = __all_sync(0xFFFFFFFFu, wait(STEP_DONE, c & 1) && ok);
      fence_after_sync();
      if (warp >= 2) {  // O rows
        const int64_t t = int64_t(c) * C + (row - 64);
        uint32_t a[32], b[32];
        tmem_ld32(tq, a);
        tmem_ld32(tq + 32, b);
        tmem_wait_ld();
        if (t < p.rows) {
          float* o = p.out + t * int64_t(p.nv) * DV + int64_t(h) * DV + vb * BV;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            reinterpret_cast<float4*>(o)[i] =
                make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                            __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3]));
            reinterpret_cast<float4*>(o + 32)[i] =
                make_float4(__uint_as_float(b[4 * i]), __uint_as_float(b[4 * i + 1]),
                            __uint_as_float(b[4 * i + 2]), __uint_as_float(b[4 * i + 3]));
          }
        }
      }
      {  // the next chunk's bf16 operand (or, after the last chunk, the state)
        uint32_t a[32], b[32];
        tmem_ld32(tq + 64, a);
        tmem_ld32(tq + 96, b);
        tmem_wait_ld();
        if (c + 1 < nc) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint32_t* v = ch < 4 ? a : b;
            const int o = (ch & 3) * 8;
            *reinterpret_cast<uint4*>(smem + S_SB + sw_off(row, ch * 8, 16384)) =
                make_uint4(pack_bf16x2(__uint_as_float(v[o]), __uint_as_float(v[o + 1])),
                           pack_bf16x2(__uint_as_float(v[o + 2]), __uint_as_float(v[o + 3])),
                           pack_bf16x2(__uint_as_float(v[o + 4]), __uint_as_float(v[o + 5])),
                           pack_bf16x2(__uint_as_float(v[o + 6]), __uint_as_float(v[o + 7])));
          }
          fence_proxy_async_smem();
          fence_before_sync();
          mbar_arrive(&bar[SBF_READY]);
        } else if (ok) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            reinterpret_cast<float4*>(sp)[i] =
                make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                            __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3]));
            reinterpret_cast<float4*>(sp + 32)[i] =
                make_float4(__uint_as_float(b[4 * i]), __uint_as_float(b[4 * i + 1]),
                            __uint_as_float(b[4 * i + 2]), __uint_as_float(b[4 * i + 3]));
          }
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    fence_after_sync();
    tmem_dealloc(tmem, 128);
  }
}

// 2-D row-major tensor [rows][cols] of `elem` bytes, boxes [box_rows][box_cols].
bool encode2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem, uint64_t rows,
              uint64_t cols, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle sw) {
  return encode_2d(m, dt, elem, base, rows, cols, cols, box_rows, box_cols, sw);
}

}  // namespace

bool gdn_prefill_serves(const hb_gdn_shape& s) {
  return s.hkd == DK && s.hvd == DV && s.nk > 0 && s.nv == 2 * s.nk;
}

GdnPrefillPlan gdn_prefill_plan(const hb_gdn_shape& s, int64_t rows) {
  GdnPrefillPlan pl;
  pl.nchunks = (rows + C - 1) / C;
  const size_t big = size_t(s.nv) * pl.nchunks * C * DK * 2;  // bf16 [nv][nc][64][128]
  pl.off_W = kWsHeader;
  pl.off_Qg = pl.off_W + align256(big);
  pl.off_Kt = pl.off_Qg + align256(big);
  pl.off_M = pl.off_Kt + align256(big);
  pl.off_U = pl.off_M + align256(size_t(s.nv) * pl.nchunks * C * C * 2);
  pl.off_gl = pl.off_U + align256(size_t(s.nv) * pl.nchunks * C * DV * 4);
  pl.bytes = pl.off_gl + align256(size_t(s.nv) * pl.nchunks * 4);
  return pl;
}

cudaError_t launch_gdn_prefill(const GdnLaunch& L, const GdnPrefillPlan& pl, void* ws,
                               cudaStream_t st) {
  char* base = static_cast<char*>(ws);
  static DeviceFlags configured;
  cudaError_t e = configured.once([] {
    cudaError_t r = cudaFuncSetAttribute(gdn_prep_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(gdn_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                S_SMEM);
  });
  if (e != cudaSuccess) return e;

  PrepParams pp;
  pp.qkv = L.call.qkv;
  pp.beta = L.call.beta;
  pp.decay = L.call.decay;
  pp.rows = L.call.rows;
  pp.nk = int(L.shape.nk);
  pp.nv = int(L.shape.nv);
  pp.nchunks = int(pl.nchunks);
  pp.l2 = L.call.l2;
  pp.eps = L.call.eps;
  pp.scale = L.scale;
  pp.W = reinterpret_cast<uint16_t*>(base + pl.off_W);
  pp.Qg = reinterpret_cast<uint16_t*>(base + pl.off_Qg);
  pp.Kt = reinterpret_cast<uint16_t*>(base + pl.off_Kt);
  pp.M = reinterpret_cast<uint16_t*>(base + pl.off_M);
  pp.U = reinterpret_cast<float*>(base + pl.off_U);
  pp.gl = reinterpret_cast<float*>(base + pl.off_gl);
  pp.status = reinterpret_cast<int*>(base);
  gdn_prep_kernel<<<dim3(unsigned(pl.nchunks), unsigned(L.shape.nk)), 128, P_SMEM, st>>>(pp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  const uint64_t rows_all = uint64_t(L.shape.nv) * pl.nchunks * C;
  CUtensorMap tW, tQ, tK, tM, tU;
  if (!encode2d(&tW, pp.W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_all, DK, 64, 64,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&tQ, pp.Qg, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_all, DK, 64, 64,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&tK, pp.Kt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_all, DK, 64, 64,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&tM, pp.M, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_all, C, 64, 64,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&tU, pp.U, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, rows_all, DV, 64, BV,
                CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  ScanParams sp;
  sp.state = L.call.state;
  sp.out = L.call.output;
  sp.gl = pp.gl;
  sp.rows = L.call.rows;
  sp.nv = int(L.shape.nv);
  sp.nchunks = int(pl.nchunks);
  sp.status = pp.status;
  gdn_scan_kernel<<<dim3(unsigned(L.shape.nv), DV / BV), 192, S_SMEM, st>>>(tW, tQ, tK, tM, tU,
                                                                             sp);
  return cudaGetLastError();
}

}  // namespace hb
