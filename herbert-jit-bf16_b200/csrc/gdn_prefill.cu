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
//    [T0'' 0; 0 T1''] times [V0; V1] gives U for both.  T comes from a blocked
//    inverse on the CUDA cores (16 x 16 diagonal blocks by forward
//    substitution, then the off-diagonal blocks block row by block row).  It
//    writes W, U, M, Qg = diag(gamma scale) Q, Kt = diag(r_{C-1,.}) K as the
//    scan's shared-memory tile images, and gamma_{C-1}.
//  * gdn_scan, one CTA per (value head, half of dv), sequential over chunks:
//    [W; Qg] S0 in one MMA (rows 0-63 W S0, rows 64-127 Q S0), D on the CUDA
//    cores, then [0; M] D accumulated onto the Q S0 rows (= O) and Kt^T D
//    accumulated onto the state, which lives in TMEM in f32 (scaled by
//    gamma_{C-1} first); its bf16 copy in shared memory is the next chunk's
//    operand.  Chunk tiles stream in by bulk copies two chunks ahead.
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

// Every per-(value head, chunk) output is written as the exact shared-memory
// image the scan's MMAs read (bf16 K-major tiles and the f32 U tile in the
// 128-byte swizzle, 1024-byte aligned), so both kernels move whole tiles
// with one-dimensional bulk copies.  Tile images in the workspace:
//   W, Qg, Kt  [2 column blocks][64 rows][128 B]       16 KB
//   M          [64 rows][128 B]                         8 KB
//   U          [4 column boxes of 32][64 rows][128 B]  32 KB (f32)
constexpr int TILE_WQK = 16384, TILE_M = 8192, TILE_U = 32768;

constexpr int P_SA = 0;          // [K; Q] bf16, 2 blocks of [128 rows x 128 B]
constexpr int P_SV = 32768;      // [V0; V1] bf16, 2 blocks of [128 rows x 128 B]
constexpr int P_S2 = 65536;      // [T0 bg0; T1 bg1] bf16, 1 block [128 x 128 B]
constexpr int P_S3 = 81920;      // blockdiag(T0 b0, T1 b1) bf16, 2 blocks
constexpr int P_AF = 114688;     // A f32 [2][64][65] (row stride 65: no bank conflicts)
constexpr int P_TF = 148480;     // T f32 [2][64][65]
constexpr int P_XS = 182272;     // X blocks f32 [2][3][16][16] of the blocked inverse
constexpr int P_VEC = 188416;    // beta[2][64], G[2][64]
constexpr int P_BAR = P_VEC + 1024;
constexpr int P_SMEM = P_BAR + 64 + 1024;
// staging of the output images (regions free at that point of the kernel)
constexpr int P_STG_M = P_TF;    // M0, M1 (16 KB, before T is computed)
// after the last MMA:
constexpr int P_STG_QK = P_S2;   // Qg0, Kt0, Qg1, Kt1 (64 KB over S2, S3, AF), read from SA
constexpr int P_STG_W = P_TF;    // W0, W1 (32 KB)
constexpr int P_STG_U = P_SA;    // U0, U1 (64 KB over SA, SV), once SA is read
constexpr int LDA = 65;          // row stride of A, T (floats)

struct PrepParams {
  const float* qkv;
  const float* beta;
  const float* decay;
  int64_t rows;
  int nk, nv, nchunks, l2;
  float eps, scale;
  uint8_t* W;   // [nv][nchunks] tile images
  uint8_t* Qg;
  uint8_t* Kt;
  uint8_t* M;
  uint8_t* U;
  float* gl;    // [nv][nchunks]
  int* status;
};

// byte offset of element (row, col) of a K-major bf16 tile whose column
// blocks of 64 are `block_bytes` apart, 128B-swizzled
HB_DEV uint32_t sw_off(int row, int col, int block_bytes) {
  return uint32_t((col >> 6) * block_bytes + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                  (col & 7) * 2);
}
// byte offset of 16-byte chunk `ch` (0..7) of row `row` in a 128B-swizzled block
HB_DEV uint32_t sw_chunk(int row, int ch) { return uint32_t(row * 128 + ((ch ^ (row & 7)) << 4)); }

__global__ void __launch_bounds__(256, 1) gdn_prep_kernel(const PrepParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + P_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 2);
  float* beta_s = reinterpret_cast<float*>(smem + P_VEC);  // [2][64]
  float* G_s = beta_s + 128;                               // [2][64]
  float* Af = reinterpret_cast<float*>(smem + P_AF);
  float* Tf = reinterpret_cast<float*>(smem + P_TF);
  float* Xs = reinterpret_cast<float*>(smem + P_XS);

  const int c = blockIdx.x, kh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t key = int64_t(p.nk) * DK, conv = 2 * key + int64_t(p.nv) * DV;
  const int64_t t0 = int64_t(c) * C;
  const int h0 = kh * 2;
  const int64_t tile0 = int64_t(h0) * p.nchunks + c, tile1 = tile0 + p.nchunks;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 256);

  // gates of both value heads, loaded first so that their latency hides
  // under the row loads
  float beta_v = 0.f, decay_v = 1.f;  // padded rows: decay 1
  if (tid < 128) {
    const int64_t t = t0 + (tid & 63);
    if (t < p.rows) {
      beta_v = p.beta[t * p.nv + h0 + (tid >> 6)];
      decay_v = p.decay[t * p.nv + h0 + (tid >> 6)];
    }
  }
  // ---- rows, a warp per row, lane = 4 columns: warp w loads 32 rows of
  // tensor w/2 (K, Q, V0, V1), K and Q L2-normalised, bf16 into SA / SV
  {
    const int ten = warp >> 1;
    const int64_t col_base = ten == 0 ? key + int64_t(kh) * DK
                           : ten == 1 ? int64_t(kh) * DK
                                      : 2 * key + int64_t(h0 + ten - 2) * DV;
    uint8_t* dst = smem + (ten < 2 ? P_SA : P_SV);
    const int row_off = (ten & 1) * 64;
    {
      float4 x[32];  // every row of the warp in flight at once
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = (warp & 1) * 32 + i;
        const int64_t t = t0 + r;
        x[i] = t < p.rows ? reinterpret_cast<const float4*>(p.qkv + t * conv + col_base)[lane]
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = (warp & 1) * 32 + i;
        float inv = 1.f;
        if (ten < 2 && p.l2) {
          float ss = x[i].x * x[i].x + x[i].y * x[i].y + x[i].z * x[i].z + x[i].w * x[i].w;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
          inv = 1.f / sqrtf(ss + p.eps);
        }
        const uint2 w = make_uint2(pack_bf16x2(x[i].x * inv, x[i].y * inv),
                                   pack_bf16x2(x[i].z * inv, x[i].w * inv));
        *reinterpret_cast<uint2*>(dst + sw_off(row_off + r, lane * 4, 16384)) = w;
      }
    }
  }
  if (tid < 128) {
    beta_s[tid] = beta_v;  // [head][row]: tid = hh * 64 + r
    G_s[tid] = logf(decay_v);
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
    const uint64_t sad = sw128_desc(sa, 16, 1024);
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      const uint64_t d = desc_add(sad, (kk >> 2) * 16384 + (kk & 3) * 32);
      mma_bf16_ss(tmem, d, d, id, kk > 0);
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

  if (tid < 2) p.gl[tid == 0 ? tile0 : tile1] = __expf(G_s[tid * 64 + 63]);
  if (!mbar_wait(&bar[0], 0)) record_status(p.status, kStatusTimeout);
  __syncthreads();
  fence_after_sync();

  // ---- K K^T (rows 0-63) -> A, Q K^T (rows 64-127) -> M images; warp w
  // reads TMEM lane quadrant w%4, columns 32 (w/4) .. + 32
  {
    const int q = warp & 3, cb = (warp >> 2) * 32;
    uint32_t ra[32];
    tmem_ld32(tmem + (uint32_t(q * 32) << 16) + cb, ra);
    tmem_wait_ld();
    const int t = (q & 1) * 32 + lane;
    if (q < 2) {  // A_h[t][j] = beta_t r_tj (k_t . k_j), j < t
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float bt = beta_s[hh * 64 + t], Gt = G_s[hh * 64 + t];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j = cb + i;
          Af[(hh * 64 + t) * LDA + j] =
              j < t ? bt * __expf(Gt - G_s[hh * 64 + j]) * __uint_as_float(ra[i]) : 0.f;
        }
      }
    } else {  // M_h[t][j] = scale r_tj (q_t . k_j), j <= t
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float Gt = G_s[hh * 64 + t];
        uint8_t* img = smem + P_STG_M + hh * TILE_M;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int i0 = c8 * 8 + 2 * i, j0 = cb + i0, j1 = j0 + 1;
            const float m0 = j0 <= t ? p.scale * __expf(Gt - G_s[hh * 64 + j0]) * __uint_as_float(ra[i0]) : 0.f;
            const float m1 = j1 <= t ? p.scale * __expf(Gt - G_s[hh * 64 + j1]) * __uint_as_float(ra[i0 + 1]) : 0.f;
            w[i] = pack_bf16x2(m0, m1);
          }
          *reinterpret_cast<uint4*>(img + sw_chunk(t, (cb >> 3) + c8)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  if (tid == 0) {
    bulk_s2g(p.M + tile0 * TILE_M, smem + P_STG_M, TILE_M);
    bulk_s2g(p.M + tile1 * TILE_M, smem + P_STG_M + TILE_M, TILE_M);
    tma_store_commit();
  }

  // ---- T = (I + A)^-1 by 16 x 16 blocks (threads 128 per head):
  //  diagonal blocks by forward substitution, then for block rows i = 1..3
  //  X_ij = sum_{k=j}^{i-1} A_ik T_kj and T_ij = -T_ii X_ij
  const int hh = tid >> 7, lt = tid & 127;
  const float* A = Af + hh * 64 * LDA;
  float* T = Tf + hh * 64 * LDA;
  if (tid == 0) tma_store_wait_read();  // the M staging lies under T
  __syncthreads();
  if (lt < 64) {  // column jj of diagonal block ib
    const int ib = lt >> 4, jj = lt & 15, o = ib * 16;
    float x[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float acc = 0.f;
#pragma unroll
      for (int s = 0; s < t; ++s) acc = fmaf(A[(o + t) * LDA + o + s], x[s], acc);
      x[t] = t == jj ? 1.f : (t < jj ? 0.f : -acc);
    }
#pragma unroll
    for (int t = 0; t < 16; ++t) T[(o + t) * LDA + o + jj] = x[t];
  }
  __syncthreads();
#pragma unroll
  for (int ib = 1; ib < 4; ++ib) {
    // X_ij for j < ib: ib * 256 elements per head, ib * 2 per thread
    float* X = Xs + hh * 768;
    for (int e = lt; e < ib * 256; e += 128) {
      const int jb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      float acc = 0.f;
#pragma unroll
      for (int kb = 0; kb < 3; ++kb) {
        if (kb < jb || kb >= ib) continue;
#pragma unroll
        for (int s = 0; s < 16; ++s)
          acc = fmaf(A[(ib * 16 + r) * LDA + kb * 16 + s], T[(kb * 16 + s) * LDA + jb * 16 + cc], acc);
      }
      X[e] = acc;
    }
    __syncthreads();
    for (int e = lt; e < ib * 256; e += 128) {
      const int jb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      float acc = 0.f;
#pragma unroll
      for (int s = 0; s < 16; ++s)
        acc = fmaf(T[(ib * 16 + r) * LDA + ib * 16 + s], X[(jb * 16 + s) * 16 + cc], acc);
      T[(ib * 16 + r) * LDA + jb * 16 + cc] = -acc;
    }
    __syncthreads();
  }

  // ---- S2 row (hh*64 + t) col j: T[t][j] beta_j gamma_j; S3 row (hh*64 + t)
  // col (hh*64 + j): T[t][j] beta_j, other half of the row zero; j > t zero
  {
    const int t = lt >> 1, half = lt & 1;
    const int row = hh * 64 + t;
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) {
      uint32_t w2[4], w3[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float a2[2], a3[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = half * 32 + c8 * 8 + 2 * i + e;
          const float tv = j <= t ? T[t * LDA + j] : 0.f;
          const float bj = beta_s[hh * 64 + j];
          a3[e] = tv * bj;
          a2[e] = a3[e] * __expf(G_s[hh * 64 + j]);
        }
        w2[i] = pack_bf16x2(a2[0], a2[1]);
        w3[i] = pack_bf16x2(a3[0], a3[1]);
      }
      const int ch = half * 4 + c8;
      *reinterpret_cast<uint4*>(smem + P_S2 + sw_chunk(row, ch)) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
      *reinterpret_cast<uint4*>(smem + P_S3 + hh * 16384 + sw_chunk(row, ch)) =
          make_uint4(w3[0], w3[1], w3[2], w3[3]);
      *reinterpret_cast<uint4*>(smem + P_S3 + (hh ^ 1) * 16384 + sw_chunk(row, ch)) =
          make_uint4(0, 0, 0, 0);
    }
  }
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();

  // ---- MMA 2: W = [T0 bg0; T1 bg1] K -> cols [0,128); MMA 3: U -> cols [128,256)
  if (tid == 0) {
    constexpr uint32_t id = idesc_bf16(128, 128, false, true);
    const uint64_t s2d = sw128_desc(smem_u32(smem + P_S2), 16, 1024),
                   s3d = sw128_desc(smem_u32(smem + P_S3), 16, 1024),
                   svd = sw128_desc(smem_u32(smem + P_SV), 16384, 1024),
                   sak = sw128_desc(sa, 16384, 1024);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      mma_bf16_ss(tmem, desc_add(s2d, kk * 32), desc_add(sak, kk * 2048), id, kk > 0);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      mma_bf16_ss(tmem + 128, desc_add(s3d, (kk >> 2) * 16384 + (kk & 3) * 32),
                  desc_add(svd, kk * 2048), id, kk > 0);
    mma_commit(&bar[1]);
  }
  __syncwarp();
  if (!mbar_wait(&bar[1], 0)) record_status(p.status, kStatusTimeout);
  fence_after_sync();

  // ---- Qg = diag(gamma scale) Q, Kt = diag(r_{63,.}) K as tile images: a
  // row scaling keeps each 16-byte chunk where the swizzle put it.  Unit =
  // (head, tensor, row, column block), 128 bytes; 512 units, 2 per thread.
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int u = tid + k * 256;
    const int blk = u & 1, r = (u >> 1) & 63, ten = (u >> 7) & 1, hq = u >> 8;
    const float G = G_s[hq * 64 + r];
    const float f = ten == 0 ? __expf(G) * p.scale : __expf(G_s[hq * 64 + 63] - G);
    const uint8_t* src = smem + P_SA + blk * 16384 + (ten == 0 ? 64 + r : r) * 128;
    uint8_t* dst = smem + P_STG_QK + (hq * 2 + ten) * TILE_WQK + blk * 8192 + r * 128;
#pragma unroll
    for (int k8 = 0; k8 < 8; ++k8) {
      const int ch = (k8 + r) & 7;  // rows of a warp start on different banks
      const uint4 v = reinterpret_cast<const uint4*>(src)[ch];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = pack_bf16x2(bf16lo(w[i]) * f, bf16hi(w[i]) * f);
      reinterpret_cast<uint4*>(dst)[ch] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();  // SA is read: the U images may overwrite it

  // ---- W (bf16) and U (f32) images: warp w reads lane quadrant w%4 (row =
  // head*64 + t), columns 64 (w/4) .. + 64 of W and of U
  {
    const int q = warp & 3, cb = (warp >> 2) * 64;
    const int row = q * 32 + lane, wh = row >> 6, t = row & 63;
    const uint32_t tq = tmem + (uint32_t(q * 32) << 16);
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      uint32_t w[32], u[32];
      tmem_ld32(tq + cb + half * 32, w);
      tmem_ld32(tq + 128 + cb + half * 32, u);
      tmem_wait_ld();
      const int col0 = cb + half * 32;  // 32 columns: 4 bf16 chunks of W, 8 f32 chunks of U
      uint8_t* wimg = smem + P_STG_W + wh * TILE_WQK + (col0 >> 6) * 8192;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8)
        *reinterpret_cast<uint4*>(wimg + sw_chunk(t, ((col0 & 63) >> 3) + c8)) =
            make_uint4(pack_bf16x2(__uint_as_float(w[8 * c8]), __uint_as_float(w[8 * c8 + 1])),
                       pack_bf16x2(__uint_as_float(w[8 * c8 + 2]), __uint_as_float(w[8 * c8 + 3])),
                       pack_bf16x2(__uint_as_float(w[8 * c8 + 4]), __uint_as_float(w[8 * c8 + 5])),
                       pack_bf16x2(__uint_as_float(w[8 * c8 + 6]), __uint_as_float(w[8 * c8 + 7])));
      uint8_t* uimg = smem + P_STG_U + wh * TILE_U + (col0 >> 5) * 8192;
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4)
        *reinterpret_cast<float4*>(uimg + sw_chunk(t, c4)) =
            make_float4(__uint_as_float(u[4 * c4]), __uint_as_float(u[4 * c4 + 1]),
                        __uint_as_float(u[4 * c4 + 2]), __uint_as_float(u[4 * c4 + 3]));
    }
  }
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  if (tid == 0) {
    bulk_s2g(p.Qg + tile0 * TILE_WQK, smem + P_STG_QK + 0 * TILE_WQK, TILE_WQK);
    bulk_s2g(p.Kt + tile0 * TILE_WQK, smem + P_STG_QK + 1 * TILE_WQK, TILE_WQK);
    bulk_s2g(p.Qg + tile1 * TILE_WQK, smem + P_STG_QK + 2 * TILE_WQK, TILE_WQK);
    bulk_s2g(p.Kt + tile1 * TILE_WQK, smem + P_STG_QK + 3 * TILE_WQK, TILE_WQK);
    bulk_s2g(p.W + tile0 * TILE_WQK, smem + P_STG_W, TILE_WQK);
    bulk_s2g(p.W + tile1 * TILE_WQK, smem + P_STG_W + TILE_WQK, TILE_WQK);
    bulk_s2g(p.U + tile0 * TILE_U, smem + P_STG_U, TILE_U);
    bulk_s2g(p.U + tile1 * TILE_U, smem + P_STG_U + TILE_U, TILE_U);
    tma_store_commit();
    tma_store_wait_read();
  }
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
constexpr int S_U = 65536;                //            U f32, 2 blocks [64 rows x 128 B], 128B-swizzled
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
  const uint8_t* W;  // tile images of the prep kernel, [nv][nchunks]
  const uint8_t* Qg;
  const uint8_t* Kt;
  const uint8_t* M;
  const uint8_t* U;
  int64_t rows;
  int nv, nchunks;
  int* status;
};

__global__ void __launch_bounds__(192, 1) gdn_scan_kernel(const ScanParams p) {
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
        const int64_t tile = int64_t(h) * nc + c;
        uint64_t* fb = &bar[FULL + s];
        mbar_arrive_expect_tx(fb, 4 * 8192 + TILE_WQK + TILE_M + TILE_U / 2);
        for (int b = 0; b < 2; ++b) {  // [W; Qg] stacked per column block
          bulk_g2s(st + S_A1 + b * 16384, p.W + tile * TILE_WQK + b * 8192, 8192, fb);
          bulk_g2s(st + S_A1 + b * 16384 + 8192, p.Qg + tile * TILE_WQK + b * 8192, 8192, fb);
        }
        bulk_g2s(st + S_KT, p.Kt + tile * TILE_WQK, TILE_WQK, fb);
        bulk_g2s(st + S_A2 + 8192, p.M + tile * TILE_M, TILE_M, fb);
        bulk_g2s(st + S_U, p.U + tile * TILE_U + vb * (TILE_U / 2), TILE_U / 2, fb);
      }
    }
  } else if (warp == 5) {  // -------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t id1 = idesc_bf16(128, BV, false, true);
      constexpr uint32_t id3 = idesc_bf16(128, BV, true, true);
      const uint64_t sbd = sw128_desc(smem_u32(smem + S_SB), 8192, 1024),
                     dld = sw128_desc(smem_u32(smem + S_D), 8192, 1024);
      for (int c = 0; c < nc; ++c) {
        const int s = c & 1;
        const uint32_t st = smem_u32(smem + s * STAGE);
        const uint64_t a1d = sw128_desc(st + S_A1, 16, 1024), a2d = sw128_desc(st + S_A2, 16, 1024),
                       ktd = sw128_desc(st + S_KT, 8192, 1024);
        if (!wait(FULL + s, (c >> 1) & 1) || !wait(SBF_READY, c & 1)) break;
        fence_after_sync();
        // D0 = [W; Qg] S0  (M128 N64 K128)
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)
          mma_bf16_ss(tmem, desc_add(a1d, (kk >> 2) * 16384 + (kk & 3) * 32),
                      desc_add(sbd, kk * 2048), id1, kk > 0);
        mma_commit(&bar[D0_FULL]);
        if (!wait(DELTA_FULL, c & 1) || !wait(S_SCALED, c & 1)) break;
        fence_after_sync();
        // D0 += [0; M] D  (rows 64-127 become O);  S += Kt^T D
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {
          mma_bf16_ss(tmem, desc_add(a2d, kk * 32), desc_add(dld, kk * 2048), id1, true);
          mma_bf16_ss(tmem + 64, desc_add(ktd, kk * 2048), desc_add(dld, kk * 2048), id3, true);
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
    float g_next = p.gl[int64_t(h) * nc];  // gamma_{C-1} of the chunk, one chunk ahead
    for (int c = 0; c < nc && ok; ++c) {
      const int s = c & 1;
      const float g = g_next;
      if (c + 1 < nc) g_next = p.gl[int64_t(h) * nc + c + 1];
      ok = __all_sync(0xFFFFFFFFu, wait(D0_FULL, c & 1));
      fence_after_sync();
      if (warp < 2) {  // D = U - W S0 for row t
        uint32_t a[32], b[32];
        tmem_ld32(tq, a);
        tmem_ld32(tq + 32, b);
        tmem_wait_ld();
        // U row `row`: columns c at block c/32, 16-byte chunk (c%32)/4 ^ (row%8)
        const uint8_t* u = smem + s * STAGE + S_U + row * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint32_t* v = ch < 4 ? a : b;
          const int o = (ch & 3) * 8;
          const int blk = (ch >> 2) * 8192, j = (ch & 3) * 2;
          const float4 u0 = *reinterpret_cast<const float4*>(u + blk + ((j ^ (row & 7)) << 4));
          const float4 u1 = *reinterpret_cast<const float4*>(u + blk + (((j + 1) ^ (row & 7)) << 4));
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
  pp.W = reinterpret_cast<uint8_t*>(base + pl.off_W);
  pp.Qg = reinterpret_cast<uint8_t*>(base + pl.off_Qg);
  pp.Kt = reinterpret_cast<uint8_t*>(base + pl.off_Kt);
  pp.M = reinterpret_cast<uint8_t*>(base + pl.off_M);
  pp.U = reinterpret_cast<uint8_t*>(base + pl.off_U);
  pp.gl = reinterpret_cast<float*>(base + pl.off_gl);
  pp.status = reinterpret_cast<int*>(base);
  gdn_prep_kernel<<<dim3(unsigned(pl.nchunks), unsigned(L.shape.nk)), 256, P_SMEM, st>>>(pp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  ScanParams sp;
  sp.state = L.call.state;
  sp.out = L.call.output;
  sp.gl = pp.gl;
  sp.W = pp.W;
  sp.Qg = pp.Qg;
  sp.Kt = pp.Kt;
  sp.M = pp.M;
  sp.U = pp.U;
  sp.rows = L.call.rows;
  sp.nv = int(L.shape.nv);
  sp.nchunks = int(pl.nchunks);
  sp.status = pp.status;
  gdn_scan_kernel<<<dim3(unsigned(L.shape.nv), DV / BV), 192, S_SMEM, st>>>(sp);
  return cudaGetLastError();
}

}  // namespace hb
