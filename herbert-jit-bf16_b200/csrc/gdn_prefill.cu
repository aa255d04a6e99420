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
//   S_C  = gamma_{C-1} S0 + Kt^T D,        Kt = diag(r_{C-1,.}) K
//
// Substituting D folds every S0-independent product into per-chunk matrices:
//
//   S_C = Ac S0 + Kt^T U,   Ac = gamma_{C-1} I - Kt^T W      (dk x dk)
//   O   = Pc S0 + M U,      Pc = diag(gamma scale) Q - M W   (C x dk)
//
// so the sequential part of a chunk is one product with S0 (Ac S0 and Pc S0
// read the same operand) and one rounding of the new state to bf16; Kt^T U
// and M U do not depend on S0 and are issued ahead.  Two kernels:
//  * gdn_prep: persistent CTAs walk the (chunk, key head) tiles in chunk
//    order, both value heads of the key head at once, so that the products
//    are M = 128 tcgen05 MMAs: [K;Q] K^T gives K K^T and Q K^T; T comes from a
//    blocked inverse (16 x 16 diagonal blocks by forward substitution, the
//    off-diagonal blocks by warp-level block products); [T0'; T1'] K gives W,
//    blockdiag(T0'', T1'') [V0; V1] gives U, Kt^T W gives Ac and
//    blockdiag(M0, M1) [W0; W1] gives M W.  It writes Ac, Pc, Kt, M and U
//    (bf16) as the scan's shared-memory tile images.
//  * gdn_scan, one CTA per (value head, half of dv), sequential over chunks:
//    the state is the bf16 operand in shared memory (two buffers, alternate
//    chunks); per chunk Ac S0 (onto Kt^T U) into TMEM is the only product on
//    the chain: the new state is read back and rounded to bf16 for the next
//    chunk while Pc S0 (onto M U, an M = 64 accumulator) runs and four warps
//    store the chunk's output.  Chunk tiles stream in by bulk copies two
//    chunks ahead, prefetched into L2 six chunks ahead.
// MMA operands are bf16, accumulators f32; the result is not the bits of the
// sequential recurrence (as for the reference's own chunked kernel) and is
// held to a relative Frobenius tolerance.
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
// image the scan's MMAs read (bf16 tiles in the 128-byte swizzle, 1024-byte
// aligned), so both kernels move whole tiles with one-dimensional bulk
// copies.  Tile images in the workspace:
//   Ac  [2 column blocks][128 rows][128 B]   32 KB   (row i = key dim, col j)
//   Pc  [2 column blocks][64 rows][128 B]    16 KB   (row t, col = key dim)
//   Kt  [2 column blocks][64 rows][128 B]    16 KB   (row t, col = key dim)
//   M   [64 rows][128 B]                      8 KB   (row t, col j)
//   U   [2 column blocks][64 rows][128 B]    16 KB   (row t, col = value dim)
constexpr int TILE_AC = 32768, TILE_PC = 16384, TILE_KT = 16384, TILE_M = 8192, TILE_U = 16384;

// Shared memory of one prep CTA (bytes; tile regions 1024-aligned).  Later
// phases of a tile reuse regions whose contents are dead by then.
constexpr int P_SA = 0;          // [K; Q] bf16 [2 blocks][128 rows][128 B]
constexpr int P_SV = 32768;      // [V0; V1] bf16 [2 blocks][128][128 B]; then U images
constexpr int P_MB = 65536;      // blockdiag(M0, M1) [2 blocks][128][128 B]; then Ac images
constexpr int P_AF = 98304;      // A f32 [2][64][65]; then W0 over W1 [2 blocks][128][128 B]
constexpr int P_TF = 132096;     // T f32 [2][64][65]; then Kt images
constexpr int P_XS = 165376;     // per warp a [16][17] f32 block of the inverse's products
constexpr int P_S2 = 174080;     // [T0 bg0; T1 bg1] [128][128 B]; then Pc images
constexpr int P_S3 = 190464;     // blockdiag(T0 b0, T1 b1) [2 blocks][128][128 B]
constexpr int P_VEC = 223232;    // beta[2][64], G2[2][64] (log2 of the decay, prefix sums)
constexpr int P_BAR = P_VEC + 1024;
constexpr int P_SMEM = P_BAR + 64 + 1024;
constexpr int P_WS = P_AF;       // W rows (hh*64 + t), MN-major B of the last products
constexpr int LDA = 65;          // row stride of A, T (floats)
constexpr int LDX = 17;          // row stride of a warp's product block (floats)
constexpr int PREP_THREADS = 256;

struct PrepParams {
  const float* qkv;
  const float* beta;
  const float* decay;
  int64_t rows;
  int nk, nv, nchunks, l2;
  float eps, scale;
  uint8_t* Ac;  // [nv][nchunks] tile images
  uint8_t* Pc;
  uint8_t* Kt;
  uint8_t* M;
  uint8_t* U;
  int* status;
};

// byte offset of element (row, col) of a bf16 tile whose column blocks of 64
// are `block_bytes` apart, 128B-swizzled
HB_DEV uint32_t sw_off(int row, int col, int block_bytes) {
  return uint32_t((col >> 6) * block_bytes + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                  (col & 7) * 2);
}
// byte offset of 16-byte chunk `ch` (0..7) of row `row` in a 128B-swizzled block
HB_DEV uint32_t sw_chunk(int row, int ch) { return uint32_t(row * 128 + ((ch ^ (row & 7)) << 4)); }

// Waits until all but the newest `N` committed bulk-store groups have read
// their shared-memory source.
template <int N>
HB_DEV void store_wait_read_but() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// 8 f32 -> one 16-byte chunk of bf16
HB_DEV uint4 pack8(const float* v) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

// One 16 x 16 x 16 product of row-major f32 blocks by a warp, accumulated in
// registers: lane l owns rows 2 (l / 4) .. +1 and columns 4 (l % 4) .. +3, so
// each step loads 2 values of `a` and 4 of `b` for 8 FMAs.
HB_DEV void warp_block_mma(const float* a, int lda, const float* b, int ldb, float (&acc)[2][4]) {
  const int lane = threadIdx.x & 31, r0 = (lane >> 2) * 2, c0 = (lane & 3) * 4;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float a0 = a[r0 * lda + k], a1 = a[(r0 + 1) * lda + k];
    float bv[4];
#pragma unroll
    for (int x = 0; x < 4; ++x) bv[x] = b[k * ldb + c0 + x];
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      acc[0][x] = fmaf(a0, bv[x], acc[0][x]);
      acc[1][x] = fmaf(a1, bv[x], acc[1][x]);
    }
  }
}

HB_DEV void warp_block_store(float* dst, int ld, const float (&acc)[2][4], float sign) {
  const int lane = threadIdx.x & 31, r0 = (lane >> 2) * 2, c0 = (lane & 3) * 4;
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int x = 0; x < 4; ++x) dst[(r0 + r) * ld + c0 + x] = sign * acc[r][x];
}

// Off-diagonal 16 x 16 block (i, j), i > j, of T = (I + A)^-1 for one head,
// once its diagonal blocks and the blocks (k, j), j <= k < i, are final:
// X = sum_{k=j}^{i-1} A_ik T_kj, then T_ij = -T_ii X (one warp).
HB_DEV void inverse_block(const float* A, float* T, float* X, int i, int j) {
  float acc[2][4] = {};
  for (int k = j; k < i; ++k)
    warp_block_mma(A + (16 * i) * LDA + 16 * k, LDA, T + (16 * k) * LDA + 16 * j, LDA, acc);
  warp_block_store(X, LDX, acc, 1.f);
  __syncwarp();
  float out[2][4] = {};
  warp_block_mma(T + (16 * i) * LDA + 16 * i, LDA, X, LDX, out);
  warp_block_store(T + (16 * i) * LDA + 16 * j, LDA, out, -1.f);
  __syncwarp();
}

// A persistent CTA per SM walks the (chunk, key head) tiles in chunk order.
// All 32 row loads of a lane are issued before the first is used, the rows of
// the next tile are then prefetched into L2 by four tensor prefetches, and a
// tile's last image stores drain while the next tile's rows load and its
// first product runs.
__global__ void __launch_bounds__(PREP_THREADS, 1)
    gdn_prep_kernel(const __grid_constant__ CUtensorMap tm_qkv, const PrepParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + P_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 3);
  float* beta_s = reinterpret_cast<float*>(smem + P_VEC);  // [2][64]
  float* G_s = beta_s + 128;                               // [2][64], log2 units
  float* Af = reinterpret_cast<float*>(smem + P_AF);
  float* Tf = reinterpret_cast<float*>(smem + P_TF);
  float* Xs = reinterpret_cast<float*>(smem + P_XS);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t key = int64_t(p.nk) * DK, conv = 2 * key + int64_t(p.nv) * DV;
  const int ntiles = p.nchunks * p.nk;

  if (tid == 0) {
    for (int b = 0; b < 3; ++b) mbar_init(&bar[b], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 512);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;  // cols [0,64) K K^T | Q K^T, then W [0,128) U [128,256),
                                 // then M W [0,128), Kt^T W [256,512)
  const uint32_t sa = smem_u32(smem + P_SA);

  // brings a tile's rows (K, Q of the key head, V of both value heads) into
  // L2: four [64 rows][128 columns] boxes
  auto prefetch_rows = [&](int tile) {
    const int c = tile / p.nk, kh = tile % p.nk, y = c * C;
    tma_prefetch_l2_2d(&tm_qkv, int(key) + kh * DK, y);
    tma_prefetch_l2_2d(&tm_qkv, kh * DK, y);
    tma_prefetch_l2_2d(&tm_qkv, int(2 * key) + 2 * kh * DV, y);
    tma_prefetch_l2_2d(&tm_qkv, int(2 * key) + (2 * kh + 1) * DV, y);
  };

  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    const int c = tile / p.nk, kh = tile % p.nk;
    const int64_t t0 = int64_t(c) * C;
    const int h0 = kh * 2;
    const int64_t tile0 = int64_t(h0) * p.nchunks + c, tile1 = tile0 + p.nchunks;
    const uint32_t par = it & 1;

    // gates of both value heads first, so that their latency hides under the rows
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
      float4 x[32];
      // all 32 loads issued before any is used (rows past the block read the
      // last row and are zeroed below)
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int64_t t = t0 + (warp & 1) * 32 + i;
        const float4* src =
            reinterpret_cast<const float4*>(p.qkv + (t < p.rows ? t : p.rows - 1) * conv + col_base) + lane;
        asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(x[i].x), "=f"(x[i].y), "=f"(x[i].z), "=f"(x[i].w)
                     : "l"(src));
      }
      if (tid == 0 && tile + int(gridDim.x) < ntiles) prefetch_rows(tile + gridDim.x);
      // SA is no store source, and SV's U images were read long ago (their
      // group precedes Ac and Pc): the rows may be written before the
      // previous tile's last stores have drained
      if (tid == 0) store_wait_read_but<1>();
      __syncthreads();
      // sums of squares of all 32 rows first, then the butterflies of all rows
      // interleaved (independent shuffles pipeline; a chain per row does not)
      float inv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (t0 + (warp & 1) * 32 + i >= p.rows) x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        inv[i] = x[i].x * x[i].x + x[i].y * x[i].y + x[i].z * x[i].z + x[i].w * x[i].w;
      }
      if (ten < 2 && p.l2) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int i = 0; i < 32; ++i) inv[i] += __shfl_xor_sync(0xFFFFFFFFu, inv[i], o);
#pragma unroll
        for (int i = 0; i < 32; ++i) inv[i] = rsqrtf(inv[i] + p.eps);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) inv[i] = 1.f;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = (warp & 1) * 32 + i;
        const uint2 w = make_uint2(pack_bf16x2(x[i].x * inv[i], x[i].y * inv[i]),
                                   pack_bf16x2(x[i].z * inv[i], x[i].w * inv[i]));
        *reinterpret_cast<uint2*>(dst + sw_off(row_off + r, lane * 4, 16384)) = w;
      }
    }
    if (tid < 128) {
      beta_s[tid] = beta_v;  // [head][row]: tid = hh * 64 + r
      G_s[tid] = log2f(decay_v);
    }
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();

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
    // ---- prefix sums of log2 decay per head (warp hh, 2 values per lane)
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
    // the previous tile's Ac and Pc stores must have read M's, W's and S2's
    // regions before they are written again
    if (tid == 0) tma_store_wait_read();
    __syncthreads();
    if (!mbar_wait(&bar[0], par)) record_status(p.status, kStatusTimeout);
    __syncthreads();
    fence_after_sync();

    // ---- A (from K K^T, TMEM lanes 0-63) and blockdiag(M0, M1) (from Q K^T,
    // lanes 64-127): warp w reads the 64 columns of lane quadrant w % 4 and
    // gates them for value head w / 4; one exponential per element
    {
      const int q = warp & 3, hh = warp >> 2;
      const int t = (q & 1) * 32 + lane;
      const bool upper_half = (q & 1) != 0;  // rows 32-63 see columns 32-63
      uint32_t ra[64];
      tmem_ld32(tmem + (uint32_t(q * 32) << 16), *reinterpret_cast<uint32_t(*)[32]>(ra));
      tmem_ld32(tmem + (uint32_t(q * 32) << 16) + 32, *reinterpret_cast<uint32_t(*)[32]>(ra + 32));
      tmem_wait_ld();
      const float Gt = G_s[hh * 64 + t];
      const float* Gh = G_s + hh * 64;
      if (q < 2) {  // A_h[t][j] = beta_t 2^(G_t - G_j) (k_t . k_j), j < t
        const float bt = beta_s[hh * 64 + t];
        float* Arow = Af + (hh * 64 + t) * LDA;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          float v = 0.f;
          if (j < 32 || upper_half)
            v = j < t ? bt * fast_exp2(Gt - Gh[j]) * __uint_as_float(ra[j]) : 0.f;
          Arow[j] = v;
        }
      } else {  // M_h[t][j] = scale 2^(G_t - G_j) (q_t . k_j), j <= t, in block hh of row hh*64+t
        const int row = hh * 64 + t;
        uint8_t* mb = smem + P_MB;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float m[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int j = c8 * 8 + i;
            m[i] = 0.f;
            if (c8 < 4 || upper_half)
              m[i] = j <= t ? p.scale * fast_exp2(Gt - Gh[j]) * __uint_as_float(ra[j]) : 0.f;
          }
          *reinterpret_cast<uint4*>(mb + hh * 16384 + sw_chunk(row, c8)) = pack8(m);
          *reinterpret_cast<uint4*>(mb + (hh ^ 1) * 16384 + sw_chunk(row, c8)) = make_uint4(0, 0, 0, 0);
        }
      }
    }
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // M_hh is rows hh*64.. of block hh: one 8 KB image each
      bulk_s2g(p.M + tile0 * TILE_M, smem + P_MB, TILE_M);
      bulk_s2g(p.M + tile1 * TILE_M, smem + P_MB + 16384 + 8192, TILE_M);
      tma_store_commit();
    }

    // ---- T = (I + A)^-1 by 16 x 16 blocks: diagonal blocks by forward
    // substitution (a thread per column), then the off-diagonal blocks by
    // warp products, level by level (one block below the diagonal, two, three)
    {
      const int hh = tid >> 7, lt = tid & 127;
      const float* A = Af + hh * 64 * LDA;
      float* T = Tf + hh * 64 * LDA;
      if (lt < 64) {  // column jj of diagonal block ib
        const int ib = lt >> 4, jj = lt & 15, o = ib * 16;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float acc = 0.f;
#pragma unroll
          for (int s = 0; s < r; ++s) acc = fmaf(A[(o + r) * LDA + o + s], x[s], acc);
          x[r] = r == jj ? 1.f : (r < jj ? 0.f : -acc);
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) T[(o + r) * LDA + o + jj] = x[r];
      }
    }
    __syncthreads();
    {
      float* X = Xs + warp * 16 * LDX;
      if (warp < 6) {  // blocks (1,0) (2,1) (3,2) of each head
        const int hh = warp / 3, i = warp % 3 + 1;
        inverse_block(Af + hh * 64 * LDA, Tf + hh * 64 * LDA, X, i, i - 1);
      }
      __syncthreads();
      if (warp < 4) {  // (2,0) (3,1)
        const int hh = warp >> 1, i = (warp & 1) + 2;
        inverse_block(Af + hh * 64 * LDA, Tf + hh * 64 * LDA, X, i, i - 2);
      }
      __syncthreads();
      if (warp < 2) inverse_block(Af + warp * 64 * LDA, Tf + warp * 64 * LDA, X, 3, 0);
      __syncthreads();
    }

    // ---- S2 row (hh*64 + t) col j: T[t][j] beta_j gamma_j; S3 row (hh*64 + t)
    // col (hh*64 + j): T[t][j] beta_j, other half of the row zero; j > t zero
    {
      const int hh = tid >> 7, lt = tid & 127;
      const float* T = Tf + hh * 64 * LDA;
      const int t = lt >> 1, half = lt & 1;
      const int row = hh * 64 + t;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float a2[8], a3[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = half * 32 + c8 * 8 + e;
          const float tv = j <= t ? T[t * LDA + j] : 0.f;
          a3[e] = tv * beta_s[hh * 64 + j];
          a2[e] = a3[e] * fast_exp2(G_s[hh * 64 + j]);
        }
        const int ch = half * 4 + c8;
        *reinterpret_cast<uint4*>(smem + P_S2 + sw_chunk(row, ch)) = pack8(a2);
        *reinterpret_cast<uint4*>(smem + P_S3 + hh * 16384 + sw_chunk(row, ch)) = pack8(a3);
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
    if (!mbar_wait(&bar[1], par)) record_status(p.status, kStatusTimeout);
    fence_after_sync();

    // ---- W (bf16, rows hh*64 + t over A's region) and U images (bf16, over
    // V's region): warp w reads lane quadrant w%4 (row = head*64 + t),
    // columns 64 (w/4) .. + 64 of W and of U
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
        const int col0 = cb + half * 32;  // 4 chunks of 8 columns
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const int ch = ((col0 & 63) >> 3) + c8;
          *reinterpret_cast<uint4*>(smem + P_WS + (col0 >> 6) * 16384 + sw_chunk(row, ch)) =
              pack8(reinterpret_cast<const float*>(w + 8 * c8));
          *reinterpret_cast<uint4*>(smem + P_SV + wh * TILE_U + (col0 >> 6) * 8192 + sw_chunk(t, ch)) =
              pack8(reinterpret_cast<const float*>(u + 8 * c8));
        }
      }
    }
    // ---- Kt = diag(r_{63,.}) K images over T's region: a row scaling keeps
    // each 16-byte chunk where the swizzle put it.  Unit = (head, row,
    // column block), 128 bytes; 256 units, one per thread.
    {
      const int blk = tid & 1, r = (tid >> 1) & 63, hq = tid >> 7;
      const float f = fast_exp2(G_s[hq * 64 + 63] - G_s[hq * 64 + r]);
      const uint8_t* src = smem + P_SA + blk * 16384 + r * 128;
      uint8_t* dst = smem + P_TF + hq * TILE_KT + blk * 8192 + r * 128;
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
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();

    // ---- MMA 4: Kt_h^T W_h -> cols [256 + 128 h, ...); MMA 5: blockdiag(M) [W0; W1] -> [0,128)
    if (tid == 0) {
      constexpr uint32_t id4 = idesc_bf16(128, 128, true, true);
      constexpr uint32_t id5 = idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint64_t ktd = sw128_desc(smem_u32(smem + P_TF + hh * TILE_KT), 8192, 1024),
                       wsd = sw128_desc(smem_u32(smem + P_WS + hh * 8192), 16384, 1024);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          mma_bf16_ss(tmem + 256 + hh * 128, desc_add(ktd, kk * 2048), desc_add(wsd, kk * 2048),
                      id4, kk > 0);
      }
      const uint64_t mbd = sw128_desc(smem_u32(smem + P_MB), 16, 1024),
                     wsd = sw128_desc(smem_u32(smem + P_WS), 16384, 1024);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_bf16_ss(tmem, desc_add(mbd, (kk >> 2) * 16384 + (kk & 3) * 32),
                    desc_add(wsd, kk * 2048), id5, kk > 0);
      mma_commit(&bar[2]);
      // U and Kt images are final: their stores overlap the products
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int64_t tl = hh ? tile1 : tile0;
        bulk_s2g(p.U + tl * TILE_U, smem + P_SV + hh * TILE_U, TILE_U);
        bulk_s2g(p.Kt + tl * TILE_KT, smem + P_TF + hh * TILE_KT, TILE_KT);
      }
      tma_store_commit();
    }
    __syncwarp();
    if (!mbar_wait(&bar[2], par)) record_status(p.status, kStatusTimeout);
    // the M stores have read blockdiag(M), which Ac overwrites next
    if (tid == 0) store_wait_read_but<1>();
    __syncthreads();
    fence_after_sync();

    // ---- Ac_h = gamma_63 I - Kt_h^T W_h (lane i = key dim, column j) over
    // M's and W's regions; warp w: head w / 4, rows 32 (w % 4) ..
    {
      const int q = warp & 3, hh = warp >> 2;
      const int i = q * 32 + lane;
      const float g63 = fast_exp2(G_s[hh * 64 + 63]);
      const uint32_t tq = tmem + (uint32_t(q * 32) << 16) + 256 + hh * 128;
      uint8_t* img = smem + P_MB + hh * TILE_AC;
#pragma unroll 1
      for (int cb = 0; cb < 128; cb += 32) {
        uint32_t v[32];
        tmem_ld32(tq + cb, v);
        tmem_wait_ld();
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float a[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = cb + c8 * 8 + e;
            a[e] = (j == i ? g63 : 0.f) - __uint_as_float(v[c8 * 8 + e]);
          }
          *reinterpret_cast<uint4*>(img + (cb >> 6) * 16384 + sw_chunk(i, ((cb & 63) >> 3) + c8)) =
              pack8(a);
        }
      }
    }
    // ---- Pc_h = diag(gamma scale) Q_h - M_h W_h (lane hh*64 + t, column j)
    // over S2/S3's region; warp w: lane quadrant w % 4, columns 64 (w / 4) ..
    {
      const int q = warp & 3, cb0 = (warp >> 2) * 64;
      const int row = q * 32 + lane, hh = row >> 6, t = row & 63;
      const float f = fast_exp2(G_s[hh * 64 + t]) * p.scale;
      const uint32_t tq = tmem + (uint32_t(q * 32) << 16);
      const int qr = 64 + t;  // Q row t of [K; Q]
#pragma unroll 1
      for (int cb = cb0; cb < cb0 + 64; cb += 32) {
        uint32_t v[32];
        tmem_ld32(tq + cb, v);
        tmem_wait_ld();
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const int ch = ((cb & 63) >> 3) + c8;
          const uint4 qv =
              *reinterpret_cast<const uint4*>(smem + P_SA + (cb >> 6) * 16384 + sw_chunk(qr, ch));
          const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
          float a[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            a[2 * e] = bf16lo(qw[e]) * f - __uint_as_float(v[c8 * 8 + 2 * e]);
            a[2 * e + 1] = bf16hi(qw[e]) * f - __uint_as_float(v[c8 * 8 + 2 * e + 1]);
          }
          *reinterpret_cast<uint4*>(smem + P_S2 + hh * TILE_PC + (cb >> 6) * 8192 +
                                    sw_chunk(t, ch)) = pack8(a);
        }
      }
    }
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // drained while the next tile's rows load
      bulk_s2g(p.Ac + tile0 * TILE_AC, smem + P_MB, TILE_AC);
      bulk_s2g(p.Ac + tile1 * TILE_AC, smem + P_MB + TILE_AC, TILE_AC);
      bulk_s2g(p.Pc + tile0 * TILE_PC, smem + P_S2, TILE_PC);
      bulk_s2g(p.Pc + tile1 * TILE_PC, smem + P_S2 + TILE_PC, TILE_PC);
      tma_store_commit();
    }
  }
  if (tid == 0) tma_store_wait_read();
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ scan

constexpr int BV = 64;            // value columns per CTA
// one stage holds one chunk's operands (1024-aligned images)
constexpr int S_AC = 0;           // Ac [2 K-blocks][128 rows][128 B]              K-major A
constexpr int S_PC = 32768;       // Pc [2 K-blocks][64 rows][128 B]               K-major A
constexpr int S_MZ = 49152;       // M [64 rows][128 B]                             K-major A
constexpr int S_KT = 57344;       // Kt [2 blocks][64 rows][128 B]     MN-major A (Kt^T)
constexpr int S_UH = 73728;       // U columns vb*64.. [64 rows][128 B]             MN-major B
constexpr int STAGE = 81920;
constexpr int S_SB = 2 * STAGE;   // state bf16, 2 x [128 rows][128 B] (alternate chunks) MN-major B
constexpr int S_OS = S_SB + 2 * 16384;  // output staging [2 buffers][4 warps][2 x [16 rows][128 B]]
constexpr int S_BAR = S_OS + 2 * 16384;
constexpr int NSBAR = 10;
constexpr int S_SMEM = S_BAR + NSBAR * 8 + 16 + 1024;
constexpr int SCAN_THREADS = 320;
constexpr int kScanPrefetch = 6;  // chunks of L2 prefetch ahead of the bulk copies

// FULL/EMPTY: stage loaded / consumed; SB_READY: bf16 state written;
// S_DONE: a chunk's products done (new state in TMEM); O_DONE/O_FREE: an
// output buffer written / read (one pair per buffer, so the output warps may
// trail the state warps by a chunk without losing a phase).
enum ScanBar { FULL = 0, EMPTY = 2, SB_READY = 4, S_DONE = 5, O_FREE = 6, O_DONE = 8 };

struct ScanParams {
  float* state;     // [nv][DK][DV]
  const uint8_t* Ac;  // tile images of the prep kernel, [nv][nchunks]
  const uint8_t* Pc;
  const uint8_t* Kt;
  const uint8_t* M;
  const uint8_t* U;
  int64_t rows;
  int nv, nchunks;
  int* status;
};

// Warps 0-3: the state (TMEM lane = key dim row; bf16 operand for the next
// chunk, the f32 state after the last); warps 4-7: the chunk outputs (an M =
// 64 accumulator: rows 16q .. 16q+15 in lanes 32q .. 32q+15), staged in
// shared memory and written by tensor stores; warp 8: bulk
// copies; warp 9: MMAs.  TMEM columns: [0,64) and [64,128) the state of
// alternate chunks, [128,192) and [192,256) the outputs of alternate chunks.
__global__ void __launch_bounds__(SCAN_THREADS, 1)
    gdn_scan_kernel(const __grid_constant__ CUtensorMap tm_out, const ScanParams p) {
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
      mbar_init(&bar[O_FREE + s], 128);
      mbar_init(&bar[O_DONE + s], 1);
    }
    mbar_init(&bar[SB_READY], 128);
    mbar_init(&bar[S_DONE], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) tmem_alloc(tslot, 256);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;

  auto wait = [&](int b, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait(&bar[b], parity)) return true;
    record_status(p.status, kStatusTimeout);
    *abort_flag = 1;
    return false;
  };

  if (warp == 8) {  // -------------------------------------------------- TMA
    if (lane == 0) {
      // a chunk's tiles are brought into L2 kScanPrefetch chunks before their
      // bulk copies, which then hit L2
      auto prefetch = [&](int c) {
        const int64_t tile = int64_t(h) * nc + c;
        bulk_prefetch_l2(p.Ac + tile * TILE_AC, TILE_AC);
        bulk_prefetch_l2(p.Pc + tile * TILE_PC, TILE_PC);
        bulk_prefetch_l2(p.M + tile * TILE_M, TILE_M);
        bulk_prefetch_l2(p.Kt + tile * TILE_KT, TILE_KT);
        bulk_prefetch_l2(p.U + tile * TILE_U + vb * (TILE_U / 2), TILE_U / 2);
      };
      for (int c = 0; c < kScanPrefetch && c < nc; ++c) prefetch(c);
      for (int c = 0; c < nc; ++c) {
        const int s = c & 1;
        if (c + kScanPrefetch < nc) prefetch(c + kScanPrefetch);
        if (c >= 2 && !wait(EMPTY + s, ((c >> 1) - 1) & 1)) break;
        uint8_t* st = smem + s * STAGE;
        const int64_t tile = int64_t(h) * nc + c;
        uint64_t* fb = &bar[FULL + s];
        mbar_arrive_expect_tx(fb, TILE_AC + TILE_PC + TILE_M + TILE_KT + TILE_U / 2);
        bulk_g2s(st + S_AC, p.Ac + tile * TILE_AC, TILE_AC, fb);
        bulk_g2s(st + S_PC, p.Pc + tile * TILE_PC, TILE_PC, fb);
        bulk_g2s(st + S_MZ, p.M + tile * TILE_M, TILE_M, fb);
        bulk_g2s(st + S_KT, p.Kt + tile * TILE_KT, TILE_KT, fb);
        bulk_g2s(st + S_UH, p.U + tile * TILE_U + vb * (TILE_U / 2), TILE_U / 2, fb);
      }
    }
  } else if (warp == 9) {  // -------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16(128, BV, false, true);  // state: M = key dim
      constexpr uint32_t id_t = idesc_bf16(128, BV, true, true);   // Kt^T (MN-major A)
      constexpr uint32_t id_o = idesc_bf16(64, BV, false, true);   // outputs: M = 64 positions
      for (int c = 0; c < nc; ++c) {
        const int s = c & 1;
        const uint32_t st = smem_u32(smem + s * STAGE);
        const uint64_t acd = sw128_desc(st + S_AC, 16, 1024), pcd = sw128_desc(st + S_PC, 16, 1024),
                       mzd = sw128_desc(st + S_MZ, 16, 1024), ktd = sw128_desc(st + S_KT, 8192, 1024),
                       uhd = sw128_desc(st + S_UH, 8192, 1024),
                       sbd = sw128_desc(smem_u32(smem + S_SB + (c & 1) * 16384), 8192, 1024);
        const uint32_t s_next = tmem + ((c + 1) & 1) * 64, o_buf = tmem + 128 + (c & 1) * 64;
        if (!wait(FULL + s, (c >> 1) & 1)) break;
        if (c >= 2 && !wait(O_FREE + (c & 1), ((c >> 1) - 1) & 1)) break;
        fence_after_sync();
        // S0-independent terms: Kt^T U onto the next state, M U onto the output
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {
          mma_bf16_ss(s_next, desc_add(ktd, kk * 2048), desc_add(uhd, kk * 2048), id_t, kk > 0);
          mma_bf16_ss(o_buf, desc_add(mzd, kk * 32), desc_add(uhd, kk * 2048), id_o, kk > 0);
        }
        if (!wait(SB_READY, c & 1)) break;
        fence_after_sync();
        // the chain: Ac S0, then the output's Pc S0 off it (the next state is
        // written into the other bf16 buffer while this one is still read)
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)
          mma_bf16_ss(s_next, desc_add(acd, (kk >> 2) * 16384 + (kk & 3) * 32),
                      desc_add(sbd, kk * 2048), id_s, true);
        mma_commit(&bar[S_DONE]);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)
          mma_bf16_ss(o_buf, desc_add(pcd, (kk >> 2) * 8192 + (kk & 3) * 32),
                      desc_add(sbd, kk * 2048), id_o, true);
        mma_commit(&bar[O_DONE + (c & 1)]);
        mma_commit(&bar[EMPTY + s]);
      }
    }
    __syncwarp();
  } else if (warp < 4) {  // ------------------------------- state (lane = dk row)
    const int row = tid;
    const uint32_t lq = uint32_t(warp * 32) << 16;
    float* sp = p.state + (int64_t(h) * DK + row) * DV + vb * BV;
    // one state row into the bf16 operand of chunk `cn`; the buffer was last
    // read by chunk cn - 2's products, which completed before S_DONE of cn - 1
    auto put_bf16 = [&](const float* v, int cn) {
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<uint4*>(smem + S_SB + (cn & 1) * 16384 + sw_chunk(row, ch)) =
            pack8(v + ch * 8);
      fence_proxy_async_smem();
      mbar_arrive(&bar[SB_READY]);
    };
    {
      float v[64];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 x = reinterpret_cast<const float4*>(sp)[i];
        v[4 * i] = x.x;
        v[4 * i + 1] = x.y;
        v[4 * i + 2] = x.z;
        v[4 * i + 3] = x.w;
      }
      put_bf16(v, 0);
    }
    bool ok = true;
    for (int c = 0; c < nc && ok; ++c) {
      ok = __all_sync(0xFFFFFFFFu, wait(S_DONE, c & 1));
      fence_after_sync();
      uint32_t a[32], b[32];
      const uint32_t sb = tmem + lq + ((c + 1) & 1) * 64;
      tmem_ld32(sb, a);
      tmem_ld32(sb + 32, b);
      tmem_wait_ld();
      if (c + 1 < nc) {
        float v[64];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __uint_as_float(a[i]);
          v[32 + i] = __uint_as_float(b[i]);
        }
        fence_before_sync();
        put_bf16(v, c + 1);
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
    if (!ok) *abort_flag = 1;
  } else {  // ------------------------------ outputs, warps 4-7 (quadrant q = warp - 4)
    // lane i < 16 of warp 4 + q holds output row 16 q + i of the chunk; the
    // warp stages its 16 rows as two [16 rows][32 f32] boxes in the 128-byte
    // swizzle and stores them with two tensor stores
    const int q = warp - 4;
    const uint32_t lq = uint32_t(q * 32) << 16;
    bool ok = true;
    for (int c = 0; c < nc && ok; ++c) {
      ok = __all_sync(0xFFFFFFFFu, wait(O_DONE + (c & 1), (c >> 1) & 1));
      fence_after_sync();
      uint32_t a[32], b[32];
      const uint32_t ob = tmem + lq + 128 + (c & 1) * 64;
      tmem_ld32(ob, a);
      tmem_ld32(ob + 32, b);
      tmem_wait_ld();
      fence_before_sync();
      mbar_arrive(&bar[O_FREE + (c & 1)]);
      uint8_t* os = smem + S_OS + (c & 1) * 16384 + q * 4096;
      if (lane == 0) store_wait_read_but<1>();  // chunk c - 2's stores have read it
      __syncwarp();
      if (lane < 16) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {  // 16-byte chunk j: columns 4j .. 4j+3
          const uint32_t* v = j < 8 ? a + 4 * j : b + 4 * (j - 8);
          *reinterpret_cast<float4*>(os + (j >> 3) * 2048 + lane * 128 + (((j & 7) ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]),
                          __uint_as_float(v[3]));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && ok) {  // rows past the block are clipped by the tensor map
        tma_store_2d(&tm_out, os, h * DV + vb * BV, c * C + q * 16);
        tma_store_2d(&tm_out, os + 2048, h * DV + vb * BV + 32, c * C + q * 16);
        tma_store_commit();
      }
    }
    if (lane == 0) tma_store_wait_all();
    if (!ok) *abort_flag = 1;
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 9) {
    fence_after_sync();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

bool gdn_prefill_serves(const hb_gdn_shape& s) {
  return s.hkd == DK && s.hvd == DV && s.nk > 0 && s.nv == 2 * s.nk;
}

GdnPrefillPlan gdn_prefill_plan(const hb_gdn_shape& s, int64_t rows) {
  GdnPrefillPlan pl;
  pl.nchunks = (rows + C - 1) / C;
  const size_t tiles = size_t(s.nv) * size_t(pl.nchunks);
  pl.off_Ac = kWsHeader;
  pl.off_Pc = pl.off_Ac + align256(tiles * TILE_AC);
  pl.off_Kt = pl.off_Pc + align256(tiles * TILE_PC);
  pl.off_M = pl.off_Kt + align256(tiles * TILE_KT);
  pl.off_U = pl.off_M + align256(tiles * TILE_M);
  pl.bytes = pl.off_U + align256(tiles * TILE_U);
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
  pp.Ac = reinterpret_cast<uint8_t*>(base + pl.off_Ac);
  pp.Pc = reinterpret_cast<uint8_t*>(base + pl.off_Pc);
  pp.Kt = reinterpret_cast<uint8_t*>(base + pl.off_Kt);
  pp.M = reinterpret_cast<uint8_t*>(base + pl.off_M);
  pp.U = reinterpret_cast<uint8_t*>(base + pl.off_U);
  pp.status = L.status;
  // qkv [rows][conv] f32 in [64 rows][128 columns] boxes (L2 prefetch only)
  CUtensorMap tm_qkv;
  const uint64_t conv = uint64_t(2 * L.shape.nk * DK + L.shape.nv * DV);
  if (!encode_2d(&tm_qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.call.qkv, uint64_t(L.call.rows),
                 conv, conv, C, DK, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const int64_t ntiles = pl.nchunks * L.shape.nk;
  const unsigned grid = unsigned(ntiles < device_sms() ? ntiles : device_sms());
  gdn_prep_kernel<<<grid, PREP_THREADS, P_SMEM, st>>>(tm_qkv, pp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  ScanParams sp;
  sp.state = L.call.state;
  sp.Ac = pp.Ac;
  sp.Pc = pp.Pc;
  sp.Kt = pp.Kt;
  sp.M = pp.M;
  sp.U = pp.U;
  sp.rows = L.call.rows;
  sp.nv = int(L.shape.nv);
  sp.nchunks = int(pl.nchunks);
  sp.status = pp.status;
  // the outputs [rows][nv*DV] f32, stored in [16 positions][32 values] boxes
  CUtensorMap tm_out;
  if (!encode_2d(&tm_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.call.output, uint64_t(L.call.rows),
                 uint64_t(L.shape.nv) * DV, uint64_t(L.shape.nv) * DV, 16, 32,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  gdn_scan_kernel<<<dim3(unsigned(L.shape.nv), DV / BV), SCAN_THREADS, S_SMEM, st>>>(tm_out, sp);
  return cudaGetLastError();
}

}  // namespace hb
