// attn_prefill.cu -- causal flash attention for sm_100a on the 5th-generation
// tensor cores (tcgen05), with the Qwen3.5 output gate in the epilogue.
//
// Replaces, in the prefill regime, the reference's attention node
// (SdpaPrefillFn blocks of 8 rows, src/jit/emit_sdpa.rs:173-304,
// src/jit/target/x86/emit_sdpa/x86/prefill.rs:733-912, remainder rows on the
// decode kernel) and the output-gate node (src/jit/target/x86/emit_elem.rs:333-420).
// Row r of the call is the query at absolute position past + r and sees keys
// [0, past + r] (src/jit/target/x86/execution/attention.rs:189-196).
//
// CTA = one tile of 128 query rows of one query head (head_dim 256), 576
// threads:
//   warp 16      TMA producers (no multicast, SWIZZLE_128B): lane 0 loads
//                the Q tile, then the K slots (a ring of four 16 KB slots,
//                slot b = column block b of a 128-key tile) and finally the
//                gate tile into the K ring; lane 1 loads the V slots (five
//                16 KB slots of 32 keys x 256 dims);
//   warp 17      MMA issuer: S_j = Q K_j^T (M128 N128 K256) into TMEM S
//                buffer j % 2; O += P_j V_j (M128 N256 K128) with P_j taken
//                from TMEM (the TS form) and V MN-major from shared memory;
//                issue order S_0, S_1, then PV_j, S_{j+2}, S_{j+2} waiting
//                for PV_j to free its buffer; every group committed to an
//                mbarrier that also frees the ring slots it read;
//   warps 0-15   softmax: warps q, q+4, q+8, q+12 own TMEM lanes 32q.. (one
//                query row per thread), each a quarter of a tile's 128 keys;
//                the row maxima meet through shared memory and a 128-thread
//                named barrier; running max and sum in the log2 domain;
//                P = 2^(s-m) written as bf16 pairs over the first 64 columns
//                of its S buffer (tcgen05.st); O rescaled in TMEM only when
//                the max grows by more than 2^8;
//   warps 0-15   epilogue: O / l, bf16, the output gate with the
//                reference's polynomial and rounding steps (hb_epilogue.cuh),
//                each thread storing 64 columns of its row.
// TMEM: S buffers at columns [0, 256), O at [256, 512) of a 512-column
// allocation.  Shared memory: Q 64 KB + K ring 64 KB + V ring 80 KB.
//
// Context-parallel hops (template CP = true) run the same pipeline over the
// K/V shard of one ring position: up to two key segments (a zig-zag shard
// holds chunks j and 2P-1-j), query rows in up to two segments, the causal
// mask taken on absolute positions.  Instead of the bf16 epilogue, the CTA
// merges its unnormalised O and its (m, l) into an f32 accumulator in the
// workspace (O_acc = O_acc 2^(m_acc - m) + O 2^(m_hop - m), the log-sum-exp
// merge); a finishing kernel divides by l, rounds and gates.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_epilogue.cuh"
#include "hb_internal.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 128, HDIM = 256;  // query rows, keys per tile, head dim
// warps 0-15 softmax and epilogue, 16 TMA, 17 MMA
constexpr int kSoftmaxWarps = 16, kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kTmaWarp = 16, kMmaWarp = 17;
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
constexpr int Q_BYTES = BM * HDIM * 2;  // 4 column blocks of [128 rows x 128 B]
constexpr int SLOT = 16384;             // one ring slot
constexpr int NSLOT = 4;                // K slots: one 128-key tile
constexpr int NVSLOT = 5;               // V slots: a tile and a quarter
constexpr int OFF_Q = 0;
// K ring: slot b holds column block b (dims 64b..64b+63) of a key tile,
// [128 keys x 128 B]; V ring: quarter g = 4 j + c of the key stream (keys
// 32c..32c+31 of tile j, [4 column blocks][32 keys][128 B]) sits in slot
// g % 5, so the first quarter of a tile loads while the previous tile's
// products still read the other four.  A slot is refilled as soon as the
// MMAs that read it have completed.
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int OFF_V = OFF_K + NSLOT * SLOT;
constexpr int OFF_BAR = OFF_V + NVSLOT * SLOT;
constexpr int NBAR = 26;
constexpr int OFF_INVL = OFF_BAR + NBAR * 8 + 16;  // 1/l (or the merge weight of O_acc)
constexpr int OFF_FB = OFF_INVL + BM * 4;          // merge weight of a CP hop's O
constexpr int OFF_XM = OFF_FB + BM * 4;            // row maxima [2 parity][4 quarters][128]
constexpr int OFF_XL = OFF_XM + 8 * BM * 4;        // row sums [4 quarters][128]
constexpr int SMEM_BYTES = OFF_XL + 4 * BM * 4 + 1024;  // + 1 KB alignment slack
constexpr uint32_t TMEM_COLS = 512;
// S_j in columns [128 (j%2), +128); P_j (bf16, two per column) overwrites
// its first 64 columns; O in [256, 512)
constexpr uint32_t S_COL = 0, O_COL = 256;
constexpr float kRescaleLog2 = 8.0f;  // keep a stale max while p stays below 2^8
// pairs c % 8 of a thread's 32 probability pairs whose 2^x comes from the
// polynomial (bit c set), the rest from the SFU
constexpr uint32_t kPolyPairs = 0xA4u;  // pairs 2, 5, 7

// 2^x on two lanes for x <= 8 (the max may be stale by up to 2^8) without
// the SFU: Cody-Waite range reduction x = j + f with j = round(x) (adding
// and removing 1.5 * 2^23 leaves j in the low bits of the sum) and f in
// [-1/2, 1/2], 2^f by a cubic fitted here for least relative error on that
// interval (max relative error 7.5e-5, far below the bf16 rounding of P),
// and j added to the exponent field.  x is clamped at -126 so that the
// exponent stays in range; such p are below 2^-125 and vanish in the sums.
HB_DEV uint64_t exp2_poly2(uint64_t x2) {
  const uint64_t x = f2(fmaxf(f2lo(x2), -126.0f), fmaxf(f2hi(x2), -126.0f));
  const uint64_t shift = f2(12582912.0f, 12582912.0f);
  const uint64_t t = f2add(x, shift);
  const uint64_t f = f2sub(x, f2sub(t, shift));
  uint64_t q = f2fma(f2(0.055171650f, 0.055171650f), f, f2(0.24261114f, 0.24261114f));
  q = f2fma(q, f, f2(0.69326097f, 0.69326097f));
  q = f2fma(q, f, f2(0.99992806f, 0.99992806f));
  const uint32_t lo = uint32_t(q) + (uint32_t(t) << 23);
  const uint32_t hi = uint32_t(q >> 32) + (uint32_t(t >> 32) << 23);
  return (uint64_t(hi) << 32) | lo;
}

enum Bar { Q_FULL = 0, K_FULL = 1, K_EMPTY = 5, V_FULL = 9, V_EMPTY = 14, S_FULL = 19,
           P_FULL = 21, PV_DONE = 23, GATE_FULL = 25 };

HB_DEV void epilogue_sync() { asm volatile("bar.sync 2, 512;" ::: "memory"); }

// Barrier of the four softmax warps of lane quadrant q (warps q, q + 4,
// q + 8, q + 12, named barrier 3 + q); returns the AND of `v` over their 128
// threads, so all four take the same early exit.
HB_DEV bool quad_sync_and(int q, bool v) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, %2, 128, p; selp.u32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(3 + q)
      : "memory");
  return r != 0;
}

// Kept at 104 bytes: with the tensor maps, a larger parameter block made
// the same kernel ~5% slower on B200 (measured).
struct PrefillParams {
  const uint16_t* q;  // gate reads
  uint16_t* out;
  int64_t q_row, out_row, gate_offset;
  int rows, heads, gqa, n_qtiles;
  int q_pos0;  // position of row 0 (= past); on a CP hop, of the first chunk's row 0
  float scale_log2;
  int* status;
  // context-parallel hop: rows [0, chunk) sit at positions q_pos0.., rows
  // [chunk, 2 chunk) at q_pos1..; the shard's K/V rows [0, chunk) hold
  // positions kpos0.., rows [chunk, 2 chunk) positions kpos1..
  int chunk, q_pos1, kpos0, kpos1;
  int merge;  // 0 on the first hop (write the accumulators only)
  // [head][q tile][256 columns][128 rows] f32 O, then [head][q tile][128] (m, l)
  float* acc;
};

// Key tiles of a CP hop's segment s that query rows at positions <= qmax see.
HB_DEV int segment_tiles(const PrefillParams& p, int s, int qmax) {
  const int pos = s ? p.kpos1 : p.kpos0;
  if (qmax < pos) return 0;
  return (min(p.chunk, qmax - pos + 1) + BN - 1) / BN;
}

template <bool CP>
__global__ void __launch_bounds__(kThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* inv_l = reinterpret_cast<float*>(smem + OFF_INVL);
  float* w_hop = reinterpret_cast<float*>(smem + OFF_FB);
  float* xmax = reinterpret_cast<float*>(smem + OFF_XM);
  float* xsum = reinterpret_cast<float*>(smem + OFF_XL);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.n_qtiles - 1 - int(blockIdx.x) / p.heads;  // heaviest tiles first
  const int h = int(blockIdx.x) % p.heads;
  const int kvh = h / p.gqa;
  const int m0 = qt * BM;
  int qlo, n0, ntiles;  // position of row 0, key tiles of segment 0 and in all
  if constexpr (CP) {
    qlo = m0 < p.chunk ? p.q_pos0 + m0 : p.q_pos1 + (m0 - p.chunk);
    const int qmax = qlo + min(BM, p.rows - m0) - 1;
    n0 = segment_tiles(p, 0, qmax);
    ntiles = n0 + segment_tiles(p, 1, qmax);
  } else {  // row r at position past + r (= q_pos0 + r) sees keys [0, past + r]
    qlo = p.q_pos0 + m0;
    n0 = ntiles = (min(qlo + BM, p.q_pos0 + p.rows) + BN - 1) / BN;
  }
  if (CP && ntiles == 0) return;  // this shard holds no key the tile sees

  if (threadIdx.x == 0) {
    mbar_init(&bar[Q_FULL], 1);
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&bar[K_FULL + s], 1);
      mbar_init(&bar[K_EMPTY + s], 1);
    }
    for (int s = 0; s < NVSLOT; ++s) {
      mbar_init(&bar[V_FULL + s], 1);
      mbar_init(&bar[V_EMPTY + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[S_FULL + s], 1);
      mbar_init(&bar[P_FULL + s], kSoftmaxThreads);
      mbar_init(&bar[PV_DONE + s], 1);
    }
    mbar_init(&bar[GATE_FULL], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](int b, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait(&bar[b], parity)) return true;
    record_status(p.status, kStatusTimeout);
    *abort_flag = 1;
    return false;
  };
  // K/V row of the first key of tile j in the K/V buffers
  auto key_row = [&](int j) -> int {
    return !CP ? j * BN : j < n0 ? j * BN : p.chunk + (j - n0) * BN;
  };

  if (warp == kTmaWarp) {  // ---------------------- TMA producers (lanes 0, 1)
    if (lane == 0) {  // Q, then the K slots, then the gate tile
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      mbar_arrive_expect_tx(&bar[Q_FULL], Q_BYTES);
      for (int c = 0; c < 4; ++c)
        tma_load_2d(smem + OFF_Q + c * SLOT, &tmQ, &bar[Q_FULL], h * HDIM + c * 64, m0);
      {  // the Q tile of the CTA one SM-count later, which starts about when
         // this one ends, into L2
        uint32_t nsm;
        asm("mov.u32 %0, %%nsmid;" : "=r"(nsm));
        const int nb = int(blockIdx.x + nsm);
        if (nb < int(gridDim.x)) {
          const int nqt = p.n_qtiles - 1 - nb / p.heads, nh = nb % p.heads;
          for (int c = 0; c < 4; ++c) tma_prefetch_l2_2d(&tmQ, nh * HDIM + c * 64, nqt * BM);
        }
      }
      bool ok = true;
      for (int j = 0; ok && j < ntiles; ++j) {
        const int kr = key_row(j);
        for (int b = 0; b < NSLOT; ++b) {
          if (j >= 1 && !wait(K_EMPTY + b, (j - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bar[K_FULL + b], SLOT);
          tma_load_3d(smem + OFF_K + b * SLOT, &tmK, &bar[K_FULL + b], b * 64, kr, kvh);
        }
      }
      // the gate tile [128 rows x 256] goes into the K ring once the last S
      // product has read it
      if (ok && !CP && p.gate_offset >= 0) {
        bool free_ring = true;
        for (int b = 0; b < NSLOT; ++b) free_ring = free_ring && wait(K_EMPTY + b, (ntiles - 1) & 1);
        if (free_ring) {
          mbar_arrive_expect_tx(&bar[GATE_FULL], Q_BYTES);
          for (int c = 0; c < 4; ++c)
            tma_load_2d(smem + OFF_K + c * SLOT, &tmQ, &bar[GATE_FULL],
                        int(p.gate_offset) + h * HDIM + c * 64, m0);
        }
      }
    } else if (lane == 1) {  // the V quarters, through five slots
      prefetch_tmap(&tmV);
      for (int g = 0; g < 4 * ntiles; ++g) {
        const int sl = g % NVSLOT, fill = g / NVSLOT;
        if (fill >= 1 && !wait(V_EMPTY + sl, (fill - 1) & 1)) break;
        mbar_arrive_expect_tx(&bar[V_FULL + sl], SLOT);
        const int kr = key_row(g >> 2) + (g & 3) * 32;
        for (int db = 0; db < 4; ++db)
          tma_load_3d(smem + OFF_V + sl * SLOT + db * 4096, &tmV, &bar[V_FULL + sl], db * 64, kr,
                      kvh);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {  // ------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idPV = idesc_bf16(BM, HDIM, false, true);
      const uint64_t qd0 = sw128_desc(smem_u32(smem + OFF_Q), 16, 1024),
                     kd0 = sw128_desc(smem_u32(smem + OFF_K), 16, 1024),
                     vd0 = sw128_desc(smem_u32(smem + OFF_V), 4096, 1024);
      // S_j = Q K_j^T (M128 N128 K256) into TMEM buffer j % 2; that buffer
      // held P_{j-2}, so PV_{j-2} must have completed
      auto issue_s = [&](int j) -> bool {
        const int sb = j & 1;
        if (j >= 2 && !wait(PV_DONE + sb, ((j - 2) >> 1) & 1)) return false;
        for (int b = 0; b < NSLOT; ++b) {
          if (!wait(K_FULL + b, j & 1)) return false;
          fence_after_sync();
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const uint64_t a = desc_add(qd0, b * SLOT + k4 * 32);
            const uint64_t bd = desc_add(kd0, b * SLOT + k4 * 32);
            mma_bf16_ss(tmem + S_COL + sb * BN, a, bd, idS, b > 0 || k4 > 0);
          }
          mma_commit(&bar[K_EMPTY + b]);
        }
        mma_commit(&bar[S_FULL + sb]);
        return true;
      };
      // order S_0, S_1, then PV_j followed by S_{j+2}
      bool ok = wait(Q_FULL, 0);
      for (int j = 0; ok && j < ntiles && j < 2; ++j) ok = issue_s(j);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int sb = j & 1;
        if (!wait(P_FULL + sb, (j >> 1) & 1)) break;
        fence_after_sync();
        // O += P_j V_j: P from TMEM (8 columns per 16 keys), V slot c holds
        // keys 32c.. (column blocks 4096 B apart)
        for (int c = 0; c < 4; ++c) {
          const int g = 4 * j + c, sl = g % NVSLOT;
          if (!wait(V_FULL + sl, (g / NVSLOT) & 1)) {
            ok = false;
            break;
          }
          fence_after_sync();
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2) {
            const int kk = c * 2 + k2;
            const uint64_t bd = desc_add(vd0, sl * SLOT + k2 * 2048);
            mma_bf16_ts(tmem + O_COL, tmem + S_COL + sb * BN + kk * 8, bd, idPV, j > 0 || kk > 0);
          }
          mma_commit(&bar[V_EMPTY + sl]);
        }
        if (!ok) break;
        mma_commit(&bar[PV_DONE + sb]);
        if (j + 2 < ntiles) ok = issue_s(j + 2);
      }
    }
    __syncwarp();
  } else {  // ----------------------------------------- softmax (warps 0-15)
    // warps q, q + 4, q + 8, q + 12 own rows 32q .. 32q + 31 (TMEM lanes);
    // warp q + 4k takes keys 32k .. 32k + 31 of each tile.  The row max is
    // exchanged through shared memory each tile, the row sum at the end.
    const int q4 = warp & 3, hq = warp >> 2;
    const int row = q4 * 32 + lane;
    const uint32_t tl = tmem + (uint32_t(q4 * 32) << 16);
    const int qpos = qlo + row;
    if (CP && p.merge && hq == 3) {
      // bring this tile's accumulator (128 KB, 1024 lines) into L2 for the merge
      const char* a = reinterpret_cast<const char*>(
          p.acc + (size_t(h) * p.n_qtiles + qt) * (size_t(HDIM) * BM));
      for (int ln = threadIdx.x - 384; ln < HDIM * BM * 4 / 128; ln += 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a + size_t(ln) * 128));
    }
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      ok = __all_sync(0xFFFFFFFFu, wait(S_FULL + sb, (j >> 1) & 1) && ok);
      fence_after_sync();
      uint32_t ra[32];
      tmem_ld32(tl + S_COL + sb * BN + hq * 32, ra);
      tmem_wait_ld();
      fence_before_sync();
      // key positions kb.. of this tile; keys from klen on lie past the
      // segment (one segment starting at position 0 outside CP hops)
      int kb = j * BN, klen = BN;
      if constexpr (CP) {
        const bool s1 = j >= n0;
        const int t = s1 ? j - n0 : j;
        kb = (s1 ? p.kpos1 : p.kpos0) + t * BN;
        klen = p.chunk - t * BN;
      }
      const int kh0 = kb + hq * 32, klh = klen - hq * 32;  // this thread's 32 keys
      const bool full = kb + BN - 1 <= qlo && (!CP || klen >= BN);  // no key masked
      if (!full) {  // masked scores become -inf (raw, before scaling)
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (!(kh0 + c <= qpos && (!CP || c < klh))) ra[c] = 0xFF800000u;
      }
      // the max of the raw scores, scaled once (scale > 0)
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) m8[c & 7] = fmaxf(m8[c & 7], __uint_as_float(ra[c]));
      float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                       fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * p.scale_log2;
      // the other quarters' maxima (and one shared decision to stop); the
      // barrier also orders all four threads' S reads before any writes P
      // over them
      float* xm = xmax + (j & 1) * 4 * BM + row;
      xm[hq * BM] = mx;
      ok = quad_sync_and(q4, ok);
      fence_after_sync();
      if (!ok) break;
      mx = fmaxf(fmaxf(xm[0], xm[BM]), fmaxf(xm[2 * BM], xm[3 * BM]));
      const float m_new = fmaxf(m, mx);
      float factor = 1.f;
      bool resc = false;
      if (m == -INFINITY) {
        m = m_new;  // first keys of the row: O holds nothing yet
      } else if (m_new > m + kRescaleLog2) {
        factor = fast_exp2(m - m_new);
        resc = true;
      }
      if (__any_sync(0xFFFFFFFFu, resc)) {
        // O holds PV_0 .. PV_{j-1}; the last of them may still be running.
        // Each thread rescales a quarter of the row's 256 columns.
        const int jp = j - 1;
        ok = __all_sync(0xFFFFFFFFu, wait(PV_DONE + (jp & 1), (jp >> 1) & 1) && ok);
        fence_after_sync();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tl + O_COL + hq * 64 + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
          tmem_st32(tl + O_COL + hq * 64 + c * 32, r);
        }
        tmem_wait_st();
        if (resc) {
          l *= factor;
          m = m_new;
        }
      }
      // P_j = 2^(s - m) in bf16 over the first 64 columns of S_j: keys
      // 32 hq .. + 31 go to columns 16 hq .. + 15, two keys per column.
      // x = s scale - m by one paired FMA; 2^x by the SFU, except, on tiles
      // with no masked key, for three pairs in eight, which go to
      // exp2_poly2 on the FMA pipe so that neither unit alone paces the
      // softmax (a masked x = -inf must give exactly 0: SFU)
      uint32_t pk[16];
      const uint64_t sc2 = f2(p.scale_log2, p.scale_log2), nm2 = f2(-m, -m);
      uint64_t s4[4] = {0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint64_t x2 =
            f2fma(f2(__uint_as_float(ra[2 * c]), __uint_as_float(ra[2 * c + 1])), sc2, nm2);
        const uint64_t p2 = full && ((kPolyPairs >> (c & 7)) & 1u)
                                ? exp2_poly2(x2)
                                : f2(fast_exp2(f2lo(x2)), fast_exp2(f2hi(x2)));
        s4[c & 3] = f2add(s4[c & 3], p2);
        pk[c] = pack_bf16x2(f2lo(p2), f2hi(p2));
      }
      const uint64_t s2 = f2add(f2add(s4[0], s4[1]), f2add(s4[2], s4[3]));
      l += f2lo(s2) + f2hi(s2);
      tmem_st16(tl + S_COL + sb * BN + hq * 16, pk);
      tmem_wait_st();
      fence_before_sync();
      mbar_arrive(&bar[P_FULL + sb]);
    }
    // the row sum of the four quarters
    xsum[hq * BM + row] = l;
    if (!ok) *abort_flag = 1;
    epilogue_sync();
    if (hq == 0) {
      l = ((l + xsum[BM + row]) + xsum[2 * BM + row]) + xsum[3 * BM + row];
      if constexpr (CP) {
        // log-sum-exp merge of (m, l) with what earlier hops left; O and l of
        // this hop are relative to m (a max that may be stale by < 2^8)
        const size_t units = size_t(p.heads) * p.n_qtiles;
        float2* ml = reinterpret_cast<float2*>(p.acc + units * (size_t(HDIM) * BM)) +
                     (size_t(h) * p.n_qtiles + qt) * BM + row;
        float wa = 0.f, wb = 1.f, mo = m, lo = l;
        if (p.merge) {
          const float2 a = *ml;
          mo = fmaxf(a.x, m);
          if (mo == -INFINITY) {
            wb = 0.f;
            lo = 0.f;
          } else {
            wa = fast_exp2(a.x - mo);
            wb = fast_exp2(m - mo);
            lo = a.y * wa + l * wb;
          }
        }
        if (ok && !*abort_flag) *ml = make_float2(mo, lo);
        inv_l[row] = wa;
        w_hop[row] = wb;
      } else {
        inv_l[row] = l > 0.f ? 1.f / l : 0.f;
      }
    }
  }

  if (warp < kSoftmaxWarps) {  // --------------------------- epilogue (warps 0-15)
    epilogue_sync();  // inv_l written
    const int jl = ntiles - 1;
    bool ok = wait(PV_DONE + (jl & 1), (jl >> 1) & 1);
    if (!CP && p.gate_offset >= 0) ok = wait(GATE_FULL, 0) && ok;
    ok = __all_sync(0xFFFFFFFFu, ok);
    fence_after_sync();
    const int qd = warp & 3, hq = warp >> 2;  // TMEM lane quadrant, column quarter
    const int rl = qd * 32 + lane;            // row within the tile
    const uint32_t tq = tmem + (uint32_t(qd * 32) << 16);
    const float inv = inv_l[rl];
    if constexpr (CP) {
      // O_acc <- O_acc * wa + O * wb; [32 columns][128 rows] per block, so a
      // warp's 32 rows are one 128-byte line per column
      const float wa = inv, wb = w_hop[rl];
      float* acc = p.acc + (size_t(h) * p.n_qtiles + qt) * (size_t(HDIM) * BM) + rl;
#pragma unroll 1
      for (int ch = 0; ch < 2; ++ch) {
        const int col0 = hq * 64 + ch * 32;
        uint32_t o[32];
        tmem_ld32(tq + O_COL + col0, o);
        tmem_wait_ld();
        float* ap = acc + size_t(col0) * BM;
        if (ok && !*abort_flag) {
          if (p.merge) {
            float a[32];  // every load in flight before the first store
#pragma unroll
            for (int i = 0; i < 32; ++i) a[i] = ap[i * BM];
#pragma unroll
            for (int i = 0; i < 32; ++i) ap[i * BM] = fmaf(a[i], wa, __uint_as_float(o[i]) * wb);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) ap[i * BM] = __uint_as_float(o[i]);
          }
        }
      }
    } else {
      // each thread writes its row's 32-byte pieces straight to global memory
      constexpr int W = kEpilogueWidth;
      const bool store = ok && !*abort_flag && m0 + rl < p.rows;
      uint16_t* orow = p.out + size_t(m0 + rl) * size_t(p.out_row) + h * HDIM;
#pragma unroll 1
      for (int blk = 0; blk < 64 / W; ++blk) {
        const int col0 = hq * 64 + blk * W;
        uint32_t o[W];
        tmem_ld16(tq + O_COL + col0, o);
        tmem_wait_ld();
        // a = bf16(O / l), then the gate y = bf16(a / (1 + exp(-g))) for W
        // columns at once (hb_epilogue.cuh); the gate tile sits in the K
        // ring as [4 column blocks][128 rows][128 B], 128B-swizzled
        uint32_t gw[W / 2], w[W / 2];
        if (p.gate_offset >= 0) {
          const int cb = col0 >> 6, c16 = (col0 & 63) >> 3;
#pragma unroll
          for (int k = 0; k < W / 8; ++k) {
            const int phys = cb * (BM * 128) + rl * 128 + (((c16 + k) ^ (rl & 7)) << 4);
            const uint4 gv = *reinterpret_cast<const uint4*>(smem + OFF_K + phys);
            gw[4 * k] = gv.x; gw[4 * k + 1] = gv.y; gw[4 * k + 2] = gv.z; gw[4 * k + 3] = gv.w;
          }
          epilogue_block<W, true>(o, inv, gw, w);
        } else {
          epilogue_block<W, false>(o, inv, gw, w);
        }
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(orow + col0);
#pragma unroll
          for (int k = 0; k < W / 8; ++k)
            dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        }
      }
    }
  }

  fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

bool encode_bf16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                 const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, base, dims, strides_bytes, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

bool prefill_serves(int64_t head_dim) { return head_dim == HDIM; }

cudaError_t launch_attn_prefill(const PrefillLaunch& L, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  const int64_t kv_rows = L.cp ? L.kv_rows : L.past + L.rows;
  const cuuint64_t qd[2] = {cuuint64_t(L.q_row), cuuint64_t(L.rows)};
  const cuuint64_t qs[1] = {cuuint64_t(L.q_row) * 2};
  const cuuint32_t qbox[2] = {64, BM};
  const cuuint64_t kd[3] = {cuuint64_t(HDIM), cuuint64_t(kv_rows), cuuint64_t(L.hkv)};
  const cuuint64_t ks[2] = {cuuint64_t(HDIM) * 2, cuuint64_t(L.kv_stride) * 2};
  const cuuint32_t kbox[3] = {64, BN, 1};  // one K slot: 128 keys of one column block
  const cuuint32_t vbox[3] = {64, 32, 1};  // a quarter of a V slot: 32 keys of one column block
  if (!encode_bf16(&tq, L.q, 2, qd, qs, qbox) || !encode_bf16(&tk, L.keys, 3, kd, ks, kbox) ||
      !encode_bf16(&tv, L.values, 3, kd, ks, vbox))
    return cudaErrorInvalidValue;
  // the epilogue writes 16-byte pieces of output rows
  if (!L.cp && ((reinterpret_cast<uintptr_t>(L.out) & 15) || (L.out_row & 7)))
    return cudaErrorInvalidValue;
  static DeviceFlags configured;
  cudaError_t e = configured.once([] {
    cudaError_t r = cudaFuncSetAttribute(attn_prefill_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(attn_prefill_kernel<true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    return r;
  });
  if (e != cudaSuccess) return e;
  PrefillParams p;
  p.q = L.q;
  p.out = L.out;
  p.q_row = L.q_row;
  p.out_row = L.out_row;
  p.gate_offset = L.cp ? -1 : L.gate_offset;
  p.rows = int(L.rows);
  p.heads = int(L.heads);
  p.gqa = int(L.gqa);
  p.n_qtiles = int((L.rows + BM - 1) / BM);
  p.q_pos0 = int(L.cp ? L.q_pos0 : L.past);
  p.chunk = int(L.chunk);
  p.q_pos1 = int(L.q_pos1);
  p.kpos0 = int(L.kpos[0]);
  p.kpos1 = int(L.kpos[1]);
  p.scale_log2 = L.scale * 1.4426950408889634f;
  p.status = L.status;
  p.acc = L.acc;
  p.merge = L.merge ? 1 : 0;
  const unsigned grid = unsigned(p.n_qtiles * p.heads);
  if (L.cp)
    attn_prefill_kernel<true><<<grid, kThreads, SMEM_BYTES, st>>>(tq, tk, tv, p);
  else
    attn_prefill_kernel<false><<<grid, kThreads, SMEM_BYTES, st>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

namespace {

// The last step of a context-parallel prefill: O_acc / l, rounded to bf16
// and gated exactly as the single-GPU epilogue does, written token-major.
// CTA = one (q tile, head); 32-column blocks of the accumulator are turned
// from [column][row] to row-major through shared memory.
__global__ void __launch_bounds__(256)
    attn_cp_finish_kernel(const float* __restrict__ acc_o, const uint16_t* __restrict__ q, uint16_t* __restrict__ out, int64_t q_row,
                          int64_t out_row, int64_t gate_offset, int rows, int heads, int n_qtiles) {
  __shared__ float tile[32][BM + 1];
  __shared__ float inv_s[BM];
  const int qt = int(blockIdx.x) / heads, h = int(blockIdx.x) % heads;
  const size_t unit = size_t(h) * n_qtiles + qt;
  const float* acc = acc_o + unit * (size_t(HDIM) * BM);
  const float2* acc_ml =
      reinterpret_cast<const float2*>(acc_o + size_t(heads) * n_qtiles * (size_t(HDIM) * BM));
  const int t = threadIdx.x;
  if (t < BM) {
    const float l = acc_ml[unit * BM + t].y;
    inv_s[t] = l > 0.f ? 1.f / l : 0.f;
  }
  const int wr = t >> 1, part = t & 1;  // write phase: row, 16-column half
  const int rr = t & (BM - 1), ih = t >> 7;  // read phase: row, 16-column half
  const int64_t grow = int64_t(qt) * BM + wr;
#pragma unroll 1
  for (int cc = 0; cc < HDIM / 32; ++cc) {
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      tile[ih * 16 + i][rr] = acc[size_t(cc * 32 + ih * 16 + i) * BM + rr];
    __syncthreads();
    if (grow < rows) {
      const float inv = inv_s[wr];
      const int col = h * HDIM + cc * 32 + part * 16;
      uint32_t g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (gate_offset >= 0) {
        const uint4* gp = reinterpret_cast<const uint4*>(q + grow * q_row + gate_offset + col);
        const uint4 g0 = gp[0], g1 = gp[1];
        g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w;
        g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
      }
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint16_t a0 = f32_to_bf16_cvtne(tile[part * 16 + 2 * k][wr] * inv);
        uint16_t a1 = f32_to_bf16_cvtne(tile[part * 16 + 2 * k + 1][wr] * inv);
        if (gate_offset >= 0) {
          a0 = gate_bf16(a0, uint16_t(g[k] & 0xFFFFu));
          a1 = gate_bf16(a1, uint16_t(g[k] >> 16));
        }
        w[k] = uint32_t(a0) | (uint32_t(a1) << 16);
      }
      uint4* op = reinterpret_cast<uint4*>(out + grow * out_row + col);
      op[0] = make_uint4(w[0], w[1], w[2], w[3]);
      op[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
}

}  // namespace

size_t cp_acc_bytes(int64_t heads, int64_t rows) {
  const int64_t nqt = (rows + BM - 1) / BM;
  return size_t(mul_sat(mul_sat(heads, nqt), int64_t(BM) * (HDIM + 2) * sizeof(float)));
}

cudaError_t launch_attn_cp_finish(const PrefillLaunch& L, cudaStream_t st) {
  const int nqt = int((L.rows + BM - 1) / BM);
  attn_cp_finish_kernel<<<unsigned(nqt * L.heads), 256, 0, st>>>(
      L.acc, L.q, L.out, L.q_row, L.out_row,
      L.gate_offset, int(L.rows), int(L.heads), nqt);
  return cudaGetLastError();
}

}  // namespace hb
