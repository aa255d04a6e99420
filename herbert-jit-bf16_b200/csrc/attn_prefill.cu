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
// CTA = one tile of 128 query rows of one query head (head_dim 256):
//   warp 4       TMA producer: Q tile once, then K and V tiles of 64 keys
//                into two-stage rings (SWIZZLE_128B, no multicast);
//   warp 5       MMA issuer: S_j = Q K_j^T (M128 N64 K256, 16 MMAs) into one
//                of two TMEM S buffers, then O += P_{j-1} V_{j-1} (M128 N256
//                K64, 4 MMAs, V read MN-major) into the TMEM O accumulator;
//                each group is committed to an mbarrier;
//   warps 0-3    softmax: one thread per query row reads its S row from TMEM,
//                applies the causal mask, keeps the running max m and sum l in
//                the log2 domain, writes P = 2^(s - m) as bf16 into shared
//                memory in the UMMA K-major swizzled layout, and rescales the
//                O row in TMEM only when the max grows by more than 2^8;
//   warps 0-7    epilogue: O / l, bf16, gate with the reference's exp
//                polynomial and rounding steps; the gate tile comes in by TMA
//                (into the K ring, free once the last S is computed) and the
//                output tile leaves by TMA store (staged in the V ring).
// TMEM: S buffers at columns [0,128), O at [256,512) of a 512-column
// allocation.  Shared memory: Q 64 KB + K 2x32 KB + V 2x32 KB + P 2x16 KB.
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
#include "hb_internal.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 64, HDIM = 256;
constexpr int kThreads = 320;  // warps 0-3 softmax, 0-7 epilogue, 8 TMA, 9 MMA
constexpr int kTmaWarp = 8, kMmaWarp = 9;
constexpr int Q_BYTES = BM * HDIM * 2;   // 4 column blocks of [128 rows x 128 B]
constexpr int KV_BYTES = BN * HDIM * 2;  // 4 column blocks of [64 rows x 128 B]
constexpr int P_BYTES = BM * BN * 2;     // 1 block of [128 rows x 128 B]
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr int NBAR = 18;
constexpr int OFF_INVL = OFF_BAR + NBAR * 8 + 16;  // 1/l (or the merge weight of O_acc)
constexpr int SMEM_BYTES = OFF_INVL + BM * 4 + 1024;  // + 1 KB alignment slack
// merge weight of a CP hop's O: in the K ring, which no MMA reads once the
// softmax has seen the last S (a hop loads no gate tile there)
constexpr int OFF_FB = OFF_K;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL = 0, O_COL = 256;
constexpr float kRescaleLog2 = 8.0f;  // keep a stale max while p stays below 2^8

enum Bar { Q_FULL = 0, K_FULL = 1, K_EMPTY = 3, V_FULL = 5, V_EMPTY = 7, S_FULL = 9,
           S_EMPTY = 11, P_FULL = 13, PV_DONE = 15, GATE_FULL = 17 };

HB_DEV void epilogue_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

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
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmO, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* inv_l = reinterpret_cast<float*>(smem + OFF_INVL);
  float* w_hop = reinterpret_cast<float*>(smem + OFF_FB);

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
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[K_FULL + s], 1);
      mbar_init(&bar[K_EMPTY + s], 1);
      mbar_init(&bar[V_FULL + s], 1);
      mbar_init(&bar[V_EMPTY + s], 1);
      mbar_init(&bar[S_FULL + s], 1);
      mbar_init(&bar[S_EMPTY + s], 128);
      mbar_init(&bar[P_FULL + s], 128);
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

  if (warp == kTmaWarp) {  // ----------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmO);
      mbar_arrive_expect_tx(&bar[Q_FULL], Q_BYTES);
      for (int c = 0; c < 4; ++c)
        tma_load_2d(smem + OFF_Q + c * (BM * 128), &tmQ, &bar[Q_FULL], h * HDIM + c * 64, m0);
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int kr = !CP ? j * BN : j < n0 ? j * BN : p.chunk + (j - n0) * BN;
        if (j >= 2 && !wait(K_EMPTY + s, ph ^ 1)) break;
        mbar_arrive_expect_tx(&bar[K_FULL + s], KV_BYTES);
        for (int c = 0; c < 4; ++c)
          tma_load_3d(smem + OFF_K + s * KV_BYTES + c * (BN * 128), &tmK, &bar[K_FULL + s], c * 64,
                      kr, kvh);
        if (j >= 2 && !wait(V_EMPTY + s, ph ^ 1)) break;
        mbar_arrive_expect_tx(&bar[V_FULL + s], KV_BYTES);
        for (int c = 0; c < 4; ++c)
          tma_load_3d(smem + OFF_V + s * KV_BYTES + c * (BN * 128), &tmV, &bar[V_FULL + s], c * 64,
                      kr, kvh);
      }
      // the gate tile [128 rows x 256] goes into the K ring once the last one
      // or two S products have read it
      if (!CP && p.gate_offset >= 0) {
        bool free_ring = true;
        for (int j = ntiles > 2 ? ntiles - 2 : 0; j < ntiles; ++j)
          free_ring = free_ring && wait(K_EMPTY + (j & 1), (j >> 1) & 1);
        if (free_ring) {
          mbar_arrive_expect_tx(&bar[GATE_FULL], Q_BYTES);
          for (int c = 0; c < 4; ++c)
            tma_load_2d(smem + OFF_K + c * (BM * 128), &tmQ, &bar[GATE_FULL],
                        int(p.gate_offset) + h * HDIM + c * 64, m0);
        }
      }
    }
  } else if (warp == kMmaWarp) {  // ------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idPV = idesc_bf16(BM, HDIM, false, true);
      const uint32_t qb = smem_u32(smem + OFF_Q);
      bool ok = wait(Q_FULL, 0);
      for (int j = 0; ok && j <= ntiles; ++j) {
        if (j < ntiles) {
          const int s = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!wait(K_FULL + s, ph)) break;
          if (j >= 2 && !wait(S_EMPTY + s, ph ^ 1)) break;
          fence_after_sync();
          const uint32_t kb = smem_u32(smem + OFF_K + s * KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < HDIM / 16; ++kk) {
            const uint64_t a = sw128_desc(qb + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
            const uint64_t b = sw128_desc(kb + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
            mma_bf16_ss(tmem + S_COL + s * BN, a, b, idS, kk > 0);
          }
          mma_commit(&bar[S_FULL + s]);
          mma_commit(&bar[K_EMPTY + s]);
        }
        if (j >= 1) {
          const int jj = j - 1, s = jj & 1;
          const uint32_t ph = (jj >> 1) & 1;
          if (!wait(P_FULL + s, ph) || !wait(V_FULL + s, ph)) break;
          fence_after_sync();
          const uint32_t pb = smem_u32(smem + OFF_P + s * P_BYTES);
          const uint32_t vb = smem_u32(smem + OFF_V + s * KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t a = sw128_desc(pb + kk * 32, 16, 1024);
            const uint64_t b = sw128_desc(vb + kk * 16 * 128, BN * 128, 1024);
            mma_bf16_ss(tmem + O_COL, a, b, idPV, jj > 0 || kk > 0);
          }
          mma_commit(&bar[PV_DONE + s]);
          mma_commit(&bar[V_EMPTY + s]);
        }
      }
    }
    __syncwarp();
  } else if (warp < 4) {  // -------------------------------------- softmax
    const int row = threadIdx.x;  // 0..127 = TMEM lane
    const uint32_t tl = tmem + (uint32_t(warp * 32) << 16);
    const int qpos = qlo + row;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      ok = __all_sync(0xFFFFFFFFu, wait(S_FULL + s, ph) && ok);
      fence_after_sync();
      uint32_t ra[32], rb[32];
      tmem_ld32(tl + S_COL + s * BN, ra);
      tmem_ld32(tl + S_COL + s * BN + 32, rb);
      tmem_wait_ld();
      fence_before_sync();
      mbar_arrive(&bar[S_EMPTY + s]);
      // key positions kb.. of this tile; keys from klen on lie past the
      // segment (one segment starting at position 0 outside CP hops)
      int kb = j * BN, klen = BN;
      if constexpr (CP) {
        const bool s1 = j >= n0;
        const int t = s1 ? j - n0 : j;
        kb = (s1 ? p.kpos1 : p.kpos0) + t * BN;
        klen = p.chunk - t * BN;
      }
      float v[64];
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = -INFINITY;
      if (kb + BN - 1 <= qlo && (!CP || klen >= BN)) {  // below the diagonal for every row
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          v[c] = __uint_as_float(ra[c]) * p.scale_log2;
          v[32 + c] = __uint_as_float(rb[c]) * p.scale_log2;
          m8[c & 7] = fmaxf(m8[c & 7], fmaxf(v[c], v[32 + c]));
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          v[c] = (kb + c <= qpos && (!CP || c < klen)) ? __uint_as_float(ra[c]) * p.scale_log2
                                                       : -INFINITY;
          v[32 + c] = (kb + 32 + c <= qpos && (!CP || 32 + c < klen))
                          ? __uint_as_float(rb[c]) * p.scale_log2
                          : -INFINITY;
          m8[c & 7] = fmaxf(m8[c & 7], fmaxf(v[c], v[32 + c]));
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
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
        // O holds PV_0 .. PV_{j-1}; the last of them may still be running
        const int jp = j - 1;
        ok = __all_sync(0xFFFFFFFFu, wait(PV_DONE + (jp & 1), (jp >> 1) & 1) && ok);
        fence_after_sync();
#pragma unroll 1
        for (int c = 0; c < HDIM / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tl + O_COL + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
          tmem_st32(tl + O_COL + c * 32, r);
        }
        tmem_wait_st();
        fence_before_sync();
        if (resc) {
          l *= factor;
          m = m_new;
        }
      }
      // P_j goes to buffer s, which PV_{j-2} read
      if (j >= 2) ok = __all_sync(0xFFFFFFFFu, wait(PV_DONE + s, ph ^ 1) && ok);
      float s8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) s8[i] = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = fast_exp2(v[2 * c] - m), p1 = fast_exp2(v[2 * c + 1] - m);
        s8[c & 7] += p0 + p1;
        pk[c] = pack_bf16x2(p0, p1);
      }
      l += ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
      uint8_t* prow = smem + OFF_P + s * P_BYTES + row * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) =
            make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
      fence_proxy_async_smem();
      mbar_arrive(&bar[P_FULL + s]);
      if (!ok) break;
    }
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
      if (ok) *ml = make_float2(mo, lo);
      inv_l[row] = wa;
      w_hop[row] = wb;
    } else {
      inv_l[row] = l > 0.f ? 1.f / l : 0.f;
    }
    if (!ok) *abort_flag = 1;
  }

  if (warp < 8) {  // ------------------------------- epilogue (warps 0-7)
    if (CP && p.merge && warp >= 4) {
      // warps 4-7 idle through the main loop: bring this tile's accumulator
      // (128 KB, 1024 lines) into L2 so the merge below reads it from there
      const char* a = reinterpret_cast<const char*>(
          p.acc + (size_t(h) * p.n_qtiles + qt) * (size_t(HDIM) * BM));
      for (int ln = threadIdx.x - 128; ln < HDIM * BM * 4 / 128; ln += 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a + size_t(ln) * 128));
    }
    epilogue_sync();  // inv_l written
    const int jl = ntiles - 1;
    bool ok = wait(PV_DONE + (jl & 1), (jl >> 1) & 1);
    if (!CP && p.gate_offset >= 0) ok = wait(GATE_FULL, 0) && ok;
    ok = __all_sync(0xFFFFFFFFu, ok);
    fence_after_sync();
    const int qd = warp & 3, hc = warp >> 2;  // TMEM lane quadrant, column half
    const int rl = qd * 32 + lane;            // row within the tile
    const uint32_t tq = tmem + (uint32_t(qd * 32) << 16);
    const float inv = inv_l[rl];
    if constexpr (CP) {
      // O_acc <- O_acc * wa + O * wb; [32 columns][128 rows] per block, so a
      // warp's 32 rows are one 128-byte line per column
      const float wa = inv, wb = w_hop[rl];
      float* acc = p.acc + (size_t(h) * p.n_qtiles + qt) * (size_t(HDIM) * BM) + rl;
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        const int col0 = hc * 128 + ch * 32;
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
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      const int col0 = hc * 128 + ch * 32;
      uint32_t o[32];
      tmem_ld32(tq + O_COL + col0, o);
      tmem_wait_ld();
      const int cb = col0 >> 6, c16 = (col0 & 63) >> 3;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int phys = cb * (BM * 128) + rl * 128 + (((c16 + k) ^ (rl & 7)) << 4);
        uint4 gv = make_uint4(0, 0, 0, 0);
        if (p.gate_offset >= 0) gv = *reinterpret_cast<const uint4*>(smem + OFF_K + phys);
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint16_t a0 = f32_to_bf16_cvtne(__uint_as_float(o[k * 8 + 2 * i]) * inv);
          uint16_t a1 = f32_to_bf16_cvtne(__uint_as_float(o[k * 8 + 2 * i + 1]) * inv);
          if (p.gate_offset >= 0) {
            a0 = gate_bf16(a0, uint16_t(gw[i] & 0xFFFFu));
            a1 = gate_bf16(a1, uint16_t(gw[i] >> 16));
          }
          w[i] = uint32_t(a0) | (uint32_t(a1) << 16);
        }
        *reinterpret_cast<uint4*>(smem + OFF_V + phys) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    fence_proxy_async_smem();
    epilogue_sync();  // the output tile is staged
    if (threadIdx.x == 0 && ok && !*abort_flag) {
      for (int c = 0; c < 4; ++c)
        tma_store_2d(&tmO, smem + OFF_V + c * (BM * 128), h * HDIM + c * 64, m0);
      tma_store_commit();
      tma_store_wait_read();
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
  CUtensorMap tq, tk, tv, to;
  const int64_t kv_rows = L.cp ? L.kv_rows : L.past + L.rows;
  const cuuint64_t qd[2] = {cuuint64_t(L.q_row), cuuint64_t(L.rows)};
  const cuuint64_t qs[1] = {cuuint64_t(L.q_row) * 2};
  const cuuint32_t qbox[2] = {64, BM};
  const cuuint64_t kd[3] = {cuuint64_t(HDIM), cuuint64_t(kv_rows), cuuint64_t(L.hkv)};
  const cuuint64_t ks[2] = {cuuint64_t(HDIM) * 2, cuuint64_t(L.kv_stride) * 2};
  const cuuint32_t kbox[3] = {64, BN, 1};
  const cuuint64_t od[2] = {cuuint64_t(L.out_row), cuuint64_t(L.rows)};
  const cuuint64_t os[1] = {cuuint64_t(L.out_row) * 2};
  if (!encode_bf16(&tq, L.q, 2, qd, qs, qbox) || !encode_bf16(&tk, L.keys, 3, kd, ks, kbox) ||
      !encode_bf16(&tv, L.values, 3, kd, ks, kbox))
    return cudaErrorInvalidValue;
  if (L.cp) {
    to = tq;  // no output store on a hop
  } else if (!encode_bf16(&to, L.out, 2, od, os, qbox)) {
    return cudaErrorInvalidValue;
  }
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
    attn_prefill_kernel<true><<<grid, kThreads, SMEM_BYTES, st>>>(tq, tk, tv, to, p);
  else
    attn_prefill_kernel<false><<<grid, kThreads, SMEM_BYTES, st>>>(tq, tk, tv, to, p);
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
  return size_t(heads * nqt) * BM * (HDIM + 2) * sizeof(float);
}

cudaError_t launch_attn_cp_finish(const PrefillLaunch& L, cudaStream_t st) {
  const int nqt = int((L.rows + BM - 1) / BM);
  attn_cp_finish_kernel<<<unsigned(nqt * L.heads), 256, 0, st>>>(
      L.acc, L.q, L.out, L.q_row, L.out_row,
      L.gate_offset, int(L.rows), int(L.heads), nqt);
  return cudaGetLastError();
}

}  // namespace hb
