// attn_decode_mma.cu -- decode SDPA of one short sequence on the sm_100a
// tensor cores: every CTA of a thread-block cluster scores one tile of 128
// cached positions against the query heads of one GQA group with tcgen05,
// and the cluster merges the partials through distributed shared memory.
//
// Replaces, as the cluster form of attn_decode.cu does, the attention node
// in the decode regime (SdpaHeadFn, src/jit/emit_sdpa.rs:131-140, driven by
// src/jit/target/x86/execution/attention.rs:56-224) and the output-gate node
// (ElemOp::SigmoidMul, src/jit/target/x86/emit_elem.rs:333-420), for rows
// that see at most 16 x 128 positions, head_dim 256.
//
// Per CTA (tile t of KV head kh, query row `row`; 160 threads):
//   S^T = K_t Q^T        tcgen05 M128 N16 K256 into TMEM: lanes = positions,
//                        columns = heads (the group's G heads are the first G
//                        of the 16 rows of the B operand, the rest zero)
//   softmax              warps 0-3, one position per thread; each head's max
//                        and sum reduced over the tile's 128 positions
//   O^T = V_t^T P^T      tcgen05 M128 N16 K128 twice (dims 0-127, 128-255):
//                        V MN-major as the A operand, P^T (bf16) as B
// Each CTA stores its (m, l) and, to CTA r, the slice of its O partial that
// r merges into r's shared memory (DSMEM stores); after one cluster barrier
// CTA r merges output slice r from its own shared memory, divides by l,
// rounds to bf16 and applies the gate with the reference's steps.  Warp 4
// loads K and V by TMA (no multicast) and issues the MMAs (lane 0).
//
// Launched with programmatic dependent launch: before griddepcontrol.wait a
// CTA only prefetches its K/V tile and its q/gate lines into L2; every load
// that returns data and every store comes after the wait.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_front.cuh"
#include "hb_internal.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

using namespace sm100;

constexpr int BT = 128;        // positions per CTA
constexpr int HDM = 256;       // head dim
constexpr int NQ = 16;         // B-operand rows (query heads, padded)
constexpr int kThreadsM = 160; // warps 0-3 softmax / epilogue / merge, warp 4 TMA + MMA
constexpr int M_OFF_K = 0;                  // K tile: 4 blocks [128 positions][128 B]
constexpr int M_OFF_V = 65536;              // V tile: the same layout
constexpr int M_OFF_Q = 131072;             // Q^T: 4 blocks [16 rows][128 B]
constexpr int M_OFF_P = M_OFF_Q + 8192;     // P^T: 2 blocks [16 rows][128 B]
constexpr int M_OFF_PART = M_OFF_P + 4096;  // partial: O [G][256] f32, then m[G], l[G]
constexpr int M_PART_MAX = 8 * HDM * 4 + 64;
constexpr int M_OFF_RED = M_OFF_PART + M_PART_MAX;  // [2][4 warps][16] maxima, sums
constexpr int M_OFF_RML = M_OFF_RED + 2 * 4 * 16 * 4;  // [16 splits][16]: m[G], l[G] received
constexpr int M_OFF_RBUF = M_OFF_RML + 16 * 16 * 4;     // received output quads (<= 528 float4)
constexpr int M_OFF_BAR = M_OFF_RBUF + 528 * 16;
constexpr int M_SMEM = M_OFF_BAR + 128 + 1024;  // + alignment slack
constexpr uint32_t M_TMEM_COLS = 64;  // S^T [0, 16), O^T [16, 48)
// K_FULL and KB1..KB3: the K tile's four 64-dim column blocks, each on its
// own barrier so that the S products start as the first block lands
// O_DONE / O_DONE2: the two 128-dim halves of O^T
enum MBar { K_FULL = 0, V_FULL = 1, S_DONE = 2, O_DONE = 3, PEERS = 4, MERGE = 5, KB1 = 6, O_DONE2 = 9,
            M_NBAR = 10 };
HB_DEV constexpr int kblock_bar(int cb) { return cb == 0 ? int(K_FULL) : int(KB1) + cb - 1; }

struct DecodeMmaParams {
  const uint16_t* q;  // query rows (and gates)
  uint16_t* out;
  int64_t q_row, q_head, out_row;
  int64_t gate_offset;  // < 0: no gate
  int64_t past;         // row r sees past + r + 1 positions
  float scale_log2;
  int* status;
};

HB_DEV void nbar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// The warp's maximum in one instruction (sm_100a; NaN inputs are ignored
// unless all are NaN, as fmaxf does).
HB_DEV float warp_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}
HB_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
HB_DEV uint32_t dsmem_addr_m(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
// Stores into a peer's shared memory that count their bytes on the peer's
// mbarrier `bar` (complete_tx): the receiver waits on its own barrier.
HB_DEV void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(addr),
               "f"(v), "r"(bar)
               : "memory");
}
// Split cluster barrier: arrive early (this CTA has started), wait later.
HB_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
HB_DEV void cluster_wait_m() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// byte offset of element (row, col) in 128B-swizzled K-major blocks of
// [rows][64 columns], `block_bytes` apart
HB_DEV uint32_t swz(int row, int col, int block_bytes) {
  return uint32_t((col >> 6) * block_bytes + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                  (col & 7) * 2);
}

template <int G>
__global__ void __launch_bounds__(kThreadsM, 1)
    attn_decode_mma_kernel(const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const DecodeMmaParams p) {
  static_assert(G * HDM * 4 + 8 * G <= M_PART_MAX, "partial fits");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + M_OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + M_NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  float* cpart = reinterpret_cast<float*>(smem + M_OFF_PART);
  float* red_m = reinterpret_cast<float*>(smem + M_OFF_RED);  // [4][16]
  float* red_l = red_m + 64;                                   // [4][16]

  const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
  const int ns = int(gridDim.x);  // the cluster: every split of this (row, KV head)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int64_t n = p.past + row + 1;  // positions this row sees
  const int64_t p0 = int64_t(split) * BT;
  const bool has = p0 < n;  // the tile holds a position of the row (uniform)
  const int h0 = kh * G;
  const uint16_t* qrow = p.q + int64_t(row) * p.q_row;

  constexpr int Q4 = G * HDM / 4;       // output quads of the unit
  const int nqs = (Q4 + ns - 1) / ns;    // quads per slice (the last one may be short)
  if (tid == 0) {
    for (int i = 0; i < M_NBAR; ++i) mbar_init(&bar[i], 1);
    *abort_flag = 0;
    // the bytes every CTA of the cluster will store here: its (m, l) and
    // the quads of this CTA's output slice
    const int nq = max(0, min(nqs, Q4 - split * nqs));
    mbar_arrive_expect_tx(&bar[MERGE], uint32_t(ns) * uint32_t(2 * G * 4 + nq * 16));
    fence_mbar_init();
  }
  if (warp == 4) tmem_alloc(tslot, M_TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;
  griddep_launch_dependents();
  cluster_arrive_relaxed();  // warp 4 waits for the whole cluster (PEERS) before any peer store

  auto wait = [&](int b, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait(&bar[b], parity)) return true;
    record_status(p.status, kStatusTimeout);
    *abort_flag = 1;
    return false;
  };

  // warps 0-3: the gate divisor 1 + exp(-g) of the thread's first output in
  // this CTA's merge slice, by the reference's steps, formed early so that
  // the merge only divides
  float gdiv0 = 1.f;
  bool peers = false;  // warps 0-3: every CTA of the cluster has started (stores into peers allowed)
  if (warp == 4) {  // ------------------------------------------ TMA + MMA
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      if (has) {
        // this tile's K and V into L2 while the previous grid finishes
        tma_prefetch_l2_3d(&tmK, 0, int(p0), kh);
        tma_prefetch_l2_3d(&tmK, 64, int(p0), kh);
        tma_prefetch_l2_3d(&tmK, 128, int(p0), kh);
        tma_prefetch_l2_3d(&tmK, 192, int(p0), kh);
        tma_prefetch_l2_3d(&tmV, 0, int(p0), kh);
        tma_prefetch_l2_3d(&tmV, 64, int(p0), kh);
        tma_prefetch_l2_3d(&tmV, 128, int(p0), kh);
        tma_prefetch_l2_3d(&tmV, 192, int(p0), kh);
      }
      griddep_wait();
      if (has) {
        for (int cb = 0; cb < 4; ++cb) {
          mbar_arrive_expect_tx(&bar[kblock_bar(cb)], 16384);
          tma_load_3d(smem + M_OFF_K + cb * 16384, &tmK, &bar[kblock_bar(cb)], cb * 64, int(p0), kh);
        }
        mbar_arrive_expect_tx(&bar[V_FULL], 4 * 16384);
        for (int cb = 0; cb < 4; ++cb)
          tma_load_3d(smem + M_OFF_V + cb * 16384, &tmV, &bar[V_FULL], cb * 64, int(p0), kh);
      }
    }
    __syncwarp();
    nbar_sync(1, kThreadsM);  // Q^T written
    if (lane == 0 && has) {
      // S^T = K Q^T: M128 (positions) N16 (heads) K256, 16 MMAs of K16
      constexpr uint32_t idS = idesc_bf16(BT, NQ, false, false);
      const uint64_t kd0 = sw128_desc(smem_u32(smem + M_OFF_K), 16, 1024),
                     qd0 = sw128_desc(smem_u32(smem + M_OFF_Q), 16, 1024);
      bool kok = true;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {  // each column block's 4 products as soon as it lands
        if (!wait(kblock_bar(cb), 0)) {
          kok = false;
          break;
        }
        fence_after_sync();
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4)
          mma_bf16_ss(tmem, desc_add(kd0, cb * 16384 + k4 * 32), desc_add(qd0, cb * 2048 + k4 * 32),
                      idS, cb > 0 || k4 > 0);
      }
      if (kok) mma_commit(&bar[S_DONE]);
    }
    __syncwarp();
    // every CTA of the cluster has started and initialised its barriers:
    // the wait runs here, beside the softmax, and releases the stores into
    // the peers through PEERS
    cluster_wait_m();
    if (lane == 0) mbar_arrive(&bar[PEERS]);
    nbar_sync(3, kThreadsM);  // P^T written
    if (lane == 0 && has && !*abort_flag) {
      // O^T = V^T P^T: M128 (dims) N16 K128, V MN-major (64-dim blocks 16 KB
      // apart, 8-position groups 1 KB apart), for dims 0-127 and 128-255
      constexpr uint32_t idPV = idesc_bf16(BT, NQ, true, false);
      const uint64_t vd0 = sw128_desc(smem_u32(smem + M_OFF_V), 16384, 1024),
                     pd0 = sw128_desc(smem_u32(smem + M_OFF_P), 16, 1024);
      if (wait(V_FULL, 0)) {
        fence_after_sync();
#pragma unroll
        for (int mm = 0; mm < 2; ++mm) {  // each half committed on its own: its read-out starts early
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ss(tmem + NQ + NQ * mm, desc_add(vd0, 2 * mm * 16384 + kk * 2048),
                        desc_add(pd0, (kk >> 2) * 2048 + (kk & 3) * 32), idPV, kk > 0);
          mma_commit(&bar[mm == 0 ? O_DONE : O_DONE2]);
        }
      }
    }
    __syncwarp();
  } else {  // ----------------------------------- warps 0-3: q, softmax, partial
    // the group's q and gate lines into L2, then wait for the previous grid
    if (tid < G * 4) {
      const int g = tid >> 2, ln = tid & 3;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(
          reinterpret_cast<const char*>(qrow + int64_t(h0 + g) * p.q_head) + ln * 128));
      if (p.gate_offset >= 0)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(
            reinterpret_cast<const char*>(qrow + p.gate_offset + int64_t(h0 + g) * HDM) + ln * 128));
    }
    griddep_wait();
    {
      const int q0 = split * nqs, nq0 = max(0, min(nqs, Q4 - q0));
      if (p.gate_offset >= 0 && tid < 4 * nq0) {
        const int e = q0 * 4 + tid;
        gdiv0 = gate_divisor(qrow[p.gate_offset + int64_t(h0 + e / HDM) * HDM + e % HDM]);
      }
    }
    // Q^T: row h = tid / 8 (zero for h >= G), dims 32 (tid % 8) ..; and the
    // padding rows G..15 of P^T
    {
      const int h = tid >> 3, dg = tid & 7;
      uint4 v[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                    make_uint4(0, 0, 0, 0)};
      if (h < G) {
        const uint4* src = reinterpret_cast<const uint4*>(qrow + int64_t(h0 + h) * p.q_head + dg * 32);
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = src[c];
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(smem + M_OFF_Q + swz(h, dg * 32 + c * 8, 2048)) = v[c];
      // P^T rows G..15: 2 blocks x (16 - G) rows x 8 chunks
      for (int i = tid; i < 2 * (NQ - G) * 8; i += 128) {
        const int blk = i / ((NQ - G) * 8), rr = G + (i / 8) % (NQ - G), ch = i & 7;
        *reinterpret_cast<uint4*>(smem + M_OFF_P + blk * 2048 + rr * 128 + (ch << 4)) =
            make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
    }
    nbar_sync(1, kThreadsM);  // Q^T ready for the MMA

    // softmax over the tile's 128 positions, one per thread (TMEM lane)
    const int pl = warp * 32 + lane;  // position within the tile
    const bool valid = has && p0 + pl < n;
    float s[G];
    bool ok = true;
    if (has) {
      ok = __all_sync(0xFFFFFFFFu, wait(S_DONE, 0));
      fence_after_sync();
      uint32_t raw[16];
      tmem_ld16(tmem + (uint32_t(warp * 32) << 16), raw);
      tmem_wait_ld();
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = valid ? __uint_as_float(raw[g]) * p.scale_log2 : -INFINITY;
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = -INFINITY;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mx = warp_max(s[g]);
      if (lane == 0) red_m[warp * 16 + g] = mx;
    }
    nbar_sync(2, 128);
    float m[G], pr[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = fmaxf(fmaxf(red_m[g], red_m[16 + g]), fmaxf(red_m[32 + g], red_m[48 + g]));
      pr[g] = m[g] == -INFINITY ? 0.f : fast_exp2(s[g] - m[g]);  // masked: 2^-inf = 0
      // P^T element (head g, position pl), bf16
      const uint16_t b = uint16_t(pack_bf16x2(pr[g], 0.f) & 0xFFFFu);
      *reinterpret_cast<uint16_t*>(smem + M_OFF_P + swz(g, pl, 2048)) = b;
    }
    fence_proxy_async_smem();
    nbar_sync(3, kThreadsM);  // P^T ready for the MMA
    // the tile's maxima, and each warp's part of the sums (added by the
    // senders below, after the block barrier that completes the partial)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sm = warp_sum(pr[g]);
      if (lane == 0) red_l[warp * 16 + g] = sm;
      if (tid == g) cpart[G * HDM + g] = m[g];
    }

    // O^T out of TMEM (thread = dim 32 warp + lane, + 128 in the second
    // half; columns = heads), each element stored straight into the CTA of
    // the cluster that merges it (quads [s nqs, (s + 1) nqs) go to CTA s)
    peers = __all_sync(0xFFFFFFFFu, mbar_wait(&bar[PEERS], 0));
    if (!peers) {
      if (lane == 0) record_status(p.status, kStatusTimeout);
      *abort_flag = 1;
    }
    float* rbf = reinterpret_cast<float*>(smem + M_OFF_RBUF);  // receivers: [split][nqs quads]
#pragma unroll
    for (int mm = 0; mm < 2; ++mm) {
      uint32_t o[16];
      bool got = false;
      if (has) {
        ok = __all_sync(0xFFFFFFFFu, wait(mm == 0 ? O_DONE : O_DONE2, 0)) && ok;
        fence_after_sync();
        tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + NQ + NQ * mm, o);
        tmem_wait_ld();
        got = ok;
      }
      if (peers) {
        const int dim = mm * 128 + pl;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const int e = g * HDM + dim, r = (e >> 2) / nqs;
          st_async_f32(dsmem_addr_m(rbf + (split * nqs - r * nqs) * 4 + e, uint32_t(r)),
                       got ? __uint_as_float(o[g]) : 0.f, dsmem_addr_m(&bar[MERGE], uint32_t(r)));
        }
      }
    }
  }

  // ------------------------------------------------ merge across the cluster
  // Every CTA stores its (m, l) into every peer, and into CTA s the output
  // quads s merges (quads [s nqs, (s + 1) nqs)); after one cluster barrier
  // each CTA merges its slice from its own shared memory and nothing reads
  // a peer any more.
  float* rml = reinterpret_cast<float*>(smem + M_OFF_RML);      // [split][16]
  float4* rbuf = reinterpret_cast<float4*>(smem + M_OFF_RBUF);  // [split][nqs]
  if (warp < 4) {
    nbar_sync(2, 128);  // the tile's maxima and every warp's part of the sums are written
    if (peers) {
      for (int i = tid; i < ns * 2 * G; i += 128) {
        const int sp = i / (2 * G), k = i % (2 * G);
        const int g = k - G;  // k >= G: the sum of head g over the four warps
        const float v = k < G ? cpart[G * HDM + k]
                              : ((red_l[g] + red_l[16 + g]) + red_l[32 + g]) + red_l[48 + g];
        st_async_f32(dsmem_addr_m(rml + split * 16 + k, uint32_t(sp)), v,
                     dsmem_addr_m(&bar[MERGE], uint32_t(sp)));
      }
    }
    // every CTA's stores into this one have landed (counted in bytes)
    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bar[MERGE], 0))) {
      if (lane == 0) record_status(p.status, kStatusTimeout);
      *abort_flag = 1;
    }
  }
  if (warp < 4) {
    // one output element per thread: its head's maximum over the splits, the
    // weights 2^(m_r - M) and the merged sum formed by the thread itself (no
    // block barrier), the weighted sum of the splits, / l, bf16, and the gate
    // with the reference's steps (its divisor formed at the start)
    const int q0 = split * nqs, nq = max(0, min(nqs, Q4 - q0));
    uint16_t* orow = p.out + int64_t(row) * p.out_row;
    if (!*abort_flag) {
      const float* rf = reinterpret_cast<const float*>(rbuf);
      for (int t = tid; t < 4 * nq; t += 128) {
        const int e = q0 * 4 + t, g = e / HDM, dd = e % HDM;
        // every split's (m, l, value) read at once (ns <= 16 splits: the
        // cluster), the weights formed in parallel, then the sums in split
        // order
        float mr[16], lr[16], vr[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          mr[r] = r < ns ? rml[r * 16 + g] : -INFINITY;
          lr[r] = r < ns ? rml[r * 16 + G + g] : 0.f;
          vr[r] = r < ns ? rf[r * nqs * 4 + t] : 0.f;
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < 16; ++r) M = fmaxf(M, mr[r]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float w[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) w[r] = fast_exp2(mr[r] - Mu);
        float acc = 0.f, Ls = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r)
          if (r < ns) {
            Ls = fmaf(lr[r], w[r], Ls);
            acc = fmaf(w[r], vr[r], acc);
          }
        const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
        uint16_t a = f32_to_bf16_cvtne(acc * inv);
        if (p.gate_offset >= 0) {  // gate_bf16's steps, the divisor formed early
          const float d = t == tid ? gdiv0 : gate_divisor(qrow[p.gate_offset + int64_t(h0 + g) * HDM + dd]);
          a = f32_to_bf16_cvtne(__fdiv_rn(bf16_to_f32(a), d));
        }
        orow[int64_t(h0 + g) * HDM + dd] = a;
      }
    }
  }
  fence_before_sync();
  __syncthreads();  // every TMEM read of this CTA is done
  if (warp == 4) {
    fence_after_sync();
    tmem_dealloc(tmem, M_TMEM_COLS);
  }
}

// Largest cluster (16, else 8) that the device co-schedules for this
// kernel; 0 if none (probed once per device).
template <int G>
int mma_cluster_limit() {
  static int cache[64];
  static DeviceFlags probed;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  cudaError_t e = probed.once([&] {
    cudaError_t r = cudaFuncSetAttribute(attn_decode_mma_kernel<G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, M_SMEM);
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(attn_decode_mma_kernel<G>,
                               cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (r != cudaSuccess) return r;
    int best = 0;
    for (int c : {16, 8}) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(c, 1, 1);
      cfg.blockDim = dim3(kThreadsM);
      cfg.dynamicSmemBytes = M_SMEM;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = c;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int nc = 0;
      if (cudaOccupancyMaxActiveClusters(&nc, attn_decode_mma_kernel<G>, &cfg) == cudaSuccess &&
          nc >= 1) {
        best = c;
        break;
      }
      cudaGetLastError();  // a refused size is not an error of this call
    }
    cache[dev] = best;
    return cudaSuccess;
  });
  return e == cudaSuccess ? cache[dev] : 0;
}

template <int G>
cudaError_t launch_mma(const DecodeLaunch& L, int nsplit, cudaStream_t st) {
  CUtensorMap tk, tv;
  const int64_t kv_rows = L.one.past + L.rows;
  const cuuint64_t kd[3] = {cuuint64_t(HDM), cuuint64_t(kv_rows), cuuint64_t(L.hkv)};
  const cuuint64_t ks[2] = {cuuint64_t(HDM) * 2, cuuint64_t(L.one.kv_stride) * 2};
  const cuuint32_t box[3] = {64, BT, 1};
  if (!encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, L.one.keys, kd, ks, box,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, L.one.values, kd, ks, box,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  DecodeMmaParams p;
  p.q = L.one.q;
  p.out = L.one.output;
  p.q_row = L.q_row;
  p.q_head = L.q_head;
  p.out_row = L.out_row;
  p.gate_offset = L.gate_offset;
  p.past = L.one.past;
  p.scale_log2 = L.scale * 1.4426950408889634f;
  p.status = L.status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(nsplit), unsigned(L.hkv), unsigned(L.rows));
  cfg.blockDim = dim3(kThreadsM);
  cfg.dynamicSmemBytes = M_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = unsigned(nsplit);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, attn_decode_mma_kernel<G>, tk, tv, p);
}

// ----------------------------------------------- long sequences: split-KV
//
// One sequence beyond the cluster forms' reach: unit = (query row, KV head),
// split = `chunk` positions (a multiple of 128) of the unit, grid = (splits,
// KV heads, rows), about one CTA per SM.  A CTA loops over its 128-position
// tiles:
//   warp 4 (TMA)   K_t, V_t into a ring of three 64 KB slots (K_0 V_0 K_1 ...)
//   warp 5 (MMA)   S_t^T = K_t Q^T into S buffer t % 2, then O_{t-1}^T =
//                  V_{t-1}^T P_{t-1}^T into O buffer (t - 1) % 2: the scores of
//                  the next tile are in flight while the softmax of this one runs
//   warps 0-3      online softmax of tile t (one position per thread: the
//                  running max M and sum L per head, P_t^T in bf16 into P
//                  buffer t % 2), then O_{t-1} out of TMEM (one dim per
//                  thread, dims d and d + 128) folded into f32 registers with
//                  the correction 2^(M_acc - M_{t-1})
// The CTA's (O, M, L) partial goes to the workspace in the layout of the
// CUDA-core kernel's partials; the last CTA of the unit to arrive (atomic
// counter, reset after use) merges them, divides, rounds to bf16 and
// applies the gate with the reference's steps.  A unit with one split
// finalises directly.
//
// FRONT: a one-row call whose front end (head-norm-rope of q and k, the
// kv-append of the row's position) runs here instead of in attn_front.cu,
// with the same arithmetic (hb_front.cuh).  Warps 0-3 norm and rotate the
// group's q heads straight into the Q^T operand; the CTA whose split holds
// the row's position also norms and rotates the k head, writes k and v into
// the cache row (and k in place) and signals the TMA warp, which loads that
// tile only then; the CTA that finalises the unit (the last to arrive, when
// every other CTA has read q) writes the normed q back in place.

constexpr int kThreadsL = 192;               // warps 0-3 softmax, 4 TMA, 5 MMA
constexpr int L_SLOT = 65536;                // one K or V tile: 4 blocks [128][128 B]
constexpr int L_OFF_Q = 3 * L_SLOT;          // Q^T: 4 blocks [16 rows][128 B]
constexpr int L_OFF_P = L_OFF_Q + 8192;      // P^T: 2 buffers x 2 blocks [16][128 B]
constexpr int L_OFF_RED = L_OFF_P + 8192;    // maxima [2][4 warps][16], then sums [2][4][16]
constexpr int L_OFF_XS = L_OFF_RED + 2 * 2 * 4 * 16 * 4;  // FRONT: 4 warps x 512 B norm scratch
constexpr int L_OFF_BAR = L_OFF_XS + 4 * 512;
constexpr int L_SMEM = L_OFF_BAR + 256 + 1024;  // + alignment slack
constexpr uint32_t L_TMEM_COLS = 128;        // S^T 2 x 16 columns, O^T 2 x 32
enum LBar { L_FULL = 0, L_EMPTY = 3, L_S_FULL = 6, L_S_FREE = 8, L_P_READY = 10, L_O_FULL = 12,
            L_O_FREE = 14, L_MERGE = 16, L_KV = 17, L_NBAR = 18 };

struct DecodeLongParams {
  const uint16_t* q;
  uint16_t* out;
  int64_t q_row, q_head, out_row;
  int64_t gate_offset;  // < 0: no gate
  int64_t past;         // row r sees past + r + 1 positions
  int hkv, chunk, nsplit;
  float scale_log2;
  int* status;
  unsigned* counters;   // one per unit
  int spread;           // every CTA of the grid resident at once: the last G CTAs of a unit merge it
  float* partials;      // [unit][split][G*HD + 2G rounded up to 4]
  // FRONT (rows == 1): the row's k and v ([hkv][256] each; k normed and
  // rotated in place), the norm weights, the RoPE table, the cache
  uint16_t* kf;
  const uint16_t* vf;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const uint16_t* cos;
  const uint16_t* sin;
  uint16_t* kcache;  // KV head 0 of the layer's K cache, heads kv_stride apart
  uint16_t* vcache;
  int64_t kv_stride;
  int rotary, gemma;
  float eps, inv_dim;
};

template <int G, bool FRONT>
__global__ void __launch_bounds__(kThreadsL, 1)
    attn_decode_long_kernel(const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const DecodeLongParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L_OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + L_NBAR);
  volatile int* flags = reinterpret_cast<volatile int*>(tslot + 1);  // [0] abort, [1] last
  float* red = reinterpret_cast<float*>(smem + L_OFF_RED);

  const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int64_t n = p.past + row + 1;  // positions this row sees
  const int64_t p0 = int64_t(split) * p.chunk;
  if (p0 >= n) return;  // beyond the row's last split: not counted
  const int64_t p1 = min(n, p0 + p.chunk);
  const int nt = int((p1 - p0 + BT - 1) / BT);
  const int active = int((n + p.chunk - 1) / p.chunk);
  const int unit = row * p.hkv + kh;
  const int h0 = kh * G;
  const uint16_t* qrow = p.q + int64_t(row) * p.q_row;
  // FRONT: this CTA's split holds the row's own position (rows == 1)
  const bool tail = FRONT && p.past >= p0 && p.past < p1;

  if (tid == 0) {
    for (int i = 0; i < L_NBAR; ++i) {
      // the S_FREE, P_READY and O_FREE barriers count the four softmax warps
      const bool four = (i >= L_S_FREE && i < L_S_FREE + 2) || (i >= L_P_READY && i < L_P_READY + 2) ||
                        (i >= L_O_FREE && i < L_O_FREE + 2);
      mbar_init(&bar[i], four ? 4u : 1u);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_mbar_init();
  }
  if (warp == 5) tmem_alloc(tslot, L_TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;
  griddep_launch_dependents();

  auto wait = [&](int b, uint32_t parity) -> bool {
    if (flags[0]) return false;
    if (mbar_wait(&bar[b], parity)) return true;
    record_status(p.status, kStatusTimeout);
    flags[0] = 1;
    return false;
  };

  if (warp == 4) {  // ------------------------------------------------- TMA
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      // K and V are read once per step: their lines are the first L2 evicts,
      // so a sweep of the cache leaves other layers' data (a DeltaNet
      // layer's state, the next step's inputs) in L2
      const uint64_t once = l2_evict_first();
      // the first tiles into L2 while the previous grid finishes
      for (int t = 0; t < nt && t < 2; ++t)
        for (int cb = 0; cb < 4; ++cb) {
          tma_prefetch_l2_3d_hint(&tmK, cb * 64, int(p0) + t * BT, kh, once);
          tma_prefetch_l2_3d_hint(&tmV, cb * 64, int(p0) + t * BT, kh, once);
        }
      griddep_wait();
      const int t_tail = tail ? int((p.past - p0) / BT) : -1;
      int issued = 0;
      for (int i = 0; i < 2 * nt; ++i) {
        const int s = i % 3;
        if (i >= 3 && !wait(L_EMPTY + s, ((i / 3) - 1) & 1)) break;
        // the tile of the row's position once its k and v are in the cache
        if (i == 2 * t_tail && !wait(L_KV, 0)) break;
        const int pos = int(p0) + (i >> 1) * BT;
        const CUtensorMap* tm = (i & 1) ? &tmV : &tmK;
        mbar_arrive_expect_tx(&bar[L_FULL + s], 4 * 16384);
        for (int cb = 0; cb < 4; ++cb)
          tma_load_3d_hint(smem + s * L_SLOT + cb * 16384, tm, &bar[L_FULL + s], cb * 64, pos, kh, once);
        issued = i + 1;
      }
      // every copy into this CTA's shared memory lands before it ends: the
      // last three (earlier slots were consumed before their reuse)
      for (int i = max(0, issued - 3); i < issued; ++i) mbar_wait(&bar[L_FULL + i % 3], (i / 3) & 1);
    }
    __syncwarp();
  } else if (warp == 5) {  // ------------------------------------------- MMA
    nbar_sync(1, 128 + 32);  // Q^T written by warps 0-3
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(BT, NQ, false, false);
      constexpr uint32_t idPV = idesc_bf16(BT, NQ, true, false);
      const uint64_t qd0 = sw128_desc(smem_u32(smem + L_OFF_Q), 16, 1024);
      bool ok = true;
      // iteration t: the scores of tile t (t < nt), then O of tile t - 1
      for (int t = 0; t <= nt && ok; ++t) {
        if (t < nt) {
          const int s = (2 * t) % 3;
          if (!(wait(L_FULL + s, ((2 * t) / 3) & 1) &&
                (t < 2 || wait(L_S_FREE + (t & 1), ((t - 2) >> 1) & 1)))) {
            ok = false;
            break;
          }
          fence_after_sync();
          const uint64_t kd0 = sw128_desc(smem_u32(smem + s * L_SLOT), 16, 1024);
#pragma unroll
          for (int cb = 0; cb < 4; ++cb)
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              mma_bf16_ss(tmem + (t & 1) * 16, desc_add(kd0, cb * 16384 + k4 * 32),
                          desc_add(qd0, cb * 2048 + k4 * 32), idS, cb > 0 || k4 > 0);
          mma_commit(&bar[L_S_FULL + (t & 1)]);
          mma_commit(&bar[L_EMPTY + s]);
        }
        if (t >= 1) {
          const int j = t - 1, s = (2 * j + 1) % 3;
          if (!(wait(L_FULL + s, ((2 * j + 1) / 3) & 1) && wait(L_P_READY + (j & 1), (j >> 1) & 1) &&
                (j < 2 || wait(L_O_FREE + (j & 1), ((j - 2) >> 1) & 1)))) {
            ok = false;
            break;
          }
          fence_after_sync();
          // O^T = V^T P^T: M128 (dims) N16 K128, V MN-major (64-dim blocks
          // 16 KB apart, 8-position groups 1 KB apart), dims 0-127 and 128-255
          const uint64_t vd0 = sw128_desc(smem_u32(smem + s * L_SLOT), 16384, 1024),
                         pd0 = sw128_desc(smem_u32(smem + L_OFF_P + (j & 1) * 4096), 16, 1024);
          const uint32_t od = tmem + 32 + (j & 1) * 32;
#pragma unroll
          for (int mm = 0; mm < 2; ++mm)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_bf16_ss(od + NQ * mm, desc_add(vd0, 2 * mm * 16384 + kk * 2048),
                          desc_add(pd0, (kk >> 2) * 2048 + (kk & 3) * 32), idPV, kk > 0);
          mma_commit(&bar[L_O_FULL + (j & 1)]);
          mma_commit(&bar[L_EMPTY + s]);
        }
      }
    }
    __syncwarp();
  } else {  // ---------------------------------------------- warps 0-3
    if (tid < G * 4) {
      const int g = tid >> 2, ln = tid & 3;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(
          reinterpret_cast<const char*>(qrow + int64_t(h0 + g) * p.q_head) + ln * 128));
    }
    griddep_wait();
    constexpr int QW = (G + 3) / 4;  // q heads per warp (FRONT)
    uint32_t qy[QW][4];              // FRONT: this warp's normed q heads, for the write-back
    if constexpr (FRONT) {
      // head-norm-rope of the group's q heads (warp w: heads w, w + 4) into
      // Q^T, and for the position's split the k head and the kv-append
      const int64_t pos = p.past;
      uint32_t* xs = reinterpret_cast<uint32_t*>(smem + L_OFF_XS) + warp * 128;
      uint32_t cw[4] = {0u, 0u, 0u, 0u}, sw[4] = {0u, 0u, 0u, 0u}, ww[4];
      const int half = p.rotary / 2;
      if (lane * 8 < p.rotary) {
        const int j0 = lane * 8 < half ? lane * 8 : lane * 8 - half;
        front::load_words<4>(cw, p.cos + pos * half + j0);
        front::load_words<4>(sw, p.sin + pos * half + j0);
      }
      front::load_words<4>(ww, p.q_norm + lane * 8);
#pragma unroll
      for (int i = 0; i < QW; ++i) {
        const int hh = warp + 4 * i;
        if (hh < G) {  // warp-uniform
          uint32_t xw[4];
          front::load_words<4>(xw, qrow + int64_t(h0 + hh) * p.q_head + lane * 8);
          front::norm_rope<HDM>(xw, ww, cw, sw, p.rotary, p.eps, p.inv_dim, p.gemma != 0, xs, lane, qy[i]);
          *reinterpret_cast<uint4*>(smem + L_OFF_Q + swz(hh, lane * 8, 2048)) =
              make_uint4(qy[i][0], qy[i][1], qy[i][2], qy[i][3]);
        }
      }
      for (int i = tid; i < (NQ - G) * 32; i += 128)
        *reinterpret_cast<uint4*>(smem + L_OFF_Q + swz(G + i / 32, (i % 32) * 8, 2048)) =
            make_uint4(0, 0, 0, 0);
      if (tail && warp == 0) {
        uint32_t kw[4], knw[4], vw[4], ky[4];
        uint16_t* krow = p.kf + int64_t(kh) * HDM + lane * 8;
        front::load_words<4>(kw, krow);
        front::load_words<4>(knw, p.k_norm + lane * 8);
        front::load_words<4>(vw, p.vf + int64_t(kh) * HDM + lane * 8);
        front::norm_rope<HDM>(kw, knw, cw, sw, p.rotary, p.eps, p.inv_dim, p.gemma != 0, xs, lane, ky);
        const int64_t dst = int64_t(kh) * p.kv_stride + pos * HDM + lane * 8;
        front::store_words<4>(p.kcache + dst, ky);
        front::store_words<4>(p.vcache + dst, vw);
        front::store_words<4>(krow, ky);
        // the cache row before the TMA warp's loads of its tile
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[L_KV]);
      }
    } else {  // Q^T rows (zero for h >= G)
      const int h = tid >> 3, dg = tid & 7;
      uint4 v[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                    make_uint4(0, 0, 0, 0)};
      if (h < G) {
        const uint4* src = reinterpret_cast<const uint4*>(qrow + int64_t(h0 + h) * p.q_head + dg * 32);
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = src[c];
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(smem + L_OFF_Q + swz(h, dg * 32 + c * 8, 2048)) = v[c];
    }
    {  // the zero rows G..15 of both P^T buffers
      for (int i = tid; i < 4 * (NQ - G) * 8; i += 128) {
        const int blk = i / ((NQ - G) * 8), rr = G + (i / 8) % (NQ - G), ch = i & 7;
        *reinterpret_cast<uint4*>(smem + L_OFF_P + blk * 2048 + rr * 128 + (ch << 4)) =
            make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
    }
    nbar_sync(1, 128 + 32);  // Q^T ready for the MMA warp

    const int pl = warp * 32 + lane;  // position in the tile; dim pl (and pl + 128) of O
    // Mt0 / Mt1: M after the last even / odd tile
    float M[G], Lsum[G], Macc[G], Mt0[G], Mt1[G], o[2][G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      M[g] = -INFINITY;
      Lsum[g] = 0.f;
      Macc[g] = -INFINITY;
      o[0][g] = 0.f;
      o[1][g] = 0.f;
      Mt0[g] = Mt1[g] = -INFINITY;
    }
    bool ok = true;
    // iteration t: the softmax of tile t (t < nt), then O of tile t - 1
    for (int t = 0; t <= nt; ++t) {
      const int b = t & 1;
      if (t < nt) {
        float sc[G];
        {
          const bool got = __all_sync(0xFFFFFFFFu, wait(L_S_FULL + b, (t >> 1) & 1));
          ok = ok && got;
          fence_after_sync();
          uint32_t raw[16];
          tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + b * 16, raw);
          tmem_wait_ld();
          fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar[L_S_FREE + b]);
          const bool valid = got && p0 + int64_t(t) * BT + pl < p1;
#pragma unroll
          for (int g = 0; g < G; ++g) sc[g] = valid ? __uint_as_float(raw[g]) * p.scale_log2 : -INFINITY;
        }
        float* rm = red + b * 64;        // [4 warps][16] maxima of tile parity b
        float* rl = red + 128 + b * 64;  // and sums
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float mx = warp_max(sc[g]);
          if (lane == 0) rm[warp * 16 + g] = mx;
        }
        nbar_sync(2, 128);
        uint8_t* pbuf = smem + L_OFF_P + b * 4096;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float tm = fmaxf(fmaxf(rm[g], rm[16 + g]), fmaxf(rm[32 + g], rm[48 + g]));
          const float mn = fmaxf(M[g], tm);
          const float pr = mn == -INFINITY ? 0.f : fast_exp2(sc[g] - mn);
          const float sm = warp_sum(pr);
          if (lane == 0) rl[warp * 16 + g] = sm;
          *reinterpret_cast<uint16_t*>(pbuf + swz(g, pl, 2048)) = uint16_t(pack_bf16x2(pr, 0.f) & 0xFFFFu);
          const float corr = M[g] == -INFINITY ? 0.f : fast_exp2(M[g] - mn);
          Lsum[g] *= corr;  // the tile's sum is added below
          M[g] = mn;
          if (b) Mt1[g] = mn; else Mt0[g] = mn;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[L_P_READY + b]);
        nbar_sync(2, 128);
#pragma unroll
        for (int g = 0; g < G; ++g) Lsum[g] += ((rl[g] + rl[16 + g]) + rl[32 + g]) + rl[48 + g];
      }
      if (t >= 1) {  // O of tile j = t - 1 out of TMEM, folded into the registers
        const int j = t - 1;
        const bool got = __all_sync(0xFFFFFFFFu, wait(L_O_FULL + (j & 1), (j >> 1) & 1));
        ok = ok && got;
        fence_after_sync();
        uint32_t r0[16], r1[16];
        const uint32_t base = tmem + (uint32_t(warp * 32) << 16) + 32 + (j & 1) * 32;
        tmem_ld16(base, r0);
        tmem_ld16(base + NQ, r1);
        tmem_wait_ld();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[L_O_FREE + (j & 1)]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float mj = (j & 1) ? Mt1[g] : Mt0[g];
          const float c = Macc[g] == -INFINITY ? 0.f : fast_exp2(Macc[g] - mj);
          o[0][g] = fmaf(o[0][g], c, got ? __uint_as_float(r0[g]) : 0.f);
          o[1][g] = fmaf(o[1][g], c, got ? __uint_as_float(r1[g]) : 0.f);
          Macc[g] = mj;
        }
      }
    }
    if (!ok && lane == 0) flags[0] = 1;

    // ------------------------------------------------ partial or finalise
    uint16_t* orow = p.out + int64_t(row) * p.out_row;
    if (active == 1) {
      if (!flags[0]) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float inv = Lsum[g] > 0.f ? 1.f / Lsum[g] : 0.f;
#pragma unroll
          for (int mm = 0; mm < 2; ++mm) {
            const int dd = mm * 128 + pl;
            uint16_t a = f32_to_bf16_cvtne(o[mm][g] * inv);
            if (p.gate_offset >= 0) a = gate_bf16(a, qrow[p.gate_offset + int64_t(h0 + g) * HDM + dd]);
            orow[int64_t(h0 + g) * HDM + dd] = a;
          }
        }
      }
      if constexpr (FRONT) {  // the only CTA of the unit: the normed q back in place
#pragma unroll
        for (int i = 0; i < QW; ++i)
          if (warp + 4 * i < G)
            front::store_words<4>(const_cast<uint16_t*>(qrow) + int64_t(h0 + warp + 4 * i) * p.q_head + lane * 8, qy[i]);
      }
    } else {
      // the partial, head-major: O rows at [unit][head][split][HD] (a head's
      // rows of every split contiguous, one bulk copy for a merger), the
      // maxima and sums at [unit][split][2G] after all the O rows
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float* orow_p = p.partials + ((int64_t(unit) * G + g) * p.nsplit + split) * HDM;
        __stcg(orow_p + pl, o[0][g]);
        __stcg(orow_p + 128 + pl, o[1][g]);
      }
      float* ml = p.partials + int64_t(gridDim.y) * gridDim.z * G * p.nsplit * HDM +
                  (int64_t(unit) * p.nsplit + split) * 2 * G;
#pragma unroll
      for (int g = 0; g < G; ++g)
        if (tid == g) {
          __stcg(ml + g, M[g]);
          __stcg(ml + G + g, Lsum[g]);
        }
      nbar_sync(2, 128);  // every partial store of this CTA precedes thread 0's release
      // The last K CTAs of the unit to count themselves merge it, one slice
      // of K of its G heads each (K = G when the launch spreads the merge:
      // every CTA of the grid resident at once; else K = 1, the last CTA
      // merges every head).  A merger that is not the last waits until
      // every split has counted itself, then adds itself once more; the one
      // that brings the count to active + K resets it for the next call.
      const int K = (p.spread && active >= G) ? G : 1;
      if (tid == 0) {
        // acquire-release at gpu scope: the CTA's partial (ordered before
        // this thread by the block barrier) is visible to whoever reads the
        // count after it, and this CTA sees every partial counted before
        unsigned prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(prev) : "l"(p.counters + unit) : "memory");
        const int mi = int(prev) - (active - K);
        flags[1] = mi >= 0 ? mi : -1;
        if (mi >= 0 && mi < K - 1) {  // wait for the splits after this one
          const long long t0 = clock64();
          unsigned c;
          for (;;) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(c) : "l"(p.counters + unit) : "memory");
            if (c >= unsigned(active)) break;
            if (clock64() - t0 > kSpinCycles) {
              record_status(p.status, kStatusTimeout);
              flags[0] = 1;
              break;
            }
          }
        }
      }
      nbar_sync(2, 128);
      const int mi = flags[1];
      if (mi >= 0) {
        // This CTA's heads [g0, g0 + GM).  Their splits' maxima and sums
        // first (one warp per head, lanes across the splits: the weights
        // 2^(m_s - M) and the merged sum), then the heads' O partials come
        // into the idle ring by bulk copies, as many splits at a time as it
        // holds, all of a batch in flight on one barrier, and each thread
        // sums its output quads from shared memory.
        const int GM = G / K, g0 = mi * GM;
        constexpr int QPT = (G * HDM / 4 + 127) / 128;
        const int NQD = GM * HDM / 4;  // output quads of this CTA's heads
        // the gate divisors 1 + exp(-g) of this thread's output quads, formed
        // while the partials come in: the gate's read is off the merge's tail
        float gd[QPT][4];
#pragma unroll
        for (int k = 0; k < QPT; ++k) {
          const int qd = tid + k * 128;
          gd[k][0] = gd[k][1] = gd[k][2] = gd[k][3] = 1.f;
          if (qd < NQD && p.gate_offset >= 0) {
            const int e = g0 * HDM + qd * 4, hq = h0 + e / HDM, dd = e % HDM;
            const uint2 gw = *reinterpret_cast<const uint2*>(qrow + p.gate_offset + int64_t(hq) * HDM + dd);
            gd[k][0] = gate_divisor(uint16_t(gw.x & 0xFFFFu));
            gd[k][1] = gate_divisor(uint16_t(gw.x >> 16));
            gd[k][2] = gate_divisor(uint16_t(gw.y & 0xFFFFu));
            gd[k][3] = gate_divisor(uint16_t(gw.y >> 16));
          }
        }
        const float* uo = p.partials + int64_t(unit) * G * p.nsplit * HDM;  // [head][split][HD]
        const float* uml = p.partials + int64_t(gridDim.y) * gridDim.z * G * p.nsplit * HDM +
                           int64_t(unit) * p.nsplit * 2 * G;  // [split][2G]
        float* sml = reinterpret_cast<float*>(smem + L_OFF_Q);  // [active][2G] m, l (Q^T, P^T are done)
        float* smw = sml + active * 2 * G;                      // [active][G] weights
        float* smL = reinterpret_cast<float*>(smem + L_OFF_RED);  // [G]
        const int ROW = GM * HDM * 4;                           // bytes of the heads' O in one split
        const int BATCH = 3 * L_SLOT / ROW;  // splits per batch; in shared memory [head][split][HD]
        const bool staged = active * 3 * G * 4 <= 16384;        // m, l and weights fit Q^T + P^T
        auto issue = [&](int b0) {  // warp 0: the heads' O rows of splits b0 .. b0 + BATCH - 1
          const int nb = min(BATCH, active - b0);
          if (lane == 0) mbar_arrive_expect_tx(&bar[L_MERGE], uint32_t(nb) * ROW);
          __syncwarp();
          if (lane < GM)  // one copy per head: its nb rows are contiguous
            bulk_g2s(smem + lane * nb * HDM * 4, uo + (int64_t(g0 + lane) * p.nsplit + b0) * HDM,
                     uint32_t(nb) * HDM * 4, &bar[L_MERGE]);
        };
        if (staged && !flags[0]) {
          if (warp == 0) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            issue(0);  // in flight while the weights are formed
          }
          for (int i = tid; i < active * 2 * G; i += 128)
            sml[i] = __ldcg(uml + i);
          nbar_sync(2, 128);
          for (int g = g0 + warp; g < g0 + GM; g += 4) {
            float Mx = -INFINITY;
            for (int sp = lane; sp < active; sp += 32) Mx = fmaxf(Mx, sml[sp * 2 * G + g]);
            Mx = warp_max(Mx);
            const float Mu = Mx == -INFINITY ? 0.f : Mx;
            float Ls = 0.f;
            for (int sp = lane; sp < active; sp += 32) {
              const float w = fast_exp2(sml[sp * 2 * G + g] - Mu);
              smw[sp * G + g] = w;
              Ls = fmaf(sml[sp * 2 * G + G + g], w, Ls);
            }
            Ls = warp_sum(Ls);
            if (lane == 0) smL[g] = Ls;
          }
        }
        nbar_sync(2, 128);
        float4 acc[QPT];
#pragma unroll
        for (int k = 0; k < QPT; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (staged && !flags[0]) {
          for (int b0 = 0, it = 0; b0 < active; b0 += BATCH, ++it) {
            const int nb = min(BATCH, active - b0);
            if (it > 0 && warp == 0) issue(b0);
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bar[L_MERGE], it & 1))) {
              if (tid == 0) {
                record_status(p.status, kStatusTimeout);
                mbar_wait(&bar[L_MERGE], it & 1);  // a second bounded wait for the copies in flight
              }
              flags[0] = 1;
            }
            if (!flags[0]) {
#pragma unroll
              for (int k = 0; k < QPT; ++k) {
                const int qd = tid + k * 128;
                if (qd < NQD) {
                  const int gh = qd * 4 / HDM, g = g0 + gh, dq = (qd * 4) % HDM;
                  const float4* hv = reinterpret_cast<const float4*>(smem + gh * nb * HDM * 4) + dq / 4;
                  for (int i = 0; i < nb; ++i) {
                    const float4 v = hv[i * (HDM / 4)];
                    const float w = smw[(b0 + i) * G + g];
                    acc[k].x = fmaf(w, v.x, acc[k].x);
                    acc[k].y = fmaf(w, v.y, acc[k].y);
                    acc[k].z = fmaf(w, v.z, acc[k].z);
                    acc[k].w = fmaf(w, v.w, acc[k].w);
                  }
                }
              }
            }
            nbar_sync(2, 128);  // the batch is summed: its buffers may take the next
            if (flags[0]) break;
          }
        } else if (tid == 0 && !staged) {
          // more splits than the weight buffer holds: the launcher does not
          // send such calls here
          record_status(p.status, kStatusArg);
        }
#pragma unroll
        for (int k = 0; k < QPT; ++k) {
          const int qd = tid + k * 128;
          if (qd >= NQD || flags[0] || !staged) continue;
          const int e = g0 * HDM + qd * 4, g = e / HDM, dd = e % HDM, hq = h0 + g;
          const float Ls = smL[g];
          const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
          uint16_t a[4] = {f32_to_bf16_cvtne(acc[k].x * inv), f32_to_bf16_cvtne(acc[k].y * inv),
                           f32_to_bf16_cvtne(acc[k].z * inv), f32_to_bf16_cvtne(acc[k].w * inv)};
          if (p.gate_offset >= 0) {  // gate_bf16's steps, the divisors formed early
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = f32_to_bf16_cvtne(__fdiv_rn(bf16_to_f32(a[i]), gd[k][i]));
          }
          *reinterpret_cast<uint2*>(orow + int64_t(hq) * HDM + dd) =
              make_uint2(uint32_t(a[0]) | (uint32_t(a[1]) << 16), uint32_t(a[2]) | (uint32_t(a[3]) << 16));
        }
        if constexpr (FRONT) {  // every other CTA of the unit has read q: the normed q in place
          if (mi == 0) {
#pragma unroll
            for (int i = 0; i < QW; ++i)
              if (warp + 4 * i < G)
                front::store_words<4>(const_cast<uint16_t*>(qrow) + int64_t(h0 + warp + 4 * i) * p.q_head + lane * 8, qy[i]);
          }
        }
        // leave the workspace reusable: the merger that completes the
        // second count (every merger is past its wait) resets it
        if (tid == 0) {
          __threadfence();
          const unsigned prev = atomicAdd(&p.counters[unit], 1u);
          if (prev == unsigned(active + K - 1)) p.counters[unit] = 0u;
        }
      }
    }
  }
  fence_before_sync();
  __syncthreads();  // every TMEM read and every MMA of this CTA is done
  if (warp == 5) {
    fence_after_sync();
    tmem_dealloc(tmem, L_TMEM_COLS);
  }
}

}  // namespace

bool launch_attn_decode_mma(const DecodeLaunch& L, cudaStream_t st, cudaError_t* err) {
  if (L.seqs != nullptr || L.nseq != 1 || L.head_dim != HDM) return false;
  if ((reinterpret_cast<uintptr_t>(L.one.q) | reinterpret_cast<uintptr_t>(L.one.keys) |
       reinterpret_cast<uintptr_t>(L.one.values) | reinterpret_cast<uintptr_t>(L.one.output)) & 15)
    return false;
  const int64_t max_n = L.one.past + L.rows;
  const int nsplit = int((max_n + BT - 1) / BT);
  if (nsplit < 2) return false;  // one tile: the CUDA-core kernel needs no merge
#define HB_MMA_CASE(G_)                                                      \
  if (L.gqa == G_) {                                                         \
    const int cmax = mma_cluster_limit<G_>();                                \
    if (nsplit > cmax) return false;                                         \
    *err = launch_mma<G_>(L, nsplit, st);                                    \
    return true;                                                             \
  }
  HB_MMA_CASE(1) HB_MMA_CASE(2) HB_MMA_CASE(4) HB_MMA_CASE(8)
#undef HB_MMA_CASE
  return false;
}

namespace {
template <int G, bool FRONT>
cudaError_t launch_long(const DecodeLaunch& L, const DecodeFront* F, int chunk, int nsplit,
                        cudaStream_t st) {
  static DeviceFlags configured;
  cudaError_t e = configured.once([] {
    return cudaFuncSetAttribute(attn_decode_long_kernel<G, FRONT>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, L_SMEM);
  });
  if (e != cudaSuccess) return e;
  CUtensorMap tk, tv;
  const int64_t kv_rows = L.one.past + L.rows;
  const cuuint64_t kd[3] = {cuuint64_t(HDM), cuuint64_t(kv_rows), cuuint64_t(L.hkv)};
  const cuuint64_t ks[2] = {cuuint64_t(HDM) * 2, cuuint64_t(L.one.kv_stride) * 2};
  const cuuint32_t box[3] = {64, BT, 1};
  if (!encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, L.one.keys, kd, ks, box,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, L.one.values, kd, ks, box,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  DecodeLongParams p;
  p.q = L.one.q;
  p.out = L.one.output;
  p.q_row = L.q_row;
  p.q_head = L.q_head;
  p.out_row = L.out_row;
  p.gate_offset = L.gate_offset;
  p.past = L.one.past;
  p.hkv = int(L.hkv);
  p.chunk = chunk;
  p.nsplit = nsplit;
  p.scale_log2 = L.scale * 1.4426950408889634f;
  p.status = L.status;
  p.counters = L.counters;
  p.partials = L.partials;
  p.kf = F ? F->k : nullptr;
  p.vf = F ? F->v : nullptr;
  p.q_norm = F ? F->q_norm : nullptr;
  p.k_norm = F ? F->k_norm : nullptr;
  p.cos = F ? F->cos : nullptr;
  p.sin = F ? F->sin : nullptr;
  p.kcache = const_cast<uint16_t*>(L.one.keys);
  p.vcache = const_cast<uint16_t*>(L.one.values);
  p.kv_stride = L.one.kv_stride;
  p.rotary = F ? int(F->rotary) : 0;
  p.gemma = F && F->gemma ? 1 : 0;
  p.eps = F ? F->eps : 0.f;
  p.inv_dim = 1.0f / float(HDM);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(nsplit), unsigned(L.hkv), unsigned(L.rows));
  cfg.blockDim = dim3(kThreadsL);
  // one CTA per SM (its shared memory): the merge waits on other CTAs only
  // when every CTA of the grid can be resident at once
  p.spread = int64_t(nsplit) * L.hkv * L.rows <= device_sms() ? 1 : 0;
  cfg.dynamicSmemBytes = L_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_decode_long_kernel<G, FRONT>, tk, tv, p);
}
}  // namespace

bool launch_attn_decode_long(const DecodeLaunch& L, cudaStream_t st, cudaError_t* err,
                             const DecodeFront* front) {
  if (L.seqs != nullptr || L.nseq != 1 || L.head_dim != HDM) return false;
  if (front && (L.rows != 1 || front->rotary < 0 || front->rotary % 32 != 0 || front->rotary > HDM))
    return false;
  if ((reinterpret_cast<uintptr_t>(L.one.q) | reinterpret_cast<uintptr_t>(L.one.keys) |
       reinterpret_cast<uintptr_t>(L.one.values) | reinterpret_cast<uintptr_t>(L.one.output)) & 15)
    return false;
  // beyond the reach of the cluster forms (16 splits of <= 256 positions);
  // splits of whole tiles, no more of them than the plan's workspace holds
  const int64_t max_n = L.one.past + L.rows;
  if (max_n <= 16 * 256) return false;
  const int64_t chunk = (int64_t(L.chunk) + BT - 1) / BT * BT;
  const int64_t nsplit = (max_n + chunk - 1) / chunk;
  if (chunk > (int64_t(1) << 30) || nsplit > L.nsplit || max_n + BT > (int64_t(1) << 31)) return false;
  // the merge keeps the splits' maxima, sums and weights in 16 KB of shared memory
  if (nsplit * L.gqa * 12 > 16384) return false;
#define HB_LONG_CASE(G_)                                                                      \
  if (L.gqa == G_) {                                                                          \
    *err = front ? launch_long<G_, true>(L, front, int(chunk), int(nsplit), st)               \
                 : launch_long<G_, false>(L, nullptr, int(chunk), int(nsplit), st);           \
    return true;                                                                              \
  }
  HB_LONG_CASE(1) HB_LONG_CASE(2) HB_LONG_CASE(4) HB_LONG_CASE(8)
#undef HB_LONG_CASE
  return false;
}

}  // namespace hb
