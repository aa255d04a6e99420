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
constexpr int M_SMEM = M_OFF_BAR + 64 + 1024;  // + alignment slack
constexpr uint32_t M_TMEM_COLS = 64;  // S^T [0, 16), O^T [16, 48)
enum MBar { K_FULL = 0, V_FULL = 1, S_DONE = 2, O_DONE = 3 };

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
HB_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
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
HB_DEV void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
HB_DEV void st_cluster_v4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
// Split cluster barrier: arrive early (this CTA has started), wait later.
HB_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
HB_DEV void cluster_wait_m() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
HB_DEV void cluster_sync_m() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
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
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 4);
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

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) tmem_alloc(tslot, M_TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;
  griddep_launch_dependents();
  cluster_arrive_relaxed();  // waited for before the first store into a peer

  auto wait = [&](int b, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait(&bar[b], parity)) return true;
    record_status(p.status, kStatusTimeout);
    *abort_flag = 1;
    return false;
  };

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
        mbar_arrive_expect_tx(&bar[K_FULL], 4 * 16384);
        for (int cb = 0; cb < 4; ++cb)
          tma_load_3d(smem + M_OFF_K + cb * 16384, &tmK, &bar[K_FULL], cb * 64, int(p0), kh);
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
      if (wait(K_FULL, 0)) {
        fence_after_sync();
#pragma unroll
        for (int cb = 0; cb < 4; ++cb)
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4)
            mma_bf16_ss(tmem, desc_add(kd0, cb * 16384 + k4 * 32), desc_add(qd0, cb * 2048 + k4 * 32),
                        idS, cb > 0 || k4 > 0);
        mma_commit(&bar[S_DONE]);
      }
    }
    __syncwarp();
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
        for (int mm = 0; mm < 2; ++mm)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ss(tmem + NQ + NQ * mm, desc_add(vd0, 2 * mm * 16384 + kk * 2048),
                        desc_add(pd0, (kk >> 2) * 2048 + (kk & 3) * 32), idPV, kk > 0);
        mma_commit(&bar[O_DONE]);
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
      const float sm = warp_sum(pr[g]);
      if (lane == 0) red_l[warp * 16 + g] = sm;
      // P^T element (head g, position pl), bf16
      const uint16_t b = uint16_t(pack_bf16x2(pr[g], 0.f) & 0xFFFFu);
      *reinterpret_cast<uint16_t*>(smem + M_OFF_P + swz(g, pl, 2048)) = b;
    }
    fence_proxy_async_smem();
    nbar_sync(2, 128);
    if (tid < G) {  // the tile's partial (m, l) of head tid
      cpart[G * HDM + tid] = m[tid];
      cpart[G * HDM + G + tid] =
          ((red_l[tid] + red_l[16 + tid]) + red_l[32 + tid]) + red_l[48 + tid];
    }
    nbar_sync(3, kThreadsM);  // P^T ready for the MMA

    // O^T out of TMEM: thread = dim 32 warp + lane (+ 128), columns = heads
    if (has) {
      ok = __all_sync(0xFFFFFFFFu, wait(O_DONE, 0)) && ok;
      fence_after_sync();
#pragma unroll
      for (int mm = 0; mm < 2; ++mm) {
        uint32_t o[16];
        tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + NQ + NQ * mm, o);
        tmem_wait_ld();
        const int dim = mm * 128 + pl;
#pragma unroll
        for (int g = 0; g < G; ++g) cpart[g * HDM + dim] = ok ? __uint_as_float(o[g]) : 0.f;
      }
    } else {
      for (int e = tid; e < G * HDM; e += 128) cpart[e] = 0.f;
    }
  }

  // ------------------------------------------------ merge across the cluster
  // Every CTA stores its (m, l) into every peer, and into CTA s the output
  // quads s merges (quads [s nqs, (s + 1) nqs)); after one cluster barrier
  // each CTA merges its slice from its own shared memory and nothing reads
  // a peer any more.
  constexpr int Q4 = G * HDM / 4;
  const int nqs = (Q4 + ns - 1) / ns;  // quads per slice (the last one may be short)
  float* rml = reinterpret_cast<float*>(smem + M_OFF_RML);      // [split][16]
  float4* rbuf = reinterpret_cast<float4*>(smem + M_OFF_RBUF);  // [split][nqs]
  if (warp < 4) nbar_sync(2, 128);  // this CTA's partial is complete
  __syncwarp();
  cluster_wait_m();  // every CTA of the cluster has started
  if (warp < 4) {
    for (int i = tid; i < ns * 2 * G; i += 128) {
      const int sp = i / (2 * G), k = i % (2 * G);
      st_cluster_f32(dsmem_addr_m(rml + split * 16 + k, uint32_t(sp)), cpart[G * HDM + k]);
    }
    for (int q = tid; q < Q4; q += 128) {
      const int sp = q / nqs, qi = q - sp * nqs;
      st_cluster_v4(dsmem_addr_m(rbuf + split * nqs + qi, uint32_t(sp)),
                    *reinterpret_cast<const float4*>(cpart + q * 4));
    }
  }
  fence_before_sync();
  __syncwarp();
  cluster_sync_m();  // every store into this CTA has landed
  if (warp < 4) {
    // the splits' weights 2^(m_r - M) and the merged sums, one warp per head
    float* wb = reinterpret_cast<float*>(smem + M_OFF_K);  // [split][16] (the K tile is done)
    float* Lb = wb + 16 * 16;                              // [G]
    for (int g = warp; g < G; g += 4) {
      const float mv = lane < ns ? rml[lane * 16 + g] : -INFINITY;
      const float lv = lane < ns ? rml[lane * 16 + G + g] : 0.f;
      const float M = warp_max(mv);
      const float Mu = M == -INFINITY ? 0.f : M;
      const float w = lane < ns ? fast_exp2(mv - Mu) : 0.f;
      const float L = warp_sum(lv * w);
      if (lane < ns) wb[lane * 16 + g] = w;
      if (lane == 0) Lb[g] = L;
    }
    nbar_sync(2, 128);
    // one output element per thread: the splits' weighted sum, / l, bf16,
    // the gate with the reference's steps
    const int q0 = split * nqs, nq = max(0, min(nqs, Q4 - q0));
    uint16_t* orow = p.out + int64_t(row) * p.out_row;
    if (!*abort_flag) {
      const float* rf = reinterpret_cast<const float*>(rbuf);
      for (int t = tid; t < 4 * nq; t += 128) {
        const int e = q0 * 4 + t, g = e / HDM, dd = e % HDM;
        float acc = 0.f;
        for (int r = 0; r < ns; ++r) acc = fmaf(wb[r * 16 + g], rf[r * nqs * 4 + t], acc);
        const float Ls = Lb[g];
        const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
        uint16_t a = f32_to_bf16_cvtne(acc * inv);
        if (p.gate_offset >= 0) a = gate_bf16(a, qrow[p.gate_offset + int64_t(h0 + g) * HDM + dd]);
        orow[int64_t(h0 + g) * HDM + dd] = a;
      }
    }
  }
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

}  // namespace hb
