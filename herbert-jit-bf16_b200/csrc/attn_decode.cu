// attn_decode.cu -- split-KV flash-decoding SDPA for sm_100a, with the
// Qwen3.5 sigmoid output gate fused into the final combine.
//
// Replaces, in the decode regime, the reference's attention node
// (SdpaHeadFn per (row, head), src/jit/emit_sdpa.rs:131-140, driven by
// src/jit/target/x86/execution/attention.rs:56-224) and the output-gate node
// (ElemOp::SigmoidMul, src/jit/target/x86/emit_elem.rs:333-420).
//
// Work decomposition.  A "unit" is (sequence, query row, KV head): the G
// query heads of one GQA group share every K/V row, so a CTA streams
// positions of one KV head once and scores them against all G heads.  The
// tiles (32 positions) of all units are laid end to end and cut into one
// range per resident CTA slot (two per SM for groups of up to 4 heads):
// every CTA moves the same bytes whatever the sequences' lengths, in one
// wave.  A CTA walks the units its range touches one segment at a time.
//
// CTA = 1 producer warp + 8 consumer warps.  The producer streams 32-position
// tiles of K and V with 1-D bulk copies (a tile of one head is contiguous in
// the reference layout) into a shared-memory ring, completion tracked by
// mbarriers: 96 KB (3 stages at head_dim 256) and two CTAs per SM for groups
// of up to 4 query heads, 128 KB and one CTA for 8.  Consumer warp w owns
// positions 4w..4w+3 of every tile and keeps its own online-softmax state
// (max, sum, G x head_dim accumulator, in the log2 domain).  A lane holds
// head_dim/32 consecutive dimensions: each K or V row is one 16-byte
// (head_dim 256) shared-memory load per lane.  The 4G partial dot products
// of a lane are reduced across the warp by a transposed butterfly (4G-1
// shuffles for 4G sums instead of 5 per sum).
//
// At a segment's end the 8 warp states merge in shared memory; a unit inside
// one range is finalised by its CTA, otherwise each CTA writes an
// unnormalised partial (O, m, l) to the workspace and the last CTA of the
// unit to arrive (atomic counter, reset after use) merges the partials,
// rounds to bf16 and applies the gate with the reference's own exp
// polynomial and rounding steps.
//
// Short sequences (one call, at most 16 splits of <= 256 positions) take
// the cluster form instead: the splits of a unit are one thread-block
// cluster, each CTA leaves its partial in its own shared memory, and after
// a cluster barrier CTA r merges output slice r from all the partials
// through distributed shared memory -- no global partials, no atomics, and
// the merge is spread over the cluster instead of one last CTA.  Both forms
// are launched with programmatic dependent launch: the next grid on the
// stream may become resident early, and before its own griddepcontrol.wait
// a cluster CTA only prefetches its K/V split and q/gate lines into L2
// (prefetches cannot change what a later load returns), so a decode step
// that follows another pulls its 8 MB from HBM while the previous one
// computes, and reads nothing, and writes nothing, before that one ends.
#include <cstdint>
#include <cuda_runtime.h>

#include "hb_common.cuh"
#include "hb_host.h"
#include "hb_internal.h"
#include "hb_sm100.cuh"

namespace hb {

// Scratch of hb_attn_decode_noalloc: a file-scope device array, so callers
// that may not allocate device memory still get split-KV decoding.  Every
// device that loads the library holds these bytes until the process exits.
// In host code the name is only a host-side stand-in for the symbol; the
// device address comes from cudaGetSymbolAddress (noalloc_scratch below),
// looked up once per device and context: a context that ends (for instance
// by cudaDeviceReset) takes its module and the array's mapping with it, and
// the next call in a new context looks the address up again.
static __device__ __align__(256) unsigned char g_noalloc_scratch[HB_NOALLOC_SCRATCH_BYTES];

cudaError_t noalloc_scratch(void** ptr) {
  static SymbolCache cache;
  return symbol_address(cache, reinterpret_cast<const void*>(&g_noalloc_scratch), ptr);
}

namespace {

constexpr int kTile = 32;           // positions per pipeline tile
// K+V tiles in flight per CTA: groups of up to 4 query heads run two CTAs
// per SM (96 KB rings: twice the warps to hide each tile's latency chain),
// larger groups one (128 KB, the registers of 8 heads' accumulators)
template <int G>
struct RingBytes { static constexpr int value = G <= 4 ? 98304 : 131072; };
template <int G>
struct CtasPerSm { static constexpr int value = G <= 4 ? 2 : 1; };
constexpr int kConsumerWarps = 8;   // 4 positions per warp per tile
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr uint32_t kFull = 0xFFFFFFFFu;
constexpr int64_t kMaxSplits = 1024;  // 3 * 8 * 1024 floats fit the ring

struct DecodeParams {
  const hb_decode_seq* seqs;  // device table, or nullptr: use `one`
  hb_decode_seq one;
  int rows;                   // query rows per sequence (table mode: 1)
  int hkv;                    // KV heads
  int64_t q_row, q_head, out_row;
  int64_t gate_offset;        // < 0: no gate
  float scale_log2;           // scale * log2(e)
  int chunk;                  // positions per split, multiple of kTile
  int nsplit;                 // cluster form: grid.x
  int units_z;                // ranges form: sequences x rows
  int* status;
  unsigned* counters;         // one per unit (ranges form)
  float* partials;            // cluster form: unused; ranges form: [range + unit][G*HD + 2G]
};

// ------------------------------------------------ cluster shared memory
HB_DEV uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
HB_DEV float dsmem_ld(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
// (not volatile: the reads of one merge are independent and overlap; the
// cluster barrier before them orders them after the peers' writes)
HB_DEV float4 dsmem_ld4(uint32_t addr) {
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "r"(addr));
  return v;
}
// Every thread of every CTA of the cluster (hardware barrier: each path
// through the kernel reaches it exactly as often).
HB_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

template <int HD>
struct LaneVec;
template <>
struct LaneVec<256> {  // 8 bf16 per lane
  static HB_DEV void load(const uint16_t* p, float (&x)[8]) {
    uint4 w = *reinterpret_cast<const uint4*>(p);
    x[0] = bf16lo(w.x); x[1] = bf16hi(w.x); x[2] = bf16lo(w.y); x[3] = bf16hi(w.y);
    x[4] = bf16lo(w.z); x[5] = bf16hi(w.z); x[6] = bf16lo(w.w); x[7] = bf16hi(w.w);
  }
};
template <>
struct LaneVec<128> {  // 4 bf16 per lane
  static HB_DEV void load(const uint16_t* p, float (&x)[4]) {
    uint2 w = *reinterpret_cast<const uint2*>(p);
    x[0] = bf16lo(w.x); x[1] = bf16hi(w.x); x[2] = bf16lo(w.y); x[3] = bf16hi(w.y);
  }
};

template <int V>
struct Log2 { static constexpr int value = 1 + Log2<V / 2>::value; };
template <>
struct Log2<1> { static constexpr int value = 0; };

// Transposed butterfly: every lane enters with NV partial sums; on exit
// lane l holds the warp-wide sum of value (l >> (5 - log2 NV)).
template <int NV>
HB_DEV float transpose_reduce(float (&v)[NV], int lane) {
  constexpr int L = Log2<NV>::value;
#pragma unroll
  for (int lvl = 0; lvl < L; ++lvl) {
    const int width = NV >> lvl, half = width >> 1, off = 16 >> lvl;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      float send = upper ? v[i] : v[i + half];
      float keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(kFull, send, off);
    }
  }
#pragma unroll
  for (int off = 16 >> L; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(kFull, v[0], off);
  return v[0];
}

HB_DEV void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory"); }

template <int HD, int G>
struct Ring { static constexpr int stages = RingBytes<G>::value / (2 * kTile * HD * 2); };

// Compile-time geometry of the CUDA-core decode kernels.
template <int HD, int G>
struct Geo {
  static constexpr int kStages = Ring<HD, G>::stages;
  static constexpr int DPL = HD / 32;             // dims per lane
  static constexpr int DP2 = DPL / 2;             // paired f32 lanes per lane
  static constexpr int NV = 4 * G;                // partial sums per lane per tile
  static constexpr int SH = 5 - Log2<NV>::value;  // lane >> SH = value index
  static constexpr int TILE_ELEMS = kTile * HD;
  static constexpr int PSTRIDE = G * HD + ((2 * G + 3) & ~3);  // floats per partial (16 B multiple)
  static constexpr int RING_BYTES = 2 * kStages * TILE_ELEMS * 2;
  static constexpr int MERGE_BYTES = kConsumerWarps * PSTRIDE * 4;
  static constexpr int BODY = ((RING_BYTES > MERGE_BYTES ? RING_BYTES : MERGE_BYTES) + 15) / 16 * 16;
  static constexpr int NOUT = G * HD;             // outputs of a unit
  static constexpr int NT = kConsumerWarps * 32;  // consumer threads
  static constexpr int PER_T = (NOUT + NT - 1) / NT;
};

// Consumer warp `warp`'s share of one ring tile (K at ktile, V at vtile):
// positions 4 warp .. 4 warp + 3, the first vc of them valid, scored against
// the G query heads in q2; online-softmax update of this lane's (m_own,
// l_own) and P.V into the accumulators o2.
template <int HD, int G>
HB_DEV void consume_tile(const uint16_t* ktile, const uint16_t* vtile, int vc, float scale_log2,
                         const uint64_t (&q2)[G][Geo<HD, G>::DP2], uint64_t (&o2)[G][Geo<HD, G>::DP2],
                         float& m_own, float& l_own, int warp, int lane) {
  using T = Geo<HD, G>;
  constexpr int DPL = T::DPL, DP2 = T::DP2, NV = T::NV, SH = T::SH;
  const uint16_t* kt = ktile + warp * 4 * HD + lane * DPL;
  const uint16_t* vt = vtile + warp * 4 * HD + lane * DPL;
  float part[NV];
  // all four rows are read whatever vc is (the reads stay inside the ring),
  // so the loads issue together; a dot of a row past vc only reaches its
  // own slot, which the mask below sets to -inf
  float kxa[4][DPL];
#pragma unroll
  for (int j = 0; j < 4; ++j) LaneVec<HD>::load(kt + j * HD, kxa[j]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float (&kx)[DPL] = kxa[j];
    uint64_t k2[DP2];
#pragma unroll
    for (int k = 0; k < DP2; ++k) k2[k] = f2(kx[2 * k], kx[2 * k + 1]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      uint64_t acc = f2mul(q2[g][0], k2[0]);
#pragma unroll
      for (int k = 1; k < DP2; ++k) acc = f2fma(q2[g][k], k2[k], acc);
      part[g * 4 + j] = f2lo(acc) + f2hi(acc);
    }
  }
  const float dot = transpose_reduce<NV>(part, lane);
  const int vidx = lane >> SH, jown = vidx & 3;
  float sc = jown < vc ? dot * scale_log2 : -INFINITY;
  // max over the 4 positions of this lane's head
  float tmax = fmaxf(sc, __shfl_xor_sync(kFull, sc, 1 << SH));
  tmax = fmaxf(tmax, __shfl_xor_sync(kFull, tmax, 2 << SH));
  const float m_new = fmaxf(m_own, tmax);
  const float m_use = m_new == -INFINITY ? 0.f : m_new;
  const float corr = fast_exp2(m_own - m_use);
  const float pr = fast_exp2(sc - m_use);
  float psum = pr + __shfl_xor_sync(kFull, pr, 1 << SH);
  psum += __shfl_xor_sync(kFull, psum, 2 << SH);
  l_own = l_own * corr + psum;
  m_own = m_new;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float cg = __shfl_sync(kFull, corr, (g * 4) << SH);
    const uint64_t cg2 = f2(cg, cg);
#pragma unroll
    for (int k = 0; k < DP2; ++k) o2[g][k] = f2mul(o2[g][k], cg2);
  }
  float vxa[4][DPL];
#pragma unroll
  for (int j = 0; j < 4; ++j) LaneVec<HD>::load(vt + j * HD, vxa[j]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    // rows past vc may hold any bits (even NaN): zero them, p is 0 there
    uint64_t v2[DP2];
#pragma unroll
    for (int k = 0; k < DP2; ++k)
      v2[k] = j < vc ? f2(vxa[j][2 * k], vxa[j][2 * k + 1]) : f2(0.f, 0.f);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pg = __shfl_sync(kFull, pr, (g * 4 + j) << SH);
      const uint64_t pg2 = f2(pg, pg);
#pragma unroll
      for (int k = 0; k < DP2; ++k) o2[g][k] = f2fma(pg2, v2[k], o2[g][k]);
    }
  }
}

// The 8 consumer warps' states merged through shared memory `ws` (the ring,
// which every warp has finished reading once the first barrier passes):
// consumer thread tid ends with (M, L, O) of output elements tid + 256 k.
template <int HD, int G>
HB_DEV void merge_warps(float* ws, const uint64_t (&o2)[G][Geo<HD, G>::DP2], float m_own,
                        float l_own, int warp, int lane, float (&om)[Geo<HD, G>::PER_T],
                        float (&ol)[Geo<HD, G>::PER_T], float (&oo)[Geo<HD, G>::PER_T]) {
  using T = Geo<HD, G>;
  constexpr int DPL = T::DPL, DP2 = T::DP2, SH = T::SH, PSTRIDE = T::PSTRIDE;
  consumer_sync();  // every warp is done reading the ring
  {
    float* mine = ws + warp * PSTRIDE;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int k = 0; k < DP2; ++k) {
        mine[g * HD + lane * DPL + 2 * k] = f2lo(o2[g][k]);
        mine[g * HD + lane * DPL + 2 * k + 1] = f2hi(o2[g][k]);
      }
    if ((lane & ((4 << SH) - 1)) == 0) {
      const int g = (lane >> SH) >> 2;
      mine[G * HD + g] = m_own;
      mine[G * HD + G + g] = l_own;
    }
  }
  consumer_sync();
  const int tid = threadIdx.x;
#pragma unroll
  for (int k = 0; k < T::PER_T; ++k) {
    const int e = min(tid + k * T::NT, T::NOUT - 1), g = e / HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, ws[w * PSTRIDE + G * HD + g]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float Ls = 0.f, Os = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float f = fast_exp2(ws[w * PSTRIDE + G * HD + g] - Mu);
      Ls += ws[w * PSTRIDE + G * HD + G + g] * f;
      Os += ws[w * PSTRIDE + e] * f;
    }
    om[k] = M; ol[k] = Ls; oo[k] = Os;
  }
}

// A unit whose positions one CTA covered: O / l, bf16, then the gate.
template <int HD, int G>
HB_DEV void finalize_own(const float (&ol)[Geo<HD, G>::PER_T], const float (&oo)[Geo<HD, G>::PER_T],
                         uint16_t* orow, const uint16_t* qrow, int64_t gate_offset, int h0) {
  using T = Geo<HD, G>;
  const int tid = threadIdx.x;
#pragma unroll
  for (int k = 0; k < T::PER_T; ++k) {
    const int e = tid + k * T::NT, g = e / HD, dd = e % HD;
    if (e >= T::NOUT) break;
    const int h = h0 + g;
    const float val = ol[k] > 0.f ? oo[k] / ol[k] : 0.f;
    uint16_t a = f32_to_bf16_cvtne(val);
    if (gate_offset >= 0) a = gate_bf16(a, qrow[gate_offset + int64_t(h) * HD + dd]);
    orow[int64_t(h) * HD + dd] = a;
  }
}

// This CTA's unnormalised partial (O, m, l) of a unit, to `mine` in global
// memory (L2).
template <int HD, int G>
HB_DEV void store_partial(float* mine, const float (&om)[Geo<HD, G>::PER_T],
                          const float (&ol)[Geo<HD, G>::PER_T], const float (&oo)[Geo<HD, G>::PER_T]) {
  using T = Geo<HD, G>;
  const int tid = threadIdx.x;
#pragma unroll
  for (int k = 0; k < T::PER_T; ++k) {
    const int e = tid + k * T::NT, g = e / HD;
    if (e >= T::NOUT) break;
    __stcg(mine + e, oo[k]);
    if ((e % HD) == 0) {
      __stcg(mine + G * HD + g, om[k]);
      __stcg(mine + G * HD + G + g, ol[k]);
    }
  }
}

// The merge of a unit's `active` partials at up[0 .. active) (stride
// PSTRIDE) by the last CTA to leave one.  The partials' maxima and sums are
// staged in `ws` first (one load per thread), the per-partial weights
// computed once per head, then each output element sums its partials with
// independent loads in flight; O / L, bf16, the gate.
template <int HD, int G>
HB_DEV void merge_partials(const float* up, int active, float* ws, uint16_t* orow,
                           const uint16_t* qrow, int64_t gate_offset, int h0) {
  using T = Geo<HD, G>;
  constexpr int PSTRIDE = T::PSTRIDE;
  const int tid = threadIdx.x;
  float* sml = ws;                       // [active][2G]: m then l
  float* smw = ws + active * 2 * G;      // [active][G]: exp2(m_s - M)
  float* smL = smw + active * G;         // [G]: merged sums
  for (int i = tid; i < active * 2 * G; i += T::NT)
    sml[i] = __ldcg(up + (i / (2 * G)) * PSTRIDE + G * HD + (i % (2 * G)));
  consumer_sync();
  if (tid < G) {
    float M = -INFINITY;
    for (int sp = 0; sp < active; ++sp) M = fmaxf(M, sml[sp * 2 * G + tid]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float Ls = 0.f;
    for (int sp = 0; sp < active; ++sp) {
      const float w = fast_exp2(sml[sp * 2 * G + tid] - Mu);
      smw[sp * G + tid] = w;
      Ls += sml[sp * 2 * G + G + tid] * w;
    }
    smL[tid] = Ls;
  }
  consumer_sync();
  // every thread owns 4 consecutive outputs (one head): one 16-byte load per
  // partial, all independent, then finalise them here
  for (int qd = tid; qd < T::NOUT / 4; qd += T::NT) {
    const int e = qd * 4, g = e / HD, dd = e % HD, hq = h0 + g;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
    for (int sp = 0; sp < active; ++sp) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(up + sp * PSTRIDE + e));
      const float w = smw[sp * G + g];
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    const float Ls = smL[g];
    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
    uint16_t a[4] = {f32_to_bf16_cvtne(acc.x * inv), f32_to_bf16_cvtne(acc.y * inv),
                     f32_to_bf16_cvtne(acc.z * inv), f32_to_bf16_cvtne(acc.w * inv)};
    if (gate_offset >= 0) {
      const uint2 gw = *reinterpret_cast<const uint2*>(qrow + gate_offset + int64_t(hq) * HD + dd);
      a[0] = gate_bf16(a[0], uint16_t(gw.x & 0xFFFFu));
      a[1] = gate_bf16(a[1], uint16_t(gw.x >> 16));
      a[2] = gate_bf16(a[2], uint16_t(gw.y & 0xFFFFu));
      a[3] = gate_bf16(a[3], uint16_t(gw.y >> 16));
    }
    *reinterpret_cast<uint2*>(orow + int64_t(hq) * HD + dd) =
        make_uint2(uint32_t(a[0]) | (uint32_t(a[1]) << 16), uint32_t(a[2]) | (uint32_t(a[3]) << 16));
  }
}

// q of the G heads of group h0 as paired f32 lanes (dims 2k, 2k+1): one
// paired FMA per two products.
template <int HD, int G>
HB_DEV void load_q(const uint16_t* qrow, int64_t q_head, int h0, int lane,
                   uint64_t (&q2)[G][Geo<HD, G>::DP2]) {
  constexpr int DPL = Geo<HD, G>::DPL;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float t[DPL];
    LaneVec<HD>::load(qrow + int64_t(h0 + g) * q_head + lane * DPL, t);
#pragma unroll
    for (int k = 0; k < DPL / 2; ++k) q2[g][k] = f2(t[2 * k], t[2 * k + 1]);
  }
}

// ------------------------------------------------------------ cluster form
// One short sequence: grid (splits, kv heads, rows), a cluster per unit.
template <int HD, int G>
__global__ void __launch_bounds__(kThreads, CtasPerSm<G>::value)
    attn_decode_cluster_kernel(const DecodeParams p) {
  using T = Geo<HD, G>;
  constexpr int kStages = T::kStages, DP2 = T::DP2, TILE_ELEMS = T::TILE_ELEMS;
  constexpr int MERGE_BYTES = T::MERGE_BYTES, BODY = T::BODY, NOUT = T::NOUT, PER_T = T::PER_T;

  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint16_t* ks = reinterpret_cast<uint16_t*>(smem_raw);
  uint16_t* vs = ks + kStages * TILE_ELEMS;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + BODY);
  uint64_t* empty = full + kStages;
  int* flags = reinterpret_cast<int*>(empty + kStages);  // [0] abort

  const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
  const hb_decode_seq d = p.one;
  const int64_t n = d.past + row + 1;  // keys visible to this row
  const int64_t p0 = int64_t(split) * p.chunk;
  // a CTA beyond the row's last position still merges its output slice,
  // with an empty partial
  const int64_t p1 = max(p0, min(n, p0 + p.chunk));
  const int ntiles = int((p1 - p0 + kTile - 1) / kTile);
  const uint16_t* kbase = d.keys + int64_t(kh) * d.kv_stride;
  const uint16_t* vbase = d.values + int64_t(kh) * d.kv_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    flags[0] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // launched with programmatic stream serialization: the next grid on the
  // stream may become resident now and run up to its own griddep_wait()
  // while this one works
  griddep_launch_dependents();

  if (warp == kConsumerWarps) {  // ---------------------------- producer
    if (lane == 0) {
      const uint64_t once = l2_evict_first();  // K and V are read once per step
      // this split's K and V into L2 while the previous grid finishes;
      // every load that returns data waits for it
      if (p1 > p0) {
        const uint32_t bytes = uint32_t(p1 - p0) * HD * 2u;
        bulk_prefetch_l2(kbase + p0 * HD, bytes);
        bulk_prefetch_l2(vbase + p0 * HD, bytes);
      }
      griddep_wait();
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(&empty[s], ((t / kStages) - 1) & 1)) {
          record_status(p.status, kStatusTimeout);
          atomicExch(&flags[0], 1);
          break;
        }
        const int64_t pos = p0 + int64_t(t) * kTile;
        const uint32_t bytes = uint32_t(min(int64_t(kTile), p1 - pos)) * HD * 2u;
        mbar_arrive_expect_tx(&full[s], 2u * bytes);
        bulk_g2s_hint(ks + s * TILE_ELEMS, kbase + pos * HD, bytes, &full[s], once);
        bulk_g2s_hint(vs + s * TILE_ELEMS, vbase + pos * HD, bytes, &full[s], once);
      }
    }
    // the producer warp takes part in both cluster barriers
    __syncwarp();
    cluster_sync_all();
    cluster_sync_all();
    return;
  }

  // ------------------------------------------------------------ consumers
  const int h0 = kh * G;  // first query head of the group
  const uint16_t* qrow = d.q + int64_t(row) * p.q_row;
  {
    // the group's q and gate lines into L2, then wait for the previous grid
    // (q, the gate and the newest K/V rows may be its outputs)
    constexpr int LINES = HD * 2 / 128;  // 128-byte lines per head
    if (int(threadIdx.x) < G * LINES) {
      const int g = threadIdx.x / LINES, ln = threadIdx.x % LINES;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(
          reinterpret_cast<const char*>(qrow + int64_t(h0 + g) * p.q_head) + ln * 128));
      if (p.gate_offset >= 0)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(
            reinterpret_cast<const char*>(qrow + p.gate_offset + int64_t(h0 + g) * HD) + ln * 128));
    }
    griddep_wait();
  }
  uint64_t q2[G][DP2];
  load_q<HD, G>(qrow, p.q_head, h0, lane, q2);
  uint64_t o2[G][DP2];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int k = 0; k < DP2; ++k) o2[g][k] = f2(0.f, 0.f);
  float m_own = -INFINITY, l_own = 0.f;  // state of value head (lane >> SH) >> 2
  // the gate values of this thread's output quad, fetched now so that the
  // final merge does not wait on them
  uint2 gate_pre = make_uint2(0u, 0u);
  if (p.gate_offset >= 0) {
    constexpr int Q4 = G * HD / 4;
    const int ns = p.nsplit, qb = split * Q4 / ns, qe = (split + 1) * Q4 / ns;
    const int tid0 = threadIdx.x;
    if (tid0 < qe - qb) {
      const int e = (qb + tid0) * 4, g = e / HD, dd = e % HD;
      gate_pre = *reinterpret_cast<const uint2*>(qrow + p.gate_offset + int64_t(h0 + g) * HD + dd);
    }
  }

  for (int t = 0; t < ntiles; ++t) {
    const int s = t % kStages;
    if (*reinterpret_cast<volatile int*>(&flags[0])) break;
    if (!mbar_wait(&full[s], (t / kStages) & 1)) {
      record_status(p.status, kStatusTimeout);
      atomicExch(&flags[0], 1);
      break;
    }
    const int64_t tile_pos = p0 + int64_t(t) * kTile;
    const int vc = int(max(int64_t(0), min(int64_t(4), p1 - tile_pos - warp * 4)));
    if (vc > 0)
      consume_tile<HD, G>(ks + s * TILE_ELEMS, vs + s * TILE_ELEMS, vc, p.scale_log2, q2, o2,
                          m_own, l_own, warp, lane);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  float* ws = reinterpret_cast<float*>(smem_raw);  // [warp][G*HD + 2G]
  const int tid = threadIdx.x;
  float om[PER_T], ol[PER_T], oo[PER_T];
  merge_warps<HD, G>(ws, o2, m_own, l_own, warp, lane, om, ol, oo);

  // this CTA's partial stays in its shared memory for the cluster merge
  float* cpart = reinterpret_cast<float*>(smem_raw + (MERGE_BYTES + 15) / 16 * 16);
#pragma unroll
  for (int k = 0; k < PER_T; ++k) {
    const int e = tid + k * T::NT, g = e / HD;
    if (e >= NOUT) break;
    cpart[e] = oo[k];
    if ((e % HD) == 0) {
      cpart[G * HD + g] = om[k];
      cpart[G * HD + G + g] = ol[k];
    }
  }
  cluster_sync_all();
  // output slice of this CTA: quads [split * Q / ns, (split + 1) * Q / ns)
  const int ns = p.nsplit;
  float* sml = ws;                 // [ns][2G]: m then l of every split
  float* smw = ws + ns * 2 * G;    // [ns][G]: exp2(m_s - M)
  float* smL = smw + ns * G;       // [G]
  for (int i = tid; i < ns * 2 * G; i += T::NT)
    sml[i] = dsmem_ld(dsmem_addr(cpart + G * HD + (i % (2 * G)), uint32_t(i / (2 * G))));
  consumer_sync();
  if (tid < G) {
    float M = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, sml[sp * 2 * G + tid]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float Ls = 0.f;
    for (int sp = 0; sp < ns; ++sp) {
      const float w = fast_exp2(sml[sp * 2 * G + tid] - Mu);
      smw[sp * G + tid] = w;
      Ls += sml[sp * 2 * G + G + tid] * w;
    }
    smL[tid] = Ls;
  }
  consumer_sync();
  constexpr int Q4 = NOUT / 4;
  const int qb = split * Q4 / ns, qe = (split + 1) * Q4 / ns, nq = qe - qb;
  // one 16-byte read per (output quad, split), all in flight at once, then
  // the splits of each quad summed through shared memory
  float4* red = reinterpret_cast<float4*>(smL + G + 3);  // [ns][nq], 16-byte aligned below
  red = reinterpret_cast<float4*>((reinterpret_cast<uintptr_t>(red) + 15) & ~uintptr_t(15));
  for (int idx = tid; idx < nq * ns; idx += T::NT) {
    const int sp = idx / nq, qi = idx % nq, e = (qb + qi) * 4, g = e / HD;
    const float4 v = dsmem_ld4(dsmem_addr(cpart + e, uint32_t(sp)));
    const float w = smw[sp * G + g];
    red[idx] = make_float4(w * v.x, w * v.y, w * v.z, w * v.w);
  }
  consumer_sync();
  uint16_t* orow_c = d.output + int64_t(row) * p.out_row;
  for (int qi = tid; qi < nq; qi += T::NT) {
    const int e = (qb + qi) * 4, g = e / HD, dd = e % HD, hq = h0 + g;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < ns; ++sp) {
      const float4 v = red[sp * nq + qi];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const float Ls = smL[g];
    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
    uint16_t a[4] = {f32_to_bf16_cvtne(acc.x * inv), f32_to_bf16_cvtne(acc.y * inv),
                     f32_to_bf16_cvtne(acc.z * inv), f32_to_bf16_cvtne(acc.w * inv)};
    if (p.gate_offset >= 0) {
      // fetched at the start when this thread owns the quad (nq <= 256)
      const uint2 gw = qi == tid ? gate_pre
                                 : *reinterpret_cast<const uint2*>(qrow + p.gate_offset +
                                                                   int64_t(hq) * HD + dd);
      a[0] = gate_bf16(a[0], uint16_t(gw.x & 0xFFFFu));
      a[1] = gate_bf16(a[1], uint16_t(gw.x >> 16));
      a[2] = gate_bf16(a[2], uint16_t(gw.y & 0xFFFFu));
      a[3] = gate_bf16(a[3], uint16_t(gw.y >> 16));
    }
    *reinterpret_cast<uint2*>(orow_c + int64_t(hq) * HD + dd) =
        make_uint2(uint32_t(a[0]) | (uint32_t(a[1]) << 16), uint32_t(a[2]) | (uint32_t(a[3]) << 16));
  }
  cluster_sync_all();  // the peers are done reading this CTA's partial
}

// --------------------------------------------------------- balanced ranges
// Every other call (batches, long sequences, blocks of rows): the tiles of
// all units laid end to end -- unit u = (z, y), query row z of the call
// (sequence z / rows, row z % rows) and KV head y, holding ceil(n_z / 32)
// tiles -- and CTA k of S streams tiles [k T / S, (k + 1) T / S), so every
// CTA moves the same bytes whatever the lengths.  A CTA walks the units of
// its range one segment at a time; a unit inside one range is finalised by
// its CTA, otherwise each CTA touching it leaves a partial in slot k + u
// (slots of one unit are contiguous: the units of consecutive ranges never
// decrease) and the last to arrive (atomic counter, reset after use) merges.
template <int HD, int G>
__global__ void __launch_bounds__(kThreads, CtasPerSm<G>::value)
    attn_decode_ranges_kernel(const DecodeParams p) {
  using T = Geo<HD, G>;
  constexpr int kStages = T::kStages, TILE_ELEMS = T::TILE_ELEMS;
  constexpr int PSTRIDE = T::PSTRIDE, BODY = T::BODY, PER_T = T::PER_T;
  constexpr int kWarps = kThreads / 32;

  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint16_t* ks = reinterpret_cast<uint16_t*>(smem_raw);
  uint16_t* vs = ks + kStages * TILE_ELEMS;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + BODY);
  uint64_t* empty = full + kStages;
  int* flags = reinterpret_cast<int*>(empty + kStages);  // [0] abort, [1] is-last
  int64_t* scan = reinterpret_cast<int64_t*>(flags + 4);  // [kWarps] totals, then z and Zpre(z)

  const int k = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // launched with programmatic stream serialization: the next grid may
  // become resident as this one's CTAs finish; the sequence table, q and the
  // newest K/V rows may be outputs of the previous grid, so every load
  // follows the wait
  griddep_launch_dependents();
  griddep_wait();

  // ---- T and the unit holding this CTA's first tile: thread i sums the
  // tiles of a contiguous block of rows z, a block scan gives Zpre (tiles of
  // the rows before z, per KV head), the thread whose block holds tile b0
  // walks it
  const int64_t hkv = p.hkv;
  const int Z = p.units_z;
  auto row_tiles = [&](int z) -> int64_t {
    const int64_t past = p.seqs ? p.seqs[z].past : p.one.past;  // table mode: one row per sequence
    return (past + (p.seqs ? 0 : z) + kTile) / kTile;           // ceil((past + row + 1) / 32)
  };
  const int per = (Z + kThreads - 1) / kThreads;
  const int z0 = min(Z, tid * per), z1 = min(Z, z0 + per);
  int64_t local = 0;
  for (int z = z0; z < z1; ++z) local += row_tiles(z);
  int64_t inc = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t v = __shfl_up_sync(kFull, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) scan[warp] = inc;
  __syncthreads();
  int64_t woff = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const int64_t v = scan[w];
    woff += w < warp ? v : 0;
    total += v;
  }
  const int64_t excl = woff + inc - local;  // Zpre(z0)
  const int64_t tiles = total * hkv;
  // at most one range per tile (the plan sizes S from the caller's totals):
  // every range then holds at least one tile, so each CTA between the first
  // and the last range touching a unit leaves a partial of it
  const int S = int(min(int64_t(gridDim.x), tiles));
  if (k >= S) return;
  const int64_t b0 = int64_t(k) * tiles / S, b1 = int64_t(k + 1) * tiles / S;
  if (local > 0 && hkv * excl <= b0 && b0 < hkv * (excl + local)) {
    int64_t pre = excl;
    int z = z0;
    for (; z + 1 < z1; ++z) {
      const int64_t t = row_tiles(z);
      if (b0 < hkv * (pre + t)) break;
      pre += t;
    }
    scan[kWarps] = z;
    scan[kWarps + 1] = pre;
  }
  __syncthreads();
  // the range containing tile x
  auto range_of = [&](int64_t x) -> int64_t { return ((x + 1) * S - 1) / tiles; };

  float* ws = reinterpret_cast<float*>(smem_raw);  // merge scratch over the ring
  int z = int(scan[kWarps]);
  int64_t pre = scan[kWarps + 1];
  uint32_t tg = 0;      // tiles through the ring so far: slot tg % kStages, phase (tg / kStages) & 1
  uint32_t issued = 0;  // producer: one past the last tile it copied
  for (int64_t g = b0; g < b1;) {
    const hb_decode_seq d = p.seqs ? p.seqs[z] : p.one;
    const int row = p.seqs ? 0 : z;
    const int64_t n = d.past + row + 1;  // keys visible to this row
    const int64_t tz = (n + kTile - 1) / kTile;
    const int64_t ubase = hkv * pre;  // first tile of unit (z, 0)
    const int y = int((g - ubase) / tz);
    const int64_t ustart = ubase + int64_t(y) * tz;
    const int64_t a = g - ustart, b = min(b1, ustart + tz) - ustart;  // tiles [a, b) of the unit
    // a table entry the bulk copies and vector accesses cannot take: no
    // loads and no outputs for its units (the status word says why), its
    // partials and counters kept consistent
    const bool bad = ((reinterpret_cast<uintptr_t>(d.keys) | reinterpret_cast<uintptr_t>(d.values) |
                       reinterpret_cast<uintptr_t>(d.q) | reinterpret_cast<uintptr_t>(d.output)) & 15) != 0 ||
                     (d.kv_stride & 7) != 0;
    const int nt = bad ? 0 : int(b - a);
    const int64_t p0 = a * kTile, p1 = min(n, b * kTile);
    const int64_t u = int64_t(z) * hkv + y;
    if (warp == kConsumerWarps) {  // -------------------------- producer
      if (lane == 0) {
        const uint64_t once = l2_evict_first();  // K and V are read once per step
        const uint16_t* kbase = d.keys + int64_t(y) * d.kv_stride;
        const uint16_t* vbase = d.values + int64_t(y) * d.kv_stride;
        for (int t = 0; t < nt; ++t) {
          const uint32_t i = tg + uint32_t(t);
          const int s = int(i % kStages);
          if (*reinterpret_cast<volatile int*>(&flags[0])) break;
          if (i >= uint32_t(kStages) && !mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) {
            record_status(p.status, kStatusTimeout);
            atomicExch(&flags[0], 1);
            break;
          }
          const int64_t pos = p0 + int64_t(t) * kTile;
          const uint32_t bytes = uint32_t(min(int64_t(kTile), p1 - pos)) * HD * 2u;
          mbar_arrive_expect_tx(&full[s], 2u * bytes);
          bulk_g2s_hint(ks + s * TILE_ELEMS, kbase + pos * HD, bytes, &full[s], once);
          bulk_g2s_hint(vs + s * TILE_ELEMS, vbase + pos * HD, bytes, &full[s], once);
          issued = i + 1;
        }
      }
      __syncwarp();
    } else {  // ------------------------------------------------ consumers
      const int h0 = y * G;
      const uint16_t* qrow = d.q + int64_t(row) * p.q_row;
      uint16_t* orow = d.output + int64_t(row) * p.out_row;
      if (bad && tid == 0) record_status(p.status, kStatusArg);
      uint64_t q2[G][T::DP2];
      if (!bad) load_q<HD, G>(qrow, p.q_head, h0, lane, q2);
      uint64_t o2[G][T::DP2];
#pragma unroll
      for (int gg = 0; gg < G; ++gg)
#pragma unroll
        for (int kk = 0; kk < T::DP2; ++kk) o2[gg][kk] = f2(0.f, 0.f);
      float m_own = -INFINITY, l_own = 0.f;
      for (int t = 0; t < nt; ++t) {
        const uint32_t i = tg + uint32_t(t);
        const int s = int(i % kStages);
        if (*reinterpret_cast<volatile int*>(&flags[0])) break;
        if (!mbar_wait(&full[s], (i / kStages) & 1)) {
          record_status(p.status, kStatusTimeout);
          atomicExch(&flags[0], 1);
          break;
        }
        const int64_t tile_pos = p0 + int64_t(t) * kTile;
        const int vc = int(max(int64_t(0), min(int64_t(4), p1 - tile_pos - warp * 4)));
        if (vc > 0)
          consume_tile<HD, G>(ks + s * TILE_ELEMS, vs + s * TILE_ELEMS, vc, p.scale_log2, q2, o2,
                              m_own, l_own, warp, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      float om[PER_T], ol[PER_T], oo[PER_T];
      merge_warps<HD, G>(ws, o2, m_own, l_own, warp, lane, om, ol, oo);
      if (a == 0 && b == tz) {
        if (!bad) finalize_own<HD, G>(ol, oo, orow, qrow, p.gate_offset, h0);
      } else {
        const int64_t ka = range_of(ustart), kb = range_of(ustart + tz - 1);
        store_partial<HD, G>(p.partials + (k + u) * PSTRIDE, om, ol, oo);
        consumer_sync();  // every partial store of this CTA precedes thread 0's release
        if (tid == 0) {
          __threadfence();
          const unsigned prev = atomicAdd(&p.counters[u], 1u);
          __threadfence();
          flags[1] = (int64_t(prev) == kb - ka);
        }
        consumer_sync();
        if (flags[1]) {
          if (!bad)
            merge_partials<HD, G>(p.partials + (ka + u) * PSTRIDE, int(kb - ka + 1), ws, orow, qrow,
                                  p.gate_offset, h0);
          if (tid == 0) p.counters[u] = 0u;  // leave the workspace reusable
        }
      }
      // the merges wrote the ring's shared memory through the generic proxy;
      // the next segment's bulk copies write it through the async proxy
      sm100::fence_proxy_async_smem();
    }
    tg += uint32_t(nt);
    // the producer starts the next segment's copies once the consumers are
    // done with the ring (tiles and merge scratch)
    asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory");
    g = ustart + b;
    if (g == ubase + hkv * tz) {  // past the row's last KV head
      ++z;
      pre += tz;
    }
  }
  // copies still in flight after a wait ran out: let them land (bounded)
  if (warp == kConsumerWarps && lane == 0 && *reinterpret_cast<volatile int*>(&flags[0])) {
    for (uint32_t i = issued > uint32_t(kStages) ? issued - kStages : 0u; i < issued; ++i)
      mbar_wait(&full[i % kStages], (i / kStages) & 1);
  }
}

// ring (or merge scratch), the ring's barriers, four flags, the ranges
// kernel's scan words
template <int HD, int G>
size_t smem_bytes() {
  using T = Geo<HD, G>;
  return size_t(T::BODY) + 2 * T::kStages * sizeof(uint64_t) + 16 +
         (kThreads / 32 + 2) * sizeof(int64_t);
}

// Largest cluster (16 with non-portable sizes, else 8) that the device can
// co-schedule for this kernel, or 0; probed once per device.
template <int HD, int G>
int cluster_limit(size_t smem) {
  static int cache[64];
  static DeviceFlags probed;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  cudaError_t e = probed.once([&] {
    int best = 0;
    for (int c : {16, 8}) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(c, 1, 1);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = c;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, attn_decode_cluster_kernel<HD, G>, &cfg) == cudaSuccess &&
          n >= 1) {
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

template <int HD, int G>
cudaError_t launch(DecodeParams p, int units_z, bool single, int64_t max_n, int ranges,
                   cudaStream_t st) {
  const size_t smem = smem_bytes<HD, G>();
  static DeviceFlags configured;  // the attributes are set once per device
  cudaError_t e = configured.once([&] {
    cudaError_t r = cudaFuncSetAttribute(attn_decode_ranges_kernel<HD, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(attn_decode_cluster_kernel<HD, G>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(attn_decode_cluster_kernel<HD, G>,
                               cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return r;
  });
  if (e != cudaSuccess) return e;
  // one short sequence: splits of <= 256 positions merged inside a cluster
  const int cmax = single ? cluster_limit<HD, G>(smem) : 0;
  if (cmax > 1) {
    int64_t c = (max_n + cmax - 1) / cmax;
    c = (c + kTile - 1) / kTile * kTile;
    if (c <= 256) {
      p.chunk = int(c);
      p.nsplit = int((max_n + c - 1) / c);
      if (p.nsplit >= 2) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(p.nsplit, p.hkv, units_z);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = p.nsplit;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        // programmatic dependent launch: resident early, K/V prefetched into
        // L2 before griddepcontrol.wait, everything else after it
        at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 2;
        return cudaLaunchKernelEx(&cfg, attn_decode_cluster_kernel<HD, G>, p);
      }
    }
  }
  // balanced ranges over all units
  p.units_z = units_z;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(ranges));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_decode_ranges_kernel<HD, G>, p);
}

}  // namespace

// Positions per split: enough CTAs to cover the SMs several times over
// (load balance across units of unequal length), at least two tiles each.
int decode_chunk(int64_t total_positions, int64_t units, int64_t max_n, int num_sms) {
  // Units of unequal length (a ragged batch) are balanced by about eight
  // waves of splits; when every unit has max_n positions (one sequence, or a
  // batch of equal lengths) a single wave of long splits streams the same
  // bytes with one CTA set-up and a short merge per SM.
  const bool uniform = total_positions >= mul_sat(units, max_n);
  const int64_t target = int64_t(num_sms) * (uniform ? 1 : 8);
  int64_t c = (total_positions + target - 1) / target;
  c = (c + kTile - 1) / kTile * kTile;
  if (c < 2 * kTile) c = 2 * kTile;
  if (c > 8192) c = 8192;
  // the last CTA stages 3G floats per split in the ring (96 or 128 KB): at most
  // 1024 splits per unit
  const int64_t min_chunk = (max_n + kMaxSplits - 1) / kMaxSplits;
  if (c < min_chunk) c = (min_chunk + kTile - 1) / kTile * kTile;
  if (c > max_n) c = (max_n + kTile - 1) / kTile * kTile;
  return int(c);
}

// Ranges of the balanced form: one per resident CTA slot (two per SM for
// groups of up to 4 query heads), at most one per two tiles of the call.
int decode_ranges(int64_t unit_positions, int64_t gqa, int num_sms) {
  const int64_t slots = int64_t(num_sms) * (gqa <= 4 ? 2 : 1);
  const int64_t half_tiles = (unit_positions + kTile - 1) / kTile / 2;
  int64_t r = slots < half_tiles ? slots : half_tiles;
  if (r > kMaxSplits) r = kMaxSplits;
  return int(r < 1 ? 1 : r);
}

size_t decode_partial_floats(int64_t gqa, int64_t head_dim) {
  return size_t(gqa * head_dim + ((2 * gqa + 3) & ~int64_t(3)));
}

cudaError_t launch_attn_decode(const DecodeLaunch& L, cudaStream_t st) {
  cudaError_t mma_err = cudaSuccess;
  if (launch_attn_decode_mma(L, st, &mma_err)) return mma_err;
  if (launch_attn_decode_long(L, st, &mma_err)) return mma_err;
  DecodeParams p;
  p.seqs = L.seqs;
  p.one = L.one;
  p.rows = int(L.rows);
  p.hkv = int(L.hkv);
  p.q_row = L.q_row;
  p.q_head = L.q_head;
  p.out_row = L.out_row;
  p.gate_offset = L.gate_offset;
  p.scale_log2 = L.scale * 1.4426950408889634f;
  p.chunk = L.chunk;
  p.nsplit = L.nsplit;
  p.status = L.status;
  p.counters = L.counters;
  p.partials = L.partials;
  const int z = int(L.nseq * L.rows);
  const bool single = L.seqs == nullptr && L.nseq == 1;
  const int64_t max_n = L.one.past + L.rows;
#define HB_DECODE_CASE(HD_, G_) \
  if (L.head_dim == HD_ && L.gqa == G_) return launch<HD_, G_>(p, z, single, max_n, L.ranges, st);
  HB_DECODE_CASE(256, 1) HB_DECODE_CASE(256, 2) HB_DECODE_CASE(256, 4) HB_DECODE_CASE(256, 8)
  HB_DECODE_CASE(128, 1) HB_DECODE_CASE(128, 2) HB_DECODE_CASE(128, 4) HB_DECODE_CASE(128, 8)
#undef HB_DECODE_CASE
  return cudaErrorInvalidValue;
}

bool decode_serves(int64_t head_dim, int64_t gqa) {
  return (head_dim == 128 || head_dim == 256) && (gqa == 1 || gqa == 2 || gqa == 4 || gqa == 8);
}

}  // namespace hb
