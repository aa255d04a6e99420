// mount.cu -- routing of a model pass to the kernels: the per-layer binding
// the reference's lowering makes when it mounts a regime
// (src/jit/model/mounted.rs:237-380), and one call per layer mixer.
//
// A layer is routed to its slice of the sequence's state exactly as the
// lowering mounts it: an attention layer to the KV cache at kv_offsets[layer]
// (keys, then values n_kv_heads x stride later; mounted.rs:337-340), the d-th
// DeltaNet layer to the conv and recurrent slots at d x their strides
// (mounted.rs:283-293).  The refusals are the lowering's: a DeltaNet layer
// with a KV cache or whose state does not fit its slots, an attention layer
// whose cache is not heads x kv_reserve x head_dim.
//
// Host code only: each mixer call issues the C entry points of its nodes in
// order on one stream, with the workspaces and scratch the mount allocated
// once.

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <vector>

#include "hb_internal.h"

struct hb_mount {
  hb_mount_desc desc;
  hb_state_geometry geo;
  hb_state_buffers state;
  std::vector<int64_t> kv_offsets;
  std::vector<int32_t> kinds;
  void* attn_ws = nullptr;
  size_t attn_ws_bytes = 0;
  void* gdn_ws = nullptr;
  size_t gdn_ws_bytes = 0;
  void* front_ws = nullptr;
  float* beta = nullptr;
  float* decay = nullptr;
  float* rec_out = nullptr;
  // Set by the first failure after a call entered execution (a node
  // launched, so state may be half updated) or by a device-side status;
  // every later mixer call is refused with it until hb_mount_reset, as a
  // failed call poisons the reference's execution session until its owner
  // resets or restores the model (src/jit/execution/runtime.rs:144-151,
  // 310-327; src/jit/execution/program.rs:289).
  hb_status poison = HB_OK;
  char poison_msg[256] = "";
};

namespace hb {
namespace {

constexpr float kDeltaL2Eps = 1e-6f;  // DN_L2_EPS (src/jit/schedule/deltanet.rs:69)

hb_status check_desc(const hb_mount_desc* d) {
  if (!d || !d->geometry || !d->state || !d->layer_kinds) return fail(HB_ERR_ARG, "mount description is incomplete");
  hb_status r = check_state_geometry(d->geometry);
  if (r != HB_OK) return r;
  const hb_state_geometry* g = d->geometry;
  // the workspaces are sized over every block size up to max_rows (create)
  constexpr int64_t kMaxBlockRows = int64_t(1) << 20;
  if (d->max_rows < 1 || d->max_rows > g->kv_reserve || d->max_rows > kMaxBlockRows)
    return fail(HB_ERR_ARG, "max_rows must be in 1 .. min(kv_reserve, 2^20)");
  bool any_attn = false, any_delta = false;
  for (int64_t l = 0; l < g->n_layers; l++) {
    if (d->layer_kinds[l] == HB_LAYER_ATTENTION) any_attn = true;
    else if (d->layer_kinds[l] == HB_LAYER_DELTA) any_delta = true;
    else return fail(HB_ERR_ARG, "layer %lld: unknown mixer kind %d", static_cast<long long>(l), d->layer_kinds[l]);
  }
  if (any_attn) {
    if ((r = check_spec(&d->attn)) != HB_OK) return r;
    if (d->attn.heads / d->attn.gqa != g->kv_heads)
      return fail(HB_DECLINE_GEOMETRY, "attention heads / gqa differ from the cache's kv_heads");
    if (!front_serves(d->attn.head_dim, d->rotary))
      return fail(HB_DECLINE_HEAD_DIM, "head norm / RoPE not served at head_dim %lld, rotary %lld",
                  static_cast<long long>(d->attn.head_dim), static_cast<long long>(d->rotary));
    if (!d->cos || !d->sin) return fail(HB_ERR_ARG, "missing RoPE table");
    if (!(d->attn_scale > 0.f) || !std::isfinite(d->attn_scale)) return fail(HB_ERR_ARG, "invalid attention scale");
    if (!d->state->kv) return fail(HB_ERR_ARG, "null KV buffer");
  }
  if (!(d->norm_eps >= 0.f) || !std::isfinite(d->norm_eps)) return fail(HB_ERR_ARG, "invalid norm eps");
  if (any_delta) {
    const hb_gdn_shape& s = d->delta;
    const int64_t lim = int64_t(1) << 16;
    if (s.nk <= 0 || s.nv <= 0 || s.nv % s.nk || s.hkd <= 0 || s.hvd <= 0 || s.nk > lim || s.nv > lim ||
        s.hkd > lim || s.hvd > lim)
      return fail(HB_DECLINE_GEOMETRY, "invalid generated DeltaNet geometry");
    if (!gdn_front_serves(2 * s.nk * s.hkd + s.nv * s.hvd, d->conv_kernel) || !gdn_decode_serves(s))
      return fail(HB_DECLINE_HEAD_DIM, "DeltaNet geometry not served (conv width a multiple of 4, ck 1..8, "
                                       "hkd 64/128, hvd a multiple of 32)");
    if (!d->state->dn_conv || !d->state->dn_recurrent) return fail(HB_ERR_ARG, "null DeltaNet state buffer");
  }
  // the lowering's per-layer checks (mounted.rs:253-280, 300-313)
  int64_t delta_layer = 0;
  for (int64_t l = 0; l < g->n_layers; l++) {
    const int64_t stride = (g->kv_offsets[l + 1] - g->kv_offsets[l]) / (2 * g->kv_heads);
    if (d->layer_kinds[l] == HB_LAYER_DELTA) {
      const hb_gdn_shape& s = d->delta;
      const int64_t conv_need = (2 * s.nk * s.hkd + s.nv * s.hvd) * d->conv_kernel;
      const int64_t rec_need = s.nv * s.hkd * s.hvd;
      if (stride != 0 || d->conv_stride <= 0 || d->recurrent_stride <= 0 || conv_need > d->conv_stride ||
          rec_need > d->recurrent_stride || (delta_layer + 1) * d->conv_stride > g->conv_len ||
          (delta_layer + 1) * d->recurrent_stride > g->recurrent_len)
        return fail(HB_DECLINE_GEOMETRY, "generated layer %lld: DeltaNet state or absent-KV plan mismatch",
                    static_cast<long long>(l));
      delta_layer++;
    } else if (stride == 0 || stride / g->kv_reserve != d->attn.head_dim) {
      return fail(HB_DECLINE_GEOMETRY, "generated layer %lld: KV geometry mismatch", static_cast<long long>(l));
    }
  }
  return HB_OK;
}

hb_layer_route route_of(const hb_mount_desc* d, int64_t layer) {
  const hb_state_geometry* g = d->geometry;
  hb_layer_route r{};
  r.kind = d->layer_kinds[layer];
  r.delta_index = -1;
  if (r.kind == HB_LAYER_ATTENTION) {
    r.kv_stride = (g->kv_offsets[layer + 1] - g->kv_offsets[layer]) / (2 * g->kv_heads);
    r.keys = d->state->kv + g->kv_offsets[layer];
    r.values = r.keys + g->kv_heads * r.kv_stride;
  } else {
    int32_t idx = 0;
    for (int64_t l = 0; l < layer; l++) idx += d->layer_kinds[l] == HB_LAYER_DELTA;
    r.delta_index = idx;
    r.conv_state = d->state->dn_conv + int64_t(idx) * d->conv_stride;
    r.recurrent_state = d->state->dn_recurrent + int64_t(idx) * d->recurrent_stride;
  }
  return r;
}

void release(hb_mount* m) {
  for (void* p : {m->attn_ws, m->gdn_ws, m->front_ws, static_cast<void*>(m->beta), static_cast<void*>(m->decay),
                  static_cast<void*>(m->rec_out)})
    if (p) cudaFree(p);
  delete m;
}

// Records the first failure of a call that entered execution and returns it.
hb_status poison(hb_mount* m, hb_status r) {
  if (r != HB_OK && m->poison == HB_OK) {
    m->poison = r;
    snprintf(m->poison_msg, sizeof m->poison_msg, "%s", hb_last_error());
  }
  return r;
}

hb_status refuse_if_poisoned(const hb_mount* m) {
  if (m->poison == HB_OK) return HB_OK;
  return fail(m->poison, "the mount needs hb_mount_reset after a failed call (%s: %s)",
              hb_status_name(m->poison), m->poison_msg);
}

// A node's status once an earlier node of the same call has launched, or
// when the node itself failed past its checks (a launch or device error):
// either way the state may be half updated.
hb_status after_entry(hb_mount* m, hb_status r, bool entered) {
  if (r == HB_OK) return r;
  if (entered || r == HB_ERR_CUDA || r == HB_ERR_TIMEOUT || r == HB_ERR_NCCL) return poison(m, r);
  return r;
}

hb_status layer_of(hb_mount* m, int64_t layer, int32_t kind, hb_layer_route* r) {
  if (!m) return fail(HB_ERR_ARG, "mount is null");
  if (layer < 0 || layer >= m->geo.n_layers) return fail(HB_ERR_ARG, "layer %lld out of range", static_cast<long long>(layer));
  if (m->kinds[layer] != kind) return fail(HB_ERR_ARG, "layer %lld has the other mixer kind", static_cast<long long>(layer));
  *r = route_of(&m->desc, layer);
  return HB_OK;
}

}  // namespace
}  // namespace hb

using namespace hb;

hb_status hb_mount_route(const hb_mount_desc* d, int64_t layer, hb_layer_route* route) {
  hb_status r = check_desc(d);
  if (r != HB_OK) return r;
  if (!route) return fail(HB_ERR_ARG, "route is null");
  if (layer < 0 || layer >= d->geometry->n_layers)
    return fail(HB_ERR_ARG, "layer %lld out of range", static_cast<long long>(layer));
  *route = route_of(d, layer);
  return HB_OK;
}

hb_status hb_mount_create(const hb_mount_desc* d, hb_mount** out) {
  if (!out) return fail(HB_ERR_ARG, "mount output is null");
  *out = nullptr;
  hb_status r = check_desc(d);
  if (r != HB_OK) return r;
  hb_mount* m = new hb_mount;
  m->desc = *d;
  m->geo = *d->geometry;
  m->state = *d->state;
  m->kv_offsets.assign(d->geometry->kv_offsets, d->geometry->kv_offsets + d->geometry->n_layers + 1);
  m->geo.kv_offsets = m->kv_offsets.data();
  m->kinds.assign(d->layer_kinds, d->layer_kinds + d->geometry->n_layers);
  m->desc.geometry = &m->geo;
  m->desc.state = &m->state;
  m->desc.layer_kinds = m->kinds.data();
  const bool any_attn = std::count(m->kinds.begin(), m->kinds.end(), HB_LAYER_ATTENTION) > 0;
  const bool any_delta = std::count(m->kinds.begin(), m->kinds.end(), HB_LAYER_DELTA) > 0;
  const int64_t res = m->geo.kv_reserve, R = d->max_rows;
  // workspaces: the largest any block of up to max_rows rows at any position needs
  if (any_attn) {
    size_t need = kWsHeader;
    hb_attn_call c{};
    c.kv_stride = res * d->attn.head_dim;
    c.capacity = res;
    for (int64_t rows = 1; rows <= R; rows++) {
      c.rows = rows;
      c.past = res - rows;
      need = std::max(need, hb_attn_prefill_workspace_bytes(&d->attn, &c));
      need = std::max(need, hb_attn_decode_workspace_bytes(&d->attn, &c));
    }
    m->attn_ws_bytes = need;
  }
  if (any_delta) {
    size_t need = kWsHeader;
    for (int64_t rows = 1; rows <= R; rows++) need = std::max(need, hb_gdn_prefill_workspace_bytes(&d->delta, rows));
    m->gdn_ws_bytes = need;
  }
  cudaError_t e = cudaSuccess;
  if (any_attn) e = cudaMalloc(&m->attn_ws, m->attn_ws_bytes);
  if (e == cudaSuccess && any_delta) {
    const size_t nv = size_t(d->delta.nv), vd = nv * size_t(d->delta.hvd);
    e = cudaMalloc(&m->gdn_ws, m->gdn_ws_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&m->front_ws, kWsHeader + kRowCounterBytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&m->beta), 4 * size_t(R) * nv);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&m->decay), 4 * size_t(R) * nv);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&m->rec_out), 4 * size_t(R) * vd);
  }
  if (e == cudaSuccess && m->attn_ws) e = cudaMemset(m->attn_ws, 0, m->attn_ws_bytes);
  if (e == cudaSuccess && m->gdn_ws) e = cudaMemset(m->gdn_ws, 0, m->gdn_ws_bytes);
  if (e == cudaSuccess && m->front_ws) e = cudaMemset(m->front_ws, 0, kWsHeader + kRowCounterBytes);
  if (e != cudaSuccess) {
    release(m);
    return cuda_fail(e, "hb_mount_create");
  }
  *out = m;
  return HB_OK;
}

void hb_mount_destroy(hb_mount* m) {
  if (m) release(m);
}

hb_status hb_mount_status(hb_mount* m, hb_stream_t stream) {
  if (!m) return fail(HB_ERR_ARG, "mount is null");
  hb_status r = HB_OK;
  if (m->attn_ws && (r = hb_workspace_status(m->attn_ws, m->attn_ws_bytes, stream)) != HB_OK)
    return poison(m, r);
  if (m->gdn_ws && (r = hb_workspace_status(m->gdn_ws, m->gdn_ws_bytes, stream)) != HB_OK)
    return poison(m, r);
  if (m->front_ws && (r = hb_workspace_status(m->front_ws, kWsHeader, stream)) != HB_OK)
    return poison(m, r);
  return refuse_if_poisoned(m);
}

int hb_mount_needs_reset(const hb_mount* m) { return m && m->poison != HB_OK; }

hb_status hb_mount_reset(hb_mount* m, hb_stream_t stream) {
  if (!m) return fail(HB_ERR_ARG, "mount is null");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  for (void* ws : {m->attn_ws, m->gdn_ws, m->front_ws})
    if (ws && e == cudaSuccess) e = cudaMemsetAsync(ws, 0, kWsHeader, st);
  // the one-row DeltaNet launches' counters (a failed call may have left
  // some counted)
  if (m->front_ws && e == cudaSuccess)
    e = cudaMemsetAsync(static_cast<char*>(m->front_ws) + kWsHeader, 0, kRowCounterBytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "hb_mount_reset");
  m->poison = HB_OK;
  m->poison_msg[0] = 0;
  return HB_OK;
}

hb_status hb_mount_attention(hb_mount* m, int64_t layer, const hb_mount_attention_call* c, hb_stream_t stream) {
  hb_layer_route rt;
  hb_status r = layer_of(m, layer, HB_LAYER_ATTENTION, &rt);
  if (r != HB_OK) return r;
  if (!c) return fail(HB_ERR_ARG, "attention call is null");
  const int64_t res = m->geo.kv_reserve;
  if (c->rows < 1 || c->rows > m->desc.max_rows) return fail(HB_ERR_ARG, "rows outside 1 .. max_rows");
  if (c->pos < 0 || c->pos + c->rows > res) return fail(HB_ERR_ARG, "positions beyond the cache");
  if ((r = refuse_if_poisoned(m)) != HB_OK) return r;
  const hb_attn_spec& spec = m->desc.attn;
  const int64_t hd = spec.head_dim;
  // head-norm-rope of q and k, kv-append (lowering.rs:549-592)
  hb_kv_spec kv{};
  kv.heads = m->geo.kv_heads;
  kv.head_dim = hd;
  kv.stride = rt.kv_stride;
  kv.capacity = res;
  kv.max_batch = m->desc.max_rows;
  hb_front_spec front{};
  front.rotary = m->desc.rotary;
  front.eps = m->desc.norm_eps;
  front.gemma = m->desc.gemma;
  hb_front_call fc{};
  fc.q = c->q;
  fc.k = c->k;
  fc.v = c->v;
  fc.q_norm = c->q_norm;
  fc.k_norm = c->k_norm;
  fc.cos = m->desc.cos;
  fc.sin = m->desc.sin;
  fc.keys = rt.keys;
  fc.values = rt.values;
  fc.rows = c->rows;
  fc.past = c->pos;
  // attention + output gate (lowering.rs:600-666), by regime
  hb_attn_call ac{};
  ac.q = c->q;
  ac.keys = rt.keys;
  ac.values = rt.values;
  ac.output = c->out;
  ac.rows = c->rows;
  ac.past = c->pos;
  ac.kv_stride = rt.kv_stride;
  ac.capacity = res;
  ac.scale = m->desc.attn_scale;
  if (c->rows == 1) {
    // a decode row over a long cache: the decode kernel runs the front end
    // too (both nodes checked first), in one launch
    bool served = false;
    r = attn_layer_row(&spec, &kv, &front, &fc, &ac, m->attn_ws, m->attn_ws_bytes, stream, &served);
    if (served) return after_entry(m, r, false);
  }
  if ((r = hb_attn_front(&spec, &kv, &front, &fc, stream)) != HB_OK) return after_entry(m, r, false);
  if (c->rows == 1)
    return after_entry(m, hb_attn_decode(&spec, &ac, m->attn_ws, m->attn_ws_bytes, stream), true);
  return after_entry(m, hb_attn_prefill(&spec, &ac, m->attn_ws, m->attn_ws_bytes, stream), true);
}

hb_status hb_mount_delta(hb_mount* m, int64_t layer, const hb_mount_delta_call* c, hb_stream_t stream) {
  hb_layer_route rt;
  hb_status r = layer_of(m, layer, HB_LAYER_DELTA, &rt);
  if (r != HB_OK) return r;
  if (!c) return fail(HB_ERR_ARG, "DeltaNet call is null");
  if (c->rows < 1 || c->rows > m->desc.max_rows) return fail(HB_ERR_ARG, "rows outside 1 .. max_rows");
  if ((r = refuse_if_poisoned(m)) != HB_OK) return r;
  const hb_gdn_shape& shape = m->desc.delta;
  // delta-causal-convolution + the gates of delta-l2-gates (lowering.rs:904-961)
  hb_gdn_front_call fc{};
  fc.qkv = c->qkv;
  fc.conv_state = rt.conv_state;
  fc.conv_weight = c->conv_weight;
  fc.ab = c->ab;
  fc.dt_bias = c->dt_bias;
  fc.a_log = c->a_log;
  fc.beta = m->beta;
  fc.decay = m->decay;
  fc.rows = c->rows;
  fc.ck = m->desc.conv_kernel;
  // the L2 of delta-l2-gates + delta-causal-recurrence (lowering.rs:935-986)
  hb_gdn_call gc{};
  gc.state = rt.recurrent_state;
  gc.output = m->rec_out;
  gc.qkv = c->qkv;
  gc.beta = m->beta;
  gc.decay = m->decay;
  gc.rows = c->rows;
  gc.l2 = 1;
  gc.eps = kDeltaL2Eps;
  // delta-gated-norm (lowering.rs:987-1010)
  hb_gdn_norm_call nc{};
  nc.x = m->rec_out;
  nc.z = c->z;
  nc.weight = c->norm_weight;
  nc.out = c->out;
  nc.out_f32 = c->out_f32;
  nc.rows = c->rows;
  nc.eps = m->desc.norm_eps;
  if (c->rows == 1) {
    // a decode row: the three nodes in one launch where the shape allows
    // (every node's checks first, so a refusal launches nothing)
    bool served = false;
    r = gdn_layer_row(&shape, &fc, &gc, &nc, m->front_ws, kWsHeader + kRowCounterBytes,
                      static_cast<int*>(m->gdn_ws), stream, &served);
    if (served) return after_entry(m, r, false);
  }
  if ((r = hb_gdn_front(&shape, &fc, m->front_ws, kWsHeader, stream)) != HB_OK)
    return after_entry(m, r, false);
  if ((r = hb_gdn_prefill(&shape, &gc, m->gdn_ws, m->gdn_ws_bytes, stream)) != HB_OK)
    return after_entry(m, r, true);
  return after_entry(m, hb_gdn_gated_norm(&shape, &nc, stream), true);
}
