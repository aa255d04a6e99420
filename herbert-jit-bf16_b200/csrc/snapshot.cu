// snapshot.cu -- snapshot / restore of a sequence's device state (KV cache,
// DeltaNet conv and recurrent states, last logits) in the reference's
// serialized Instantaneous format, version 1 (src/jit/model.rs:100-326,
// 675-857).
//
// The slot is the serialized image in host memory: the header and every
// length are written by the host, and the payload moves by DMA straight into
// (take) or out of (restore) its place in the image -- one 2-D copy per
// (layer, K|V half) covers the kv_heads rows of `pos` positions with the
// device pitch on one side and the snapshot's pitch on the other.  Nothing
// is staged on the device and nothing is allocated.
//
// Host code only (CUDA runtime copies); every refusal happens before the
// first copy.

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "hb_internal.h"

namespace hb {
namespace {

static_assert(__BYTE_ORDER__ == __ORDER_LITTLE_ENDIAN__, "the image format is little-endian");

constexpr uint32_t kSnapshotFormat = 1;                  // SNAPSHOT_FORMAT, model.rs:103
constexpr uint64_t kMaxBlockBytes = uint64_t(64) << 30;  // MAX_BLOCK_SNAPSHOT, model.rs:108

uint64_t rd64(const uint8_t* p) {
  uint64_t v;
  std::memcpy(&v, p, 8);
  return v;
}
void wr64(uint8_t* p, uint64_t v) { std::memcpy(p, &v, 8); }

// One validated geometry: per layer the head stride (elements) and head_dim.
struct Geo {
  const hb_state_geometry* g;
  bool ok = false;
  int64_t stride(int64_t l) const { return (g->kv_offsets[l + 1] - g->kv_offsets[l]) / (2 * g->kv_heads); }
  int64_t head_dim(int64_t l) const { return stride(l) / g->kv_reserve; }
  int64_t cap(int64_t l, int64_t max_positions) const {
    return stride(l) == 0 ? 0 : std::min(g->kv_reserve, max_positions);
  }
};

hb_status check_geometry_(const hb_state_geometry* g, Geo* out) {
  out->g = g;
  if (!g || !g->kv_offsets) return fail(HB_ERR_ARG, "state geometry or kv_offsets is null");
  const int64_t lim = int64_t(1) << 40;
  if (g->n_layers < 0 || g->n_layers > 65536 || g->kv_heads <= 0 || g->kv_heads > 65536 ||
      g->kv_reserve <= 0 || g->kv_reserve > (int64_t(1) << 31) || g->conv_len < 0 ||
      g->conv_len > lim || g->recurrent_len < 0 || g->recurrent_len > lim || g->logits_len < 0 ||
      g->logits_len > lim)
    return fail(HB_DECLINE_GEOMETRY, "invalid state geometry");
  if (g->kv_offsets[0] != 0) return fail(HB_DECLINE_GEOMETRY, "kv_offsets[0] must be 0");
  for (int64_t l = 0; l < g->n_layers; l++) {
    const int64_t d = g->kv_offsets[l + 1] - g->kv_offsets[l];
    if (d < 0 || d > lim || d % (2 * g->kv_heads * g->kv_reserve))
      return fail(HB_DECLINE_GEOMETRY, "kv_offsets of layer %lld are not 2 x kv_heads x kv_reserve x head_dim",
                  static_cast<long long>(l));
  }
  out->ok = true;
  return HB_OK;
}

// The image's sections, located without copying anything.
struct Image {
  const uint8_t* base = nullptr;
  size_t bytes = 0;
  size_t at = 0;
  uint64_t n_kv_offsets = 0, n_snap_offsets = 0, n_snap_positions = 0;
  size_t kv_offsets_at = 0, snap_offsets_at = 0, snap_positions_at = 0;
  uint64_t kv_n = 0, logits_n = 0, conv_n = 0, rec_n = 0;
  size_t kv_at = 0, logits_at = 0, conv_at = 0, rec_at = 0;
  uint64_t pos = 0;

  bool need(size_t n) const { return n <= bytes && at <= bytes - n; }
  // length (model.rs:110-121): the element count, refused beyond 64 GiB
  hb_status block(size_t elem, uint64_t* n, size_t* data_at) {
    if (!need(8)) return fail(HB_ERR_ARG, "snapshot image truncated");
    *n = rd64(base + at);
    at += 8;
    if (*n > kMaxBlockBytes / elem) return fail(HB_ERR_ARG, "snapshot block of %llu elements: beyond the ceiling",
                                                static_cast<unsigned long long>(*n));
    if (!need(*n * elem)) return fail(HB_ERR_ARG, "snapshot image truncated");
    *data_at = at;
    at += *n * elem;
    return HB_OK;
  }
  uint64_t u(size_t array_at, uint64_t i) const { return rd64(base + array_at + 8 * i); }
};

// Instantaneous::read (model.rs:291-316).
hb_status parse(const void* image, size_t bytes, Image* im) {
  if (!image) return fail(HB_ERR_ARG, "snapshot image is null");
  im->base = static_cast<const uint8_t*>(image);
  im->bytes = bytes;
  if (!im->need(4)) return fail(HB_ERR_ARG, "snapshot image truncated");
  uint32_t v;
  std::memcpy(&v, im->base, 4);
  if (v != kSnapshotFormat) return fail(HB_ERR_ARG, "snapshot of another version of format (%u)", v);
  im->at = 4;
  hb_status r;
  if ((r = im->block(8, &im->n_kv_offsets, &im->kv_offsets_at)) != HB_OK) return r;
  if ((r = im->block(8, &im->n_snap_offsets, &im->snap_offsets_at)) != HB_OK) return r;
  if ((r = im->block(8, &im->n_snap_positions, &im->snap_positions_at)) != HB_OK) return r;
  if ((r = im->block(2, &im->kv_n, &im->kv_at)) != HB_OK) return r;
  if ((r = im->block(2, &im->logits_n, &im->logits_at)) != HB_OK) return r;
  if ((r = im->block(4, &im->conv_n, &im->conv_at)) != HB_OK) return r;
  if ((r = im->block(4, &im->rec_n, &im->rec_at)) != HB_OK) return r;
  if (!im->need(8)) return fail(HB_ERR_ARG, "snapshot image truncated");
  im->pos = rd64(im->base + im->at);
  im->at += 8;
  return HB_OK;
}

// The snapshot's own offsets must describe its kv block (a corrupted image
// must not steer a copy out of bounds): snap_offsets[0] = 0, each layer
// 2 x kv_heads x snap_positions x head_dim, the last one the kv length, and
// pos within every slot.  Against the geometry that compatible_snapshot
// (model.rs:709-723) compares.
hb_status check_against(const Geo& G, const Image& im) {
  const hb_state_geometry* g = G.g;
  const uint64_t L = static_cast<uint64_t>(g->n_layers);
  bool same = im.n_kv_offsets == L + 1 && im.conv_n == uint64_t(g->conv_len) &&
              im.rec_n == uint64_t(g->recurrent_len) && im.logits_n == uint64_t(g->logits_len);
  for (uint64_t i = 0; same && i <= L; i++) same = im.u(im.kv_offsets_at, i) == uint64_t(g->kv_offsets[i]);
  if (!same)
    return fail(HB_DECLINE_GEOMETRY,
                "the snapshot has been reserved for a different Runner geometry (KV cache, pass, or model differ)");
  if (im.n_snap_offsets != L + 1 || im.n_snap_positions != L || im.u(im.snap_offsets_at, 0) != 0)
    return fail(HB_ERR_ARG, "corrupted snapshot: slot offsets");
  for (uint64_t l = 0; l < L; l++) {
    const uint64_t cap = im.u(im.snap_positions_at, l);
    const uint64_t hd = uint64_t(G.head_dim(int64_t(l)));
    const uint64_t lo = im.u(im.snap_offsets_at, l), hi = im.u(im.snap_offsets_at, l + 1);
    if (cap > uint64_t(g->kv_reserve) || (hd == 0 && cap != 0) || hi < lo ||
        hi - lo != 2 * uint64_t(g->kv_heads) * cap * hd || (hd != 0 && im.pos > cap))
      return fail(HB_ERR_ARG, "corrupted snapshot: layer %llu", static_cast<unsigned long long>(l));
  }
  if (im.u(im.snap_offsets_at, L) != im.kv_n) return fail(HB_ERR_ARG, "corrupted snapshot: kv length");
  return HB_OK;
}

size_t image_bytes_for(const Geo& G, int64_t max_positions) {
  const hb_state_geometry* g = G.g;
  size_t kv = 0;
  for (int64_t l = 0; l < g->n_layers; l++)
    kv += size_t(2) * g->kv_heads * G.cap(l, max_positions) * G.head_dim(l);
  const size_t L = size_t(g->n_layers);
  return 4 + (8 + 8 * (L + 1)) * 2 + (8 + 8 * L) + (8 + 2 * kv) + (8 + 2 * size_t(g->logits_len)) +
         (8 + 4 * size_t(g->conv_len)) + (8 + 4 * size_t(g->recurrent_len)) + 8;
}

cudaError_t copy_flat(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t st) {
  return bytes ? cudaMemcpyAsync(dst, src, bytes, kind, st) : cudaSuccess;
}

}  // namespace

hb_status check_state_geometry(const hb_state_geometry* g) {
  Geo G;
  return check_geometry_(g, &G);
}

}  // namespace hb

using namespace hb;

size_t hb_snapshot_bytes(const hb_state_geometry* g, int64_t max_positions) {
  Geo G;
  if (check_geometry_(g, &G) != HB_OK || max_positions < 0) return 0;
  return image_bytes_for(G, max_positions);
}

hb_status hb_snapshot_take(const hb_state_geometry* g, const hb_state_buffers* b, int64_t pos,
                           int64_t max_positions, void* image, size_t image_bytes, hb_stream_t stream) {
  Geo G;
  hb_status r = check_geometry_(g, &G);
  if (r != HB_OK) return r;
  if (!b || !image) return fail(HB_ERR_ARG, "state buffers or image is null");
  if (pos < 0 || max_positions < 0 || pos > g->kv_reserve)
    return fail(HB_ERR_ARG, "position %lld outside the cache", static_cast<long long>(pos));
  // snapshot_take's named refusal (model.rs:752-758): never a silent truncation
  for (int64_t l = 0; l < g->n_layers; l++)
    if (G.stride(l) && pos > G.cap(l, max_positions))
      return fail(HB_ERR_ARG,
                  "snapshot rejected: layer %lld holds %lld positions, the slot buffer holds %lld "
                  "(increase positions_max)",
                  static_cast<long long>(l), static_cast<long long>(pos),
                  static_cast<long long>(G.cap(l, max_positions)));
  const size_t need = image_bytes_for(G, max_positions);
  if (image_bytes < need) return fail(HB_ERR_ARG, "image of %zu bytes, the slot needs %zu", image_bytes, need);
  const int64_t kv_total = g->kv_offsets[g->n_layers];
  if ((kv_total && !b->kv) || (g->conv_len && !b->dn_conv) || (g->recurrent_len && !b->dn_recurrent) ||
      (g->logits_len && !b->logits))
    return fail(HB_ERR_ARG, "null state buffer");

  // Instantaneous::write_to (model.rs:270-287), the header by the host
  uint8_t* out = static_cast<uint8_t*>(image);
  size_t at = 0;
  std::memcpy(out, &kSnapshotFormat, 4);
  at = 4;
  const int64_t L = g->n_layers;
  wr64(out + at, uint64_t(L + 1));
  at += 8;
  for (int64_t i = 0; i <= L; i++, at += 8) wr64(out + at, uint64_t(g->kv_offsets[i]));
  wr64(out + at, uint64_t(L + 1));
  at += 8;
  uint64_t snap = 0;
  for (int64_t l = 0; l <= L; l++, at += 8) {
    wr64(out + at, snap);
    if (l < L) snap += uint64_t(2) * g->kv_heads * G.cap(l, max_positions) * G.head_dim(l);
  }
  wr64(out + at, uint64_t(L));
  at += 8;
  for (int64_t l = 0; l < L; l++, at += 8) wr64(out + at, uint64_t(G.cap(l, max_positions)));
  wr64(out + at, snap);
  at += 8;
  uint8_t* kv_img = out + at;
  at += 2 * snap;
  wr64(out + at, uint64_t(g->logits_len));
  uint8_t* logits_img = out + at + 8;
  at += 8 + 2 * size_t(g->logits_len);
  wr64(out + at, uint64_t(g->conv_len));
  uint8_t* conv_img = out + at + 8;
  at += 8 + 4 * size_t(g->conv_len);
  wr64(out + at, uint64_t(g->recurrent_len));
  uint8_t* rec_img = out + at + 8;
  at += 8 + 4 * size_t(g->recurrent_len);
  wr64(out + at, uint64_t(pos));

  // the payload: per owning layer and half, `pos` positions of every head
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint64_t snap_at = 0;
  for (int64_t l = 0; l < L; l++) {
    const int64_t stride = G.stride(l), hd = G.head_dim(l), cap = G.cap(l, max_positions);
    if (stride == 0) continue;
    const int64_t snap_st = cap * hd;
    for (int half = 0; half < 2; half++) {
      uint8_t* dst0 = kv_img + 2 * (snap_at + uint64_t(half) * g->kv_heads * snap_st);
      const uint16_t* src0 = b->kv + g->kv_offsets[l] + int64_t(half) * g->kv_heads * stride;
      if (cap > pos)  // positions beyond pos: the zeros of a fresh slot
        for (int64_t h = 0; h < g->kv_heads; h++)
          std::memset(dst0 + 2 * (h * snap_st + pos * hd), 0, size_t(2) * (cap - pos) * hd);
      if (pos > 0) {
        cudaError_t e = cudaMemcpy2DAsync(dst0, size_t(2) * snap_st, src0, size_t(2) * stride,
                                          size_t(2) * pos * hd, size_t(g->kv_heads), cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) return cuda_fail(e, "snapshot kv copy");
      }
    }
    snap_at += uint64_t(2) * g->kv_heads * snap_st;
  }
  cudaError_t e = copy_flat(logits_img, b->logits, 2 * size_t(g->logits_len), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = copy_flat(conv_img, b->dn_conv, 4 * size_t(g->conv_len), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess)
    e = copy_flat(rec_img, b->dn_recurrent, 4 * size_t(g->recurrent_len), cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return cuda_fail(e, "snapshot state copy");
  return HB_OK;
}

hb_status hb_snapshot_restore(const hb_state_geometry* g, const hb_state_buffers* b, const void* image,
                              size_t image_bytes, int64_t p, hb_stream_t stream) {
  Geo G;
  hb_status r = check_geometry_(g, &G);
  if (r != HB_OK) return r;
  if (!b) return fail(HB_ERR_ARG, "state buffers are null");
  Image im;
  if ((r = parse(image, image_bytes, &im)) != HB_OK) return r;
  if ((r = check_against(G, im)) != HB_OK) return r;
  // restore_from's named refusals (model.rs:786-810)
  if (p < 0 || uint64_t(p) > im.pos)
    return fail(HB_ERR_ARG, "restoration refused: p=%lld beyond snapshot (%llu positions)",
                static_cast<long long>(p), static_cast<unsigned long long>(im.pos));
  if (uint64_t(p) < im.pos && g->recurrent_len > 0)
    return fail(HB_ERR_ARG,
                "restoration refused: the recurrent state (DeltaNet) is at position %llu, it does not "
                "revert to p=%lld; only an EXACT prefix is restorable on this model",
                static_cast<unsigned long long>(im.pos), static_cast<long long>(p));
  const int64_t kv_total = g->kv_offsets[g->n_layers];
  if ((kv_total && !b->kv) || (g->conv_len && !b->dn_conv) || (g->recurrent_len && !b->dn_recurrent) ||
      (g->logits_len && !b->logits))
    return fail(HB_ERR_ARG, "null state buffer");

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int64_t l = 0; l < g->n_layers; l++) {
    const int64_t stride = G.stride(l), hd = G.head_dim(l);
    if (stride == 0 || p == 0) continue;
    const int64_t snap_st = int64_t(im.u(im.snap_positions_at, uint64_t(l))) * hd;
    const uint64_t snap_at = im.u(im.snap_offsets_at, uint64_t(l));
    for (int half = 0; half < 2; half++) {
      const uint8_t* src0 = im.base + im.kv_at + 2 * (snap_at + uint64_t(half) * g->kv_heads * snap_st);
      uint16_t* dst0 = b->kv + g->kv_offsets[l] + int64_t(half) * g->kv_heads * stride;
      cudaError_t e = cudaMemcpy2DAsync(dst0, size_t(2) * stride, src0, size_t(2) * snap_st,
                                        size_t(2) * p * hd, size_t(g->kv_heads), cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) return cuda_fail(e, "restore kv copy");
    }
  }
  cudaError_t e = copy_flat(b->logits, im.base + im.logits_at, 2 * im.logits_n, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = copy_flat(b->dn_conv, im.base + im.conv_at, 4 * im.conv_n, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = copy_flat(b->dn_recurrent, im.base + im.rec_at, 4 * im.rec_n, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "restore state copy");
  return HB_OK;
}

hb_status hb_snapshot_info(const void* image, size_t image_bytes, int64_t* pos, int32_t* restorable_below) {
  Image im;
  hb_status r = parse(image, image_bytes, &im);
  if (r != HB_OK) return r;
  if (im.pos > uint64_t(INT64_MAX)) return fail(HB_ERR_ARG, "corrupted snapshot: position");
  if (pos) *pos = static_cast<int64_t>(im.pos);
  if (restorable_below) *restorable_below = im.rec_n == 0 ? 1 : 0;
  return HB_OK;
}
