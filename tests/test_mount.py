"""Routing of a pass to the kernels (src/jit/model/mounted.rs:237-380).

CPU: ``hb_mount_route`` binds each layer to its slice of the state exactly as
the lowering mounts it, and refuses the lowering's plan mismatches (host only,
no device access).  GPU: a mount over a hybrid state runs an attention layer
(decode and prefill blocks) and a DeltaNet layer (recurrent and chunked
blocks) against the oracle's chains, writing only that layer's slices.
"""
import numpy as np
import pytest

import herbert_b200 as hb
import oracle as O
from harness import assert_sdpa_close, rel_frob
from herbert_b200.inputs import DeltaFrontInputs, FrontInputs

KINDS = [hb.HB_LAYER_DELTA, hb.HB_LAYER_ATTENTION, hb.HB_LAYER_DELTA, hb.HB_LAYER_ATTENTION]
RESERVE, HKV, HD = 320, 4, 256
NK, NV, HKD, HVD, CK = 2, 4, 128, 128, 4
CONV = 2 * NK * HKD + NV * HVD
CONV_STRIDE, REC_STRIDE = CONV * CK, NV * HKD * HVD


def _geometry(kinds=KINDS, hd=HD, n_delta=None):
    offsets = [0]
    for k in kinds:
        offsets.append(offsets[-1] + (2 * HKV * RESERVE * hd if k == hb.HB_LAYER_ATTENTION else 0))
    n_delta = kinds.count(hb.HB_LAYER_DELTA) if n_delta is None else n_delta
    return hb.Geometry(offsets, HKV, RESERVE, n_delta * CONV_STRIDE, n_delta * REC_STRIDE, 16)


def _desc(geo, kinds=KINDS, base=1 << 20, **over):
    kw = dict(kv=base, dn_conv=base << 8, dn_recurrent=base << 12, logits=base << 16,
              attn=hb.attention_spec(16, 4, HD, True), attn_scale=1 / 16.0, rotary=64,
              cos=base << 4, sin=base << 5, delta=hb.DeltaShape(nk=NK, nv=NV, hkd=HKD, hvd=HVD),
              conv_kernel=CK, conv_stride=CONV_STRIDE, recurrent_stride=REC_STRIDE, max_rows=256)
    kw.update(over)
    return hb.mount_desc(geo, kinds, **kw)


# ----------------------------------------------------------------- CPU only

def test_layers_are_routed_to_their_slices():
    kinds = [hb.HB_LAYER_DELTA] * 3 + [hb.HB_LAYER_ATTENTION] + [hb.HB_LAYER_DELTA] * 3 + \
            [hb.HB_LAYER_ATTENTION]
    geo = _geometry(kinds)
    base = 1 << 20
    desc, keep = _desc(geo, kinds, base)
    r = hb.mount_route(desc, 3)
    assert (r.kind, r.delta_index) == (hb.HB_LAYER_ATTENTION, -1)
    assert r.kv_stride == RESERVE * HD
    assert r.keys == base and r.values == base + 2 * HKV * RESERVE * HD   # bf16 elements -> bytes
    r = hb.mount_route(desc, 7)
    assert r.keys == base + 2 * geo.offsets[7] and r.values == r.keys + 2 * HKV * RESERVE * HD
    r = hb.mount_route(desc, 5)   # DeltaNet layers 0, 1, 2, 4 come before it
    assert (r.kind, r.delta_index) == (hb.HB_LAYER_DELTA, 4)
    assert r.conv_state == (base << 8) + 4 * 4 * CONV_STRIDE
    assert r.recurrent_state == (base << 12) + 4 * 4 * REC_STRIDE
    assert hb.mount_route(desc, 0).delta_index == 0


def _status(desc):
    import ctypes
    r = hb.LayerRoute()
    return hb.lib().hb_mount_route(ctypes.byref(desc), 0, ctypes.byref(r))


def test_the_lowerings_refusals():
    geo = _geometry()
    assert _status(_desc(geo)[0]) == hb.HB_OK
    # a DeltaNet layer that owns a KV cache
    kinds = [hb.HB_LAYER_DELTA, hb.HB_LAYER_DELTA, hb.HB_LAYER_DELTA, hb.HB_LAYER_ATTENTION]
    assert _status(_desc(geo, kinds)[0]) == hb.HB_DECLINE_GEOMETRY
    assert "absent-KV" in hb.last_error()
    # an attention layer whose cache is not kv_heads x reserve x head_dim
    assert _status(_desc(_geometry(hd=128))[0]) == hb.HB_DECLINE_GEOMETRY
    assert "KV geometry" in hb.last_error()
    # slots too small or too few
    assert _status(_desc(geo, conv_stride=CONV_STRIDE - 1)[0]) == hb.HB_DECLINE_GEOMETRY
    assert _status(_desc(_geometry(n_delta=1))[0]) == hb.HB_DECLINE_GEOMETRY
    # heads / gqa against the cache's kv_heads
    assert _status(_desc(geo, attn=hb.attention_spec(16, 2, HD, True))[0]) == hb.HB_DECLINE_GEOMETRY
    assert _status(_desc(geo, rotary=48)[0]) == hb.HB_DECLINE_HEAD_DIM
    assert _status(_desc(geo, max_rows=RESERVE + 1)[0]) == hb.HB_ERR_ARG
    big = hb.Geometry([0, 0, 2 * HKV * (1 << 21) * HD, 2 * HKV * (1 << 21) * HD,
                       4 * HKV * (1 << 21) * HD], HKV, 1 << 21, 2 * CONV_STRIDE, 2 * REC_STRIDE, 16)
    assert _status(_desc(big, max_rows=(1 << 20) + 1)[0]) == hb.HB_ERR_ARG
    assert _status(_desc(big, max_rows=1 << 20)[0]) == hb.HB_OK
    assert _status(_desc(geo, cos=0)[0]) == hb.HB_ERR_ARG
    assert _status(_desc(geo, norm_eps=float("nan"))[0]) == hb.HB_ERR_ARG
    assert _status(_desc(geo, [1, 2, 9, 2])[0]) == hb.HB_ERR_ARG


# ---------------------------------------------------------------------- GPU

class _Model:
    """A hybrid state on the device: layers 0, 2 DeltaNet, 1, 3 attention."""

    def __init__(self, seed, max_rows=256):
        import torch
        self.geo = _geometry()
        rng = np.random.default_rng(seed)
        # the caches hold finite bf16 values: attention computes on them
        self.kv0 = O.normal_bf16((self.geo.offsets[-1],), seed)
        self.conv0 = rng.standard_normal(2 * CONV_STRIDE, dtype=np.float32)
        self.rec0 = (rng.standard_normal(2 * REC_STRIDE) * 0.1).astype(np.float32)
        self.kv = torch.from_numpy(self.kv0.view(np.int16).copy()).cuda()
        self.conv = torch.from_numpy(self.conv0.copy()).cuda()
        self.rec = torch.from_numpy(self.rec0.copy()).cuda()
        self.logits = torch.zeros(16, dtype=torch.int16, device="cuda")
        self.front = FrontInputs(1, 0, capacity=RESERVE, seed=seed + 1)
        self.cos = torch.from_numpy(self.front.cos.view(np.int16).copy()).cuda()
        self.sin = torch.from_numpy(self.front.sin.view(np.int16).copy()).cuda()
        desc, keep = _desc(self.geo, kv=self.kv, dn_conv=self.conv, dn_recurrent=self.rec,
                           logits=self.logits, cos=self.cos, sin=self.sin, max_rows=max_rows)
        self.mount = hb.Mount(desc, keep + (self.cos, self.sin))

    def kv_layer(self, l):
        a, b = self.geo.offsets[l], self.geo.offsets[l + 1]
        return self.kv[a:b].cpu().numpy().view(np.uint16)


def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a.copy()).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,pos", [(1, 300), (40, 9), (1, 0)])
def test_attention_layer_matches_the_oracle(rows, pos):
    import torch
    m = _Model(0xA11 + rows)
    f = FrontInputs(rows, pos, capacity=RESERVE, seed=0xA12 + pos)
    f.cos, f.sin = m.front.cos, m.front.sin
    layer = 3
    a = m.geo.offsets[layer]
    cache = m.kv0[a:a + 2 * HKV * RESERVE * HD].reshape(2, HKV, RESERVE, HD)
    f.keys, f.values = cache[0].copy(), cache[1].copy()
    q, k, keys, values = O.attn_front(f.q, f.k, f.v, f.q_norm, f.k_norm, f.cos, f.sin, heads=16,
                                      kv_heads=HKV, head_dim=HD, rotary=64, past=pos,
                                      keys=f.keys, values=f.values)
    want = O.attention(q, keys, values, rows=rows, past=pos, heads=16, gqa=4, head_dim=HD,
                       q_row=f.q_row, q_head=HD, out_row=16 * HD, kv_stride=RESERVE * HD,
                       gate_offset=16 * HD, scale=1 / 16.0)
    gq, gk = _dev(f.q), _dev(f.k)
    out = torch.zeros((rows, 16 * HD), dtype=torch.int16, device="cuda")
    m.mount.attention(layer, gq, gk, _dev(f.v), _dev(f.q_norm), _dev(f.k_norm), out, rows=rows,
                      pos=pos)
    torch.cuda.synchronize()
    m.mount.status()
    assert_sdpa_close(out.cpu().numpy().view(np.uint16).ravel(), want, "mount attention")
    assert np.array_equal(m.kv_layer(layer), np.concatenate([keys.ravel(), values.ravel()]))
    assert np.array_equal(m.kv_layer(1), m.kv0[m.geo.offsets[1]:m.geo.offsets[2]])
    assert np.array_equal(m.conv.cpu().numpy(), m.conv0)


def _delta_oracle(inp, conv_state, rec_state):
    y, st = O.gdn_conv(inp.qkv, conv_state, inp.conv_weight)
    beta, decay = O.gdn_gates(inp.ab, inp.dt_bias, inp.a_log)
    out, rec, _ = O.gdn_layer(y, rec_state.reshape(NV, HKD, HVD), beta, decay, nk=NK, nv=NV,
                              hkd=HKD, hvd=HVD)
    yn, yb = O.gdn_gated_norm(out, inp.z, inp.norm_weight)
    return st, rec, yn, yb


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [6, 1, 200])
def test_delta_layer_matches_the_oracle(rows):
    import torch
    m = _Model(0xD11 + rows)
    inp = DeltaFrontInputs(rows, nk=NK, nv=NV, hkd=HKD, hvd=HVD, seed=0xD12 + rows)
    layer, slot = 2, 1
    st, rec, yn, yb = _delta_oracle(inp, m.conv0[slot * CONV_STRIDE:(slot + 1) * CONV_STRIDE]
                                    .reshape(CONV, CK),
                                    m.rec0[slot * REC_STRIDE:(slot + 1) * REC_STRIDE])
    out = torch.empty((rows, NV * HVD), dtype=torch.int16, device="cuda")
    out_f32 = torch.empty((rows, NV * HVD), dtype=torch.float32, device="cuda")
    m.mount.delta(layer, _dev(inp.qkv), _dev(inp.ab), _dev(inp.z), _dev(inp.conv_weight),
                  _dev(inp.dt_bias), _dev(inp.a_log), _dev(inp.norm_weight), out, rows=rows,
                  out_f32=out_f32)
    torch.cuda.synchronize()
    m.mount.status()
    conv, recs = m.conv.cpu().numpy(), m.rec.cpu().numpy()
    assert np.array_equal(conv[CONV_STRIDE:], st.ravel())              # conv + gates: exact
    assert np.array_equal(conv[:CONV_STRIDE], m.conv0[:CONV_STRIDE])   # layer 0 untouched
    assert np.array_equal(recs[:REC_STRIDE], m.rec0[:REC_STRIDE])
    if rows < 128:   # the recurrence in the reference's order: the reference's bits
        assert np.array_equal(recs[REC_STRIDE:].view(np.uint32), rec.ravel().view(np.uint32))
        assert np.array_equal(out_f32.cpu().numpy().view(np.uint32), yn.view(np.uint32))
        assert np.array_equal(out.cpu().numpy().view(np.uint16), yb)
    else:            # chunked: the DeltaNet bar
        assert rel_frob(recs[REC_STRIDE:], rec.ravel()) <= 1e-2
        assert rel_frob(out_f32.cpu().numpy(), yn) <= 1e-2
    assert np.array_equal(m.kv.cpu().numpy().view(np.uint16), m.kv0)  # no KV touched


@pytest.mark.gpu
def test_a_failed_call_poisons_the_mount_until_reset():
    """A call that fails after its first node launched leaves the layer's
    state half updated: the mount refuses every later mixer call (before any
    launch) until its owner restores the state and resets it, as a failed
    call poisons the reference's execution session."""
    import torch
    m = _Model(0xD77)
    rows, layer, slot = 6, 2, 1
    inp = DeltaFrontInputs(rows, nk=NK, nv=NV, hkd=HKD, hvd=HVD, seed=0xD78)
    out = torch.empty((rows, NV * HVD), dtype=torch.int16, device="cuda")
    args = [_dev(inp.qkv), _dev(inp.ab), _dev(inp.z), _dev(inp.conv_weight), _dev(inp.dt_bias),
            _dev(inp.a_log), _dev(inp.norm_weight), out]
    bad = list(args)
    bad[2] = None  # the gated norm refuses a null z, after the conv and the recurrence ran
    assert not m.mount.needs_reset
    with pytest.raises(hb.HBError) as e:
        m.mount.delta(layer, *bad, rows=rows)
    assert e.value.status == hb.HB_ERR_ARG
    assert m.mount.needs_reset
    torch.cuda.synchronize()
    conv_after, rec_after = m.conv.clone(), m.rec.clone()
    assert not torch.equal(m.conv.cpu(), torch.from_numpy(m.conv0))  # the conv state moved
    # refused, nothing launched: the state stays as the failed call left it
    for call in (lambda: m.mount.delta(layer, *args, rows=rows),
                 lambda: m.mount.delta(0, *args, rows=rows)):
        with pytest.raises(hb.HBError) as e2:
            call()
        assert e2.value.status == hb.HB_ERR_ARG and "hb_mount_reset" in str(e2.value)
    with pytest.raises(hb.HBError):
        m.mount.status()
    torch.cuda.synchronize()
    assert torch.equal(m.conv, conv_after) and torch.equal(m.rec, rec_after)
    # the owner restores the state it holds, then resets the mount
    m.conv.copy_(torch.from_numpy(m.conv0))
    m.rec.copy_(torch.from_numpy(m.rec0))
    m.mount.reset()
    assert not m.mount.needs_reset
    args[0] = _dev(inp.qkv)  # the conv ran in place on the failed call's qkv
    m.mount.delta(layer, *args, rows=rows)
    torch.cuda.synchronize()
    m.mount.status()
    st, rec, yn, yb = _delta_oracle(inp, m.conv0[slot * CONV_STRIDE:(slot + 1) * CONV_STRIDE]
                                    .reshape(CONV, CK),
                                    m.rec0[slot * REC_STRIDE:(slot + 1) * REC_STRIDE])
    assert np.array_equal(m.conv.cpu().numpy()[CONV_STRIDE:], st.ravel())
    assert np.array_equal(out.cpu().numpy().view(np.uint16), yb)
