"""One-row attention layers over long caches through the mount (a decode
step of the lowering's attention nodes, src/jit/model/lowering.rs:549-666).

For one row over more than 16 x 256 cached positions the mount runs the
head-norm-rope and kv-append nodes inside the split-KV decode launch.
Checked here bit for bit against the two node calls (hb_attn_front, then
hb_attn_decode) on copies of the same inputs and cache: the gated output,
q and k normed and rotated in place, and the whole cache (the new row and
nothing else); at one size also against the oracle's front end and
attention within the SDPA tolerance.
"""
import numpy as np
import pytest

import herbert_b200 as hb
import oracle as O
from harness import assert_sdpa_close
from herbert_b200.inputs import FrontInputs

HD = 256


def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a.copy()).cuda()


def _bits(t):
    return t.cpu().numpy().view(np.uint16)


class _Layer:
    """A mount over one attention layer with a cache of `reserve` positions."""

    def __init__(self, heads, gqa, reserve, seed):
        import torch
        self.heads, self.hkv, self.reserve = heads, heads // gqa, reserve
        self.f = FrontInputs(1, 0, heads=heads, kv_heads=self.hkv, capacity=reserve, seed=seed)
        self.cache0 = np.concatenate([self.f.keys.ravel(), self.f.values.ravel()])
        self.kv = _dev(self.cache0)
        self.cos, self.sin = _dev(self.f.cos), _dev(self.f.sin)
        geo = hb.Geometry([0, 2 * self.hkv * reserve * HD], self.hkv, reserve, 0, 0, 16)
        self.logits = torch.zeros(16, dtype=torch.int16, device="cuda")
        self.spec = hb.attention_spec(heads, gqa, HD, True)
        desc, keep = hb.mount_desc(geo, [hb.HB_LAYER_ATTENTION], kv=self.kv, logits=self.logits,
                                   attn=self.spec, attn_scale=1 / 16.0, rotary=64, cos=self.cos,
                                   sin=self.sin, max_rows=1)
        self.mount = hb.Mount(desc, keep + (self.cos, self.sin))


@pytest.mark.gpu
@pytest.mark.parametrize("heads,gqa,pos", [(16, 4, 32767), (16, 4, 5000), (16, 8, 9000),
                                           (8, 1, 4096)])
def test_one_row_layer_is_the_two_nodes_bits(heads, gqa, pos):
    import torch
    lay = _Layer(heads, gqa, pos + 8, seed=0xA70 + pos + gqa)
    f = lay.f
    kv_u = lay.kv.clone()
    stride = lay.reserve * HD
    ks, vs = kv_u[:lay.hkv * stride], kv_u[lay.hkv * stride:]
    q_m, k_m, v = _dev(f.q), _dev(f.k), _dev(f.v)
    q_u, k_u = q_m.clone(), k_m.clone()
    qn, kn = _dev(f.q_norm), _dev(f.k_norm)
    out_m = torch.zeros((1, heads * HD), dtype=torch.int16, device="cuda")
    out_u = torch.zeros_like(out_m)
    for _ in range(2):  # the second call repeats the first (the split counters reset themselves)
        q_m.copy_(_dev(f.q)); k_m.copy_(_dev(f.k))
        lay.mount.attention(0, q_m, k_m, v, qn, kn, out_m, rows=1, pos=pos)
    kvs = hb.KvSpec(heads=lay.hkv, head_dim=HD, stride=stride, capacity=lay.reserve, max_batch=1)
    hb.attn_front(lay.spec, kvs, q_u, k_u, v, qn, kn, lay.cos, lay.sin, rows=1, past=pos,
                  rotary=64, keys=ks, values=vs)
    hb.attention(lay.spec, q_u, ks, vs, out_u, rows=1, past=pos, kv_stride=stride,
                 capacity=lay.reserve, scale=1 / 16.0)
    torch.cuda.synchronize()
    lay.mount.status()
    assert np.array_equal(_bits(q_m), _bits(q_u)), "q in place"
    assert np.array_equal(_bits(k_m), _bits(k_u)), "k in place"
    assert np.array_equal(_bits(lay.kv), _bits(kv_u)), "cache"
    assert np.array_equal(_bits(out_m), _bits(out_u)), "output"
    changed = np.nonzero(_bits(lay.kv) != lay.cache0)[0]
    rows = np.unique((changed % stride) // HD)
    assert set(rows.tolist()) <= {pos}, "only the row's position is written"


@pytest.mark.gpu
def test_one_row_layer_matches_the_oracle():
    import torch
    pos = 6000
    lay = _Layer(16, 4, pos + 4, seed=0xA90)
    f = lay.f
    keys, values = f.keys.copy(), f.values.copy()
    q, k, keys, values = O.attn_front(f.q, f.k, f.v, f.q_norm, f.k_norm, f.cos, f.sin, heads=16,
                                      kv_heads=4, head_dim=HD, rotary=64, past=pos,
                                      keys=keys, values=values)
    want = O.attention(q, keys, values, rows=1, past=pos, heads=16, gqa=4, head_dim=HD,
                       q_row=f.q_row, q_head=HD, out_row=16 * HD, kv_stride=lay.reserve * HD,
                       gate_offset=16 * HD, scale=1 / 16.0)
    gq = _dev(f.q)
    out = torch.zeros((1, 16 * HD), dtype=torch.int16, device="cuda")
    lay.mount.attention(0, gq, _dev(f.k), _dev(f.v), _dev(f.q_norm), _dev(f.k_norm), out, rows=1,
                        pos=pos)
    torch.cuda.synchronize()
    lay.mount.status()
    assert_sdpa_close(_bits(out).ravel(), want, "fused one-row attention")
    assert np.array_equal(_bits(lay.kv), np.concatenate([keys.ravel(), values.ravel()]))
    assert np.array_equal(_bits(gq)[:, :16 * HD], q[:, :16 * HD].view(np.uint16))
