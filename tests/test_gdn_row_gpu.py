"""One-row DeltaNet layers through the mount (a decode step of the
lowering's delta nodes, src/jit/model/lowering.rs:904-1010).

The mount runs a one-row block of a served geometry as one launch (conv +
SiLU, gates, L2, recurrence, gated norm).  Here that launch is checked bit
for bit against the three node calls (hb_gdn_front, hb_gdn_decode,
hb_gdn_gated_norm) on copies of the same inputs and state, over several
tokens and over the served geometries (key/value head ratios 1, 2, 4;
hkd 64 and 128; hvd 32 to 128), and, at Qwen3.5's DeltaNet geometry,
against the oracle's chains.  A one-row call that a node refuses launches
nothing: the state is untouched and the mount is not poisoned.
"""
import numpy as np
import pytest

import herbert_b200 as hb
import oracle as O
from herbert_b200.inputs import DeltaFrontInputs

L2_EPS, NORM_EPS = 1e-6, 1e-6

SHAPES = [(2, 4, 128, 128), (4, 4, 64, 64), (1, 4, 64, 32), (2, 8, 128, 96), (16, 32, 128, 128)]


def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a.copy()).cuda()


class _Layer:
    """A mount over one DeltaNet layer and its state, seeded."""

    def __init__(self, nk, nv, hkd, hvd, seed):
        import torch
        self.shape = hb.DeltaShape(nk=nk, nv=nv, hkd=hkd, hvd=hvd)
        self.conv = 2 * nk * hkd + nv * hvd
        self.rec_len = nv * hkd * hvd
        rng = np.random.default_rng(seed)
        self.conv0 = rng.standard_normal(self.conv * 4, dtype=np.float32)
        self.rec0 = (rng.standard_normal(self.rec_len) * 0.1).astype(np.float32)
        self.conv_state = torch.from_numpy(self.conv0.copy()).cuda()
        self.rec = torch.from_numpy(self.rec0.copy()).cuda()
        geo = hb.Geometry([0, 0], 1, 8, self.conv * 4, self.rec_len, 0)
        desc, keep = hb.mount_desc(geo, [hb.HB_LAYER_DELTA], dn_conv=self.conv_state,
                                   dn_recurrent=self.rec, delta=self.shape, conv_kernel=4,
                                   conv_stride=self.conv * 4, recurrent_stride=self.rec_len,
                                   max_rows=1, norm_eps=NORM_EPS)
        self.mount = hb.Mount(desc, keep)


def _bits(a):
    return a.cpu().numpy().view(np.uint32 if a.element_size() == 4 else np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("nk,nv,hkd,hvd", SHAPES)
def test_one_row_layer_is_the_three_nodes_bits(nk, nv, hkd, hvd):
    import torch
    lay = _Layer(nk, nv, hkd, hvd, seed=0x5E0 + nk * 7 + nv + hkd + hvd)
    conv_u, rec_u = lay.conv_state.clone(), lay.rec.clone()   # the node path's own state
    beta = torch.empty(nv, dtype=torch.float32, device="cuda")
    decay = torch.empty_like(beta)
    x = torch.empty(nv * hvd, dtype=torch.float32, device="cuda")
    for t in range(5):
        inp = DeltaFrontInputs(1, nk=nk, nv=nv, hkd=hkd, hvd=hvd, seed=0x5E1 + 31 * t + hvd)
        qkv_m = _dev(inp.qkv)
        qkv_u = qkv_m.clone()
        ab, z, cw = _dev(inp.ab), _dev(inp.z), _dev(inp.conv_weight)
        dtb, alog, nw = _dev(inp.dt_bias), _dev(inp.a_log), _dev(inp.norm_weight)
        out_m = torch.empty(nv * hvd, dtype=torch.int16, device="cuda")
        outf_m = torch.empty(nv * hvd, dtype=torch.float32, device="cuda")
        out_u, outf_u = torch.empty_like(out_m), torch.empty_like(outf_m)
        lay.mount.delta(0, qkv_m, ab, z, cw, dtb, alog, nw, out_m, rows=1, out_f32=outf_m)
        hb.delta_front(lay.shape, qkv_u, conv_u, cw, ab, dtb, alog, beta, decay, rows=1)
        hb.delta_recurrence(lay.shape, rec_u, x, qkv_u, beta, decay, rows=1, eps=L2_EPS)
        hb.delta_gated_norm(lay.shape, x, z, nw, out_u, rows=1, eps=NORM_EPS, out_f32=outf_u)
        torch.cuda.synchronize()
        lay.mount.status()
        assert np.array_equal(_bits(qkv_m), _bits(qkv_u)), f"qkv, token {t}"
        assert np.array_equal(_bits(lay.conv_state), _bits(conv_u)), f"conv state, token {t}"
        assert np.array_equal(_bits(lay.rec), _bits(rec_u)), f"recurrent state, token {t}"
        assert np.array_equal(_bits(outf_m), _bits(outf_u)), f"f32 output, token {t}"
        assert np.array_equal(_bits(out_m), _bits(out_u)), f"bf16 output, token {t}"
    assert not np.array_equal(lay.rec.cpu().numpy(), lay.rec0)


@pytest.mark.gpu
def test_one_row_tokens_match_the_oracle():
    """Four tokens in a row at Qwen3.5's DeltaNet geometry against the
    oracle's conv, gates, recurrence and gated norm chains: the
    reference's bits."""
    import torch
    nk, nv, hkd, hvd = 16, 32, 128, 128
    lay = _Layer(nk, nv, hkd, hvd, seed=0x5F0)
    conv_state = lay.conv0.reshape(lay.conv, 4).copy()
    rec = lay.rec0.reshape(nv, hkd, hvd).copy()
    for t in range(4):
        inp = DeltaFrontInputs(1, nk=nk, nv=nv, hkd=hkd, hvd=hvd, seed=0x5F1 + t)
        qkv = _dev(inp.qkv)
        out = torch.empty(nv * hvd, dtype=torch.int16, device="cuda")
        out_f32 = torch.empty(nv * hvd, dtype=torch.float32, device="cuda")
        lay.mount.delta(0, qkv, _dev(inp.ab), _dev(inp.z), _dev(inp.conv_weight),
                        _dev(inp.dt_bias), _dev(inp.a_log), _dev(inp.norm_weight), out, rows=1,
                        out_f32=out_f32)
        y, conv_state = O.gdn_conv(inp.qkv, conv_state, inp.conv_weight)
        beta, decay = O.gdn_gates(inp.ab, inp.dt_bias, inp.a_log)
        o, rec, _ = O.gdn_layer(y, rec, beta, decay, nk=nk, nv=nv, hkd=hkd, hvd=hvd)
        yn, yb = O.gdn_gated_norm(o, inp.z, inp.norm_weight)
        torch.cuda.synchronize()
        lay.mount.status()
        assert np.array_equal(qkv.cpu().numpy().ravel().view(np.uint32), y.ravel().view(np.uint32))
        assert np.array_equal(out_f32.cpu().numpy().view(np.uint32), yn.ravel().view(np.uint32))
        assert np.array_equal(out.cpu().numpy().view(np.uint16), yb.ravel())
    assert np.array_equal(lay.conv_state.cpu().numpy().view(np.uint32),
                          conv_state.ravel().view(np.uint32))
    assert np.array_equal(lay.rec.cpu().numpy().view(np.uint32), rec.ravel().view(np.uint32))


@pytest.mark.gpu
def test_a_refused_one_row_call_launches_nothing():
    """Every node's checks run before the one launch: a null z is refused
    with the state untouched and the mount usable."""
    import torch
    lay = _Layer(2, 4, 128, 128, seed=0x5D0)
    inp = DeltaFrontInputs(1, nk=2, nv=4, hkd=128, hvd=128, seed=0x5D1)
    out = torch.empty(4 * 128, dtype=torch.int16, device="cuda")
    qkv = _dev(inp.qkv)
    args = [qkv, _dev(inp.ab), None, _dev(inp.conv_weight), _dev(inp.dt_bias), _dev(inp.a_log),
            _dev(inp.norm_weight), out]
    with pytest.raises(hb.HBError) as e:
        lay.mount.delta(0, *args, rows=1)
    assert e.value.status == hb.HB_ERR_ARG
    assert not lay.mount.needs_reset
    torch.cuda.synchronize()
    assert np.array_equal(lay.conv_state.cpu().numpy(), lay.conv0)
    assert np.array_equal(lay.rec.cpu().numpy(), lay.rec0)
    assert np.array_equal(qkv.cpu().numpy(), inp.qkv)
    args[2] = _dev(inp.z)
    lay.mount.delta(0, *args, rows=1)
    torch.cuda.synchronize()
    lay.mount.status()
