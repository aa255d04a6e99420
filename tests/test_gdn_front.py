"""DeltaNet front and back ends: causal conv + SiLU, beta/decay gates, gated
RMS norm (src/jit/target/x86/execution/delta.rs:290-389, 609-774).

CPU: the oracle's scalar exp/log equal glibc's expf/logf (the same published
algorithm) on a sweep of bit patterns, and their tables follow from their
definitions; the oracle's conv and gated-norm restatements equal their
AVX-512 transcriptions of the emitted kernels bit for bit; the outputs are
accurate against f64; the golden fixture reproduces; the C ABI refuses bad
calls before any launch.  GPU: ``hb_gdn_front`` and ``hb_gdn_gated_norm``
give the oracle's bits, alone and chained with ``hb_gdn_decode``.
"""
import ctypes
import os
import struct
from decimal import Decimal, getcontext

import numpy as np
import pytest

import herbert_b200 as hb
import oracle as O
from herbert_b200.inputs import DeltaFrontInputs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "gdn_front_rows5.npz")


def bits_equal(a, b):
    """Bit equality of f32 arrays, any NaN equal to any NaN (payloads are not
    reproduced)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    return a.shape == b.shape and bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | both_nan))


def oracle_front(inp, impl=0):
    y, st = O.gdn_conv(inp.qkv, inp.conv_state, inp.conv_weight, impl)
    beta, decay = O.gdn_gates(inp.ab, inp.dt_bias, inp.a_log)
    return y, st, beta, decay


def oracle_norm(inp, impl=0, eps=1e-6):
    return O.gdn_gated_norm(inp.x, inp.z, inp.norm_weight, eps, impl)


CASES = [
    # rows, nk, nv, hkd, hvd, ck
    (1, 16, 32, 128, 128, 4),     # decode, Qwen3.5
    (5, 16, 32, 128, 128, 4),
    (200, 2, 4, 128, 128, 4),     # four boxes, the last one ragged
    (700, 1, 2, 64, 64, 4),       # eleven boxes: every ring slot reused
    (67, 1, 1, 18, 16, 4),        # conv 52: a ragged last block (scalar body), a partial strip
    (9, 2, 4, 32, 16, 3),         # ck 3: the scalar body everywhere
    (3, 1, 2, 16, 32, 8),
]


def _ids(c):
    return "r{}nk{}nv{}k{}v{}ck{}".format(*c)


def _inputs(c, seed=0xDE17A):
    rows, nk, nv, hkd, hvd, ck = c
    inp = DeltaFrontInputs(rows, nk=nk, nv=nv, hkd=hkd, hvd=hvd, ck=ck, seed=seed)
    # specials through every path: zeros, a huge and a tiny value, infinities
    flat = inp.qkv.reshape(-1)
    flat[:6] = [0.0, -0.0, 1e30, 1e-40, np.inf, -np.inf]
    specials_ab = [25.0, -120.0, 95.0, 20.0]
    n = min(4, inp.ab.shape[1])
    inp.ab[0, :n] = specials_ab[:n]
    if inp.ab.shape[1] > 4:
        inp.ab[0, -2:] = [np.inf, -np.inf]
    inp.z.reshape(-1)[:4] = [100.0, -100.0, 0.0, -0.0]
    return inp


# ----------------------------------------------------------------- CPU only

def test_scalar_exp_log_equal_glibc():
    # stride 101 visits every exponent and sign with ~42 M patterns; the full
    # 2^32 sweep (stride 1) also shows no difference but takes a minute
    assert O.mathf_sweep(101, 0) == 0
    assert O.mathf_sweep(101, 1) == 0
    sp = np.array([0.0, -0.0, np.inf, -np.inf, 1.0, 1e-40, -1.0, 88.0, 88.72283, 88.72284,
                   -103.97208, -104.0, 89.0, 20.0, -87.5], np.float32)
    assert bits_equal(O.expf_arm(sp), O.expf_libm(sp))
    assert bits_equal(O.logf_arm(sp), O.logf_libm(sp))


def test_scalar_exp_log_tables_follow_their_definitions():
    getcontext().prec = 80
    e, g = O.mathf_tables()
    as_bits = lambda x: struct.unpack("<Q", struct.pack("<d", float(x)))[0]  # noqa: E731
    as_f64 = lambda b: struct.unpack("<d", struct.pack("<Q", int(b)))[0]  # noqa: E731
    for i in range(32):
        want = (as_bits(Decimal(2) ** (Decimal(i) / 32)) - (i << 47)) % (1 << 64)
        assert int(e[i]) == want, i
    for i in range(16):
        invc = as_f64(g[i, 0])
        assert int(g[i, 1]) == as_bits(-Decimal(invc).ln()) % (1 << 64), i
        # subinterval i of [0x3f330000, 2 * 0x3f330000) holds 1 / invc
        lo = struct.unpack("<f", struct.pack("<I", 0x3F330000 + (i << 19)))[0]
        hi = struct.unpack("<f", struct.pack("<I", 0x3F330000 + ((i + 1) << 19)))[0]
        assert lo <= 1.0 / invc <= hi, i


@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_oracle_restatements_equal_avx512_transcriptions(case):
    if not O.has_avx512bf16():
        pytest.skip("this CPU has no AVX-512")
    inp = _inputs(case)
    y0, s0 = O.gdn_conv(inp.qkv, inp.conv_state, inp.conv_weight, 0)
    y1, s1 = O.gdn_conv(inp.qkv, inp.conv_state, inp.conv_weight, 1)
    assert bits_equal(y0, y1) and bits_equal(s0, s1)
    n0, b0 = oracle_norm(inp, 0)
    n1, b1 = oracle_norm(inp, 1)
    assert bits_equal(n0, n1) and np.array_equal(b0, b1)


def test_oracle_is_accurate():
    inp = DeltaFrontInputs(33, nk=2, nv=4, hkd=64, hvd=128, seed=0xACC)
    y, st, beta, decay = oracle_front(inp)
    # conv + SiLU in f64
    x = np.concatenate([inp.conv_state[:, 1:].T.astype(np.float64), inp.qkv.astype(np.float64)])
    w = O.bf16_to_f32(inp.conv_weight).astype(np.float64)
    g = sum(x[j:j + inp.rows] * w[:, j] for j in range(4))
    want = g / (1 + np.exp(-g))
    # the SiLU's exp is the reference's degree-4 polynomial (~5e-5 relative)
    assert np.max(np.abs(y - want)) <= 1e-4 * max(1.0, np.max(np.abs(want)))
    assert np.array_equal(st, x[-4:].T.astype(np.float32))
    a = inp.ab[:, :inp.nv].astype(np.float64)
    b = inp.ab[:, inp.nv:].astype(np.float64)
    dt = a + O.bf16_to_f32(inp.dt_bias).astype(np.float64)
    dt = np.where(dt > 20, dt, np.log1p(np.exp(dt)))
    assert np.max(np.abs(beta - 1 / (1 + np.exp(-b)))) < 1e-6
    want_decay = np.exp(-np.exp(inp.a_log.astype(np.float64)) * dt)
    assert np.max(np.abs(decay - want_decay) / want_decay) < 1e-5
    yn, ob = oracle_norm(inp)
    xv = inp.x.reshape(-1, inp.hvd).astype(np.float64)
    zv = inp.z.reshape(-1, inp.hvd).astype(np.float64)
    inv = 1 / np.sqrt((xv * xv).mean(axis=1, keepdims=True) + 1e-6)
    want = xv * inv * O.bf16_to_f32(inp.norm_weight) * zv / (1 + np.exp(-zv))
    assert np.max(np.abs(yn.reshape(want.shape) - want)) < 1e-4 * np.max(np.abs(want))
    assert np.array_equal(ob, O.f32_to_bf16(yn))


def test_oracle_reproduces_the_golden_fixture():
    z = np.load(GOLDEN)
    y, st = O.gdn_conv(z["qkv"], z["conv_state"], z["conv_weight"])
    beta, decay = O.gdn_gates(z["ab"], z["dt_bias"], z["a_log"])
    yn, ob = O.gdn_gated_norm(z["x"], z["z"], z["norm_weight"])
    assert bits_equal(y, z["qkv_out"]) and bits_equal(st, z["conv_state_out"])
    assert bits_equal(beta, z["beta"]) and bits_equal(decay, z["decay"])
    assert bits_equal(yn, z["norm_f32"]) and np.array_equal(ob, z["norm_bf16"])


def _front_refusal(shape=None, ws=256, **over):
    shape = shape or hb.DeltaShape(nk=16, nv=32, hkd=128, hvd=128)
    base = dict(qkv=256, conv_state=256, conv_weight=256, ab=256, dt_bias=256, a_log=256,
                beta=256, decay=256, rows=4, ck=4)
    base.update(over)
    call = hb.GdnFrontCall(**base)
    return hb.lib().hb_gdn_front(ctypes.byref(shape), ctypes.byref(call), ctypes.c_void_p(ws),
                                 256, None)


def _norm_refusal(shape=None, **over):
    shape = shape or hb.DeltaShape(nk=16, nv=32, hkd=128, hvd=128)
    base = dict(x=256, z=256, weight=256, out=256, out_f32=None, rows=4, eps=1e-6)
    base.update(over)
    call = hb.GdnNormCall(**base)
    return hb.lib().hb_gdn_gated_norm(ctypes.byref(shape), ctypes.byref(call), None)


def test_refusals_happen_before_any_launch():
    # fake (aligned, non-null) pointers: every case must be refused by the
    # host checks; never run where a GPU could receive a launch
    import torch
    if torch.cuda.is_available():
        pytest.skip("fake-pointer refusals run on hosts without a GPU only")
    assert _front_refusal(ck=0) == hb.HB_DECLINE_GEOMETRY
    assert _front_refusal(ck=9) == hb.HB_DECLINE_GEOMETRY
    assert _front_refusal(hb.DeltaShape(nk=1, nv=1, hkd=1, hvd=1)) == hb.HB_DECLINE_GEOMETRY
    assert _front_refusal(hb.DeltaShape(nk=2, nv=3, hkd=8, hvd=8)) == hb.HB_DECLINE_GEOMETRY
    assert _front_refusal(rows=0) == hb.HB_DECLINE_EMPTY
    assert _front_refusal(qkv=260) == hb.HB_ERR_ARG  # TMA needs 16-byte alignment
    assert _front_refusal(a_log=None) == hb.HB_ERR_ARG
    assert _front_refusal(ws=None) == hb.HB_ERR_WORKSPACE
    assert _norm_refusal(rows=0) == hb.HB_DECLINE_EMPTY
    assert _norm_refusal(z=None) == hb.HB_ERR_ARG
    assert _norm_refusal(eps=float("nan")) == hb.HB_ERR_ARG
    assert "eps" in hb.last_error()
    assert _norm_refusal(hb.DeltaShape(nk=0, nv=32, hkd=128, hvd=128)) == hb.HB_DECLINE_GEOMETRY


# ---------------------------------------------------------------------- GPU

def _dev(a, dtype=None):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


def _gpu_front(inp):
    import torch
    shape = hb.DeltaShape(nk=inp.nk, nv=inp.nv, hkd=inp.hkd, hvd=inp.hvd)
    qkv, st = _dev(inp.qkv), _dev(inp.conv_state)
    beta = torch.empty((inp.rows, inp.nv), dtype=torch.float32, device="cuda")
    decay = torch.empty_like(beta)
    ws = hb.delta_front(shape, qkv, st, _dev(inp.conv_weight), _dev(inp.ab), _dev(inp.dt_bias),
                        _dev(inp.a_log), beta, decay, rows=inp.rows, ck=inp.ck)
    ws.status()
    return qkv.cpu().numpy(), st.cpu().numpy(), beta.cpu().numpy(), decay.cpu().numpy()


def _gpu_norm(inp, in_place=False, f32=True, eps=1e-6):
    import torch
    shape = hb.DeltaShape(nk=inp.nk, nv=inp.nv, hkd=inp.hkd, hvd=inp.hvd)
    x = _dev(inp.x)
    out = torch.empty(inp.x.shape, dtype=torch.int16, device="cuda")
    of = x if in_place else (torch.empty_like(x) if f32 else None)
    hb.delta_gated_norm(shape, x, _dev(inp.z), _dev(inp.norm_weight), out, rows=inp.rows,
                        eps=eps, out_f32=of)
    torch.cuda.synchronize()
    return (None if of is None else of.cpu().numpy()), out.cpu().numpy().view(np.uint16), x


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_front_matches_oracle_bit_for_bit(case):
    inp = _inputs(case)
    want = oracle_front(inp)
    got = _gpu_front(inp)
    for name, g, w in zip(("qkv", "conv_state", "beta", "decay"), got, want):
        assert bits_equal(g, w), f"{name}: {np.count_nonzero(~np.isclose(g, w, 0, 0, True))} differ"


@pytest.mark.gpu
@pytest.mark.parametrize("hvd", [128, 64, 16, 48, 100, 256])
def test_gated_norm_matches_oracle_bit_for_bit(hvd):
    inp = _inputs((7, 2, 4, 64, hvd, 4), seed=0xD0 + hvd)
    yf, yb = oracle_norm(inp)
    gf, gb, _ = _gpu_norm(inp)
    assert bits_equal(gf, yf.reshape(gf.shape))
    assert np.array_equal(gb, yb.reshape(gb.shape))


@pytest.mark.gpu
def test_gated_norm_in_place_and_without_f32():
    inp = _inputs((5, 16, 32, 128, 128, 4), seed=0xD1)
    yf, yb = oracle_norm(inp)
    gf, gb, _ = _gpu_norm(inp, in_place=True)
    assert bits_equal(gf, yf) and np.array_equal(gb, yb)
    gf, gb, x = _gpu_norm(inp, f32=False)
    assert gf is None and np.array_equal(gb, yb)
    assert bits_equal(x.cpu().numpy(), inp.x)


@pytest.mark.gpu
def test_golden_fixture_on_the_device():
    z = np.load(GOLDEN)
    m = z["meta"]
    inp = DeltaFrontInputs(int(m[0]), nk=int(m[1]), nv=int(m[2]), hkd=int(m[3]), hvd=int(m[4]),
                           ck=int(m[5]))
    for k in ("qkv", "conv_state", "conv_weight", "ab", "dt_bias", "a_log", "x", "z",
              "norm_weight"):
        setattr(inp, k, z[k])
    y, st, beta, decay = _gpu_front(inp)
    assert bits_equal(y, z["qkv_out"]) and bits_equal(st, z["conv_state_out"])
    assert bits_equal(beta, z["beta"]) and bits_equal(decay, z["decay"])
    gf, gb, _ = _gpu_norm(inp)
    assert bits_equal(gf, z["norm_f32"]) and np.array_equal(gb, z["norm_bf16"])


@pytest.mark.gpu
def test_mixer_chain_matches_the_oracle_bit_for_bit():
    """conv + gates -> L2 + recurrence (decode kernel) -> gated norm on the
    device equals the oracle's chain: the DeltaNet mixer between its
    projections, in the reference's bits."""
    import torch
    inp = DeltaFrontInputs(6, seed=0xC4A1)
    y, _, beta, decay = oracle_front(inp)
    state0 = (np.random.default_rng(3).standard_normal((inp.nv, inp.hkd, inp.hvd)) * 0.1
              ).astype(np.float32)
    out, _, _ = O.gdn_layer(y, state0, beta, decay, nk=inp.nk, nv=inp.nv, hkd=inp.hkd,
                            hvd=inp.hvd)
    yn, yb = O.gdn_gated_norm(out, inp.z, inp.norm_weight)

    shape = hb.DeltaShape(nk=inp.nk, nv=inp.nv, hkd=inp.hkd, hvd=inp.hvd)
    qkv, cst = _dev(inp.qkv), _dev(inp.conv_state)
    gbeta = torch.empty((inp.rows, inp.nv), dtype=torch.float32, device="cuda")
    gdecay = torch.empty_like(gbeta)
    hb.delta_front(shape, qkv, cst, _dev(inp.conv_weight), _dev(inp.ab), _dev(inp.dt_bias),
                   _dev(inp.a_log), gbeta, gdecay, rows=inp.rows)
    st = _dev(state0)
    gout = torch.empty((inp.rows, inp.nv * inp.hvd), dtype=torch.float32, device="cuda")
    hb.delta_recurrence(shape, st, gout, qkv, gbeta, gdecay, rows=inp.rows, regime="decode")
    ob = torch.empty(gout.shape, dtype=torch.int16, device="cuda")
    hb.delta_gated_norm(shape, gout, _dev(inp.z), _dev(inp.norm_weight), ob, rows=inp.rows)
    torch.cuda.synchronize()
    assert bits_equal(gout.cpu().numpy(), out)
    assert np.array_equal(ob.cpu().numpy().view(np.uint16), yb)
