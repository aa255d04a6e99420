"""Attention front end: head-norm-rope of q and k, then kv-append
(src/jit/schedule/lowering.rs:549-592).

CPU: the oracle's scalar restatement equals its AVX-512 BF16 transcription of
the emitted instructions (src/jit/target/x86/emit_elem.rs:242-330, 479-514)
bit for bit, is accurate against an f64 evaluation, and reproduces the
committed golden fixture; the C ABI refuses bad calls with the named statuses
before any launch.  GPU: ``hb_attn_front`` gives the oracle's bits for q, k
and both caches.
"""
import ctypes
import os

import numpy as np
import pytest

import herbert_b200 as hb
import oracle as O
from herbert_b200.inputs import FrontInputs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "front_rows5_past9.npz")


def oracle_front(inp, impl=0, append=True):
    return O.attn_front(inp.q, inp.k, inp.v, inp.q_norm, inp.k_norm, inp.cos, inp.sin,
                        heads=inp.heads, kv_heads=inp.kv_heads, head_dim=inp.head_dim,
                        rotary=inp.rotary, past=inp.past, gemma=inp.gemma,
                        keys=inp.keys if append else None,
                        values=inp.values if append else None, impl=impl)


CASES = [
    # rows, past, heads, kv_heads, head_dim, rotary, gated, gemma
    (1, 2047, 16, 4, 256, 64, True, True),
    (5, 9, 16, 4, 256, 64, True, True),
    (37, 0, 16, 4, 256, 64, True, True),
    (3, 100, 8, 8, 256, 256, False, False),
    (7, 11, 4, 2, 128, 32, False, True),
    (2, 3, 4, 1, 128, 0, True, False),
]


def _ids(c):
    return "r{}p{}h{}k{}d{}rot{}{}{}".format(c[0], c[1], c[2], c[3], c[4], c[5],
                                             "g" if c[6] else "", "G" if c[7] else "")


def _inputs(c, seed=0xF407):
    rows, past, h, kh, d, rot, gated, gemma = c
    return FrontInputs(rows, past, heads=h, kv_heads=kh, head_dim=d, rotary=rot, gated=gated,
                       gemma=gemma, seed=seed)


# ----------------------------------------------------------------- CPU only

@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_oracle_scalar_equals_avx512_transcription(case):
    if not O.has_avx512bf16():
        pytest.skip("this CPU has no AVX512-BF16")
    inp = _inputs(case)
    for a, b in zip(oracle_front(inp, impl=0), oracle_front(inp, impl=1)):
        assert np.array_equal(a, b)


def test_oracle_is_accurate_and_leaves_the_rest_alone():
    inp = FrontInputs(4, 30)
    q, k, keys, values = oracle_front(inp)
    d, r, half = inp.head_dim, inp.rotary, inp.rotary // 2
    x = O.bf16_to_f32(inp.q[:, : inp.heads * d]).astype(np.float64).reshape(4, inp.heads, d)
    w = 1.0 + O.bf16_to_f32(inp.q_norm).astype(np.float64)
    y = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w
    c = O.bf16_to_f32(inp.cos[30:34]).astype(np.float64)[:, None, :]
    s = O.bf16_to_f32(inp.sin[30:34]).astype(np.float64)[:, None, :]
    a, b = y[..., :half].copy(), y[..., half:r].copy()
    y[..., :half], y[..., half:r] = a * c - b * s, a * s + b * c
    got = O.bf16_to_f32(q[:, : inp.heads * d]).astype(np.float64).reshape(4, inp.heads, d)
    assert np.abs(got - y).max() <= 2 ** -7 * np.abs(y).max()
    # the gate half of q, the cache outside rows [30, 34) and v are untouched
    assert np.array_equal(q[:, inp.heads * d:], inp.q[:, inp.heads * d:])
    assert np.array_equal(keys[:, :30], inp.keys[:, :30])
    assert np.array_equal(keys[:, 34:], inp.keys[:, 34:])
    assert np.array_equal(values[:, 30:34].transpose(1, 0, 2).reshape(4, -1), inp.v)
    assert np.array_equal(keys[:, 30:34].transpose(1, 0, 2).reshape(4, -1), k)


def test_oracle_reproduces_the_golden_fixture():
    z = np.load(GOLDEN)
    m = z["meta"]
    q, k, keys, values = O.attn_front(
        z["q"], z["k"], z["v"], z["q_norm"], z["k_norm"], z["cos"], z["sin"], heads=int(m[2]),
        kv_heads=int(m[3]), head_dim=int(m[4]), rotary=int(m[5]), past=int(m[1]),
        gemma=bool(m[6]), keys=z["keys0"], values=z["values0"])
    for got, want in ((q, z["q_out"]), (k, z["k_out"]), (keys, z["keys"]), (values, z["values"])):
        assert np.array_equal(got, want)


def _front_refusal(spec=None, kv=None, front=None, **over):
    spec = spec or hb.attention_spec(16, 4, 256, True)
    kv = kv or hb.KvSpec(heads=4, head_dim=256, stride=64 * 256, capacity=64, max_batch=16)
    front = front or hb.FrontSpec(rotary=64, eps=1e-6, gemma=1)
    base = dict(q=256, k=256, v=256, q_norm=256, k_norm=256, cos=256, sin=256, keys=256,
                values=256, rows=2, past=5)
    base.update(over)
    call = hb.FrontCall(**base)
    return hb.lib().hb_attn_front(ctypes.byref(spec), ctypes.byref(kv), ctypes.byref(front),
                                  ctypes.byref(call), None)


def test_front_refusals_happen_before_any_launch():
    # fake (aligned, non-null) pointers: every case must be refused by the
    # host checks; never run where a GPU could receive a launch
    import torch
    if torch.cuda.is_available():
        pytest.skip("fake-pointer refusals run on hosts without a GPU only")
    assert _front_refusal(front=hb.FrontSpec(rotary=48, eps=1e-6, gemma=1)) == hb.HB_DECLINE_HEAD_DIM
    assert _front_refusal(front=hb.FrontSpec(rotary=288, eps=1e-6, gemma=1)) == hb.HB_DECLINE_HEAD_DIM
    assert _front_refusal(rows=0) == hb.HB_DECLINE_EMPTY
    assert _front_refusal(q=258) == hb.HB_ERR_ARG  # misaligned
    assert _front_refusal(cos=None) == hb.HB_ERR_ARG
    assert _front_refusal(keys=None) == hb.HB_ERR_ARG  # keys without values
    assert _front_refusal(past=63) == hb.HB_ERR_ARG  # past + rows beyond the capacity
    assert _front_refusal(rows=17) == hb.HB_ERR_ARG  # above max_batch
    assert _front_refusal(kv=hb.KvSpec(heads=2, head_dim=256, stride=64 * 256, capacity=64,
                                       max_batch=16)) == hb.HB_DECLINE_GEOMETRY
    assert _front_refusal(front=hb.FrontSpec(rotary=64, eps=float("nan"), gemma=1)) == hb.HB_ERR_ARG
    assert "eps" in hb.last_error()


# ---------------------------------------------------------------------- GPU

def _gpu_front(inp, append=True):
    import torch
    dev = "cuda"
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)  # noqa: E731
    q, k, v = t(inp.q), t(inp.k), t(inp.v)
    qn, kn, cs, sn = t(inp.q_norm), t(inp.k_norm), t(inp.cos), t(inp.sin)
    keys, values = t(inp.keys), t(inp.values)
    spec = hb.attention_spec(inp.heads, inp.heads // inp.kv_heads, inp.head_dim,
                             inp.gated)
    kv = hb.KvSpec(heads=inp.kv_heads, head_dim=inp.head_dim,
                   stride=inp.capacity * inp.head_dim, capacity=inp.capacity,
                   max_batch=inp.rows)
    hb.attn_front(spec, kv, q, k, v, qn, kn, cs, sn, rows=inp.rows, past=inp.past,
                  rotary=inp.rotary, gemma=inp.gemma, keys=keys if append else None,
                  values=values if append else None)
    torch.cuda.synchronize()
    u = lambda x: x.cpu().numpy().view(np.uint16)  # noqa: E731
    return u(q), u(k), u(keys), u(values)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_front_matches_oracle_bit_for_bit(case):
    inp = _inputs(case)
    want = oracle_front(inp)
    got = _gpu_front(inp)
    for name, g, w in zip(("q", "k", "keys", "values"), got, want):
        assert np.array_equal(g, w), f"{name}: {np.count_nonzero(g != w)} elements differ"


@pytest.mark.gpu
def test_front_without_append_leaves_the_cache():
    inp = FrontInputs(9, 40, seed=0xF500)
    q, k, _, _ = oracle_front(inp, append=False)
    gq, gk, gkeys, gvalues = _gpu_front(inp, append=False)
    assert np.array_equal(gq, q) and np.array_equal(gk, k)
    assert np.array_equal(gkeys, inp.keys) and np.array_equal(gvalues, inp.values)


@pytest.mark.gpu
def test_front_golden_fixture():
    z = np.load(GOLDEN)
    m = z["meta"]
    inp = FrontInputs(int(m[0]), int(m[1]), heads=int(m[2]), kv_heads=int(m[3]),
                      head_dim=int(m[4]), rotary=int(m[5]), gated=bool(m[7]),
                      gemma=bool(m[6]), capacity=z["keys0"].shape[1])
    inp.q, inp.k, inp.v = z["q"], z["k"], z["v"]
    inp.q_norm, inp.k_norm, inp.cos, inp.sin = z["q_norm"], z["k_norm"], z["cos"], z["sin"]
    inp.keys, inp.values = z["keys0"], z["values0"]
    got = _gpu_front(inp)
    for g, w in zip(got, (z["q_out"], z["k_out"], z["keys"], z["values"])):
        assert np.array_equal(g, w)


@pytest.mark.gpu
def test_front_then_decode_matches_the_oracle_layer():
    """The front end feeding the decode SDPA on the device equals the oracle's
    front end feeding its own attention (the attention node's tolerance)."""
    import torch
    from harness import assert_sdpa_close
    inp = FrontInputs(1, 300, capacity=301, seed=0xF600)
    q, k, keys, values = oracle_front(inp)
    want = O.attention(q, keys, values, rows=1, past=300, heads=16, gqa=4, head_dim=256,
                       q_row=inp.q_row, q_head=256, out_row=16 * 256, kv_stride=301 * 256,
                       gate_offset=16 * 256, scale=1 / 16.0)
    gq, _, gkeys, gvalues = _gpu_front(inp)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()  # noqa: E731
    out = torch.zeros((1, 16 * 256), dtype=torch.int16, device="cuda")
    spec = hb.attention_spec(16, 4, 256, True)
    hb.attention(spec, t(gq), t(gkeys), t(gvalues), out, rows=1, past=300, kv_stride=301 * 256,
                 regime="decode")
    torch.cuda.synchronize()
    assert_sdpa_close(out.cpu().numpy().view(np.uint16), want, "front + decode")
