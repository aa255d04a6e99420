"""Shared helpers of the tests: the oracle side of each comparison, the GPU
side through the C ABI, and the tolerance checks.

Tolerances (stated by the port's contract):
  SDPA     max |gpu - oracle| <= 2 bf16 ulp of the output scale (max |oracle|)
           and relative Frobenius error <= 5e-3;
  DeltaNet relative Frobenius error <= 1e-2 for the chunked prefill; the
           recurrent kernel is required to be bit-exact.
"""
from __future__ import annotations

import numpy as np

import oracle
from herbert_b200.inputs import AttentionInputs, DeltaInputs, bf16_bits_to_f32

SDPA_ULPS = 2.0
SDPA_REL_FROB = 5e-3
GDN_REL_FROB = 1e-2


def bf16_ulp(x: float) -> float:
    return float(2.0 ** (np.floor(np.log2(x)) - 7))


def sdpa_errors(got_bits, ref_bits):
    g = bf16_bits_to_f32(got_bits).astype(np.float64)
    r = bf16_bits_to_f32(ref_bits).astype(np.float64)
    scale = float(np.abs(r).max())
    maxabs = float(np.abs(g - r).max())
    rel = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
    return maxabs, rel, SDPA_ULPS * bf16_ulp(scale) if scale > 0 else 0.0


def assert_sdpa_close(got_bits, ref_bits, what=""):
    assert np.all(np.isfinite(bf16_bits_to_f32(got_bits))), f"{what}: non-finite output"
    maxabs, rel, tol = sdpa_errors(got_bits, ref_bits)
    assert maxabs <= tol and rel <= SDPA_REL_FROB, (
        f"{what}: max abs {maxabs:.3e} (tol {tol:.3e}), rel frob {rel:.3e} (tol {SDPA_REL_FROB})")
    return maxabs, rel


def rel_frob(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


# ------------------------------------------------------------------ oracle

def oracle_attention(inp: AttentionInputs, threads: int = 0, impl=None) -> np.ndarray:
    # the AVX512-BF16 transcription (row by row) and the portable emulation
    # (8-row blocks) give identical bits (tests/test_oracle.py); the first is
    # ~40x faster where the CPU has it
    if impl is None:
        impl = 1 if oracle.has_avx512bf16() else 0
    out = oracle.attention(inp.q.ravel(), inp.keys.ravel(), inp.values.ravel(), rows=inp.rows,
                           past=inp.past, heads=inp.heads, gqa=inp.gqa, head_dim=inp.head_dim,
                           q_row=inp.q_row, q_head=inp.head_dim, out_row=inp.out_row,
                           gate_offset=inp.gate_offset if inp.gated else None,
                           kv_stride=inp.kv_stride, scale=inp.scale, impl=impl,
                           use_block=0 if impl == 1 else 1, threads=threads)
    return out.reshape(inp.rows, inp.out_row)


def oracle_gdn(inp: DeltaInputs, l2=True, threads=0):
    out, state, _ = oracle.gdn_layer(inp.qkv, inp.state, inp.beta, inp.decay, nk=inp.nk,
                                     nv=inp.nv, hkd=inp.hkd, hvd=inp.hvd, l2=l2,
                                     threads=threads)
    return out, state


# --------------------------------------------------------------------- GPU

def to_dev_bf16(a: np.ndarray, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device)


def to_dev_f32(a: np.ndarray, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


def bits_of(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def gpu_attention(inp: AttentionInputs, regime="decode", workspace=None, out=None):
    import torch
    import herbert_b200 as hb
    q = to_dev_bf16(inp.q)
    keys = to_dev_bf16(inp.keys)
    values = to_dev_bf16(inp.values)
    if out is None:
        out = torch.zeros((inp.rows, inp.out_row), dtype=torch.int16, device="cuda")
    spec = hb.attention_spec(inp.heads, inp.gqa, inp.head_dim, inp.gated)
    ws = hb.attention(spec, q, keys, values, out, rows=inp.rows, past=inp.past,
                      kv_stride=inp.kv_stride, capacity=inp.capacity, scale=inp.scale,
                      regime=regime, workspace=workspace)
    torch.cuda.synchronize()
    ws.status()
    return bits_of(out), ws


def gpu_gdn(inp: DeltaInputs, regime="decode", l2=True, workspace=None):
    import torch
    import herbert_b200 as hb
    state = to_dev_f32(inp.state)
    qkv = to_dev_f32(inp.qkv)
    beta = to_dev_f32(inp.beta)
    decay = to_dev_f32(inp.decay)
    out = torch.zeros((inp.rows, inp.nv * inp.hvd), dtype=torch.float32, device="cuda")
    shape = hb.DeltaShape(nk=inp.nk, nv=inp.nv, hkd=inp.hkd, hvd=inp.hvd)
    ws = hb.delta_recurrence(shape, state, out, qkv, beta, decay, rows=inp.rows, l2=l2,
                             regime=regime, workspace=workspace)
    torch.cuda.synchronize()
    return out.cpu().numpy(), state.cpu().numpy(), ws


# --------------------------------------------------------------- fixtures

GOLDEN_DIR = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden")
ATTN_FIXTURES = ["attn_decode_n38", "attn_decode_n1", "attn_rows11_past5", "attn_hd128_g2_nogate"]
GDN_FIXTURES = ["gdn_rows5_zero_state", "gdn_rows3_warm_state"]


def load_attn_fixture(name):
    import os
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    rows, past, heads, kvh, hd, gated = (int(x) for x in z["meta"])
    inp = AttentionInputs.__new__(AttentionInputs)
    inp.rows, inp.past, inp.heads, inp.kv_heads, inp.head_dim = rows, past, heads, kvh, hd
    inp.gqa, inp.gated = heads // kvh, bool(gated)
    inp.capacity = z["keys"].shape[1]
    qd = heads * hd
    inp.q_row, inp.out_row = (2 * qd if gated else qd), qd
    inp.gate_offset = qd if gated else -1
    inp.kv_stride = inp.capacity * hd
    inp.scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    inp.q, inp.keys, inp.values = z["q"], z["keys"], z["values"]
    return inp, z["out"]


def load_gdn_fixture(name):
    import os
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    rows, nk, nv, hkd, hvd = (int(x) for x in z["meta"])
    inp = DeltaInputs.__new__(DeltaInputs)
    inp.rows, inp.nk, inp.nv, inp.hkd, inp.hvd = rows, nk, nv, hkd, hvd
    inp.conv = 2 * nk * hkd + nv * hvd
    inp.qkv, inp.beta, inp.decay, inp.state = z["qkv"], z["beta"], z["decay"], z["state0"]
    return inp, z["out"], z["state"]
