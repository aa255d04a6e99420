"""CPU tests of the oracle (no GPU).

The reference ships no tests and no golden vectors and cannot be built here,
so the oracle is pinned by (1) the hardware: its portable emulation of every
x86 instruction the reference emits must equal the same instruction sequence
run with intrinsics on an AVX512-BF16 CPU, and (2) the reference's own stated
invariants, each cited.
"""
import numpy as np
import pytest

import oracle
from herbert_b200.inputs import AttentionInputs, DeltaInputs, bf16_bits_to_f32
from harness import oracle_attention, oracle_gdn, rel_frob

needs_bf16 = pytest.mark.skipif(not oracle.has_avx512bf16(),
                                reason="CPU without AVX512-BF16: hardware pin unavailable")


@needs_bf16
def test_vdpbf16ps_emulation_matches_hardware():
    rng = np.random.default_rng(1)
    L = oracle.lib()
    for t in range(3000):
        acc = (rng.standard_normal(16) * rng.choice([1e-3, 1.0, 1e3])).astype(np.float32)
        a = oracle.f32_to_bf16(rng.standard_normal(32).astype(np.float32) *
                               np.float32(rng.choice([1.0, 1e-19, 1e19, 1e-38])))
        b = oracle.f32_to_bf16(rng.standard_normal(32).astype(np.float32))
        s, h = acc.copy(), acc.copy()
        L.orc_dpbf16_scalar(oracle._p(s, oracle._f32p), oracle._p(a, oracle._u16p),
                            oracle._p(b, oracle._u16p))
        assert L.orc_dpbf16_hw(oracle._p(h, oracle._f32p), oracle._p(a, oracle._u16p),
                               oracle._p(b, oracle._u16p)) == 0
        assert np.array_equal(s.view(np.uint32), h.view(np.uint32)), t


@needs_bf16
def test_exp_polynomial_matches_hardware():
    L = oracle.lib()
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.uniform(-100, 0, 8000), rng.uniform(-2, 2, 8000),
                        [-np.inf, 0.0, -0.0, 88.0, -87.33654, -87.4, -126.0, 1e-30]])
    x = x[: len(x) // 16 * 16].astype(np.float32)
    for i in range(0, len(x), 16):
        xi = np.ascontiguousarray(x[i:i + 16])
        yh = np.empty(16, np.float32)
        assert L.orc_exp_poly_hw16(oracle._p(xi, oracle._f32p), oracle._p(yh, oracle._f32p)) == 0
        ys = np.array([L.orc_exp_poly(float(v)) for v in xi], np.float32)
        assert np.array_equal(ys.view(np.uint32), yh.view(np.uint32))


@needs_bf16
@pytest.mark.parametrize("n", [1, 2, 7, 15, 16, 17, 33, 100, 257])
@pytest.mark.parametrize("chains", [1, 4])
def test_sdpa_head_emulation_equals_avx512_transcription(n, chains):
    d = 256
    q = oracle.normal_bf16((d,), 10 + n)
    k = oracle.normal_bf16((n, d), 20 + n)
    v = oracle.normal_bf16((n, d), 30 + n)
    a = oracle.sdpa_head(q, k, v, n, 1 / 16, impl=0, qk_chains=chains)
    b = oracle.sdpa_head(q, k, v, n, 1 / 16, impl=1, qk_chains=chains)
    assert np.array_equal(a, b)


@needs_bf16
def test_gate_emulation_equals_avx512_transcription():
    a = oracle.normal_bf16((8192,), 40)
    g = oracle.f32_to_bf16(bf16_bits_to_f32(oracle.normal_bf16((8192,), 41)) * np.float32(30))
    assert np.array_equal(oracle.sigmoid_mul(a, g, 0), oracle.sigmoid_mul(a, g, 1))


@pytest.mark.parametrize("past", [0, 1, 8, 15, 16, 100])
def test_prefill_block_equals_repeated_decode(past):
    """src/jit/emit_sdpa.rs:163-171: the block is bitwise equal to the
    decode kernel called row by row."""
    d, rows = 256, 8
    q = oracle.normal_bf16((rows, d), 50 + past)
    k = oracle.normal_bf16((past + rows, d), 60 + past)
    v = oracle.normal_bf16((past + rows, d), 70 + past)
    blk = oracle.sdpa_prefill_block(q, k, v, past, 1 / 16)
    dec = np.stack([oracle.sdpa_head(q[i], k, v, past + i + 1, 1 / 16) for i in range(rows)])
    assert np.array_equal(blk, dec)


def test_attention_node_block_and_row_paths_agree():
    inp = AttentionInputs(rows=19, past=5)
    args = dict(rows=inp.rows, past=inp.past, heads=inp.heads, gqa=inp.gqa,
                head_dim=inp.head_dim, q_row=inp.q_row, q_head=inp.head_dim, out_row=inp.out_row,
                gate_offset=inp.gate_offset, kv_stride=inp.kv_stride, scale=inp.scale)
    a = oracle.attention(inp.q.ravel(), inp.keys.ravel(), inp.values.ravel(), use_block=1, **args)
    b = oracle.attention(inp.q.ravel(), inp.keys.ravel(), inp.values.ravel(), use_block=0, **args)
    assert np.array_equal(a, b)


def test_qk_group_moves_outputs_at_most_one_bf16_step():
    """src/jit/emit_sdpa.rs:231-247: one accumulation chain instead of four
    moves a score by at most one bf16 step."""
    d, n = 256, 300
    worst = 0
    for s in range(20):
        q = oracle.normal_bf16((d,), 80 + s)
        k = oracle.normal_bf16((n, d), 90 + s)
        v = oracle.normal_bf16((n, d), 100 + s)
        a = oracle.sdpa_head(q, k, v, n, 1 / 16, qk_chains=1).astype(np.int32)
        b = oracle.sdpa_head(q, k, v, n, 1 / 16, qk_chains=4).astype(np.int32)
        worst = max(worst, int(np.abs(a - b).max()))
    assert worst <= 1


def _f64_attention(inp: AttentionInputs):
    q = bf16_bits_to_f32(inp.q).astype(np.float64)
    K = bf16_bits_to_f32(inp.keys).astype(np.float64)
    V = bf16_bits_to_f32(inp.values).astype(np.float64)
    out = np.zeros((inp.rows, inp.out_row))
    for r in range(inp.rows):
        n = inp.past + r + 1
        for h in range(inp.heads):
            qh = q[r, h * inp.head_dim:(h + 1) * inp.head_dim]
            kh = h // inp.gqa
            s = K[kh, :n] @ qh * inp.scale
            p = np.exp(s - s.max())
            p /= p.sum()
            o = p @ V[kh, :n]
            if inp.gated:
                g = q[r, inp.gate_offset + h * inp.head_dim:inp.gate_offset + (h + 1) * inp.head_dim]
                o = o / (1 + np.exp(-g))
            out[r, h * inp.head_dim:(h + 1) * inp.head_dim] = o
    return out


@pytest.mark.parametrize("rows,past", [(1, 0), (1, 511), (9, 40)])
def test_sdpa_oracle_is_accurate(rows, past):
    inp = AttentionInputs(rows=rows, past=past)
    got = bf16_bits_to_f32(oracle_attention(inp)).astype(np.float64)
    ref = _f64_attention(inp)
    assert rel_frob(got, ref) < 4e-3


def _f64_gdn(inp: DeltaInputs):
    key = inp.nk * inp.hkd
    S = inp.state.astype(np.float64).copy()
    out = np.zeros((inp.rows, inp.nv * inp.hvd))
    scale = 1.0 / np.sqrt(inp.hkd)
    for t in range(inp.rows):
        row = inp.qkv[t].astype(np.float64)
        for h in range(inp.nv):
            kh = h // (inp.nv // inp.nk)
            q = row[kh * inp.hkd:(kh + 1) * inp.hkd]
            k = row[key + kh * inp.hkd:key + (kh + 1) * inp.hkd]
            q = q / np.sqrt((q * q).sum() + 1e-6)
            k = k / np.sqrt((k * k).sum() + 1e-6)
            v = row[2 * key + h * inp.hvd:2 * key + (h + 1) * inp.hvd]
            S[h] *= inp.decay[t, h]
            delta = (v - S[h].T @ k) * inp.beta[t, h]
            S[h] += np.outer(k, delta)
            out[t, h * inp.hvd:(h + 1) * inp.hvd] = S[h].T @ q * scale
    return out, S


def test_gdn_oracle_is_accurate():
    inp = DeltaInputs(rows=24, nk=2, nv=4)
    out, state = oracle_gdn(inp)
    ref_out, ref_state = _f64_gdn(inp)
    assert rel_frob(out, ref_out) < 1e-5
    assert rel_frob(state, ref_state) < 1e-5


def test_gdn_fma_form_differs_only_in_last_bits():
    """src/jit/target/x86/emit_recurrence.rs:31-41: the FMA form returns the
    bits of a scalar written with mul_add, differing at the last bit."""
    inp = DeltaInputs(rows=6, nk=2, nv=4)
    a, sa, _ = oracle.gdn_layer(inp.qkv, inp.state, inp.beta, inp.decay, nk=2, nv=4, hkd=128,
                                hvd=128, fma=0)
    b, sb, _ = oracle.gdn_layer(inp.qkv, inp.state, inp.beta, inp.decay, nk=2, nv=4, hkd=128,
                                hvd=128, fma=1)
    assert not np.array_equal(a, b)
    assert rel_frob(a, b) < 1e-6 and rel_frob(sa, sb) < 1e-6


def test_l2norm_matches_sequential_definition():
    x = np.random.default_rng(3).standard_normal(128).astype(np.float32)
    y = oracle.l2norm(x)
    s = np.float32(0)
    for v in x:
        s = np.float32(s + np.float32(v * v))
    inv = np.float32(1) / np.sqrt(np.float32(s + np.float32(1e-6)))
    assert np.array_equal(y, (x * inv).astype(np.float32))
