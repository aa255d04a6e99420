"""Seeded synthetic inputs in the reference's layouts (numpy, host side).

The configurations are the reference's attention path at Qwen3.5 geometry:
16 query heads, 4 KV heads, head_dim 256 (SDPA); 16 key heads, 32 value
heads, dk = dv = 128 (GatedDeltaNet).  Values are N(0,1) rounded to bf16
(round to nearest even), drawn from numpy's PCG64 with a fixed seed per
tensor; no dataset is involved.
"""
from __future__ import annotations

import numpy as np

QWEN_HEADS, QWEN_KV_HEADS, QWEN_HEAD_DIM = 16, 4, 256
QWEN_NK, QWEN_NV, QWEN_HKD, QWEN_HVD = 16, 32, 128, 128


def f32_to_bf16_bits(x) -> np.ndarray:
    """float -> bf16 bits, round to nearest even (finite values)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal_bf16(shape, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))


class AttentionInputs:
    """q rows [Q | gate], head-major K/V caches, as the engine lays them out.

    q      : [rows, q_row]                 bf16 bits (q_row = 2*heads*head_dim)
    keys   : [kv_heads, capacity, head_dim] bf16 bits
    values : [kv_heads, capacity, head_dim] bf16 bits
    Row r is the query at position past + r; positions [0, past + rows) of
    the caches are filled, the rest of the reserve is zero.
    """

    def __init__(self, rows, past, heads=QWEN_HEADS, kv_heads=QWEN_KV_HEADS,
                 head_dim=QWEN_HEAD_DIM, capacity=None, gated=True, seed=0x5EED0001):
        self.rows, self.past = rows, past
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.gqa = heads // kv_heads
        self.capacity = capacity or (past + rows)
        self.gated = gated
        qd = heads * head_dim
        self.q_row = 2 * qd if gated else qd
        self.out_row = qd
        self.gate_offset = qd if gated else -1
        self.kv_stride = self.capacity * head_dim
        self.scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
        n = past + rows
        self.q = normal_bf16((rows, self.q_row), seed)
        self.keys = np.zeros((kv_heads, self.capacity, head_dim), np.uint16)
        self.values = np.zeros((kv_heads, self.capacity, head_dim), np.uint16)
        self.keys[:, :n] = normal_bf16((kv_heads, n, head_dim), seed + 1)
        self.values[:, :n] = normal_bf16((kv_heads, n, head_dim), seed + 2)


class DeltaInputs:
    """One GatedDeltaNet block in the reference layout (f32).

    qkv   : [rows, 2*nk*hkd + nv*hvd]  q, k ~ bf16 N(0,1) (L2 applied by the
            kernels), v ~ bf16 N(0,1)
    beta  : [rows, nv]  sigmoid(N(0,1))
    decay : [rows, nv]  exp(-softplus(N(0,1)))
    state : [nv, hkd, hvd] zeros (or a given state)
    """

    def __init__(self, rows, nk=QWEN_NK, nv=QWEN_NV, hkd=QWEN_HKD, hvd=QWEN_HVD,
                 seed=0x5EED0003, state=None):
        self.rows, self.nk, self.nv, self.hkd, self.hvd = rows, nk, nv, hkd, hvd
        key, value = nk * hkd, nv * hvd
        self.conv = 2 * key + value
        self.qkv = bf16_bits_to_f32(normal_bf16((rows, self.conv), seed)).copy()
        rng = np.random.default_rng(seed + 1)
        b = rng.standard_normal((rows, nv))
        g = rng.standard_normal((rows, nv))
        self.beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)
        self.decay = np.exp(-np.logaddexp(0.0, g)).astype(np.float32)
        self.state = (np.zeros((nv, hkd, hvd), np.float32) if state is None
                      else np.ascontiguousarray(state, dtype=np.float32))


def batch_lengths(nseq=64, lo=1024, hi=32768, seed=0x5EED0004) -> np.ndarray:
    """KV lengths of the batched-decode configuration, uniform in [lo, hi]."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=nseq)


class FrontInputs:
    """One call of the attention front end (head-norm-rope + kv-append).

    q      : [rows, q_row] bf16 bits (the heads' part is transformed)
    k, v   : [rows, kv_heads*head_dim] bf16 bits
    q_norm, k_norm : [head_dim] bf16 bits, N(0, 0.1) (Gemma-form weights
             are small deviations around 0)
    cos, sin : [capacity, rotary/2] bf16 bits of the RoPE angles
             pos * 1e7^(-2j/rotary) (Qwen3.5's rope theta)
    keys, values : [kv_heads, capacity, head_dim] bf16 bits (prior content)
    """

    def __init__(self, rows, past, heads=QWEN_HEADS, kv_heads=QWEN_KV_HEADS,
                 head_dim=QWEN_HEAD_DIM, rotary=64, gated=True, gemma=True, capacity=None,
                 seed=0xF407):
        self.rows, self.past, self.heads, self.kv_heads = rows, past, heads, kv_heads
        self.head_dim, self.rotary, self.gemma = head_dim, rotary, gemma
        self.capacity = capacity or past + rows + 3
        qd = heads * head_dim
        self.q_row = 2 * qd if gated else qd
        self.gated = gated
        self.q = normal_bf16((rows, self.q_row), seed)
        self.k = normal_bf16((rows, kv_heads * head_dim), seed + 1)
        self.v = normal_bf16((rows, kv_heads * head_dim), seed + 2)
        self.q_norm = f32_to_bf16_bits(np.random.default_rng(seed + 3).standard_normal(head_dim) * 0.1)
        self.k_norm = f32_to_bf16_bits(np.random.default_rng(seed + 4).standard_normal(head_dim) * 0.1)
        half = max(rotary // 2, 1)
        pos = np.arange(self.capacity, dtype=np.float64)[:, None]
        inv_freq = 1e7 ** (-np.arange(half, dtype=np.float64) * 2 / max(rotary, 2))
        self.cos = f32_to_bf16_bits(np.cos(pos * inv_freq))
        self.sin = f32_to_bf16_bits(np.sin(pos * inv_freq))
        self.keys = normal_bf16((kv_heads, self.capacity, head_dim), seed + 5)
        self.values = normal_bf16((kv_heads, self.capacity, head_dim), seed + 6)


class DeltaFrontInputs:
    """One call of the DeltaNet front end (conv + SiLU, gates) and of the gated
    norm, Qwen3.5 geometry by default.

    qkv        : [rows, conv] f32 projection output, N(0, 1)
    conv_state : [conv, ck] f32, N(0, 1) (the last ck inputs of an earlier block)
    conv_weight: [conv, ck] bf16 bits, N(0, 0.25)
    ab         : [rows, 2*nv] f32, a then b projections, N(0, 2)
    dt_bias    : [nv] bf16 bits, softplus^-1 of dt ~ logU(1e-3, 1e-1) (the usual init)
    a_log      : [nv] f32, log U(1, 16)
    x, z       : [rows, nv*hvd] f32, recurrence output N(0, 0.05) and gate N(0, 1)
    norm_weight: [hvd] bf16 bits, 1 + N(0, 0.1)
    """

    def __init__(self, rows, nk=QWEN_NK, nv=QWEN_NV, hkd=QWEN_HKD, hvd=QWEN_HVD, ck=4,
                 seed=0xDE17A):
        self.rows, self.nk, self.nv, self.hkd, self.hvd, self.ck = rows, nk, nv, hkd, hvd, ck
        self.conv = 2 * nk * hkd + nv * hvd
        rng = np.random.default_rng(seed)
        f32 = np.float32
        self.qkv = rng.standard_normal((rows, self.conv), dtype=f32)
        self.conv_state = rng.standard_normal((self.conv, ck), dtype=f32)
        self.conv_weight = f32_to_bf16_bits(rng.standard_normal((self.conv, ck)) * 0.25)
        self.ab = (rng.standard_normal((rows, 2 * nv)) * 2.0).astype(f32)
        dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), nv))
        self.dt_bias = f32_to_bf16_bits(dt + np.log(-np.expm1(-dt)))
        self.a_log = np.log(rng.uniform(1.0, 16.0, nv)).astype(f32)
        self.x = (rng.standard_normal((rows, nv * hvd)) * 0.05).astype(f32)
        self.z = rng.standard_normal((rows, nv * hvd), dtype=f32)
        self.norm_weight = f32_to_bf16_bits(1.0 + rng.standard_normal(hvd) * 0.1)
