"""ctypes/numpy wrapper of the CPU oracle (``libherbert_oracle.so``).

TEST INFRASTRUCTURE ONLY.  Imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline / reference legs of ``bench.py`` -- as the checker, never
as the thing measured on the GPU path.

The C file restates the reference's x86 AVX-512 BF16 attention-path kernels
(xigh/herbert-jit-bf16):

* decode SDPA ``SdpaHeadFn``  -- src/jit/emit_sdpa.rs:131-140,
  src/jit/target/x86/emit_sdpa/x86/decode.rs:59-428, prefill.rs:496-605;
* prefill block ``SdpaPrefillFn`` -- src/jit/emit_sdpa.rs:173-304,
  src/jit/target/x86/emit_sdpa/x86/prefill.rs:733-912;
* output gate ``ElemOp::SigmoidMul`` -- src/jit/target/x86/emit_elem.rs:333-420;
* DeltaNet L2 norm and recurrence -- src/jit/target/x86/execution/delta.rs:28-62,
  519-607; src/jit/target/x86/emit_recurrence.rs:108-217;
* attention front end (head-norm-rope of q and k, kv-append) --
  src/jit/schedule/lowering.rs:549-592, src/jit/target/x86/emit_elem.rs:242-330,
  479-514, src/jit/target/x86/execution/transforms.rs:30-81;
* DeltaNet front end: causal conv + SiLU, beta/decay gates, gated RMS norm --
  src/jit/target/x86/execution/delta.rs:290-389, 609-774, delta_scalar.rs:85-239,
  src/jit/target/x86/emit_conv.rs, emit_gated_norm.rs, execution/math.rs.

Parity is unpinned by reference outputs (the Rust reference cannot be built
in this image and ships no golden vectors); the restatement is pinned to the
x86 semantics of the emitted instructions instead (see the C header).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libherbert_oracle.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_sz = ctypes.c_size_t

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
        os.path.join(HERE, "herbert_oracle.c")
    ):
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_has_avx512bf16.restype = ctypes.c_int
        L.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_bf16_to_f32.restype = ctypes.c_float
        L.orc_f32_to_bf16_cvtne.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16_cvtne.restype = ctypes.c_uint16
        L.orc_f32_to_bf16_array.argtypes = [_f32p, _u16p, _sz]
        L.orc_bf16_to_f32_array.argtypes = [_u16p, _f32p, _sz]
        L.orc_dpbf16_scalar.argtypes = [_f32p, _u16p, _u16p]
        L.orc_dpbf16_hw.argtypes = [_f32p, _u16p, _u16p]
        L.orc_dpbf16_hw.restype = ctypes.c_int
        L.orc_exp_poly.argtypes = [ctypes.c_float]
        L.orc_exp_poly.restype = ctypes.c_float
        L.orc_exp_poly_hw16.argtypes = [_f32p, _f32p]
        L.orc_exp_poly_hw16.restype = ctypes.c_int
        L.orc_sdpa_head.argtypes = [_u16p, _u16p, _u16p, _f32p, _u16p, _sz, _sz,
                                    ctypes.c_float, ctypes.c_int, ctypes.c_int]
        L.orc_sdpa_head.restype = ctypes.c_int
        L.orc_sdpa_prefill_block.argtypes = [_u16p, _u16p, _u16p, _u16p, _sz, _sz, _sz,
                                             _sz, _sz, ctypes.c_float]
        L.orc_sdpa_prefill_block.restype = ctypes.c_int
        L.orc_sigmoid_mul.argtypes = [_u16p, _u16p, _u16p, _sz, ctypes.c_int]
        L.orc_sigmoid_mul.restype = ctypes.c_int
        L.orc_attention.argtypes = [_u16p, _u16p, _u16p, _u16p, _sz, _sz, _sz, _sz, _sz,
                                    _sz, _sz, _sz, ctypes.c_ssize_t, _sz, ctypes.c_float,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_attention.restype = ctypes.c_int
        L.orc_l2norm.argtypes = [_f32p, _sz, ctypes.c_float]
        L.orc_gdn_recurrence.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _sz, _sz,
                                         ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_int]
        L.orc_gdn_layer.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz,
                                    _sz, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                    ctypes.c_int]
        L.orc_gdn_layer.restype = ctypes.c_int
        L.orc_attn_front.argtypes = [_u16p, _sz, _sz, _u16p, _u16p, _sz, _sz, _sz, _u16p, _u16p,
                                     _u16p, _u16p, _sz, ctypes.c_float, ctypes.c_int, _u16p,
                                     _u16p, _sz, _sz, _sz, ctypes.c_int]
        L.orc_attn_front.restype = ctypes.c_int
        _u64p = ctypes.POINTER(ctypes.c_uint64)
        for fn in ("orc_expf_arm_array", "orc_logf_arm_array", "orc_expf_libm_array",
                   "orc_logf_libm_array"):
            getattr(L, fn).argtypes = [_f32p, _f32p, _sz]
        L.orc_mathf_tables.argtypes = [_u64p, _u64p]
        L.orc_mathf_sweep.argtypes = [ctypes.c_uint32, ctypes.c_int]
        L.orc_mathf_sweep.restype = ctypes.c_uint64
        L.orc_gdn_conv.argtypes = [_f32p, _sz, _sz, _u16p, _f32p, _sz, ctypes.c_int]
        L.orc_gdn_conv.restype = ctypes.c_int
        L.orc_gdn_gates.argtypes = [_f32p, _u16p, _f32p, _f32p, _f32p, _sz, _sz]
        L.orc_gdn_gated_norm.argtypes = [_f32p, _f32p, _u16p, _u16p, _sz, _sz, ctypes.c_float,
                                         ctypes.c_int]
        L.orc_gdn_gated_norm.restype = ctypes.c_int
        L.orc_fill_normal_bf16.argtypes = [_u16p, _sz, ctypes.c_uint64]
        L.orc_fill_normal_f64.argtypes = [_f64p, _sz, ctypes.c_uint64]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(t)


def has_avx512bf16() -> bool:
    return bool(lib().orc_has_avx512bf16())


# ------------------------------------------------------------ conversions

def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    """Exact widening: bf16 bits (uint16) -> float32."""
    return (x.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """vcvtneps2bf16 semantics (RNE; zero/denormal -> signed zero)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16_array(_p(x, _f32p), _p(y, _u16p), x.size)
    return y


def normal_bf16(shape, seed: int) -> np.ndarray:
    """Seeded N(0,1) rounded to bf16 bits (splitmix64 + Box-Muller)."""
    n = int(np.prod(shape))
    y = np.empty(n, dtype=np.uint16)
    lib().orc_fill_normal_bf16(_p(y, _u16p), n, ctypes.c_uint64(seed & (2**64 - 1)))
    return y.reshape(shape)


def normal_f64(shape, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    y = np.empty(n, dtype=np.float64)
    lib().orc_fill_normal_f64(_p(y, _f64p), n, ctypes.c_uint64(seed & (2**64 - 1)))
    return y.reshape(shape)


# ------------------------------------------------------------------ SDPA

def sdpa_head(q, k, v, n, scale, impl=0, qk_chains=1):
    """One decode head: q [d], k/v [>=n, d] bf16 bits -> out [d] bf16 bits."""
    d = q.shape[-1]
    out = np.empty(d, dtype=np.uint16)
    q = np.ascontiguousarray(q); k = np.ascontiguousarray(k); v = np.ascontiguousarray(v)
    rc = lib().orc_sdpa_head(_p(q, _u16p), _p(k, _u16p), _p(v, _u16p), None, _p(out, _u16p),
                             n, d, ctypes.c_float(scale), impl, qk_chains)
    if rc != 0:
        raise RuntimeError(f"orc_sdpa_head rc={rc}")
    return out


def sdpa_prefill_block(q, k, v, past, scale):
    """q [rows, d] (rows <= 8) against k/v [past+rows, d] -> out [rows, d]."""
    rows, d = q.shape
    out = np.empty((rows, d), dtype=np.uint16)
    q = np.ascontiguousarray(q); k = np.ascontiguousarray(k); v = np.ascontiguousarray(v)
    rc = lib().orc_sdpa_prefill_block(_p(q, _u16p), _p(k, _u16p), _p(v, _u16p), _p(out, _u16p),
                                      past, rows, d, d, d, ctypes.c_float(scale))
    if rc != 0:
        raise RuntimeError(f"orc_sdpa_prefill_block rc={rc}")
    return out


def sigmoid_mul(a, b, impl=0):
    a = np.ascontiguousarray(a); b = np.ascontiguousarray(b)
    y = np.empty_like(a)
    rc = lib().orc_sigmoid_mul(_p(a, _u16p), _p(b, _u16p), _p(y, _u16p), a.size, impl)
    if rc != 0:
        raise RuntimeError(f"orc_sigmoid_mul rc={rc}")
    return y


def attention(q, keys, values, *, rows, past, heads, gqa, head_dim, q_row, q_head, out_row,
              gate_offset, kv_stride, scale, impl=0, use_block=1, threads=0, out=None):
    """The attention node plus the gate node over flat bf16-bit buffers.

    q: flat uint16 holding `rows` query rows at stride q_row; keys/values:
    flat uint16 caches, KV head h at h*kv_stride; returns flat out
    [rows*out_row]."""
    q = np.ascontiguousarray(q); keys = np.ascontiguousarray(keys)
    values = np.ascontiguousarray(values)
    if out is None:
        out = np.zeros(rows * out_row, dtype=np.uint16)
    rc = lib().orc_attention(_p(q, _u16p), _p(keys, _u16p), _p(values, _u16p), _p(out, _u16p),
                             rows, past, heads, gqa, head_dim, q_row, q_head, out_row,
                             -1 if gate_offset is None else gate_offset, kv_stride,
                             ctypes.c_float(scale), impl, use_block, threads)
    if rc != 0:
        raise RuntimeError(f"orc_attention rc={rc}")
    return out


# -------------------------------------------------------------- DeltaNet

def attn_front(q, k, v, q_norm, k_norm, cos, sin, *, heads, kv_heads, head_dim, rotary, past,
               eps=1e-6, gemma=True, keys=None, values=None, impl=0):
    """Head-norm-rope of q and k, then kv-append (src/jit/schedule/lowering.rs:549-592).

    q [rows][q_row], k/v [rows][kv_heads*head_dim], norms [head_dim], tables
    [positions][rotary/2], caches [kv_heads][capacity][head_dim] (bf16 bits).
    Returns (q, k, keys, values) as new arrays; the inputs are not modified."""
    q = np.ascontiguousarray(q, dtype=np.uint16).copy()
    k = np.ascontiguousarray(k, dtype=np.uint16).copy()
    v = np.ascontiguousarray(v, dtype=np.uint16)
    rows = q.shape[0]
    if keys is not None:
        keys = np.ascontiguousarray(keys, dtype=np.uint16).copy()
        values = np.ascontiguousarray(values, dtype=np.uint16).copy()
        kv_stride = keys.shape[1] * keys.shape[2]
        kp, vp = _p(keys, _u16p), _p(values, _u16p)
    else:
        kv_stride, kp, vp = 0, None, None
    qn = np.ascontiguousarray(q_norm, dtype=np.uint16)
    kn = np.ascontiguousarray(k_norm, dtype=np.uint16)
    ct = np.ascontiguousarray(cos, dtype=np.uint16)
    st = np.ascontiguousarray(sin, dtype=np.uint16)
    rc = lib().orc_attn_front(_p(q, _u16p), q.shape[1], heads, _p(k, _u16p), _p(v, _u16p),
                              k.shape[1], kv_heads, head_dim, _p(qn, _u16p), _p(kn, _u16p),
                              _p(ct, _u16p), _p(st, _u16p), rotary, eps, int(gemma), kp, vp,
                              kv_stride, rows, past, impl)
    if rc != 0:
        raise RuntimeError(f"orc_attn_front refused (impl={impl})")
    return q, k, keys, values


def l2norm(x, eps=1e-6):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().orc_l2norm(_p(x, _f32p), x.size, ctypes.c_float(eps))
    return x


def gdn_layer(qkv, state, beta, decay, *, nk, nv, hkd, hvd, l2=True, eps=1e-6, fma=0,
              threads=0):
    """delta-l2-gates (L2 part) + delta-causal-recurrence over all rows.

    qkv [rows, 2*nk*hkd + nv*hvd] f32 (copied; returned normalised),
    state [nv, hkd, hvd] f32 (copied; returned updated), beta/decay [rows, nv].
    Returns (out [rows, nv*hvd] f32, state, qkv_normalised)."""
    qkv = np.array(qkv, dtype=np.float32, copy=True, order="C")
    state = np.array(state, dtype=np.float32, copy=True, order="C")
    beta = np.ascontiguousarray(beta, dtype=np.float32)
    decay = np.ascontiguousarray(decay, dtype=np.float32)
    rows = qkv.shape[0]
    out = np.zeros((rows, nv * hvd), dtype=np.float32)
    rc = lib().orc_gdn_layer(_p(qkv, _f32p), _p(state, _f32p), _p(out, _f32p), _p(beta, _f32p),
                             _p(decay, _f32p), rows, nk, nv, hkd, hvd, int(l2),
                             ctypes.c_float(eps), fma, threads)
    if rc != 0:
        raise RuntimeError(f"orc_gdn_layer rc={rc}")
    return out, state, qkv


# ------------------------------------------------------ DeltaNet front end

def _f32_array(fn, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    getattr(lib(), fn)(_p(x, _f32p), _p(y, _f32p), x.size)
    return y


def expf_arm(x):
    """The reference's scalar exp (Arm optimized-routines expf, FMA form)."""
    return _f32_array("orc_expf_arm_array", x)


def logf_arm(x):
    """The reference's scalar log (Arm optimized-routines logf, FMA form)."""
    return _f32_array("orc_logf_arm_array", x)


def expf_libm(x):
    return _f32_array("orc_expf_libm_array", x)


def logf_libm(x):
    return _f32_array("orc_logf_libm_array", x)


def mathf_sweep(stride, which):
    """Bit patterns at `stride` through the restatement and glibc (0 exp, 1 log):
    the count of differing results."""
    return int(lib().orc_mathf_sweep(stride, which))


def mathf_tables():
    """(exp table [32] u64, log table [16][2] u64) of the restatement."""
    e = np.empty(32, dtype=np.uint64)
    g = np.empty(32, dtype=np.uint64)
    lib().orc_mathf_tables(e.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                           g.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)))
    return e, g.reshape(16, 2)


def gdn_conv(qkv, state, weight, impl=0):
    """delta-causal-convolution: qkv [rows, conv] f32, state [conv, ck] f32,
    weight [conv, ck] bf16 bits.  Returns (y, new_state) as new arrays."""
    y = np.array(qkv, dtype=np.float32, copy=True, order="C")
    st = np.array(state, dtype=np.float32, copy=True, order="C")
    w = np.ascontiguousarray(weight, dtype=np.uint16)
    rows, conv = y.shape
    rc = lib().orc_gdn_conv(_p(y, _f32p), rows, conv, _p(w, _u16p), _p(st, _f32p), st.shape[1],
                            impl)
    if rc != 0:
        raise RuntimeError(f"orc_gdn_conv rc={rc} (impl={impl})")
    return y, st


def gdn_gates(ab, dt_bias, a_log):
    """beta, decay [rows, nv] from ab [rows, 2*nv] f32, dt_bias [nv] bf16 bits,
    a_log [nv] f32."""
    ab = np.ascontiguousarray(ab, dtype=np.float32)
    rows, nv = ab.shape[0], ab.shape[1] // 2
    db = np.ascontiguousarray(dt_bias, dtype=np.uint16)
    al = np.ascontiguousarray(a_log, dtype=np.float32)
    beta = np.empty((rows, nv), dtype=np.float32)
    decay = np.empty((rows, nv), dtype=np.float32)
    lib().orc_gdn_gates(_p(ab, _f32p), _p(db, _u16p), _p(al, _f32p), _p(beta, _f32p),
                        _p(decay, _f32p), rows, nv)
    return beta, decay


def gdn_gated_norm(x, z, weight, eps=1e-6, impl=0):
    """delta-gated-norm over rows of width weight.size: x, z [..., dim] f32.
    Returns (y f32, y bf16 bits)."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    zz = np.ascontiguousarray(z, dtype=np.float32)
    w = np.ascontiguousarray(weight, dtype=np.uint16)
    dim = w.size
    ob = np.empty(y.shape, dtype=np.uint16)
    rc = lib().orc_gdn_gated_norm(_p(y, _f32p), _p(zz, _f32p), _p(w, _u16p), _p(ob, _u16p),
                                  y.size // dim, dim, ctypes.c_float(eps), impl)
    if rc != 0:
        raise RuntimeError(f"orc_gdn_gated_norm rc={rc} (impl={impl})")
    return y, ob
