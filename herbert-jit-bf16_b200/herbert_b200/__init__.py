"""Python binding of ``libherbert_b200.so`` -- the B200 attention hot path of
the herbert-jit-bf16 Qwen3.5 engine behind the C ABI of
``include/herbert_b200.h``.

The records mirror the reference's call records field for field
(src/jit/execution/abi.rs): ``AttentionSpec`` / ``AttentionCall`` (:136-180),
``KvSpec`` / ``KvCall`` (:57-130), ``DeltaShape`` (``Shape``, :266-307) and
``RecurrenceCall`` (:310-317).  The entry points mirror the node kernels of
``trait KernelSet`` (src/jit/target/mod.rs:194-240): ``attention`` (the
attention tile selector plus the output-gate node), ``kv_append`` and
``delta_recurrence``.  A shape the kernels do not serve raises ``Decline``
(the reference's named refusal, src/jit/ir.rs:177-230) so a caller can fall
back; any other failure raises ``HBError``.

There is no CPU path here: every call runs the CUDA library, and importing
the binding without the built library fails loudly.  torch is used only for
device memory and streams.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int32, c_int64, c_size_t, c_void_p

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libherbert_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(PKG_DIR), "include", "herbert_b200.h")

HB_OK = 0
HB_DECLINE_EMPTY = 1
HB_DECLINE_HEAD_DIM = 2
HB_DECLINE_GEOMETRY = 3
HB_DECLINE_SINK = 4
HB_ERR_ARG = 10
HB_ERR_WORKSPACE = 11
HB_ERR_CUDA = 12
HB_ERR_TIMEOUT = 13
HB_ERR_NCCL = 14


class HBError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{status_name(status)}: {message}")


class Decline(HBError):
    """The kernels refuse this shape; the caller falls back."""


class AttentionSpec(ctypes.Structure):
    _fields_ = [("heads", c_int64), ("gqa", c_int64), ("head_dim", c_int64),
                ("q_row", c_int64), ("q_head", c_int64), ("out_row", c_int64),
                ("gate_offset", c_int64), ("grouped", c_int32), ("sink", c_int32)]


class AttentionCall(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("keys", c_void_p), ("values", c_void_p),
                ("output", c_void_p), ("rows", c_int64), ("past", c_int64),
                ("kv_stride", c_int64), ("capacity", c_int64), ("scale", c_float),
                ("sink", c_float)]


class AttentionHostCall(ctypes.Structure):
    _fields_ = [("dev", AttentionCall), ("q_host", c_void_p), ("keys_host", c_void_p),
                ("values_host", c_void_p), ("out_host", c_void_p), ("block_rows", c_int64)]


class DecodeSeq(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("keys", c_void_p), ("values", c_void_p),
                ("output", c_void_p), ("past", c_int64), ("kv_stride", c_int64)]


class KvSpec(ctypes.Structure):
    _fields_ = [("heads", c_int64), ("head_dim", c_int64), ("stride", c_int64),
                ("capacity", c_int64), ("max_batch", c_int64)]


class KvCall(ctypes.Structure):
    _fields_ = [("keys", c_void_p), ("values", c_void_p), ("input_keys", c_void_p),
                ("input_values", c_void_p), ("rows", c_int64), ("past", c_int64)]


class FrontSpec(ctypes.Structure):
    """hb_front_spec: rotated elements per head, RMSNorm epsilon, Gemma weight form."""
    _fields_ = [("rotary", c_int64), ("eps", c_float), ("gemma", c_int32)]


class FrontCall(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("q_norm", c_void_p),
                ("k_norm", c_void_p), ("cos", c_void_p), ("sin", c_void_p), ("keys", c_void_p),
                ("values", c_void_p), ("rows", c_int64), ("past", c_int64)]


class DeltaShape(ctypes.Structure):
    _fields_ = [("nk", c_int64), ("nv", c_int64), ("hkd", c_int64), ("hvd", c_int64)]


class RecurrenceCall(ctypes.Structure):
    _fields_ = [("state", c_void_p), ("output", c_void_p), ("qkv", c_void_p),
                ("beta", c_void_p), ("decay", c_void_p), ("rows", c_int64),
                ("l2", c_int32), ("eps", c_float)]


class RecurrenceHostCall(ctypes.Structure):
    _fields_ = [("dev", RecurrenceCall), ("qkv_host", c_void_p), ("beta_host", c_void_p),
                ("decay_host", c_void_p), ("output_host", c_void_p), ("block_rows", c_int64)]


class GdnFrontCall(ctypes.Structure):
    """hb_gdn_front_call: conv + SiLU in place over qkv, then the beta/decay gates."""
    _fields_ = [("qkv", c_void_p), ("conv_state", c_void_p), ("conv_weight", c_void_p),
                ("ab", c_void_p), ("dt_bias", c_void_p), ("a_log", c_void_p), ("beta", c_void_p),
                ("decay", c_void_p), ("rows", c_int64), ("ck", c_int64)]


class GdnNormCall(ctypes.Structure):
    """hb_gdn_norm_call: the gated RMS norm of the recurrence output."""
    _fields_ = [("x", c_void_p), ("z", c_void_p), ("weight", c_void_p), ("out", c_void_p),
                ("out_f32", c_void_p), ("rows", c_int64), ("eps", c_float)]


class StateGeometry(ctypes.Structure):
    """hb_state_geometry: where a sequence's state lives on the device."""
    _fields_ = [("kv_offsets", c_void_p), ("n_layers", c_int64), ("kv_heads", c_int64),
                ("kv_reserve", c_int64), ("conv_len", c_int64), ("recurrent_len", c_int64),
                ("logits_len", c_int64)]


class StateBuffers(ctypes.Structure):
    _fields_ = [("kv", c_void_p), ("dn_conv", c_void_p), ("dn_recurrent", c_void_p),
                ("logits", c_void_p)]


HB_LAYER_ATTENTION, HB_LAYER_DELTA = 1, 2


class MountDesc(ctypes.Structure):
    """hb_mount_desc: the model's layers bound to one sequence's state."""
    _fields_ = [("geometry", ctypes.POINTER(StateGeometry)), ("state", ctypes.POINTER(StateBuffers)),
                ("layer_kinds", c_void_p), ("attn", AttentionSpec), ("attn_scale", c_float),
                ("rotary", c_int64), ("cos", c_void_p), ("sin", c_void_p), ("norm_eps", c_float),
                ("gemma", c_int32), ("delta", DeltaShape), ("conv_kernel", c_int64),
                ("conv_stride", c_int64), ("recurrent_stride", c_int64), ("max_rows", c_int64)]


class LayerRoute(ctypes.Structure):
    _fields_ = [("kind", c_int32), ("delta_index", c_int32), ("keys", c_void_p),
                ("values", c_void_p), ("kv_stride", c_int64), ("conv_state", c_void_p),
                ("recurrent_state", c_void_p)]


class MountAttentionCall(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("q_norm", c_void_p),
                ("k_norm", c_void_p), ("out", c_void_p), ("rows", c_int64), ("pos", c_int64)]


class MountDeltaCall(ctypes.Structure):
    _fields_ = [("qkv", c_void_p), ("ab", c_void_p), ("z", c_void_p), ("conv_weight", c_void_p),
                ("dt_bias", c_void_p), ("a_log", c_void_p), ("norm_weight", c_void_p),
                ("out", c_void_p), ("out_f32", c_void_p), ("rows", c_int64)]


class CpSpec(ctypes.Structure):
    """hb_cp_spec: a zig-zag sharded sequence of 2*ranks*chunk positions."""
    _fields_ = [("ranks", c_int32), ("rank", c_int32), ("chunk", c_int64)]


HB_CP_ID_BYTES = 128

_P = ctypes.POINTER
_lib = None

# name -> (restype, argtypes); every function the header declares.
_SIGNATURES = {
    "hb_version": (ctypes.c_int, []),
    "hb_last_error": (ctypes.c_char_p, []),
    "hb_status_name": (ctypes.c_char_p, [ctypes.c_int]),
    "hb_workspace_init": (ctypes.c_int, [c_void_p, c_size_t, c_void_p]),
    "hb_workspace_status": (ctypes.c_int, [c_void_p, c_size_t, c_void_p]),
    "hb_device_status": (ctypes.c_int, [c_void_p]),
    "hb_attn_decode_workspace_bytes": (c_size_t, [_P(AttentionSpec), _P(AttentionCall)]),
    "hb_attn_decode": (ctypes.c_int, [_P(AttentionSpec), _P(AttentionCall), c_void_p, c_size_t,
                                      c_void_p]),
    "hb_attn_decode_noalloc": (ctypes.c_int, [_P(AttentionSpec), _P(AttentionCall), c_void_p]),
    "hb_attn_decode_batch_workspace_bytes": (c_size_t, [_P(AttentionSpec), c_int64, c_int64,
                                                        c_int64]),
    "hb_attn_decode_batch": (ctypes.c_int, [_P(AttentionSpec), c_void_p, c_int64, c_int64,
                                            c_int64, c_void_p, c_size_t, c_void_p]),
    "hb_decode_shard_plan": (ctypes.c_int, [_P(c_int64), c_int64, c_int32, _P(c_int32),
                                            _P(c_int64)]),
    "hb_attn_prefill_workspace_bytes": (c_size_t, [_P(AttentionSpec), _P(AttentionCall)]),
    "hb_attn_prefill": (ctypes.c_int, [_P(AttentionSpec), _P(AttentionCall), c_void_p, c_size_t,
                                       c_void_p]),
    "hb_attn_prefill_host_workspace_bytes": (c_size_t, [_P(AttentionSpec), _P(AttentionHostCall)]),
    "hb_attn_prefill_host": (ctypes.c_int, [_P(AttentionSpec), _P(AttentionHostCall), c_void_p,
                                            c_size_t, c_void_p]),
    "hb_gdn_prefill_host_workspace_bytes": (c_size_t, [_P(DeltaShape), _P(RecurrenceHostCall)]),
    "hb_gdn_prefill_host": (ctypes.c_int, [_P(DeltaShape), _P(RecurrenceHostCall), c_void_p,
                                           c_size_t, c_void_p]),
    "hb_kv_append": (ctypes.c_int, [_P(KvSpec), _P(KvCall), c_void_p]),
    "hb_attn_front": (ctypes.c_int, [_P(AttentionSpec), _P(KvSpec), _P(FrontSpec), _P(FrontCall),
                                     c_void_p]),
    "hb_gdn_decode": (ctypes.c_int, [_P(DeltaShape), _P(RecurrenceCall), c_void_p]),
    "hb_gdn_prefill_workspace_bytes": (c_size_t, [_P(DeltaShape), c_int64]),
    "hb_gdn_prefill": (ctypes.c_int, [_P(DeltaShape), _P(RecurrenceCall), c_void_p, c_size_t,
                                      c_void_p]),
    "hb_gdn_front": (ctypes.c_int, [_P(DeltaShape), _P(GdnFrontCall), c_void_p, c_size_t,
                                    c_void_p]),
    "hb_gdn_gated_norm": (ctypes.c_int, [_P(DeltaShape), _P(GdnNormCall), c_void_p]),
    "hb_snapshot_bytes": (c_size_t, [_P(StateGeometry), c_int64]),
    "hb_snapshot_take": (ctypes.c_int, [_P(StateGeometry), _P(StateBuffers), c_int64, c_int64,
                                        c_void_p, c_size_t, c_void_p]),
    "hb_snapshot_restore": (ctypes.c_int, [_P(StateGeometry), _P(StateBuffers), c_void_p,
                                           c_size_t, c_int64, c_void_p]),
    "hb_snapshot_info": (ctypes.c_int, [c_void_p, c_size_t, _P(c_int64), _P(c_int32)]),
    "hb_mount_route": (ctypes.c_int, [_P(MountDesc), c_int64, _P(LayerRoute)]),
    "hb_mount_create": (ctypes.c_int, [_P(MountDesc), _P(c_void_p)]),
    "hb_mount_destroy": (None, [c_void_p]),
    "hb_mount_status": (ctypes.c_int, [c_void_p, c_void_p]),
    "hb_mount_needs_reset": (ctypes.c_int, [c_void_p]),
    "hb_mount_reset": (ctypes.c_int, [c_void_p, c_void_p]),
    "hb_mount_attention": (ctypes.c_int, [c_void_p, c_int64, _P(MountAttentionCall), c_void_p]),
    "hb_mount_delta": (ctypes.c_int, [c_void_p, c_int64, _P(MountDeltaCall), c_void_p]),
    "hb_cp_hop_source": (c_int32, [_P(CpSpec), c_int32]),
    "hb_cp_row_position": (c_int64, [_P(CpSpec), c_int32, c_int64]),
    "hb_attn_prefill_cp_workspace_bytes": (c_size_t, [_P(AttentionSpec), _P(CpSpec)]),
    "hb_attn_prefill_cp_hop": (ctypes.c_int, [_P(AttentionSpec), _P(CpSpec), _P(AttentionCall),
                                              c_int32, c_void_p, c_size_t, c_void_p]),
    "hb_attn_prefill_cp_finish": (ctypes.c_int, [_P(AttentionSpec), _P(CpSpec),
                                                 _P(AttentionCall), c_void_p, c_size_t,
                                                 c_void_p]),
    "hb_cp_comm_unique_id": (ctypes.c_int, [c_void_p]),
    "hb_cp_comm_init": (ctypes.c_int, [_P(c_void_p), c_int32, c_void_p, c_int32]),
    "hb_cp_comm_destroy": (ctypes.c_int, [c_void_p]),
    "hb_cp_wait": (ctypes.c_int, [c_void_p, c_void_p, ctypes.c_double]),
    "hb_attn_prefill_cp": (ctypes.c_int, [_P(AttentionSpec), _P(CpSpec), _P(AttentionCall),
                                          c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
}


def lib():
    """Load the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libherbert_b200.so is missing at {LIB_PATH}: run __graft_entry__.build() "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


SELFTEST_LIB_PATH = os.path.join(PKG_DIR, "libherbert_b200_selftest.so")
_selftest = None

# the test-only companion library (csrc/selftest/hb_selftest.h)
_SELFTEST_SIGNATURES = {
    "hbt_last_error": (ctypes.c_char_p, []),
    "hbt_prefill_epilogue": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint64), c_void_p]),
    "hbt_wait_timeout": (ctypes.c_int, [c_void_p, c_size_t, ctypes.c_longlong, ctypes.c_int,
                                        c_void_p]),
}


def selftest_lib():
    """Load the test-only library of device self-tests (never used by the
    product path)."""
    global _selftest
    if _selftest is None:
        if not os.path.exists(SELFTEST_LIB_PATH):
            raise ImportError(f"{SELFTEST_LIB_PATH} is missing: run __graft_entry__.build()")
        L = ctypes.CDLL(SELFTEST_LIB_PATH)
        for name, (res, args) in _SELFTEST_SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _selftest = L
    return _selftest


def status_name(status: int) -> str:
    return lib().hb_status_name(status).decode()


def last_error() -> str:
    return lib().hb_last_error().decode()


def check(status: int) -> None:
    if status == HB_OK:
        return
    msg = last_error()
    if status < HB_ERR_ARG:
        raise Decline(status, msg)
    raise HBError(status, msg)


def version() -> tuple:
    v = lib().hb_version()
    return (v >> 16, v & 0xFFFF)


# ----------------------------------------------------------- torch plumbing

def _stream(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return c_void_p(stream.cuda_stream)


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


class Workspace:
    """Caller-owned device scratch for one or more calls (zeroed once)."""

    def __init__(self, nbytes: int, device=None, stream=None):
        import torch
        self.nbytes = max(256, int(nbytes))
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device or "cuda")
        check(lib().hb_workspace_init(c_void_p(self.ptr), self.nbytes, _stream(stream)))

    @property
    def ptr(self) -> int:
        return int(self.buf.data_ptr())

    def ensure(self, nbytes: int, stream=None) -> "Workspace":
        if nbytes > self.nbytes:
            self.__init__(nbytes, self.buf.device, stream)
        return self

    def status(self, stream=None) -> None:
        check(lib().hb_workspace_status(c_void_p(self.ptr), self.nbytes, _stream(stream)))


def attention_spec(heads=16, gqa=4, head_dim=256, gated=True, q_row=None, out_row=None,
                   q_head=None) -> AttentionSpec:
    """The Qwen3.5 layer geometry: q rows [Q | gate] (src/jit/schedule.rs:172-186)."""
    qd = heads * head_dim
    return AttentionSpec(heads=heads, gqa=gqa, head_dim=head_dim,
                         q_row=q_row if q_row is not None else (2 * qd if gated else qd),
                         q_head=q_head if q_head is not None else head_dim,
                         out_row=out_row if out_row is not None else qd,
                         gate_offset=qd if gated else -1, grouped=0, sink=0)


def attention(spec: AttentionSpec, q, keys, values, out, *, rows: int, past: int,
              kv_stride: int, capacity: int = 0, scale: float | None = None,
              regime: str = "decode", workspace: Workspace | None = None, stream=None):
    """The attention node + output-gate node over device tensors (bf16 or int16/uint16 views).

    regime "decode" runs the split-KV kernel, "prefill" the causal flash
    attention kernel.  Returns the workspace used (reuse it across calls)."""
    call = AttentionCall(q=_ptr(q), keys=_ptr(keys), values=_ptr(values), output=_ptr(out),
                         rows=rows, past=past, kv_stride=kv_stride, capacity=capacity,
                         scale=(1.0 / spec.head_dim ** 0.5) if scale is None else scale, sink=0.0)
    L = lib()
    if regime == "decode":
        need, run = L.hb_attn_decode_workspace_bytes, L.hb_attn_decode
    elif regime == "prefill":
        need, run = L.hb_attn_prefill_workspace_bytes, L.hb_attn_prefill
    else:
        raise ValueError(regime)
    nbytes = need(ctypes.byref(spec), ctypes.byref(call))
    if nbytes == 0:
        # the size query refuses what the call refuses: let the call name it
        check(run(ctypes.byref(spec), ctypes.byref(call), None, 0, _stream(stream)))
    if workspace is None:
        workspace = Workspace(nbytes, q.device, stream)
    else:
        workspace.ensure(nbytes, stream)
    check(run(ctypes.byref(spec), ctypes.byref(call), c_void_p(workspace.ptr), workspace.nbytes,
              _stream(stream)))
    return workspace


def prefill_host(spec: AttentionSpec, q_host, keys_host, values_host, out_host, q, keys, values,
                 out, *, rows: int, past: int, kv_stride: int, capacity: int = 0,
                 scale: float | None = None, block_rows: int = 0,
                 workspace: Workspace | None = None, stream=None) -> Workspace:
    """hb_attn_prefill_host: prefill whose q rows, new K/V positions and output
    are host tensors (pin them for asynchronous copies) mirroring the device
    tensors q, keys, values, out; copies and computation overlap block by
    block.  Returns the workspace used."""
    dev = AttentionCall(q=_ptr(q), keys=_ptr(keys), values=_ptr(values), output=_ptr(out),
                        rows=rows, past=past, kv_stride=kv_stride, capacity=capacity,
                        scale=(1.0 / spec.head_dim ** 0.5) if scale is None else scale, sink=0.0)
    call = AttentionHostCall(dev=dev, q_host=q_host.data_ptr(), keys_host=keys_host.data_ptr(),
                             values_host=values_host.data_ptr(), out_host=out_host.data_ptr(),
                             block_rows=block_rows)
    L = lib()
    nbytes = L.hb_attn_prefill_host_workspace_bytes(ctypes.byref(spec), ctypes.byref(call))
    if nbytes == 0:
        check(L.hb_attn_prefill_host(ctypes.byref(spec), ctypes.byref(call), None, 0,
                                     _stream(stream)))
    if workspace is None:
        workspace = Workspace(nbytes, q.device, stream)
    else:
        workspace.ensure(nbytes, stream)
    check(L.hb_attn_prefill_host(ctypes.byref(spec), ctypes.byref(call), c_void_p(workspace.ptr),
                                 workspace.nbytes, _stream(stream)))
    return workspace


def decode_batch(spec: AttentionSpec, seqs_table, nseq: int, max_past: int, sum_past: int = 0,
                 workspace: Workspace | None = None, stream=None, device=None):
    """Batched decode over a device table of DecodeSeq records (uint8 tensor)."""
    L = lib()
    nbytes = L.hb_attn_decode_batch_workspace_bytes(ctypes.byref(spec), nseq, max_past, sum_past)
    if workspace is None:
        workspace = Workspace(nbytes, device or seqs_table.device, stream)
    else:
        workspace.ensure(nbytes, stream)
    check(L.hb_attn_decode_batch(ctypes.byref(spec), c_void_p(_ptr(seqs_table)), nseq, max_past,
                                 sum_past, c_void_p(workspace.ptr), workspace.nbytes,
                                 _stream(stream)))
    return workspace


def seq_table(entries, device="cuda"):
    """Pack DecodeSeq records into a device uint8 tensor."""
    import torch
    arr = (DecodeSeq * len(entries))(*entries)
    raw = bytes(arr)
    host = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
    return host.to(device)


def shard_plan(costs, parts: int):
    """hb_decode_shard_plan: the GPU of each sequence (longest first, each to
    the least-loaded GPU) and each GPU's total cost.  Returns (part, load)."""
    n = len(costs)
    c = (c_int64 * n)(*[int(x) for x in costs])
    part = (c_int32 * n)()
    load = (c_int64 * parts)()
    check(lib().hb_decode_shard_plan(c, n, parts, part, load))
    return list(part), list(load)


def shard_of(costs, parts: int, rank: int):
    """Indices of the sequences GPU ``rank`` serves, in input order."""
    part, _ = shard_plan(costs, parts)
    return [i for i, g in enumerate(part) if g == rank]


def kv_append(spec: KvSpec, keys, values, input_keys, input_values, *, rows: int, past: int,
              stream=None) -> None:
    call = KvCall(keys=_ptr(keys), values=_ptr(values), input_keys=_ptr(input_keys),
                  input_values=_ptr(input_values), rows=rows, past=past)
    check(lib().hb_kv_append(ctypes.byref(spec), ctypes.byref(call), _stream(stream)))


def attn_front(spec: AttentionSpec, kv: KvSpec, q, k, v, q_norm, k_norm, cos, sin, *,
               rows: int, past: int, rotary: int, eps: float = 1e-6, gemma: bool = True,
               keys=None, values=None, stream=None) -> None:
    """Head-norm-rope of q and k in place, then k and v into the cache (keys/values None:
    no append).  Device tensors of bf16 bits."""
    front = FrontSpec(rotary=rotary, eps=eps, gemma=int(gemma))
    call = FrontCall(q=_ptr(q), k=_ptr(k), v=_ptr(v), q_norm=_ptr(q_norm), k_norm=_ptr(k_norm),
                     cos=_ptr(cos), sin=_ptr(sin), keys=_ptr(keys), values=_ptr(values),
                     rows=rows, past=past)
    check(lib().hb_attn_front(ctypes.byref(spec), ctypes.byref(kv), ctypes.byref(front),
                              ctypes.byref(call), _stream(stream)))


def delta_recurrence(shape: DeltaShape, state, out, qkv, beta, decay, *, rows: int,
                     l2: bool = True, eps: float = 1e-6, regime: str = "decode",
                     workspace: Workspace | None = None, stream=None):
    """The delta-l2-gates L2 step + delta-causal-recurrence node (f32 tensors).

    regime "decode": positions in order with the reference's rounding;
    "prefill": the chunked kernel."""
    call = RecurrenceCall(state=_ptr(state), output=_ptr(out), qkv=_ptr(qkv), beta=_ptr(beta),
                          decay=_ptr(decay), rows=rows, l2=int(l2), eps=eps)
    L = lib()
    if regime == "decode":
        check(L.hb_gdn_decode(ctypes.byref(shape), ctypes.byref(call), _stream(stream)))
        return workspace
    nbytes = L.hb_gdn_prefill_workspace_bytes(ctypes.byref(shape), rows)
    if workspace is None:
        workspace = Workspace(nbytes, state.device, stream)
    else:
        workspace.ensure(nbytes, stream)
    check(L.hb_gdn_prefill(ctypes.byref(shape), ctypes.byref(call), c_void_p(workspace.ptr),
                           workspace.nbytes, _stream(stream)))
    return workspace


def delta_prefill_host(shape: DeltaShape, state, out, qkv, beta, decay, qkv_host, beta_host,
                       decay_host, out_host, *, rows: int, l2: bool = True, eps: float = 1e-6,
                       block_rows: int = 0, workspace: Workspace | None = None,
                       stream=None) -> Workspace:
    """hb_gdn_prefill_host: the chunked prefill of rows whose qkv, beta,
    decay and output are host tensors (pin them for asynchronous copies)
    mirroring the device tensors; copies and computation overlap block by
    block, the state carried in place.  Returns the workspace used."""
    dev = RecurrenceCall(state=_ptr(state), output=_ptr(out), qkv=_ptr(qkv), beta=_ptr(beta),
                         decay=_ptr(decay), rows=rows, l2=int(l2), eps=eps)
    call = RecurrenceHostCall(dev=dev, qkv_host=qkv_host.data_ptr(), beta_host=beta_host.data_ptr(),
                              decay_host=decay_host.data_ptr(), output_host=out_host.data_ptr(),
                              block_rows=block_rows)
    L = lib()
    nbytes = L.hb_gdn_prefill_host_workspace_bytes(ctypes.byref(shape), ctypes.byref(call))
    if nbytes == 0:
        check(L.hb_gdn_prefill_host(ctypes.byref(shape), ctypes.byref(call), None, 0,
                                    _stream(stream)))
    if workspace is None:
        workspace = Workspace(nbytes, state.device, stream)
    else:
        workspace.ensure(nbytes, stream)
    check(L.hb_gdn_prefill_host(ctypes.byref(shape), ctypes.byref(call), c_void_p(workspace.ptr),
                                workspace.nbytes, _stream(stream)))
    return workspace


def delta_front(shape: DeltaShape, qkv, conv_state, conv_weight, ab, dt_bias, a_log, beta,
                decay, *, rows: int, ck: int = 4, workspace: Workspace | None = None,
                stream=None) -> Workspace:
    """The delta-causal-convolution node (conv + SiLU in place over qkv, conv_state
    updated) and the gate part of delta-l2-gates (beta, decay) in one launch.
    f32 tensors except conv_weight and dt_bias (bf16 bits)."""
    if workspace is None:
        workspace = Workspace(256, qkv.device, stream)
    call = GdnFrontCall(qkv=_ptr(qkv), conv_state=_ptr(conv_state), conv_weight=_ptr(conv_weight),
                        ab=_ptr(ab), dt_bias=_ptr(dt_bias), a_log=_ptr(a_log), beta=_ptr(beta),
                        decay=_ptr(decay), rows=rows, ck=ck)
    check(lib().hb_gdn_front(ctypes.byref(shape), ctypes.byref(call), c_void_p(workspace.ptr),
                             workspace.nbytes, _stream(stream)))
    return workspace


def delta_gated_norm(shape: DeltaShape, x, z, weight, out, *, rows: int, eps: float = 1e-6,
                     out_f32=None, stream=None) -> None:
    """The delta-gated-norm node: out (bf16 bits) = ((x inv_rms) w) silu(z) per V head;
    out_f32 (optional, may be x) receives the f32 values."""
    call = GdnNormCall(x=_ptr(x), z=_ptr(z), weight=_ptr(weight), out=_ptr(out),
                       out_f32=_ptr(out_f32), rows=rows, eps=eps)
    check(lib().hb_gdn_gated_norm(ctypes.byref(shape), ctypes.byref(call), _stream(stream)))


# --------------------------------------------------------------- snapshot

class Geometry:
    """hb_state_geometry plus the kv_offsets array it points to (kept alive)."""

    def __init__(self, kv_offsets, kv_heads, kv_reserve, conv_len=0, recurrent_len=0,
                 logits_len=0):
        import numpy as np
        self.offsets = np.ascontiguousarray(kv_offsets, dtype=np.int64)
        self.c = StateGeometry(kv_offsets=self.offsets.ctypes.data, n_layers=self.offsets.size - 1,
                               kv_heads=kv_heads, kv_reserve=kv_reserve, conv_len=conv_len,
                               recurrent_len=recurrent_len, logits_len=logits_len)


def _host_ptr(image):
    """Address and byte size of a host image: a numpy array or a CPU torch tensor."""
    if hasattr(image, "data_ptr"):
        return int(image.data_ptr()), int(image.numel() * image.element_size())
    return int(image.ctypes.data), int(image.nbytes)


def snapshot_bytes(geo: Geometry, max_positions: int) -> int:
    return int(lib().hb_snapshot_bytes(ctypes.byref(geo.c), max_positions))


def snapshot_take(geo: Geometry, kv, dn_conv, dn_recurrent, logits, image, *, pos: int,
                  max_positions: int, stream=None) -> None:
    """snapshot_take + write_to: the state at `pos` into the host image (stream-ordered;
    synchronise before reading the image)."""
    bufs = StateBuffers(kv=_ptr(kv), dn_conv=_ptr(dn_conv), dn_recurrent=_ptr(dn_recurrent),
                        logits=_ptr(logits))
    ptr, nbytes = _host_ptr(image)
    check(lib().hb_snapshot_take(ctypes.byref(geo.c), ctypes.byref(bufs), pos, max_positions,
                                 c_void_p(ptr), nbytes, _stream(stream)))


def snapshot_restore(geo: Geometry, kv, dn_conv, dn_recurrent, logits, image, *, p: int,
                     stream=None) -> None:
    """Instantaneous::read + restore_from: the image's state truncated to `p` positions."""
    bufs = StateBuffers(kv=_ptr(kv), dn_conv=_ptr(dn_conv), dn_recurrent=_ptr(dn_recurrent),
                        logits=_ptr(logits))
    ptr, nbytes = _host_ptr(image)
    check(lib().hb_snapshot_restore(ctypes.byref(geo.c), ctypes.byref(bufs), c_void_p(ptr),
                                    nbytes, p, _stream(stream)))


def snapshot_info(image) -> tuple:
    """(pos, restorable_below) of an image."""
    ptr, nbytes = _host_ptr(image)
    pos, below = c_int64(0), c_int32(0)
    check(lib().hb_snapshot_info(c_void_p(ptr), nbytes, ctypes.byref(pos), ctypes.byref(below)))
    return int(pos.value), bool(below.value)


# ------------------------------------------------------------------ mount

def mount_desc(geo: Geometry, kinds, *, kv=None, dn_conv=None, dn_recurrent=None, logits=None,
               attn: AttentionSpec | None = None, attn_scale=0.0625, rotary=64, cos=None,
               sin=None, norm_eps=1e-6, gemma=True, delta: DeltaShape | None = None,
               conv_kernel=4, conv_stride=0, recurrent_stride=0, max_rows=1):
    """An hb_mount_desc and the objects it points to (returned together so that
    they stay alive).  Buffers are device tensors or raw addresses."""
    import numpy as np
    addr = lambda t: t if isinstance(t, int) else _ptr(t)  # noqa: E731
    k = np.ascontiguousarray(kinds, dtype=np.int32)
    bufs = StateBuffers(kv=addr(kv), dn_conv=addr(dn_conv), dn_recurrent=addr(dn_recurrent),
                        logits=addr(logits))
    d = MountDesc(geometry=ctypes.pointer(geo.c), state=ctypes.pointer(bufs),
                  layer_kinds=k.ctypes.data, attn=attn or attention_spec(),
                  attn_scale=attn_scale, rotary=rotary, cos=addr(cos), sin=addr(sin),
                  norm_eps=norm_eps, gemma=int(gemma),
                  delta=delta or DeltaShape(nk=16, nv=32, hkd=128, hvd=128),
                  conv_kernel=conv_kernel, conv_stride=conv_stride,
                  recurrent_stride=recurrent_stride, max_rows=max_rows)
    return d, (geo, k, bufs)


def mount_route(desc: MountDesc, layer: int) -> LayerRoute:
    r = LayerRoute()
    check(lib().hb_mount_route(ctypes.byref(desc), layer, ctypes.byref(r)))
    return r


class Mount:
    """hb_mount: the per-layer routing of a pass (owns its workspaces)."""

    def __init__(self, desc: MountDesc, keep=()):
        self._keep = keep
        self.h = c_void_p()
        check(lib().hb_mount_create(ctypes.byref(desc), ctypes.byref(self.h)))

    def close(self):
        if self.h:
            lib().hb_mount_destroy(self.h)
            self.h = c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def status(self, stream=None):
        check(lib().hb_mount_status(self.h, _stream(stream)))

    @property
    def needs_reset(self) -> bool:
        return bool(lib().hb_mount_needs_reset(self.h))

    def reset(self, stream=None):
        """Clear the poison of a failed call, once the caller has restored or
        cleared the state it may have touched."""
        check(lib().hb_mount_reset(self.h, _stream(stream)))

    def attention(self, layer, q, k, v, q_norm, k_norm, out, *, rows, pos, stream=None):
        c = MountAttentionCall(q=_ptr(q), k=_ptr(k), v=_ptr(v), q_norm=_ptr(q_norm),
                               k_norm=_ptr(k_norm), out=_ptr(out), rows=rows, pos=pos)
        check(lib().hb_mount_attention(self.h, layer, ctypes.byref(c), _stream(stream)))

    def delta(self, layer, qkv, ab, z, conv_weight, dt_bias, a_log, norm_weight, out, *, rows,
              out_f32=None, stream=None):
        c = MountDeltaCall(qkv=_ptr(qkv), ab=_ptr(ab), z=_ptr(z), conv_weight=_ptr(conv_weight),
                           dt_bias=_ptr(dt_bias), a_log=_ptr(a_log),
                           norm_weight=_ptr(norm_weight), out=_ptr(out), out_f32=_ptr(out_f32),
                           rows=rows)
        check(lib().hb_mount_delta(self.h, layer, ctypes.byref(c), _stream(stream)))


# ------------------------------------------------- context-parallel prefill

def cp_spec(ranks: int, rank: int, chunk: int) -> CpSpec:
    return CpSpec(ranks=ranks, rank=rank, chunk=chunk)


def cp_hop_source(cp: CpSpec, hop: int) -> int:
    """Rank whose K/V shard ``cp.rank`` computes at ``hop`` (0 = its own)."""
    return lib().hb_cp_hop_source(ctypes.byref(cp), hop)


def cp_row_position(cp: CpSpec, rank: int, row: int) -> int:
    """Absolute position of local row ``row`` of ``rank`` (zig-zag shards)."""
    return lib().hb_cp_row_position(ctypes.byref(cp), rank, row)


def cp_positions(cp: CpSpec, rank: int):
    """The 2*chunk absolute positions of ``rank``'s local rows, in order."""
    c = cp.chunk
    a = rank * c
    b = (2 * cp.ranks - 1 - rank) * c
    return list(range(a, a + c)) + list(range(b, b + c))


def _cp_call(cp, q, keys, values, out, kv_stride, capacity, scale, spec):
    return AttentionCall(q=_ptr(q), keys=_ptr(keys), values=_ptr(values), output=_ptr(out),
                         rows=2 * cp.chunk, past=0, kv_stride=kv_stride, capacity=capacity,
                         scale=(1.0 / spec.head_dim ** 0.5) if scale is None else scale, sink=0.0)


def _cp_workspace(spec, cp, workspace, device, stream):
    nbytes = lib().hb_attn_prefill_cp_workspace_bytes(ctypes.byref(spec), ctypes.byref(cp))
    if nbytes == 0:
        raise Decline(HB_DECLINE_GEOMETRY, "context-parallel prefill refuses this geometry")
    if workspace is None:
        return Workspace(nbytes, device, stream)
    return workspace.ensure(nbytes, stream)


def prefill_cp_hop(spec: AttentionSpec, cp: CpSpec, q, keys, values, out, hop: int, *,
                   kv_stride: int, capacity: int = 0, scale: float | None = None,
                   workspace: Workspace | None = None, stream=None) -> Workspace:
    """One hop of the ring without transport: ``keys``/``values`` hold the shard of
    ``cp_hop_source(cp, hop)``; hop 0 first."""
    call = _cp_call(cp, q, keys, values, out, kv_stride, capacity, scale, spec)
    workspace = _cp_workspace(spec, cp, workspace, q.device, stream)
    check(lib().hb_attn_prefill_cp_hop(ctypes.byref(spec), ctypes.byref(cp), ctypes.byref(call),
                                       hop, c_void_p(workspace.ptr), workspace.nbytes,
                                       _stream(stream)))
    return workspace


def prefill_cp_finish(spec: AttentionSpec, cp: CpSpec, q, keys, values, out, *, kv_stride: int,
                      capacity: int = 0, scale: float | None = None,
                      workspace: Workspace, stream=None) -> None:
    call = _cp_call(cp, q, keys, values, out, kv_stride, capacity, scale, spec)
    check(lib().hb_attn_prefill_cp_finish(ctypes.byref(spec), ctypes.byref(cp),
                                          ctypes.byref(call), c_void_p(workspace.ptr),
                                          workspace.nbytes, _stream(stream)))


class CpComm:
    """The ring's NCCL communicator over the ranks of a torch.distributed group
    (one GPU per rank, current before construction)."""

    def __init__(self, group=None):
        import torch
        import torch.distributed as dist
        self.ranks = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        uid = ctypes.create_string_buffer(HB_CP_ID_BYTES)
        if self.rank == 0:
            check(lib().hb_cp_comm_unique_id(uid))
        obj = [bytes(uid.raw) if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0,
                                   group=group)
        uid = ctypes.create_string_buffer(obj[0], HB_CP_ID_BYTES)
        handle = c_void_p()
        torch.cuda.synchronize()
        check(lib().hb_cp_comm_init(ctypes.byref(handle), self.ranks, uid, self.rank))
        self.handle = handle

    def close(self):
        if self.handle is not None and self.handle.value:
            check(lib().hb_cp_comm_destroy(self.handle))
        self.handle = None

    def wait(self, stream=None, timeout_s: float = 60.0) -> None:
        """Wait for the ring's work on ``stream`` with a deadline; on a timeout
        or a communicator error the communicator is aborted (and released) and
        the error raised."""
        rc = lib().hb_cp_wait(self.handle, _stream(stream), float(timeout_s))
        if rc in (HB_ERR_TIMEOUT, HB_ERR_NCCL, HB_ERR_CUDA):
            self.handle = None  # aborted by the library: never destroy it again
        check(rc)


def prefill_cp(spec: AttentionSpec, cp: CpSpec, q, keys, values, out, *, kv_stride: int,
               capacity: int = 0, scale: float | None = None, comm: CpComm | None = None,
               workspace: Workspace | None = None, stream=None, comm_stream=None) -> Workspace:
    """The whole ring (every rank calls it): P hops with the shards moving by NCCL
    send/recv on ``comm_stream``, then the bf16 gated output of the local rows."""
    call = _cp_call(cp, q, keys, values, out, kv_stride, capacity, scale, spec)
    workspace = _cp_workspace(spec, cp, workspace, q.device, stream)
    handle = comm.handle if comm is not None else None
    cs = c_void_p(comm_stream.cuda_stream) if comm_stream is not None else None
    check(lib().hb_attn_prefill_cp(ctypes.byref(spec), ctypes.byref(cp), ctypes.byref(call),
                                   handle, c_void_p(workspace.ptr), workspace.nbytes,
                                   _stream(stream), cs))
    return workspace
