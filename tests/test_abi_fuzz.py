"""The C ABI under hostile arguments, on CPU: every entry point given records
whose fields are drawn from zero, negative, huge and typical values, null
and misaligned pointers, NaN scales, must return a status (or a size) and
never crash the host or overflow its own arithmetic.

Device pointers are fake: a record that happens to be valid would launch, so
these run only on hosts without a GPU (there a launch fails with
HB_ERR_CUDA).  Host-side arrays (kv_offsets, layer kinds) are real and sized
as their counts say -- that is the caller's part of the contract.
"""
import ctypes

import numpy as np
import pytest

import herbert_b200 as hb

STATUSES = {hb.HB_OK, hb.HB_DECLINE_EMPTY, hb.HB_DECLINE_HEAD_DIM, hb.HB_DECLINE_GEOMETRY,
            hb.HB_DECLINE_SINK, hb.HB_ERR_ARG, hb.HB_ERR_WORKSPACE, hb.HB_ERR_CUDA,
            hb.HB_ERR_TIMEOUT, hb.HB_ERR_NCCL}
I64 = [0, 1, -1, 2, 3, 4, 16, 31, 64, 100, 128, 255, 256, 257, 1000, 4096, 32768, 2**31 - 1,
       2**31, 2**40, 2**62, -2**63, 2**63 - 1]
PTRS = [0, 256, 1 << 20, (1 << 20) + 2, (1 << 20) + 8, 1 << 40]
FLOATS = [0.0, 1e-6, 0.0625, 1.0, -1.0, float("nan"), float("inf"), 1e30]


@pytest.fixture(autouse=True)
def _cpu_only():
    import torch
    if torch.cuda.is_available():
        pytest.skip("fake-pointer fuzzing runs on hosts without a GPU only")


def _pick(rng, pool):
    return pool[int(rng.integers(0, len(pool)))]


def _fill(rng, struct_type, typical=None):
    """A record of `struct_type`: each field typical (if given) or hostile."""
    rec = struct_type()
    for name, ctype in struct_type._fields_:
        if typical and name in typical and rng.random() < 0.6:
            setattr(rec, name, typical[name])
        elif ctype in (ctypes.c_void_p,):
            setattr(rec, name, _pick(rng, PTRS))
        elif ctype is ctypes.c_float:
            setattr(rec, name, _pick(rng, FLOATS))
        elif ctype in (ctypes.c_int32, ctypes.c_int64):
            setattr(rec, name, _pick(rng, I64))  # ctypes wraps to the field's width
    return rec


ATTN = dict(heads=16, gqa=4, head_dim=256, q_row=8192, q_head=256, out_row=4096,
            gate_offset=4096, grouped=0, sink=0)
CALL = dict(q=256, keys=256, values=256, output=256, rows=1, past=100, kv_stride=256 * 256,
            capacity=256, scale=0.0625, sink=0.0)
SHAPE = dict(nk=16, nv=32, hkd=128, hvd=128)


def _ok(st):
    assert st in STATUSES, st


def test_attention_entry_points():
    L = hb.lib()
    rng = np.random.default_rng(0xF0221)
    ws = ctypes.c_void_p(1 << 20)
    for _ in range(600):
        spec = _fill(rng, hb.AttentionSpec, ATTN)
        call = _fill(rng, hb.AttentionCall, CALL)
        s, c = ctypes.byref(spec), ctypes.byref(call)
        L.hb_attn_decode_workspace_bytes(s, c)
        L.hb_attn_prefill_workspace_bytes(s, c)
        L.hb_attn_decode_batch_workspace_bytes(s, _pick(rng, I64), _pick(rng, I64), _pick(rng, I64))
        nbytes = _pick(rng, [0, 255, 256, 1 << 20, 1 << 40])
        _ok(L.hb_attn_decode(s, c, ws, nbytes, None))
        _ok(L.hb_attn_prefill(s, c, ws, nbytes, None))
        hc = hb.AttentionHostCall(dev=call, q_host=_pick(rng, PTRS), keys_host=_pick(rng, PTRS),
                                  values_host=_pick(rng, PTRS), out_host=_pick(rng, PTRS),
                                  block_rows=_pick(rng, I64 + [0, 128, 1024]))
        L.hb_attn_prefill_host_workspace_bytes(s, ctypes.byref(hc))
        _ok(L.hb_attn_prefill_host(s, ctypes.byref(hc), ws, nbytes, None))
        _ok(L.hb_attn_decode_batch(s, ctypes.c_void_p(_pick(rng, PTRS)), _pick(rng, I64),
                                   _pick(rng, I64), _pick(rng, I64), ws, nbytes, None))
        kv = _fill(rng, hb.KvSpec, dict(heads=4, head_dim=256, stride=256 * 256, capacity=256,
                                        max_batch=16))
        kc = _fill(rng, hb.KvCall, dict(keys=256, values=256, input_keys=256, input_values=256,
                                        rows=2, past=5))
        _ok(L.hb_kv_append(ctypes.byref(kv), ctypes.byref(kc), None))
        front = _fill(rng, hb.FrontSpec, dict(rotary=64, eps=1e-6, gemma=1))
        fc = _fill(rng, hb.FrontCall, dict(q=256, k=256, v=256, q_norm=256, k_norm=256, cos=256,
                                           sin=256, keys=256, values=256, rows=2, past=5))
        _ok(L.hb_attn_front(s, ctypes.byref(kv), ctypes.byref(front), ctypes.byref(fc), None))


def test_context_parallel_host_logic():
    L = hb.lib()
    rng = np.random.default_rng(0xF0222)
    for _ in range(600):
        cp = _fill(rng, hb.CpSpec, dict(ranks=2, rank=0, chunk=1024))
        L.hb_cp_hop_source(ctypes.byref(cp), _pick(rng, [0, 1, -1, 7, 2**31 - 1]))
        L.hb_cp_row_position(ctypes.byref(cp), _pick(rng, [0, 1, -1, 5]), _pick(rng, I64))
        spec = _fill(rng, hb.AttentionSpec, ATTN)
        L.hb_attn_prefill_cp_workspace_bytes(ctypes.byref(spec), ctypes.byref(cp))


def test_deltanet_entry_points():
    L = hb.lib()
    rng = np.random.default_rng(0xF0223)
    ws = ctypes.c_void_p(1 << 20)
    for _ in range(600):
        shape = _fill(rng, hb.DeltaShape, SHAPE)
        sh = ctypes.byref(shape)
        call = _fill(rng, hb.RecurrenceCall, dict(state=256, output=256, qkv=256, beta=256,
                                                  decay=256, rows=3, l2=1, eps=1e-6))
        L.hb_gdn_prefill_workspace_bytes(sh, _pick(rng, I64))
        _ok(L.hb_gdn_decode(sh, ctypes.byref(call), None))
        _ok(L.hb_gdn_prefill(sh, ctypes.byref(call), ws, _pick(rng, [0, 256, 1 << 30]), None))
        hc = hb.RecurrenceHostCall(dev=call, qkv_host=_pick(rng, PTRS), beta_host=_pick(rng, PTRS),
                                   decay_host=_pick(rng, PTRS), output_host=_pick(rng, PTRS),
                                   block_rows=_pick(rng, I64 + [0, 64, 128, 256]))
        L.hb_gdn_prefill_host_workspace_bytes(sh, ctypes.byref(hc))
        _ok(L.hb_gdn_prefill_host(sh, ctypes.byref(hc), ws, _pick(rng, [0, 256, 1 << 30]), None))
        fc = _fill(rng, hb.GdnFrontCall, dict(qkv=256, conv_state=256, conv_weight=256, ab=256,
                                              dt_bias=256, a_log=256, beta=256, decay=256,
                                              rows=3, ck=4))
        _ok(L.hb_gdn_front(sh, ctypes.byref(fc), ws, _pick(rng, [0, 255, 256]), None))
        nc = _fill(rng, hb.GdnNormCall, dict(x=256, z=256, weight=256, out=256, out_f32=0,
                                             rows=3, eps=1e-6))
        _ok(L.hb_gdn_gated_norm(sh, ctypes.byref(nc), None))


def test_state_geometry_entry_points():
    L = hb.lib()
    rng = np.random.default_rng(0xF0224)
    for _ in range(400):
        n = int(rng.integers(0, 6))
        heads, res = _pick(rng, [1, 2, 4, 0, -1, 2**31]), _pick(rng, [1, 8, 40, 0, -5, 2**40])
        steps = [_pick(rng, [0, 2 * 4 * 40 * 64, 7, -8, 2**50]) for _ in range(n)]
        offsets = np.concatenate([[_pick(rng, [0, 0, 0, 3])], np.cumsum(steps)]).astype(np.int64)
        geo = hb.Geometry(offsets, heads, res, _pick(rng, [0, 16, -1, 2**41]),
                          _pick(rng, [0, 64, 2**41]), _pick(rng, [0, 16]))
        L.hb_snapshot_bytes(ctypes.byref(geo.c), _pick(rng, I64))
        kinds = np.array([_pick(rng, [1, 2, 2, 0, 7]) for _ in range(n)], np.int32)
        desc, keep = hb.mount_desc(geo, kinds, kv=256, dn_conv=256, dn_recurrent=256, logits=256,
                                   cos=_pick(rng, PTRS), sin=256,
                                   attn_scale=_pick(rng, FLOATS), rotary=_pick(rng, [64, 48, 0]),
                                   conv_stride=_pick(rng, I64), recurrent_stride=_pick(rng, I64),
                                   max_rows=_pick(rng, I64))
        route = hb.LayerRoute()
        _ok(L.hb_mount_route(ctypes.byref(desc), _pick(rng, [0, 1, -1, n, 2**40]),
                             ctypes.byref(route)))
