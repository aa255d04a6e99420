"""The C ABI on CPU: the library loads, exports every function the header
declares, its record layouts match the ctypes mirror, and the host-side
refusals return the reference's named statuses (no kernel launches)."""
import ctypes
import os
import re
import subprocess

import pytest

import herbert_b200 as hb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(hb.HEADER_PATH).read()
    return sorted(set(re.findall(r"HB_API\s+[\w\s\*]+?\b(hb_\w+)\s*\(", text)))


def test_library_exports_every_declared_function():
    names = declared_functions()
    assert len(names) >= 15
    L = hb.lib()
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(hb._SIGNATURES), "binding and header disagree"
    nm = subprocess.run(["nm", "-D", "--defined-only", hb.LIB_PATH], capture_output=True,
                        text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(hb_\w+)", nm))
    assert exported == set(names)


def test_record_layouts_match_the_header(tmp_path):
    src = tmp_path / "layout.c"
    recs = {"hb_attn_spec": hb.AttentionSpec, "hb_attn_call": hb.AttentionCall,
            "hb_decode_seq": hb.DecodeSeq, "hb_kv_spec": hb.KvSpec, "hb_kv_call": hb.KvCall,
            "hb_gdn_shape": hb.DeltaShape, "hb_gdn_call": hb.RecurrenceCall,
            "hb_cp_spec": hb.CpSpec, "hb_front_spec": hb.FrontSpec,
            "hb_front_call": hb.FrontCall, "hb_gdn_front_call": hb.GdnFrontCall,
            "hb_gdn_norm_call": hb.GdnNormCall, "hb_state_geometry": hb.StateGeometry,
            "hb_state_buffers": hb.StateBuffers, "hb_attn_host_call": hb.AttentionHostCall,
            "hb_gdn_host_call": hb.RecurrenceHostCall}
    body = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{hb.HEADER_PATH}"',
            "int main(void){"]
    for c, py in recs.items():
        body.append(f'printf("{c} %zu\\n", sizeof({c}));')
        for f, _ in py._fields_:
            body.append(f'printf("{c}.{f} %zu\\n", offsetof({c}, {f}));')
    body.append("return 0;}")
    src.write_text("\n".join(body))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for c, py in recs.items():
        assert int(out[c]) == ctypes.sizeof(py), c
        for f, _ in py._fields_:
            assert int(out[f"{c}.{f}"]) == getattr(py, f).offset, f"{c}.{f}"


def _call(spec, **kw):
    base = dict(q=16, keys=16, values=16, output=16, rows=1, past=10, kv_stride=11 * 256,
                capacity=0, scale=0.0625, sink=0.0)
    base.update(kw)
    return hb.AttentionCall(**base)


@pytest.mark.parametrize("mutate,status", [
    (dict(sink=1), hb.HB_DECLINE_SINK),
    (dict(heads=0), hb.HB_DECLINE_EMPTY),
    (dict(gqa=3), hb.HB_DECLINE_GEOMETRY),
    (dict(q_head=128), hb.HB_DECLINE_GEOMETRY),
    (dict(out_row=1024), hb.HB_DECLINE_GEOMETRY),
    (dict(head_dim=96, q_head=96, q_row=2 * 16 * 96, out_row=16 * 96, gate_offset=16 * 96),
     hb.HB_DECLINE_HEAD_DIM),
    (dict(gate_offset=8000), hb.HB_DECLINE_GEOMETRY),
])
def test_spec_refusals(mutate, status):
    spec = hb.attention_spec()
    for k, v in mutate.items():
        setattr(spec, k, v)
    rc = hb.lib().hb_attn_decode(ctypes.byref(spec), ctypes.byref(_call(spec)), None, 0, None)
    assert rc == status, hb.last_error()
    assert hb.last_error()


@pytest.mark.parametrize("mutate,status", [
    (dict(rows=0), hb.HB_DECLINE_EMPTY),
    (dict(q=0), hb.HB_ERR_ARG),
    (dict(keys=24), hb.HB_ERR_ARG),
    (dict(past=-1), hb.HB_ERR_ARG),
    (dict(kv_stride=10 * 256), hb.HB_ERR_ARG),
    (dict(capacity=5), hb.HB_ERR_ARG),
])
def test_call_refusals(mutate, status):
    spec = hb.attention_spec()
    rc = hb.lib().hb_attn_decode(ctypes.byref(spec), ctypes.byref(_call(spec, **mutate)), None, 0,
                                 None)
    assert rc == status, hb.last_error()


def test_python_binding_raises_decline():
    spec = hb.attention_spec()
    spec.sink = 1
    with pytest.raises(hb.Decline):
        hb.check(hb.lib().hb_attn_decode(ctypes.byref(spec), ctypes.byref(_call(spec)), None, 0,
                                         None))


def test_kv_and_delta_refusals():
    L = hb.lib()
    ks = hb.KvSpec(heads=4, head_dim=256, stride=100, capacity=8, max_batch=4)
    kc = hb.KvCall(keys=16, values=16, input_keys=16, input_values=16, rows=1, past=0)
    assert L.hb_kv_append(ctypes.byref(ks), ctypes.byref(kc), None) == hb.HB_DECLINE_GEOMETRY
    ks.stride = 8 * 256
    kc.rows = 5
    assert L.hb_kv_append(ctypes.byref(ks), ctypes.byref(kc), None) == hb.HB_ERR_ARG
    sh = hb.DeltaShape(nk=16, nv=30, hkd=128, hvd=128)
    rc = hb.RecurrenceCall(state=16, output=16, qkv=16, beta=16, decay=16, rows=1, l2=1, eps=1e-6)
    assert L.hb_gdn_decode(ctypes.byref(sh), ctypes.byref(rc), None) == hb.HB_DECLINE_GEOMETRY
    sh.nv, sh.hkd = 32, 96
    assert L.hb_gdn_decode(ctypes.byref(sh), ctypes.byref(rc), None) == hb.HB_DECLINE_HEAD_DIM
    sh.hkd = 128
    rc.rows = 0
    assert L.hb_gdn_decode(ctypes.byref(sh), ctypes.byref(rc), None) == hb.HB_DECLINE_EMPTY


def test_host_call_refusals():
    # the host-buffer prefills check their calls before any CUDA call
    L = hb.lib()
    sh = hb.DeltaShape(nk=2, nv=4, hkd=128, hvd=128)
    dev = hb.RecurrenceCall(state=16, output=16, qkv=16, beta=16, decay=16, rows=256, l2=1, eps=1e-6)
    call = hb.RecurrenceHostCall(dev=dev, qkv_host=16, beta_host=16, decay_host=16, output_host=16,
                                 block_rows=100)
    assert L.hb_gdn_prefill_host_workspace_bytes(ctypes.byref(sh), ctypes.byref(call)) == 0
    assert L.hb_gdn_prefill_host(ctypes.byref(sh), ctypes.byref(call), None, 0, None) == hb.HB_ERR_ARG
    assert "block_rows" in hb.last_error()
    call.block_rows = 128
    assert L.hb_gdn_prefill_host_workspace_bytes(ctypes.byref(sh), ctypes.byref(call)) > 0
    assert (L.hb_gdn_prefill_host(ctypes.byref(sh), ctypes.byref(call), None, 0, None)
            == hb.HB_ERR_WORKSPACE)
    call.decay_host = None
    assert L.hb_gdn_prefill_host(ctypes.byref(sh), ctypes.byref(call), None, 0, None) == hb.HB_ERR_ARG
    call.decay_host, call.dev.rows = 16, 0
    assert (L.hb_gdn_prefill_host(ctypes.byref(sh), ctypes.byref(call), None, 0, None)
            == hb.HB_DECLINE_EMPTY)
    spec = hb.attention_spec()
    acall = hb.AttentionHostCall(dev=_call(spec, rows=256, past=0, kv_stride=256 * 256),
                                 q_host=16, keys_host=16, values_host=16, out_host=16,
                                 block_rows=64)
    assert L.hb_attn_prefill_host(ctypes.byref(spec), ctypes.byref(acall), None, 0, None) == hb.HB_ERR_ARG
    assert "block_rows" in hb.last_error()


def test_status_names():
    assert hb.status_name(0) == "HB_OK"
    assert hb.status_name(hb.HB_ERR_TIMEOUT) == "HB_ERR_TIMEOUT"
    assert hb.version() >= (0, 1)


def test_ring_wait_refuses_a_bad_deadline():
    # checked on the host before any CUDA or NCCL call
    for t in (float("nan"), -1.0):
        assert hb.lib().hb_cp_wait(None, None, t) == hb.HB_ERR_ARG
        assert "timeout" in hb.last_error()


def test_selftests_live_outside_the_product_library():
    # the device self-tests are in the test-only companion library
    nm = subprocess.run(["nm", "-D", "--defined-only", hb.LIB_PATH], capture_output=True,
                        text=True, check=True).stdout
    assert "selftest" not in nm and "hbt_" not in nm
    T = hb.selftest_lib()
    for name in hb._SELFTEST_SIGNATURES:
        assert hasattr(T, name), name
