"""The allocation-free decode entry point, hb_attn_decode_noalloc.

Some callers cannot give this library device memory: an engine that plans
all its device memory once at start-up and allocates nothing while it runs,
a plugin host that hands its plugins no workspace, or a decode loop that
cannot afford cudaMalloc's implicit synchronisation.  For them the entry
point uses a static device array as its scratch instead of a caller
workspace.  This test calls it through the C ABI twice in a row and checks
both outputs against the workspace entry point, hb_attn_decode, with the
tolerance the other SDPA tests use.  It lives in its own file, named so that
pytest collects it last.
"""
import ctypes

import pytest

import herbert_b200 as hb
from herbert_b200.inputs import AttentionInputs
from harness import assert_sdpa_close, bits_of, gpu_attention, to_dev_bf16

pytestmark = pytest.mark.gpu


def _noalloc(inp, q, k, v, out):
    spec = hb.attention_spec(inp.heads, inp.gqa, inp.head_dim, inp.gated)
    call = hb.AttentionCall(q=q.data_ptr(), keys=k.data_ptr(), values=v.data_ptr(),
                            output=out.data_ptr(), rows=inp.rows, past=inp.past,
                            kv_stride=inp.kv_stride, capacity=inp.capacity, scale=inp.scale,
                            sink=0.0)
    return hb.lib().hb_attn_decode_noalloc(ctypes.byref(spec), ctypes.byref(call), None)


@pytest.mark.parametrize("rows,past", [(1, 2047), (3, 5000)])
def test_noalloc_matches_workspace_entry_point(cuda_device, rows, past):
    import torch
    inp = AttentionInputs(rows, past, capacity=past + rows)
    ref, _ = gpu_attention(inp, "decode")  # hb_attn_decode with a caller workspace
    q, k, v = to_dev_bf16(inp.q), to_dev_bf16(inp.keys), to_dev_bf16(inp.values)
    for _ in range(2):  # two calls in a row share (and must re-clear) the static scratch
        out = torch.zeros((inp.rows, inp.out_row), dtype=torch.int16, device="cuda")
        rc = _noalloc(inp, q, k, v, out)
        assert rc == hb.HB_OK, hb.last_error()
        torch.cuda.synchronize()
        assert_sdpa_close(bits_of(out), ref, f"noalloc rows={rows} past={past}")
    # no bounded wait ran out: the per-device status word these calls report
    # through is clear
    assert hb.lib().hb_device_status(None) == hb.HB_OK, hb.last_error()


def test_noalloc_refuses_calls_beyond_its_scratch(cuda_device):
    # a 4M-position cache needs more split partials than the static array
    # holds: refused before anything is launched (the pointers are never read)
    inp = AttentionInputs.__new__(AttentionInputs)
    inp.heads, inp.gqa, inp.head_dim, inp.gated = 16, 4, 256, True
    inp.rows, inp.past, inp.capacity = 1, (1 << 22) - 1, 0
    inp.kv_stride, inp.scale = (1 << 22) * 256, 0.0625

    class _P:  # aligned stand-in pointers
        def data_ptr(self):
            return 1 << 20

    rc = _noalloc(inp, _P(), _P(), _P(), _P())
    assert rc == hb.HB_ERR_WORKSPACE
    assert "HB_NOALLOC_SCRATCH_BYTES" in hb.last_error()
