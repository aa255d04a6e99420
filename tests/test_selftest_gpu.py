"""Device code paths that random parity inputs do not reach, run through the
test-only companion library (libherbert_b200_selftest.so).

The prefill epilogue's fast arithmetic over its whole input domain:
hb_attn_prefill rounds O / l to bf16 and applies the output gate with a fast
path (hardware conversions, SFU reciprocal plus one Newton step) that hands
rare column pairs to the exact per-element steps.  Random parity inputs
almost never reach those cases, so the library's self-test runs the same
device code over every (a, g) pair of bf16 values and every f32 O / l and
counts results that differ from the exact steps: there must be none.

A bounded device wait that runs out: every product kernel that waits on an
mbarrier gives up after about a second, records HB_ERR_TIMEOUT in its
workspace's status word and returns, so that a lost copy or peer leaves the
context usable and the caller learns of it from hb_workspace_status.  The
self-test kernel waits on a barrier phase nothing completes, with a short
limit, and nothing is in flight when it returns."""
import ctypes

import pytest

import herbert_b200 as hb

pytestmark = pytest.mark.gpu


def test_prefill_epilogue_fast_path_is_exact(cuda_device):
    out = (ctypes.c_uint64 * 8)()
    rc = hb.selftest_lib().hbt_prefill_epilogue(out, None)
    assert rc == hb.HB_OK, hb.selftest_lib().hbt_last_error()
    gate_bad, gate_slow, gate_first, gate_bits = out[0], out[1], out[2], out[3]
    plain_bad, plain_slow, plain_first, plain_bits = out[4], out[5], out[6], out[7]
    assert gate_bad == 0, (f"{gate_bad} gated results differ; first a|g<<16 = "
                           f"{gate_first - 1:#010x}, got|want<<16 = {gate_bits:#010x}")
    assert plain_bad == 0, (f"{plain_bad} O/l roundings differ; first f32 bits = "
                            f"{plain_first - 1:#010x}, got|want<<16 = {plain_bits:#010x}")
    # the exact steps are the exception even over the whole domain (NaN, zero
    # and tiny operands included): under half of the 2^31 column pairs
    assert gate_slow < (1 << 30) and plain_slow < (1 << 30), (gate_slow, plain_slow)


def test_bounded_wait_that_runs_out_reports_timeout(cuda_device):
    """The wait gives up after its limit (~1 ms here), the status word reads
    HB_ERR_TIMEOUT once and is then clear, and the context still runs the
    product kernels with correct results."""
    import torch
    from harness import assert_sdpa_close, gpu_attention, oracle_attention
    from herbert_b200.inputs import AttentionInputs
    ws = hb.Workspace(256)
    T = hb.selftest_lib()
    # the phase completes: no timeout recorded
    assert T.hbt_wait_timeout(ctypes.c_void_p(ws.ptr), ws.nbytes, 2_000_000, 1, None) == hb.HB_OK
    torch.cuda.synchronize()
    assert hb.lib().hb_workspace_status(ctypes.c_void_p(ws.ptr), ws.nbytes, None) == hb.HB_OK
    # nothing completes the phase: the wait runs out after 2e6 cycles
    assert T.hbt_wait_timeout(ctypes.c_void_p(ws.ptr), ws.nbytes, 2_000_000, 0, None) == hb.HB_OK
    torch.cuda.synchronize()
    rc = hb.lib().hb_workspace_status(ctypes.c_void_p(ws.ptr), ws.nbytes, None)
    assert rc == hb.HB_ERR_TIMEOUT, hb.status_name(rc)
    assert "bounded device wait" in hb.last_error()
    # read and cleared
    assert hb.lib().hb_workspace_status(ctypes.c_void_p(ws.ptr), ws.nbytes, None) == hb.HB_OK
    inp = AttentionInputs(1, 700)
    got, _ = gpu_attention(inp, "decode")
    assert_sdpa_close(got, oracle_attention(inp), "decode after a timed-out wait")
