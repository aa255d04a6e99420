"""The prefill epilogue's fast arithmetic over its whole input domain.

hb_attn_prefill rounds O / l to bf16 and applies the output gate with a fast
path (hardware conversions, SFU reciprocal plus one Newton step) that hands
rare column pairs to the exact per-element steps.  Random parity inputs
almost never reach those cases, so the library's self-test runs the same
device code over every (a, g) pair of bf16 values and every f32 O / l and
counts results that differ from the exact steps: there must be none."""
import ctypes

import pytest

import herbert_b200 as hb

pytestmark = pytest.mark.gpu


def test_prefill_epilogue_fast_path_is_exact(cuda_device):
    out = (ctypes.c_uint64 * 8)()
    rc = hb.lib().hb_selftest_prefill_epilogue(out, None)
    assert rc == hb.HB_OK, hb.last_error()
    gate_bad, gate_slow, gate_first, gate_bits = out[0], out[1], out[2], out[3]
    plain_bad, plain_slow, plain_first, plain_bits = out[4], out[5], out[6], out[7]
    assert gate_bad == 0, (f"{gate_bad} gated results differ; first a|g<<16 = "
                           f"{gate_first - 1:#010x}, got|want<<16 = {gate_bits:#010x}")
    assert plain_bad == 0, (f"{plain_bad} O/l roundings differ; first f32 bits = "
                            f"{plain_first - 1:#010x}, got|want<<16 = {plain_bits:#010x}")
    # the exact steps are the exception even over the whole domain (NaN, zero
    # and tiny operands included): under half of the 2^31 column pairs
    assert gate_slow < (1 << 30) and plain_slow < (1 << 30), (gate_slow, plain_slow)
