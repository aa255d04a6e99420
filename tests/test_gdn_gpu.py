"""GPU parity of the GatedDeltaNet kernels against the CPU oracle, through
the C ABI.  The recurrent kernel keeps the reference's non-FMA order, so its
outputs and final state must be bit-identical to the oracle's."""
import numpy as np
import pytest

from herbert_b200.inputs import DeltaInputs
from harness import GDN_FIXTURES, gpu_gdn, load_gdn_fixture, oracle_gdn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,nk,nv,hkd,hvd,l2,warm", [
    (1, 16, 32, 128, 128, True, False),    # one decode step at Qwen3.5 geometry
    (7, 16, 32, 128, 128, True, True),
    (4, 2, 4, 128, 64, False, True),
    (3, 4, 4, 64, 96, True, False),
])
def test_recurrent_is_bit_exact(cuda_device, rows, nk, nv, hkd, hvd, l2, warm):
    state = (np.random.default_rng(9).standard_normal((nv, hkd, hvd)).astype(np.float32) * 0.1
             if warm else None)
    inp = DeltaInputs(rows, nk=nk, nv=nv, hkd=hkd, hvd=hvd, state=state)
    out, st, _ = gpu_gdn(inp, "decode", l2=l2)
    ref_out, ref_st = oracle_gdn(inp, l2=l2)
    assert np.array_equal(out.view(np.uint32), ref_out.view(np.uint32))
    assert np.array_equal(st.view(np.uint32), ref_st.view(np.uint32))


@pytest.mark.parametrize("name", GDN_FIXTURES)
def test_golden_fixtures_bit_exact(cuda_device, name):
    inp, out, state = load_gdn_fixture(name)
    o, s, _ = gpu_gdn(inp, "decode")
    assert np.array_equal(o.view(np.uint32), out.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), state.view(np.uint32))


def test_decode_steps_chain(cuda_device):
    """Prefill block then single-row steps equals one long block."""
    inp = DeltaInputs(12, nk=2, nv=4)
    full_out, full_state, _ = gpu_gdn(inp, "decode")
    first = DeltaInputs.__new__(DeltaInputs)
    first.__dict__.update(inp.__dict__)
    first.rows, first.qkv, first.beta, first.decay = 8, inp.qkv[:8], inp.beta[:8], inp.decay[:8]
    o1, s1, _ = gpu_gdn(first, "decode")
    outs = [o1]
    state = s1
    for t in range(8, 12):
        step = DeltaInputs.__new__(DeltaInputs)
        step.__dict__.update(inp.__dict__)
        step.rows, step.qkv = 1, inp.qkv[t:t + 1]
        step.beta, step.decay, step.state = inp.beta[t:t + 1], inp.decay[t:t + 1], state
        o, state, _ = gpu_gdn(step, "decode")
        outs.append(o)
    assert np.array_equal(np.concatenate(outs).view(np.uint32), full_out.view(np.uint32))
    assert np.array_equal(state.view(np.uint32), full_state.view(np.uint32))
