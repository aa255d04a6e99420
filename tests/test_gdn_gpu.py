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
    (1, 16, 32, 128, 128, True, True),     # the one-row form, warm state
    (1, 4, 8, 64, 128, False, True),       # the one-row form at hkd 64, no L2 step
    (1, 2, 4, 128, 96, True, True),        # one row at hvd 96: the pipelined form
    (7, 16, 32, 128, 128, True, True),     # a short block: the split form
    (40, 16, 32, 128, 128, True, True),    # a longer block: the pipelined form
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
    import herbert_b200 as hb  # the recurrence reports through the per-device status word
    assert hb.lib().hb_device_status(None) == hb.HB_OK, hb.last_error()


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


@pytest.mark.parametrize("rows,nk,nv,warm", [
    (4096, 16, 32, False),   # the prefill of the benchmark configuration
    (200, 2, 4, True),       # partial last chunk, warm state
    (130, 4, 8, False),
    (1000, 16, 32, True),
])
def test_chunked_prefill_within_tolerance(cuda_device, rows, nk, nv, warm):
    """The chunk-64 tensor-core prefill reassociates the sums: relative
    Frobenius error <= 1e-2 on the outputs and the final state."""
    from harness import GDN_REL_FROB, rel_frob
    state = (np.random.default_rng(11).standard_normal((nv, 128, 128)).astype(np.float32) * 0.1
             if warm else None)
    inp = DeltaInputs(rows, nk=nk, nv=nv, state=state, seed=0x5EED0003 + rows)
    out, st, ws = gpu_gdn(inp, "prefill")
    ws.status()
    ref_out, ref_st = oracle_gdn(inp)
    assert np.all(np.isfinite(out)) and np.all(np.isfinite(st))
    eo, es = rel_frob(out, ref_out), rel_frob(st, ref_st)
    assert eo <= GDN_REL_FROB and es <= GDN_REL_FROB, (eo, es)


def test_chunked_prefill_then_decode(cuda_device):
    """Prefill on the chunked kernels, then exact decode steps from its state."""
    from harness import GDN_REL_FROB, rel_frob
    inp = DeltaInputs(512 + 8, nk=2, nv=4)
    ref_out, ref_st = oracle_gdn(inp)
    pre = DeltaInputs.__new__(DeltaInputs)
    pre.__dict__.update(inp.__dict__)
    pre.rows, pre.qkv, pre.beta, pre.decay = 512, inp.qkv[:512], inp.beta[:512], inp.decay[:512]
    o1, s1, _ = gpu_gdn(pre, "prefill")
    dec = DeltaInputs.__new__(DeltaInputs)
    dec.__dict__.update(inp.__dict__)
    dec.rows, dec.qkv, dec.beta, dec.decay, dec.state = 8, inp.qkv[512:], inp.beta[512:], inp.decay[512:], s1
    o2, s2, _ = gpu_gdn(dec, "decode")
    assert rel_frob(np.concatenate([o1, o2]), ref_out) <= GDN_REL_FROB
    assert rel_frob(s2, ref_st) <= GDN_REL_FROB
