"""hb_gdn_prefill_host: the chunked DeltaNet prefill from host buffers, the
copies overlapped with the computation block by block.  Blocks start on
chunk boundaries and each takes the chunked kernels (a remainder below 128
rows joins the block before it), and the kernels carry the state between
chunks only through its bf16 rounding, so the output and the final state
must be bit-identical to one hb_gdn_prefill call over all the rows."""
import numpy as np
import pytest

from herbert_b200.inputs import DeltaInputs
from harness import GDN_REL_FROB, gpu_gdn, oracle_gdn, rel_frob

pytestmark = pytest.mark.gpu

CASES = [
    # rows, block_rows, nk, nv, hkd, hvd, warm state
    (1024, 256, 2, 4, 128, 128, False),   # four full blocks
    (700, 256, 2, 4, 128, 128, True),     # a ragged last block of 188 rows
    (600, 256, 4, 8, 128, 128, True),     # an 88-row remainder joins the block before it
    (2048, 0, 16, 32, 128, 128, True),    # Qwen3.5 geometry, the library's block size
    (640, 128, 4, 8, 64, 64, False),      # hkd 64: every block takes the recurrence in order
]


def _pin(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


@pytest.mark.parametrize("rows,block,nk,nv,hkd,hvd,warm", CASES)
def test_prefill_host_matches_one_device_call(cuda_device, rows, block, nk, nv, hkd, hvd, warm):
    import torch
    import herbert_b200 as hb
    state0 = (np.random.default_rng(rows).standard_normal((nv, hkd, hvd)).astype(np.float32) * 0.1
              if warm else None)
    inp = DeltaInputs(rows, nk=nk, nv=nv, hkd=hkd, hvd=hvd, seed=0x5EED00F0 + rows, state=state0)
    want_out, want_state, _ = gpu_gdn(inp, "prefill")  # one hb_gdn_prefill call on device buffers

    h_qkv, h_beta, h_decay = _pin(inp.qkv), _pin(inp.beta), _pin(inp.decay)
    h_out = torch.zeros((rows, nv * hvd), dtype=torch.float32).pin_memory()
    state = torch.from_numpy(inp.state.copy()).cuda()
    qkv = torch.zeros(h_qkv.shape, dtype=torch.float32, device="cuda")
    beta = torch.zeros(h_beta.shape, dtype=torch.float32, device="cuda")
    decay = torch.zeros(h_decay.shape, dtype=torch.float32, device="cuda")
    out = torch.zeros((rows, nv * hvd), dtype=torch.float32, device="cuda")
    shape = hb.DeltaShape(nk=nk, nv=nv, hkd=hkd, hvd=hvd)
    ws = hb.delta_prefill_host(shape, state, out, qkv, beta, decay, h_qkv, h_beta, h_decay, h_out,
                               rows=rows, block_rows=block)
    torch.cuda.synchronize()
    ws.status()
    got = h_out.numpy()
    assert np.array_equal(got.view(np.uint32), want_out.view(np.uint32)), \
        f"{int((got != want_out).sum())} outputs differ from one call"
    assert np.array_equal(state.cpu().numpy().view(np.uint32), want_state.view(np.uint32))
    # the device copies hold the host rows and the output
    assert np.array_equal(qkv.cpu().numpy().view(np.uint32), inp.qkv.view(np.uint32))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want_out.view(np.uint32))


def test_prefill_host_against_the_oracle(cuda_device):
    import torch
    import herbert_b200 as hb
    rows, nk, nv = 384, 2, 4
    inp = DeltaInputs(rows, nk=nk, nv=nv, seed=0x5EED00E1)
    h_qkv, h_beta, h_decay = _pin(inp.qkv), _pin(inp.beta), _pin(inp.decay)
    h_out = torch.zeros((rows, nv * 128), dtype=torch.float32).pin_memory()
    state = torch.zeros((nv, 128, 128), dtype=torch.float32, device="cuda")
    qkv, beta, decay = (torch.zeros(t.shape, dtype=torch.float32, device="cuda")
                        for t in (h_qkv, h_beta, h_decay))
    out = torch.zeros((rows, nv * 128), dtype=torch.float32, device="cuda")
    shape = hb.DeltaShape(nk=nk, nv=nv, hkd=128, hvd=128)
    hb.delta_prefill_host(shape, state, out, qkv, beta, decay, h_qkv, h_beta, h_decay, h_out,
                          rows=rows, block_rows=128)
    torch.cuda.synchronize()
    ref_out, ref_state = oracle_gdn(inp)
    assert rel_frob(h_out.numpy(), ref_out) <= GDN_REL_FROB
    assert rel_frob(state.cpu().numpy(), ref_state) <= GDN_REL_FROB


def test_prefill_host_refuses_bad_blocks(cuda_device):
    import ctypes
    import torch
    import herbert_b200 as hb
    t = torch.zeros(64, dtype=torch.float32, device="cuda")
    h = torch.zeros(64, dtype=torch.float32).pin_memory()
    shape = hb.DeltaShape(nk=2, nv=4, hkd=128, hvd=128)
    dev = hb.RecurrenceCall(state=t.data_ptr(), output=t.data_ptr(), qkv=t.data_ptr(),
                            beta=t.data_ptr(), decay=t.data_ptr(), rows=256, l2=1, eps=1e-6)
    call = hb.RecurrenceHostCall(dev=dev, qkv_host=h.data_ptr(), beta_host=h.data_ptr(),
                                 decay_host=h.data_ptr(), output_host=h.data_ptr(), block_rows=100)
    assert hb.lib().hb_gdn_prefill_host_workspace_bytes(ctypes.byref(shape), ctypes.byref(call)) == 0
    rc = hb.lib().hb_gdn_prefill_host(ctypes.byref(shape), ctypes.byref(call), None, 0, None)
    assert rc == hb.HB_ERR_ARG and "block_rows" in hb.last_error()
    call.block_rows = 0
    call.beta_host = None
    rc = hb.lib().hb_gdn_prefill_host(ctypes.byref(shape), ctypes.byref(call), None, 0, None)
    assert rc == hb.HB_ERR_ARG and "host" in hb.last_error()
