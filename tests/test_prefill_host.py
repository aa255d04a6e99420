"""hb_attn_prefill_host: prefill from host buffers, copies overlapped with the
computation block by block.  Every row must come out bit-identical to one
hb_attn_prefill call over all the rows (block boundaries are query-tile
boundaries, and a remainder too small for the tensor-core kernel joins the
last block), and the host inputs must land where the device call reads
them (K/V positions past .. past+rows-1 of every KV head)."""
import numpy as np
import pytest

from herbert_b200.inputs import AttentionInputs
from harness import assert_sdpa_close, bits_of, gpu_attention, oracle_attention

pytestmark = pytest.mark.gpu

CASES = [
    # rows, past, block_rows, heads, gqa (KV heads = heads / gqa), gated
    (1536, 0, 512, 16, 4, True),     # three full blocks
    (1000, 256, 384, 16, 4, True),   # past > 0 (positions 0..255 already on the device), ragged last block
    (700, 0, 640, 16, 4, True),      # a 60-row remainder joins the block before it
    (2048, 0, 0, 16, 4, True),       # the library's block size
    (640, 128, 128, 8, 8, False),    # gqa 1, no gate, blocks of one query tile
]


@pytest.mark.parametrize("rows,past,block,heads,gqa,gated", CASES)
def test_prefill_host_matches_one_device_call(cuda_device, rows, past, block, heads, gqa, gated):
    import torch
    import herbert_b200 as hb
    inp = AttentionInputs(rows, past, heads=heads, kv_heads=heads // gqa, head_dim=256,
                          gated=gated, capacity=past + rows, seed=9100 + rows)
    want, _ = gpu_attention(inp, "prefill")  # one hb_attn_prefill call on device buffers

    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).pin_memory()
    h_q, h_k, h_v = pin(inp.q), pin(inp.keys), pin(inp.values)
    h_out = torch.zeros((rows, inp.out_row), dtype=torch.int16).pin_memory()
    q = torch.zeros(h_q.shape, dtype=torch.int16, device="cuda")
    k = torch.zeros(h_k.shape, dtype=torch.int16, device="cuda")
    v = torch.zeros(h_v.shape, dtype=torch.int16, device="cuda")
    # the cached positions 0..past-1 are on the device before the call
    hkv, hd = heads // gqa, 256
    kv_k = k.view(hkv, -1)
    kv_v = v.view(hkv, -1)
    kv_k[:, :past * hd] = h_k.view(hkv, -1)[:, :past * hd].cuda()
    kv_v[:, :past * hd] = h_v.view(hkv, -1)[:, :past * hd].cuda()
    out = torch.zeros((rows, inp.out_row), dtype=torch.int16, device="cuda")
    spec = hb.attention_spec(inp.heads, inp.gqa, inp.head_dim, inp.gated)
    ws = hb.prefill_host(spec, h_q, h_k, h_v, h_out, q, k, v, out, rows=rows, past=past,
                         kv_stride=inp.kv_stride, capacity=inp.capacity, scale=inp.scale,
                         block_rows=block)
    torch.cuda.synchronize()
    ws.status()
    got = h_out.numpy().view(np.uint16)
    assert np.array_equal(got, want), f"{int((got != want).sum())} outputs differ from one call"
    # the device copy of the output and the inputs moved in are the host's
    assert np.array_equal(bits_of(out), want)
    assert np.array_equal(bits_of(kv_k[:, past * hd:(past + rows) * hd]),
                          h_k.view(hkv, -1)[:, past * hd:(past + rows) * hd].numpy().view(np.uint16))


def test_prefill_host_against_the_oracle(cuda_device):
    import torch
    import herbert_b200 as hb
    rows = 384
    inp = AttentionInputs(rows, 0, capacity=rows, seed=9301)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).pin_memory()
    h_q, h_k, h_v = pin(inp.q), pin(inp.keys), pin(inp.values)
    h_out = torch.zeros((rows, inp.out_row), dtype=torch.int16).pin_memory()
    q, k, v = (torch.zeros(t.shape, dtype=torch.int16, device="cuda") for t in (h_q, h_k, h_v))
    out = torch.zeros((rows, inp.out_row), dtype=torch.int16, device="cuda")
    spec = hb.attention_spec(inp.heads, inp.gqa, inp.head_dim, inp.gated)
    hb.prefill_host(spec, h_q, h_k, h_v, h_out, q, k, v, out, rows=rows, past=0,
                    kv_stride=inp.kv_stride, capacity=inp.capacity, scale=inp.scale,
                    block_rows=128)
    torch.cuda.synchronize()
    assert_sdpa_close(h_out.numpy().view(np.uint16), oracle_attention(inp), "prefill_host")


def test_prefill_host_refuses_bad_blocks(cuda_device):
    import ctypes
    import torch
    import herbert_b200 as hb
    inp = AttentionInputs(256, 0, capacity=256, seed=9302)
    t = torch.zeros(16, dtype=torch.int16, device="cuda")
    h = torch.zeros(16, dtype=torch.int16).pin_memory()
    spec = hb.attention_spec()
    dev = hb.AttentionCall(q=t.data_ptr(), keys=t.data_ptr(), values=t.data_ptr(),
                           output=t.data_ptr(), rows=256, past=0, kv_stride=inp.kv_stride,
                           capacity=256, scale=inp.scale, sink=0.0)
    call = hb.AttentionHostCall(dev=dev, q_host=h.data_ptr(), keys_host=h.data_ptr(),
                                values_host=h.data_ptr(), out_host=h.data_ptr(), block_rows=100)
    assert hb.lib().hb_attn_prefill_host_workspace_bytes(ctypes.byref(spec), ctypes.byref(call)) == 0
    rc = hb.lib().hb_attn_prefill_host(ctypes.byref(spec), ctypes.byref(call), None, 0, None)
    assert rc == hb.HB_ERR_ARG and "block_rows" in hb.last_error()
    call.block_rows = 0
    call.q_host = None
    rc = hb.lib().hb_attn_prefill_host(ctypes.byref(spec), ctypes.byref(call), None, 0, None)
    assert rc == hb.HB_ERR_ARG and "host" in hb.last_error()
