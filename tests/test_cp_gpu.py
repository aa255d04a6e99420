"""Context-parallel prefill on the GPU through the C ABI.

On one GPU the ring is emulated: every rank's shard sits on the same device
and each rank's hops run in the library's schedule order through
hb_attn_prefill_cp_hop (the transport is the only part left out); the
assembled sequence is checked against the oracle's causal attention with
the SDPA tolerance.  A ring of one (hop + finish) must give the bits of the
single-GPU prefill kernel.  With two or more GPUs the whole ring, NCCL
send/recv included, runs under torchrun (tests/cp_ring_worker.py)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from harness import assert_sdpa_close, bits_of, gpu_attention, oracle_attention, to_dev_bf16
from herbert_b200.inputs import AttentionInputs

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def shard_inputs(inp, cp_positions):
    """q rows, K and V of one rank's zig-zag shard ([kv_head][2*chunk][head_dim])."""
    pos = np.asarray(cp_positions)
    return (inp.q[pos], np.ascontiguousarray(inp.keys[:, pos]),
            np.ascontiguousarray(inp.values[:, pos]))


def emulated_ring(inp, ranks, chunk, workspaces=None):
    """The assembled output of every rank; `workspaces` (one per rank) are
    filled on the first call and reused when given again."""
    import torch
    import herbert_b200 as hb
    spec = hb.attention_spec(inp.heads, inp.gqa, inp.head_dim, inp.gated)
    shards = []
    for r in range(ranks):
        pos = hb.cp_positions(hb.cp_spec(ranks, r, chunk), r)
        q, k, v = shard_inputs(inp, pos)
        shards.append((pos, to_dev_bf16(q), to_dev_bf16(k), to_dev_bf16(v)))
    full = np.zeros((inp.rows, inp.out_row), np.uint16)
    if workspaces is None:
        workspaces = []
    for r in range(ranks):
        cp = hb.cp_spec(ranks, r, chunk)
        pos, q, _, _ = shards[r]
        out = torch.zeros((2 * chunk, inp.out_row), dtype=torch.int16, device="cuda")
        ws = workspaces[r] if r < len(workspaces) else None
        for hop in range(ranks):
            _, _, k, v = shards[hb.cp_hop_source(cp, hop)]
            ws = hb.prefill_cp_hop(spec, cp, q, k, v, out, hop, kv_stride=2 * chunk * inp.head_dim,
                                   scale=inp.scale, workspace=ws)
        hb.prefill_cp_finish(spec, cp, q, shards[r][2], shards[r][3], out,
                             kv_stride=2 * chunk * inp.head_dim, scale=inp.scale, workspace=ws)
        torch.cuda.synchronize()
        ws.status()
        full[np.asarray(pos)] = bits_of(out)
        if r >= len(workspaces):
            workspaces.append(ws)
    return full


@pytest.mark.parametrize("ranks,chunk,gated", [(2, 128, True), (4, 128, True), (2, 256, False),
                                               (3, 128, True), (8, 128, True)])
def test_emulated_ring_matches_oracle(cuda_device, oracle_lib, ranks, chunk, gated):
    inp = AttentionInputs(rows=2 * ranks * chunk, past=0, gated=gated, seed=0x5EED0005 + ranks)
    got = emulated_ring(inp, ranks, chunk)
    ref = oracle_attention(inp)
    assert_sdpa_close(got, ref, f"cp ranks={ranks} chunk={chunk}")


def test_ring_of_one_is_the_prefill_kernel(cuda_device):
    """hop 0 + finish over the whole sequence: the accumulator path (f32 O,
    (m, l), the finishing kernel) gives the single-GPU epilogue's bits."""
    import torch
    import herbert_b200 as hb
    inp = AttentionInputs(rows=1024, past=0, seed=0x5EED0015)
    plain, _ = gpu_attention(inp, regime="prefill")
    spec = hb.attention_spec()
    cp = hb.cp_spec(1, 0, 512)
    q, k, v = to_dev_bf16(inp.q), to_dev_bf16(inp.keys), to_dev_bf16(inp.values)
    out = torch.zeros((1024, inp.out_row), dtype=torch.int16, device="cuda")
    ws = hb.prefill_cp_hop(spec, cp, q, k, v, out, 0, kv_stride=inp.kv_stride, scale=inp.scale)
    hb.prefill_cp_finish(spec, cp, q, k, v, out, kv_stride=inp.kv_stride, scale=inp.scale,
                         workspace=ws)
    torch.cuda.synchronize()
    ws.status()
    assert np.array_equal(bits_of(out), plain)
    out.zero_()
    hb.prefill_cp(spec, cp, q, k, v, out, kv_stride=inp.kv_stride, scale=inp.scale, workspace=ws)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(out), plain)


def test_ring_workspace_reuse(cuda_device, oracle_lib):
    """Two calls on one workspace: hop 0 rewrites the accumulators."""
    inp = AttentionInputs(rows=512, past=0, seed=0x5EED0025)
    wss = []
    a = emulated_ring(inp, 2, 128, wss)
    b = emulated_ring(inp, 2, 128, wss)
    assert len(wss) == 2
    assert np.array_equal(a, b)


def test_nccl_ring_two_gpus(cuda_device):
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("the NCCL ring needs two GPUs")
    world = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", "29531", os.path.join(HERE, "cp_ring_worker.py"), "--chunk", "256"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "cp ring ok" in r.stdout
