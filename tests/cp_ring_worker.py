"""One rank of the NCCL ring test (launched by tests/test_cp_gpu.py under
torchrun, one GPU per rank): shards a seeded sequence zig-zag, runs
hb_attn_prefill_cp with the K/V shards moving by NCCL send/recv, gathers the
outputs on rank 0 and checks them against the oracle's causal attention
with the SDPA tolerance.  Prints "cp ring ok" on rank 0 when it passes."""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "herbert-jit-bf16_b200"), os.path.join(ROOT, "oracle"), HERE):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import herbert_b200 as hb  # noqa: E402
from harness import assert_sdpa_close, bits_of, oracle_attention, to_dev_bf16  # noqa: E402
from herbert_b200.inputs import AttentionInputs  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--chunk", type=int, default=256)
    ap.add_argument("--repeat", type=int, default=2)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    from datetime import timedelta
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=timedelta(seconds=120))
    comm = None
    try:
        chunk = a.chunk
        inp = AttentionInputs(rows=2 * world * chunk, past=0, seed=0x5EED0035)
        cp = hb.cp_spec(world, rank, chunk)
        pos = np.asarray(hb.cp_positions(cp, rank))
        q = to_dev_bf16(inp.q[pos])
        k = to_dev_bf16(np.ascontiguousarray(inp.keys[:, pos]))
        v = to_dev_bf16(np.ascontiguousarray(inp.values[:, pos]))
        out = torch.zeros((2 * chunk, inp.out_row), dtype=torch.int16, device="cuda")
        comm = hb.CpComm()
        side = torch.cuda.Stream(priority=-1)
        spec = hb.attention_spec()
        ws = None
        outs = []
        for _ in range(a.repeat):  # the second call reuses the workspace
            out.zero_()
            ws = hb.prefill_cp(spec, cp, q, k, v, out, kv_stride=2 * chunk * 256, scale=inp.scale,
                               comm=comm, workspace=ws, comm_stream=side)
            torch.cuda.synchronize()
            ws.status()
            outs.append(bits_of(out).copy())
        assert all(np.array_equal(outs[0], o) for o in outs[1:]), "repeat differs"
        # NCCL moves no int16: gather the bits as bf16
        gathered = [torch.zeros_like(out).view(torch.bfloat16) for _ in range(world)]
        dist.all_gather(gathered, out.view(torch.bfloat16))
        gathered = [g.view(torch.int16) for g in gathered]
        if rank == 0:
            full = np.zeros((inp.rows, inp.out_row), np.uint16)
            for r in range(world):
                full[np.asarray(hb.cp_positions(hb.cp_spec(world, r, chunk), r))] = \
                    bits_of(gathered[r])
            ref = oracle_attention(inp)
            err = assert_sdpa_close(full, ref, f"nccl ring world={world}")
            print(f"cp ring ok world={world} chunk={chunk} max_abs={err[0]:.3e} rel={err[1]:.3e}",
                  flush=True)
        dist.barrier()
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
