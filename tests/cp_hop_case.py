"""One rank of an emulated context-parallel ring on one GPU, for timing and
profiling the hop kernel (not collected by pytest): rank 3 of 8, random bf16
shards, all 8 hops through hb_attn_prefill_cp_hop then
hb_attn_prefill_cp_finish, the same calls tests/test_cp_gpu.py checks
against the oracle.  CP_CHUNK sets the chunk (default 1024)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(ROOT, "herbert-jit-bf16_b200")]

import torch  # noqa: E402

import herbert_b200 as hb  # noqa: E402

P, RANK = 8, 3
HQ, HKV, HD = 16, 4, 256


def main():
    c = int(os.environ.get("CP_CHUNK", "1024"))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn((2 * c, 2 * HQ * HD), generator=g, device=dev).to(torch.bfloat16)
    kv = torch.randn((2, HKV, 2 * c, HD), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty((2 * c, HQ * HD), dtype=torch.bfloat16, device=dev)
    spec = hb.attention_spec()
    cp = hb.cp_spec(P, RANK, c)
    ws = None
    for hop in range(P):
        ws = hb.prefill_cp_hop(spec, cp, q, kv[0], kv[1], out, hop, kv_stride=2 * c * HD,
                               workspace=ws)
    hb.prefill_cp_finish(spec, cp, q, kv[0], kv[1], out, kv_stride=2 * c * HD, workspace=ws)
    torch.cuda.synchronize()
    ws.status()
    print("ok")


if __name__ == "__main__":
    main()
