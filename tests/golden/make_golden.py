"""Writes the golden fixtures of this directory from the CPU oracle.

The reference (xigh/herbert-jit-bf16) has no tests, no golden vectors and
cannot be built in this image, so these fixtures are the oracle's own
outputs on small seeded inputs, committed so that (a) any change to the
oracle shows up as a fixture mismatch and (b) the GPU parity tests have
inputs/outputs that do not depend on the host that runs them.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "herbert-jit-bf16_b200"),
                os.path.join(ROOT, "tests")]

from herbert_b200.inputs import AttentionInputs, DeltaFrontInputs, DeltaInputs, FrontInputs  # noqa: E402,E501
from harness import oracle_attention, oracle_gdn  # noqa: E402
import oracle as O  # noqa: E402

ATTN_CASES = {
    # name: (rows, past, heads, kv_heads, head_dim, gated)
    "attn_decode_n38": (1, 37, 16, 4, 256, True),
    "attn_decode_n1": (1, 0, 16, 4, 256, True),
    "attn_rows11_past5": (11, 5, 16, 4, 256, True),
    "attn_hd128_g2_nogate": (3, 20, 4, 2, 128, False),
}
GDN_CASES = {
    # name: (rows, nk, nv, hkd, hvd, state_scale)
    "gdn_rows5_zero_state": (5, 2, 4, 128, 128, 0.0),
    "gdn_rows3_warm_state": (3, 2, 4, 128, 128, 0.1),
}


def main():
    for name, (rows, past, heads, kvh, hd, gated) in ATTN_CASES.items():
        inp = AttentionInputs(rows, past, heads=heads, kv_heads=kvh, head_dim=hd, gated=gated,
                              seed=0x60D0 + len(name))
        out = oracle_attention(inp)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), q=inp.q, keys=inp.keys,
                            values=inp.values, out=out,
                            meta=np.array([rows, past, heads, kvh, hd, int(gated)], np.int64))
    for name, (rows, nk, nv, hkd, hvd, ss) in GDN_CASES.items():
        state = np.random.default_rng(7).standard_normal((nv, hkd, hvd)).astype(np.float32) * ss
        inp = DeltaInputs(rows, nk=nk, nv=nv, hkd=hkd, hvd=hvd, seed=0x60D1 + len(name),
                          state=state)
        out, st = oracle_gdn(inp)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), qkv=inp.qkv, beta=inp.beta,
                            decay=inp.decay, state0=inp.state, out=out, state=st,
                            meta=np.array([rows, nk, nv, hkd, hvd], np.int64))
    # attention front end (head-norm-rope + kv-append), Qwen3.5 geometry
    f = FrontInputs(5, 9, seed=0x60D2)
    q, k, keys, values = O.attn_front(f.q, f.k, f.v, f.q_norm, f.k_norm, f.cos, f.sin,
                                      heads=f.heads, kv_heads=f.kv_heads, head_dim=f.head_dim,
                                      rotary=f.rotary, past=f.past, gemma=f.gemma, keys=f.keys,
                                      values=f.values)
    np.savez_compressed(os.path.join(HERE, "front_rows5_past9.npz"), q=f.q, k=f.k, v=f.v,
                        q_norm=f.q_norm, k_norm=f.k_norm, cos=f.cos, sin=f.sin, keys0=f.keys,
                        values0=f.values, q_out=q, k_out=k, keys=keys, values=values,
                        meta=np.array([f.rows, f.past, f.heads, f.kv_heads, f.head_dim, f.rotary,
                                       int(f.gemma), int(f.gated)], np.int64))
    # DeltaNet front end (conv + SiLU, gates) and gated norm: conv width 68
    # (four vector blocks and a scalar tail of 4), V head width 16
    d = DeltaFrontInputs(5, nk=1, nv=2, hkd=18, hvd=16, seed=0x60D3)
    d.qkv.reshape(-1)[:3] = [0.0, 1e30, -np.inf]
    y, st = O.gdn_conv(d.qkv, d.conv_state, d.conv_weight)
    beta, decay = O.gdn_gates(d.ab, d.dt_bias, d.a_log)
    yn, ob = O.gdn_gated_norm(d.x, d.z, d.norm_weight)
    np.savez_compressed(os.path.join(HERE, "gdn_front_rows5.npz"), qkv=d.qkv,
                        conv_state=d.conv_state, conv_weight=d.conv_weight, ab=d.ab,
                        dt_bias=d.dt_bias, a_log=d.a_log, x=d.x, z=d.z, norm_weight=d.norm_weight,
                        qkv_out=y, conv_state_out=st, beta=beta, decay=decay, norm_f32=yn,
                        norm_bf16=ob, meta=np.array([d.rows, d.nk, d.nv, d.hkd, d.hvd, d.ck],
                                                    np.int64))
    # snapshot image of a hybrid state (two cached layers among eight, DeltaNet
    # states, logits) at position 21 in a 32-position slot, as the reference's
    # Instantaneous::write_to lays it out
    import snapshot as S
    r = S.seeded_runner(2, 40, [0, 0, 0, 64, 0, 0, 0, 64], 6 * 96 * 4, 6 * 2 * 16 * 16, 48, 21,
                        0x60D4)
    slot = S.snapshot_reserve(r, 32)
    S.snapshot_take(r, slot)
    with open(os.path.join(HERE, "snapshot_hybrid.bin"), "wb") as f:
        f.write(S.write_to(slot))
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith((".npz", ".bin"))))


if __name__ == "__main__":
    main()
