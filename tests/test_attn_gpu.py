"""GPU parity of the SDPA kernels against the CPU oracle, through the C ABI.

Tolerance: max abs error <= 2 bf16 ulp of the output scale and relative
Frobenius error <= 5e-3 (tests/harness.py).  The gate epilogue reproduces the
reference's exp polynomial and rounding, so with the gate the outputs differ
from the oracle only through the SDPA sum order.
"""
import numpy as np
import pytest

from herbert_b200.inputs import AttentionInputs, normal_bf16
from harness import (ATTN_FIXTURES, assert_sdpa_close, gpu_attention, load_attn_fixture,
                     oracle_attention, to_dev_bf16, bits_of)

pytestmark = pytest.mark.gpu

DECODE_CASES = [
    # rows, past, heads, kv_heads, head_dim, gated
    (1, 2047, 16, 4, 256, True),    # the single decode step of the Qwen3.5 layer, n = 2048
    (1, 0, 16, 4, 256, True),       # n = 1
    (1, 15, 16, 4, 256, True),
    (1, 16, 16, 4, 256, True),
    (1, 100, 16, 4, 256, False),
    (1, 4999, 16, 4, 256, True),    # several splits, ragged last tile
    (3, 50, 16, 4, 256, True),      # rows > 1 in the decode regime
    (1, 700, 8, 8, 128, False),     # gqa 1, head_dim 128
    (2, 300, 16, 2, 128, True),     # gqa 8
    (1, 333, 8, 4, 256, True),      # gqa 2
    # one sequence of 129 .. 2048 positions at head_dim 256: the tensor-core
    # cluster form (one 128-position tile per CTA)
    (1, 128, 16, 4, 256, True),     # two tiles, the second holding one position
    (3, 382, 16, 4, 256, True),     # rows > 1: the fourth tile is empty for rows 0 and 1
    (1, 1000, 16, 2, 256, True),    # gqa 8
    (1, 600, 4, 4, 256, False),     # gqa 1, no gate
    (2, 1500, 16, 4, 256, True),
    # one sequence beyond 16 x 256 positions at head_dim 256: split-KV on the
    # tensor cores, 128-position tiles, partials merged by the last G CTAs of
    # a unit (one q head each) when the whole grid is resident at once
    (1, 32767, 16, 4, 256, True),   # the mixers' attention layer, n = 32768
    (1, 9000, 16, 2, 256, True),    # gqa 8, ragged last tile
    (2, 6000, 8, 8, 256, False),    # gqa 1, rows > 1, no gate
    (1, 20000, 8, 4, 256, True),    # gqa 2
    (3, 4094, 16, 4, 256, True),    # rows 0-1 at the cluster forms' limit, row 2 beyond it
    (2, 32000, 16, 4, 256, True),   # more CTAs than SMs: the last CTA of a unit merges every head
]


@pytest.mark.parametrize("case", DECODE_CASES, ids=lambda c: "r{}p{}h{}k{}d{}{}".format(
    c[0], c[1], c[2], c[3], c[4], "g" if c[5] else ""))
def test_decode_matches_oracle(cuda_device, case):
    rows, past, heads, kvh, hd, gated = case
    inp = AttentionInputs(rows, past, heads=heads, kv_heads=kvh, head_dim=hd, gated=gated,
                          capacity=past + rows + 7)
    got, _ = gpu_attention(inp, "decode")
    assert_sdpa_close(got, oracle_attention(inp), f"decode {case}")


def test_decode_workspace_reuse_is_stable(cuda_device):
    """The split counters reset themselves: the same workspace serves calls
    back to back with identical results."""
    inp = AttentionInputs(1, 3000)
    a, ws = gpu_attention(inp, "decode")
    b, _ = gpu_attention(inp, "decode", workspace=ws)
    c, _ = gpu_attention(inp, "decode", workspace=ws)
    assert np.array_equal(a, b) and np.array_equal(b, c)
    assert_sdpa_close(a, oracle_attention(inp), "reuse")


PREFILL_CASES = [
    # rows, past, heads, kv_heads, gated
    (64, 0, 16, 4, True),       # one partial 128-row tile on the tensor cores
    (37, 11, 16, 4, True),      # below 64 rows: the decode kernel
    (200, 300, 16, 4, True),
    (256, 0, 16, 4, True),
    (1000, 24, 16, 4, False),   # ragged last tile, no gate
    (129, 5000, 8, 8, True),    # long past, gqa 1
    (384, 0, 8, 1, True),       # gqa 8
    (4096, 0, 16, 4, True),     # the prefill configuration of the benchmark
]


@pytest.mark.parametrize("case", PREFILL_CASES, ids=lambda c: "r{}p{}h{}k{}{}".format(
    c[0], c[1], c[2], c[3], "g" if c[4] else ""))
def test_prefill_matches_oracle(cuda_device, case):
    rows, past, heads, kvh, gated = case
    inp = AttentionInputs(rows, past, heads=heads, kv_heads=kvh, gated=gated,
                          capacity=past + rows)
    got, _ = gpu_attention(inp, "prefill")
    assert_sdpa_close(got, oracle_attention(inp), f"prefill {case}")


@pytest.mark.parametrize("name", ATTN_FIXTURES)
def test_golden_fixtures(cuda_device, name):
    inp, ref = load_attn_fixture(name)
    for regime in ("decode", "prefill"):
        got, _ = gpu_attention(inp, regime)
        assert_sdpa_close(got, ref, f"{name} {regime}")


def test_batched_decode_ragged(cuda_device):
    import torch
    import herbert_b200 as hb
    lens = [1, 2, 31, 32, 33, 1000, 4097]
    spec = hb.attention_spec()
    seqs, keep, refs = [], [], []
    for i, n in enumerate(lens):
        inp = AttentionInputs(1, n - 1, capacity=n + 3, seed=1000 + 10 * i)
        q, k, v = to_dev_bf16(inp.q), to_dev_bf16(inp.keys), to_dev_bf16(inp.values)
        out = torch.zeros((1, inp.out_row), dtype=torch.int16, device="cuda")
        keep.append((q, k, v, out))
        seqs.append(hb.DecodeSeq(q=q.data_ptr(), keys=k.data_ptr(), values=v.data_ptr(),
                                 output=out.data_ptr(), past=n - 1, kv_stride=inp.kv_stride))
        refs.append(oracle_attention(inp))
    table = hb.seq_table(seqs)
    ws = hb.decode_batch(spec, table, len(lens), max(lens) - 1, sum(lens) - len(lens))
    torch.cuda.synchronize()
    ws.status()
    for (q, k, v, out), ref, n in zip(keep, refs, lens):
        assert_sdpa_close(bits_of(out), ref, f"batch n={n}")


@pytest.mark.parametrize("case", ["300 short", "upper-bound sum", "reuse"])
def test_batched_decode_balanced_ranges(cuda_device, case):
    # The batch kernel lays the tiles of all (sequence, KV head) units end to
    # end and cuts them into one range per CTA: many short sequences (a
    # range crossing many units, more sequences than threads in the CTA's
    # scan), a plan from the upper-bound total (sum_past 0: more ranges than
    # tiles), and two calls through one workspace (counters left at zero).
    import numpy as np
    import torch
    import herbert_b200 as hb
    if case == "300 short":
        lens = [int(x) for x in np.random.default_rng(7).integers(1, 100, 300)]
    else:
        lens = [1, 3, 40, 64, 65, 700]
    spec = hb.attention_spec()
    seqs, keep, refs = [], [], []
    for i, n in enumerate(lens):
        inp = AttentionInputs(1, n - 1, capacity=n, seed=5000 + 7 * i)
        q, k, v = to_dev_bf16(inp.q), to_dev_bf16(inp.keys), to_dev_bf16(inp.values)
        out = torch.zeros((1, inp.out_row), dtype=torch.int16, device="cuda")
        keep.append((q, k, v, out))
        seqs.append(hb.DecodeSeq(q=q.data_ptr(), keys=k.data_ptr(), values=v.data_ptr(),
                                 output=out.data_ptr(), past=n - 1, kv_stride=inp.kv_stride))
        refs.append(oracle_attention(inp))
    table = hb.seq_table(seqs)
    sum_past = 0 if case == "upper-bound sum" else sum(lens) - len(lens)
    ws = None
    for _ in range(2 if case == "reuse" else 1):
        for _, _, _, out in keep:
            out.zero_()
        ws = hb.decode_batch(spec, table, len(lens), max(lens) - 1, sum_past, workspace=ws)
        torch.cuda.synchronize()
        ws.status()
        for (q, k, v, out), ref, n in zip(keep, refs, lens):
            assert_sdpa_close(bits_of(out), ref, f"{case} n={n}")


def test_batched_decode_misaligned_entry_is_skipped(cuda_device):
    # One table entry whose K pointer is 2 bytes off: the kernel checks each
    # entry before its bulk copies, issues no load and writes no output for
    # it, and reports HB_ERR_ARG through the workspace; the other sequences
    # match the oracle, and the workspace serves the next (good) call.  The entry
    # spans several ranges, so its partials and counter still run.
    import torch
    import herbert_b200 as hb
    lens = [300, 5000, 700]
    spec = hb.attention_spec()
    keep, refs = [], []
    for i, n in enumerate(lens):
        inp = AttentionInputs(1, n - 1, capacity=n + 8, seed=7000 + 3 * i)
        q, k, v = to_dev_bf16(inp.q), to_dev_bf16(inp.keys), to_dev_bf16(inp.values)
        out = torch.zeros((1, inp.out_row), dtype=torch.int16, device="cuda")
        keep.append((q, k, v, out, inp))
        refs.append(oracle_attention(inp))

    def table(bad):
        return hb.seq_table([hb.DecodeSeq(q=q.data_ptr(), keys=k.data_ptr() + (2 if bad and i == 1 else 0),
                                          values=v.data_ptr(), output=out.data_ptr(), past=n - 1,
                                          kv_stride=inp.kv_stride)
                             for i, ((q, k, v, out, inp), n) in enumerate(zip(keep, lens))])

    t_bad, t_good = table(True), table(False)
    ws = hb.decode_batch(spec, t_bad, len(lens), max(lens) - 1, sum(lens) - len(lens))
    torch.cuda.synchronize()
    with pytest.raises(hb.HBError) as err:
        ws.status()
    assert err.value.status == hb.HB_ERR_ARG
    assert not bits_of(keep[1][3]).any(), "no output for the skipped entry"
    for j in (0, 2):
        assert_sdpa_close(bits_of(keep[j][3]), refs[j], f"batch n={lens[j]} beside a bad entry")
    hb.decode_batch(spec, t_good, len(lens), max(lens) - 1, sum(lens) - len(lens), workspace=ws)
    torch.cuda.synchronize()
    ws.status()
    for (q, k, v, out, inp), ref, n in zip(keep, refs, lens):
        assert_sdpa_close(bits_of(out), ref, f"batch n={n} after the bad call")


def test_workspace_too_small_is_refused(cuda_device):
    import ctypes
    import torch
    import herbert_b200 as hb
    inp = AttentionInputs(1, 2047)
    small = hb.Workspace(256)
    q, k, v = to_dev_bf16(inp.q), to_dev_bf16(inp.keys), to_dev_bf16(inp.values)
    out = torch.zeros((1, inp.out_row), dtype=torch.int16, device="cuda")
    spec = hb.attention_spec()
    call = hb.AttentionCall(q=q.data_ptr(), keys=k.data_ptr(), values=v.data_ptr(),
                            output=out.data_ptr(), rows=1, past=2047, kv_stride=inp.kv_stride,
                            capacity=0, scale=inp.scale, sink=0.0)
    rc = hb.lib().hb_attn_decode(ctypes.byref(spec), ctypes.byref(call),
                                 ctypes.c_void_p(small.ptr), small.nbytes, None)
    assert rc == hb.HB_ERR_WORKSPACE, hb.last_error()


def test_kv_append_copies_into_the_reference_layout(cuda_device):
    import torch
    import herbert_b200 as hb
    heads, hd, cap, rows, past = 4, 256, 64, 9, 17
    keys = torch.zeros((heads, cap, hd), dtype=torch.int16, device="cuda")
    values = torch.zeros_like(keys)
    ik = normal_bf16((rows, heads, hd), 5)
    iv = normal_bf16((rows, heads, hd), 6)
    spec = hb.KvSpec(heads=heads, head_dim=hd, stride=cap * hd, capacity=cap, max_batch=16)
    hb.kv_append(spec, keys, values, to_dev_bf16(ik), to_dev_bf16(iv), rows=rows, past=past)
    torch.cuda.synchronize()
    K, V = bits_of(keys), bits_of(values)
    assert np.array_equal(K[:, past:past + rows], ik.transpose(1, 0, 2))
    assert np.array_equal(V[:, past:past + rows], iv.transpose(1, 0, 2))
    assert not K[:, :past].any() and not K[:, past + rows:].any()
