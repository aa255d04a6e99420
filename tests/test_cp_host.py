"""Context-parallel prefill, host side, on CPU: the ring schedule and the
zig-zag positions exported by the C ABI, the refusals of the CP entry
points, and a world_size-2 (and 3) gloo run of the whole ring -- shards
moving by send/recv in the library's hop order, each hop's partial attention
merged by log-sum-exp in the log2 domain as the hop kernel does -- checked
against single-process causal attention in f64.  No kernel launches."""
import ctypes
import os
import socket

import numpy as np
import pytest

import herbert_b200 as hb


@pytest.mark.parametrize("ranks", [1, 2, 3, 4, 8])
def test_every_rank_sees_every_shard_once(ranks):
    for rank in range(ranks):
        cp = hb.cp_spec(ranks, rank, 128)
        src = [hb.cp_hop_source(cp, h) for h in range(ranks)]
        assert src[0] == rank
        assert sorted(src) == list(range(ranks))
        # shard j reaches rank r after (r - j) mod P forwards along r-1 -> r
        assert all(src[h] == (rank - h) % ranks for h in range(ranks))
        assert hb.cp_hop_source(cp, ranks) == -1 and hb.cp_hop_source(cp, -1) == -1


@pytest.mark.parametrize("ranks,chunk", [(1, 128), (2, 128), (4, 256), (8, 128)])
def test_zigzag_positions_cover_the_sequence_and_balance_work(ranks, chunk):
    seen = []
    work = []
    for rank in range(ranks):
        cp = hb.cp_spec(ranks, rank, chunk)
        pos = [hb.cp_row_position(cp, rank, r) for r in range(2 * chunk)]
        assert pos == hb.cp_positions(cp, rank)
        assert hb.cp_row_position(cp, rank, 2 * chunk) == -1
        seen += pos
        work.append(sum(p + 1 for p in pos))  # keys seen by the rank's rows
    assert sorted(seen) == list(range(2 * ranks * chunk))
    assert len(set(work)) == 1  # zig-zag: every rank does the same causal work


def _call(chunk, **kw):
    base = dict(q=256, keys=256, values=256, output=256, rows=2 * chunk, past=0,
                kv_stride=2 * chunk * 256, capacity=0, scale=0.0625, sink=0.0)
    base.update(kw)
    return hb.AttentionCall(**base)


def _cp(spec, cp, call, comm=None, ws=1 << 20, nbytes=1 << 40):
    return hb.lib().hb_attn_prefill_cp(ctypes.byref(spec), ctypes.byref(cp), ctypes.byref(call),
                                       comm, ctypes.c_void_p(ws), nbytes, None, None)


def test_cp_refusals():
    spec = hb.attention_spec()
    assert _cp(spec, hb.cp_spec(2, 0, 100), _call(100)) == hb.HB_DECLINE_GEOMETRY
    assert _cp(spec, hb.cp_spec(2, 2, 128), _call(128)) == hb.HB_ERR_ARG
    assert _cp(spec, hb.cp_spec(0, 0, 128), _call(128)) == hb.HB_ERR_ARG
    assert _cp(spec, hb.cp_spec(2, 0, 128), _call(128, rows=128)) == hb.HB_ERR_ARG
    assert _cp(spec, hb.cp_spec(2, 0, 128), _call(128, past=4)) == hb.HB_ERR_ARG
    assert _cp(spec, hb.cp_spec(2, 0, 128), _call(128, kv_stride=128 * 256)) == hb.HB_ERR_ARG
    # a ring of two needs a communicator (checked before any launch)
    assert _cp(spec, hb.cp_spec(2, 0, 128), _call(128)) == hb.HB_ERR_ARG
    assert "communicator" in hb.last_error()
    assert _cp(spec, hb.cp_spec(2, 0, 128), _call(128), nbytes=4096) == hb.HB_ERR_WORKSPACE
    assert _cp(spec, hb.cp_spec(1 << 20, 0, 1 << 12), _call(1 << 12)) == hb.HB_DECLINE_GEOMETRY
    small = hb.attention_spec(heads=16, gqa=4, head_dim=128)
    assert _cp(small, hb.cp_spec(2, 0, 128), _call(128, kv_stride=256 * 128)) == \
        hb.HB_DECLINE_HEAD_DIM
    rc = hb.lib().hb_attn_prefill_cp_hop(ctypes.byref(spec), ctypes.byref(hb.cp_spec(2, 0, 128)),
                                         ctypes.byref(_call(128)), 2, ctypes.c_void_p(1 << 20),
                                         1 << 40, None)
    assert rc == hb.HB_ERR_ARG


def test_cp_workspace_size():
    spec = hb.attention_spec()
    one = hb.lib().hb_attn_prefill_cp_workspace_bytes(ctypes.byref(spec),
                                                      ctypes.byref(hb.cp_spec(1, 0, 1024)))
    two = hb.lib().hb_attn_prefill_cp_workspace_bytes(ctypes.byref(spec),
                                                      ctypes.byref(hb.cp_spec(2, 0, 1024)))
    acc = 16 * (2048 // 128) * 128 * (2 + 256) * 4
    assert one >= 256 + acc
    shard = 4 * 2048 * 256 * 2  # K (or V) of one shard
    assert two == one + 4 * shard


# ----------------------------------------------------------- gloo ring

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(ranks, chunk, heads=2, kv_heads=1, hd=16, seed=7):
    rng = np.random.default_rng(seed)
    S = 2 * ranks * chunk
    q = rng.standard_normal((S, heads, hd))
    k = rng.standard_normal((kv_heads, S, hd))
    v = rng.standard_normal((kv_heads, S, hd))
    return q, k, v, 1.0 / np.sqrt(hd)


def _full_causal(q, k, v, scale):
    S, heads, _ = q.shape
    gqa = heads // k.shape[0]
    out = np.zeros_like(q)
    for h in range(heads):
        s = q[:, h] @ k[h // gqa].T * scale
        s[np.triu_indices(S, 1)] = -np.inf
        p = np.exp(s - s.max(1, keepdims=True))
        out[:, h] = (p / p.sum(1, keepdims=True)) @ v[h // gqa]
    return out


def _ring_rank(rank, world, port, chunk, result):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, scale = _problem(world, chunk)
        cp = hb.cp_spec(world, rank, chunk)
        pos = np.array([hb.cp_row_position(cp, rank, r) for r in range(2 * chunk)])
        ql = q[pos]
        heads, gqa = q.shape[1], q.shape[1] // k.shape[0]
        # the shard in transit: K/V of the rank's own positions
        shard = torch.from_numpy(np.stack([k[:, pos], v[:, pos]]).copy())
        m = np.full((2 * chunk, heads), -np.inf)
        l = np.zeros((2 * chunk, heads))
        o = np.zeros_like(ql)
        for hop in range(world):
            src = hb.cp_hop_source(cp, hop)
            kpos = np.array([hb.cp_row_position(hb.cp_spec(world, src, chunk), src, r)
                             for r in range(2 * chunk)])
            ks, vs = shard[0].numpy(), shard[1].numpy()
            if hop + 1 < world:  # forward this shard, receive the next
                nxt = torch.empty_like(shard)
                reqs = [dist.isend(shard, (rank + 1) % world),
                        dist.irecv(nxt, (rank - 1) % world)]
            mask = kpos[None, :] <= pos[:, None]
            for h in range(heads):
                s = (ql[:, h] @ ks[h // gqa].T) * scale * np.log2(np.e)
                s = np.where(mask, s, -np.inf)
                mh = s.max(1)
                seen = np.isfinite(mh)
                p = np.where(seen[:, None], np.exp2(s - np.where(seen, mh, 0)[:, None]), 0.0)
                lh, oh = p.sum(1), p @ vs[h // gqa]
                # the hop kernel's merge: m' = max, weights 2^(m_old - m'), 2^(m_hop - m')
                mn = np.maximum(m[:, h], mh)
                live = np.isfinite(mn)
                wa = np.where(live, np.exp2(np.where(live, m[:, h] - mn, 0)), 0.0)
                wb = np.where(live & seen, np.exp2(np.where(seen, mh - mn, 0)), 0.0)
                o[:, h] = o[:, h] * wa[:, None] + oh * wb[:, None]
                l[:, h] = l[:, h] * wa + lh * wb
                m[:, h] = mn
            if hop + 1 < world:
                for r in reqs:
                    r.wait()
                shard = nxt
        out = o / l[:, :, None]
        full = torch.zeros(q.shape, dtype=torch.float64)
        full[torch.from_numpy(pos)] = torch.from_numpy(out)
        dist.all_reduce(full)  # disjoint rows: the sum assembles the sequence
        if rank == 0:
            ref = _full_causal(q, k, v, scale)
            result.put(float(np.abs(full.numpy() - ref).max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ring_matches_single_process_attention(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_rank, args=(r, world, port, 8, result))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = result.get(timeout=5)
    assert err < 1e-12, err
