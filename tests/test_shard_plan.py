"""Batched decode over several GPUs (one process per GPU, no collective):
hb_decode_shard_plan assigns the sequences to the GPUs by their KV cost,
longest first, each to the least-loaded GPU.  CPU only: coverage, the
rule's tie order, its guarantee against brute-force optima, refusals, and
that every rank of a gloo group derives the same disjoint cover."""
import itertools
import os

import numpy as np
import pytest

import herbert_b200 as hb
from herbert_b200.inputs import batch_lengths


def test_every_sequence_goes_to_exactly_one_gpu():
    lens = batch_lengths()
    for parts in (1, 2, 4, 8, 64, 100):
        part, load = hb.shard_plan(lens, parts)
        assert len(part) == len(lens) and all(0 <= g < parts for g in part)
        assert sum(load) == int(lens.sum())
        for g in range(parts):
            assert load[g] == int(sum(int(lens[i]) for i, x in enumerate(part) if x == g))
        # list scheduling: the busiest GPU exceeds the mean by at most one sequence
        assert max(load) <= lens.sum() / parts + lens.max()


def test_longest_first_least_loaded_lowest_index_on_ties():
    part, load = hb.shard_plan([5, 5, 5, 5], 2)
    assert part == [0, 1, 0, 1] and load == [10, 10]
    part, load = hb.shard_plan([1, 7, 3, 3, 2], 3)
    # 7 -> 0; 3 -> 1; 3 -> 2; 2 -> 1 (3 < 7, 1 < 2); 1 -> 2
    assert part == [2, 0, 1, 2, 1] and load == [7, 5, 4]
    assert hb.shard_plan([0, 0, 0], 2)[0] == [0, 0, 0]  # loads stay tied at zero: GPU 0


def test_within_the_lpt_guarantee_of_the_optimum():
    rng = np.random.default_rng(7)
    for _ in range(60):
        n, m = int(rng.integers(2, 9)), int(rng.integers(2, 4))
        w = [int(x) for x in rng.integers(1, 1000, size=n)]
        _, load = hb.shard_plan(w, m)
        opt = min(max(sum(w[i] for i in range(n) if a[i] == g) for g in range(m))
                  for a in itertools.product(range(m), repeat=n))
        assert max(load) <= (4 / 3 - 1 / (3 * m)) * opt + 1e-9, (w, m, load, opt)


def test_refusals():
    import ctypes
    L = hb.lib()
    c = (ctypes.c_int64 * 2)(1, -1)
    part = (ctypes.c_int32 * 2)()
    assert L.hb_decode_shard_plan(c, 2, 2, part, None) == hb.HB_ERR_ARG
    c = (ctypes.c_int64 * 2)(1, 1)
    assert L.hb_decode_shard_plan(c, 2, 0, part, None) == hb.HB_ERR_ARG
    assert L.hb_decode_shard_plan(c, 2, 4097, part, None) == hb.HB_ERR_ARG
    assert L.hb_decode_shard_plan(c, 0, 2, part, None) == hb.HB_DECLINE_EMPTY
    assert L.hb_decode_shard_plan(None, 2, 2, part, None) == hb.HB_ERR_ARG
    big = (ctypes.c_int64 * 2)(1 << 61, 1 << 61)
    assert L.hb_decode_shard_plan(big, 2, 2, part, None) == hb.HB_ERR_ARG


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = hb.shard_of(batch_lengths(), world, rank)
        got = [None] * world
        dist.all_gather_object(got, mine)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_ranks_agree_on_a_disjoint_cover(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    res = dict(q.get(timeout=5) for _ in range(world))
    views = list(res.values())
    assert all(v == views[0] for v in views)  # every rank derived the same plan
    flat = sorted(i for shard in views[0] for i in shard)
    assert flat == list(range(64))
