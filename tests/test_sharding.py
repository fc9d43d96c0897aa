"""Sequence sharding host logic, single process and as two gloo ranks on CPU."""

from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp

from augur_b200 import sharding


def test_lpt_is_a_partition_and_balanced():
    lens = sharding.box_lengths()
    assert lens.shape == (2048,) and lens.min() >= 64 and lens.max() <= 8192
    for n in (1, 2, 4, 8):
        shards = sharding.lpt_assign(lens, n)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(2048))
        tok = sharding.shard_tokens(shards, lens)
        assert sum(tok) == int(lens.sum())
        # LPT bound: max load <= mean + the longest sequence
        assert max(tok) <= lens.sum() / n + lens.max()


def test_lpt_small_known_answer():
    # longest first: 9 -> r0 (9), 7 -> r1 (7), 5 -> r1 (12), 3 -> r0 (12), 1 -> tie, lowest rank r0
    assert sharding.lpt_assign([5, 9, 1, 7, 3], 2) == [[1, 2, 4], [0, 3]]
    assert sharding.lpt_assign([4, 4, 4], 3) == [[0], [1], [2]]
    assert sharding.lpt_assign([], 2) == [[], []]
    with pytest.raises(ValueError):
        sharding.lpt_assign([1], 0)


def test_aggregate():
    reps = [sharding.ShardReport(0, 3, 100, 1000, 2.0), sharding.ShardReport(1, 2, 60, 600, 4.0)]
    agg = sharding.aggregate(reps)
    assert agg["bytes"] == 1600 and agg["max_device_ms"] == 4.0
    assert agg["GBps"] == pytest.approx(1600 / 4e-3 / 1e9)
    assert agg["token_imbalance"] == pytest.approx(100 / 80)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = sharding.box_lengths(n_seqs=256, seed=1)
        shards = sharding.lpt_assign(lens, world)
        mine = shards[rank]
        tok = int(lens[mine].sum())
        rep = sharding.ShardReport(rank, len(mine), tok, tok * 24576, 1.0 + rank)
        reps = sharding.gather_reports(rep)
        q.put((rank, [r.rank for r in reps], [r.sequences for r in reps], sharding.aggregate(reps),
               sorted(mine)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_plan_and_report():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort(key=lambda x: x[0])
    lens = sharding.box_lengths(n_seqs=256, seed=1)
    expect = sharding.lpt_assign(lens, 2)
    for rank, ranks, seqs, agg, mine in results:
        assert ranks == [0, 1]
        assert seqs == [len(s) for s in expect]
        assert agg["max_device_ms"] == 2.0 and agg["bytes"] == int(lens.sum()) * 24576
        assert mine == expect[rank]
    assert sorted(results[0][4] + results[1][4]) == list(range(256))
