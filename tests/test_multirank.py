"""The bench's multi-rank host logic with two gloo ranks on CPU: disjoint stream shards, the max-over-ranks
device time every rank receives, and the whole-job rate computed from it (one process per GPU on the GPU box,
streams sharded with no collective on the data path)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids = bench.rank_streams(4, rank)
        t = bench.max_over_ranks(10.0 + 5.0 * rank, dist, torch.device("cpu"))
        rate = bench.whole_job_rate(4, 3, world, t)
        gathered = [None] * world
        dist.all_gather_object(gathered, ids)
        out.put((rank, ids, t, rate, gathered))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_streams_and_agree_on_the_slowest_time():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    all_ids = [i for _, ids, *_ in res for i in ids]
    assert len(set(all_ids)) == len(all_ids) == 8            # disjoint shards covering 8 streams
    assert all(t == pytest.approx(15.0) for _, _, t, _, _ in res)   # every rank sees the slowest rank's time
    assert all(rate == pytest.approx(4 * 3 * 2 / 0.015) for *_, rate, _ in res)
    assert res[0][4] == res[1][4]


def test_single_process_has_no_collective():
    assert bench.max_over_ranks(7.5, None, None) == 7.5
    assert bench.rank_streams(3, 0) == [0, 1, 2]
