"""Multi-process host logic of the clip-sharded benchmark on CPU (gloo, two
ranks): each rank codes its own clips with no data-path exchange, the timed
region ends in a max over ranks, the whole-job rate counts every rank's clips
against the slowest rank's time, and the result gather (the one collective on
the data path) delivers every rank's streams to rank 0."""
from __future__ import annotations

import os
import pathlib
import socket
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import datetime

    import torch
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        seeds = bench.clip_seeds(rank, 4)
        gathered = [None] * world
        dist.all_gather_object(gathered, seeds)
        # Per-rank elapsed times differ; every rank must see the slowest.
        elapsed = 100.0 + 50.0 * rank
        slowest = bench.max_over_ranks(elapsed, world, torch, dist)
        rate = bench.whole_job_rate(4 * 30.0, world, slowest)
        # Result gather: ragged per-rank stream lists reach rank 0 intact.
        mine = [bytes([rank, i]) * (i + 1) for i in range(rank + 2)]
        streams = bench.gather_streams(mine, world, rank, torch, dist)
        results[rank] = {"gathered": gathered, "slowest": slowest, "rate": rate,
                         "streams": streams}
    finally:
        dist.destroy_process_group()


def test_clip_sharding_and_max_over_ranks():
    import torch.multiprocessing as tmp

    world = 2
    manager = tmp.get_context("spawn").Manager()
    results = manager.dict()
    tmp.start_processes(_rank_main, args=(world, _free_port(), results), nprocs=world,
                        start_method="spawn", join=True)
    assert sorted(results.keys()) == [0, 1]
    for rank in range(world):
        r = results[rank]
        flat = [s for seeds in r["gathered"] for s in seeds]
        assert len(flat) == len(set(flat)) == 4 * world  # disjoint shards
        assert r["gathered"][0][0] == 0  # rank 0 clip 0 is the cfg0 clip
        assert r["slowest"] == pytest.approx(150.0)
        assert r["rate"] == pytest.approx(4 * 30.0 * world / 0.150)
    expected = [bytes([r, i]) * (i + 1) for r in range(world) for i in range(r + 2)]
    assert results[0]["streams"] == expected
    assert results[1]["streams"] is None


def test_host_thread_share(monkeypatch):
    import bench

    monkeypatch.delenv("LOCAL_WORLD_SIZE", raising=False)
    assert bench.host_thread_share(1) == 0  # alone: the library chooses
    cpus = len(os.sched_getaffinity(0))
    for world in (2, 4, 8):
        share = bench.host_thread_share(world)
        assert 1 <= share and (share * world <= cpus or share == 1)
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "1")
    assert bench.host_thread_share(8) == 0  # one rank per host
