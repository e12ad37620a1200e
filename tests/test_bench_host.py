"""CPU tests of bench.py's host logic: the BASELINE config 4 clip set, its static longest-first
partition over ranks, and the multi-rank reduction bench.py performs, on two gloo ranks."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_clip_set_is_config4():
    clips = bench.clip_set()
    assert len(clips) == 256
    assert [c[0] for c in clips] == list(range(256))
    secs = np.array([c[1] for c in clips])
    assert secs.min() >= 5.0 and secs.max() <= 30.0
    assert all(c[2] == int(round(7.5 * c[1])) for c in clips)
    assert clips == bench.clip_set()  # seeded


@pytest.mark.parametrize('world', [1, 2, 3, 4, 8])
def test_partition_covers_every_clip_once_and_balances(world):
    clips = bench.clip_set()
    parts = bench.partition(clips, world)
    assert sorted(i for p in parts for i in p) == list(range(len(clips)))
    loads = [sum(clips[i][2] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(c[2] for c in clips)
    for p in parts:  # longest first within a rank
        toks = [clips[i][2] for i in p]
        assert toks == sorted(toks, reverse=True)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        clips = bench.clip_set()
        mine = bench.partition(clips, world)[rank]
        load = float(sum(clips[i][2] for i in mine))
        t = torch.tensor([load], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the max-over-ranks time reduction of bench.py
        total = torch.tensor([float(len(mine))], dtype=torch.float64)
        dist.all_reduce(total, op=dist.ReduceOp.SUM)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        out.put((rank, float(t), float(total), gathered))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_partition_and_reductions():
    world = 2
    ctx = mp.get_context('spawn')
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    clips = bench.clip_set()
    parts = bench.partition(clips, world)
    expect_max = max(float(sum(clips[i][2] for i in p)) for p in parts)
    for rank, tmax, total, gathered in results:
        assert tmax == expect_max
        assert total == len(clips)
        assert gathered == parts
