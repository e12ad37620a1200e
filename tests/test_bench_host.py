"""CPU tests of bench.py's host logic: the BASELINE config 4 clip set, its static longest-first
partition over ranks, the clock record parsed from nvidia-smi's CSV samples, and the multi-rank
reduction bench.py performs, on two gloo ranks."""

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


def test_clock_summary_parses_samples_and_reasons():
    """The clock record of a timed region: median SM clock under load, the max clock, and every throttle
    reason seen Active in any sample (fields as bench.ClockSampler.FIELDS asks nvidia-smi for them)."""
    cs = bench.ClockSampler(0)
    cs.lines = ['0, 1965, 1965, 612.3, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active',
                '0, 1950, 1965, 998.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active',
                '0, 1965, 1965, 640.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active',
                'garbage line']
    s = cs.summary()
    assert s == {'sm_mhz': 1965.0, 'sm_max_mhz': 1965.0, 'reasons': ['sw_power_cap'], 'samples': 3}
    cs.lines = ['0, 1200, 1965, 700.0, 0x0000000000000008, Active, Not Active, Active, Not Active']
    assert cs.summary()['reasons'] == ['hw_slowdown', 'sw_thermal_slowdown']
    cs.lines = []
    assert cs.summary() == {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unavailable']}


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
