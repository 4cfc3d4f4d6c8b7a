"""The benchmark's multi-rank plumbing on CPU: two gloo ranks on 127.0.0.1 run the same
``bench.Ranks`` code the NCCL job runs (barrier, max over ranks of the step time, agreed
repetition count), and the per-rank shard seeds and whole-job value follow weak scaling."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ranks = bench.Ranks(world, rank, torch.device("cpu"), dist)
        ranks.barrier()
        # Each rank times a different step; the job's step time is the slowest rank's.
        step_ms = ranks.max_float(0.05 + 0.01 * rank)
        reps = ranks.max_int(3 + rank)
        per_rank = ranks.gather_floats([10.0 + rank, 20.0 + rank])
        seeds = [bench.shard_seed(rank, r) for r in range(4)]
        gathered = [None] * world
        dist.all_gather_object(gathered, seeds)
        ranks.barrier()
        out[rank] = (step_ms, reps, gathered, per_rank)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    for rank in range(world):
        step_ms, reps, seeds, per_rank = out[rank]
        assert step_ms == pytest.approx(0.06)   # max over ranks, identical on every rank
        assert reps == 4
        assert per_rank == [[10.0, 20.0], [11.0, 21.0]]  # every rank's figures, in rank order
        assert not set(seeds[0]) & set(seeds[1])  # disjoint input sets per rank


def test_whole_job_value_is_weak_scaling():
    one = bench.whole_job_value(bench.B * bench.LQ, 1, 0.07)
    eight = bench.whole_job_value(bench.B * bench.LQ, 8, 0.07)
    assert eight == pytest.approx(8 * one)
    assert one == pytest.approx(bench.B * bench.LQ / 0.07e-3)


def test_single_rank_needs_no_process_group():
    ranks = bench.Ranks(1, 0, torch.device("cpu"))
    ranks.barrier()
    assert ranks.max_float(1.5) == 1.5 and ranks.max_int(7) == 7
    assert ranks.gather_floats([2, 3]) == [[2.0, 3.0]]
