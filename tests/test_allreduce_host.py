"""The peer all-reduce's host logic on CPU: two gloo ranks exchange their (fake) IPC exports over
the process group, and each rank maps exactly its peer's exports, in rank order, keeping its own
pointers; mismatched sizes raise on every rank.  The device kernel needs two GPUs
(``tests/test_allreduce_gpu.py``)."""

from __future__ import annotations

import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, sizes, out):
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    from rfdetr_jax_b200 import collective as C

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        n = sizes[rank]
        exports = [(f"buf{rank}".encode(), 64 * rank), (f"flags{rank}".encode(), 0)]
        entries = C.exchange_exports(None, rank, world, n, exports)
        opened = []

        def fake_open(handle, offset):
            opened.append((handle, offset))
            return 1000 * (len(opened)) + offset

        try:
            bufs, flags = C.peer_pointers(entries, rank, n, [11 + rank, 22 + rank], fake_open)
            out[rank] = ("ok", bufs, flags, opened)
        except ValueError as e:
            out[rank] = ("error", str(e))
        assert pkg.PeerAllReduce is C.PeerAllReduce
    finally:
        dist.destroy_process_group()


def _run(sizes):
    world = len(sizes)
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), sizes, out), nprocs=world, start_method="spawn",
                       join=True)
    return dict(out)


def test_two_ranks_map_each_other():
    out = _run([4096, 4096])
    for rank in range(2):
        status, bufs, flags, opened = out[rank]
        peer = 1 - rank
        assert status == "ok"
        assert (bufs[rank], flags[rank]) == (11 + rank, 22 + rank)  # own pointers kept
        assert opened == [(f"buf{peer}".encode(), 64 * peer), (f"flags{peer}".encode(), 0)]
        assert (bufs[peer], flags[peer]) == (1000 + 64 * peer, 2000)


def test_size_mismatch_raises_on_every_rank():
    out = _run([4096, 4100])
    for rank in range(2):
        assert out[rank][0] == "error" and "registered" in out[rank][1]


def test_rejects_host_buffers():
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    with pytest.raises(ValueError, match="CUDA"):
        pkg.PeerAllReduce(torch.zeros(16))
