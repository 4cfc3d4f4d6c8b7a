"""The NVLink peer-memory gradient all-reduce (``PeerAllReduce`` / ``rfdetr_allreduce_sum_f32``)
on two GPUs, one process each: bit-exact against the rank-order float32 sum computed on the CPU,
over whole buffers, bucket ranges and sizes that are not a multiple of the vector width; then
against NCCL's all-reduce within float32 rounding.  Needs two GPUs (skipped otherwise)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, root: str, out_dir: str) -> None:
    import sys

    import torch.distributed as dist

    sys.path.insert(0, root)
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    results = {}
    try:
        for n in (1, 7, 4096 + 3, 1_000_003):
            host = [np.random.default_rng(100 * n + r).standard_normal(n).astype(np.float32) for r in range(world)]
            buf = torch.tensor(host[rank], device=f"cuda:{rank}")
            ar = pkg.PeerAllReduce(buf, ctas=16)
            want = host[0].copy()
            for r in range(1, world):
                want = (want + host[r]).astype(np.float32)
            for _ in range(3):  # the same sum repeated: every epoch must land
                buf.copy_(torch.tensor(host[rank], device=f"cuda:{rank}"))
                ar()
                torch.cuda.synchronize()
                ar.check()
                np.testing.assert_array_equal(buf.cpu().numpy(), want, err_msg=f"n={n}")
            if n >= 4096:
                # Bucket ranges of one registration, reduced in separate calls.
                buf.copy_(torch.tensor(host[rank], device=f"cuda:{rank}"))
                cut = (n // 3) & ~3
                ar(offset=0, count=cut)
                ar(offset=cut)
                torch.cuda.synchronize()
                ar.check()
                np.testing.assert_array_equal(buf.cpu().numpy(), want, err_msg=f"n={n} in two ranges")
            dist.barrier()
            ar.close()
            results[n] = True
        # Against NCCL on the same data (a different summation tree: float32 rounding apart).
        n = 1 << 20
        host = [np.random.default_rng(7 + r).standard_normal(n).astype(np.float32) for r in range(world)]
        a = torch.tensor(host[rank], device=f"cuda:{rank}")
        ar = pkg.PeerAllReduce(a, ctas=64)
        ar()
        torch.cuda.synchronize()
        ar.check()
        ar.close()
        want = np.sum(np.stack(host).astype(np.float64), 0)
        np.testing.assert_allclose(a.cpu().numpy(), want, rtol=1e-6, atol=1e-6)
        with open(os.path.join(out_dir, f"rank{rank}.ok"), "w") as f:
            f.write(repr(results))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_allreduce_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), root, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}.ok").exists()
