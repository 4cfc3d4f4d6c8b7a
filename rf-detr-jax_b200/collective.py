"""Data-parallel gradient all-reduce over NVLink peer memory (``rfdetr_allreduce_sum_f32``).

The reference's train step sums its gradients across the batch-sharded devices with
``jax.lax.psum`` (``src/rfdetr_jax/training/trainer.py:462-469``), an NCCL all-reduce under XLA.
:class:`PeerAllReduce` is that sum for one float32 buffer per rank, one process per GPU on one
node: the ranks map each other's buffers once (CUDA IPC handles exchanged over the process
group), then each call is one kernel launch per rank that reduces this rank's chunk from every
rank's buffer over NVLink and writes the sum back to all of them.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N


def exchange_exports(group, rank: int, world: int, n: int, exported: list) -> list:
    """Every rank's ``(rank, n, exported)`` in rank order, over the process group (the ranks'
    IPC handles and offsets travel on the host channel)."""
    import torch.distributed as dist

    entries = [None] * world
    dist.all_gather_object(entries, (rank, n, exported), group=group)
    return sorted(entries, key=lambda e: e[0])


def peer_pointers(entries: list, rank: int, n: int, own: list[int], open_export) -> tuple[list[int], ...]:
    """Per registered array (the buffer, then the flags): the device pointer of every rank, in
    rank order -- this rank's own, the peers' mapped through ``open_export(handle, offset)``.
    Raises when the ranks registered different sizes."""
    out = tuple([0] * len(entries) for _ in own)
    for r, (er, en, exported) in enumerate(entries):
        if er != r:
            raise ValueError(f"rank {er} answered in slot {r}")
        if en != n:
            raise ValueError(f"rank {er} registered {en} elements, rank {rank} {n}")
        for j, ptr in enumerate(own):
            out[j][r] = ptr if r == rank else open_export(*exported[j])
    return out


class PeerAllReduce:
    """In-place sum of ``buffer`` across the ranks of ``group`` (a ``torch.distributed`` process
    group, any backend: it only carries the IPC handles at construction).

    ``buffer`` is a contiguous float32 CUDA tensor, 16-byte aligned, of the same size on every
    rank; it stays registered until :meth:`close` (register one buffer once: gradient buckets are
    ranges of it, see :meth:`__call__`).  Calling the object launches the reduction on ``stream``
    (default: the current stream) after the work already queued there; every rank must make the
    same calls.  A peer that never arrives makes the launch give up after about a second:
    :meth:`check` then raises.
    """

    def __init__(self, buffer: torch.Tensor, group=None, ctas: int = 64):
        import torch.distributed as dist

        if not buffer.is_cuda or buffer.dtype != torch.float32 or not buffer.is_contiguous():
            raise ValueError("buffer must be a contiguous float32 CUDA tensor")
        if buffer.data_ptr() % 16:
            raise ValueError("buffer must be 16-byte aligned")
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one node)")
        self.buffer = buffer
        self.n = buffer.numel()
        self.ctas = int(ctas)
        lib = N.lib()
        self._lib = lib
        self.flags = torch.zeros(lib.rfdetr_allreduce_flag_bytes() // 4, dtype=torch.int32, device=buffer.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=buffer.device)
        self.epoch = 0
        self._opened: list[int] = []
        self._bufs = self._flags = None
        own = [buffer.data_ptr(), self.flags.data_ptr()]
        if self.world == 1:
            self._bufs, self._flags = ((ctypes.c_void_p * 1)(p) for p in own)
            return
        entries = exchange_exports(group, self.rank, self.world, self.n, [self._export(p) for p in own])
        bufs, flags = peer_pointers(entries, self.rank, self.n, own, self._open)
        self._bufs = (ctypes.c_void_p * self.world)(*bufs)
        self._flags = (ctypes.c_void_p * self.world)(*flags)

    def _export(self, ptr: int) -> tuple[bytes, int]:
        handle = ctypes.create_string_buffer(self._lib.rfdetr_ipc_handle_bytes())
        offset = ctypes.c_size_t(0)
        N.check(self._lib.rfdetr_ipc_get_handle(ptr, handle, ctypes.byref(offset)), "rfdetr_ipc_get_handle")
        return handle.raw, int(offset.value)

    def _open(self, handle: bytes, offset: int) -> int:
        base = ctypes.c_void_p(0)
        N.check(self._lib.rfdetr_ipc_open_handle(handle, ctypes.byref(base)), "rfdetr_ipc_open_handle")
        self._opened.append(int(base.value))
        return int(base.value) + int(offset)

    def __call__(self, stream=None, offset: int = 0, count: int | None = None) -> None:
        """Sums elements ``[offset, offset + count)`` of the buffer (default: all of it) across the
        ranks; ``offset`` a multiple of 4 (16-byte alignment).  Every rank makes the same calls in
        the same order."""
        if self._bufs is None:
            raise RuntimeError("PeerAllReduce is closed")
        count = self.n - offset if count is None else int(count)
        if offset < 0 or count < 0 or offset + count > self.n or offset % 4:
            raise ValueError(f"range [{offset}, {offset + count}) of a {self.n}-element buffer (offset a multiple of 4)")
        if self.world == 1 or count == 0:
            return
        self.epoch = (self.epoch % 0xFFFFFFFF) + 1
        s = (stream if stream is not None else torch.cuda.current_stream(self.buffer.device)).cuda_stream
        bufs = (ctypes.c_void_p * self.world)(*[b + 4 * offset for b in self._bufs])
        N.check(self._lib.rfdetr_allreduce_sum_f32(s, bufs, self._flags, self.rank, self.world, count, self.epoch,
                                                   self.ctas, self.status.data_ptr()),
                "rfdetr_allreduce_sum_f32")

    def check(self) -> None:
        """Raises if a launch gave up waiting for a peer (reads the device status word)."""
        N.check_device_status(self.status, "rfdetr_allreduce_sum_f32")

    def close(self) -> None:
        """Unmaps the peers' allocations (after this rank's launches have completed)."""
        if self._bufs is None:
            return
        torch.cuda.synchronize(self.buffer.device)
        for base in self._opened:
            N.check(self._lib.rfdetr_ipc_close_handle(base), "rfdetr_ipc_close_handle")
        self._opened = []
        self._bufs = self._flags = None
