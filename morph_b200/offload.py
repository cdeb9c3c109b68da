"""Row-sparse AdamW on optimizer state held in pinned host memory (kernel 5).

``OffloadedRowTable`` keeps a [rows, cols] table's FP32 w, m, v in pinned,
device-mapped host memory (the bounded-VRAM role of the reference's CPU/disk
masters, streamtrain/disk.py:287-359) and updates the rows named by a sorted
index list through two 256 MiB device windows: gathers on an H2D stream,
kernel-1 updates on the compute stream, scatters on a D2H stream, all ordered
by events (the ping-pong Slot protocol of streamtrain/engine.py:60-163). The
arithmetic is DiskState.update's (streamtrain/disk.py:207-215) with the table's
step clock, as the conditional AdamW of streamtrain/sparse_disk.py:122-138
applies it.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .disk import disk_host_scalars


class OffloadedRowTable:
    def __init__(self, rows: int, cols: int, init=None, device="cuda", window_bytes: int = 256 << 20):
        self.rows, self.cols = int(rows), int(cols)
        self.device = torch.device(device)
        self.w = torch.empty(self.rows, self.cols, dtype=torch.float32, pin_memory=True)
        self.m = torch.zeros(self.rows, self.cols, dtype=torch.float32, pin_memory=True)
        self.v = torch.zeros(self.rows, self.cols, dtype=torch.float32, pin_memory=True)
        if init is not None:
            self.w.copy_(torch.as_tensor(init, dtype=torch.float32).reshape(self.rows, self.cols))
        else:
            self.w.zero_()
        self.window_rows = max(1, int(window_bytes) // (3 * self.cols * 4))
        self.windows = [torch.empty(3 * self.window_rows * self.cols, dtype=torch.float32, device=self.device)
                        for _ in range(2)]
        self.h2d = torch.cuda.Stream(device=self.device)
        self.d2h = torch.cuda.Stream(device=self.device)
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def step(self, index: torch.Tensor, grads: torch.Tensor, step: int, lr: float, clip: float = 1.0,
             loss_scale: float = 1.0) -> None:
        """Enqueue one update of rows ``index`` (sorted unique int64, on the device)
        with gradient rows ``grads`` [k, cols] (FP32/FP16/BF16, on the device)."""
        k = index.numel()
        if index.dtype != torch.int64 or not index.is_cuda or not index.is_contiguous():
            raise ValueError("index must be a contiguous int64 CUDA tensor")
        if grads.shape != (k, self.cols) or not grads.is_cuda or not grads.is_contiguous():
            raise ValueError(f"grads must be a contiguous CUDA tensor of shape ({k}, {self.cols})")
        s = disk_host_scalars(float(lr), int(step), float(clip), float(loss_scale))
        with torch.cuda.device(self.device):
            compute = torch.cuda.current_stream()
            _lib.check(_lib.lib().mb_offload_rows_step(
                _lib.ptr(self.w), _lib.ptr(self.m), _lib.ptr(self.v), self.rows, self.cols, _lib.ptr(index), k,
                _lib.ptr(grads), _lib.dtype_code(grads.dtype), ctypes.byref(s), _lib.ptr(self.windows[0]),
                _lib.ptr(self.windows[1]), self.window_rows, _lib.stream_handle(compute),
                _lib.stream_handle(self.h2d), _lib.stream_handle(self.d2h), _lib.ptr(self._err)),
                "offload_rows_step")

    def synchronize(self, timeout: float | None = None) -> None:
        """Wait for every enqueued step; raise IndexError if an index was out of
        range. With ``timeout`` (seconds) the wait is bounded: TimeoutError is
        raised if the steps have not finished by then (they keep running)."""
        stream = torch.cuda.current_stream(self.device)
        if timeout is None:
            stream.synchronize()
        else:
            with torch.cuda.device(self.device):
                _lib.check(_lib.lib().mb_stream_wait(_lib.stream_handle(stream), int(timeout * 1e6)),
                           "offloaded rows still in flight")
        if int(self._err.item()):
            self._err.zero_()
            raise IndexError("row index out of range")


class ShardedRowTable:
    """An offloaded row table sharded by contiguous row blocks over the ranks of
    a process group, one GPU (and its own host link) per rank.

    Rank r owns rows [rows*r/N, rows*(r+1)/N) in its own ``OffloadedRowTable``.
    ``step`` takes the full sorted index list and gradient rows (as every rank
    holds them after the gradient reduction) and updates the contiguous slice of
    the list that falls in this rank's block; the arithmetic per row is exactly
    the unsharded table's, and no collective is needed."""

    def __init__(self, rows: int, cols: int, init=None, device="cuda", window_bytes: int = 256 << 20,
                 process_group=None, table_factory=None):
        import torch.distributed as dist
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.rows, self.cols = int(rows), int(cols)
        self.lo = self.rows * self.rank // self.world
        self.hi = self.rows * (self.rank + 1) // self.world
        block = None if init is None else torch.as_tensor(init).reshape(self.rows, self.cols)[self.lo:self.hi]
        make = table_factory or (lambda r, c, i: OffloadedRowTable(r, c, init=i, device=device,
                                                                  window_bytes=window_bytes))
        self.local = make(self.hi - self.lo, self.cols, block)

    def local_slice(self, index: torch.Tensor):
        """(a, b): the positions of this rank's rows in the sorted index list."""
        bounds = torch.tensor([self.lo, self.hi], dtype=index.dtype, device=index.device)
        a, b = torch.searchsorted(index, bounds).tolist()
        return a, b

    def step(self, index: torch.Tensor, grads: torch.Tensor, step: int, lr: float, clip: float = 1.0,
             loss_scale: float = 1.0) -> int:
        """Update this rank's rows of ``index``; returns how many rows that was."""
        a, b = self.local_slice(index)
        if b > a:
            self.local.step(index[a:b] - self.lo, grads[a:b], step, lr, clip, loss_scale)
        return b - a

    def synchronize(self, timeout: float | None = None) -> None:
        self.local.synchronize(timeout)
