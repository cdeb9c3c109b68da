"""DiskState.update on the reference's state files with the arithmetic on the GPU.

The reference keeps each parameter's optimizer state in one file of FP32
planes ``(3, size)`` = ``[w; m; v]`` (streamtrain/disk.py:68-69) and updates it
in place chunk by chunk on the CPU (disk.py:203-223): read the chunk's three
planes, apply the AdamW step, write them back, call the
``fault('partial_state_write')`` hook, and finally flush and fsync the file.

``GpuDiskUpdater.update`` keeps the file, its layout, the per-chunk write order,
the fault hook, the flush and the fsync, and moves the arithmetic to the GPU
through two pinned staging windows:

  host:      read window j's planes from the file into pinned buffer j % 2;
  h2d:       copy them (and window j's gradient slice, if it is on the host)
             to device window j % 2;
  compute:   kernel 1 (``mb_adamw_update``) on the device window;
  d2h:       copy the planes back into the pinned buffer;
  host:      write the planes back to the file chunk by chunk (chunk_elements,
             as the reference does), calling the fault hook after each chunk.

The host reads window j + 1 while the GPU processes window j, so the file I/O
(the reference's bound) overlaps the transfers and the arithmetic. ``install``
swaps a store's ``update`` for the GPU one, so an engine that calls
``store.update(name, gradient, step, lr, clip)`` (disk.py:464,
sparse_disk.py:133, single_pass.py:179) uses it unchanged.
"""
from __future__ import annotations

import ctypes
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from . import _lib
from .disk import disk_host_scalars


_POOL = None


def _pool():
    """Host copy threads (numpy releases the GIL while copying)."""
    global _POOL
    if _POOL is None:
        _POOL = ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1)))
    return _POOL


def _parallel_copy(dst: np.ndarray, src: np.ndarray, pieces: int = 8) -> None:
    """dst[...] = src for (3, n) arrays, split by columns over the host threads."""
    n = dst.shape[1]
    step = max(1, -(-n // pieces))
    if n <= step or n < (1 << 16):
        np.copyto(dst, src)
        return
    futures = [_pool().submit(np.copyto, dst[:, a:a + step], src[:, a:a + step]) for a in range(0, n, step)]
    for f in futures:
        f.result()


class GpuDiskUpdater:
    """GPU arithmetic for a store with ``root`` (directory), ``entries``
    (name -> {'file', 'size'}) and optionally ``fault(label)``."""

    def __init__(self, store, device="cuda", window_elements: int = 1 << 24):
        self.store = store
        self.device = torch.device(device)
        self.window = int(window_elements)
        self._alloc(self.window)
        self.gdev = [None, None]
        self.h2d = torch.cuda.Stream(device=self.device)
        self.d2h = torch.cuda.Stream(device=self.device)
        self.loaded = [torch.cuda.Event() for _ in range(2)]
        self.updated = [torch.cuda.Event() for _ in range(2)]
        self.done = [torch.cuda.Event() for _ in range(2)]

    def _alloc(self, elements):
        # flat [3 * window] buffers, viewed as a contiguous (3, n) block per window
        self.capacity = elements
        self.host = [torch.empty(3 * elements, dtype=torch.float32, pin_memory=True) for _ in range(2)]
        self.dev = [torch.empty(3 * elements, dtype=torch.float32, device=self.device) for _ in range(2)]

    def _fault(self, label):
        fault = getattr(self.store, "fault", None)
        if fault is not None:
            fault(label)

    def update(self, name, gradient, step, lr, clip, chunk_elements=1048576):
        """disk.py:203-223 for entry ``name``; ``gradient`` (FP32/FP16/BF16, host
        or CUDA) has the entry's size."""
        entry = self.store.entries[name]
        size = int(entry["size"])
        path = os.path.join(str(self.store.root), entry["file"])
        mapped = np.memmap(path, dtype=np.float32, mode="r+", shape=(3, size))
        self._run(name, mapped, [mapped], gradient, step, lr, clip, chunk_elements)
        _flush_and_fsync(mapped, path)

    def update_cached(self, name, values, gradient, step, lr, clip, chunk_elements=1048576):
        """The cache-hit path of CachedDiskState.update (state_cache.py:111-137):
        the entry's planes come from ``values`` (its RAM copy, (3, size) FP32)
        and every chunk is written to both ``values`` and the file before the
        fault hook, then the file is flushed and fsynced."""
        entry = self.store.entries[name]
        size = int(entry["size"])
        if values.shape != (3, size) or values.dtype != np.float32:
            raise ValueError(f"{name}: cached planes must be float32 of shape (3, {size})")
        path = os.path.join(str(self.store.root), entry["file"])
        mapped = np.memmap(path, dtype=np.float32, mode="r+", shape=(3, size))
        self._run(name, values, [values, mapped], gradient, step, lr, clip, chunk_elements)
        _flush_and_fsync(mapped, path)

    def _run(self, name, source, sinks, gradient, step, lr, clip, chunk_elements):
        """Stream the (3, size) planes of ``source`` through the device windows
        and write the updated planes to every array of ``sinks`` chunk by chunk."""
        size = int(source.shape[1])
        g = gradient.reshape(-1)
        if g.numel() != size:
            raise ValueError(f"{name}: gradient must have {size} elements")
        if g.is_cuda and g.device != self.device:
            raise ValueError(f"{name}: gradient is on {g.device}, the updater on {self.device}")
        g = g.contiguous()
        s = disk_host_scalars(float(lr), int(step), float(clip))
        # windows hold whole reference chunks, so writes and fault calls fall where the reference's do
        W = max(chunk_elements, self.window // chunk_elements * chunk_elements)
        if W > self.capacity:
            torch.cuda.synchronize(self.device)
            self._alloc(W)
        n_win = -(-size // W)
        if n_win == 0:
            return
        lib = _lib.lib()
        compute = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(compute)  # the gradient is produced on the caller's stream
        self.h2d.wait_event(start)

        def stage(j):
            """Read window j from the source and enqueue its copies and update."""
            b, lo = j % 2, j * W
            n = min(W, size - lo)
            host = self.host[b][:3 * n].view(3, n)
            dev = self.dev[b][:3 * n].view(3, n)
            _parallel_copy(host.numpy(), source[:, lo:lo + n])  # buffer b was written back already
            with torch.cuda.stream(self.h2d):
                if j >= 2:
                    self.h2d.wait_event(self.done[b])  # device window b's copy-back is complete
                dev.copy_(host, non_blocking=True)
                if g.is_cuda:
                    gw = g[lo:lo + n]
                else:
                    if self.gdev[b] is None or self.gdev[b].numel() < W or self.gdev[b].dtype != g.dtype:
                        self.gdev[b] = torch.empty(W, dtype=g.dtype, device=self.device)
                    gw = self.gdev[b][:n]
                    gw.copy_(g[lo:lo + n], non_blocking=True)
                self.loaded[b].record(self.h2d)
            compute.wait_event(self.loaded[b])
            with torch.cuda.device(self.device):
                _lib.check(lib.mb_adamw_update(
                    _lib.ptr(dev[0]), _lib.ptr(dev[1]), _lib.ptr(dev[2]), _lib.ptr(gw), _lib.dtype_code(g.dtype),
                    None, _lib.MB_NONE, n, ctypes.byref(s), _lib.stream_handle(compute)), f"update {name}")
            self.updated[b].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.updated[b])
                host.copy_(dev, non_blocking=True)
                self.done[b].record(self.d2h)

        def write_back(j):
            b, lo = j % 2, j * W
            n = min(W, size - lo)
            self.done[b].synchronize()
            host = self.host[b][:3 * n].view(3, n).numpy()
            for c0 in range(0, n, chunk_elements):  # the reference's write and fault granularity
                c1 = min(c0 + chunk_elements, n)
                for sink in sinks:
                    _parallel_copy(sink[:, lo + c0:lo + c1], host[:, c0:c1])
                self._fault('partial_state_write')

        stage(0)
        for j in range(n_win):
            if j + 1 < n_win:
                stage(j + 1)  # window (j + 1) % 2 was written back in iteration j - 1
            write_back(j)
        compute.wait_event(self.done[(n_win - 1) % 2])


def _flush_and_fsync(mapped, path):
    mapped.flush()
    del mapped
    fd = os.open(path, os.O_RDWR)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def install(store, device="cuda", window_elements: int = 1 << 24) -> GpuDiskUpdater:
    """Route ``store.update`` through a GpuDiskUpdater; returns the updater."""
    updater = GpuDiskUpdater(store, device, window_elements)
    store.update = updater.update
    return updater


def patch_class(cls, device="cuda", window_elements: int = 1 << 24):
    """Route ``cls.update`` (a DiskState-like class: instances have ``root``,
    ``entries`` and ``fault``) through one GpuDiskUpdater per instance, created
    on first use. For engines that build their store internally (e.g.
    streamtrain/delta_cycle.py:130-156), call this once before they run.
    Returns a function that restores the original method."""
    original = cls.update

    def update(self, name, gradient, step, lr, clip, chunk_elements=1048576):
        updater = self.__dict__.get("_mb_gpu_updater")
        if updater is None:
            updater = self.__dict__["_mb_gpu_updater"] = GpuDiskUpdater(self, device, window_elements)
        return updater.update(name, gradient, step, lr, clip, chunk_elements)

    cls.update = update

    def restore():
        cls.update = original
    return restore


def patch_cached_class(cls, device="cuda", window_elements: int = 1 << 24):
    """The same for a CachedDiskState-like class (state_cache.py:103-140: a
    bounded RAM cache ``_cache`` of (3, size) planes under ``_cache_lock``,
    counters in ``_cache_stats``, ``_drop`` on failure): a cache hit updates the
    RAM copy and the file from the GPU (``update_cached``), a miss runs the
    file path. Returns a function that restores the original method."""
    original = cls.update

    def update(self, name, gradient, step, lr, clip, chunk_elements=1048576):
        updater = self.__dict__.get("_mb_gpu_updater")
        if updater is None:
            updater = self.__dict__["_mb_gpu_updater"] = GpuDiskUpdater(self, device, window_elements)
        with self._cache_lock:
            values = self._cache.get(name)
            if values is None:
                self._cache_stats["misses"] += 1
                return updater.update(name, gradient, step, lr, clip, chunk_elements)
            self._cache.move_to_end(name)
            self._cache_stats["hits"] += 1
            self._cache_stats["estimated_bytes_avoided"] += values.nbytes
            try:
                updater.update_cached(name, values, gradient, step, lr, clip, chunk_elements)
            except BaseException:
                self._drop(name)
                raise

    cls.update = update

    def restore():
        cls.update = original
    return restore
