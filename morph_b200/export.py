"""FP16 export of FP32 masters held on the GPU (the device side of
streamtrain/export.py:16-43).

``export_fp16`` writes the bytes export.py writes for one tensor (little-endian
FP16, round to nearest even) to a binary file handle, checking every
``chunk_elements`` chunk for nonfinite values or |x| > 65504 like export.py:33
and raising the same ValueError after writing the chunks before the first bad
one. The GPU converts staging chunks straight into two pinned host buffers
(kernel ``k_export_f16`` through the buffers' device mapping) while the host
writes and hashes the previous one. The manifest, fsync, locking and file
naming stay with the caller.
"""
from __future__ import annotations

import torch

from . import _lib

_ERR = 'weights cannot be represented by finite FP16'


def export_fp16(src: torch.Tensor, handle, chunk_elements: int = 1048576, digest=None,
                staging_elements: int = 1 << 24) -> int:
    """Write ``src`` (FP32, CUDA) as FP16 to ``handle``; update ``digest``
    (hashlib object, optional) with the same bytes. Returns the bytes written."""
    if not src.is_cuda or src.dtype != torch.float32:
        raise ValueError("src must be a float32 CUDA tensor")
    if chunk_elements <= 0:
        raise ValueError("chunk_elements must be positive")
    flat = src.contiguous().reshape(-1)
    n = flat.numel()
    if n == 0:
        return 0
    stage = max(chunk_elements, staging_elements // chunk_elements * chunk_elements)
    stage = min(stage, -(-n // chunk_elements) * chunk_elements)
    dev = flat.device
    bufs = [torch.empty(stage, dtype=torch.float16, pin_memory=True) for _ in range(2)]
    flags = torch.empty(2, dtype=torch.int64, device=dev)
    flags_host = torch.empty(2, dtype=torch.int64, pin_memory=True)
    events = [torch.cuda.Event() for _ in range(2)]
    n_stage = -(-n // stage)
    lib = _lib.lib()

    def launch(j):
        b, lo = j % 2, j * stage
        cnt = min(stage, n - lo)
        flags[b].fill_(-1)  # UINT64_MAX: no bad element yet
        _lib.check(lib.mb_export_f16(_lib.ptr(flat[lo:]), cnt, _lib.ptr(bufs[b]), _lib.ptr(flags[b:]),
                                     _lib.stream_handle()), "export_f16")
        flags_host[b].copy_(flags[b], non_blocking=True)
        events[b].record()

    written = 0
    with torch.cuda.device(dev):
        launch(0)
        for j in range(n_stage):
            if j + 1 < n_stage:
                launch(j + 1)  # its buffer was written out in iteration j - 1
            b, lo = j % 2, j * stage
            cnt = min(stage, n - lo)
            events[b].synchronize()
            bad = int(flags_host[b])
            good = cnt if bad < 0 else (lo + bad) // chunk_elements * chunk_elements - lo
            if good > 0:
                data = memoryview(bufs[b][:good].numpy()).cast("B")
                handle.write(data)
                if digest is not None:
                    digest.update(data)
                written += 2 * good
            if bad >= 0:
                torch.cuda.current_stream(dev).synchronize()  # the launched next stage, before its buffers go
                raise ValueError(_ERR)
    return written
