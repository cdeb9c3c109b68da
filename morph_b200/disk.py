"""DiskState.update arithmetic on device-resident optimizer state.

``DeviceDiskState`` keeps, per parameter name, the reference's ``(3, size)``
FP32 layout ``[w; m; v]`` (streamtrain/disk.py:68-69, 206) in GPU memory and
offers the store interface the engines call: ``update(name, gradient, step,
lr, clip, chunk_elements)`` (disk.py:203 callers: disk.py:464,
sparse_disk.py:133, single_pass.py:179), ``read_into(name, destination)`` and
``weight(name)``. File I/O, journals and the ``fault`` hook stay with the
caller; ``update`` only does the arithmetic, in one kernel launch per call.

``update_rows`` is the row-sparse variant: only the listed rows of a 2-D entry
are read and written (kernel 3).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib


def disk_host_scalars(lr: float, step: int, clip: float = 1.0, loss_scale: float = 1.0) -> _lib.HostScalars:
    """Float32 step scalars of DiskState.update, derived as disk.py:210-215 does:
    lerp weight .1, beta2 .999, addcmul value .001, ``math.sqrt(1 - .999**step)``,
    eps 1e-8, ``1 - lr*.01`` and ``-lr / (1 - .9**step)``; the gradient is
    ``g / loss_scale * clip`` (sparse_disk.py:107, disk.py:210)."""
    f = lambda x: float(np.float32(x))  # noqa: E731
    return _lib.HostScalars(f(1 - lr * .01), f(.1), f(.999), f(.001), f(math.sqrt(1 - .999 ** step)), f(1e-8),
                            f(-lr / (1 - .9 ** step)), f(loss_scale), f(clip))


def _check_plane(t: torch.Tensor, name: str):
    if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError(f"{name}: state must be a contiguous float32 CUDA tensor")


class DeviceDiskState:
    """Per-name ``(3, size)`` FP32 ``[w; m; v]`` planes on one CUDA device."""

    def __init__(self, planes: dict[str, torch.Tensor], shapes: dict[str, tuple] | None = None):
        self.planes = {}
        self.shapes = {}
        for name, t in planes.items():
            if t.dim() != 2 or t.shape[0] != 3:
                raise ValueError(f"{name}: expected a (3, size) tensor")
            _check_plane(t, name)
            self.planes[name] = t
            self.shapes[name] = tuple(shapes[name]) if shapes and name in shapes else (t.shape[1],)
        self.device = next(iter(self.planes.values())).device if self.planes else None
        self._err = None

    @classmethod
    def from_model(cls, model: torch.nn.Module, device="cuda"):
        """Masters from the model's parameters, moments zero (DiskState.create with source=model)."""
        planes, shapes = {}, {}
        for name, p in model.named_parameters():
            t = torch.zeros(3, p.numel(), dtype=torch.float32, device=device)
            t[0].copy_(p.detach().reshape(-1))
            planes[name] = t
            shapes[name] = tuple(p.shape)
        return cls(planes, shapes)

    # -- reads ---------------------------------------------------------------------
    def read_into(self, name: str, destination: torch.Tensor) -> None:
        destination.reshape(-1).copy_(self.planes[name][0])

    def weight(self, name: str) -> torch.Tensor:
        return self.planes[name][0].reshape(self.shapes[name]).clone()

    # -- updates -------------------------------------------------------------------
    def update(self, name, gradient, step, lr, clip, chunk_elements=1048576, loss_scale=1.0, out=None):
        """One DiskState.update step of entry ``name`` (``chunk_elements`` only
        bounded host memory in the reference and is accepted for signature
        compatibility). ``gradient`` is a CUDA FP32/FP16/BF16 tensor of the
        entry's size; ``out`` (optional F16/BF16 tensor) receives the new w."""
        planes = self.planes[name]
        size = planes.shape[1]
        g = gradient.reshape(-1)
        if not g.is_cuda or g.device != planes.device or g.numel() != size or not g.is_contiguous():
            raise ValueError(f"{name}: gradient must be a contiguous CUDA tensor of {size} elements")
        s = disk_host_scalars(float(lr), int(step), float(clip), float(loss_scale))
        odt = _lib.MB_NONE
        optr = None
        if out is not None:
            odt = _lib.dtype_code(out.dtype)
            optr = _lib.ptr(out)
        with torch.cuda.device(planes.device):
            _lib.check(_lib.lib().mb_adamw_update(
                _lib.ptr(planes[0]), _lib.ptr(planes[1]), _lib.ptr(planes[2]), _lib.ptr(g), _lib.dtype_code(g.dtype),
                optr, odt, size, ctypes.byref(s), _lib.stream_handle()), f"update {name}")

    def update_rows(self, name, index, grads, step, lr, clip=1.0, loss_scale=1.0, check=True):
        """Lazy row-sparse update of a 2-D entry: rows ``index`` (int64 CUDA
        tensor, sorted unique in the reference's use) take one DiskState.update
        step with ``grads[r]`` for row ``index[r]``; other rows are untouched.
        With ``check`` an out-of-range index raises IndexError after the launch
        (in-range rows are updated); without it the flag is left for ``errors()``."""
        planes = self.planes[name]
        rows, cols = self.shapes[name]
        if index.dtype != torch.int64 or not index.is_cuda or index.dim() != 1 or not index.is_contiguous():
            raise ValueError("index must be a 1-D contiguous int64 CUDA tensor")
        k = index.numel()
        if grads.shape != (k, cols) or not grads.is_cuda or not grads.is_contiguous():
            raise ValueError(f"grads must be a contiguous CUDA tensor of shape ({k}, {cols})")
        if self._err is None or self._err.device != planes.device:
            self._err = torch.zeros(1, dtype=torch.int32, device=planes.device)
        s = disk_host_scalars(float(lr), int(step), float(clip), float(loss_scale))
        with torch.cuda.device(planes.device):
            _lib.check(_lib.lib().mb_sparse_rows_update(
                _lib.ptr(planes[0]), _lib.ptr(planes[1]), _lib.ptr(planes[2]), rows, cols, _lib.ptr(index), k,
                _lib.ptr(grads), _lib.dtype_code(grads.dtype), ctypes.byref(s), _lib.ptr(self._err),
                _lib.stream_handle()), f"update_rows {name}")
        if check:
            self.errors()

    def errors(self) -> None:
        """Raise IndexError (and clear the flag) if a row index was out of range."""
        if self._err is not None and int(self._err.item()):
            self._err.zero_()
            raise IndexError("row index out of range")


def cast_f32(src: torch.Tensor, dtype: torch.dtype, export_check: bool = False) -> torch.Tensor:
    """FP32 -> FP16/BF16 copy (round to nearest even). With ``export_check``
    (FP16 only) it raises ValueError like streamtrain/export.py:33 when a value
    is nonfinite or exceeds 65504."""
    if not src.is_cuda or src.dtype != torch.float32 or not src.is_contiguous():
        raise ValueError("src must be a contiguous float32 CUDA tensor")
    dst = torch.empty(src.shape, dtype=dtype, device=src.device)
    err = torch.zeros(1, dtype=torch.int32, device=src.device) if export_check else None
    with torch.cuda.device(src.device):
        _lib.check(_lib.lib().mb_cast_f32(_lib.ptr(src), _lib.ptr(dst), _lib.dtype_code(dtype), src.numel(),
                                          int(export_check), _lib.ptr(err) if err is not None else None,
                                          _lib.stream_handle()), "cast")
    if export_check and int(err.item()):
        raise ValueError('weights cannot be represented by finite FP16')
    return dst


class _AccWorkspace:
    """Per-device scratch of mb_grad_accumulate's statistics (zeroed once)."""

    def __init__(self):
        self.buf = {}

    def get(self, device):
        t = self.buf.get(device)
        if t is None:
            t = self.buf[device] = torch.zeros(_lib.lib().mb_accumulate_workspace_bytes(), dtype=torch.uint8,
                                               device=device)
        return t


_ACC_WS = _AccWorkspace()


def norm_record(device) -> torch.Tensor:
    """A zeroed device record {sum of squares, nonfinite} (2 x FP64) for accumulate_."""
    return torch.zeros(2, dtype=torch.float64, device=device)


def accumulate_(acc: torch.Tensor, gradient: torch.Tensor, loss_scale: float = 1.0, *, first: bool = False,
                record: torch.Tensor = None) -> torch.Tensor:
    """acc.add_(gradient.float() / loss_scale) on the device, the microbatch
    accumulation of streamtrain/sparse_disk.py:82-110 (``first=True`` is the
    window's zero_() followed by the first add). With ``record`` (from
    ``norm_record``) the same pass adds the updated acc's FP64 sum of squares and
    a nonfinite flag to it, the statistics of the norm pass
    (sparse_disk.py:119-120). Calls on one device must share one stream."""
    if not acc.is_cuda or acc.dtype != torch.float32 or not acc.is_contiguous():
        raise ValueError("acc must be a contiguous float32 CUDA tensor")
    if gradient.shape != acc.shape or gradient.device != acc.device or not gradient.is_contiguous():
        raise ValueError("gradient must be contiguous, on acc's device and of acc's shape")
    if record is not None and (record.dtype != torch.float64 or record.numel() != 2 or record.device != acc.device):
        raise ValueError("record must be a 2-element float64 tensor on acc's device")
    with torch.cuda.device(acc.device):
        _lib.check(_lib.lib().mb_grad_accumulate(
            _lib.ptr(acc), _lib.ptr(gradient), _lib.dtype_code(gradient.dtype), acc.numel(), float(loss_scale),
            int(bool(first)), None if record is None else _lib.ptr(record),
            _lib.ptr(_ACC_WS.get(acc.device)) if record is not None else None, _lib.stream_handle()),
            "grad_accumulate")
    return acc


def record_norm(record: torch.Tensor) -> float:
    """sqrt of the accumulated sum of squares (inf/nan when a value was nonfinite)."""
    s, bad = record.tolist()
    return float("nan") if bad else math.sqrt(s)
