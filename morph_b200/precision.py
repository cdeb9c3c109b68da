"""Dynamic FP16 loss scaling with the state resident on the GPU.

Drop-in for ``DynamicLossScale`` of streamtrain/precision.py:6-17 (same
constructor, attributes, ``overflow()``, ``success()``, ``state_dict()`` and
``load_state_dict()``, same exceptions). The scale and good-step counter live
in a device ``mb_step_state`` record, so an optimizer that is given this object
(``AdamW(..., loss_scale=scaler)``) decides skip-and-back-off or success on the
device without a host round trip. Reading an attribute synchronises with the
current stream and returns the device value.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


class DynamicLossScale:
    """Loss scale S: gradients arrive multiplied by S and are divided by it
    before the update. On an overflow step the update is skipped and S halves
    (never below 1; at 1 the overflow raises FloatingPointError and leaves the
    state unchanged). After ``growth_interval`` good steps S doubles, capped
    at 65536."""

    def __init__(self, scale=128., growth_interval=2000, device=None):
        self.device = (torch.device(device) if device is not None
                       else torch.device("cuda", torch.cuda.current_device()))
        st = _lib.StepState()
        _lib.check(_lib.lib().mb_step_state_init(ctypes.byref(st), float(scale), int(growth_interval)),
                   "DynamicLossScale")
        self._buf = torch.zeros(ctypes.sizeof(_lib.StepState), dtype=torch.uint8, device=self.device)
        self._write(st)

    # -- device record ------------------------------------------------------
    @property
    def state_buffer(self) -> torch.Tensor:
        """The 96-byte device ``mb_step_state`` shared with attached optimizers."""
        return self._buf

    def _read(self) -> _lib.StepState:
        host = self._buf.cpu()
        return _lib.StepState.from_buffer_copy(host.numpy().tobytes())

    def _write(self, st: _lib.StepState) -> None:
        src = torch.frombuffer(bytearray(bytes(st)), dtype=torch.uint8)
        self._buf.copy_(src)

    # -- reference attributes -------------------------------------------------
    @property
    def scale(self) -> float:
        return float(self._read().scale)

    @scale.setter
    def scale(self, value) -> None:
        st = self._read()
        st.scale = float(value)
        self._write(st)

    @property
    def good_steps(self) -> int:
        return int(self._read().good_steps)

    @good_steps.setter
    def good_steps(self, value) -> None:
        st = self._read()
        st.good_steps = int(value)
        self._write(st)

    @property
    def growth_interval(self) -> int:
        return int(self._read().growth_interval)

    @growth_interval.setter
    def growth_interval(self, value) -> None:
        st = self._read()
        st.growth_interval = int(value)
        self._write(st)

    # -- reference methods (host-driven transitions) ---------------------------
    def overflow(self) -> None:
        st = self._read()
        if st.scale <= 1:
            raise FloatingPointError('FP16 overflow at minimum loss scale; state unchanged')
        st.scale = max(1., st.scale / 2)
        st.good_steps = 0
        self._write(st)

    def success(self) -> None:
        st = self._read()
        st.good_steps += 1
        if st.good_steps >= st.growth_interval:
            st.scale = min(st.scale * 2, 65536.)
            st.good_steps = 0
        self._write(st)

    def state_dict(self) -> dict:
        st = self._read()
        return dict(scale=float(st.scale), good_steps=int(st.good_steps), growth_interval=int(st.growth_interval))

    def load_state_dict(self, state) -> None:
        st = self._read()
        st.scale = float(state['scale'])
        st.good_steps = int(state['good_steps'])
        st.growth_interval = int(state['growth_interval'])
        self._write(st)

    # -- device-side results of the last fused step ---------------------------
    def last_step(self) -> dict:
        """Outcome of the last finalized optimizer step that used this scaler."""
        st = self._read()
        return dict(skipped=bool(st.skip), status=int(st.status), norm=float(st.norm),
                    step_scale=float(st.step_scale), clip_coef=float(st.clip_coef),
                    steps_applied=int(st.steps_applied), steps_skipped=int(st.steps_skipped))


def pack_fp8(value: torch.Tensor, block_size: int = 256):
    """streamtrain/precision.py:24-30 on the GPU: E4M3FN codes (uint8, one per
    element) and FP32 per-256-block scales of ``value`` (any shape, on a CUDA
    device, converted to FP32 first)."""
    if block_size != 256:
        raise ValueError("the B200 kernels use 256-element blocks")
    flat = value.detach().float().contiguous().reshape(-1)
    if not flat.is_cuda:
        raise ValueError("pack_fp8 expects a CUDA tensor")
    n = flat.numel()
    codes = torch.empty(n, dtype=torch.uint8, device=flat.device)
    scales = torch.empty((n + 255) // 256, dtype=torch.float32, device=flat.device)
    with torch.cuda.device(flat.device):
        _lib.check(_lib.lib().mb_fp8_pack(_lib.ptr(flat), n, _lib.ptr(codes), _lib.ptr(scales),
                                          _lib.stream_handle()), "fp8_pack")
    return codes, scales


def unpack_fp8(encoded: torch.Tensor, scales: torch.Tensor, dtype=torch.float16, block_size: int = 256):
    """streamtrain/precision.py:33-37 on the GPU: values = code * scale, rounded
    to ``dtype`` (float16, bfloat16 or float32), flat."""
    if block_size != 256:
        raise ValueError("the B200 kernels use 256-element blocks")
    if not encoded.is_cuda or encoded.dtype != torch.uint8 or not encoded.is_contiguous():
        raise ValueError("encoded must be contiguous uint8 on a CUDA device")
    n = encoded.numel()
    sc = scales.contiguous().float()
    if sc.numel() != (n + 255) // 256:
        raise ValueError("one scale per 256-element block expected")
    out = torch.empty(n, dtype=dtype, device=encoded.device)
    with torch.cuda.device(encoded.device):
        _lib.check(_lib.lib().mb_fp8_unpack(_lib.ptr(encoded), _lib.ptr(sc), n, _lib.ptr(out),
                                            _lib.dtype_code(dtype), _lib.stream_handle()), "fp8_unpack")
    return out


def fp8_eligible(name: str) -> bool:
    """streamtrain/precision.py:20-21: the SwiGLU projections may travel as FP8."""
    return any(name.endswith(suffix) for suffix in ('ffn.gate.weight', 'ffn.up.weight', 'ffn.down.weight'))
