"""TEST INFRASTRUCTURE — CPU parity oracle for MORPH's optimizer-step hot path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker (or as the timed CPU
baseline). The product package ``morph_b200`` never imports it.

The elementwise arithmetic is in ``oracle.c`` (built to ``liboracle.so`` by
``oracle/Makefile``); this module restates the host-side scalar derivations
in Python double precision, exactly as the reference's Python computes them,
and the control logic (loss scale, finiteness gate, clip) line by line.

Reference lines restated (paths inside the MORPH project):
  - ``adamw_scalars``: torch/optim/adam.py ``_single_tensor_adam`` (torch 2.11.0,
    installed file lines 414-547), reached through streamtrain/optimizer.py:40,62
    and morph/training/runner.py:46,101.
  - ``disk_scalars``: streamtrain/disk.py:207-215.
  - ``DynamicLossScale``: streamtrain/precision.py:6-17.
  - ``clip_coef_torch``: torch/nn/utils/clip_grad.py:165-169 as called at
    morph/training/runner.py:100 (``max_norm / t`` is ``t.reciprocal()*max_norm``).
  - ``clip_coef_disk``: streamtrain/disk.py:489.
  - ``orthogonalize``: streamtrain/optimizer.py:13-22.
  - ``partition``-independent Muon step: streamtrain/optimizer.py:52-61.
  - ``grad_accumulate_``: streamtrain/sparse_disk.py:82-110 (window zeroed, then
    ``destination.add_(g.float() / loss_scale)`` per microbatch).
  - ``export_f16_chunks``: streamtrain/export.py:30-35 (chunked check and cast).
  - ``pack_fp8`` / ``unpack_fp8``: streamtrain/precision.py:20-37.

Parity pin: tests/test_oracle_cpu.py checks this oracle against golden vectors
produced by running the reference itself (tests/golden/make_golden.py) and
against the installed torch AdamW live.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

F32, F16, BF16 = 0, 1, 2


def build() -> str:
    """Compile liboracle.so in place (gcc, no reference sources involved)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "liboracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        p, i64, f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
        L.orc_adamw.argtypes = [p, p, p, p, i64, p]
        L.orc_grad_prepare.argtypes = [p, ctypes.c_int, i64, f, f, p]
        L.orc_sumsq.argtypes = [p, i64, p]
        L.orc_sumsq.restype = ctypes.c_double
        for name in ("orc_f16_to_f32", "orc_bf16_to_f32", "orc_f32_to_f16", "orc_f32_to_bf16"):
            getattr(L, name).argtypes = [p, p, i64]
        L.orc_export_f16.argtypes = [p, p, i64]
        L.orc_export_f16.restype = ctypes.c_int
        L.orc_sparse_rows.argtypes = [p, p, p, i64, i64, p, i64, p, p]
        L.orc_sparse_rows.restype = ctypes.c_int
        L.orc_muon_momentum.argtypes = [p, p, p, i64, f, f]
        L.orc_muon_apply.argtypes = [p, p, i64, f, f, f]
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return ctypes.c_void_p(a.ctypes.data)


class Scalars(ctypes.Structure):
    _fields_ = [(n, ctypes.c_float) for n in ("cwd", "omb1", "b2", "omb2", "bc2s", "eps", "nss")]


# ------------------------------------------------------------ scalar rules --

def adamw_scalars(lr, beta1, beta2, eps, weight_decay, step) -> Scalars:
    """Scalars of one torch AdamW step at clock ``step`` (after increment).

    adam.py: ``param.mul_(1 - lr * weight_decay)``; ``exp_avg.lerp_(grad, 1 - beta1)``;
    ``exp_avg_sq.mul_(beta2).addcmul_(grad, grad, value=1 - beta2)``;
    ``bias_correction1 = 1 - beta1 ** step``; ``bias_correction2 = 1 - beta2 ** step``;
    ``step_size = lr / bias_correction1``; ``bias_correction2_sqrt = bias_correction2 ** 0.5``;
    ``denom = (exp_avg_sq.sqrt() / bias_correction2_sqrt).add_(eps)``;
    ``param.addcdiv_(exp_avg, denom, value=-step_size)``. ``step`` is a Python float
    there (``_get_value`` of a float32 tensor).
    """
    step = float(step)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    return Scalars(1 - lr * weight_decay, 1 - beta1, beta2, 1 - beta2, bc2 ** 0.5, eps, -(lr / bc1))


def disk_scalars(lr, step) -> Scalars:
    """Scalars of DiskState.update (disk.py:211-215): fixed beta1 .9 (lerp .1),
    beta2 .999, eps 1e-8, weight decay .01; ``math.sqrt`` (not ``** 0.5``)."""
    return Scalars(1 - lr * .01, .1, .999, .001, math.sqrt(1 - .999 ** step), 1e-8,
                   -lr / (1 - .9 ** step))


def bc_table(beta1, beta2, length, kind="torch"):
    """Double bias corrections per clock t = 0..length-1: (1 - b1**t, sqrt-ish(1 - b2**t)).
    ``kind='torch'`` uses ``** 0.5`` (adam.py), ``'disk'`` uses ``math.sqrt`` (disk.py:213)."""
    out = np.ones((2, length), np.float64)
    for t in range(1, length):
        out[0, t] = 1 - beta1 ** float(t)
        b = 1 - beta2 ** float(t)
        out[1, t] = b ** 0.5 if kind == "torch" else math.sqrt(b)
    return out


def clip_coef_torch(total_norm: float, max_norm: float) -> np.float32:
    """clip_grad.py:165-169 on a float32 total norm: ``max_norm / (total_norm + 1e-6)``
    evaluates as ``(total_norm + 1e-6).reciprocal() * max_norm``, then ``clamp(max=1)``."""
    t = np.float32(np.float32(total_norm) + np.float32(1e-6))
    c = np.float32(np.float32(1.0) / t) * np.float32(max_norm)
    return np.float32(min(c, np.float32(1.0)))


def clip_coef_disk(norm: float, max_norm: float) -> np.float32:
    """disk.py:489: ``clip = min(1., max_norm / (norm + 1e-6))`` in double, applied as
    ``gradient * clip`` (float32 multiply, disk.py:210)."""
    return np.float32(min(1.0, max_norm / (norm + 1e-6)))


class DynamicLossScale:
    """precision.py:6-17, restated."""

    def __init__(self, scale=128., growth_interval=2000):
        self.scale = float(scale)
        self.good_steps = 0
        self.growth_interval = growth_interval

    def overflow(self):
        if self.scale <= 1:
            raise FloatingPointError('FP16 overflow at minimum loss scale; state unchanged')
        self.scale = max(1., self.scale / 2)
        self.good_steps = 0

    def success(self):
        self.good_steps += 1
        if self.good_steps >= self.growth_interval:
            self.scale = min(self.scale * 2, 65536.)
            self.good_steps = 0

    def state_dict(self):
        return dict(scale=self.scale, good_steps=self.good_steps, growth_interval=self.growth_interval)


# -------------------------------------------------------------- elementwise --

def grad_prepare(g: np.ndarray, scale=1.0, coef=1.0) -> np.ndarray:
    """float32 gradient = (float(g) / scale) * coef (see oracle.c)."""
    g = np.ascontiguousarray(g)
    dt = {np.dtype(np.float32): F32, np.dtype(np.float16): F16, np.dtype(np.uint16): BF16}[g.dtype]
    out = np.empty(g.size, np.float32)
    lib().orc_grad_prepare(_ptr(g), dt, g.size, float(np.float32(scale)), float(np.float32(coef)), _ptr(out))
    return out.reshape(g.shape)


def sumsq(g32: np.ndarray):
    """(FP64 sum of squares, nonfinite count) of a float32 array (disk.py:466-468)."""
    g32 = np.ascontiguousarray(g32, np.float32)
    bad = ctypes.c_int64(0)
    s = lib().orc_sumsq(_ptr(g32), g32.size, ctypes.byref(bad))
    return s, bad.value


def adamw_(w, m, v, g32, scalars: Scalars):
    """One in-place AdamW step on float32 arrays."""
    for a in (w, m, v, g32):
        assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    assert w.size == m.size == v.size == g32.size
    lib().orc_adamw(_ptr(w), _ptr(m), _ptr(v), _ptr(g32), w.size, ctypes.byref(scalars))


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_ptr(x), _ptr(out), x.size)
    return out


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.uint16)
    out = np.empty(x.shape, np.float32)
    lib().orc_bf16_to_f32(_ptr(x), _ptr(out), x.size)
    return out


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.float16)
    lib().orc_f32_to_f16(_ptr(x), _ptr(out), x.size)
    return out


def export_f16(x: np.ndarray) -> np.ndarray:
    """export.py:33-34: ValueError if nonfinite or |w| > 65504, else RNE float16."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.float16)
    if lib().orc_export_f16(_ptr(x), _ptr(out), x.size):
        raise ValueError('weights cannot be represented by finite FP16')
    return out


def export_f16_chunks(x: np.ndarray, chunk_elements=1048576):
    """export.py:30-35 for one tensor: (bytes the reference writes, whether it
    raised). Chunks are checked in order; the first bad chunk raises after the
    chunks before it were written."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = []
    for start in range(0, x.size, chunk_elements):
        value = x[start:start + chunk_elements]
        if not np.isfinite(value).all() or np.abs(value).max(initial=0) > 65504:
            return b"".join(out), True
        out.append(value.astype('<f2').tobytes())
    return b"".join(out), False


def grad_accumulate_(acc: np.ndarray, g32: np.ndarray, loss_scale=1.0, first=False) -> None:
    """sparse_disk.py:82-110: the window is zeroed, then each microbatch adds
    g.float() / loss_scale (float32 division and addition)."""
    if first:
        acc[...] = np.float32(0)
    acc += np.asarray(g32, np.float32) / np.float32(loss_scale)


def sparse_rows_(w, m, v, idx, grads32, scalars: Scalars):
    """DiskState.update applied to the gathered rows ``idx`` of [rows, cols] planes."""
    rows, cols = w.shape
    idx = np.ascontiguousarray(idx, np.int64)
    grads32 = np.ascontiguousarray(grads32, np.float32)
    assert grads32.shape == (idx.size, cols)
    if lib().orc_sparse_rows(_ptr(w), _ptr(m), _ptr(v), rows, cols, _ptr(idx), idx.size,
                             _ptr(grads32), ctypes.byref(scalars)):
        raise IndexError('row index out of range')


def pack_fp8(x: np.ndarray, block_size=256):
    """streamtrain/precision.py:24-30 restated with torch CPU ops (the float8
    conversion is torch's): (uint8 codes, float32 per-block scales)."""
    import torch
    flat = torch.from_numpy(np.ascontiguousarray(x, np.float32)).reshape(-1)
    padding = (-flat.numel()) % block_size
    padded = torch.nn.functional.pad(flat, (0, padding)).reshape(-1, block_size)
    scales = (padded.abs().amax(1) / 448.).clamp_min(1e-30)
    codes = (padded / scales[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    return codes.reshape(-1)[:flat.numel()].numpy(), scales.numpy()


def unpack_fp8(codes: np.ndarray, scales: np.ndarray, dtype="float16", block_size=256):
    """streamtrain/precision.py:33-37 restated with torch CPU ops."""
    import torch
    c = torch.from_numpy(np.ascontiguousarray(codes, np.uint8))
    n = c.numel()
    padded = torch.nn.functional.pad(c, (0, (-n) % block_size))
    values = padded.view(torch.float8_e4m3fn).float().reshape(-1, block_size)
    return (values * torch.from_numpy(scales)[:, None]).to(getattr(torch, dtype)).reshape(-1)[:n].numpy()


# --------------------------------------------------------------------- Muon --

def orthogonalize(g: np.ndarray, steps=5) -> np.ndarray:
    """optimizer.py:13-22 in float32 (BLAS matmul; summation order is BLAS's)."""
    x = np.asarray(g, np.float32)
    transpose = x.shape[0] > x.shape[1]
    if transpose:
        x = x.T
    x = (x / (np.float32(np.linalg.norm(x.astype(np.float64))) + np.float32(1e-7))).astype(np.float32)
    a, b, c = np.float32(3.4445), np.float32(-4.775), np.float32(2.0315)
    for _ in range(steps):
        gram = x @ x.T
        x = (a * x + (b * gram + c * (gram @ gram)) @ x).astype(np.float32)
    return np.ascontiguousarray(x.T if transpose else x)


def muon_momentum_(mom: np.ndarray, g32: np.ndarray, beta_lerp=.05, nesterov_w=.95) -> np.ndarray:
    """optimizer.py:58-59: momentum.lerp_(g, .05) in place; returns g.lerp(momentum, .95)."""
    u = np.empty_like(mom)
    lib().orc_muon_momentum(_ptr(mom), _ptr(np.ascontiguousarray(g32, np.float32)), _ptr(u),
                            mom.size, beta_lerp, nesterov_w)
    return u


def muon_apply_(w: np.ndarray, o: np.ndarray, lr, wd):
    """optimizer.py:60-61 on the orthogonalised update ``o`` (rows, cols of w)."""
    rows, cols = w.shape
    shape_scale = max(1, rows / cols) ** .5
    lib().orc_muon_apply(_ptr(w), _ptr(np.ascontiguousarray(o, np.float32)), w.size,
                         shape_scale, 1 - lr * wd, -lr)


# ---------------------------------------------------------- seeded inputs --

def rng(seed: int) -> np.random.Generator:
    """Seeded generator shared by fixtures and tests (numpy PCG64; stable across hosts)."""
    return np.random.Generator(np.random.PCG64(seed))


def config1_inputs(seed=1234, tensors=64, shape=(128, 128)):
    """Config 1: ``tensors`` FP32 masters ~N(0, 0.02); m = v = 0."""
    r = rng(seed)
    return [(r.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            for _ in range(tensors)]


def config1_grads(step: int, tensors=64, shape=(128, 128), scale=65536.0, seed=1234):
    """FP16 grads of step ``step``: (N(0, 1e-3) * scale).half(), seed = seed + step."""
    r = rng(seed + step)
    out = []
    for _ in range(tensors):
        g = r.standard_normal(shape, dtype=np.float32) * np.float32(1e-3)
        out.append((g * np.float32(scale)).astype(np.float16))
    return out


def config3_injection(step: int, tensors=64, shape=(128, 128), seed=1234):
    """Config 3: at steps 3 and 7 one seeded element becomes +inf (step 3) or NaN
    (step 7). Returns (tensor index, flat index, value) or None."""
    if step not in (3, 7):
        return None
    r = rng(10_000 + seed + step)
    t = int(r.integers(tensors))
    i = int(r.integers(shape[0] * shape[1]))
    return t, i, (np.float16(np.inf) if step == 3 else np.float16(np.nan))
