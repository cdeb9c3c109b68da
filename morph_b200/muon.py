"""Hybrid Muon + AdamW on the B200 kernels.

``gemm_bf16`` exposes kernel 4's tcgen05 GEMM. The Newton-Schulz
orthogonalisation (streamtrain/optimizer.py:13-22) and the HybridMuonAdamW
drop-in (streamtrain/optimizer.py:25-70) are built on it.
"""
from __future__ import annotations

import torch

from . import _lib


def _check_bf16_matrix(t, name):
    if not t.is_cuda or t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D row-major BF16 CUDA tensor")


def gemm_bf16(a, b, alpha=1.0, beta=0.0, c=None, out=True, out_t=False, out_f32=False):
    """alpha * (a @ b.T) + beta * c on the tensor cores. a [m, k], b [n, k] BF16
    row-major; m % 128 == 0, n % 256 == 0, k % 64 == 0. Returns (d, dt, df):
    BF16 [m, n], BF16 [n, m] (transposed copy) and FP32 [m, n], each or None."""
    _check_bf16_matrix(a, "a")
    _check_bf16_matrix(b, "b")
    m, k = a.shape
    n, k2 = b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    if c is not None:
        _check_bf16_matrix(c, "c")
        if c.shape != (m, n):
            raise ValueError("c must be [m, n]")
    dev = a.device
    d = torch.empty(m, n, dtype=torch.bfloat16, device=dev) if out else None
    dt = torch.empty(n, m, dtype=torch.bfloat16, device=dev) if out_t else None
    df = torch.empty(m, n, dtype=torch.float32, device=dev) if out_f32 else None
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    P = lambda t: None if t is None else _lib.ptr(t)  # noqa: E731
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mb_gemm_bf16(
            _lib.ptr(a), a.stride(0), _lib.ptr(b), b.stride(0), m, n, k, float(alpha), float(beta),
            P(c), c.stride(0) if c is not None else 0, P(d), n, P(dt), m, P(df), n, _lib.ptr(err),
            _lib.stream_handle()), "gemm_bf16")
    if int(err.item()):
        raise RuntimeError("gemm_bf16: a bounded wait expired on the device")
    return d, dt, df
