"""ZeRO-1 sharded AdamW across the GPUs of one node (one process per GPU).

The reference is single-process; this is the one parallel strategy the B200
build adds. The flat parameter space (all tensors in order) is cut into N
contiguous, 16-element-aligned shards. Rank r owns the FP32 master weights and
the two moments of its shard; every rank holds the full low-precision (BF16)
weights the model computes with. One step:

  1. kernel 2 over this rank's slice of the (already reduced) gradients
     writes the 16-byte record {sum of squares, nonfinite} (FP64);
  2. all_reduce(SUM) of that record, so every rank takes the same skip /
     clip / loss-scale decision;
  3. the one-CTA finalize (clip coefficient, clocks, step scalars);
  4. kernel 1 updates the shard and writes its BF16 copy into this rank's
     slice of the full weight buffer;
  5. all_gather_into_tensor of the BF16 shards, in place.

Only those two collectives exist (NCCL over NVLink on B200 nodes). The kernel
calls go through a backend object: ``CudaZeroBackend`` (the C-ABI library) is
the only one this package provides.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .optim import StepEngine

ALIGN = 16


def shard_bounds(total: int, world: int, rank: int, align: int = ALIGN):
    """[lo, hi) of rank's shard and the padded shard length (same on every rank)."""
    per = -(-total // world)
    per = -(-per // align) * align
    lo = min(total, rank * per)
    hi = min(total, lo + per)
    return lo, hi, per


def shard_pieces(sizes, lo, hi):
    """(tensor index, offset in tensor, offset in shard, length) of every piece of
    the tensors inside [lo, hi) of the flat space."""
    pieces, off = [], 0
    for i, n in enumerate(sizes):
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            pieces.append((i, a - off, a - lo, b - a))
        off += n
    return pieces


class CudaZeroBackend:
    """Kernel calls of one ZeRO step on the rank's GPU (C-ABI library)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.engine = StepEngine(self.device)
        self._plan = None

    def record(self) -> torch.Tensor:
        """The device record {sumsq, nonfinite} as a 2-element FP64 view."""
        return self.engine.state_buf[:16].view(torch.float64)

    def prepare(self, keys, entries, lr, betas, eps, weight_decay, grad_dtype, out_dtype):
        for k in keys:
            self.engine.slot(k, 0)
        groups = [(float(lr), float(betas[0]), float(betas[1]), float(eps), float(weight_decay), "torch")]
        self._plan = self.engine.prepare(entries, groups, _lib.dtype_code(grad_dtype), _lib.dtype_code(out_dtype),
                                         keys=keys)

    def stats(self, fin_flags, max_norm):
        fin = self.engine.finalize_opts(fin_flags, max_norm)
        with torch.cuda.device(self.device):
            _lib.check(self.engine.lib.mb_grad_stats(ctypes.byref(self._plan), None, _lib.stream_handle()),
                       "mb_grad_stats")
        self._fin = fin

    def finalize_and_apply(self):
        with torch.cuda.device(self.device):
            s = _lib.stream_handle()
            _lib.check(self.engine.lib.mb_step_finalize(ctypes.byref(self._plan), ctypes.byref(self._fin), s),
                       "mb_step_finalize")
            _lib.check(self.engine.lib.mb_adamw_apply(ctypes.byref(self._plan), s), "mb_adamw_apply")
        self.engine.max_clock += 1

    def last_step(self) -> dict:
        st = self.engine.read_state()
        return dict(norm=float(st.norm), skipped=bool(st.skip), status=int(st.status),
                    clip_coef=float(st.clip_coef))


class ZeroAdamW:
    """ZeRO-1 AdamW (torch AdamW arithmetic, decoupled weight decay).

    params: the model's FP32 tensors with identical initial values on every
    rank (only this rank's shard is copied into the masters). After each
    ``step(grads)`` the full updated weights are in ``weights`` (one
    low-precision tensor per parameter, views of one flat buffer)."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, *, max_norm=None,
                 clip_mode="torch", gate=False, low_precision=torch.bfloat16, process_group=None, device=None,
                 backend=None):
        params = list(params)
        if not params:
            raise ValueError("ZeroAdamW needs parameters")
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.device = torch.device(device) if device is not None else params[0].device
        self.lr, self.betas, self.eps, self.weight_decay = lr, tuple(betas), eps, weight_decay
        self.max_norm, self.clip_mode, self.gate = max_norm, clip_mode, gate
        if clip_mode not in ("torch", "disk"):
            raise ValueError("clip_mode must be 'torch' or 'disk'")
        self.low_precision = low_precision
        self.shapes = [tuple(p.shape) for p in params]
        self.sizes = [p.numel() for p in params]
        self.total = sum(self.sizes)
        self.lo, self.hi, self.per = shard_bounds(self.total, self.world, self.rank)
        self.pieces = shard_pieces(self.sizes, self.lo, self.hi)
        self.master = torch.zeros(self.per, dtype=torch.float32, device=self.device)
        for i, t_off, s_off, n in self.pieces:
            src = params[i].detach().reshape(-1)[t_off:t_off + n]
            self.master[s_off:s_off + n].copy_(src.to(self.device, torch.float32))
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.flat_weights = torch.zeros(self.per * self.world, dtype=low_precision, device=self.device)
        off = 0
        self.weights = []
        for shape, n in zip(self.shapes, self.sizes):
            self.weights.append(self.flat_weights[off:off + n].view(shape))
            off += n
        for i, t_off, s_off, n in self.pieces:  # this rank's slice starts out as the initial weights
            self.flat_weights[self.lo + s_off:self.lo + s_off + n].copy_(self.master[s_off:s_off + n])
        if self.world > 1:  # every rank starts from the full initial weights
            dist.all_gather_into_tensor(self.flat_weights, self.flat_weights[self.lo:self.lo + self.per].clone(),
                                        group=self.group)
        self.backend = backend if backend is not None else CudaZeroBackend(self.device)
        # one clock key per piece (stable objects)
        self._keys = [object() for _ in self.pieces]
        self._prepared_for = None

    def _fin_flags(self):
        flags = _lib.MB_FIN_GATE if self.gate else 0
        if self.max_norm is not None:
            flags |= _lib.MB_FIN_CLIP_TORCH if self.clip_mode == "torch" else _lib.MB_FIN_CLIP_DISK
        return flags

    @torch.no_grad()
    def step(self, grads) -> None:
        """One step with the full, already reduced gradients (one tensor per
        parameter, same shapes; FP32, FP16 or BF16, one dtype)."""
        grads = list(grads)
        if len(grads) != len(self.sizes):
            raise ValueError("one gradient per parameter expected")
        gdt = grads[0].dtype
        if any(g.dtype != gdt for g in grads):
            raise ValueError("all gradients must share a dtype")
        flat = [g.reshape(-1) for g in grads]
        own = self.flat_weights[self.lo:self.lo + self.per]
        entries = []
        for i, t_off, s_off, n in self.pieces:
            g = flat[i][t_off:t_off + n]
            if g.device != self.device or not g.is_contiguous():
                raise ValueError("gradients must be contiguous and on the optimizer's device")
            entries.append((self.master[s_off:s_off + n], self.exp_avg[s_off:s_off + n],
                            self.exp_avg_sq[s_off:s_off + n], g, own[s_off:s_off + n], 0))
        if entries:
            self.backend.prepare(self._keys, entries, self.lr, self.betas, self.eps, self.weight_decay, gdt,
                                 self.low_precision)
            self.backend.stats(self._fin_flags(), self.max_norm)
        else:
            self.backend.record().zero_()
        if self.world > 1:
            dist.all_reduce(self.backend.record(), group=self.group)
        if entries:
            self.backend.finalize_and_apply()
        if self.world > 1:
            dist.all_gather_into_tensor(self.flat_weights, own, group=self.group)
        if self.gate:
            info = self.backend.last_step()
            if info["status"]:
                _lib.check(info["status"], "optimizer not updated")

    def last_step(self) -> dict:
        return self.backend.last_step()

    def state_dict(self) -> dict:
        """This rank's shard: masters, moments, bounds and hyperparameters."""
        return dict(rank=self.rank, world=self.world, lo=self.lo, hi=self.hi, per=self.per,
                    master=self.master.cpu(), exp_avg=self.exp_avg.cpu(), exp_avg_sq=self.exp_avg_sq.cpu(),
                    lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.weight_decay)
