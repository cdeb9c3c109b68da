"""Drop-in AdamW for the reference's resident and streamed optimizer steps.

``AdamW`` replaces ``torch.optim.AdamW(..., foreach=False)`` where MORPH builds
it (streamtrain/optimizer.py:40, morph/training/runner.py:46,
morph/training/proof_runner.py:103): same constructor, ``param_groups``,
``state`` layout (``step``, ``exp_avg``, ``exp_avg_sq``) and ``state_dict()``.
One ``step()`` is two launches of the C-ABI library for all parameters:

  * kernel 2 (``mb_grad_stats``) — FP64 sum of squares and nonfinite count of
    every gradient, then in its last CTA the finalize: loss-scale back-off or
    success, skip decision, clip coefficient, clock advance, step scalars;
  * kernel 1 (``mb_adamw_apply``) — the fused AdamW update of w, m, v reading
    FP32/FP16/BF16 gradients, optionally writing a BF16/FP16 copy of w.

Extras beyond torch's signature, all off by default: ``max_norm`` (fused
``clip_grad_norm_``, morph/training/runner.py:100, or the disk engines' FP64
rule with ``clip_mode='disk'``), ``loss_scale`` (a device
``DynamicLossScale``: gradients are divided by its scale, overflow skips the
step and backs off), ``gate`` (nonfinite gradients raise FloatingPointError and
change nothing, streamtrain/optimizer.py:50-51) and ``low_precision`` (dtype of
a per-parameter compute copy written by the same kernel).
"""
from __future__ import annotations

import collections
import ctypes
import math

import numpy as np
import torch

from . import _lib
from .precision import DynamicLossScale

_SEG_DTYPE = np.dtype([("w", "<u8"), ("m", "<u8"), ("v", "<u8"), ("g", "<u8"), ("out", "<u8"),
                       ("numel", "<i8"), ("tile_begin", "<i8"), ("clock", "<i4"), ("group", "<i4")])
_GROUP_DTYPE = np.dtype([("lr", "<f8"), ("cwd", "<f4"), ("omb1", "<f4"), ("beta2", "<f4"), ("omb2", "<f4"),
                         ("eps", "<f4"), ("table", "<i4")])
assert _SEG_DTYPE.itemsize == 64 and _GROUP_DTYPE.itemsize == 32
TILE = 2048  # elements per tile (must match mb_common.cuh kTile)


def _to_device_bytes(arr: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(arr.view(np.uint8).copy()).to(device, non_blocking=False)


class BiasCorrectionTables:
    """Device table of the bias corrections per clock t, computed on the host in
    Python double exactly as the reference does: ``1 - beta1 ** t`` and
    ``(1 - beta2 ** t) ** 0.5`` (kind 'torch', adam.py) or
    ``math.sqrt(1 - beta2 ** t)`` (kind 'disk', disk.py:213). Once both have
    rounded to 1.0 they stay there, so the table stops at that clock and the
    kernel clamps larger clocks to the last entry."""

    def __init__(self, device):
        self.device = device
        self.keys: list[tuple] = []
        self.length = 0
        self.tensor = None

    def index(self, beta1, beta2, kind="torch") -> int:
        key = (float(beta1), float(beta2), kind)
        if key not in self.keys:
            self.keys.append(key)
            self.tensor = None
        return self.keys.index(key)

    @staticmethod
    def _saturation(beta) -> float:
        if beta <= 0.0:
            return 2
        if beta >= 1.0:
            return math.inf
        return math.ceil(60 * math.log(2) / -math.log(beta)) + 2

    # longest table built (entries per row); clocks past it use its last entry,
    # which is exact once both corrections have reached 1.0 (beta2 <= 0.99998)
    MAX_LENGTH = 1 << 20

    def ensure(self, max_clock: int):
        """The table for every registered (beta1, beta2, rule), long enough for
        clocks up to ``max_clock``. It is built to saturation up front (bounded by
        MAX_LENGTH), so later steps never rebuild it: a captured CUDA graph can
        replay the step for any number of steps."""
        sat = max(max(self._saturation(b1), self._saturation(b2)) for b1, b2, _ in self.keys)
        need = max_clock + 2
        if self.tensor is not None and (need <= self.length or self.length >= min(sat, self.MAX_LENGTH)):
            return self.tensor, self.length
        length = int(min(max(sat, need, 2), self.MAX_LENGTH))
        rows = []
        for b1, b2, kind in self.keys:
            t1 = np.ones(length, np.float64)
            t2 = np.ones(length, np.float64)
            t = np.arange(1, length, dtype=np.float64)
            t1[1:] = [1 - b1 ** ft for ft in t.tolist()]
            bb = [1 - b2 ** ft for ft in t.tolist()]
            t2[1:] = [x ** 0.5 for x in bb] if kind == "torch" else [math.sqrt(x) for x in bb]
            rows += [t1, t2]
        self.tensor = torch.from_numpy(np.stack(rows)).to(self.device)
        self.length = length
        return self.tensor, self.length


class StepEngine:
    """Plans and launches fused multi-tensor AdamW steps on one device.

    Owns the device clocks (one int32 per parameter slot), the bias-correction
    tables, the kernel workspace and the step-state record (its own, or the
    one of an attached DynamicLossScale)."""

    SEG_CACHE = 4  # distinct segment tables kept on the device

    def __init__(self, device, loss_scale: DynamicLossScale | None = None):
        self.device = torch.device(device)
        self.lib = _lib.lib()
        self.tables = BiasCorrectionTables(self.device)
        self.slots: dict[int, int] = {}
        self.clocks = torch.zeros(0, dtype=torch.int32, device=self.device)
        self.generation = 0
        self.max_clock = 0
        self.loss_scale = loss_scale
        if loss_scale is not None:
            if loss_scale.device != self.device:
                raise ValueError("loss scale lives on another device")
            self.state_buf = loss_scale.state_buffer
        else:
            st = _lib.StepState()
            _lib.check(self.lib.mb_step_state_init(ctypes.byref(st), 1.0, 1 << 62))
            self.state_buf = torch.frombuffer(bytearray(bytes(st)), dtype=torch.uint8).to(self.device)
        self.workspace = None
        # device segment tables of the last few distinct layouts (a caller that
        # alternates gradient buffers alternates between two of them)
        self._seg_cache = collections.OrderedDict()
        self._group_bytes = None
        self._groups_dev = None

    # -- clocks ------------------------------------------------------------------
    def reserve(self, n: int) -> None:
        """Grow the clock array to at least n slots. Growing moves it, so views
        handed out by clock_view() before a growth must be refreshed
        (``generation`` changes when that happens)."""
        if n > self.clocks.numel():
            grown = torch.zeros(max(16, n, 2 * self.clocks.numel()), dtype=torch.int32, device=self.device)
            grown[: self.clocks.numel()] = self.clocks
            self.clocks = grown
            self.generation += 1
            self.invalidate_segments()

    def slot(self, p: torch.Tensor, initial_clock: int = 0) -> int:
        key = id(p)
        if key not in self.slots:
            s = len(self.slots)
            self.reserve(s + 1)
            self.slots[key] = s
            self.clocks[s] = int(initial_clock)
            self.max_clock = max(self.max_clock, int(initial_clock))
        return self.slots[key]

    def set_clock(self, p, value: int) -> None:
        s = self.slot(p)
        self.clocks[s] = int(value)
        self.max_clock = max(self.max_clock, int(value))

    def clock_view(self, p) -> torch.Tensor:
        s = self.slot(p)
        return self.clocks[s]

    # -- state record ---------------------------------------------------------------
    def read_state(self) -> _lib.StepState:
        return _lib.StepState.from_buffer_copy(self.state_buf.cpu().numpy().tobytes())

    # -- launch -------------------------------------------------------------------------
    def prepare(self, entries, groups, grad_dtype, out_dtype, keys=None) -> _lib.Plan:
        """Build (or reuse) the device segment table and return the launch plan.

        entries: list of (p, m, v, g, out_or_None, group_index) where p, m, v are
        FP32 and may be any contiguous ranges (whole tensors or shard pieces);
        groups: list of (lr, beta1, beta2, eps, weight_decay, table_kind);
        keys: objects whose clock slots the segments use (default: each p)."""
        n = len(entries)
        keys = [e[0] for e in entries] if keys is None else keys
        slots = [self.slots[id(k)] for k in keys]
        key = tuple((p.data_ptr(), m.data_ptr(), v.data_ptr(), g.data_ptr(),
                     0 if o is None else o.data_ptr(), g.numel(), sl, gi)
                    for (p, m, v, g, o, gi), sl in zip(entries, slots))
        hit = self._seg_cache.get(key)
        if hit is None:
            segs = np.zeros(n, _SEG_DTYPE)
            tiles = 0
            for i, ((p, m, v, g, o, gi), sl) in enumerate(zip(entries, slots)):
                segs[i] = (p.data_ptr(), m.data_ptr(), v.data_ptr(), g.data_ptr(),
                           0 if o is None else o.data_ptr(), g.numel(), tiles, sl, gi)
                tiles += (g.numel() + TILE - 1) // TILE
            hit = (_to_device_bytes(segs, self.device), tiles)
            self._seg_cache[key] = hit
            while len(self._seg_cache) > self.SEG_CACHE:
                self._seg_cache.popitem(last=False)
            need = self.lib.mb_workspace_bytes(n)
            if self.workspace is None or self.workspace.numel() < need:
                self.workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)
        else:
            self._seg_cache.move_to_end(key)
        segs_dev, n_tiles = hit
        garr = np.zeros(len(groups), _GROUP_DTYPE)
        for i, (lr, b1, b2, eps, wd, kind) in enumerate(groups):
            garr[i] = (lr, np.float32(1 - lr * wd), np.float32(1 - b1), np.float32(b2), np.float32(1 - b2),
                       np.float32(eps), self.tables.index(b1, b2, kind))
        gbytes = garr.tobytes()
        if gbytes != self._group_bytes:
            self._groups_dev = _to_device_bytes(garr, self.device)
            self._group_bytes = gbytes
        bc, bc_len = self.tables.ensure(self.max_clock + 1)
        return _lib.Plan(segs_dev.data_ptr(), self._groups_dev.data_ptr(), bc.data_ptr(),
                         self.clocks.data_ptr(), self.workspace.data_ptr(), self.state_buf.data_ptr(),
                         n_tiles, bc_len, n, len(groups), grad_dtype, out_dtype)

    def invalidate_segments(self) -> None:
        """Forget the cached segment tables (clock slots or layouts changed)."""
        self._seg_cache.clear()

    @staticmethod
    def finalize_opts(fin_flags, max_norm) -> _lib.FinalizeOpts:
        return _lib.FinalizeOpts(int(fin_flags), 0, float(max_norm or 0.0), 0.5, 2.0)

    def launch(self, plan, fin, stream=None, stats=True):
        """One optimizer step on ``plan``: kernel 2 with the fused finalize (or the
        one-block finalize alone when no gradient statistics are needed), then
        kernel 1. Advances the host bound on the device clocks."""
        s = _lib.stream_handle(stream)
        self.max_clock += 1
        if stats:
            _lib.check(self.lib.mb_grad_stats(ctypes.byref(plan), ctypes.byref(fin), s), "mb_grad_stats")
        else:
            _lib.check(self.lib.mb_step_finalize(ctypes.byref(plan), ctypes.byref(fin), s), "mb_step_finalize")
        _lib.check(self.lib.mb_adamw_apply(ctypes.byref(plan), s), "mb_adamw_apply")

    def step(self, entries, groups, grad_dtype, out_dtype, fin_flags, max_norm, stream=None, stats=None):
        """One step; ``stats=False`` skips kernel 2 and finalizes from the
        {sum of squares, nonfinite} record already in the state (written by an
        earlier statistics launch over a superset of the gradients)."""
        plan = self.prepare(entries, groups, grad_dtype, out_dtype)
        if stats is None:
            stats = bool(fin_flags & (_lib.MB_FIN_LOSS_SCALE | _lib.MB_FIN_GATE | _lib.MB_FIN_CLIP_TORCH
                                      | _lib.MB_FIN_CLIP_DISK))
        self.launch(plan, self.finalize_opts(fin_flags, max_norm), stream, stats)
        return plan


class AdamW(torch.optim.Optimizer):
    """torch.optim.AdamW on the B200 kernels (decoupled weight decay, no amsgrad).

    Parameters must be contiguous FP32 CUDA tensors on one device; gradients
    contiguous FP32/FP16/BF16 of the parameter's shape, one dtype per step.

    With ``sync=False`` (the default unless ``gate``) ``step`` only enqueues
    kernels: clocks, the skip decision, the loss scale and the clip coefficient
    all live on the device. After one eager step it can be captured in a CUDA
    graph and replayed for any number of steps, provided the gradients stay at
    the same addresses (as for torch's capturable optimizers)."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, amsgrad=False, *,
                 maximize=False, foreach=None, capturable=False, differentiable=False, fused=None,
                 max_norm=None, clip_mode="torch", loss_scale: DynamicLossScale | None = None,
                 gate=False, low_precision=None, sync=None):
        if amsgrad or maximize or differentiable:
            raise NotImplementedError("amsgrad, maximize and differentiable are not supported")
        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= eps:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameters: {betas}")
        if clip_mode not in ("torch", "disk"):
            raise ValueError("clip_mode must be 'torch' or 'disk'")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=False, maximize=False,
                        foreach=foreach, capturable=capturable, differentiable=False, fused=fused,
                        decoupled_weight_decay=True)
        super().__init__(params, defaults)
        self.max_norm = max_norm
        self.clip_mode = clip_mode
        self.loss_scale = loss_scale
        self.gate = gate
        self.low_precision = low_precision
        self.sync = gate if sync is None else sync
        self.low_precision_copies: dict[torch.Tensor, torch.Tensor] = {}
        self._engine: StepEngine | None = None
        self._generation = 0
        # set by HybridMuonAdamW: the statistics of this step were computed over
        # all of the hybrid's gradients into this engine's record already
        self._shared_record = False
        # per parameter, after its first step: (p, its state dict, copy, device, shape)
        self._prepared: dict[int, tuple] = {}

    # -- helpers ---------------------------------------------------------------------
    def _engine_for(self, device) -> StepEngine:
        if self._engine is None:
            self._engine = StepEngine(device, self.loss_scale)
            self._engine.reserve(sum(len(g["params"]) for g in self.param_groups))
            self._generation = self._engine.generation
        elif self._engine.device != device:
            raise ValueError("all parameters of one AdamW must live on one CUDA device")
        return self._engine

    def _init_state(self, p, eng: StepEngine):
        state = self.state[p]
        if len(state) == 0:
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            eng.slot(p, 0)
            state["step"] = eng.clock_view(p)
        elif not (torch.is_tensor(state.get("step")) and state["step"].device == eng.device
                  and state["step"].dtype == torch.int32):
            eng.set_clock(p, int(float(state.get("step", 0))))
            state["step"] = eng.clock_view(p)
        return state

    def _fin_flags(self) -> int:
        flags = 0
        if self.loss_scale is not None:
            flags |= _lib.MB_FIN_LOSS_SCALE
        elif self.gate:
            flags |= _lib.MB_FIN_GATE
        if self.max_norm is not None:
            flags |= _lib.MB_FIN_CLIP_TORCH if self.clip_mode == "torch" else _lib.MB_FIN_CLIP_DISK
        return flags

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        entries, groups, gdt, device, last_dtype = [], [], None, None, None
        prepared = self._prepared
        for gi, group in enumerate(self.param_groups):
            b1, b2 = group["betas"]
            groups.append((float(group["lr"]), float(b1), float(b2), float(group["eps"]),
                           float(group["weight_decay"]), "torch"))
            for p in group["params"]:
                g = p.grad
                if g is None:
                    continue
                ready = prepared.get(id(p))
                if ready is None or ready[0] is not p:
                    # first step of this parameter (or after a state change): validate, create state
                    if not p.is_cuda or p.dtype != torch.float32 or not p.is_contiguous():
                        raise ValueError("parameters must be contiguous float32 CUDA tensors")
                    eng = self._engine_for(p.device)
                    st = self._init_state(p, eng)
                    out = None
                    if self.low_precision is not None:
                        out = self.low_precision_copies.get(p)
                        if out is None:
                            out = torch.empty_like(p, dtype=self.low_precision)
                            self.low_precision_copies[p] = out
                    ready = prepared[id(p)] = (p, st, out, p.device, p.shape)
                if g.shape != ready[4] or g.device != ready[3] or not g.is_contiguous():
                    raise ValueError("gradient must be contiguous, on the parameter's device and shape")
                if g.dtype is not last_dtype:
                    code = _lib.dtype_code(g.dtype)
                    if gdt is None:
                        gdt = code
                    elif code != gdt:
                        raise ValueError("all gradients of one step must share a dtype")
                    last_dtype = g.dtype
                device = ready[3]
                st = ready[1]
                entries.append((p, st["exp_avg"], st["exp_avg_sq"], g, ready[2], gi))
        if not entries:
            return loss
        eng = self._engine_for(device)
        if eng.generation != self._generation:  # the clock array moved: refresh the step views
            for p, st in self.state.items():
                if id(p) in eng.slots:
                    st["step"] = eng.clock_view(p)
            self._generation = eng.generation
            self._prepared.clear()
        odt = _lib.dtype_code(self.low_precision) if self.low_precision is not None else _lib.MB_NONE
        with torch.cuda.device(device):
            eng.step(entries, groups, gdt, odt, self._fin_flags(), self.max_norm,
                     stats=False if self._shared_record else None)
        if self.sync:
            self.check()
        return loss

    def check(self) -> None:
        """Synchronise and raise FloatingPointError if the last step was refused
        (nonfinite gradient under ``gate``, or overflow at loss scale 1)."""
        if self._engine is None:
            return
        st = self._engine.read_state()
        if st.status:
            _lib.check(int(st.status), "optimizer not updated")

    def last_step(self) -> dict:
        """Device outcome of the last step: grad norm, skip flag, clip coefficient."""
        st = self._engine.read_state() if self._engine else _lib.StepState()
        return dict(norm=float(st.norm), skipped=bool(st.skip), status=int(st.status),
                    clip_coef=float(st.clip_coef), step_scale=float(st.step_scale))

    # -- checkpoints in torch's CPU layout ----------------------------------------
    def state_dict(self):
        """torch's layout: per-parameter ``step`` as a 0-dim float32 CPU tensor
        (one device read of all clocks), ``exp_avg``/``exp_avg_sq`` as stored."""
        sd = super().state_dict()
        clocks = self._engine.clocks.cpu() if self._engine is not None else None
        index = {}
        for group, packed in zip(self.param_groups, sd["param_groups"]):
            for p, i in zip(group["params"], packed["params"]):
                index[i] = p
        state = {}
        for i, st in sd["state"].items():
            st = dict(st)  # never hand out the live per-parameter dict
            step = st.get("step")
            if torch.is_tensor(step) and step.is_cuda:
                p = index[i]
                value = int(clocks[self._engine.slots[id(p)]]) if id(p) in self._engine.slots else int(step.item())
                st["step"] = torch.tensor(float(value), dtype=torch.float32)
            state[i] = st
        sd["state"] = state
        return sd

    def load_state_dict(self, state_dict):
        self._prepared.clear()
        super().load_state_dict(state_dict)
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if st and "step" in st:
                    if p.is_cuda:
                        eng = self._engine_for(p.device)
                        eng.set_clock(p, int(float(st["step"])))
                        st["step"] = eng.clock_view(p)
        if self._engine is not None:
            self._engine.invalidate_segments()
