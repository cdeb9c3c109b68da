"""Hybrid Muon + AdamW on the B200 kernels.

``gemm16`` exposes kernel 4's tcgen05 GEMM (BF16 or FP16 operands, FP32
accumulation). The Newton-Schulz orthogonalisation
(streamtrain/optimizer.py:13-22), the batched Muon step and the
HybridMuonAdamW drop-in (streamtrain/optimizer.py:25-70) are built on it.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib


def _check_matrix(t, name, dtype):
    if not t.is_cuda or t.dtype != dtype or t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D row-major {dtype} CUDA tensor")


def gemm16(a, b, alpha=1.0, beta=0.0, c=None, out=True, out_t=False, out_f32=False):
    """alpha * (a @ b.T) + beta * c on the tensor cores, FP32 accumulation.
    a [m, k], b [n, k] row-major BF16 or FP16 (one type); m % 128 == 0,
    n % 256 == 0, k % 64 == 0. Returns (d, dt, df): 16-bit [m, n], 16-bit [n, m]
    (transposed copy) and FP32 [m, n], each or None."""
    dtype = a.dtype
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("gemm16 operands must be bfloat16 or float16")
    _check_matrix(a, "a", dtype)
    _check_matrix(b, "b", dtype)
    m, k = a.shape
    n, k2 = b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    if c is not None:
        _check_matrix(c, "c", dtype)
        if c.shape != (m, n):
            raise ValueError("c must be [m, n]")
    dev = a.device
    d = torch.empty(m, n, dtype=dtype, device=dev) if out else None
    dt = torch.empty(n, m, dtype=dtype, device=dev) if out_t else None
    df = torch.empty(m, n, dtype=torch.float32, device=dev) if out_f32 else None
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    P = lambda t: None if t is None else _lib.ptr(t)  # noqa: E731
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mb_gemm16(
            _lib.dtype_code(dtype), _lib.ptr(a), a.stride(0), _lib.ptr(b), b.stride(0), m, n, k, float(alpha),
            float(beta), P(c), c.stride(0) if c is not None else 0, P(d), n, P(dt), m, P(df), n, _lib.ptr(err),
            _lib.stream_handle()), "gemm16")
    if int(err.item()):
        raise RuntimeError("gemm16: a bounded wait expired on the device")
    return d, dt, df


# ------------------------------------------------------------------ Muon ----

NS_COEFFS = (3.4445, -4.775, 2.0315)
# Newton-Schulz operands: FP16 and BF16 run on the same tensor-core path at the
# same rate. The iterates are normalised (entries bounded by the power-of-two
# prescale of the first one, singular values near 1 afterwards), so FP16's range
# suffices and its 10-bit mantissa keeps the result 6-8x closer to the FP32
# reference than BF16's 7 bits: relative Frobenius error ~0.1 % vs 0.7-1.0 % on
# Gaussian inputs, 0.5 % vs 4-6 % with singular values spread over 1e-4..1
# (exact CPU emulation of the roundings). BF16 stays selectable; below a
# smaller dimension of 256 it exceeds the 1e-2 bar even on Gaussian inputs.
BF16_MIN_DIM = 256


def ns_operand_dtype(rows, cols, ns_dtype="auto"):
    """Operand type of Newton-Schulz: 'bf16', 'fp16', or 'auto' (FP16)."""
    if ns_dtype in ("bf16", torch.bfloat16):
        return _lib.MB_BF16
    if ns_dtype in ("fp16", torch.float16, "auto"):
        return _lib.MB_F16
    raise ValueError("ns_dtype must be 'auto', 'bf16' or 'fp16'")


class _Workspace:
    """Grow-only device workspace for one matrix at a time, per device."""

    def __init__(self):
        self.buf = {}

    def get(self, device, nbytes):
        t = self.buf.get(device)
        if t is None or t.numel() < nbytes:
            t = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            self.buf[device] = t
        return t


_WS = _Workspace()


def _workspace_for(device, rows, cols):
    nbytes = _lib.lib().mb_muon_workspace_bytes(rows, cols)
    if nbytes == 0:
        raise ValueError(f"unsupported matrix shape {(rows, cols)}")
    return _WS.get(device, nbytes), nbytes


def orthogonalize(gradient: torch.Tensor, steps: int = 5, ns_dtype="auto") -> torch.Tensor:
    """streamtrain/optimizer.py:13-22 on the GPU: FP32 in, FP32 out, Newton-Schulz
    on 16-bit tensor-core GEMMs with FP32 accumulation (see ns_operand_dtype)."""
    if gradient.dim() != 2 or not gradient.is_cuda:
        raise ValueError("orthogonalize expects a 2-D CUDA tensor")
    x = gradient.float().contiguous()
    rows, cols = x.shape
    out = torch.empty_like(x)
    ws, nbytes = _workspace_for(x.device, rows, cols)
    err = torch.zeros(1, dtype=torch.int32, device=x.device)
    coeffs = torch.tensor(NS_COEFFS, dtype=torch.float32)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().mb_newton_schulz(
            _lib.ptr(x), rows, cols, int(steps), coeffs.numpy().ctypes.data, ns_operand_dtype(rows, cols, ns_dtype),
            _lib.ptr(out), _lib.ptr(ws), nbytes,
            _lib.ptr(err), _lib.stream_handle()), "newton_schulz")
    if int(err.item()):
        raise RuntimeError("newton_schulz: a bounded wait expired on the device")
    return out


def batch_plan(count, rows, cols, workspace_limit):
    """Sizes of the batches that step ``count`` [rows, cols] matrices: as few
    launches as the workspace limit and MB_MUON_MAX_BATCH allow, evenly filled."""
    if count <= 0:
        return []
    per = _lib.lib().mb_muon_batch_workspace_bytes(1, rows, cols)
    if per == 0:
        raise ValueError(f"unsupported matrix shape {(rows, cols)}")
    cap = max(1, min(_lib.MB_MUON_MAX_BATCH, int(workspace_limit) // per))
    n = -(-count // cap)
    size = -(-count // n)
    return [min(size, count - b) for b in range(0, count, size)]


def muon_step_batched(params, moms, grads, outs, lr, weight_decay, ns_dtype="auto", err=None, skip=None,
                      max_sms=0):
    """optimizer.py:52-61 for each of ``params`` (same-shape contiguous FP32 CUDA
    matrices on one device) in one kernel-4 call: momentum (FP32, in place),
    Nesterov blend, Newton-Schulz, shape scale, decoupled weight decay; ``outs``
    (optional, one 16-bit tensor each) receive the updated weights. ``err``
    (int32 device flag) is raised when a bounded wait expires. ``skip`` (device
    address of an int32 flag, e.g. a finalized gate's skip) makes every launch
    of the step return at once when the flag is set: nothing changes.
    ``max_sms`` (0: all) caps the SMs the GEMMs occupy, leaving the rest to
    kernels on other streams (a collective); the results are the same bits."""
    batch = len(params)
    if batch == 0:
        return
    rows, cols = params[0].shape
    dev = params[0].device
    gdt = grads[0].dtype
    for p, m, g in zip(params, moms, grads):
        if (p.dim() != 2 or not p.is_cuda or p.dtype != torch.float32 or not p.is_contiguous()
                or tuple(p.shape) != (rows, cols) or p.device != dev):
            raise ValueError("Muon parameters must be contiguous same-shape 2-D float32 CUDA tensors")
        if m.shape != p.shape or m.dtype != torch.float32 or not m.is_contiguous():
            raise ValueError("momentum must match its parameter")
        if g.shape != p.shape or g.dtype != gdt or not g.is_contiguous():
            raise ValueError("gradients must be contiguous, of the parameter's shape and one dtype")
    if outs is not None:
        for o in outs:
            if (o.shape != (rows, cols) or not o.is_contiguous() or o.dtype != outs[0].dtype
                    or o.dtype not in (torch.bfloat16, torch.float16)):
                raise ValueError("copies must be contiguous BF16 or FP16 tensors of the parameters' shape")
    nbytes = _lib.lib().mb_muon_batch_workspace_bytes(batch, rows, cols)
    if nbytes == 0:
        raise ValueError(f"unsupported batch {batch} of {(rows, cols)}")
    ws = _WS.get(dev, nbytes)
    f = lambda x: float(np.float32(x))  # noqa: E731
    args = _lib.MuonArgs(f(.05), f(.95), f(NS_COEFFS[0]), f(NS_COEFFS[1]), f(NS_COEFFS[2]), 5,
                         f(max(1, rows / cols) ** .5), f(1 - lr * weight_decay), f(-lr),
                         ns_operand_dtype(rows, cols, ns_dtype), skip, int(max_sms))
    odt = _lib.MB_NONE if outs is None else _lib.dtype_code(outs[0].dtype)
    table = ctypes.c_void_p * batch
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mb_muon_step_batched(
            table(*[_lib.ptr(p) for p in params]), table(*[_lib.ptr(m) for m in moms]),
            table(*[_lib.ptr(g) for g in grads]), _lib.dtype_code(gdt),
            None if outs is None else table(*[_lib.ptr(o) for o in outs]), odt, batch, rows, cols,
            ctypes.byref(args), _lib.ptr(ws), nbytes, None if err is None else _lib.ptr(err),
            _lib.stream_handle()), "muon_step")


def partition(model):
    """streamtrain/optimizer.py:25-31: weights of nn.Linear modules not named
    'lm_head' go to Muon, every other parameter to AdamW."""
    hidden = {id(module.weight) for name, module in model.named_modules()
              if isinstance(module, torch.nn.Linear) and name != 'lm_head'}
    muon, adam = [], []
    for param in model.parameters():
        (muon if id(param) in hidden else adam).append(param)
    return muon, adam


class HybridMuonAdamW:
    """Drop-in for streamtrain/optimizer.py:34-70 on the B200 kernels.

    Same constructor, attributes (muon, adam, momentum, lr, weight_decay),
    zero_grad, step and state_dict/load_state_dict format. ``step`` enqueues
    one device-side finiteness gate over every gradient (kernel 2 and its
    finalize, optimizer.py:50-51), then each shape's Muon matrices (kernel 4,
    batched) and the AdamW group (finalize and kernel 1); every launch reads the
    gate's skip flag first, so a nonfinite gradient changes nothing anywhere.
    The host reads the outcome once, at the end: with ``sync=True`` (the
    default, the reference's behaviour) ``step`` raises FloatingPointError when
    the gate refused the step; with ``sync=False`` it only enqueues and
    ``check()`` raises later."""

    def __init__(self, model, lr=1e-3, muon_lr=None, weight_decay=.01, low_precision=None, ns_dtype="auto",
                 workspace_limit=4 << 30, sync=True):
        from .optim import AdamW
        self.muon, adam = partition(model)
        self.lr = lr if muon_lr is None else muon_lr
        self.weight_decay = weight_decay
        self.momentum = {}
        self.low_precision = low_precision
        self.low_precision_copies = {}
        self.ns_dtype = ns_dtype
        self.workspace_limit = int(workspace_limit)
        self.sync = bool(sync)
        # the AdamW group finalizes from the gate's record over all gradients (gate on, no host read)
        self.adam = AdamW(adam, lr=lr, weight_decay=weight_decay, betas=(.9, .95), foreach=False,
                          low_precision=low_precision, gate=True, sync=False)
        self.adam._shared_record = True
        self._gate_engines = {}
        self._err = {}
        self._new_momentum = []

    def zero_grad(self, set_to_none=True):
        for p in self.muon:
            p.grad = None if set_to_none else torch.zeros_like(p)
        self.adam.zero_grad(set_to_none=set_to_none)

    def _record_engine(self, device):
        """The step engine whose device record the gate writes and every launch
        of the step reads: the AdamW group's (it finalizes from it)."""
        adam_params = [p for g in self.adam.param_groups for p in g["params"]]
        if adam_params:
            return self.adam._engine_for(adam_params[0].device)
        from .optim import StepEngine
        eng = self._gate_engines.get(("record", device))
        if eng is None:
            eng = self._gate_engines[("record", device)] = StepEngine(device)
        return eng

    def _gate(self, params):
        """Enqueue kernel 2 over every gradient into the shared record and finalize
        it with the finiteness gate (optimizer.py:50-51). Returns the record's
        engine, or None when no parameter has a gradient."""
        from .optim import StepEngine
        grads = [(p, p.grad) for p in params if p.grad is not None]
        if not grads:
            return None
        dev = grads[0][1].device
        rec_eng = self._record_engine(dev)
        by_dtype = {}
        for p, g in grads:
            if g.device != dev:
                raise ValueError("all gradients of one HybridMuonAdamW must live on one CUDA device")
            by_dtype.setdefault(g.dtype, []).append((p, g.contiguous()))
        fin = None
        plans = []
        for dtype, items in by_dtype.items():
            eng = self._gate_engines.get((dev, dtype))
            if eng is None:
                eng = self._gate_engines[(dev, dtype)] = StepEngine(dev)
            eng.state_buf = rec_eng.state_buf
            for p, _ in items:
                eng.slot(p, 0)
            entries = [(g, g, g, g, None, 0) for _, g in items]
            plan = eng.prepare(entries, [(0.0, 0.9, 0.9, 1e-8, 0.0, "torch")], _lib.dtype_code(dtype), _lib.MB_NONE,
                               keys=[p for p, _ in items])
            fin = eng.finalize_opts(_lib.MB_FIN_GATE, None)
            plans.append((eng, plan))
        record = rec_eng.state_buf[:16].view(torch.float64)
        with torch.cuda.device(dev):
            s = _lib.stream_handle()
            if len(plans) == 1:
                eng, plan = plans[0]
                _lib.check(eng.lib.mb_grad_stats(ctypes.byref(plan), ctypes.byref(fin), s))
            else:  # one record over several gradient dtypes, then one finalize
                acc = torch.zeros(2, dtype=torch.float64, device=dev)
                for eng, plan in plans:
                    _lib.check(eng.lib.mb_grad_stats(ctypes.byref(plan), None, s))
                    acc += record
                record.copy_(acc)
                eng, plan = plans[-1]
                _lib.check(eng.lib.mb_step_finalize(ctypes.byref(plan), ctypes.byref(fin), s))
        return rec_eng

    @torch.no_grad()
    def step(self):
        all_params = self.muon + [p for g in self.adam.param_groups for p in g['params']]
        rec_eng = self._gate(all_params)
        if rec_eng is None:
            return
        skip = rec_eng.state_buf.data_ptr() + _lib.StepState.skip.offset
        # matrices of one shape and gradient dtype share every launch (kernel 4 batches them)
        groups = {}
        self._new_momentum = []
        for i, p in enumerate(self.muon):
            if p.grad is None:
                continue
            if p.dim() != 2 or not p.is_cuda or p.dtype != torch.float32 or not p.is_contiguous():
                raise ValueError("Muon parameters must be contiguous 2-D float32 CUDA tensors")
            if i not in self.momentum:
                self.momentum[i] = torch.zeros_like(p)
                self._new_momentum.append(i)
            g = p.grad.contiguous()
            groups.setdefault((p.device, tuple(p.shape), g.dtype), []).append((p, self.momentum[i], g))
        for (dev, (rows, cols), _), items in groups.items():
            b = 0
            for size in batch_plan(len(items), rows, cols, self.workspace_limit):
                self._muon_batch(items[b:b + size], rows, cols, skip)
                b += size
        self.adam.step()
        if self.sync:
            self.check()

    def check(self):
        """Wait for the last step and raise what it reported: FloatingPointError
        if the gate refused it (nothing changed; momentum buffers it created are
        dropped, as the reference never creates them), RuntimeError if a
        bounded device wait expired."""
        for dev, err in self._err.items():
            if int(err.item()):
                err.zero_()
                raise RuntimeError("muon step: a bounded wait expired on the device")
        adam_params = [p for g in self.adam.param_groups for p in g["params"]]
        dev = adam_params[0].device if adam_params else (self.muon[0].device if self.muon else None)
        if dev is None:
            return
        st = self._record_engine(dev).read_state()
        if st.status:
            for i in self._new_momentum:
                self.momentum.pop(i, None)
            self._new_momentum = []
            if int(st.status) == _lib.MB_ERR_NONFINITE:
                raise FloatingPointError('nonfinite gradient; optimizer not updated')
            _lib.check(int(st.status), "optimizer not updated")
        self._new_momentum = []

    def _muon_batch(self, items, rows, cols, skip=None):
        """One kernel-4 step over matrices of one shape (optimizer.py:52-61 per matrix)."""
        dev = items[0][0].device
        outs = None
        if self.low_precision is not None:
            outs = []
            for p, _, _ in items:
                out = self.low_precision_copies.get(p)
                if out is None:
                    out = self.low_precision_copies[p] = torch.empty_like(p, dtype=self.low_precision)
                outs.append(out)
        err = self._err.get(dev)
        if err is None:
            err = self._err[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
        muon_step_batched([p for p, _, _ in items], [m for _, m, _ in items], [g for _, _, g in items], outs,
                          self.lr, self.weight_decay, self.ns_dtype, err, skip)

    def state_dict(self):
        return dict(momentum=self.momentum, adam=self.adam.state_dict(), lr=self.lr, weight_decay=self.weight_decay)

    def load_state_dict(self, state):
        self.momentum = {i: value.to(self.muon[i].device) for i, value in state['momentum'].items()}
        self.adam.load_state_dict(state['adam'])
        self.lr, self.weight_decay = state['lr'], state['weight_decay']
