"""mb_adamw_step_noalloc: the optimizer step for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc: a host framework whose
pool allocator already holds the whole GPU, or a binding that is handed fixed
device buffers and has no allocator of its own. For them the C ABI offers
mb_adamw_step_noalloc, which runs the fused step with its scratch in a fixed
array inside the library instead of a caller-allocated workspace.

These tests call it through the C ABI (ctypes) and compare it with the
allocating entry point mb_adamw_step on identical inputs, over two calls in a
row, with this suite's tolerance for the same arithmetic on the same inputs:
bit-exact. This file is named to be collected last, and it builds all of its
own state, so it passes alone in a fresh process and after the other tests.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(300, 200), (4096,), (37,), (64, 64), (5000,)]


def _setup(cuda, seed):
    from morph_b200 import _lib
    from morph_b200.optim import StepEngine
    gen = torch.Generator(device=cuda).manual_seed(seed)
    sizes = [int(torch.tensor(s).prod()) for s in SHAPES]
    n = sum(sizes)
    w = torch.randn(n, device=cuda, generator=gen) * 0.02
    m = torch.zeros_like(w)
    v = torch.zeros_like(w)
    g = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    out = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    eng = StepEngine(cuda)
    entries, off = [], 0
    for s in sizes:
        piece = w[off:off + s]
        eng.slot(piece, 0)
        entries.append((piece, m[off:off + s], v[off:off + s], g[off:off + s], out[off:off + s], 0))
        off += s
    plan = eng.prepare(entries, [(3e-4, .9, .95, 1e-8, .1, "torch")], _lib.MB_BF16, _lib.MB_BF16)
    fin = eng.finalize_opts(_lib.MB_FIN_CLIP_TORCH | _lib.MB_FIN_GATE, 1.0)
    return dict(eng=eng, plan=plan, fin=fin, w=w, m=m, v=v, g=g, out=out)


def test_noalloc_step_matches_allocating_step_on_two_calls(cuda):
    from morph_b200 import _lib
    L = _lib.lib()
    a = _setup(cuda, 7)   # reference: mb_adamw_step with a caller workspace
    b = _setup(cuda, 7)   # mb_adamw_step_noalloc with no workspace at all
    b["plan"].workspace = None
    stream = _lib.stream_handle()
    gen = torch.Generator(device=cuda).manual_seed(99)
    for call in range(2):
        grad = (torch.randn(a["g"].numel(), device=cuda, generator=gen) * (0.05 if call else 1e-3))
        a["g"].copy_(grad.to(torch.bfloat16))
        b["g"].copy_(a["g"])
        _lib.check(L.mb_adamw_step(ctypes.byref(a["plan"]), ctypes.byref(a["fin"]), stream))
        _lib.check(L.mb_adamw_step_noalloc(ctypes.byref(b["plan"]), ctypes.byref(b["fin"]), stream))
        torch.cuda.synchronize()
        for key in ("w", "m", "v"):
            assert torch.equal(a[key], b[key]), f"{key} differs on call {call + 1}"
        assert torch.equal(a["out"].view(torch.int16), b["out"].view(torch.int16))
        assert torch.equal(a["eng"].clocks, b["eng"].clocks)
        sa, sb = a["eng"].read_state(), b["eng"].read_state()
        assert (sa.norm, sa.clip_coef, sa.skip, sa.status) == (sb.norm, sb.clip_coef, sb.skip, sb.status)
        assert sa.skip == 0 and int(b["eng"].clocks[0]) == call + 1
    assert sb.clip_coef < 1.0  # the second call's gradients were clipped


def test_noalloc_takes_a_plan_at_its_segment_limit(cuda):
    """8192 segments (the scratch's capacity) run, and equal mb_adamw_step."""
    from morph_b200 import _lib
    from morph_b200.optim import StepEngine
    L = _lib.lib()
    n_segs = 8192
    sizes = [1 + (i * 7) % 13 for i in range(n_segs)]  # ragged, tiny segments
    n = sum(sizes)
    runs = []
    for _ in range(2):
        gen = torch.Generator(device=cuda).manual_seed(3)
        w = torch.randn(n, device=cuda, generator=gen) * 0.02
        m, v = torch.zeros_like(w), torch.zeros_like(w)
        g = (torch.randn(n, device=cuda, generator=gen) * 1e-3).to(torch.bfloat16)
        eng = StepEngine(cuda)
        entries, off = [], 0
        for s in sizes:
            piece = w[off:off + s]
            eng.slot(piece, 0)
            entries.append((piece, m[off:off + s], v[off:off + s], g[off:off + s], None, 0))
            off += s
        plan = eng.prepare(entries, [(3e-4, .9, .95, 1e-8, .1, "torch")], _lib.MB_BF16, _lib.MB_NONE)
        fin = eng.finalize_opts(_lib.MB_FIN_CLIP_TORCH | _lib.MB_FIN_GATE, 1.0)
        runs.append((eng, plan, fin, w, m, v, entries))
    (ea, pa, fa, wa, ma, va, _), (eb, pb, fb, wb, mb, vb, _) = runs
    pb.workspace = None
    stream = _lib.stream_handle()
    _lib.check(L.mb_adamw_step(ctypes.byref(pa), ctypes.byref(fa), stream))
    assert L.mb_adamw_step_noalloc(ctypes.byref(pb), ctypes.byref(fb), stream) == _lib.MB_OK
    torch.cuda.synchronize()
    assert torch.equal(wa, wb) and torch.equal(ma, mb) and torch.equal(va, vb)
    assert torch.equal(ea.clocks, eb.clocks) and int(eb.clocks[n_segs - 1]) == 1


def test_noalloc_requires_finalize_options(cuda):
    """fin = NULL is refused before anything is queued (mb_adamw_step would
    accept it and skip the finalize)."""
    from morph_b200 import _lib
    L = _lib.lib()
    a = _setup(cuda, 5)
    a["plan"].workspace = None
    w0 = a["w"].clone()
    rc = L.mb_adamw_step_noalloc(ctypes.byref(a["plan"]), None, _lib.stream_handle())
    assert rc == _lib.MB_ERR_ARG
    torch.cuda.synchronize()
    assert torch.equal(a["w"], w0) and int(a["eng"].clocks[0]) == 0


def test_noalloc_rejects_plans_beyond_its_scratch(cuda):
    from morph_b200 import _lib
    L = _lib.lib()
    plan = _lib.Plan()
    plan.n_segs = 8193  # one more segment than the fixed scratch holds
    fin = _lib.FinalizeOpts(0, 0, 0.0, 0.5, 2.0)
    rc = L.mb_adamw_step_noalloc(ctypes.byref(plan), ctypes.byref(fin), _lib.stream_handle())
    assert rc == _lib.MB_ERR_TOO_LARGE
    with pytest.raises(ValueError, match="no-allocation scratch"):
        _lib.check(rc)
