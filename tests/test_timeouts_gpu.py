"""Device-side bounded waits that run out, on purpose and without a fault.

Kernels 1 and 2 (their bulk-staged forms) and the kernel-4 GEMM wait on
mbarriers for the copies their producer issues, and every such wait is bounded.
mb_debug_arm_fault makes the next launch of one of them withhold one unit's
copy and bound its waits by a few milliseconds: the consumers' wait for that
unit expires, the CTA stops issuing, waits (bounded) for its own copies still
in flight, frees what it holds (the GEMM's TMEM) and reports. Nothing faults,
traps or waits forever, and the process keeps a usable context:

* kernel 2 (statistics): the step is refused with MB_ERR_TIMEOUT
  (TimeoutError) and nothing changes -- w, m, v and the clocks keep their
  bits; the next step is bit-exact with the oracle;
* kernel 1 (update): the launch returns and the step state reports
  MB_ERR_TIMEOUT; a following optimizer step on fresh state is bit-exact with
  the oracle;
* kernel-4 GEMM: the error flag is raised (RuntimeError); the next GEMMs, on
  every SM, equal the result computed before the fault bit for bit, which
  they could not if the aborted CTA had left TMEM allocated or a copy landing.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LIMIT_NS = 5_000_000  # 5 ms bound for the armed launch
SHAPES = [(128, 128)] * 16 + [(4097,), (3, 67)]


@pytest.fixture(autouse=True)
def _disarm_after():
    """No armed fault outlives its test (a failure between arming and the
    launch would otherwise hit a later test's launch)."""
    yield
    from morph_b200 import _lib
    _lib.check(_lib.lib().mb_debug_arm_fault(0, -1, 0), "disarm")


def _arm(kernel, unit=0):
    from morph_b200 import _lib
    _lib.check(_lib.lib().mb_debug_arm_fault(kernel, unit, LIMIT_NS), "arm fault")


def _setup(cuda, seed):
    from morph_b200 import AdamW
    r = orc.rng(seed)
    w0 = [r.standard_normal(s, dtype=np.float32) * np.float32(.02) for s in SHAPES]
    g = [(r.standard_normal(s, dtype=np.float32) * np.float32(1e-3)).astype(np.float16) for s in SHAPES]
    params = [torch.nn.Parameter(torch.from_numpy(x.copy()).to(cuda)) for x in w0]
    for p, gg in zip(params, g):
        p.grad_dtype = None
        p.grad = torch.from_numpy(gg).to(cuda)
    opt = AdamW(params, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, max_norm=1.0, gate=True,
                low_precision=torch.bfloat16, sync=True)
    return opt, params, w0, g


def _check_one_step_against_oracle(opt, params, w0, g):
    g32 = orc.grad_prepare(np.concatenate([x.reshape(-1) for x in g]))
    total, bad = orc.sumsq(g32)
    assert bad == 0
    coef = orc.clip_coef_torch(total ** .5, 1.0)
    assert np.float32(opt.last_step()["clip_coef"]) == coef
    off = 0
    for p, x in zip(params, w0):
        n = x.size
        w = x.reshape(-1).copy()
        m, v = np.zeros_like(w), np.zeros_like(w)
        orc.adamw_(w, m, v, orc.grad_prepare(g32[off:off + n], coef=coef), orc.adamw_scalars(3e-4, .9, .95, 1e-8,
                                                                                              .1, 1))
        off += n
        st = opt.state[p]
        np.testing.assert_array_equal(p.detach().cpu().numpy().reshape(-1), w)
        np.testing.assert_array_equal(st["exp_avg"].cpu().numpy().reshape(-1), m)
        np.testing.assert_array_equal(st["exp_avg_sq"].cpu().numpy().reshape(-1), v)
        bf = opt.low_precision_copies[p].view(torch.int16).cpu().numpy().reshape(-1).view(np.uint16)
        np.testing.assert_array_equal(bf, orc.f32_to_bf16(w))
        assert int(st["step"]) == 1


def test_statistics_wait_expires_and_the_step_is_refused(cuda):
    from morph_b200 import _lib
    opt, params, w0, g = _setup(cuda, 32)
    _arm(_lib.MB_FAULT_STATS)
    t0 = time.perf_counter()
    with pytest.raises(TimeoutError):
        opt.step()
    assert time.perf_counter() - t0 < 2.0
    last = opt.last_step()
    assert last["status"] == _lib.MB_ERR_TIMEOUT and last["skipped"]
    for p, x in zip(params, w0):
        np.testing.assert_array_equal(p.detach().cpu().numpy(), x)
        assert int(opt.state[p]["step"]) == 0
        assert not opt.state[p]["exp_avg"].any() and not opt.state[p]["exp_avg_sq"].any()
    opt.step()  # nothing armed: the same step again, bit-exact
    assert opt.last_step()["status"] == 0
    _check_one_step_against_oracle(opt, params, w0, g)


def test_update_wait_expires_and_reports_timeout(cuda):
    from morph_b200 import _lib
    opt, params, w0, g = _setup(cuda, 33)
    _arm(_lib.MB_FAULT_APPLY)
    t0 = time.perf_counter()
    with pytest.raises(TimeoutError):
        opt.step()
    assert time.perf_counter() - t0 < 2.0
    assert opt.last_step()["status"] == _lib.MB_ERR_TIMEOUT
    torch.cuda.synchronize()
    opt, params, w0, g = _setup(cuda, 34)  # the context is intact: a normal step on fresh state
    opt.step()
    _check_one_step_against_oracle(opt, params, w0, g)


def test_gemm_wait_expires_raises_the_flag_and_frees_tmem(cuda):
    from morph_b200 import _lib
    from morph_b200.muon import gemm16
    gen = torch.Generator(device=cuda).manual_seed(35)
    a = torch.randn(256, 128, device=cuda, generator=gen).to(torch.bfloat16)
    b = torch.randn(512, 128, device=cuda, generator=gen).to(torch.bfloat16)
    want = gemm16(a, b)[0]
    big_a = torch.randn(4096, 1024, device=cuda, generator=gen).to(torch.bfloat16)
    big_want = gemm16(big_a, big_a)[0]  # 512 tiles: every SM takes several
    _arm(_lib.MB_FAULT_GEMM)
    t0 = time.perf_counter()
    with pytest.raises(RuntimeError, match="bounded wait"):
        gemm16(a, b)
    assert time.perf_counter() - t0 < 2.0
    for _ in range(3):
        assert torch.equal(gemm16(big_a, big_a)[0], big_want)
    assert torch.equal(gemm16(a, b)[0], want)


def test_arm_rejects_unknown_kernels_and_bounds(cuda):
    from morph_b200 import _lib
    L = _lib.lib()
    assert L.mb_debug_arm_fault(3, 0, LIMIT_NS) == _lib.MB_ERR_ARG
    assert L.mb_debug_arm_fault(_lib.MB_FAULT_APPLY, -1, LIMIT_NS) == _lib.MB_ERR_ARG
    assert L.mb_debug_arm_fault(_lib.MB_FAULT_APPLY, 0, 10) == _lib.MB_ERR_ARG
    assert L.mb_debug_arm_fault(_lib.MB_FAULT_APPLY, 0, 3_000_000_000) == _lib.MB_ERR_ARG
