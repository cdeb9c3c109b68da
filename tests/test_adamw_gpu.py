"""Parity of the fused AdamW kernels (C-ABI via morph_b200.AdamW) with the oracle.

Bit-exact: w, m, v, clocks, the FP16/BF16 copies, skip decisions and the
loss-scale sequence against the CPU oracle on the same inputs. Against the
reference's golden vectors: m and v digests bit-exact, w within 1e-6 relative
with a floor of 1e-6 x lr (the reference's CPU sqrt is MKL's, see
tests/test_oracle_cpu.py).
"""
import hashlib

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _digest(a):
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


def _flat(ts):
    return np.concatenate([t.detach().float().cpu().numpy().reshape(-1) for t in ts])


def _config1(cuda, inject):
    from morph_b200 import AdamW, DynamicLossScale
    masters = orc.config1_inputs()
    params = [torch.nn.Parameter(torch.from_numpy(w.copy()).to(cuda)) for w in masters]
    for p in params:
        p.grad_dtype = None  # FP16 gradients on FP32 masters
    scaler = DynamicLossScale(scale=65536., growth_interval=2000, device=cuda)
    opt = AdamW(params, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, foreach=False,
                loss_scale=scaler, low_precision=torch.float16)
    # oracle twin
    w = np.concatenate([x.reshape(-1) for x in masters])
    m, v = np.zeros_like(w), np.zeros_like(w)
    oscale = orc.DynamicLossScale(scale=65536., growth_interval=2000)
    clock = 0
    rec = []
    for step in range(1, 11):
        scale = oscale.scale
        grads = orc.config1_grads(step, scale=scale)
        hit = orc.config3_injection(step) if inject else None
        if hit is not None:
            t, i, val = hit
            grads[t].reshape(-1)[i] = val
        for p, g in zip(params, grads):
            p.grad = torch.from_numpy(g).to(cuda)
        opt.step()
        g32 = orc.grad_prepare(np.concatenate([g.reshape(-1) for g in grads]), scale=scale)
        if orc.sumsq(g32)[1]:
            oscale.overflow()
            skipped = 1
        else:
            clock += 1
            orc.adamw_(w, m, v, g32, orc.adamw_scalars(3e-4, .9, .95, 1e-8, .1, clock))
            oscale.success()
            skipped = 0
        last = scaler.last_step()
        gw = _flat(params)
        gm = _flat([opt.state[p]["exp_avg"] for p in params])
        gv = _flat([opt.state[p]["exp_avg_sq"] for p in params])
        half = np.concatenate([opt.low_precision_copies[p].cpu().numpy().reshape(-1) for p in params])
        np.testing.assert_array_equal(gw, w, err_msg=f"w step {step}")
        np.testing.assert_array_equal(gm, m, err_msg=f"m step {step}")
        np.testing.assert_array_equal(gv, v, err_msg=f"v step {step}")
        if not skipped:
            np.testing.assert_array_equal(half, orc.export_f16(w), err_msg=f"f16 copy step {step}")
        assert last["skipped"] == bool(skipped)
        assert last["step_scale"] == scale
        assert scaler.scale == oscale.scale and scaler.good_steps == oscale.good_steps
        assert all(int(opt.state[p]["step"]) == clock for p in params)
        rec.append(dict(w=gw, m=_digest(gm), v=_digest(gv), scale=scale, skipped=skipped,
                        good=scaler.good_steps, clock=clock))
    return rec


@pytest.mark.parametrize("prefix,inject", [("cfg1_", False), ("cfg3_", True)])
def test_config_1_and_3_bit_exact_vs_oracle_and_reference(cuda, golden, prefix, inject):
    rec = _config1(cuda, inject)
    idx = golden["sample_index"]
    assert [r["skipped"] for r in rec] == list(golden[prefix + "skipped"])
    assert [r["scale"] for r in rec] == list(golden[prefix + "scale_used"])
    assert [r["good"] for r in rec] == list(golden[prefix + "good_steps"])
    assert [r["clock"] for r in rec] == list(golden[prefix + "clock"])
    for s, r in enumerate(rec):
        assert (r["m"] == golden[prefix + "m_digest"][s]).all()
        assert (r["v"] == golden[prefix + "v_digest"][s]).all()
        np.testing.assert_allclose(r["w"][idx], golden[prefix + "w_sample"][s], rtol=1e-6, atol=1e-6 * 3e-4)


SIZES = [1, 3, 5, 2047, 2048, 2049, 4100, 70001]


@pytest.mark.parametrize("gdt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("odt", [None, torch.bfloat16, torch.float16])
def test_ragged_sizes_dtypes_and_unaligned_views(cuda, gdt, odt):
    from morph_b200 import AdamW
    r = orc.rng(11)
    base = torch.from_numpy(r.standard_normal(sum(SIZES) + 8, dtype=np.float32) * np.float32(.02)).to(cuda)
    params = []
    off = 1  # the first views start 4 bytes past a 16-byte boundary: scalar path
    for i, n in enumerate(SIZES):
        if i < 3:
            params.append(torch.nn.Parameter(base[off:off + n]))
            off += n
        else:
            params.append(torch.nn.Parameter(torch.from_numpy(r.standard_normal(n, dtype=np.float32)
                                                              * np.float32(.02)).to(cuda)))
    for p in params:
        p.grad_dtype = None
    opt = AdamW(params, lr=1e-3, betas=(.9, .999), eps=1e-8, weight_decay=1e-2, low_precision=odt)
    ws = [p.detach().cpu().numpy().copy() for p in params]
    ms = [np.zeros_like(x) for x in ws]
    vs = [np.zeros_like(x) for x in ws]
    for step in range(1, 4):
        gs = [(r.standard_normal(p.numel(), dtype=np.float32) * np.float32(1e-3)) for p in params]
        for p, g in zip(params, gs):
            p.grad = torch.from_numpy(g).to(cuda).to(gdt)
        opt.step()
        for i, p in enumerate(params):
            g32 = p.grad.float().cpu().numpy()
            orc.adamw_(ws[i], ms[i], vs[i], g32, orc.adamw_scalars(1e-3, .9, .999, 1e-8, 1e-2, step))
            np.testing.assert_array_equal(p.detach().cpu().numpy(), ws[i])
            np.testing.assert_array_equal(opt.state[p]["exp_avg"].cpu().numpy(), ms[i])
            np.testing.assert_array_equal(opt.state[p]["exp_avg_sq"].cpu().numpy(), vs[i])
            if odt is not None:
                got = opt.low_precision_copies[p].cpu()
                want = torch.from_numpy(ws[i]).to(odt)
                assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("mode", ["torch", "disk"])
def test_fused_clip_matches_reference_rules(cuda, mode):
    from morph_b200 import AdamW
    r = orc.rng(21)
    shapes = [(300, 200), (4096,), (37,), (64, 64)]
    w0 = [r.standard_normal(s, dtype=np.float32) * np.float32(.02) for s in shapes]
    params = [torch.nn.Parameter(torch.from_numpy(x.copy()).to(cuda)) for x in w0]
    for p in params:
        p.grad_dtype = None
    opt = AdamW(params, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, max_norm=1.0, clip_mode=mode)
    ws = [x.reshape(-1).copy() for x in w0]
    ms = [np.zeros_like(x) for x in ws]
    vs = [np.zeros_like(x) for x in ws]
    for step, gscale in enumerate((1e-2, 1e-4, 5e-2), start=1):
        gs = [(r.standard_normal(s, dtype=np.float32) * np.float32(gscale)).astype(np.float32) for s in shapes]
        bf = [torch.from_numpy(g).to(torch.bfloat16) for g in gs]
        for p, g in zip(params, bf):
            p.grad = g.to(cuda)
        opt.step()
        g32 = [g.float().numpy().reshape(-1) for g in bf]
        total, _ = orc.sumsq(np.concatenate(g32))
        norm = total ** 0.5
        want = orc.clip_coef_torch(norm, 1.0) if mode == "torch" else orc.clip_coef_disk(norm, 1.0)
        got = opt.last_step()
        assert abs(got["norm"] - norm) <= 1e-12 * max(norm, 1.0)
        assert abs(np.float32(got["clip_coef"]) - want) <= np.spacing(want)
        if mode == "torch":  # against torch's own clip_grad_norm_ on the CPU
            # a one-element probe gradient 2**-60 (negligible in the norm) reads
            # torch's applied coefficient back exactly: probe * coef * 2**60
            ref = [torch.nn.Parameter(torch.zeros(s)) for s in shapes] + [torch.nn.Parameter(torch.zeros(1))]
            for q, g in zip(ref, bf):
                q.grad = g.float().reshape(q.shape)
            ref[-1].grad = torch.full((1,), 2.0 ** -60)
            torch.nn.utils.clip_grad_norm_(ref, 1.0)
            tcoef = float(ref[-1].grad[0]) * 2.0 ** 60
            assert abs(got["clip_coef"] - tcoef) <= 2e-6 * tcoef
        coef = np.float32(got["clip_coef"])
        for i, p in enumerate(params):
            gc = orc.grad_prepare(g32[i], coef=coef)
            orc.adamw_(ws[i], ms[i], vs[i], gc, orc.adamw_scalars(3e-4, .9, .95, 1e-8, .1, step))
            np.testing.assert_array_equal(p.detach().cpu().numpy().reshape(-1), ws[i])
            np.testing.assert_array_equal(opt.state[p]["exp_avg_sq"].cpu().numpy().reshape(-1), vs[i])


def test_gate_raises_and_leaves_state_bit_identical(cuda):
    from morph_b200 import AdamW
    params = [torch.nn.Parameter(torch.randn(1000, device=cuda)) for _ in range(3)]
    opt = AdamW(params, lr=.003, betas=(.9, .95), weight_decay=.01, gate=True)
    for p in params:
        p.grad = torch.full_like(p, .2)
    opt.step()
    before = [(p.detach().clone(), opt.state[p]["exp_avg"].clone(), opt.state[p]["exp_avg_sq"].clone(),
               int(opt.state[p]["step"])) for p in params]
    params[1].grad[17] = float("nan")
    with pytest.raises(FloatingPointError):
        opt.step()
    for p, (w, m, v, c) in zip(params, before):
        assert torch.equal(p, w) and torch.equal(opt.state[p]["exp_avg"], m)
        assert torch.equal(opt.state[p]["exp_avg_sq"], v) and int(opt.state[p]["step"]) == c == 1


def test_overflow_at_minimum_scale_raises(cuda):
    from morph_b200 import AdamW, DynamicLossScale
    p = torch.nn.Parameter(torch.ones(10, device=cuda))
    p.grad_dtype = None
    scaler = DynamicLossScale(scale=1., growth_interval=5, device=cuda)
    opt = AdamW([p], loss_scale=scaler, sync=True)
    p.grad = torch.full((10,), float("inf"), device=cuda, dtype=torch.float16)
    with pytest.raises(FloatingPointError, match="minimum loss scale"):
        opt.step()
    assert scaler.scale == 1. and torch.equal(p, torch.ones(10, device=cuda))


def test_loss_scale_host_methods_match_reference(cuda, golden):
    from morph_b200 import DynamicLossScale
    events = bytes(golden["ls_events"]).decode()
    got = []
    s = DynamicLossScale(device=cuda)
    s.overflow()
    got.append((s.scale, s.good_steps))
    s = DynamicLossScale(scale=4., growth_interval=3, device=cuda)
    for e in events[1:14]:
        try:
            s.overflow() if e == "o" else s.success()
            got.append((s.scale, s.good_steps))
        except FloatingPointError:
            got.append((-1.0, s.good_steps))
    s = DynamicLossScale(scale=32768., growth_interval=2, device=cuda)
    for _ in range(6):
        s.success()
        got.append((s.scale, s.good_steps))
    np.testing.assert_array_equal(np.array(got), golden["ls_sequence"])
    assert s.state_dict() == dict(scale=65536., good_steps=0, growth_interval=2)


def test_state_dict_round_trips_through_torch_adamw(cuda):
    from morph_b200 import AdamW
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(257, 3, device=cuda)), torch.nn.Parameter(torch.randn(11, device=cuda))]
    opt = AdamW(params, lr=2e-3, betas=(.9, .95), weight_decay=.05)
    for _ in range(3):
        for p in params:
            p.grad = torch.randn_like(p) * 1e-2
        opt.step()
    sd = opt.state_dict()
    assert all(st["step"].device.type == "cpu" and st["step"].dtype == torch.float32 and float(st["step"]) == 3
               for st in sd["state"].values())
    cpu_params = [torch.nn.Parameter(p.detach().cpu().clone()) for p in params]
    ref = torch.optim.AdamW(cpu_params, lr=2e-3, betas=(.9, .95), weight_decay=.05, foreach=False)
    ref.load_state_dict({**sd, "state": {k: {kk: vv.cpu() for kk, vv in v.items()} for k, v in sd["state"].items()}})
    opt2 = AdamW([torch.nn.Parameter(p.detach().clone()) for p in params], lr=2e-3, betas=(.9, .95), weight_decay=.05)
    opt2.load_state_dict(ref.state_dict())
    g = [torch.randn(p.shape) * 1e-2 for p in params]
    for q, gg in zip(cpu_params, g):
        q.grad = gg.clone()
    ref.step()
    for q, gg in zip(opt2.param_groups[0]["params"], g):
        q.grad = gg.to(cuda)
    opt2.step()
    for q, r in zip(opt2.param_groups[0]["params"], cpu_params):
        torch.testing.assert_close(q.detach().cpu(), r.detach(), rtol=1e-6, atol=1e-6 * 2e-3)
        assert int(opt2.state[q]["step"]) == 4


def test_hundred_steps_against_torch_adamw_on_cpu(cuda):
    """The north star's drift bound: config-1 shapes (64 x [128, 128]), FP16
    grads x 2^16 unscaled on the device, 100 steps against torch.optim.AdamW
    (foreach=False, the reference's optimizer) on the CPU with the same unscaled
    grads: masters and moments within 1e-5 relative after 100 steps (1e-6 per
    step), and bit-exact with the oracle throughout."""
    from morph_b200 import AdamW, DynamicLossScale
    r = orc.rng(101)
    shapes = [(128, 128)] * 64
    init = [r.standard_normal(s).astype(np.float32) * np.float32(.02) for s in shapes]
    ps = [torch.nn.Parameter(torch.from_numpy(x).to(cuda)) for x in init]
    for p in ps:
        p.grad_dtype = None
    ref = [torch.nn.Parameter(torch.from_numpy(x.copy())) for x in init]
    scaler = DynamicLossScale(scale=65536.0, growth_interval=2000, device=cuda)
    opt = AdamW(ps, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, loss_scale=scaler)
    topt = torch.optim.AdamW(ref, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, foreach=False)
    for step in range(1, 101):
        gs = [(torch.from_numpy(r.standard_normal(s).astype(np.float32) * np.float32(1e-3)) * 65536.0).half()
              for s in shapes]
        for p, q, g in zip(ps, ref, gs):
            p.grad = g.to(cuda)
            q.grad = g.float() / 65536.0
        opt.step()
        topt.step()
        if step in (1, 100):
            tol = 1e-6 if step == 1 else 1e-5
            for p, q in zip(ps, ref):
                np.testing.assert_allclose(p.detach().cpu().numpy(), q.detach().numpy(), rtol=tol, atol=tol * 3e-4)
                np.testing.assert_allclose(opt.state[p]["exp_avg"].cpu().numpy(), topt.state[q]["exp_avg"].numpy(),
                                           rtol=tol, atol=0)
                np.testing.assert_allclose(opt.state[p]["exp_avg_sq"].cpu().numpy(),
                                           topt.state[q]["exp_avg_sq"].numpy(), rtol=tol, atol=0)
    assert scaler.scale == 65536.0 and not scaler.last_step()["skipped"]
