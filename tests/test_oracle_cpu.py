"""Pin the CPU oracle against the reference (golden vectors + installed torch).

The golden file was produced by running MORPH's own code
(tests/golden/make_golden.py). Tolerances: m, v, clocks, skips and loss-scale
sequences bit-exact; w within 1e-6 relative with an absolute floor of 1e-6 x lr
(the size of one step's update), because torch's CPU sqrt on large tensors is
MKL's and may differ from the IEEE square root by one ulp, which matters only
relative to the update, not to a near-zero weight.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as orc


def _digest(a):
    import hashlib
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


def _run_config(inject):
    masters = orc.config1_inputs()
    w = np.concatenate([x.reshape(-1) for x in masters])
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    scaler = orc.DynamicLossScale(scale=65536., growth_interval=2000)
    clock = 0
    rec = dict(w=[], m=[], v=[], export=[], scale=[], good=[], skipped=[], clock=[])
    for step in range(1, 11):
        scale = scaler.scale
        grads = orc.config1_grads(step, scale=scale)
        hit = orc.config3_injection(step) if inject else None
        if hit is not None:
            t, i, val = hit
            grads[t].reshape(-1)[i] = val
        g16 = np.concatenate([g.reshape(-1) for g in grads])
        g32 = orc.grad_prepare(g16, scale=scale)
        _, bad = orc.sumsq(g32)
        if bad:
            scaler.overflow()
            rec['skipped'].append(1)
        else:
            clock += 1
            orc.adamw_(w, m, v, g32, orc.adamw_scalars(3e-4, .9, .95, 1e-8, .1, clock))
            scaler.success()
            rec['skipped'].append(0)
        rec['w'].append(w.copy()); rec['m'].append(_digest(m)); rec['v'].append(_digest(v))
        rec['export'].append(orc.export_f16(w)); rec['scale'].append(scale)
        rec['good'].append(scaler.good_steps); rec['clock'].append(clock)
    return rec


@pytest.mark.parametrize("prefix,inject", [("cfg1_", False), ("cfg3_", True)])
def test_oracle_matches_reference_configs_1_and_3(golden, prefix, inject):
    rec = _run_config(inject)
    idx = golden['sample_index']
    np.testing.assert_array_equal(rec['skipped'], golden[prefix + 'skipped'])
    np.testing.assert_array_equal(rec['scale'], golden[prefix + 'scale_used'])
    np.testing.assert_array_equal(rec['good'], golden[prefix + 'good_steps'])
    np.testing.assert_array_equal(rec['clock'], golden[prefix + 'clock'])
    for s in range(10):
        assert (rec['m'][s] == golden[prefix + 'm_digest'][s]).all(), f"m differs at step {s + 1}"
        assert (rec['v'][s] == golden[prefix + 'v_digest'][s]).all(), f"v differs at step {s + 1}"
        np.testing.assert_allclose(rec['w'][s][idx], golden[prefix + 'w_sample'][s], rtol=1e-6, atol=1e-6 * 3e-4)
        exp = rec['export'][s][idx]
        ulps = np.abs(exp.view(np.int16).astype(np.int32) - golden[prefix + 'export_sample'][s].view(np.int16))
        assert ulps.max() <= 1 and (ulps > 0).sum() <= 2


def test_config3_scale_sequence_is_the_stated_one(golden):
    seq = golden['cfg3_scale_used']
    assert list(seq) == [65536.] * 3 + [32768.] * 4 + [16384.] * 3
    assert list(golden['cfg3_skipped']) == [0, 0, 1, 0, 0, 0, 1, 0, 0, 0]


def test_oracle_matches_reference_disk_update(golden):
    sizes = golden['disk_sizes']
    w = golden['disk_init_w'].copy()
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    for step, (g, clip) in enumerate(zip(golden['disk_grads'], golden['disk_clips']), start=1):
        off = 0
        for s in sizes:
            sl = slice(off, off + s)
            g32 = orc.grad_prepare(np.ascontiguousarray(g[sl]), coef=clip)  # disk.py:210 gradient * clip
            ww, mm, vv = w[sl].copy(), m[sl].copy(), v[sl].copy()
            orc.adamw_(ww, mm, vv, g32, orc.disk_scalars(3e-3, step))
            w[sl], m[sl], v[sl] = ww, mm, vv
            off += s
    final = golden['disk_final']
    np.testing.assert_array_equal(m, final[1])
    np.testing.assert_array_equal(v, final[2])
    np.testing.assert_allclose(w, final[0], rtol=1e-6, atol=1e-6 * 3e-3)


def test_oracle_matches_reference_row_update(golden):
    table = golden['rows_table']
    idx = golden['rows_idx']
    w, m, v = table.copy(), np.zeros_like(table), np.zeros_like(table)
    g32 = orc.grad_prepare(golden['rows_grads'])
    for step in (1, 2):
        orc.sparse_rows_(w, m, v, idx, g32, orc.disk_scalars(1e-4, step))
    final = golden['rows_final']
    np.testing.assert_array_equal(m[idx], final[1])
    np.testing.assert_array_equal(v[idx], final[2])
    np.testing.assert_allclose(w[idx], final[0], rtol=1e-6, atol=1e-6 * 1e-4)
    untouched = np.setdiff1d(np.arange(table.shape[0]), idx)
    np.testing.assert_array_equal(w[untouched], table[untouched])
    assert not m[untouched].any() and not v[untouched].any()
    with pytest.raises(IndexError):
        orc.sparse_rows_(w, m, v, np.array([table.shape[0]]), g32[:1], orc.disk_scalars(1e-4, 1))


def test_oracle_clip_coefficient_matches_torch(golden):
    for total, coef in zip(golden['clip_total_norm'], golden['clip_coef']):
        assert orc.clip_coef_torch(float(total), 1.0) == coef


def test_oracle_loss_scale_matches_reference(golden):
    events = bytes(golden['ls_events']).decode()
    seq = golden['ls_sequence']
    got = []
    s = orc.DynamicLossScale()
    s.overflow()
    got.append((s.scale, s.good_steps))
    s = orc.DynamicLossScale(scale=4., growth_interval=3)
    for e in events[1:14]:
        try:
            s.overflow() if e == 'o' else s.success()
            got.append((s.scale, s.good_steps))
        except FloatingPointError:
            got.append((-1.0, s.good_steps))
    s = orc.DynamicLossScale(scale=32768., growth_interval=2)
    for _ in range(6):
        s.success()
        got.append((s.scale, s.good_steps))
    np.testing.assert_array_equal(np.array(got), seq)


def test_oracle_orthogonalize_and_muon_match_reference(golden):
    for tag in ('wide', 'tall'):
        out = orc.orthogonalize(golden[f'muon_ortho_{tag}_in'])
        ref = golden[f'muon_ortho_{tag}_out']
        assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-5
    w = golden['muon_init'].copy()
    mom = np.zeros_like(w)
    for g in golden['muon_grads']:
        u = orc.muon_momentum_(mom, g)
        orc.muon_apply_(w, orc.orthogonalize(u), .02, .01)
    np.testing.assert_array_equal(mom, golden['muon_momentum'])
    np.testing.assert_allclose(w, golden['muon_final'], rtol=1e-5, atol=1e-7)


def test_muon_known_answer_diagonal():
    """tests/test_training.py:50-64 of the reference, on the oracle."""
    w = np.eye(2, dtype=np.float32) * np.float32(0.3)
    before = w.copy()
    mom = np.zeros_like(w)
    g = np.diag(np.array([1., 2.], np.float32))
    u = orc.muon_momentum_(mom, g)
    np.testing.assert_allclose(u, .0975 * g, rtol=1e-6)
    o = orc.orthogonalize(u)
    orc.muon_apply_(w, o, .02, .01)
    d = np.array([.0975, .195])
    d = d / (np.linalg.norm(d) + 1e-7)
    for _ in range(5):
        d = 3.4445 * d - 4.775 * d ** 3 + 2.0315 * d ** 5
    expected = before * (1 - .02 * .01) - .02 * np.diag(d).astype(np.float32)
    np.testing.assert_allclose(w, expected, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("n", [16384 * 4, 16384 * 4 + 13])
def test_oracle_matches_installed_torch_adamw(n):
    """Live pin against torch.optim.AdamW(foreach=False), the optimizer the
    reference builds at streamtrain/optimizer.py:40."""
    r = orc.rng(5)
    w0 = r.standard_normal(n, dtype=np.float32) * np.float32(.02)
    p = torch.nn.Parameter(torch.from_numpy(w0.copy()))
    opt = torch.optim.AdamW([p], lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, foreach=False)
    w, m, v = w0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    for step in range(1, 6):
        g = r.standard_normal(n, dtype=np.float32) * np.float32(1e-3)
        p.grad = torch.from_numpy(g.copy())
        opt.step()
        orc.adamw_(w, m, v, g, orc.adamw_scalars(3e-4, .9, .95, 1e-8, .1, step))
        st = opt.state[p]
        np.testing.assert_array_equal(m, st['exp_avg'].numpy())
        np.testing.assert_array_equal(v, st['exp_avg_sq'].numpy())
        np.testing.assert_allclose(w, p.detach().numpy(), rtol=1e-6, atol=1e-6 * 3e-4)
        assert (w != p.detach().numpy()).mean() < 0.02


def test_export_rejects_unrepresentable():
    with pytest.raises(ValueError):
        orc.export_f16(np.array([1.0, 65520.0], np.float32))
    with pytest.raises(ValueError):
        orc.export_f16(np.array([np.nan], np.float32))
    x = np.array([65504.0, -65504.0, 1e-8, 0.1], np.float32)
    np.testing.assert_array_equal(orc.export_f16(x), x.astype(np.float16))


def test_bf16_cast_is_round_to_nearest_even():
    r = orc.rng(3)
    x = r.standard_normal(100_000, dtype=np.float32)
    got = orc.f32_to_bf16(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(got, ref)
    np.testing.assert_array_equal(orc.bf16_to_f32(got), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_oracle_fp8_matches_reference(golden):
    codes, scales = orc.pack_fp8(golden["fp8_in"])
    np.testing.assert_array_equal(codes, golden["fp8_encoded"])
    np.testing.assert_array_equal(scales, golden["fp8_scales"])
    np.testing.assert_array_equal(orc.unpack_fp8(codes, scales, "float16"), golden["fp8_unpacked_f16"])
    x = golden["fp8_in"]
    back = orc.unpack_fp8(codes, scales, "float32")
    assert np.linalg.norm(back - x) / np.linalg.norm(x) < .04  # tests/test_fp16.py:16-19


@pytest.mark.parametrize("scale", [1.0, 1024.0, 3.7])
def test_oracle_accumulate_matches_reference_torch_ops(scale):
    """sparse_disk.py:82-110 run literally with torch on the CPU: zero_() the
    window, then destination.add_(g.detach().float() / loss_scale) per microbatch."""
    r = orc.rng(17)
    grads = [torch.from_numpy(r.standard_normal(5003).astype(np.float32) * 30).half() for _ in range(4)]
    grads[1][7] = -0.0
    dest = torch.empty(5003).fill_(123.0)
    dest.zero_()
    for g in grads:
        dest.add_(g.detach().float() / scale)
    acc = np.full(5003, 123.0, np.float32)
    for k, g in enumerate(grads):
        orc.grad_accumulate_(acc, g.float().numpy(), scale, first=k == 0)
    np.testing.assert_array_equal(acc.view(np.uint32), dest.numpy().view(np.uint32))


def test_oracle_export_chunks_follow_the_reference_order():
    x = orc.rng(18).standard_normal(10_007).astype(np.float32)
    data, raised = orc.export_f16_chunks(x, 1000)
    assert not raised and data == x.astype('<f2').tobytes()
    x[5500] = 70000.0
    data, raised = orc.export_f16_chunks(x, 1000)
    assert raised and data == x[:5000].astype('<f2').tobytes()
    x[0] = np.nan
    assert orc.export_f16_chunks(x, 1000) == (b"", True)
