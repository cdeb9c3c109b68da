"""Generate the golden fixtures by running the MORPH reference itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/MORPH

It imports the reference's own modules (streamtrain.optimizer,
streamtrain.precision, streamtrain.disk, morph) and records what they compute
on seeded inputs into ``tests/golden/golden.npz``. The tests read only that
file; nothing at test time touches the reference checkout.

Cases:
  cfg1_*  config 1 through the reference HybridMuonAdamW's AdamW
          (streamtrain/optimizer.py:40,62): 64 x [128,128] FP32, FP16 grads x 2^16
          unscaled as g.float()/scale, lr 3e-4, betas (.9,.95), eps 1e-8, wd .1,
          10 steps, FP16 export after each step.
  cfg3_*  config 3: same shapes, scale 2^16, growth 2000; +inf at step 3 and NaN
          at step 7; the reference gate raises (optimizer.py:50-51), the
          reference DynamicLossScale backs off (precision.py:9-11).
  disk_*  DiskState.update (streamtrain/disk.py:203-223) on a tiny model's
          parameters, 3 steps, clip .25/1/.1, chunk_elements 7 (exercises chunks).
  rows_*  the row-sparse oracle: DiskState.update on a gathered [k, cols] tensor.
  muon_*  HybridMuonAdamW on a small Linear (optimizer.py:52-61), 3 steps, and
          orthogonalize (optimizer.py:13-22) on rectangular inputs.
  clip_*  torch clip_grad_norm_ (morph/training/runner.py:100) coefficients.
  ls_*    DynamicLossScale sequences (tests/test_fp16.py:59-72 pattern and
          growth/cap/minimum-scale behaviour).
  fp8_*   pack_fp8 / unpack_fp8 (streamtrain/precision.py:24-37) block transport.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as orc  # noqa: E402  (seeded inputs only)

SAMPLE = np.random.Generator(np.random.PCG64(77)).choice(64 * 128 * 128, 4096, replace=False)
SAMPLE.sort()


def digest(a: np.ndarray) -> np.ndarray:
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


def run_config(out, prefix, inject):
    from streamtrain.optimizer import HybridMuonAdamW
    from streamtrain.precision import DynamicLossScale
    masters = orc.config1_inputs()
    model = torch.nn.ParameterList([torch.nn.Parameter(torch.from_numpy(w.copy())) for w in masters])
    opt = HybridMuonAdamW(model, lr=3e-4, weight_decay=0.1)
    assert not opt.muon and len(opt.adam.param_groups[0]['params']) == 64
    scaler = DynamicLossScale(scale=65536., growth_interval=2000)
    scales, goods, skipped = [], [], []
    w_s, m_d, v_d, w_d, e_s, st = [], [], [], [], [], []
    for step in range(1, 11):
        scale_used = scaler.scale
        grads = orc.config1_grads(step, scale=scale_used)
        hit = orc.config3_injection(step) if inject else None
        if hit is not None:
            t, i, val = hit
            grads[t].reshape(-1)[i] = val
        for p, g in zip(model, grads):
            # engine.py:207 / sparse_disk.py:107: g.float() / loss_scale
            p.grad = torch.from_numpy(g).float() / scale_used
        try:
            opt.step()
            scaler.success()
            skipped.append(0)
        except FloatingPointError:
            scaler.overflow()
            skipped.append(1)
        scales.append(scale_used)
        goods.append(scaler.good_steps)
        w = torch.cat([p.detach().flatten() for p in model]).numpy()
        state = [opt.adam.state[p] for p in model] if opt.adam.state else []
        m = torch.cat([s['exp_avg'].flatten() for s in state]).numpy() if state else np.zeros_like(w)
        v = torch.cat([s['exp_avg_sq'].flatten() for s in state]).numpy() if state else np.zeros_like(w)
        st.append(float(state[0]['step']) if state else 0.0)
        w_s.append(w[SAMPLE].copy())
        w_d.append(digest(w))
        m_d.append(digest(m))
        v_d.append(digest(v))
        e_s.append(w.astype(np.float16)[SAMPLE].copy())  # export.py:34 astype('<f2')
    out[prefix + 'w_sample'] = np.stack(w_s)
    out[prefix + 'w_digest'] = np.stack(w_d)
    out[prefix + 'm_digest'] = np.stack(m_d)
    out[prefix + 'v_digest'] = np.stack(v_d)
    out[prefix + 'export_sample'] = np.stack(e_s)
    out[prefix + 'scale_used'] = np.array(scales)
    out[prefix + 'good_steps'] = np.array(goods)
    out[prefix + 'skipped'] = np.array(skipped)
    out[prefix + 'clock'] = np.array(st)
    out['sample_index'] = SAMPLE


def run_disk(out):
    from morph import MorphConfig, MorphModel
    from streamtrain.disk import DiskState
    torch.manual_seed(5)
    cfg = MorphConfig(vocab_size=16, d_model=8, num_layers=1, d_ff=16, d_state=2, head_dim=4)
    model = MorphModel(cfg)
    with tempfile.TemporaryDirectory() as tmp:
        store = DiskState.create(os.path.join(tmp, 's'), model, source=model)
        names = [n for n, _ in model.named_parameters()]
        sizes = [store.entries[n]['size'] for n in names]
        r = orc.rng(99)
        init = np.concatenate([np.fromfile(os.path.join(store.root, store.entries[n]['file']), np.float32)
                               .reshape(3, -1)[0] for n in names])
        grads, clips = [], [.25, 1., .1]
        for step, clip in zip((1, 2, 3), clips):
            g = r.standard_normal(sum(sizes), dtype=np.float32) * np.float32(1e-2)
            grads.append(g)
            off = 0
            for n, s in zip(names, sizes):
                store.update(n, torch.from_numpy(g[off:off + s].copy()), step, 3e-3, clip, chunk_elements=7)
                off += s
        final = np.concatenate([np.fromfile(os.path.join(store.root, store.entries[n]['file']), np.float32)
                                .reshape(3, -1) for n in names], axis=1)
    out['disk_sizes'] = np.array(sizes)
    out['disk_init_w'] = init
    out['disk_grads'] = np.stack(grads)
    out['disk_clips'] = np.array(clips)
    out['disk_final'] = final  # (3, total): w, m, v


def run_rows(out):
    """Row-sparse oracle: DiskState.update on the gathered [k, cols] rows."""
    from streamtrain.disk import DiskState
    rows, cols, k = 64, 96, 9
    r = orc.rng(2024)
    table = (r.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    idx = np.sort(r.choice(rows, k, replace=False)).astype(np.int64)
    grads = (r.standard_normal((k, cols), dtype=np.float32) * np.float32(1e-3)).astype(np.float16)

    class Gathered(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.rows = torch.nn.Parameter(torch.from_numpy(table[idx].copy()))
            self.config = type('C', (), {'to_dict': lambda self: {}})()

    model = Gathered()
    with tempfile.TemporaryDirectory() as tmp:
        store = DiskState.create(os.path.join(tmp, 's'), model, source=model)
        for step in (1, 2):
            store.update('rows', torch.from_numpy(grads).float() * 1.0, step, 1e-4, 1.0)
        final = np.fromfile(os.path.join(store.root, store.entries['rows']['file']), np.float32).reshape(3, k, cols)
    out['rows_table'] = table
    out['rows_idx'] = idx
    out['rows_grads'] = grads
    out['rows_final'] = final


def run_muon(out):
    from streamtrain.optimizer import HybridMuonAdamW, orthogonalize
    r = orc.rng(31)
    for tag, shape in (('wide', (48, 80)), ('tall', (80, 48))):
        g = r.standard_normal(shape, dtype=np.float32)
        out[f'muon_ortho_{tag}_in'] = g
        out[f'muon_ortho_{tag}_out'] = orthogonalize(torch.from_numpy(g)).numpy()
    model = torch.nn.Sequential(torch.nn.Linear(80, 48, bias=False), torch.nn.LayerNorm(48))
    with torch.no_grad():
        model[0].weight.copy_(torch.from_numpy(r.standard_normal((48, 80), dtype=np.float32) * np.float32(.02)))
    init = model[0].weight.detach().numpy().copy()
    opt = HybridMuonAdamW(model, lr=.02)
    grads = []
    for _ in range(3):
        g = r.standard_normal((48, 80), dtype=np.float32) * np.float32(1e-2)
        grads.append(g)
        model[0].weight.grad = torch.from_numpy(g.copy())
        for p in opt.adam.param_groups[0]['params']:
            p.grad = torch.zeros_like(p)
        opt.step()
    out['muon_init'] = init
    out['muon_grads'] = np.stack(grads)
    out['muon_final'] = model[0].weight.detach().numpy()
    out['muon_momentum'] = opt.momentum[0].numpy()


def run_clip(out):
    """clip_grad_norm_ as called at morph/training/runner.py:100. A one-element
    parameter with gradient 1.0 reads the applied coefficient back exactly."""
    r = orc.rng(7)
    norms, coefs = [], []
    for scale in (1e-4, 1e-2, 0.2, 1.0, 3.0):
        ps = [torch.nn.Parameter(torch.zeros(n)) for n in (1000, 37, 4096, 1)]
        for p in ps[:3]:
            p.grad = torch.from_numpy(r.standard_normal(p.numel(), dtype=np.float32) * np.float32(scale))
        ps[3].grad = torch.ones(1)
        total = torch.nn.utils.clip_grad_norm_(ps, 1.0, error_if_nonfinite=True)
        norms.append(float(total))
        coefs.append(float(ps[3].grad[0]))
    out['clip_total_norm'] = np.array(norms, np.float32)
    out['clip_coef'] = np.array(coefs, np.float32)


def run_loss_scale(out):
    from streamtrain.precision import DynamicLossScale
    seq = []
    s = DynamicLossScale()
    s.overflow()                      # tests/test_fp16.py:72 pattern: 128 -> 64
    seq.append((s.scale, s.good_steps))
    s = DynamicLossScale(scale=4., growth_interval=3)
    for event in 'sssosssssoooo':
        try:
            s.overflow() if event == 'o' else s.success()
            seq.append((s.scale, s.good_steps))
        except FloatingPointError:
            seq.append((-1.0, s.good_steps))
    s = DynamicLossScale(scale=32768., growth_interval=2)
    for _ in range(6):
        s.success()
        seq.append((s.scale, s.good_steps))
    out['ls_sequence'] = np.array(seq, np.float64)
    out['ls_events'] = np.frombuffer(b'o' + b'sssosssssoooo' + b'ssssss', np.uint8)


def run_fp8(out):
    """precision.py:24-37 pack_fp8 / unpack_fp8 on seeded inputs (a ragged size,
    an all-zero block, a block with one huge value)."""
    from streamtrain.precision import pack_fp8, unpack_fp8
    r = orc.rng(519)
    x = r.standard_normal(519 + 256 * 3, dtype=np.float32)
    x[256:512] = 0.0
    x[600] = 3.0e4
    enc, scales = pack_fp8(torch.from_numpy(x))
    out['fp8_in'] = x
    out['fp8_encoded'] = enc.numpy()
    out['fp8_scales'] = scales.numpy()
    out['fp8_unpacked_f16'] = unpack_fp8(enc, scales, torch.float16).numpy()
    out['fp8_unpacked_f32'] = unpack_fp8(enc, scales, torch.float32).numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', default=os.environ.get('MORPH_REFERENCE', ''))
    ap.add_argument('--out', default=os.path.join(HERE, 'golden.npz'))
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        raise SystemExit('pass --reference <MORPH checkout>')
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    torch.set_num_threads(1)
    out = {}
    run_config(out, 'cfg1_', inject=False)
    run_config(out, 'cfg3_', inject=True)
    run_disk(out)
    run_rows(out)
    run_muon(out)
    run_clip(out)
    run_loss_scale(out)
    run_fp8(out)
    np.savez_compressed(args.out, **out)
    print('wrote', args.out, os.path.getsize(args.out), 'bytes,', len(out), 'arrays')


if __name__ == '__main__':
    main()
