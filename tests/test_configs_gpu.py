"""Parity at the BASELINE configs' own sizes, on one B200.

The smaller parity tests pin every kernel on ragged and unaligned shapes; these
run the exact plans the benchmark measures, so the segment planner, the tile
walk, the bias-correction clocks and the window arithmetic are checked at the
sizes where the headline numbers are taken:

* config 2: the 463-tensor, 4,165,459,968-parameter plan through the public
  ``morph_b200.AdamW`` (BF16 gradients N(0, 1e-4), clip at 1.0 by torch's
  rule, BF16 copy), two steps. The global norm is recomputed in full on the
  host each step (oracle FP64 sums, chunked; within 1e-12 relative, clip
  coefficient identical), and w, m, v and the BF16 copy are compared bit for
  bit with the oracle on every 16th tensor, all 168 vectors and windows at the
  start, middle and end of the [65536, 3072] embedding.
* config 4: one full-shape layer (3 x [4096, 11008] + 4 x [4096, 4096]) with
  BF16 Newton-Schulz operands, plus the AdamW group ([65536, 4096] embedding
  and 64 x [4096] vectors), two steps through ``HybridMuonAdamW``. Momentum is
  bit-exact with the oracle (optimizer.py:58), each matrix's weight delta is
  within 1e-2 relative Frobenius of a plain PyTorch FP32 restatement of
  optimizer.py:59-61 (TF32 off), and the AdamW group is bit-exact with the
  oracle.
* config 5: the [262144, 3072] table in pinned host memory with 256 MiB
  windows (7,281 rows each) and 26,214 sorted rows per step, two steps through
  ``OffloadedRowTable``. Touched rows are bit-exact with the oracle on a seeded
  sample of 512 rows plus the first and last row of every window; every
  untouched row keeps its bytes (per-row digests of w, m and v before and
  after).
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

CHUNK = 1 << 26


def _need(cuda, gib):
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info(cuda)
    if free < gib << 30:
        pytest.skip(f"needs {gib} GiB of free device memory")


def _bits(t):
    """A 16-bit CUDA tensor's bytes as a host uint16 array (the oracle's BF16 form)."""
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _normal_(t, std, gen):
    """Fill a flat tensor with N(0, std) in chunks (any dtype; drawn in FP32)."""
    n = t.numel()
    for s in range(0, n, 1 << 28):
        e = min(n, s + (1 << 28))
        t[s:e] = torch.empty(e - s, device=t.device).normal_(0.0, std, generator=gen).to(t.dtype)
    return t


def _host_norm(g):
    """sqrt of the oracle's FP64 sum of squares over a flat BF16 CUDA tensor."""
    total = 0.0
    for s in range(0, g.numel(), CHUNK):
        s_, bad = orc.sumsq(orc.grad_prepare(_bits(g[s:s + CHUNK])))
        assert bad == 0
        total += s_
    return math.sqrt(total)


# ------------------------------------------------------------------ config 2 --

def _config2_shapes():
    shapes = []
    for _ in range(42):
        shapes += [(3072, 6144)] * 3 + [(3072, 3072)] * 4 + [(3072,)] * 4
    return shapes + [(65536, 3072)]


def test_config2_full_plan_two_steps(cuda):
    from morph_b200 import AdamW
    _need(cuda, 72)
    shapes = _config2_shapes()
    sizes = [int(np.prod(s)) for s in shapes]
    total = sum(sizes)
    assert len(shapes) == 463 and total == 4165459968
    gen = torch.Generator(device=cuda).manual_seed(1234)
    wflat = _normal_(torch.empty(total, device=cuda), 0.02, gen)
    gflat = torch.empty(total, dtype=torch.bfloat16, device=cuda)
    offs = np.concatenate([[0], np.cumsum(sizes)]).tolist()
    params = []
    for shape, o, n in zip(shapes, offs, sizes):
        p = torch.nn.Parameter(wflat[o:o + n].view(shape))
        p.grad_dtype = None  # BF16 gradients on FP32 masters
        p.grad = gflat[o:o + n].view(shape)
        params.append(p)
    opt = AdamW(params, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, foreach=False, max_norm=1.0,
                gate=True, low_precision=torch.bfloat16, sync=True)
    emb = len(shapes) - 1
    # (tensor, first element, one past the last) of every checked range
    checks = [(i, 0, sizes[i]) for i in range(0, len(shapes), 16)]
    checks += [(i, 0, sizes[i]) for i, s in enumerate(shapes) if len(s) == 1]
    n_emb = sizes[emb]
    checks += [(emb, 0, 1 << 20), (emb, n_emb // 2 - (1 << 19), n_emb // 2 + (1 << 19)), (emb, n_emb - (1 << 20), n_emb)]
    ref = {}
    for i, a, b in checks:
        w = params[i].detach().reshape(-1)[a:b].cpu().numpy()
        ref[(i, a, b)] = [w, np.zeros_like(w), np.zeros_like(w)]
    for step in (1, 2):
        _normal_(gflat, 1e-4, gen)
        opt.step()
        last = opt.last_step()
        assert last["status"] == 0 and not last["skipped"]
        norm = _host_norm(gflat)
        assert abs(last["norm"] - norm) <= 1e-12 * norm
        coef = orc.clip_coef_torch(norm, 1.0)
        assert coef < 1 and np.float32(last["clip_coef"]) == coef
        sc = orc.adamw_scalars(3e-4, .9, .95, 1e-8, .1, step)
        for (i, a, b), (w, m, v) in ref.items():
            p = params[i]
            g = orc.grad_prepare(_bits(p.grad.reshape(-1)[a:b]), coef=coef)
            orc.adamw_(w, m, v, g, sc)
            st = opt.state[p]
            where = f"tensor {i} {shapes[i]} [{a}, {b}) step {step}"
            np.testing.assert_array_equal(p.detach().reshape(-1)[a:b].cpu().numpy(), w, err_msg="w " + where)
            np.testing.assert_array_equal(st["exp_avg"].reshape(-1)[a:b].cpu().numpy(), m, err_msg="m " + where)
            np.testing.assert_array_equal(st["exp_avg_sq"].reshape(-1)[a:b].cpu().numpy(), v, err_msg="v " + where)
            np.testing.assert_array_equal(_bits(opt.low_precision_copies[p].reshape(-1)[a:b]), orc.f32_to_bf16(w),
                                          err_msg="bf16 copy " + where)
        clocks = opt._engine.clocks[:len(params)].cpu()
        assert bool((clocks == step).all())


# ------------------------------------------------------------------ config 4 --

class _Config4Layer(torch.nn.Module):
    """One config-4 layer (3 x [4096, 11008] + 4 x [4096, 4096] Linear weights)
    and the AdamW group: a [65536, 4096] embedding and 64 vectors of 4096
    (32 LayerNorms' weights and biases)."""

    def __init__(self):
        super().__init__()
        self.embedding = torch.nn.Embedding(65536, 4096)
        self.ffn = torch.nn.ModuleList([torch.nn.Linear(11008, 4096, bias=False) for _ in range(3)])
        self.ssm = torch.nn.ModuleList([torch.nn.Linear(4096, 4096, bias=False) for _ in range(4)])
        self.norms = torch.nn.ModuleList([torch.nn.LayerNorm(4096) for _ in range(32)])


def _fp32_muon_reference(w, mom, g, lr, wd):
    """optimizer.py:58-61 in plain PyTorch FP32 on the GPU (TF32 off): momentum
    lerp, Nesterov blend, orthogonalize (optimizer.py:13-22), shape scale,
    decoupled weight decay. Returns the new weights."""
    mom = mom.lerp(g.float(), .05)
    x = g.float().lerp(mom, .95)
    transpose = x.shape[0] > x.shape[1]
    if transpose:
        x = x.T
    x = x / (x.norm() + 1e-7)
    for _ in range(5):
        a = x @ x.T
        x = 3.4445 * x + (-4.775 * a + 2.0315 * (a @ a)) @ x
    u = x.T if transpose else x
    u = u * max(1, w.shape[0] / w.shape[1]) ** .5
    return w * (1 - lr * wd) - lr * u


def test_config4_full_shape_layer_bf16_two_steps(cuda):
    from morph_b200 import HybridMuonAdamW
    _need(cuda, 24)
    torch.manual_seed(4)
    model = _Config4Layer().to(cuda)
    lr, muon_lr, wd = 3e-4, .02, .01
    opt = HybridMuonAdamW(model, lr=lr, muon_lr=muon_lr, weight_decay=wd, ns_dtype="bf16")
    assert len(opt.muon) == 7
    adam_params = opt.adam.param_groups[0]["params"]
    assert len(adam_params) == 65
    gen = torch.Generator(device=cuda).manual_seed(44)
    adam_ref = {id(p): [p.detach().reshape(-1).cpu().numpy(), None, None] for p in adam_params}
    for v in adam_ref.values():
        v[1], v[2] = np.zeros_like(v[0]), np.zeros_like(v[0])
    mom_ref = [np.zeros(p.numel(), np.float32) for p in opt.muon]
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for step in (1, 2):
            for p in opt.muon + adam_params:
                p.grad_dtype = None  # BF16 gradients on FP32 masters
                p.grad = _normal_(torch.empty(p.shape, dtype=torch.bfloat16, device=cuda).reshape(-1), 1e-4,
                                  gen).view(p.shape)
            w_before = [p.detach().clone() for p in opt.muon]
            mom_before = [opt.momentum[i].clone() if i in opt.momentum else torch.zeros_like(p)
                          for i, p in enumerate(opt.muon)]
            opt.step()
            torch.cuda.synchronize()
            for i, p in enumerate(opt.muon):
                g32 = orc.grad_prepare(_bits(p.grad.reshape(-1)))
                orc.muon_momentum_(mom_ref[i], g32)
                np.testing.assert_array_equal(opt.momentum[i].reshape(-1).cpu().numpy(), mom_ref[i],
                                              err_msg=f"momentum of matrix {i} {tuple(p.shape)} step {step}")
                want = _fp32_muon_reference(w_before[i], mom_before[i], p.grad, muon_lr, wd)
                d_ref = want - w_before[i]
                err = float((p.detach() - w_before[i] - d_ref).norm() / d_ref.norm())
                assert err < 1e-2, (i, tuple(p.shape), step, err)
            sc = orc.adamw_scalars(lr, .9, .95, 1e-8, wd, step)
            for p in adam_params:
                w, m, v = adam_ref[id(p)]
                orc.adamw_(w, m, v, orc.grad_prepare(_bits(p.grad.reshape(-1))), sc)
                st = opt.adam.state[p]
                where = f"AdamW {tuple(p.shape)} step {step}"
                np.testing.assert_array_equal(p.detach().reshape(-1).cpu().numpy(), w, err_msg="w " + where)
                np.testing.assert_array_equal(st["exp_avg"].reshape(-1).cpu().numpy(), m, err_msg="m " + where)
                np.testing.assert_array_equal(st["exp_avg_sq"].reshape(-1).cpu().numpy(), v,
                                              err_msg="v " + where)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


# ------------------------------------------------------------------ config 5 --

def _row_digests(plane):
    """Per-row (sum, xor) of a [rows, cols] FP32 host tensor's 64-bit words."""
    words = plane.view(torch.int64)
    return words.sum(1), torch.from_numpy(np.bitwise_xor.reduce(words.numpy(), axis=1))


def test_config5_full_table_two_steps(cuda):
    from morph_b200.offload import OffloadedRowTable
    _need(cuda, 4)
    rows, cols, k, lr = 262144, 3072, 26214, 1e-4
    table = OffloadedRowTable(rows, cols, device=cuda)  # 256 MiB windows
    assert table.window_rows == 7281
    gen = torch.Generator(device=cuda).manual_seed(5)
    for s in range(0, rows, 16384):
        table.w[s:s + 16384].copy_(torch.empty(16384, cols, device=cuda).normal_(0.0, .02, generator=gen))
    r = orc.rng(55)
    for step in (1, 2):
        cpu_gen = torch.Generator().manual_seed(1234 + step)
        idx = torch.randperm(rows, generator=cpu_gen)[:k].sort().values
        grads = torch.empty(k, cols, dtype=torch.float16, device=cuda).normal_(0.0, 1e-3, generator=gen)
        # checked positions of the index list: a seeded sample and both ends of every window
        pos = set(r.choice(k, 512, replace=False).tolist())
        for a in range(0, k, table.window_rows):
            pos |= {a, min(k, a + table.window_rows) - 1}
        pos = np.array(sorted(pos))
        rows_chk = idx.numpy()[pos]
        before = [t.numpy()[rows_chk].copy() for t in (table.w, table.m, table.v)]
        untouched = torch.ones(rows, dtype=torch.bool)
        untouched[idx] = False
        dig0 = [_row_digests(t) for t in (table.w, table.m, table.v)]
        table.step(idx.to(cuda), grads, step, lr, clip=1.0)
        table.synchronize(timeout=120)
        w, m, v = before
        g32 = orc.grad_prepare(grads.cpu().numpy()[pos])
        orc.sparse_rows_(w, m, v, np.arange(pos.size, dtype=np.int64), g32, orc.disk_scalars(lr, step))
        for name, t, want in (("w", table.w, w), ("m", table.m, m), ("v", table.v, v)):
            np.testing.assert_array_equal(t.numpy()[rows_chk], want, err_msg=f"{name} step {step}")
        for (s0, x0), t in zip(dig0, (table.w, table.m, table.v)):
            s1, x1 = _row_digests(t)
            assert torch.equal(s0[untouched], s1[untouched]) and torch.equal(x0[untouched], x1[untouched])
            assert not torch.equal(s0[~untouched], s1[~untouched])
