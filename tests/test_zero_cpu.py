"""ZeRO-1 host logic on CPU with world_size 2 (gloo): shard bounds, pieces that
straddle shard edges, the all-reduced {sumsq, nonfinite} record (one clip and
skip decision on every rank) and the in-place all-gather of the BF16 weights.

The kernels are replaced by an oracle-backed test double defined here (the
product class always uses the CUDA library); the 2-rank result must equal the
1-rank result."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from morph_b200.zero import ZeroAdamW, shard_bounds, shard_pieces

SHAPES = [(37,), (100, 3), (64, 64), (5,), (1000,)]
LR, BETAS, EPS, WD = 3e-4, (.9, .95), 1e-8, .1


class OracleBackend:
    """Test double of CudaZeroBackend computing with the CPU oracle."""

    def __init__(self, max_norm):
        self._record = torch.zeros(2, dtype=torch.float64)
        self.max_norm = max_norm
        self.clock = 0
        self.info = dict(norm=0.0, skipped=False, status=0, clip_coef=1.0)

    def record(self):
        return self._record

    def prepare(self, keys, entries, lr, betas, eps, weight_decay, grad_dtype, out_dtype):
        self.entries, self.hyper = entries, (lr, betas, eps, weight_decay)

    def stats(self, fin_flags, max_norm):
        from oracle import oracle as orc
        total, bad = 0.0, 0
        for _, _, _, g, _, _ in self.entries:
            s, b = orc.sumsq(g.float().numpy())
            total, bad = total + s, bad + b
        self._record[0], self._record[1] = total, bad

    def finalize_and_apply(self):
        from oracle import oracle as orc
        total, bad = float(self._record[0]), float(self._record[1])
        if bad:
            self.info = dict(norm=total ** .5, skipped=True, status=5, clip_coef=1.0)
            return
        norm = total ** .5
        coef = orc.clip_coef_torch(norm, self.max_norm) if self.max_norm else np.float32(1)
        self.clock += 1
        lr, betas, eps, wd = self.hyper
        sc = orc.adamw_scalars(lr, betas[0], betas[1], eps, wd, self.clock)
        for w, m, v, g, out, _ in self.entries:
            orc.adamw_(w.numpy(), m.numpy(), v.numpy(), orc.grad_prepare(g.float().numpy(), coef=coef), sc)
            out.copy_(w.to(out.dtype))
        self.info = dict(norm=norm, skipped=False, status=0, clip_coef=float(coef))

    def last_step(self):
        return self.info


def _inputs():
    g = torch.Generator().manual_seed(3)
    params = [torch.randn(s, generator=g) * .02 for s in SHAPES]
    grads = [[(torch.randn(s, generator=g) * 2e-2).to(torch.bfloat16) for s in SHAPES] for _ in range(3)]
    return params, grads


def _run(world, rank):
    params, grads = _inputs()
    opt = ZeroAdamW(params, LR, BETAS, EPS, WD, max_norm=1.0, device="cpu", backend=OracleBackend(1.0))
    coefs = []
    for gs in grads:
        opt.step(gs)
        coefs.append(opt.last_step()["clip_coef"])
    total = sum(p.numel() for p in params)
    return (opt.lo, opt.hi, opt.master[:opt.hi - opt.lo].clone(), opt.flat_weights[:total].clone(), coefs)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, _run(world, rank)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_and_pieces_cover_the_flat_space():
    sizes = [37, 300, 4096, 5, 1000]
    total = sum(sizes)
    for world in (1, 2, 3, 8):
        covered = []
        for r in range(world):
            lo, hi, per = shard_bounds(total, world, r)
            assert per % 16 == 0 and hi - lo <= per and lo % 16 == 0
            for i, t_off, s_off, n in shard_pieces(sizes, lo, hi):
                start = sum(sizes[:i]) + t_off
                assert start == lo + s_off
                covered += list(range(start, start + n))
        assert covered == list(range(total))


def test_two_gloo_ranks_equal_one_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lo0, hi0, m0, full0, c0 = results[0]
    lo1, hi1, m1, full1, c1 = results[1]
    assert lo0 == 0 and hi0 == lo1 and c0 == c1  # one clip decision on both ranks
    single = _run(1, 0)
    assert single[4] == c0
    torch.testing.assert_close(torch.cat([m0, m1]), single[2], rtol=1e-6, atol=1e-6 * LR)
    assert torch.equal(full0, full1)  # both ranks hold the same gathered weights
    torch.testing.assert_close(full0.float(), single[3].float(), rtol=1e-2, atol=0)
