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

from _mp import from_host, to_host

from morph_b200.zero import ZeroAdamW, chunk_size, rank_chunks, shard_pieces

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

    def prepare(self, keys, entries, rounds, lr, betas, eps, weight_decay, grad_dtype, out_dtype):
        self.entries, self.rounds, self.hyper = entries, rounds, (lr, betas, eps, weight_decay)

    def finalize_opts(self, fin_flags, max_norm):
        pass  # the double always gates and clips with its own max_norm

    def stats(self, fin_flags, max_norm):
        from oracle import oracle as orc
        total, bad = 0.0, 0
        for _, _, _, g, _, _ in self.entries:
            s, b = orc.sumsq(g.float().numpy())
            total, bad = total + s, bad + b
        self._record[0], self._record[1] = total, bad

    def finalize(self):
        from oracle import oracle as orc
        total, bad = float(self._record[0]), float(self._record[1])
        self.skip = bool(bad)
        norm = total ** .5
        if self.skip:
            self.info = dict(norm=norm, skipped=True, status=5, clip_coef=1.0)
            return
        self.coef = orc.clip_coef_torch(norm, self.max_norm) if self.max_norm else np.float32(1)
        self.clock += 1
        self.info = dict(norm=norm, skipped=False, status=0, clip_coef=float(self.coef))

    def apply_round(self, k):
        from oracle import oracle as orc
        if self.skip:
            return
        lr, betas, eps, wd = self.hyper
        sc = orc.adamw_scalars(lr, betas[0], betas[1], eps, wd, self.clock)
        for (w, m, v, g, out, _), r in zip(self.entries, self.rounds):
            if r == k:
                orc.adamw_(w.numpy(), m.numpy(), v.numpy(), orc.grad_prepare(g.float().numpy(), coef=self.coef), sc)
                out.copy_(w.to(out.dtype))

    def last_step(self):
        return self.info


def _inputs():
    g = torch.Generator().manual_seed(3)
    params = [torch.randn(s, generator=g) * .02 for s in SHAPES]
    grads = [[(torch.randn(s, generator=g) * 2e-2).to(torch.bfloat16) for s in SHAPES] for _ in range(3)]
    return params, grads


def _run(world, rank, rounds=3):
    params, grads = _inputs()
    opt = ZeroAdamW(params, LR, BETAS, EPS, WD, max_norm=1.0, device="cpu", backend=OracleBackend(1.0),
                    rounds=rounds)
    coefs = []
    for gs in grads:
        opt.step(gs)
        coefs.append(opt.last_step()["clip_coef"])
    total = sum(p.numel() for p in params)
    # this rank's masters placed at their flat positions (NaN elsewhere)
    flat = torch.full((total,), float("nan"))
    for k, lo, hi in opt.chunks:
        flat[lo:hi] = opt.master[k * opt.cs:k * opt.cs + hi - lo]
    return (flat, opt.flat_weights[:total].clone(), coefs)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, to_host(_run(world, rank))))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_round_robin_chunks_cover_the_flat_space():
    sizes = [37, 300, 4096, 5, 1000]
    total = sum(sizes)
    for world in (1, 2, 3, 8):
        for rounds in (1, 3, 8):
            cs = chunk_size(total, world, rounds)
            assert cs % 16 == 0 and rounds * world * cs >= total
            covered = []
            for r in range(world):
                for k, lo, hi in rank_chunks(total, world, r, rounds, cs):
                    assert lo == min(total, (k * world + r) * cs)
                    for i, t_off, c_off, n in shard_pieces(sizes, lo, hi):
                        start = sum(sizes[:i]) + t_off
                        assert start == lo + c_off
                        covered += list(range(start, start + n))
            assert sorted(covered) == list(range(total))


def test_two_gloo_ranks_equal_one_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {r: from_host(v) for r, v in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    flat0, full0, c0 = results[0]
    flat1, full1, c1 = results[1]
    assert c0 == c1  # one clip decision on both ranks
    masters = torch.where(torch.isnan(flat0), flat1, flat0)
    assert not torch.isnan(masters).any()  # the two ranks' chunks cover everything
    single = _run(1, 0)
    assert single[2] == c0
    torch.testing.assert_close(masters, single[0], rtol=1e-6, atol=1e-6 * LR)
    assert torch.equal(full0, full1)  # both ranks hold the same gathered weights
    torch.testing.assert_close(full0.float(), single[1].float(), rtol=1e-2, atol=0)


@pytest.mark.parametrize("sync", [None, False])
def test_refused_step_changes_nothing_and_raises(sync):
    """gate: a nonfinite gradient leaves masters and weights unchanged. The
    default (sync=gate) raises FloatingPointError inside step(); sync=False only
    enqueues the step and check() raises afterwards."""
    params, grads = _inputs()
    opt = ZeroAdamW(params, LR, BETAS, EPS, WD, max_norm=1.0, gate=True, device="cpu", backend=OracleBackend(1.0),
                    rounds=2, sync=sync)
    opt.step(grads[0])
    master, weights = opt.master.clone(), opt.flat_weights.clone()
    bad = [g.clone() for g in grads[1]]
    bad[2][5, 7] = float("inf")
    if sync is None:
        with pytest.raises(FloatingPointError):
            opt.step(bad)
    else:
        opt.step(bad)
        assert opt.last_step()["skipped"]
        with pytest.raises(FloatingPointError):
            opt.check()
    assert torch.equal(opt.master, master) and torch.equal(opt.flat_weights, weights)
    opt.step(grads[2])  # the next finite step proceeds
    opt.check()
    assert not torch.equal(opt.master, master)


def test_peer_writes_need_the_cuda_backend_and_several_ranks():
    """Peer stores are a CUDA-IPC path: asking for them with another backend
    (or on one rank) is an error; "auto" quietly falls back to the NCCL rounds."""
    params, _ = _inputs()
    with pytest.raises(ValueError):
        ZeroAdamW(params, LR, BETAS, EPS, WD, device="cpu", backend=OracleBackend(None), peer_writes=True)
    opt = ZeroAdamW(params, LR, BETAS, EPS, WD, device="cpu", backend=OracleBackend(None), peer_writes="auto")
    assert opt.peer_writes is False and opt.rounds == 1  # one rank: one round
    with pytest.raises(ValueError):
        ZeroAdamW(params, LR, BETAS, EPS, WD, device="cpu", backend=OracleBackend(None), peer_writes="yes")
