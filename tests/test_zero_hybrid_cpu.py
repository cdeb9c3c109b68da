"""Sharded Hybrid Muon + AdamW host logic on CPU with world_size 2 (gloo):
whole-matrix dealing, the per-round blocks of the low-precision buffer and
their in-place all-gather, the shared finiteness decision, and the AdamW
group's ZeRO-1 shard.

The kernels are replaced by oracle-backed test doubles defined here (the
product classes always use the CUDA library); the 2-rank result must equal the
1-rank result bit for bit."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _mp import from_host, to_host

from morph_b200.zero import ZeroHybridMuonAdamW, deal_matrices
from test_zero_cpu import OracleBackend

LR, WD = .02, .01


class OracleHybridBackend:
    """Test double of CudaHybridBackend computing with the CPU oracle."""

    def gate_record(self, grads):
        from oracle import oracle as orc
        total, bad = 0.0, 0
        for g in grads:
            s, b = orc.sumsq(g.float().numpy())
            total, bad = total + s, bad + b
        return torch.tensor([total, float(bad)], dtype=torch.float64)

    @staticmethod
    def batch_plan(n, rows, cols):
        return [2] * (n // 2) + ([n % 2] if n % 2 else [])

    def gate_finalize(self, record):
        """The skip decision as a one-element tensor (the device flag's stand-in)."""
        return torch.tensor([int(float(record[1]) != 0.0)], dtype=torch.int32)

    def muon_batch(self, params, moms, grads, outs, lr, weight_decay, skip=None):
        from oracle import oracle as orc
        assert len({tuple(p.shape) for p in params}) == 1
        if skip is not None and int(skip[0]):
            return  # the kernels read the flag first and change nothing
        for p, m, g, o in zip(params, moms, grads, outs):
            u = orc.muon_momentum_(m.numpy(), g.float().numpy())
            orc.muon_apply_(p.numpy(), orc.orthogonalize(u), lr, weight_decay)
            o.copy_(p.to(o.dtype))

    def check_errors(self):
        pass


def _model():
    torch.manual_seed(5)
    return torch.nn.Sequential(
        torch.nn.Embedding(50, 24),
        *[torch.nn.Linear(24, 40, bias=False) for _ in range(3)],
        *[torch.nn.Linear(40, 24, bias=True) for _ in range(2)],
        torch.nn.Linear(24, 24, bias=False),
        torch.nn.LayerNorm(24))


def _grads(model, steps=3, poison=None):
    g = torch.Generator().manual_seed(7)
    out = []
    for s in range(steps):
        gs = [(torch.randn(p.shape, generator=g) * 1e-2).to(torch.bfloat16) for p in model.parameters()]
        if poison is not None and s == poison[0]:
            gs[poison[1]].view(-1)[0] = float("nan")
        out.append(gs)
    return out


def _run(poison=None, sync=True):
    """Three steps; with sync=False a refused step is reported by check()
    after it was enqueued, and the next step still proceeds."""
    model = _model()
    opt = ZeroHybridMuonAdamW(model, lr=LR, weight_decay=WD, device="cpu", backend=OracleHybridBackend(),
                              adam_backend=OracleBackend(None), adam_rounds=2, sync=sync)
    raised = []
    for s, gs in enumerate(_grads(model, poison=poison)):
        try:
            opt.step(gs)
            if not sync:
                opt.check()
        except FloatingPointError:
            raised.append(s)
    masters = {i: t.clone() for i, t in opt.master.items()}
    weights = [w.float().clone() for w in opt.weights]
    return masters, weights, raised, [sorted(rd[opt.rank]) for rd in opt.rounds], sorted(opt.momentum)


def _worker(rank, world, port, q, poison, sync):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, to_host(_run(poison, sync))))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_ranks(poison=None, sync=True):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, poison, sync)) for r in range(2)]
    for p in procs:
        p.start()
    results = {r: from_host(v) for r, v in (q.get(timeout=180) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return results


def test_deal_matrices_balances_each_shape():
    shapes = [(64, 96)] * 7 + [(96, 64)] * 4 + [(32, 32)] * 3
    plan = lambda n, r, c: [3] * (n // 3) + ([n % 3] if n % 3 else [])  # noqa: E731
    for world in (1, 2, 3, 4, 8):
        rounds = deal_matrices(shapes, world, plan)
        seen = []
        for rd in rounds:
            assert set(rd) == set(range(world))
            assert len({shapes[i] for r in rd for i in rd[r]}) == 1  # one shape per round
            assert all(len(rd[r]) <= 3 for r in rd)
            for r in rd:
                seen += rd[r]
        assert sorted(seen) == list(range(len(shapes)))
        for shape in set(shapes):
            counts = [sum(1 for rd in rounds for i in rd[r] if shapes[i] == shape) for r in range(world)]
            assert max(counts) - min(counts) <= 1


def test_two_gloo_ranks_equal_one_rank():
    results = _two_ranks()
    single_masters, single_weights, raised, _, _ = _run()
    assert raised == []
    m0, w0, r0, own0, _ = results[0]
    m1, w1, r1, own1, _ = results[1]
    assert r0 == r1 == []
    assert not set(m0) & set(m1) and set(m0) | set(m1) == set(single_masters)  # each matrix on one rank
    for i, t in {**m0, **m1}.items():
        assert torch.equal(t, single_masters[i]), i
    for a, b, c in zip(w0, w1, single_weights):
        assert torch.equal(a, b)  # both ranks hold the same gathered weights
    # Muon weights are the BF16 copies of the same FP32 masters: identical to one rank;
    # the AdamW shard's clip-free update is bit-exact per element too
    for a, c in zip(w0, single_weights):
        assert torch.equal(a, c)


@pytest.mark.parametrize("sync", [True, False])
def test_nonfinite_gradient_raises_on_every_rank_and_changes_nothing(sync):
    """The gate decides on the device from the all-reduced record: the Muon
    launches and the AdamW group skip, the all-gathers carry unchanged weights,
    and every rank raises (inside step with sync=True, from check() with
    sync=False)."""
    # step 1 poisons the first Muon matrix (parameter index 1: after the embedding)
    results = _two_ranks(poison=(1, 1), sync=sync)
    clean_masters, clean_weights, _, _, _ = _run()
    for rank in (0, 1):
        masters, weights, raised, _, _ = results[rank]
        assert raised == [1]
    # steps 0 and 2 applied, step 1 skipped: equals a 1-rank run with the same poison
    single_masters, single_weights, raised, _, _ = _run(poison=(1, 1))
    assert raised == [1]
    for rank in (0, 1):
        for i, t in results[rank][0].items():
            assert torch.equal(t, single_masters[i])
        for a, c in zip(results[rank][1], single_weights):
            assert torch.equal(a, c)
    assert any(not torch.equal(a, c) for a, c in zip(single_weights, clean_weights))


def test_refused_first_step_creates_no_momentum():
    """A step refused before any Muon momentum existed leaves none behind
    (the reference raises before creating it); the next step creates it."""
    model = _model()
    opt = ZeroHybridMuonAdamW(model, lr=LR, weight_decay=WD, device="cpu", backend=OracleHybridBackend(),
                              adam_backend=OracleBackend(None), adam_rounds=2, sync=False)
    before = [w.float().clone() for w in opt.weights]
    grads = _grads(model, poison=(0, 1))
    opt.step(grads[0])
    with pytest.raises(FloatingPointError):
        opt.check()
    assert opt.momentum == {}
    assert all(torch.equal(a.float(), b) for a, b in zip(opt.weights, before))
    opt.step(grads[1])
    opt.check()
    assert sorted(opt.momentum) == sorted(opt.master)
