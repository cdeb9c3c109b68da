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

    def muon_batch(self, params, moms, grads, outs, lr, weight_decay):
        from oracle import oracle as orc
        assert len({tuple(p.shape) for p in params}) == 1
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


def _run(poison=None):
    model = _model()
    opt = ZeroHybridMuonAdamW(model, lr=LR, weight_decay=WD, device="cpu", backend=OracleHybridBackend(),
                              adam_backend=OracleBackend(None), adam_rounds=2)
    raised = []
    for s, gs in enumerate(_grads(model, poison=poison)):
        try:
            opt.step(gs)
        except FloatingPointError:
            raised.append(s)
    masters = {i: t.clone() for i, t in opt.master.items()}
    weights = [w.float().clone() for w in opt.weights]
    return masters, weights, raised, [sorted(rd[opt.rank]) for rd in opt.rounds]


def _worker(rank, world, port, q, poison):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, to_host(_run(poison))))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_ranks(poison=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, poison)) for r in range(2)]
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
    single_masters, single_weights, raised, _ = _run()
    assert raised == []
    m0, w0, r0, own0 = results[0]
    m1, w1, r1, own1 = results[1]
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


def test_nonfinite_gradient_raises_on_every_rank_and_changes_nothing():
    # step 1 poisons the first Muon matrix (parameter index 1: after the embedding)
    results = _two_ranks(poison=(1, 1))
    clean_masters, clean_weights, _, _ = _run()
    for rank in (0, 1):
        masters, weights, raised, _ = results[rank]
        assert raised == [1]
    # steps 0 and 2 applied, step 1 skipped: equals a 1-rank run with the same poison
    single_masters, single_weights, raised, _ = _run(poison=(1, 1))
    assert raised == [1]
    for rank in (0, 1):
        for i, t in results[rank][0].items():
            assert torch.equal(t, single_masters[i])
        for a, c in zip(results[rank][1], single_weights):
            assert torch.equal(a, c)
    assert any(not torch.equal(a, c) for a, c in zip(single_weights, clean_weights))
