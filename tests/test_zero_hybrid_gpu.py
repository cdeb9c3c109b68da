"""Sharded Hybrid Muon + AdamW on the GPU: on one GPU it equals
HybridMuonAdamW bit for bit (same kernels, same batches), refused steps
included; on 2 GPUs (NCCL, one process per GPU) every rank holds the same
gathered weights, equal to the 1-GPU run, each Muon master lives on exactly one
rank, and a nonfinite gradient in one rank's share refuses the step on both."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _mp import from_host, to_host

pytestmark = pytest.mark.gpu

LR, WD = .02, .01


def _model(device):
    torch.manual_seed(11)
    return torch.nn.Sequential(
        torch.nn.Embedding(300, 256),
        *[torch.nn.Linear(256, 512, bias=False) for _ in range(3)],
        *[torch.nn.Linear(512, 256, bias=True) for _ in range(3)],
        torch.nn.Linear(256, 256, bias=False),
        torch.nn.LayerNorm(256)).to(device)


# (step, parameter index) of a NaN: parameter 2 is Muon matrix 1, which rank 1 holds on 2 GPUs
POISON = (2, 2)


def _grads(model, device, steps=3, poison=None):
    g = torch.Generator().manual_seed(13)
    out = []
    for s in range(steps):
        gs = [(torch.randn(p.shape, generator=g) * 1e-2).to(torch.bfloat16) for p in model.parameters()]
        if poison is not None and s == poison[0]:
            gs[poison[1]].view(-1)[7] = float("nan")
        out.append([x.to(device) for x in gs])
    return out


def _run_zero(device, poison=None, steps=3, sync=True):
    from morph_b200.zero import ZeroHybridMuonAdamW
    model = _model(device)
    opt = ZeroHybridMuonAdamW(model, lr=LR, weight_decay=WD, device=device, sync=sync)
    raised = []
    for s, gs in enumerate(_grads(model, device, steps, poison)):
        try:
            opt.step(gs)
            if not sync:
                opt.check()
        except FloatingPointError:
            raised.append(s)
    torch.cuda.synchronize(device)
    out = ({i: t.cpu() for i, t in opt.master.items()}, [w.cpu() for w in opt.weights],
           {i: t.cpu() for i, t in opt.momentum.items()}, raised)
    opt.close()
    return out


@pytest.mark.parametrize("poison,sync", [(None, True), ((0, 1), True), (POISON, False)])
def test_one_gpu_equals_hybrid(cuda, poison, sync):
    """Same bits as HybridMuonAdamW; a refused step (first step: no momentum
    is left behind) raises in step() or, with sync=False, in check()."""
    from morph_b200 import HybridMuonAdamW
    steps = 4 if poison else 3
    masters, weights, moms, raised = _run_zero(cuda, poison, steps, sync)
    model = _model(cuda)
    for p in model.parameters():
        p.grad_dtype = None
    opt = HybridMuonAdamW(model, lr=LR, weight_decay=WD, low_precision=torch.bfloat16)
    ref_raised = []
    for s, gs in enumerate(_grads(model, cuda, steps, poison)):
        for p, g in zip(model.parameters(), gs):
            p.grad = g
        try:
            opt.step()
        except FloatingPointError:
            ref_raised.append(s)
    assert raised == ref_raised == ([poison[0]] if poison else [])
    assert sorted(moms) == sorted(opt.momentum)
    for i, p in enumerate(opt.muon):
        assert torch.equal(masters[i], p.detach().cpu()), i
        assert torch.equal(moms[i], opt.momentum[i].cpu()), i
    for w, p in zip(weights, model.parameters()):
        assert torch.equal(w, p.detach().bfloat16().cpu())


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        q.put((rank, to_host(_run_zero(torch.device("cuda", rank), POISON, 4))))
    finally:
        dist.destroy_process_group()


def test_two_gpus_equal_one_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {r: from_host(v) for r, v in (q.get(timeout=180) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    single_m, single_w, _, single_r = _run_zero(cuda, POISON, 4)
    m0, w0, _, r0 = results[0]
    m1, w1, _, r1 = results[1]
    assert r0 == r1 == single_r == [POISON[0]]  # rank 0 holds no NaN, yet refuses too
    assert not set(m0) & set(m1) and set(m0) | set(m1) == set(single_m)
    for i, t in {**m0, **m1}.items():
        assert torch.equal(t, single_m[i]), i
    for a, b in zip(w0, w1):
        assert torch.equal(a, b)
    for a, c, p in zip(w0, single_w, _model("cpu").parameters()):
        if p.dim() == 2 and p.shape[0] != 300:  # Muon matrices: same kernels, same bits
            assert torch.equal(a, c)
        else:  # AdamW group: ZeRO chunks vs one chunk (torch AdamW tolerance on the masters)
            torch.testing.assert_close(a.float(), c.float(), rtol=1e-2, atol=0)
