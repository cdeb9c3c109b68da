"""Sharded Hybrid Muon + AdamW on the GPU: on one GPU it equals
HybridMuonAdamW bit for bit (same kernels, same batches); on 2 GPUs (NCCL, one
process per GPU) every rank holds the same gathered weights, equal to the
1-GPU run, and each Muon master lives on exactly one rank."""
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


def _grads(model, device, steps=3):
    g = torch.Generator().manual_seed(13)
    return [[(torch.randn(p.shape, generator=g) * 1e-2).to(torch.bfloat16).to(device) for p in model.parameters()]
            for _ in range(steps)]


def _run_zero(device):
    from morph_b200.zero import ZeroHybridMuonAdamW
    model = _model(device)
    opt = ZeroHybridMuonAdamW(model, lr=LR, weight_decay=WD, device=device)
    for gs in _grads(model, device):
        opt.step(gs)
    torch.cuda.synchronize(device)
    out = ({i: t.cpu() for i, t in opt.master.items()}, [w.cpu() for w in opt.weights],
           {i: t.cpu() for i, t in opt.momentum.items()})
    opt.close()
    return out


def test_one_gpu_equals_hybrid(cuda):
    from morph_b200 import HybridMuonAdamW
    masters, weights, moms = _run_zero(cuda)
    model = _model(cuda)
    for p in model.parameters():
        p.grad_dtype = None
    opt = HybridMuonAdamW(model, lr=LR, weight_decay=WD, low_precision=torch.bfloat16)
    for gs in _grads(model, cuda):
        for p, g in zip(model.parameters(), gs):
            p.grad = g
        opt.step()
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
        q.put((rank, to_host(_run_zero(torch.device("cuda", rank)))))
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
    single_m, single_w, _ = _run_zero(cuda)
    m0, w0, _ = results[0]
    m1, w1, _ = results[1]
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
