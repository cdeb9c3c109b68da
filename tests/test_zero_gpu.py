"""ZeRO-1 on 2 GPUs (NCCL, one process per GPU) equals the same optimizer on
one GPU: masters within 1e-6 relative (floor 1e-6 x lr), gathered BF16 weights
identical on both ranks, one clip decision. Skipped on hosts with one GPU."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _mp import from_host, to_host

pytestmark = pytest.mark.gpu

SHAPES = [(37,), (3072, 300), (4096, 64), (5,), (100000,)]
LR, BETAS, EPS, WD = 3e-4, (.9, .95), 1e-8, .1


def _inputs():
    g = torch.Generator().manual_seed(3)
    params = [torch.randn(s, generator=g) * .02 for s in SHAPES]
    grads = [[(torch.randn(s, generator=g) * 2e-3).to(torch.bfloat16) for s in SHAPES] for _ in range(3)]
    return params, grads


def _run(device, peer_writes="auto", low=torch.bfloat16):
    from morph_b200.zero import ZeroAdamW
    params, grads = _inputs()
    opt = ZeroAdamW([p.to(device) for p in params], LR, BETAS, EPS, WD, max_norm=1.0, gate=True, device=device,
                    peer_writes=peer_writes, low_precision=low)
    coefs = []
    for gs in grads:
        opt.step([g.to(device) for g in gs])
        coefs.append(opt.last_step()["clip_coef"])
    total = sum(p.numel() for p in params)
    flat = torch.full((total,), float("nan"))
    for k, lo, hi in opt.chunks:
        flat[lo:hi] = opt.master[k * opt.cs:k * opt.cs + hi - lo].cpu()
    out = (flat, opt.flat_weights[:total].cpu(), coefs, opt.peer_writes)
    opt.close()
    return out


def _worker(rank, world, port, q, peer_writes="auto", low=torch.bfloat16):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        q.put((rank, to_host(_run(torch.device("cuda", rank), peer_writes, low))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("peer_writes,low", [(True, torch.bfloat16), (False, torch.bfloat16),
                                             (True, torch.float16)])
def test_zero_two_gpus_equal_one_gpu(cuda, peer_writes, low):
    """peer_writes=True: kernel 1 stores the BF16 copies into both GPUs' buffers
    (fused all-gather); False: NCCL all-gather rounds. Both equal one GPU."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, peer_writes, low)) for r in range(2)]
    for p in procs:
        p.start()
    results = {r: from_host(v) for r, v in (q.get(timeout=180) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    flat0, full0, c0, p0 = results[0]
    flat1, full1, c1, p1 = results[1]
    assert p0 == p1 == peer_writes
    assert c0 == c1
    masters = torch.where(torch.isnan(flat0), flat1, flat0)
    assert not torch.isnan(masters).any()
    single = _run(cuda, low=low)
    torch.testing.assert_close(masters, single[0], rtol=1e-6, atol=1e-6 * LR)
    assert torch.equal(full0, full1)
    torch.testing.assert_close(full0.float(), single[1].float(), rtol=1e-2, atol=0)
