"""Row-sharded offload table host logic on CPU with world_size 2 (gloo): every
touched row goes to exactly one rank, as a local row number, with its own
gradient row. The per-rank table is a recording test double here (the product
class uses the CUDA kernel 5)."""
import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from morph_b200.offload import ShardedRowTable

ROWS, COLS = 1001, 3


class Recorder:
    def __init__(self, rows, cols, init):
        self.rows, self.cols, self.init = rows, cols, init
        self.calls = []

    def step(self, index, grads, step, lr, clip, loss_scale):
        assert index.dtype == torch.int64 and int(index.min()) >= 0 and int(index.max()) < self.rows
        self.calls.append((index.clone(), grads.clone(), step, lr, clip))

    def synchronize(self, timeout=None):
        pass


def _run():
    init = torch.arange(ROWS * COLS, dtype=torch.float32).reshape(ROWS, COLS)
    t = ShardedRowTable(ROWS, COLS, init=init, device="cpu", table_factory=Recorder)
    assert torch.equal(t.local.init, init[t.lo:t.hi])
    g = torch.Generator().manual_seed(0)
    seen = []
    for step in range(1, 4):
        idx = torch.randperm(ROWS, generator=g)[:137].sort().values
        grads = idx.float()[:, None].repeat(1, COLS)  # row r's gradient holds r
        n = t.step(idx, grads, step, 1e-4, .5)
        rec = t.local.calls[-1] if n else None
        if rec is not None:
            gi, gg, s, lr, clip = rec
            assert s == step and clip == .5
            assert torch.equal(gg[:, 0], (gi + t.lo).float())  # each row keeps its own gradient
            seen.append((gi + t.lo).tolist())
        else:
            seen.append([])
    return t.lo, t.hi, seen


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, _run()))
    finally:
        dist.destroy_process_group()


def test_two_ranks_split_the_rows():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (lo0, hi0, s0), (lo1, hi1, s1) = res[0], res[1]
    assert lo0 == 0 and hi0 == lo1 and hi1 == ROWS
    g = torch.Generator().manual_seed(0)
    for step in range(3):
        idx = torch.randperm(ROWS, generator=g)[:137].sort().values.tolist()
        assert s0[step] + s1[step] == idx
        assert all(r < hi0 for r in s0[step]) and all(r >= lo1 for r in s1[step])
