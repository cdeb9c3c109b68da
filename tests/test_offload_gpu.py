"""Kernel 5: row-sparse DiskState.update on pinned-host state through the
ping-pong windows, bit-exact with the CPU oracle on the same seeded inputs;
rows outside the index set are untouched."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cols,gdt", [(96, torch.float16), (37, torch.bfloat16), (3072, torch.float16)])
def test_offloaded_rows_match_oracle_over_many_windows(cuda, cols, gdt):
    from morph_b200.offload import OffloadedRowTable
    rows = 1000 if cols < 1000 else 300
    r = orc.rng(cols)
    w0 = r.standard_normal((rows, cols), dtype=np.float32) * np.float32(.02)
    # windows of 7 rows: every step crosses many windows and both buffers
    table = OffloadedRowTable(rows, cols, init=w0, device=cuda, window_bytes=7 * 3 * cols * 4)
    assert table.window_rows == 7
    w, m, v = w0.copy(), np.zeros_like(w0), np.zeros_like(w0)
    touched = set()
    for step in (1, 2, 3):
        idx = np.sort(r.choice(rows, rows // 10, replace=False)).astype(np.int64)
        touched |= set(idx.tolist())
        g = (r.standard_normal((idx.size, cols), dtype=np.float32) * np.float32(1e-3))
        gt = torch.from_numpy(g).to(gdt)
        table.step(torch.from_numpy(idx).to(cuda), gt.to(cuda), step, 1e-4, clip=0.5)
        orc.sparse_rows_(w, m, v, idx, orc.grad_prepare(gt.float().numpy(), coef=0.5), orc.disk_scalars(1e-4, step))
    table.synchronize()
    np.testing.assert_array_equal(table.w.numpy(), w)
    np.testing.assert_array_equal(table.m.numpy(), m)
    np.testing.assert_array_equal(table.v.numpy(), v)
    untouched = np.array(sorted(set(range(rows)) - touched))
    np.testing.assert_array_equal(table.w.numpy()[untouched], w0[untouched])


def test_offloaded_rows_out_of_range_reported(cuda):
    from morph_b200.offload import OffloadedRowTable
    table = OffloadedRowTable(16, 8, device=cuda, window_bytes=2 * 3 * 8 * 4)
    table.step(torch.tensor([3, 16], dtype=torch.int64, device=cuda), torch.ones(2, 8, device=cuda), 1, 1e-3)
    with pytest.raises(IndexError):
        table.synchronize()
    assert table.w[3].abs().sum() > 0 or table.m[3].abs().sum() > 0


def _sharded_worker(rank, world, port, q):
    import datetime
    import os
    import torch.distributed as dist
    from morph_b200.offload import ShardedRowTable
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cuda", rank)
        rows, cols = 500, 96
        w0 = orc.rng(5).standard_normal((rows, cols), dtype=np.float32) * np.float32(.02)
        t = ShardedRowTable(rows, cols, init=w0, device=dev, window_bytes=9 * 3 * cols * 4)
        r = orc.rng(6)
        for step in (1, 2):
            idx = np.sort(r.choice(rows, 60, replace=False)).astype(np.int64)
            g = torch.from_numpy(r.standard_normal((60, cols), dtype=np.float32) * np.float32(1e-3)).half()
            t.step(torch.from_numpy(idx).to(dev), g.to(dev), step, 1e-4, clip=.5)
        t.synchronize()
        q.put((rank, (t.lo, t.hi, t.local.w.numpy().copy(), t.local.m.numpy().copy())))
    finally:
        dist.destroy_process_group()


def test_row_sharded_two_gpus_equal_oracle(cuda):
    """Two GPUs, each with its own pinned block of rows: every row bit-exact with
    the oracle's unsharded update."""
    import socket
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rows, cols = 500, 96
    w = orc.rng(5).standard_normal((rows, cols), dtype=np.float32) * np.float32(.02)
    m, v = np.zeros_like(w), np.zeros_like(w)
    r = orc.rng(6)
    for step in (1, 2):
        idx = np.sort(r.choice(rows, 60, replace=False)).astype(np.int64)
        g = torch.from_numpy(r.standard_normal((60, cols), dtype=np.float32) * np.float32(1e-3)).half()
        orc.sparse_rows_(w, m, v, idx, orc.grad_prepare(g.float().numpy(), coef=.5), orc.disk_scalars(1e-4, step))
    for rank in (0, 1):
        lo, hi, wl, ml = res[rank]
        np.testing.assert_array_equal(wl, w[lo:hi])
        np.testing.assert_array_equal(ml, m[lo:hi])
    assert res[0][1] == res[1][0] and res[1][1] == rows


def test_bounded_stream_wait(cuda):
    """mb_stream_wait returns MB_ERR_TIMEOUT while work is still queued (the
    work keeps running) and MB_OK once it has finished; the offload table's
    synchronize(timeout=...) raises TimeoutError the same way."""
    from morph_b200 import _lib
    from morph_b200.offload import OffloadedRowTable
    s = torch.cuda.current_stream(cuda)
    torch.cuda._sleep(int(1.5e9))  # ~1 s of GPU time at B200 clocks (a bounded spin)
    assert _lib.lib().mb_stream_wait(_lib.stream_handle(s), 1000) == _lib.MB_ERR_TIMEOUT
    assert _lib.lib().mb_stream_wait(_lib.stream_handle(s), 30_000_000) == _lib.MB_OK
    table = OffloadedRowTable(64, 8, device=cuda, window_bytes=2 * 3 * 8 * 4)
    torch.cuda._sleep(int(1.5e9))
    with pytest.raises(TimeoutError):
        table.synchronize(timeout=1e-3)
    table.synchronize(timeout=30.0)
