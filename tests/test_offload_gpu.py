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
