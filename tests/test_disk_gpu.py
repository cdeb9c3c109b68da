"""DiskState.update on device (kernel 1, host scalars), the row-sparse update
(kernel 3) and the FP16/BF16 cast/export, against the oracle and the
reference's golden vectors."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_disk_update_matches_reference_golden(cuda, golden):
    from morph_b200.disk import DeviceDiskState
    sizes = golden["disk_sizes"]
    w0 = golden["disk_init_w"]
    planes, off = {}, 0
    for i, s in enumerate(sizes):
        t = torch.zeros(3, int(s), device=cuda)
        t[0] = torch.from_numpy(w0[off:off + s].copy())
        planes[f"p{i}"] = t
        off += s
    store = DeviceDiskState(planes)
    w, m, v = w0.copy(), np.zeros_like(w0), np.zeros_like(w0)
    for step, (g, clip) in enumerate(zip(golden["disk_grads"], golden["disk_clips"]), start=1):
        off = 0
        for i, s in enumerate(sizes):
            sl = slice(off, off + s)
            store.update(f"p{i}", torch.from_numpy(g[sl].copy()).to(cuda), step, 3e-3, float(clip), chunk_elements=7)
            g32 = orc.grad_prepare(np.ascontiguousarray(g[sl]), coef=clip)
            ww, mm, vv = w[sl].copy(), m[sl].copy(), v[sl].copy()
            orc.adamw_(ww, mm, vv, g32, orc.disk_scalars(3e-3, step))
            w[sl], m[sl], v[sl] = ww, mm, vv
            off += s
    got = np.concatenate([store.planes[f"p{i}"].cpu().numpy() for i in range(len(sizes))], axis=1)
    np.testing.assert_array_equal(got[0], w)  # oracle: bit-exact
    np.testing.assert_array_equal(got[1], m)
    np.testing.assert_array_equal(got[2], v)
    final = golden["disk_final"]  # reference: m, v bit-exact; w within tolerance
    np.testing.assert_array_equal(got[1], final[1])
    np.testing.assert_array_equal(got[2], final[2])
    np.testing.assert_allclose(got[0], final[0], rtol=1e-6, atol=1e-6 * 3e-3)


@pytest.mark.parametrize("gdt", [torch.float16, torch.bfloat16, torch.float32])
def test_row_sparse_update_matches_oracle_and_leaves_other_rows(cuda, golden, gdt):
    from morph_b200.disk import DeviceDiskState
    table = golden["rows_table"]
    idx = golden["rows_idx"]
    rows, cols = table.shape
    planes = torch.zeros(3, rows * cols, device=cuda)
    planes[0] = torch.from_numpy(table.reshape(-1).copy())
    store = DeviceDiskState({"t": planes}, {"t": (rows, cols)})
    g16 = torch.from_numpy(golden["rows_grads"])
    grads = g16.float().to(gdt)
    w, m, v = table.copy(), np.zeros_like(table), np.zeros_like(table)
    for step in (1, 2):
        store.update_rows("t", torch.from_numpy(idx).to(cuda), grads.to(cuda), step, 1e-4, 1.0)
        orc.sparse_rows_(w, m, v, idx, grads.float().numpy(), orc.disk_scalars(1e-4, step))
    got = planes.cpu().numpy().reshape(3, rows, cols)
    np.testing.assert_array_equal(got[0], w)
    np.testing.assert_array_equal(got[1], m)
    np.testing.assert_array_equal(got[2], v)
    if gdt == torch.float16:
        final = golden["rows_final"]
        np.testing.assert_array_equal(got[1][idx], final[1])
        np.testing.assert_array_equal(got[2][idx], final[2])
        np.testing.assert_allclose(got[0][idx], final[0], rtol=1e-6, atol=1e-6 * 1e-4)
    untouched = np.setdiff1d(np.arange(rows), idx)
    np.testing.assert_array_equal(got[0][untouched], table[untouched])
    assert not got[1][untouched].any() and not got[2][untouched].any()


def test_row_index_out_of_range_is_reported(cuda):
    from morph_b200.disk import DeviceDiskState
    planes = torch.zeros(3, 8 * 16, device=cuda)
    store = DeviceDiskState({"t": planes}, {"t": (8, 16)})
    idx = torch.tensor([2, 8], dtype=torch.int64, device=cuda)
    with pytest.raises(IndexError):
        store.update_rows("t", idx, torch.ones(2, 16, device=cuda), 1, 1e-3)
    assert planes[:, 2 * 16:3 * 16].abs().sum() > 0  # the in-range row was updated
    store.update_rows("t", idx[:1], torch.ones(1, 16, device=cuda), 2, 1e-3)  # flag was cleared


def test_row_update_empty_and_ragged_columns(cuda):
    from morph_b200.disk import DeviceDiskState
    r = orc.rng(4)
    rows, cols = 50, 37  # cols % 4 != 0: scalar path
    table = r.standard_normal((rows, cols), dtype=np.float32)
    planes = torch.zeros(3, rows * cols, device=cuda)
    planes[0] = torch.from_numpy(table.reshape(-1).copy())
    store = DeviceDiskState({"t": planes}, {"t": (rows, cols)})
    store.update_rows("t", torch.zeros(0, dtype=torch.int64, device=cuda), torch.zeros(0, cols, device=cuda), 1, 1e-3)
    np.testing.assert_array_equal(planes[0].cpu().numpy(), table.reshape(-1))
    idx = np.array([0, 7, 49], np.int64)
    g = r.standard_normal((3, cols), dtype=np.float32)
    store.update_rows("t", torch.from_numpy(idx).to(cuda), torch.from_numpy(g).to(cuda), 1, 1e-3, clip=.5)
    w, m, v = table.copy(), np.zeros_like(table), np.zeros_like(table)
    orc.sparse_rows_(w, m, v, idx, orc.grad_prepare(g, coef=.5), orc.disk_scalars(1e-3, 1))
    np.testing.assert_array_equal(planes.cpu().numpy().reshape(3, rows, cols)[0], w)


def test_cast_and_fp16_export_check(cuda):
    from morph_b200.disk import cast_f32
    r = orc.rng(8)
    x = r.standard_normal(100_003, dtype=np.float32) * np.float32(100)
    xt = torch.from_numpy(x).to(cuda)
    np.testing.assert_array_equal(cast_f32(xt, torch.float16, export_check=True).cpu().numpy(), orc.export_f16(x))
    np.testing.assert_array_equal(cast_f32(xt, torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16),
                                  orc.f32_to_bf16(x))
    bad = xt.clone()
    bad[99_999] = 65520.0
    with pytest.raises(ValueError):
        cast_f32(bad, torch.float16, export_check=True)
    bad[99_999] = float("nan")
    with pytest.raises(ValueError):
        cast_f32(bad, torch.float16, export_check=True)
    edge = torch.tensor([65504.0, -65504.0], device=cuda)
    assert cast_f32(edge, torch.float16, export_check=True).tolist() == [65504.0, -65504.0]


def test_disk_update_step_gap_and_clips_bit_exact(cuda):
    """tests/test_state_cache.py:34-46 of the reference: clips .25 / 1 / .1 and a
    step gap (clocks 1, 2, 5); every plane bit-exact with the oracle."""
    from morph_b200.disk import DeviceDiskState
    r = orc.rng(31)
    n = 10_001
    w0 = r.standard_normal(n).astype(np.float32) * np.float32(.02)
    planes = torch.zeros(3, n, device=cuda)
    planes[0] = torch.from_numpy(w0).to(cuda)
    store = DeviceDiskState({"p": planes})
    w, m, v = w0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    for step, clip in ((1, .25), (2, 1.0), (5, .1)):
        g = r.standard_normal(n).astype(np.float32) * np.float32(1e-2)
        store.update("p", torch.from_numpy(g).to(cuda), step, 1e-3, clip)
        orc.adamw_(w, m, v, orc.grad_prepare(g, coef=clip), orc.disk_scalars(1e-3, step))
    got = planes.cpu().numpy()
    np.testing.assert_array_equal(got[0], w)
    np.testing.assert_array_equal(got[1], m)
    np.testing.assert_array_equal(got[2], v)
