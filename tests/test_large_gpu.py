"""Maximum sizes: one tensor of more than 2**31 elements through the statistics
pass (kernel 2), the fused update (kernel 1), the disk-rule update, the
microbatch accumulation and the FP16 export cast, i.e. every element and tile
offset past the int32 range.

The oracle cannot redo 2**31 elements in a test's time, so the check is split:
the global norm is recomputed in full on the host, chunk by chunk (FP64 sums of
the oracle, within 1e-12 relative of the kernel's FP64 sum, and the clip
coefficient derived from it identical), and w, m, v and the low-precision copy
are compared bit for bit with the oracle on windows at the start, across the
2**31 boundary and at the ragged end. The update is elementwise, so a window's
result depends only on its own inputs and the step's scalars."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

N = 2 ** 31 + 4099  # past int32, with a tail that is not a multiple of any tile
WINDOWS = [(0, 4096), (2 ** 31 - 2048, 2 ** 31 + 2048), (N - 4096, N)]
CHUNK = 1 << 26


def _need(cuda, gib):
    free, _ = torch.cuda.mem_get_info(cuda)
    if free < gib << 30:
        pytest.skip(f"needs {gib} GiB of free device memory")


def _bf16_normal(n, std, gen, device):
    g = torch.empty(n, dtype=torch.bfloat16, device=device)
    for s in range(0, n, 1 << 28):
        e = min(n, s + (1 << 28))
        g[s:e] = torch.empty(e - s, device=device).normal_(0.0, std, generator=gen).to(torch.bfloat16)
    return g


def _bits(t):
    """A 16-bit CUDA tensor's bytes as a host uint16 array (the oracle's BF16 form)."""
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _host_norm(g):
    total = 0.0
    for s in range(0, g.numel(), CHUNK):
        s_, bad = orc.sumsq(orc.grad_prepare(_bits(g[s:s + CHUNK])))
        assert bad == 0
        total += s_
    return math.sqrt(total)


def test_adamw_tensor_past_int32(cuda):
    from morph_b200 import AdamW
    _need(cuda, 40)
    gen = torch.Generator(device=cuda).manual_seed(11)
    p = torch.nn.Parameter(torch.empty(N, device=cuda).normal_(0.0, .02, generator=gen))
    p.grad_dtype = None  # BF16 gradient on an FP32 master
    p.grad = _bf16_normal(N, 1e-4, gen, cuda)
    w0 = {win: p.detach()[win[0]:win[1]].cpu().numpy() for win in WINDOWS}
    opt = AdamW([p], lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, max_norm=1.0,
                low_precision=torch.bfloat16, sync=True)
    opt.step()
    last = opt.last_step()
    norm = _host_norm(p.grad)
    assert abs(last["norm"] - norm) <= 1e-12 * norm
    coef = orc.clip_coef_torch(norm, 1.0)
    assert coef < 1 and np.float32(last["clip_coef"]) == coef
    sc = orc.adamw_scalars(3e-4, .9, .95, 1e-8, .1, 1)
    st = opt.state[p]
    assert int(st["step"]) == 1
    for a, b in WINDOWS:
        w = w0[(a, b)].copy()
        m, v = np.zeros_like(w), np.zeros_like(w)
        orc.adamw_(w, m, v, orc.grad_prepare(_bits(p.grad[a:b]), coef=coef), sc)
        np.testing.assert_array_equal(p.detach()[a:b].cpu().numpy(), w, err_msg=f"w [{a}, {b})")
        np.testing.assert_array_equal(st["exp_avg"][a:b].cpu().numpy(), m, err_msg=f"m [{a}, {b})")
        np.testing.assert_array_equal(st["exp_avg_sq"][a:b].cpu().numpy(), v, err_msg=f"v [{a}, {b})")
        np.testing.assert_array_equal(_bits(opt.low_precision_copies[p][a:b]), orc.f32_to_bf16(w),
                                      err_msg=f"bf16 copy [{a}, {b})")


def test_disk_accumulate_export_past_int32(cuda):
    from morph_b200.disk import DeviceDiskState, accumulate_, cast_f32, norm_record, record_norm
    from morph_b200.export import export_fp16
    _need(cuda, 48)
    gen = torch.Generator(device=cuda).manual_seed(12)
    g1 = _bf16_normal(N, 1e-3, gen, cuda)
    g2 = _bf16_normal(N, 1e-3, gen, cuda)
    # two microbatches, unscaled by 2 (exact), statistics of the sum in the same pass
    acc = torch.empty(N, device=cuda)
    rec = norm_record(cuda)
    accumulate_(acc, g1, 2.0, first=True)
    accumulate_(acc, g2, 2.0, record=rec)
    def oracle_acc(a, b):
        out = np.empty(b - a, np.float32)
        orc.grad_accumulate_(out, orc.bf16_to_f32(_bits(g1[a:b])), 2.0, first=True)
        orc.grad_accumulate_(out, orc.bf16_to_f32(_bits(g2[a:b])), 2.0)
        return out

    total = 0.0
    for s in range(0, N, CHUNK):
        total += orc.sumsq(oracle_acc(s, min(N, s + CHUNK)))[0]
    norm = record_norm(rec)
    assert abs(norm - math.sqrt(total)) <= 1e-12 * norm
    acc_win = {}
    for a, b in WINDOWS:
        acc_win[(a, b)] = oracle_acc(a, b)
        np.testing.assert_array_equal(acc[a:b].cpu().numpy(), acc_win[(a, b)], err_msg=f"acc [{a}, {b})")
    del g1, g2
    # one DiskState.update step of the accumulated gradient on (3, N) planes
    planes = torch.zeros(3, N, device=cuda)
    planes[0].normal_(0.0, .02, generator=gen)
    w0 = {win: planes[0, win[0]:win[1]].cpu().numpy() for win in WINDOWS}
    clip = float(orc.clip_coef_disk(norm, 1.0))
    store = DeviceDiskState({"e": planes})
    store.update("e", acc, 1, 1e-4, clip)
    for a, b in WINDOWS:
        w = w0[(a, b)].copy()
        m, v = np.zeros_like(w), np.zeros_like(w)
        orc.adamw_(w, m, v, orc.grad_prepare(acc_win[(a, b)], coef=clip), orc.disk_scalars(1e-4, 1))
        got = planes[:, a:b].cpu().numpy()
        np.testing.assert_array_equal(got[0], w, err_msg=f"w [{a}, {b})")
        np.testing.assert_array_equal(got[1], m, err_msg=f"m [{a}, {b})")
        np.testing.assert_array_equal(got[2], v, err_msg=f"v [{a}, {b})")
    del acc
    w = planes[0]
    want = {win: orc.export_f16(w[win[0]:win[1]].cpu().numpy()) for win in WINDOWS}
    # the FP16 cast (one launch over all N elements) and the staged export writer
    half = cast_f32(w, torch.float16, export_check=True)
    for (a, b), x in want.items():
        np.testing.assert_array_equal(half[a:b].cpu().numpy(), x, err_msg=f"f16 cast [{a}, {b})")
    del half
    sink = _WindowSink()
    assert export_fp16(w, sink) == 2 * N
    for (a, b), x in want.items():
        assert sink.windows[(a, b)] == x.tobytes(), f"export bytes [{a}, {b})"
    # a value past 65504 near the end: the cast raises, the writer stops at its chunk
    bad = N - 5
    w[bad] = 70000.0
    with pytest.raises(ValueError):
        cast_f32(w, torch.float16, export_check=True)
    sink = _WindowSink()
    with pytest.raises(ValueError):
        export_fp16(w, sink)
    assert sink.offset == 2 * (bad // 1048576 * 1048576)


class _WindowSink:
    """A file handle that keeps only the bytes of WINDOWS (FP16: 2 bytes each)."""

    def __init__(self):
        self.offset = 0
        self.windows = {win: b"" for win in WINDOWS}

    def write(self, data):
        data = memoryview(data).cast("B")
        lo, hi = self.offset, self.offset + len(data)
        for a, b in WINDOWS:
            s, e = max(lo, 2 * a), min(hi, 2 * b)
            if s < e:
                self.windows[(a, b)] += bytes(data[s - lo:e - lo])
        self.offset = hi
        return len(data)
