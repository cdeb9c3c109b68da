"""Device gradient accumulation (sparse_disk.py:82-110) and the streaming FP16
export (export.py:30-35) against the CPU oracle: accumulated values bit-exact,
the norm record equal to the FP64 sum within 1e-12 relative, exported bytes
identical to numpy's astype('<f2'), the same good prefix written before the
ValueError."""
import hashlib
import io

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gdt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("scale", [1.0, 1024.0, 3.7])
@pytest.mark.parametrize("n", [1, 4099, 1 << 20])
def test_accumulate_matches_oracle(cuda, gdt, scale, n):
    from morph_b200.disk import accumulate_, norm_record, record_norm
    r = orc.rng(n + int(scale))
    grads = [torch.from_numpy(r.standard_normal(n).astype(np.float32) * 20).to(gdt) for _ in range(3)]
    grads[0][0] = -0.0
    acc = torch.full((n,), 7.0, device=cuda)
    rec = norm_record(cuda)
    ref = np.empty(n, np.float32)
    for k, g in enumerate(grads):
        last = k == len(grads) - 1
        accumulate_(acc, g.to(cuda), scale, first=k == 0, record=rec if last else None)
        orc.grad_accumulate_(ref, g.float().numpy(), scale, first=k == 0)
    np.testing.assert_array_equal(acc.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    s, bad = rec.tolist()
    assert bad == 0
    assert abs(s - float((ref.astype(np.float64) ** 2).sum())) <= 1e-12 * s
    assert abs(record_norm(rec) - float(np.sqrt((ref.astype(np.float64) ** 2).sum()))) <= 1e-12 * s ** .5


def test_accumulate_record_adds_over_tensors_and_flags_nonfinite(cuda):
    from morph_b200.disk import accumulate_, norm_record
    a = torch.zeros(1000, device=cuda)
    b = torch.zeros(3000, device=cuda)
    rec = norm_record(cuda)
    accumulate_(a, torch.ones(1000, device=cuda, dtype=torch.float16), 2.0, first=True, record=rec)
    accumulate_(b, torch.ones(3000, device=cuda, dtype=torch.float16), 1.0, first=True, record=rec)
    assert rec.tolist() == [1000 * .25 + 3000.0, 0.0]
    g = torch.ones(3000, device=cuda, dtype=torch.float16)
    g[1234] = float("inf")
    accumulate_(b, g, 1.0, record=rec)
    assert rec.tolist()[1] == 1.0


def test_accumulate_rejects_bad_arguments(cuda):
    from morph_b200.disk import accumulate_
    acc = torch.zeros(10, device=cuda)
    with pytest.raises(ValueError):
        accumulate_(acc, torch.zeros(11, device=cuda))
    with pytest.raises(ValueError):
        accumulate_(acc, torch.zeros(10, device=cuda), 0.0)


@pytest.mark.parametrize("n,chunk,stage", [(10_007, 1000, 4000), (1 << 20, 1 << 18, 1 << 24), (5, 1048576, 1 << 24)])
def test_export_bytes_and_digest_match_reference(cuda, n, chunk, stage):
    from morph_b200.export import export_fp16
    x = orc.rng(n).standard_normal(n).astype(np.float32)
    x[: min(n, 4)] = [65504.0, -65504.0, 1e-7, -0.0][: min(n, 4)]  # edge, subnormal, negative zero
    buf, h = io.BytesIO(), hashlib.sha256()
    written = export_fp16(torch.from_numpy(x).to(cuda), buf, chunk_elements=chunk, digest=h, staging_elements=stage)
    ref, raised = orc.export_f16_chunks(x, chunk)
    assert not raised and written == len(ref) and buf.getvalue() == ref
    assert h.hexdigest() == hashlib.sha256(ref).hexdigest()


@pytest.mark.parametrize("bad_at,value", [(5500, 70000.0), (0, float("nan")), (9999, float("-inf")),
                                          (3999, 65505.0)])
def test_export_writes_the_good_prefix_then_raises(cuda, bad_at, value):
    from morph_b200.export import export_fp16
    x = orc.rng(3).standard_normal(10_007).astype(np.float32)
    x[bad_at] = value
    x[bad_at + 3] = np.inf  # a later bad value does not move the boundary
    buf = io.BytesIO()
    with pytest.raises(ValueError, match="finite FP16"):
        export_fp16(torch.from_numpy(x).to(cuda), buf, chunk_elements=1000, staging_elements=4000)
    ref, raised = orc.export_f16_chunks(x, 1000)
    assert raised and buf.getvalue() == ref
