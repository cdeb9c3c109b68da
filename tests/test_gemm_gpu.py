"""Kernel 4's tcgen05 BF16 GEMM against torch.matmul in FP32 (the matmuls of
orthogonalize, streamtrain/optimizer.py:20-21). FP32 output within FP32
summation-order tolerance (rtol 1e-5 of the row scale); BF16 output within one
BF16 rounding of the FP32 result; the transposed copy equals the BF16 output
bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 192), (512, 768, 1024), (384, 256, 4096)])
def test_gemm_matches_fp32_matmul(cuda, m, n, k, dtype):
    from morph_b200.muon import gemm16
    g = torch.Generator(device=cuda).manual_seed(m + n + k)
    a = torch.randn(m, k, device=cuda, generator=g).to(dtype)
    b = torch.randn(n, k, device=cuda, generator=g).to(dtype)
    d, dt, df = gemm16(a, b, out=True, out_t=True, out_f32=True)
    ref = a.float() @ b.float().T
    scale = ref.abs().max().item()
    torch.testing.assert_close(df, ref, rtol=1e-5, atol=1e-5 * scale)
    torch.testing.assert_close(d.float(), df.to(dtype).float(), rtol=0, atol=0)
    assert torch.equal(dt, d.T.contiguous())


def test_gemm_alpha_beta_and_c(cuda):
    from morph_b200.muon import gemm16
    g = torch.Generator(device=cuda).manual_seed(5)
    m, n, k = 256, 256, 320
    a = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, device=cuda, generator=g).to(torch.bfloat16)
    c = torch.randn(m, n, device=cuda, generator=g).to(torch.bfloat16)
    _, _, df = gemm16(a, b, alpha=2.0315, beta=-4.775, c=c, out=False, out_f32=True)
    ref = 2.0315 * (a.float() @ b.float().T) - 4.775 * c.float()
    torch.testing.assert_close(df, ref, rtol=1e-5, atol=1e-5 * ref.abs().max().item())


def test_gemm_rejects_untiled_shapes(cuda):
    from morph_b200.muon import gemm16
    a = torch.zeros(100, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        gemm16(a, torch.zeros(256, 64, dtype=torch.bfloat16, device=cuda))
