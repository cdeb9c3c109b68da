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


def _pair_cases(device):
    """GEMM, Newton-Schulz and fused-update outputs on shapes whose M is a
    multiple of 256 (the pair-CTA kernel's tiles)."""
    from morph_b200.muon import gemm16, muon_step_batched, orthogonalize
    g = torch.Generator(device=device).manual_seed(21)
    out = []
    a = torch.randn(512, 1024, device=device, generator=g).to(torch.bfloat16)
    b = torch.randn(768, 1024, device=device, generator=g).to(torch.bfloat16)
    out += list(gemm16(a, b, out=True, out_t=True, out_f32=True))
    c = torch.randn(512, 768, device=device, generator=g).to(torch.bfloat16)
    out += [x for x in gemm16(a, b, alpha=1.5, beta=-0.25, c=c, out=True, out_f32=True) if x is not None]
    x = torch.randn(1024, 2752, device=device, generator=g)
    out += [orthogonalize(x, ns_dtype="bf16"), orthogonalize(x.T.contiguous(), ns_dtype="fp16")]
    ps = [torch.randn(512, 1024, device=device, generator=g) * .02 for _ in range(3)]
    ms = [torch.zeros_like(p) for p in ps]
    gs = [torch.randn(512, 1024, device=device, generator=g).to(torch.bfloat16) for _ in range(3)]
    outs = [torch.empty(512, 1024, dtype=torch.bfloat16, device=device) for _ in range(3)]
    for _ in range(2):
        muon_step_batched(ps, ms, gs, outs, .02, .01, "bf16")
    out += ps + ms + outs
    torch.cuda.synchronize(device)
    return [t.cpu() for t in out]


def _single_cta_worker(q):
    import os

    from _mp import to_host
    os.environ["MB_GEMM_PAIR"] = "0"  # read by the library at its first GEMM in this process
    q.put(to_host(_pair_cases(torch.device("cuda", 0))))


def test_pair_cta_kernel_matches_single_cta_kernel_bit_for_bit(cuda):
    """The default pair-CTA GEMM (M = 256 over two SMs) against the single-CTA
    kernel, run in a child process with MB_GEMM_PAIR=0: every output equal."""
    import os

    import torch.multiprocessing as mp
    from _mp import from_host
    if os.environ.get("MB_GEMM_PAIR", "1")[:1] == "0":
        pytest.skip("pair mode switched off in this environment")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_single_cta_worker, args=(q,))
    p.start()
    single = from_host(q.get(timeout=300))
    p.join(timeout=60)
    assert p.exitcode == 0
    pair = _pair_cases(cuda)
    assert len(pair) == len(single)
    for i, (x, y) in enumerate(zip(pair, single)):
        assert torch.equal(x, y), i
