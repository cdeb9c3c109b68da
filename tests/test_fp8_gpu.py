"""Block-scaled FP8 transport on the GPU against the reference's pack_fp8 /
unpack_fp8 (golden vectors) and the oracle: codes, scales and unpacked values
bit-exact."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_fp8_pack_unpack_match_reference_golden(cuda, golden):
    from morph_b200.precision import pack_fp8, unpack_fp8
    x = torch.from_numpy(golden["fp8_in"]).to(cuda)
    codes, scales = pack_fp8(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), golden["fp8_encoded"])
    np.testing.assert_array_equal(scales.cpu().numpy(), golden["fp8_scales"])
    np.testing.assert_array_equal(unpack_fp8(codes, scales, torch.float16).cpu().numpy(), golden["fp8_unpacked_f16"])
    np.testing.assert_array_equal(unpack_fp8(codes, scales, torch.float32).cpu().numpy(), golden["fp8_unpacked_f32"])


@pytest.mark.parametrize("n", [1, 255, 256, 257, 100_000, 3_000_001])
def test_fp8_random_sizes_match_oracle(cuda, n):
    from morph_b200.precision import pack_fp8, unpack_fp8
    r = orc.rng(n)
    x = (r.standard_normal(n, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    codes, scales = pack_fp8(torch.from_numpy(x).to(cuda))
    oc, osc = orc.pack_fp8(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), oc)
    np.testing.assert_array_equal(scales.cpu().numpy(), osc)
    for dt in ("float16", "bfloat16"):
        got = unpack_fp8(codes, scales, getattr(torch, dt)).cpu()
        want = torch.from_numpy(orc.unpack_fp8(oc, osc, "float32")).to(getattr(torch, dt))
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_fp8_nan_block_propagates(cuda):
    from morph_b200.precision import pack_fp8
    x = torch.zeros(512, device=cuda)
    x[300] = float("nan")
    codes, scales = pack_fp8(x)
    assert scales[0].item() == 1e-30 or scales[0].item() == np.float32(1e-30)
    assert torch.isnan(scales[1])
