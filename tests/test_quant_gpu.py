"""Weight-only quantised GEMMs (FP8 128x128 block, AWQ int4 g128, NVFP4) vs
an fp32 reference computed from the CPU dequantiser of the checkpoint
layout; plus the standalone dequantiser must be bit-identical to the fused
path's math."""
import pytest
import torch

from vllm_sm70_b200.ops import quant

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


@pytest.mark.parametrize("fmt", ["fp8", "awq", "nvfp4"])
@pytest.mark.parametrize("M", [1, 16, 48, 128, 256])
def test_wq_gemm(b200_ops, fmt, M):
    torch.manual_seed(0)
    N, K = 768, 1024
    w = torch.randn(N, K, device="cuda") * 0.05
    lin = quant.make_linear(fmt, w)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    ref = lin.reference_forward(a)
    out = lin.forward(a)
    torch.cuda.synchronize()
    assert _rel(out, ref) < 1e-2, (fmt, M)


@pytest.mark.parametrize("fmt", ["fp8", "awq", "nvfp4"])
def test_dequant_matches_reference_bitwise(b200_ops, fmt):
    torch.manual_seed(1)
    w = torch.randn(384, 512, device="cuda") * 0.05
    lin = quant.make_linear(fmt, w)
    got = lin.dequant(with_global=False)
    ref = lin.dequant_ref().to(torch.bfloat16)
    assert torch.equal(got.cpu(), ref.cpu()), (got.float() - ref.float()).abs().max()


@pytest.mark.parametrize("fmt", ["fp8", "awq", "nvfp4"])
def test_wq_prefill_path(b200_ops, fmt):
    torch.manual_seed(2)
    w = torch.randn(512, 1024, device="cuda") * 0.05
    lin = quant.make_linear(fmt, w)
    a = torch.randn(1000, 1024, device="cuda", dtype=torch.bfloat16)
    ref = lin.reference_forward(a)
    assert _rel(lin.forward(a), ref) < 1e-2


def test_quant_error_is_small(b200_ops):
    torch.manual_seed(3)
    w = torch.randn(256, 512, device="cuda") * 0.05
    for fmt, tol in (("fp8", 0.07), ("awq", 0.2), ("nvfp4", 0.25)):
        lin = quant.make_linear(fmt, w)
        err = (lin.reference_weight() - w).norm() / w.norm()
        assert err < tol, (fmt, float(err))
