"""Block-scaled FP8 (W8A8) on the kind::f8f6f4 tensor cores: the activation
quantiser against its torch oracle (bit for bit), and the dense and grouped
GEMMs against an fp32 oracle built from the same e4m3 operands and scales
(dequantised exactly), across the normal and swap-AB tile forms."""
import pytest
import torch

from vllm_sm70_b200.ops import quant

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def _deq_act(xq, sa, M, K):
    q = xq.view(torch.float8_e4m3fn).float()
    s = sa[:, :M].t().repeat_interleave(128, 1)[:, :K]
    return q * s


@pytest.mark.parametrize("M,K", [(1, 128), (7, 1024), (300, 2000), (64, 768)])
def test_quant_fp8_act_matches_oracle_bitwise(b200_ops, M, K):
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) * 3
    x[0, :64] = 0  # a partly zero group
    xq, sa = quant.quant_fp8_act(x)
    q_ref, s_ref = quant.quant_fp8_act_ref(x)
    torch.cuda.synchronize()
    assert torch.equal(xq.cpu(), q_ref.view(torch.uint8).cpu())
    assert torch.equal(sa[:, :M].t().cpu(), s_ref.cpu())


@pytest.mark.parametrize("M,N,K", [(1, 768, 1024), (17, 384, 2048), (64, 1536, 768),
                                   (65, 512, 4096), (300, 1000, 1024), (1024, 2048, 2048)])
@pytest.mark.parametrize("bn", [0, 32, 64, 128])
def test_gemm_fp8_vs_fp32(b200_ops, M, N, K, bn):
    torch.manual_seed(1)
    w = torch.randn(N, K, device="cuda") * 0.05
    lin = quant.make_linear("fp8", w)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    xq, sa = quant.quant_fp8_act(x)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.ops._b200_C.gemm_fp8_out(out, xq, sa, lin.raw, lin.scales, bn)
    ref = _deq_act(xq, sa, M, K) @ lin.exact_weight().t()
    torch.cuda.synchronize()
    assert _rel(out, ref) < 5e-3, (M, N, K, bn)
    # Repeatable bit for bit (fixed promotion order).
    out2 = torch.empty_like(out)
    torch.ops._b200_C.gemm_fp8_out(out2, xq, sa, lin.raw, lin.scales, bn)
    assert torch.equal(out, out2)


def test_fp8_linear_w8a8_close_to_unquantised(b200_ops):
    """End to end: the W8A8 layer stays close to the unquantised product."""
    torch.manual_seed(2)
    w = torch.randn(1024, 2048, device="cuda") * 0.05
    lin = quant.make_linear("fp8", w)
    x = torch.randn(200, 2048, device="cuda", dtype=torch.bfloat16)
    out = lin.forward(x)
    assert _rel(out, lin.reference_forward(x)) < 5e-3
    assert _rel(out, x.float() @ w.t()) < 6e-2


@pytest.mark.parametrize("bn", [0, 32, 64, 128])
def test_gemm_fp8_grouped_vs_fp32(b200_ops, bn):
    torch.manual_seed(3)
    E, N, K = 8, 256, 512
    counts = torch.tensor([5, 0, 70, 1, 33, 0, 129, 16], dtype=torch.int32)
    rows = int(counts.sum())
    row_off = torch.zeros(E + 1, dtype=torch.int32)
    row_off[1:] = torch.cumsum(counts, 0)
    w = torch.randn(E * N, K, device="cuda") * 0.05
    lin = quant.make_linear("fp8", w)
    x = torch.randn(rows, K, device="cuda", dtype=torch.bfloat16)
    xq, sa = quant.quant_fp8_act(x)
    out = torch.full((rows, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    tile_off = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    torch.ops._b200_C.gemm_fp8_grouped_out(out, xq, sa, lin.raw, lin.scales, E, N,
                                           row_off.cuda(), tile_off, bn)
    xd = _deq_act(xq, sa, rows, K)
    wd = lin.exact_weight().view(E, N, K)
    ref = torch.cat([xd[row_off[e]:row_off[e + 1]] @ wd[e].t() for e in range(E)])
    torch.cuda.synchronize()
    assert not torch.isnan(out.float()).any()
    assert _rel(out, ref) < 5e-3, bn
