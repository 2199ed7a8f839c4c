"""NVFP4 W4A4 on the kind::mxf4nvf4 tensor cores (block scales in TMEM): the
activation quantiser against its torch oracle (values, scale atoms and row
scales bit for bit), and the dense (normal and swap-AB tiles) and grouped
GEMMs against an fp32 oracle of the same e2m1 operands and scales."""
import pytest
import torch

from vllm_sm70_b200.ops import quant

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def _unpack(xq, K):
    lut = quant.E2M1.to(xq.device)
    return torch.stack([lut[(xq & 0xF).long()], lut[(xq >> 4).long()]], -1).view(xq.shape[0], K)


def _deq_act(xq, sf_atoms, rs, M, K):
    """fp32 value of the kernel's quantised activations (values x scale x rs)."""
    Mp = (M + 127) // 128 * 128
    a = sf_atoms[: Mp // 128 * (K // 64) * 512].view(Mp // 128, K // 64, 32, 4, 4)
    # atom [nb, kg, m0, m1, j] -> rows nb*128 + m1*32 + m0, scale column kg*4 + j
    s = a.permute(0, 3, 2, 1, 4).reshape(Mp, K // 16)[:M]
    sc = s.view(torch.float8_e4m3fn).float()
    return _unpack(xq[:M], K) * (sc * rs[:M, None]).repeat_interleave(16, 1)


@pytest.mark.parametrize("M,K", [(1, 256), (7, 1024), (300, 2048), (129, 512)])
def test_quant_nvfp4_act_matches_oracle(b200_ops, M, K):
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) * 3
    x[0, :32] = 0
    if M > 2:
        x[2] *= 1e-3
    xq, sf, rs = quant.quant_nvfp4_act(x)
    q_ref, s_ref, rs_ref = quant.quant_nvfp4_act_ref(x)
    torch.cuda.synchronize()
    assert torch.equal(rs[:M].cpu(), rs_ref.cpu())
    assert torch.equal(_unpack(xq, K).cpu(), q_ref.cpu())
    ref_atoms = quant.nvfp4_sf_atoms(s_ref.to(torch.float8_e4m3fn).view(torch.uint8))
    assert torch.equal(sf.cpu(), ref_atoms.cpu())
    # the round trip stays within the e2m1 / e4m3 grid of each block
    back = _deq_act(xq, sf, rs, M, K)
    assert _rel(back, x.float()) < 0.25


@pytest.mark.parametrize("M,N,K", [(1, 768, 1024), (17, 384, 2048), (128, 1536, 512),
                                   (200, 520, 1024), (1024, 2048, 2048)])
@pytest.mark.parametrize("swap", [-1, 0, 1])
def test_gemm_nvfp4_vs_fp32(b200_ops, M, N, K, swap):
    torch.manual_seed(1)
    w = torch.randn(N, K, device="cuda") * 0.05
    lin = quant.make_linear("nvfp4", w)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    xq, sf, rs = quant.quant_nvfp4_act(x)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.ops._b200_C.gemm_nvfp4_out(out, xq, sf, rs, lin.raw, lin.sf_atoms(), lin.out_scale,
                                     swap)
    ref = (_deq_act(xq, sf, rs, M, K) @ lin.exact_weight().t()) * lin.out_scale
    torch.cuda.synchronize()
    assert _rel(out, ref) < 5e-3, (M, N, K, swap)
    out2 = torch.empty_like(out)
    torch.ops._b200_C.gemm_nvfp4_out(out2, xq, sf, rs, lin.raw, lin.sf_atoms(), lin.out_scale,
                                     swap)
    assert torch.equal(out, out2)


def test_nvfp4_linear_w4a4_close_to_unquantised(b200_ops):
    torch.manual_seed(2)
    w = torch.randn(1024, 2048, device="cuda") * 0.05
    lin = quant.make_linear("nvfp4", w)
    x = torch.randn(200, 2048, device="cuda", dtype=torch.bfloat16)
    out = lin.forward(x)
    assert _rel(out, lin.reference_forward(x)) < 5e-3
    assert _rel(out, x.float() @ w.t()) < 0.25


def test_gemm_nvfp4_grouped_vs_fp32(b200_ops):
    torch.manual_seed(3)
    E, N, K = 6, 256, 512
    counts = [5, 0, 130, 1, 128, 17]
    row_off = [0]
    for c in counts:  # expert blocks start at multiples of 128 (padded permutation)
        row_off.append(row_off[-1] + (c + 127) // 128 * 128)
    rows = row_off[-1]
    w = torch.randn(E * N, K, device="cuda") * 0.05
    lin = quant.make_linear("nvfp4", w)
    x = torch.randn(rows, K, device="cuda", dtype=torch.bfloat16)
    xq, sf, rs = quant.quant_nvfp4_act(x)
    out = torch.zeros(rows, N, device="cuda", dtype=torch.bfloat16)
    tile_off = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    ro = torch.tensor(row_off, dtype=torch.int32, device="cuda")
    torch.ops._b200_C.gemm_nvfp4_grouped_out(out, xq, sf, rs, lin.raw, lin.sf_atoms(),
                                             lin.out_scale, E, N, ro, tile_off)
    xd = _deq_act(xq, sf, rs, rows, K)
    wd = lin.exact_weight().view(E, N, K) * lin.out_scale
    torch.cuda.synchronize()
    for e in range(E):
        a, b = row_off[e], row_off[e] + counts[e]
        if b > a:
            assert _rel(out[a:b], xd[a:b] @ wd[e].t()) < 5e-3, e
