"""CPU checks of the quantised-weight formats: AWQ pack/unpack round trip in
the AutoAWQ column order, quantise/dequantise error bounds, NVFP4 e2m1 table
and nibble order, FP8 block-scale layout."""
import torch

from vllm_sm70_b200.ops import quant


def test_awq_pack_roundtrip():
    g = torch.Generator().manual_seed(0)
    q = torch.randint(0, 16, (64, 256), generator=g, dtype=torch.int32)  # [K, N]
    packed = torch.zeros(64, 32, dtype=torch.int32)
    v = q.view(64, 32, 8)
    for i in range(8):
        packed |= v[:, :, quant.AWQ_ORDER[i]] << (4 * i)
    assert torch.equal(quant.unpack_awq(packed), q)


def test_awq_layer_dequant_matches_checkpoint_math():
    torch.manual_seed(1)
    w = torch.randn(256, 512) * 0.05
    qw, qz, sc = quant.quantize_awq(w)
    lin = quant.AwqLinear(qw, qz, sc)
    # checkpoint-layout reference: (q - z) * s
    q = quant.unpack_awq(qw).float()                      # [K, N]
    z = quant.unpack_awq(qz).float().repeat_interleave(128, 0)
    s = sc.float().repeat_interleave(128, 0)
    ref = ((q - z) * s).t()
    got = lin.dequant_ref().float()
    assert (got - ref).abs().max() < 2e-2 * ref.abs().max()
    assert (lin.reference_weight() - w).norm() / w.norm() < 0.2


def test_nvfp4_codes_and_order():
    lin = quant.Nvfp4Linear(torch.tensor([[0x21, 0x9F]], dtype=torch.uint8).repeat(1, 8),
                            torch.full((1, 2), 1.0).to(torch.float8_e4m3fn), 1.0)
    w = lin.dequant_ref()[0, :4].float().tolist()
    # byte 0x21: low nibble 1 (0.5) is element 0, high nibble 2 (1.0) element 1;
    # byte 0x9F: low nibble 0xF (-6), high nibble 9 (-0.5)
    assert w == [0.5, 1.0, -6.0, -0.5]


def test_fp8_block_scale_shape_and_error():
    torch.manual_seed(2)
    w = torch.randn(300, 520) * 0.1
    q, s = quant.quantize_fp8_block(w)
    assert q.shape == (300, 520) and s.shape == (3, 5)
    lin = quant.Fp8BlockLinear(q, s)
    assert (lin.reference_weight() - w).norm() / w.norm() < 0.07


def test_cpu_forward_uses_reference_weight():
    torch.manual_seed(3)
    w = torch.randn(128, 256) * 0.05
    for fmt in ("fp8", "awq", "nvfp4"):
        lin = quant.make_linear(fmt, w)
        x = torch.randn(5, 256).to(torch.bfloat16)
        out = lin.forward(x)
        ref = lin.reference_forward(x)
        assert (out.float() - ref).abs().max() < 2e-2 * ref.abs().max() + 1e-3


def test_fp8_act_quant_oracle():
    """Per-token, 128-group e4m3 activation quantisation: scale = amax / 448,
    the round trip stays within e4m3's half-ulp, zero groups stay zero, and
    W8A16 (switch off) multiplies the unquantised activations."""
    torch.manual_seed(4)
    x = torch.randn(6, 300) * 5
    x[1, :128] = 0
    q, s = quant.quant_fp8_act_ref(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (6, 3)
    assert torch.allclose(s[0, 0], x[0, :128].abs().max() / 448)
    assert float(s[1, 0]) == 1.0 and q[1, :128].float().abs().max() == 0
    back = quant.fp8_act_dequant_ref(x)
    assert ((back - x).abs() <= x.abs() * 2 ** -4 + 1e-6).all()
