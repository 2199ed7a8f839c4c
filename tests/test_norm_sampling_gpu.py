"""RMSNorm / fused add+RMSNorm / argmax / embedding / silu_mul kernels vs torch."""
import pytest
import torch

from vllm_sm70_b200.ops import linear, norm, sampling

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H", [2048, 4096, 8192, 5120])
def test_rms_norm(b200_ops, H):
    torch.manual_seed(0)
    x = torch.randn(33, H, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    out = norm.rms_norm(x, w, 1e-5)
    ref = norm.rms_norm_ref(x.cpu(), w.cpu(), 1e-5)
    assert (out.cpu().float() - ref.float()).abs().max() <= 0.02 * ref.float().abs().max()


@pytest.mark.parametrize("H", [2048, 4096])
def test_fused_add_rms_norm_matches_unfused_bitwise(b200_ops, H):
    torch.manual_seed(1)
    x = torch.randn(17, H, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(17, H, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    x1, r1 = x.clone(), r.clone()
    norm.fused_add_rms_norm(x1, r1, w, 1e-5)
    s = (x.float() + r.float()).to(torch.bfloat16)
    assert torch.equal(r1, s)
    x2 = norm.rms_norm(s, w, 1e-5)
    assert torch.equal(x1, x2)


def test_argmax(b200_ops):
    torch.manual_seed(2)
    lg = torch.randn(9, 128256, device="cuda", dtype=torch.bfloat16)
    lg[1, 5] = lg[1, 900] = 100.0  # tie -> lower id
    lg[2, 77] = float("nan")
    ids, vals = sampling.argmax(lg)
    rid, _ = sampling.argmax_ref(lg.cpu())
    assert torch.equal(ids.cpu(), rid)
    assert int(ids[1]) == 5 and int(ids[2]) == 77


def test_silu_mul_and_embedding(b200_ops):
    torch.manual_seed(3)
    x = torch.randn(10, 2 * 1024, device="cuda", dtype=torch.bfloat16)
    out = linear.silu_mul(x)
    ref = linear.silu_mul_ref(x[:, :1024], x[:, 1024:])
    assert (out.float() - ref.float()).abs().max() < 0.05
    tab = torch.randn(1000, 256, device="cuda", dtype=torch.bfloat16)
    ids = torch.randint(0, 1000, (13,), device="cuda")
    e = torch.empty(13, 256, device="cuda", dtype=torch.bfloat16)
    torch.ops._b200_C.embedding(e, ids, tab, 0)
    assert torch.equal(e, tab[ids])
