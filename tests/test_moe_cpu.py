"""MoE oracles on CPU (the contracts the router / grouped-GEMM kernels are
tested against): top-k order and tie rule (lower expert id), NaN logits,
sigmoid scores with and without renormalisation; the routed-expert oracle
against a vectorised dense formulation; expert slices over ranks summing to
the whole (the TP expert-slice layout); stacked quantised expert weights
encoding the dense ones."""
import pytest
import torch

from vllm_sm70_b200.ops import moe


def test_topk_ties_nan_sigmoid():
    lg = torch.tensor([[1.0, 3.0, 3.0, 0.0], [float("nan"), 2.0, 2.0, 2.0]])
    w, ids = moe.topk_ref(lg, 2)
    assert ids.tolist() == [[1, 2], [1, 2]]          # ties -> lower id; NaN never picked
    assert torch.allclose(w.sum(-1), torch.ones(2))  # renormalised
    w2, ids2 = moe.topk_ref(lg[:1], 3, use_sigmoid=True, renorm=False)
    assert ids2.tolist() == [[1, 2, 0]]
    assert torch.allclose(w2, torch.sigmoid(torch.tensor([[3.0, 3.0, 1.0]])))
    w3, _ = moe.topk_ref(lg[:1], 3, use_sigmoid=True, renorm=True)
    assert torch.allclose(w3, w2 / w2.sum())
    # CPU wrapper fills caller buffers
    wb, ib = torch.empty(2, 2), torch.empty(2, 2, dtype=torch.int32)
    moe.topk(lg, 2, w=wb, ids=ib)
    assert torch.equal(ib, ids) and torch.equal(wb, w)


def _experts(E=6, H=16, I=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(E, 2 * I, H, generator=g) * 0.3, torch.randn(E, H, I, generator=g) * 0.3


def test_experts_oracle_matches_vectorised_form():
    E, H, I, T, K = 6, 16, 8, 5, 2
    w13, w2 = _experts(E, H, I)
    ew = moe.ExpertWeights.from_dense("bf16", w13, w2)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(1))
    w, ids = moe.topk_ref(torch.randn(T, E, generator=torch.Generator().manual_seed(2)), K)
    got = moe.experts_forward_ref(x, w, ids, ew)
    W13, W2 = ew.dense_ref()
    h = torch.einsum("tkih,th->tki", W13[ids.long()], x)          # [T, K, 2I]
    act = (torch.nn.functional.silu(h[..., :I]) * h[..., I:]).to(torch.bfloat16).float()
    y = torch.einsum("tkhi,tki->tkh", W2[ids.long()], act)
    assert torch.allclose(got, (w[..., None] * y).sum(1), atol=1e-5)


@pytest.mark.parametrize("ranks", [2, 3])
def test_expert_slices_sum_to_whole(ranks):
    E, H, I, T, K = 6, 16, 8, 7, 3
    w13, w2 = _experts(E, H, I, seed=3)
    full = moe.ExpertWeights.from_dense("bf16", w13, w2)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(4))
    w, ids = moe.topk_ref(torch.randn(T, E, generator=torch.Generator().manual_seed(5)), K)
    El = E // ranks
    parts = [moe.experts_forward_ref(x, w, ids, moe.ExpertWeights.from_dense(
        "bf16", w13[r * El:(r + 1) * El], w2[r * El:(r + 1) * El]), r * El) for r in range(ranks)]
    assert torch.allclose(sum(parts), moe.experts_forward_ref(x, w, ids, full), atol=1e-5)


@pytest.mark.parametrize("fmt,tol", [("fp8", 0.08), ("awq", 0.15), ("nvfp4", 0.25)])
def test_quantised_expert_stacks_encode_dense(fmt, tol):
    E, H, I = 4, 128, 128
    w13, w2 = _experts(E, H, I, seed=6)
    ew = moe.ExpertWeights.from_dense(fmt, w13, w2)
    d13, d2 = ew.dense_ref()
    for d, ref in ((d13, w13), (d2, w2)):
        rel = float((d - ref).abs().max() / ref.abs().max())
        assert rel < tol, (fmt, rel)
    assert ew.bytes() < (w13.numel() + w2.numel()) * 2  # smaller than bf16
