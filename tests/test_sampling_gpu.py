"""Random sampling kernels: Gumbel-max sampling matches the softmax
distribution (chi-square on a small vocab), is reproducible per seed, and
shards merge exactly; top-K candidates equal torch.topk; candidate sampling
respects top-k / top-p and temperature 0 is greedy."""
import pytest
import torch

from vllm_sm70_b200.ops import sampling

pytestmark = pytest.mark.gpu


def test_gumbel_distribution(b200_ops):
    V, n = 8, 20000
    logits = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, 0.3, 1.5, -0.5], device="cuda")
    lg = logits.expand(n, V).contiguous()
    T = 0.7
    temp = torch.full((n,), T, device="cuda")
    seeds = torch.arange(n, device="cuda", dtype=torch.int64)
    ids, _ = sampling.gumbel_sample(lg, temp, seeds, offset=0)
    counts = torch.bincount(ids.long().cpu(), minlength=V).float()
    p = torch.softmax(logits.cpu() / T, -1)
    chi2 = float(((counts - n * p) ** 2 / (n * p)).sum())
    assert chi2 < 30.0, (chi2, counts, n * p)  # 7 dof, p ~ 1e-4 threshold


def test_gumbel_reproducible_and_shard_merge(b200_ops):
    torch.manual_seed(0)
    lg = torch.randn(16, 4096, device="cuda", dtype=torch.bfloat16)
    temp = torch.full((16,), 0.9, device="cuda")
    temp[3] = 0.0
    seeds = torch.randint(0, 2**40, (16,), device="cuda")
    a, _ = sampling.gumbel_sample(lg, temp, seeds, offset=5)
    b, _ = sampling.gumbel_sample(lg, temp, seeds, offset=5)
    assert torch.equal(a, b)
    assert int(a[3]) == int(lg[3].float().argmax())
    ids, vals = [], []
    for r in range(4):
        i, v = sampling.gumbel_sample(lg[:, r * 1024:(r + 1) * 1024].contiguous(), temp, seeds,
                                      offset=5, id_offset=r * 1024)
        ids.append(i)
        vals.append(v)
    merged = sampling.merge_rank_top1(torch.stack(vals), torch.stack(ids))
    assert torch.equal(merged.cpu(), a.cpu())


@pytest.mark.parametrize("K", [1, 17, 64])
def test_topk_candidates(b200_ops, K):
    torch.manual_seed(1)
    lg = torch.randn(9, 50000, device="cuda")
    lg[2, 100:140] = 7.0  # ties -> lower ids first
    v, i = sampling.topk_candidates(lg, K)
    rv, ri = sampling.topk_candidates(lg.cpu(), K)
    assert torch.equal(i.cpu(), ri) and torch.allclose(v.cpu(), rv)


def test_sample_candidates_topk_topp_greedy(b200_ops):
    rows, C = 512, 64
    v = torch.linspace(3, -3, C, device="cuda").expand(rows, C).contiguous()
    i = torch.arange(C, device="cuda", dtype=torch.int32).expand(rows, C).contiguous()
    seeds = torch.arange(rows, device="cuda", dtype=torch.int64)
    t = torch.ones(rows, device="cuda")
    k = torch.full((rows,), 5, device="cuda", dtype=torch.int32)
    p = torch.ones(rows, device="cuda")
    out = sampling.sample_candidates(v, i, t, k, p, seeds, 0)
    assert int(out.max()) < 5 and int(out.min()) >= 0
    k.fill_(-1)
    p.fill_(0.3)
    out = sampling.sample_candidates(v, i, t, k, p, seeds, 1)
    probs = torch.softmax(v[0].cpu(), -1)
    keep = int((torch.cumsum(probs, 0) < 0.3).sum()) + 1
    assert int(out.max()) < keep
    t.fill_(0.0)
    out = sampling.sample_candidates(v, i, t, k, p, seeds, 2)
    assert int(out.max()) == 0


def test_rejection_sampler_preserves_target_distribution(b200_ops):
    """With drafts sampled from q, the emitted first token must follow p
    exactly (the defining property of speculative sampling)."""
    V, rows, k = 6, 30000, 1
    torch.manual_seed(4)
    tl = torch.tensor([1.0, 0.2, -0.5, 2.0, 0.0, -1.0])
    dl = torch.tensor([0.0, 1.5, 0.3, -0.2, 1.0, 0.5])
    T = 0.8
    p = torch.softmax(tl / T, -1)
    q = torch.softmax(dl / T, -1)
    drafts = torch.multinomial(q, rows, replacement=True).view(rows, 1).to(torch.int32).cuda()
    tgt = tl.to(torch.bfloat16).expand(rows, k + 1, V).contiguous().cuda()
    drf = dl.to(torch.bfloat16).expand(rows, k, V).contiguous().cuda()
    temp = torch.full((rows,), T, device="cuda")
    seeds = torch.arange(rows, device="cuda", dtype=torch.int64) * 7 + 1
    out, n = sampling.rejection_sample(tgt, drf, drafts, temp, seeds, 0)
    first = out[:, 0].long().cpu()
    assert int(first.min()) >= 0
    pb = torch.softmax(tl.to(torch.bfloat16).float() / T, -1)
    counts = torch.bincount(first, minlength=V).float()
    chi2 = float(((counts - rows * pb) ** 2 / (rows * pb)).sum())
    assert chi2 < 30.0, (chi2, counts / rows, pb)
    acc = (n.cpu() == 2).float().mean()
    expect = float(torch.minimum(p, q).sum())  # acceptance rate of one draft
    assert abs(float(acc) - expect) < 0.02


def test_rejection_greedy(b200_ops):
    V, k = 50, 3
    tgt = torch.randn(4, k + 1, V, device="cuda").to(torch.bfloat16)
    am = tgt.float().argmax(-1).to(torch.int32)
    drafts = am[:, :k].clone()
    drafts[1, 1] = (drafts[1, 1] + 1) % V  # row 1 rejects at position 1
    temp = torch.zeros(4, device="cuda")
    seeds = torch.zeros(4, device="cuda", dtype=torch.int64)
    out, n = sampling.rejection_sample(tgt, tgt[:, :k].contiguous(), drafts, temp, seeds, 0)
    assert n.tolist() == [4, 2, 4, 4]
    assert out[0].tolist() == am[0].tolist()
    assert out[1, :2].tolist() == am[1, :2].tolist() and out[1, 2:].tolist() == [-1, -1]
