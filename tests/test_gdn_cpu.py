"""Gated-DeltaNet oracles on CPU (the contracts the CUDA kernels are tested
against), each checked against an independent formulation:

* causal conv1d == a depthwise ``F.conv1d`` over [state | x] with left
  history, and the rolling state holds the last W-1 inputs;
* the delta rule == the closed form S_t = e^g S_{t-1} (I - beta k k^T) +
  beta v k^T, batched over heads; GQA maps v-head h to k-head h // (HV/HK);
* prefill-then-decode (state carried through slots) == one prefill, for both;
* slot < 0 runs from a zero state and leaves every stored state untouched;
* gated RMSNorm == rmsnorm(o) (rounded to bf16) * w * silu(z) per head.
"""
import torch
import torch.nn.functional as F

from vllm_sm70_b200.ops import gdn


def test_conv1d_matches_depthwise_conv():
    g = torch.Generator().manual_seed(0)
    C, W, L = 12, 4, 9
    x = torch.randn(L, C, generator=g)
    w = torch.randn(C, W, generator=g)
    bias = torch.randn(C, generator=g)
    hist = torch.randn(C, W - 1, generator=g)
    state = hist[None].clone()
    y = gdn.causal_conv1d_ref(x, w, bias, state, torch.tensor([0, L]), torch.tensor([0]))
    ref = F.conv1d(torch.cat([hist, x.t()], 1)[None], w[:, None, :], bias, groups=C)[0].t()
    assert torch.allclose(y, F.silu(ref), atol=1e-5)
    assert torch.equal(state[0], x.t()[:, -(W - 1):])


def _gdn_inputs(T, HK, HV, DK, DV, seed=1):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    return (r(T, HK * DK), r(T, HK * DK), r(T, HV * DV), r(T, HV), r(T, HV), r(HV) * 0.3,
            r(HV) * 0.3)


def _closed_form(q, k, v, a, b, A_log, dt_bias, HK, HV, S0):
    """Delta rule as S <- e^g S (I - beta k k^T) + beta v k^T, all heads at once."""
    T = q.shape[0]
    DK, DV = q.shape[1] // HK, v.shape[1] // HV
    rep = HV // HK
    S = S0.clone()                                                   # [HV, DV, DK]
    out = torch.empty(T, HV, DV)
    eye = torch.eye(DK)
    for t in range(T):
        qt = q[t].view(HK, DK).repeat_interleave(rep, 0)
        kt = k[t].view(HK, DK).repeat_interleave(rep, 0)
        qt = qt / (qt.pow(2).sum(-1, keepdim=True) + 1e-6).sqrt() * DK ** -0.5
        kt = kt / (kt.pow(2).sum(-1, keepdim=True) + 1e-6).sqrt()
        gt = -A_log.exp() * F.softplus(a[t] + dt_bias)              # [HV]
        beta = torch.sigmoid(b[t])
        vt = v[t].view(HV, DV)
        P = eye - beta[:, None, None] * kt[:, :, None] * kt[:, None, :]
        S = gt.exp()[:, None, None] * (S @ P) + beta[:, None, None] * vt[:, :, None] * kt[:, None, :]
        out[t] = (S @ qt[:, :, None])[..., 0]
    return out.reshape(T, HV * DV), S


def test_delta_rule_matches_closed_form_with_gqa():
    HK, HV, DK, DV, T = 2, 4, 8, 6, 7
    q, k, v, a, b, A_log, dt = _gdn_inputs(T, HK, HV, DK, DV)
    S0 = torch.randn(HV, DV, DK, generator=torch.Generator().manual_seed(5))
    state = S0[None].clone()
    o = gdn.gdn_recurrent_ref(q, k, v, a, b, A_log, dt, state, torch.tensor([0, T]),
                              torch.tensor([0]), HK, HV)
    ref, S_end = _closed_form(q, k, v, a, b, A_log, dt, HK, HV, S0)
    assert torch.allclose(o, ref, atol=1e-5)
    assert torch.allclose(state[0], S_end, atol=1e-5)
    # v-heads 0, 1 read k-head 0 only: changing k-head 1 leaves them alone
    q2, k2 = q.clone(), k.clone()
    q2[:, DK:] += 1.0
    k2[:, DK:] -= 1.0
    o2 = gdn.gdn_recurrent_ref(q2, k2, v, a, b, A_log, dt, S0[None].clone(),
                               torch.tensor([0, T]), torch.tensor([0]), HK, HV)
    assert torch.equal(o2[:, : 2 * DV], o[:, : 2 * DV])
    assert not torch.allclose(o2[:, 2 * DV:], o[:, 2 * DV:])


def test_prefill_then_decode_equals_one_prefill():
    HK, HV, DK, DV, T, split = 1, 2, 8, 8, 9, 5
    q, k, v, a, b, A_log, dt = _gdn_inputs(T, HK, HV, DK, DV, seed=3)
    one = torch.zeros(2, HV, DV, DK)
    o_all = gdn.gdn_recurrent_ref(q, k, v, a, b, A_log, dt, one, torch.tensor([0, T]),
                                  torch.tensor([1]), HK, HV)
    st = torch.zeros(2, HV, DV, DK)
    parts = [gdn.gdn_recurrent_ref(q[:split], k[:split], v[:split], a[:split], b[:split], A_log,
                                   dt, st, torch.tensor([0, split]), torch.tensor([1]), HK, HV)]
    for t in range(split, T):  # decode: one token per call, state carried in slot 1
        parts.append(gdn.gdn_recurrent_ref(q[t:t + 1], k[t:t + 1], v[t:t + 1], a[t:t + 1],
                                           b[t:t + 1], A_log, dt, st, torch.tensor([0, 1]),
                                           torch.tensor([1]), HK, HV))
    assert torch.allclose(torch.cat(parts), o_all, atol=1e-5)
    assert torch.allclose(st, one, atol=1e-5) and not st[0].any()
    # conv1d, likewise
    g = torch.Generator().manual_seed(4)
    C, W = 6, 4
    x, w = torch.randn(T, C, generator=g), torch.randn(C, W, generator=g)
    s_all, s_inc = torch.zeros(1, C, W - 1), torch.zeros(1, C, W - 1)
    y_all = gdn.causal_conv1d_ref(x, w, None, s_all, torch.tensor([0, T]), torch.tensor([0]))
    ys = [gdn.causal_conv1d_ref(x[:split], w, None, s_inc, torch.tensor([0, split]),
                                torch.tensor([0]))]
    ys += [gdn.causal_conv1d_ref(x[t:t + 1], w, None, s_inc, torch.tensor([0, 1]),
                                 torch.tensor([0])) for t in range(split, T)]
    assert torch.allclose(torch.cat(ys), y_all, atol=1e-6) and torch.equal(s_inc, s_all)


def test_negative_slot_is_stateless():
    HK, HV, DK, DV, T = 1, 1, 4, 4, 5
    q, k, v, a, b, A_log, dt = _gdn_inputs(T, HK, HV, DK, DV, seed=6)
    st = torch.randn(1, HV, DV, DK)
    keep = st.clone()
    o = gdn.gdn_recurrent_ref(q, k, v, a, b, A_log, dt, st, torch.tensor([0, T]),
                              torch.tensor([-1]), HK, HV)
    ref, _ = _closed_form(q, k, v, a, b, A_log, dt, HK, HV, torch.zeros(HV, DV, DK))
    assert torch.allclose(o, ref, atol=1e-5) and torch.equal(st, keep)


def test_gated_rmsnorm_formula():
    g = torch.Generator().manual_seed(7)
    T, H, D = 3, 2, 8
    o, z, w = torch.randn(T, H * D, generator=g), torch.randn(T, H * D, generator=g), \
        torch.randn(D, generator=g)
    got = gdn.gated_rmsnorm_ref(o, z, w, H, 1e-6)
    of = o.view(T, H, D)
    n = (of / (of.pow(2).mean(-1, keepdim=True) + 1e-6).sqrt()).to(torch.bfloat16).float()
    assert torch.allclose(got, (n * w * F.silu(z.view(T, H, D))).view(T, H * D), atol=1e-6)
