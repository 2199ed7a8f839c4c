"""Gated-DeltaNet kernels vs the fp32 torch oracle: causal conv1d with
rolling state (prefill then decode continues exactly), the gated delta rule
(varlen prefill; decode steps continuing the state; slot < 0 = no state),
gated RMSNorm."""
import pytest
import torch

from vllm_sm70_b200.ops import gdn

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


def test_conv1d_prefill_then_decode(b200_ops):
    torch.manual_seed(0)
    C, W = 256, 4
    lens = [5, 1, 17]
    T = sum(lens)
    x = torch.randn(T, C, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(C, W, device="cuda", dtype=torch.bfloat16) * 0.5
    cu = torch.tensor([0, 5, 6, 23], device="cuda", dtype=torch.int32)
    slots = torch.tensor([2, 0, 1], device="cuda", dtype=torch.int32)
    st = torch.randn(4, C, W - 1, device="cuda")
    st_ref = st.clone()
    y = gdn.causal_conv1d(x, w, None, st, cu, slots)
    yr = gdn.causal_conv1d_ref(x, w, None, st_ref, cu, slots)
    assert _rel(y, yr) < 1e-2
    assert torch.allclose(st, st_ref)
    # one decode token per sequence continues the state
    x2 = torch.randn(3, C, device="cuda", dtype=torch.bfloat16)
    cu2 = torch.arange(4, device="cuda", dtype=torch.int32)
    y2 = gdn.causal_conv1d(x2, w, None, st, cu2, slots)
    y2r = gdn.causal_conv1d_ref(x2, w, None, st_ref, cu2, slots)
    assert _rel(y2, y2r) < 1e-2


@pytest.mark.parametrize("HK,HV,D", [(2, 4, 128), (1, 1, 64)])
def test_gdn_recurrent_prefill_and_decode(b200_ops, HK, HV, D):
    torch.manual_seed(1)
    lens = [7, 30, 1]
    T = sum(lens)
    cu = torch.tensor([0, 7, 37, 38], device="cuda", dtype=torch.int32)
    slots = torch.tensor([1, -1, 0], device="cuda", dtype=torch.int32)

    def inputs(T):
        return (torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16),
                torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16),
                torch.randn(T, HV * D, device="cuda", dtype=torch.bfloat16),
                torch.randn(T, HV, device="cuda", dtype=torch.bfloat16),
                torch.randn(T, HV, device="cuda", dtype=torch.bfloat16))

    A_log = torch.randn(HV, device="cuda") * 0.5
    dt = torch.randn(HV, device="cuda") * 0.5
    st = torch.randn(2, HV, D, D, device="cuda") * 0.1
    st_ref = st.clone()
    q, k, v, a, b = inputs(T)
    o = gdn.gdn_recurrent(q, k, v, a, b, A_log, dt, st, cu, slots, HK, HV)
    orf = gdn.gdn_recurrent_ref(q, k, v, a, b, A_log, dt, st_ref, cu, slots, HK, HV)
    assert _rel(o, orf) < 2e-2
    assert torch.allclose(st, st_ref, atol=1e-3, rtol=1e-3)
    for _ in range(3):  # decode continues from the stored states
        cu1 = torch.arange(4, device="cuda", dtype=torch.int32)
        q, k, v, a, b = inputs(3)
        o = gdn.gdn_recurrent(q, k, v, a, b, A_log, dt, st, cu1, slots, HK, HV)
        orf = gdn.gdn_recurrent_ref(q, k, v, a, b, A_log, dt, st_ref, cu1, slots, HK, HV)
        assert _rel(o, orf) < 2e-2


def test_gated_rmsnorm(b200_ops):
    torch.manual_seed(2)
    o = torch.randn(9, 4 * 128, device="cuda", dtype=torch.bfloat16)
    z = torch.randn(9, 4 * 128, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(128, device="cuda", dtype=torch.bfloat16)
    ref = gdn.gated_rmsnorm_ref(o, z, w, 4, 1e-6)
    gdn.gated_rmsnorm(o, z, w, 4, 1e-6)
    assert _rel(o, ref) < 2e-2


def _gdn_ref_fast(q, k, v, a, b, A_log, dt_bias, state, cu, slots, HK, HV):
    """fp32 oracle vectorised over heads (token loop only): long sequences."""
    import torch.nn.functional as F

    T = q.shape[0]
    DK = q.shape[1] // HK
    DV = v.shape[1] // HV
    o = torch.empty(T, HV * DV, dtype=torch.float32, device=q.device)
    rep = HV // HK
    for s in range(len(slots)):
        t0, t1 = int(cu[s]), int(cu[s + 1])
        slot = int(slots[s])
        S = (state[slot].clone() if slot >= 0 else torch.zeros(HV, DV, DK, device=q.device))
        qs = q[t0:t1].float().view(-1, HK, DK).repeat_interleave(rep, 1)
        ks = k[t0:t1].float().view(-1, HK, DK).repeat_interleave(rep, 1)
        qs = qs / (qs.pow(2).sum(-1, keepdim=True) + 1e-6).sqrt() * DK ** -0.5
        ks = ks / (ks.pow(2).sum(-1, keepdim=True) + 1e-6).sqrt()
        g = -torch.exp(A_log)[None] * F.softplus(a[t0:t1].float() + dt_bias[None])
        beta = torch.sigmoid(b[t0:t1].float())
        vs = v[t0:t1].float().view(-1, HV, DV)
        for t in range(t1 - t0):
            S = S * torch.exp(g[t])[:, None, None]
            kt = ks[t]
            u = torch.einsum("hvk,hk->hv", S, kt)
            S = S + beta[t][:, None, None] * torch.einsum("hv,hk->hvk", vs[t] - u, kt)
            o[t0 + t] = torch.einsum("hvk,hk->hv", S, qs[t]).reshape(-1)
        if slot >= 0:
            state[slot] = S
    return o


@pytest.mark.parametrize("HK,HV", [(2, 4), (16, 32)])
def test_gdn_chunked_prefill_matches_recurrence(b200_ops, HK, HV):
    """Chunked (64-token WY/UT) prefill vs the fp32 token-serial oracle: chunk
    boundaries, partial chunks, carried-in states, slot < 0, state write-back."""
    torch.manual_seed(5)
    D = 128
    lens = [1, 63, 64, 65, 300, 200]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device="cuda", dtype=torch.int32)
    slots = torch.tensor([0, 1, -1, 2, 3, 4], device="cuda", dtype=torch.int32)
    q = torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, HV * D, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(T, HV, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(T, HV, device="cuda", dtype=torch.bfloat16)
    A_log = torch.randn(HV, device="cuda") * 0.5
    dt = torch.randn(HV, device="cuda") * 0.5
    st = torch.randn(5, HV, D, D, device="cuda") * 0.1
    st_ref = st.clone()
    o = gdn.gdn_recurrent(q, k, v, a, b, A_log, dt, st, cu, slots, HK, HV, chunked=True)
    orf = _gdn_ref_fast(q, k, v, a, b, A_log, dt, st_ref, cu, slots, HK, HV)
    torch.cuda.synchronize()
    assert _rel(o, orf) < 3e-2
    assert _rel(st, st_ref) < 3e-2


def test_gdn_chunked_long_sequence(b200_ops):
    """8192 tokens (the Qwen3-Next prompt length) in one sequence: the chunked
    kernel stays on the fp32 recurrence over 128 chunks of carried state."""
    torch.manual_seed(6)
    HK, HV, D, T = 1, 2, 128, 8192
    cu = torch.tensor([0, T], device="cuda", dtype=torch.int32)
    slots = torch.tensor([0], device="cuda", dtype=torch.int32)
    q = torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, HV * D, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(T, HV, device="cuda", dtype=torch.bfloat16) - 2
    b = torch.randn(T, HV, device="cuda", dtype=torch.bfloat16)
    A_log = torch.randn(HV, device="cuda") * 0.5 - 1
    dt = torch.randn(HV, device="cuda") * 0.5
    st = torch.zeros(1, HV, D, D, device="cuda")
    st_ref = st.clone()
    o = gdn.gdn_recurrent(q, k, v, a, b, A_log, dt, st, cu, slots, HK, HV, reset_state=True,
                          chunked=True)
    orf = _gdn_ref_fast(q, k, v, a, b, A_log, dt, st_ref, cu, slots, HK, HV)
    torch.cuda.synchronize()
    assert _rel(o, orf) < 3e-2
    assert _rel(st, st_ref) < 3e-2


@pytest.mark.parametrize("chunked", [False, True])
def test_gdn_paged_state_and_fresh_sequences(b200_ops, chunked):
    """State slots padded apart (vLLM's paged hybrid cache: slot stride past
    the dense [HV, DV, DK] block) and per-sequence ``has_init`` (False: start
    from zero, still store the final state): both kernels vs the fp32 oracle
    on a dense copy; slots nobody owns and the padding floats stay untouched."""
    torch.manual_seed(7)
    HK, HV, D = 2, 4, 128
    lens = [70, 1, 33, 5]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device="cuda", dtype=torch.int32)
    slots = torch.tensor([4, 1, 2, -1], device="cuda", dtype=torch.int32)
    has_init = torch.tensor([True, False, True, False], device="cuda")
    q = torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, HK * D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, HV * D, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(T, HV, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(T, HV, device="cuda", dtype=torch.bfloat16)
    A_log = torch.randn(HV, device="cuda") * 0.5
    dt = torch.randn(HV, device="cuda") * 0.5
    blk, pad, nslot = HV * D * D, 12, 5
    store = torch.randn(nslot * (blk + pad), device="cuda") * 0.1
    st = store.as_strided((nslot, HV, D, D), (blk + pad, D * D, D, 1))
    st_ref = st.clone()  # dense
    st_ref[1].zero_()  # slot 1's sequence has no initial state
    before = store.clone()
    o = gdn.gdn_recurrent(q, k, v, a, b, A_log, dt, st, cu, slots, HK, HV, chunked=chunked,
                          has_init=has_init)
    orf = _gdn_ref_fast(q, k, v, a, b, A_log, dt, st_ref, cu, slots, HK, HV)
    torch.cuda.synchronize()
    tol = 3e-2 if chunked else 2e-2
    assert _rel(o, orf) < tol
    for s in (4, 1, 2):
        assert _rel(st[s], st_ref[s]) < tol
    for s in (0, 3):  # no sequence owns them
        assert torch.equal(st[s], before.as_strided(st.shape, st.stride())[s])
    gaps = store.view(nslot, blk + pad)[:, blk:]
    assert torch.equal(gaps, before.view(nslot, blk + pad)[:, blk:])
