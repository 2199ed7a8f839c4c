"""vLLM's Qwen GDN layers on this library's gated-delta-rule route, on CPU
(the op wrappers' fp32 oracles stand in for the kernels): the core reads and
writes vLLM's paged fp32 state in place, sequences without an initial state
start from zero, padding rows of a decode batch (the null block) touch no
slot, and the route declines what it does not serve. The layer subclass is
installed in vLLM's out-of-tree registry under the upstream name."""
import types

import pytest
import torch

from vllm_sm70_b200.integration import gdn as G
from vllm_sm70_b200.ops import gdn as gdn_ops

HK, HV, D = 1, 2, 128
KD, VD = HK * D, HV * D
CONV = 2 * KD + VD


def _layer():
    torch.manual_seed(0)
    return types.SimpleNamespace(
        num_k_heads=HK, num_v_heads=HV, head_k_dim=D, head_v_dim=D, tp_size=1,
        A_log=torch.nn.Parameter(torch.randn(HV) * 0.5, requires_grad=False),
        dt_bias=torch.nn.Parameter((torch.randn(HV) * 0.5).to(torch.bfloat16),
                                   requires_grad=False))


def _paged_state(slots: int, pad: int = 4) -> torch.Tensor:
    """[slots, HV, D, D] fp32 whose slots sit ``pad`` floats apart beyond the
    dense block (as pages of a hybrid cache)."""
    blk = HV * D * D
    store = torch.randn(slots * (blk + pad)) * 0.1
    return store.as_strided((slots, HV, D, D), (blk + pad, D * D, D, 1))


def _md(**kw):
    base = dict(num_prefills=0, num_decodes=0, num_actual_tokens=0, has_initial_state=None,
                non_spec_query_start_loc=None, non_spec_state_indices_tensor=None,
                spec_sequence_masks=None)
    base.update(kw)
    return types.SimpleNamespace(**base)


def _conv_identity(x, *_):
    return x  # conv1d is vLLM's; the core is checked on its output


def _oracle(layer, x, a, b, state, cu, slots, has_init):
    st = state.clone()  # dense copy
    for s, ok in enumerate(has_init):
        if not ok and int(slots[s]) >= 0:
            st[int(slots[s])].zero_()
    o = gdn_ops.gdn_recurrent_ref(x[:, :KD], x[:, KD:2 * KD], x[:, 2 * KD:], a, b,
                                  layer.A_log.float(), layer.dt_bias.float(), st, cu, slots,
                                  HK, HV)
    return o, st


def test_prefill_on_paged_state_with_fresh_sequences():
    layer = _layer()
    lens = [5, 1, 9]
    T = sum(lens)
    x = torch.randn(T, CONV, dtype=torch.bfloat16)
    ba = torch.randn(T, 2 * HV, dtype=torch.bfloat16)
    b, a = ba[:, :HV], ba[:, HV:]  # column views of one projection, as vLLM splits them
    state = _paged_state(5)
    cu = torch.tensor([0, 5, 6, 15], dtype=torch.int32)
    slots = torch.tensor([3, 1, 4], dtype=torch.int32)
    has_init = torch.tensor([True, False, True])
    md = _md(num_prefills=2, num_decodes=1, num_actual_tokens=T, has_initial_state=has_init,
             non_spec_query_start_loc=cu, non_spec_state_indices_tensor=slots)
    ref_o, ref_st = _oracle(layer, x, a, b, state, cu, slots, has_init.tolist())
    out = torch.full((T + 3, HV, D), float("nan"), dtype=torch.bfloat16)
    untouched = state[0].clone(), state[2].clone()
    assert G.gdn_core(layer, x, b, a, out, md, None, state, _conv_identity, _conv_identity)
    assert torch.equal(out[:T].reshape(T, VD), ref_o.to(torch.bfloat16))
    assert torch.isnan(out[T:].float()).all()  # rows past the batch are not written
    for s in slots.tolist():
        assert torch.allclose(state[s], ref_st[s])
    assert torch.equal(state[0], untouched[0]) and torch.equal(state[2], untouched[1])


def test_decode_skips_null_block_padding():
    layer = _layer()
    n = 4  # two live rows, two captured-batch padding rows on the null block
    x = torch.randn(n, CONV, dtype=torch.bfloat16)
    a = torch.randn(n, HV, dtype=torch.bfloat16)
    b = torch.randn(n, HV, dtype=torch.bfloat16)
    state = _paged_state(4)
    idx = torch.tensor([2, 3, 0, 0], dtype=torch.int32)
    md = _md(num_decodes=n, num_actual_tokens=n, non_spec_state_indices_tensor=idx)
    null_before = state[0].clone()
    ref_o, ref_st = _oracle(layer, x[:2], a[:2], b[:2], state,
                            torch.tensor([0, 1, 2], dtype=torch.int32), idx[:2], [True, True])
    out = torch.empty(n, HV, D, dtype=torch.bfloat16)
    seen = {}

    def conv_decode(xx, ii):
        seen["idx"] = ii
        return xx

    assert G.gdn_core(layer, x, b, a, out, md, None, state, None, conv_decode)
    assert torch.equal(seen["idx"], idx)  # vLLM's conv update gets vLLM's indices
    assert torch.equal(out[:2].reshape(2, VD), ref_o.to(torch.bfloat16))
    assert torch.equal(state[0], null_before)  # the null block is neither read nor written
    for s in (2, 3):
        assert torch.allclose(state[s], ref_st[s])


def test_route_declines_what_it_does_not_serve():
    layer = _layer()
    d = G.GdnDims.of(layer)
    st = _paged_state(2)
    dec = _md(num_decodes=1, num_actual_tokens=1)
    assert G.can_serve(dec, st, d)
    assert not G.can_serve(dec, st.to(torch.bfloat16), d)  # vLLM's default bf16 state
    assert not G.can_serve(_md(num_decodes=1, spec_sequence_masks=torch.ones(1, dtype=torch.bool)),
                           st, d)
    assert not G.can_serve(_md(), st, d)  # nothing to do
    blk = HV * D * D
    odd = torch.zeros(2 * (blk + 1)).as_strided((2, HV, D, D), (blk + 1, D * D, D, 1))
    assert not G.can_serve(dec, odd, d)  # slot stride breaks the 16-byte alignment
    d64 = G.GdnDims(HK, HV, 64, 64)
    st64 = torch.zeros(2, HV, 64, 64)
    assert G.can_serve(dec, st64, d64)  # decode kernel takes 64
    assert not G.can_serve(_md(num_prefills=1, num_actual_tokens=3), st64, d64)  # chunked: 128
    # declining leaves everything untouched
    out = torch.zeros(1, HV, D, dtype=torch.bfloat16)
    assert not G.gdn_core(layer, torch.zeros(1, CONV, dtype=torch.bfloat16),
                          torch.zeros(1, HV, dtype=torch.bfloat16),
                          torch.zeros(1, HV, dtype=torch.bfloat16), out, dec, None,
                          st.to(torch.bfloat16), None, None)
    assert not out.any()


def test_gate_parameters_cached_as_fp32_and_refreshed():
    layer = _layer()
    f1 = G._fp32(layer, "dt_bias")
    assert f1.dtype == torch.float32 and G._fp32(layer, "dt_bias") is f1
    with torch.no_grad():
        layer.dt_bias.copy_(torch.ones(HV))  # a weight load writes in place
    f2 = G._fp32(layer, "dt_bias")
    assert f2 is not f1 and torch.equal(f2, torch.ones(HV))
    assert G._fp32(layer, "A_log").data_ptr() == layer.A_log.data_ptr()  # fp32 already


def test_layer_subclass_registered_out_of_tree(monkeypatch):
    pytest.importorskip("vllm")
    from vllm.model_executor.custom_op import op_registry_oot
    from vllm.model_executor.layers.mamba.gdn import qwen_gdn_linear_attn as up

    from vllm_sm70_b200.integration import vllm_models

    name = "QwenGatedDeltaNetAttention"
    monkeypatch.setattr(vllm_models, "_b200_active", lambda: False)
    monkeypatch.setattr(G, "INSTALLED", {})
    assert G.register() == {}  # not on a B200: upstream stays
    assert name not in op_registry_oot
    monkeypatch.setattr(vllm_models, "_b200_active", lambda: True)
    try:
        got = G.register()
        cls = got[name]
        assert op_registry_oot[name] is cls
        assert issubclass(cls, up.QwenGatedDeltaNetAttention)
        assert cls._forward_core is not up.QwenGatedDeltaNetAttention._forward_core
        assert G.register() == got  # idempotent
    finally:
        op_registry_oot.pop(name, None)
