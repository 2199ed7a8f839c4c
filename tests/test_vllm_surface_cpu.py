"""The vLLM-facing surface of the plugin, on CPU: packaging entry points,
model registration, quantisation configs, the RMSNorm IR-op provider, the
fused-MoE method, and the U3 / U4 call sites installed by runtime wrapping
(checked on stand-in runner classes: with no hook answering, the wrapped
methods behave exactly as the originals)."""
import tomllib
import types
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
vllm = pytest.importorskip("vllm")


def test_pyproject_declares_both_plugin_groups():
    import importlib

    d = tomllib.loads((ROOT / "pyproject.toml").read_text())
    eps = d["project"]["entry-points"]
    assert eps["vllm.general_plugins"] == {"b200": "vllm_sm70_b200:register"}
    assert eps["vllm.platform_plugins"] == {"b200": "vllm_sm70_b200.platform:activate"}
    for target in (*eps["vllm.general_plugins"].values(), *eps["vllm.platform_plugins"].values()):
        mod, _, fn = target.partition(":")
        assert callable(getattr(importlib.import_module(mod), fn))


def test_models_registered_with_vllm_registry():
    from vllm.model_executor.models import ModelRegistry

    from vllm_sm70_b200.integration import models

    got = models.register_models()
    assert set(got) == set(models.VLLM_ARCHS)
    for arch, target in models.VLLM_ARCHS.items():
        entry = ModelRegistry.models[arch]
        assert (entry.module_name, entry.class_name) == tuple(target.split(":"))
    # The lazy targets resolve to vLLM model subclasses.
    from vllm.model_executor.models.llama import LlamaForCausalLM
    from vllm.model_executor.models.qwen3_moe import Qwen3MoeForCausalLM

    from vllm_sm70_b200.integration import vllm_models

    assert issubclass(vllm_models.B200LlamaForCausalLM, LlamaForCausalLM)
    assert issubclass(vllm_models.B200Qwen3MoeForCausalLM, Qwen3MoeForCausalLM)


def test_interleave_rows_inplace_matches_engine_layout():
    from vllm_sm70_b200.integration.vllm_models import interleave_rows_inplace
    from vllm_sm70_b200.ops.linear import interleave_gate_up

    g, u = torch.randn(256, 32), torch.randn(256, 32)
    w = torch.cat([g, u]).clone()
    ptr = w.data_ptr()
    interleave_rows_inplace(w)
    assert w.data_ptr() == ptr and torch.equal(w, interleave_gate_up(g, u))


def test_quant_configs_registered_and_routed(monkeypatch):
    from vllm.model_executor.layers.quantization import get_quantization_config

    from vllm_sm70_b200.integration import quant

    reg = quant.register()
    assert set(reg) == {"fp8", "awq", "modelopt_fp4"}
    for name, cls in reg.items():
        assert get_quantization_config(name) is cls
    fp8 = quant.CONFIGS["fp8"].from_config({"quant_method": "fp8", "activation_scheme": "dynamic",
                                            "weight_block_size": [128, 128]})
    awq = quant.CONFIGS["awq"].from_config({"quant_method": "awq", "bits": 4, "group_size": 128,
                                            "zero_point": True})
    from vllm.model_executor.layers.linear import ReplicatedLinear
    from vllm.model_executor.layers.quantization.awq import AWQLinearMethod
    from vllm.model_executor.layers.quantization.fp8 import Fp8LinearMethod

    # Upstream method constructors read the running engine's config; the
    # routing decision is what is checked here.
    monkeypatch.setattr(Fp8LinearMethod, "__init__", lambda self, qc: setattr(self, "quant_config", qc))
    layer = object.__new__(ReplicatedLinear)  # a LinearBase instance
    monkeypatch.setattr(quant, "_active", lambda: False)  # not on a B200: upstream stays
    assert type(fp8.get_quant_method(layer, "x")) is Fp8LinearMethod
    assert type(awq.get_quant_method(layer, "y")) is AWQLinearMethod
    monkeypatch.setattr(quant, "_active", lambda: True)
    m = fp8.get_quant_method(layer, "x")
    assert type(m) is quant.METHODS["fp8"]
    assert type(awq.get_quant_method(layer, "y")) is quant.METHODS["awq"]
    # The B200 method converts the loaded tensors into this library's layout.
    from vllm_sm70_b200.ops import quant as Q

    w = torch.randn(256, 256) * 0.05
    q, sc = Q.quantize_fp8_block(w)
    lin = types.SimpleNamespace(weight=torch.nn.Parameter(q, requires_grad=False),
                                weight_scale_inv=torch.nn.Parameter(sc, requires_grad=False),
                                output_size_per_partition=256)
    m.process_weights_after_loading(lin)
    x = torch.randn(3, 256, dtype=torch.bfloat16)
    y = m.apply(lin, x)
    ref = lin._b200_linear.reference_forward(x)
    assert (y.float() - ref).abs().max() < 0.05


def test_ir_op_provider_first_in_priority():
    from vllm import ir
    from vllm.config.kernel import IrOpPriorityConfig

    from vllm_sm70_b200.integration import ir_ops

    assert ir_ops.register()
    assert "b200" in ir.ops.rms_norm.impls and "b200" in ir.ops.fused_add_rms_norm.impls
    p = ir_ops.with_b200_first(IrOpPriorityConfig.with_default(["native"]))
    assert p.rms_norm[0] == "b200" and p.fused_add_rms_norm[0] == "b200"
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    w = torch.ones(64, dtype=torch.bfloat16)
    assert not ir_ops.rms_supported(x, w, 1e-5)  # CPU tensors go to the next provider


class _FakeRouter:
    def select_experts(self, hidden_states, router_logits, input_ids=None):
        return ("upstream", None)


class _FakeQuant:
    is_monolithic = False

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        return topk_weights, topk_ids


class _FakeMoERunner:
    def __init__(self):
        self.router = _FakeRouter()
        self._quant_method = _FakeQuant()

    def _apply_quant_method(self, layer, hidden_states, router_logits, shared_experts_input,
                            input_ids=None):
        w, ids = self.router.select_experts(hidden_states=hidden_states,
                                            router_logits=router_logits, input_ids=input_ids)
        return self._quant_method.apply(layer, hidden_states, w, ids)


def test_u3_call_site_uses_the_route_and_is_inert_without_one():
    from vllm_sm70_b200.integration import hooks

    answer = {"route": None}

    class Route:
        def try_route(self, h, logits):
            return ("b200-w", "b200-ids")

    plat = types.SimpleNamespace(get_moe_router_provider=lambda: (lambda runner: answer["route"]))
    hooks._install_u3(plat, _FakeMoERunner, key="test_u3")
    r = _FakeMoERunner()
    assert r._apply_quant_method(None, 1, 2, None) == ("upstream", None)
    answer["route"] = Route()
    assert r._apply_quant_method(None, 1, 2, None) == ("b200-w", "b200-ids")
    assert "select_experts" not in vars(r.router)  # the override was for one call
    answer["route"] = None
    assert r._apply_quant_method(None, 1, 2, None) == ("upstream", None)


def test_u3_route_for_vllm_fused_topk_router():
    from vllm_sm70_b200.ops import moe

    FusedTopKRouter = type("FusedTopKRouter", (), {})
    router = FusedTopKRouter()
    router.top_k, router.renormalize, router.scoring_func, router.eplb_state = 8, True, \
        "softmax", None
    route = moe.make_route_for_runner(types.SimpleNamespace(router=router))
    assert isinstance(route, moe.TopKRoute) and route.top_k == 8 and not route.use_sigmoid
    router.scoring_func = "sqrtsoftplus"
    assert moe.make_route_for_runner(types.SimpleNamespace(router=router)) is None
    assert route.try_route(None, torch.randn(3, 16)) is None  # CPU logits: vLLM routes


class _FakeBatch:
    sampling_metadata = "md"

    def update_async_output_token_ids(self):
        pass


class _FakeModel:
    def compute_logits(self, h):
        return h * 2


class _FakeGPURunner:
    is_pooling_model = False

    def __init__(self):
        self.model = _FakeModel()
        self.input_batch = _FakeBatch()

    def execute_model(self, scheduler_output):
        self.logits = self.model.compute_logits(torch.ones(2, 3))

    def _sample(self, logits, spec_decode_metadata):
        return ("upstream", logits.shape)


def test_u4_call_site_skips_compute_logits_when_the_sampler_answers():
    from vllm_sm70_b200.integration import hooks

    class Sampler:
        answer = None

        def try_sample(self, model, h, md, so, spec):
            return self.answer

    smp = Sampler()
    plat = types.SimpleNamespace(get_hidden_state_sampler=lambda: smp)
    hooks._install_u4(plat, _FakeGPURunner, key="test_u4")
    so = types.SimpleNamespace(has_structured_output_requests=False,
                               scheduled_spec_decode_tokens={})
    r = _FakeGPURunner()
    r.execute_model(so)  # sampler defers: upstream logits
    assert torch.equal(r.logits, torch.full((2, 3), 2.0))
    assert r._sample(r.logits, None) == ("upstream", (2, 3))
    smp.answer = "b200-out"
    r.execute_model(so)
    assert r.logits.shape == (2, 0)  # no logits materialised
    assert r._sample(r.logits, None) == "b200-out"
    # Structured output or spec decode: the sampler is not consulted.
    so2 = types.SimpleNamespace(has_structured_output_requests=True,
                                scheduled_spec_decode_tokens={})
    r.execute_model(so2)
    assert r.logits.shape == (2, 3)
    assert not hooks.u4_admits(types.SimpleNamespace(has_structured_output_requests=False,
                                                     scheduled_spec_decode_tokens={"a": [1]}))


def test_hidden_state_sampler_rejects_what_it_does_not_serve():
    from vllm_sm70_b200.engine import hidden_state_sampler as hss

    s = hss.HiddenStateSampler()
    s.prepared = True
    md = types.SimpleNamespace(all_greedy=False)
    assert s.try_sample(None, None, md) is None
    md = types.SimpleNamespace(all_greedy=True, max_num_logprobs=5)
    assert s.try_sample(None, None, md) is None
    md = types.SimpleNamespace(all_greedy=True, max_num_logprobs=None, no_penalties=True,
                               allowed_token_ids_mask=None, bad_words_token_ids={},
                               logitsprocs=None)
    head = types.SimpleNamespace(weight=torch.zeros(4, 4, dtype=torch.bfloat16), bias=None,
                                 shard_indices=types.SimpleNamespace(org_vocab_start_index=0,
                                                                     org_vocab_end_index=4),
                                 tp_size=1)
    model = types.SimpleNamespace(lm_head=head,
                                  logits_processor=types.SimpleNamespace(soft_cap=30.0, scale=1.0))
    assert hss.vllm_lm_head(model) is None  # soft cap: upstream path
    model.logits_processor.soft_cap = None
    rows, start, tp = hss.vllm_lm_head(model)
    assert rows.shape == (4, 4) and start == 0 and tp == 1
