"""Flint (hybrid sliding / full attention with learned sinks, no-RoPE layers,
dense + sigmoid-routed MoE layers with an ungated shared expert) on CPU:
HF config parsing, greedy decoding equal to an independent dense forward,
an HF checkpoint round trip, the window / sinks actually taking effect, and
TP2 (gloo ranks: sink heads sharded, dense layers row-parallel) equal to
TP1."""
import json

import torch

from vllm_sm70_b200.engine import LLM, SamplingParams
from vllm_sm70_b200.models.config import ModelConfig

from . import _mp
from ._flint_ref import greedy_reference

HF = {"architectures": ["FlintForCausalLM"], "model_type": "flint", "hidden_size": 128,
      "num_hidden_layers": 4, "num_attention_heads": 4, "num_key_value_heads": 2,
      "head_dim": 32, "intermediate_size": 256, "vocab_size": 512, "rms_norm_eps": 1e-6,
      "max_position_embeddings": 512, "tie_word_embeddings": False,
      "layer_types": ["sliding_attention", "full_attention", "sliding_attention",
                      "full_attention"],
      "sliding_window": 8, "no_rope_layer_indices": [1], "mlp_only_layers": [0],
      "rope_parameters": {"sliding_attention": {"rope_theta": 10000.0},
                          "full_attention": {"rope_theta": 1000000.0}},
      "num_experts": 8, "num_experts_per_tok": 2, "moe_intermediate_size": 64,
      "shared_expert_intermediate_size": 128, "norm_topk_prob": True,
      "router_score_function": "sigmoid"}
KW = dict(max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
          enforce_eager=True, max_num_batched_tokens=24)


def _prompts():
    g = torch.Generator().manual_seed(9)
    return [torch.randint(0, 512, (n,), generator=g) for n in (30, 11, 45)]


def test_config_parse():
    cfg = ModelConfig.from_hf(HF)
    assert cfg.arch == "flint" and cfg.qk_norm and cfg.num_experts == 8
    assert cfg.extra["sliding_window"] == 8 and cfg.extra["no_rope_layers"] == [1]
    assert cfg.extra["mlp_only_layers"] == [0]
    assert cfg.extra["rope_theta_by_type"] == {"sliding_attention": 10000.0,
                                               "full_attention": 1000000.0}


def test_greedy_matches_dense_reference():
    llm = LLM(ModelConfig.from_hf(HF), **KW)
    m = llm.model
    assert "experts" not in m.layers[0] and "experts" in m.layers[1]
    assert "shared_gate" not in m.layers[1] and m.layers[1]["sinks"].shape == (4,)
    outs = llm.generate(_prompts(), SamplingParams(max_tokens=5))
    for p, o in zip(_prompts(), outs):
        assert o.output_token_ids == greedy_reference(m, p, 5)


def test_window_and_sinks_take_effect():
    a = LLM(ModelConfig.from_hf(HF), **KW)
    base = a.score(_prompts()[:1])[0]
    no_window = LLM(ModelConfig.from_hf({**HF, "sliding_window": 0}), **KW)
    assert not torch.allclose(no_window.score(_prompts()[:1])[0], base, atol=1e-4)
    for L in a.model.layers:
        L["sinks"] = torch.full_like(L["sinks"], -1e4)  # a sink that takes no mass
    assert not torch.allclose(a.score(_prompts()[:1])[0], base, atol=1e-4)


def _write(path, sd):
    from safetensors.torch import save_file

    (path / "config.json").write_text(json.dumps(HF))
    save_file(sd, str(path / "model.safetensors"))


def test_checkpoint_roundtrip(tmp_path):
    a = LLM(ModelConfig.from_hf(HF), **KW)
    sd = a.model.hf_state_dict()
    assert "model.layers.1.self_attn.softmax_offset" in sd
    assert "model.layers.0.mlp.gate_proj.weight" in sd and "model.layers.0.mlp.gate.weight" not in sd
    assert "model.layers.1.mlp.shared_expert.gate_proj.weight" in sd
    assert not any("shared_expert_gate" in k for k in sd)
    _write(tmp_path, sd)
    b = LLM(str(tmp_path), load_format="safetensors", **KW)
    sp = SamplingParams(max_tokens=5)
    assert ([o.output_token_ids for o in a.generate(_prompts(), sp)]
            == [o.output_token_ids for o in b.generate(_prompts(), sp)])


def _tp_body(rank, world, path, out):
    from pathlib import Path

    from vllm_sm70_b200.parallel import state

    state.init(tp_size=world, backend="gloo", timeout_s=120)
    llm = LLM(path, tensor_parallel_size=world, load_format="safetensors", **KW)
    assert llm.model.layers[1]["sinks"].shape == (4 // world,)
    toks = [o.output_token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=5))]
    if rank == 0:
        Path(out).write_text(json.dumps(toks))
    llm.shutdown()
    state.shutdown()


def test_tp2_equals_tp1(tmp_path):
    a = LLM(ModelConfig.from_hf(HF), **KW)
    _write(tmp_path, a.model.hf_state_dict())
    one = LLM(str(tmp_path), load_format="safetensors", **KW)
    want = [o.output_token_ids for o in one.generate(_prompts(), SamplingParams(max_tokens=5))]
    out = tmp_path / "tp2.json"
    _mp.run(_tp_body, 2, args=(str(tmp_path), str(out)), timeout=300)
    assert json.loads(out.read_text()) == want
