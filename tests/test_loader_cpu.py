"""HF-layout safetensors checkpoints through ``LLM(path, load_format=...)``:
export -> load round trips (Llama, Qwen3-MoE), block-FP8, AutoAWQ int4 and
ModelOpt NVFP4 checkpoints kept in their formats (dense projections, fused
q/k/v and gate/up, MoE experts), and an explicit error where loading is not
built."""
import json

import pytest
import torch

from vllm_sm70_b200.engine import LLM, SamplingParams
from vllm_sm70_b200.models.config import ModelConfig
from vllm_sm70_b200.ops import quant

KW = dict(max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
          enforce_eager=True, max_num_batched_tokens=64)


def _hf_config(cfg: ModelConfig, **extra) -> dict:
    d = {"model_type": "qwen3_moe" if cfg.arch == "qwen3_moe" else "llama",
         "hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_layers,
         "num_attention_heads": cfg.num_heads, "num_key_value_heads": cfg.num_kv_heads,
         "head_dim": cfg.head_dim, "intermediate_size": cfg.intermediate_size,
         "vocab_size": cfg.vocab_size, "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.rms_eps,
         "max_position_embeddings": cfg.max_position, "tie_word_embeddings": False}
    if cfg.arch == "qwen3_moe":
        d.update(num_experts=cfg.num_experts, num_experts_per_tok=cfg.top_k,
                 moe_intermediate_size=cfg.moe_intermediate_size, norm_topk_prob=True)
    d.update(extra)
    return d


def _write(tmp_path, cfg_json: dict, sd: dict):
    from safetensors.torch import save_file

    (tmp_path / "config.json").write_text(json.dumps(cfg_json))
    save_file(sd, str(tmp_path / "model.safetensors"))
    return str(tmp_path)


def _prompts():
    g = torch.Generator().manual_seed(3)
    return [torch.randint(0, 512, (n,), generator=g) for n in (9, 30, 4)]


def _tokens(llm):
    return [o.output_token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=5))]


TINY = ModelConfig(arch="llama", hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=4,
                   head_dim=32, intermediate_size=256, vocab_size=512, rope_theta=10000.0,
                   rms_eps=1e-5, max_position=512)


def test_llama_roundtrip(tmp_path):
    a = LLM(TINY, **KW)
    path = _write(tmp_path, _hf_config(TINY), a.model.hf_state_dict())
    b = LLM(path, load_format="safetensors", **KW)
    assert _tokens(a) == _tokens(b)
    for La, Lb in zip(a.model.layers, b.model.layers):
        assert torch.equal(La["qkv"].w, Lb["qkv"].w) and torch.equal(La["gate_up"].w, Lb["gate_up"].w)


def test_fp8_checkpoint_stays_fp8(tmp_path):
    a = LLM(TINY, **KW)
    sd = a.model.hf_state_dict()
    dense = dict(sd)
    for name in list(sd):
        if name.endswith("_proj.weight"):
            wq, s = quant.quantize_fp8_block(sd[name].float())
            sd[name] = wq
            sd[name.replace(".weight", ".weight_scale_inv")] = s
            dense[name] = quant.Fp8BlockLinear(wq, s).dequant_ref().float()
    cfg = _hf_config(TINY, quantization_config={"quant_method": "fp8",
                                                "weight_block_size": [128, 128]})
    b = LLM(_write(tmp_path, cfg, sd), load_format="safetensors", **KW)
    L0 = b.model.layers[0]
    assert isinstance(L0["qkv"], quant.Fp8BlockLinear) and isinstance(L0["o"], quant.Fp8BlockLinear)
    q = dense["model.layers.0.self_attn.q_proj.weight"]
    k = dense["model.layers.0.self_attn.k_proj.weight"]
    v = dense["model.layers.0.self_attn.v_proj.weight"]
    ref = torch.cat([q, k, v])
    assert torch.allclose(L0["qkv"].reference_weight(), ref, atol=1e-6)
    assert all(len(t) == 5 for t in _tokens(b))


def test_qwen3_moe_roundtrip(tmp_path):
    cfg = ModelConfig(arch="qwen3_moe", hidden_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=32, intermediate_size=256, vocab_size=512,
                      rope_theta=10000.0, rms_eps=1e-6, max_position=512, qk_norm=True,
                      num_experts=8, top_k=2, moe_intermediate_size=64)
    a = LLM(cfg, **KW)
    path = _write(tmp_path, _hf_config(cfg), a.model.hf_state_dict())
    b = LLM(path, load_format="safetensors", **KW)
    assert _tokens(a) == _tokens(b)


def test_missing_checkpoint_is_a_clear_error(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps(_hf_config(TINY)))
    with pytest.raises(FileNotFoundError):
        LLM(str(tmp_path), load_format="safetensors", **KW)


def test_qwen3_next_roundtrip(tmp_path):
    """Hybrid gated-DeltaNet / gated-attention model: HF layouts (per key-head
    group qkvz / ba rows, zero-centred norms) round-trip exactly."""
    cfg = ModelConfig.from_hf({
        "model_type": "qwen3_next", "hidden_size": 128, "num_hidden_layers": 4,
        "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 32,
        "intermediate_size": 256, "vocab_size": 512, "rope_theta": 10000.0,
        "rms_norm_eps": 1e-6, "max_position_embeddings": 512, "tie_word_embeddings": False,
        "num_experts": 8, "num_experts_per_tok": 2, "moe_intermediate_size": 64,
        "shared_expert_intermediate_size": 64, "norm_topk_prob": True,
        "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 32,
        "linear_value_head_dim": 32, "linear_conv_kernel_dim": 4, "full_attention_interval": 2,
        "partial_rotary_factor": 0.25, "num_nextn_predict_layers": 1})
    a = LLM(cfg, **KW)
    g = torch.Generator().manual_seed(11)
    m = a.model
    # non-trivial norms and GDN parameters so every conversion is exercised
    m.final_norm += torch.randn(m.final_norm.shape, generator=g) * 0.1
    for L in m.layers:
        for k in ("in_norm", "post_norm", "q_norm", "k_norm", "gnorm"):
            if k in L:
                L[k] += torch.randn(L[k].shape, generator=g) * 0.1
    hf_json = {"model_type": "qwen3_next", "hidden_size": 128, "num_hidden_layers": 4,
               "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 32,
               "intermediate_size": 256, "vocab_size": 512, "rope_theta": 10000.0,
               "rms_norm_eps": 1e-6, "max_position_embeddings": 512,
               "tie_word_embeddings": False, "num_experts": 8, "num_experts_per_tok": 2,
               "moe_intermediate_size": 64, "shared_expert_intermediate_size": 64,
               "norm_topk_prob": True, "linear_num_key_heads": 2, "linear_num_value_heads": 4,
               "linear_key_head_dim": 32, "linear_value_head_dim": 32,
               "linear_conv_kernel_dim": 4, "full_attention_interval": 2,
               "partial_rotary_factor": 0.25, "num_nextn_predict_layers": 1}
    sd = m.hf_state_dict()
    # HF stores the gated-DeltaNet projection per key-head group: group 1's q
    # rows follow group 0's [q | k | v | z] block.
    w = sd["model.layers.0.linear_attn.in_proj_qkvz.weight"]
    S = 2 * 32 + 2 * 32 * 2
    assert torch.equal(w[S:S + 32], m.layers[0]["qkvz"].w[32:64])
    path = _write(tmp_path, hf_json, sd)
    b = LLM(path, load_format="safetensors", **KW)
    for La, Lb in zip(a.model.layers, b.model.layers):
        for k, va in La.items():
            vb = Lb[k]
            if isinstance(va, torch.Tensor):
                assert torch.allclose(va.float(), vb.float(), atol=1e-6), k
            elif hasattr(va, "w") and isinstance(va.w, torch.Tensor):
                assert torch.equal(va.w, vb.w), k
    assert _tokens(a) == _tokens(b)


def test_qwen3_next_mtp_roundtrip(tmp_path):
    """The MTP draft layer (``mtp.*``, gated attention + MoE, zero-centred
    norms) loads from the checkpoint; speculative greedy decoding then equals
    plain greedy decoding of the same weights."""
    hf_json = {"model_type": "qwen3_next", "hidden_size": 128, "num_hidden_layers": 4,
               "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 32,
               "intermediate_size": 256, "vocab_size": 512, "rope_theta": 10000.0,
               "rms_norm_eps": 1e-6, "max_position_embeddings": 512,
               "tie_word_embeddings": False, "num_experts": 8, "num_experts_per_tok": 2,
               "moe_intermediate_size": 64, "shared_expert_intermediate_size": 64,
               "norm_topk_prob": True, "linear_num_key_heads": 2, "linear_num_value_heads": 4,
               "linear_key_head_dim": 32, "linear_value_head_dim": 32,
               "linear_conv_kernel_dim": 4, "full_attention_interval": 2,
               "partial_rotary_factor": 0.25, "num_nextn_predict_layers": 1}
    cfg = ModelConfig.from_hf(hf_json)
    a = LLM(cfg, speculative_k=2, **KW)
    head = a.runner.mtp
    g = torch.Generator().manual_seed(12)
    for k in ("norm_e", "norm_h", "final_norm"):
        getattr(head, k).add_(torch.randn(getattr(head, k).shape, generator=g) * 0.1)
    sd = dict(a.model.hf_state_dict())
    sd.update(head.hf_state_dict())
    path = _write(tmp_path, hf_json, sd)
    b = LLM(path, load_format="safetensors", speculative_k=2, **KW)
    hb = b.runner.mtp
    assert torch.allclose(hb.norm_e.float(), head.norm_e.float(), atol=1e-6)
    assert torch.equal(hb.fc.w, head.fc.w) and torch.equal(hb.layer["qkv"].w, head.layer["qkv"].w)
    plain = LLM(path, load_format="safetensors", **KW)
    assert _tokens(b) == _tokens(plain)


def _quantize_sd(sd, fmt):
    """Quantise every ``*_proj`` weight of an HF state dict the way AutoAWQ /
    ModelOpt store it. NVFP4: q/k/v and gate/up are quantised jointly (one
    global scale per fused group, as ModelOpt exports them). Returns the
    quantised dict and, per projection prefix, the dense weight it encodes."""
    out, want = {}, {}
    groups = {}
    for k in sd:
        if k.endswith("_proj.weight"):
            pre = k[: -len(".weight")]
            base, proj = pre.rsplit(".", 1)
            key = {"q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv", "gate_proj": "gu",
                   "up_proj": "gu"}.get(proj, proj)
            groups.setdefault((base, key), []).append(pre)
        else:
            out[k] = sd[k]
    for (_, _), pres in groups.items():
        ws = [sd[p + ".weight"].float() for p in pres]
        if fmt == "awq":
            for p, w in zip(pres, ws):
                qw, qz, sc = quant.quantize_awq(w)
                out[p + ".qweight"], out[p + ".qzeros"], out[p + ".scales"] = qw, qz, sc
                want[p] = quant.AwqLinear(qw, qz, sc).reference_weight()
            continue
        packed, bs, g = quant.quantize_nvfp4(torch.cat(ws))
        r0 = 0
        for p, w in zip(pres, ws):
            n = w.shape[0]
            out[p + ".weight"] = packed[r0:r0 + n].contiguous()
            out[p + ".weight_scale"] = bs[r0:r0 + n].contiguous()
            out[p + ".weight_scale_2"] = torch.tensor(g, dtype=torch.float32)
            out[p + ".input_scale"] = torch.tensor(1.0, dtype=torch.float32)
            want[p] = quant.Nvfp4Linear(packed[r0:r0 + n], bs[r0:r0 + n], g).reference_weight()
            r0 += n
    return out, want


QCFG = {"awq": {"quant_method": "awq", "bits": 4, "group_size": 128, "version": "gemm"},
        "nvfp4": {"quant_method": "modelopt", "quant_algo": "NVFP4"}}


@pytest.mark.parametrize("fmt", ["awq", "nvfp4"])
def test_quantized_dense_checkpoint(tmp_path, fmt):
    a = LLM(TINY, **KW)
    sd, want = _quantize_sd(a.model.hf_state_dict(), fmt)
    b = LLM(_write(tmp_path, _hf_config(TINY, quantization_config=QCFG[fmt]), sd),
            load_format="safetensors", **KW)
    assert b.cfg.quant == fmt
    cls = {"awq": quant.AwqLinear, "nvfp4": quant.Nvfp4Linear}[fmt]
    for i, L in enumerate(b.model.layers):
        p = f"model.layers.{i}."
        assert isinstance(L["qkv"], cls) and isinstance(L["down"], cls)
        qkv = torch.cat([want[p + f"self_attn.{x}_proj"] for x in "qkv"])
        assert torch.equal(L["qkv"].reference_weight(), qkv)
        assert torch.equal(L["o"].reference_weight(), want[p + "self_attn.o_proj"])
        gu = torch.cat([want[p + "mlp.gate_proj"], want[p + "mlp.up_proj"]])
        assert torch.equal(L["gate_up"].lin.reference_weight(), gu)
        assert torch.equal(L["down"].reference_weight(), want[p + "mlp.down_proj"])
    assert all(len(t) == 5 for t in _tokens(b))


@pytest.mark.parametrize("fmt", ["awq", "nvfp4"])
def test_quantized_moe_checkpoint(tmp_path, fmt):
    cfg = ModelConfig(arch="qwen3_moe", hidden_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=4, head_dim=32, intermediate_size=256, vocab_size=512,
                      rope_theta=10000.0, rms_eps=1e-5, max_position=512, qk_norm=True,
                      num_experts=4, top_k=2, moe_intermediate_size=128)
    a = LLM(cfg, **KW)
    sd, want = _quantize_sd(a.model.hf_state_dict(), fmt)
    b = LLM(_write(tmp_path, _hf_config(cfg, quantization_config=QCFG[fmt]), sd),
            load_format="safetensors", **KW)
    ew = b.model.layers[1]["experts"]
    assert ew.fmt == fmt and ew.E == 4
    w13, w2 = ew.dense_ref()
    p = "model.layers.1.mlp.experts."
    for e in range(4):
        ref13 = torch.cat([want[f"{p}{e}.gate_proj"], want[f"{p}{e}.up_proj"]])
        if fmt == "nvfp4":  # per-expert globals are folded into the block scales
            rel = ((w13[e] - ref13).abs() / ref13.abs().clamp_min(1e-3)).max().item()
            assert rel < 0.07, rel
        else:
            assert torch.equal(w13[e], ref13)
            assert torch.equal(w2[e], want[f"{p}{e}.down_proj"])
    assert all(len(t) == 5 for t in _tokens(b))


def test_merge_nvfp4_parts_rescales_block_scales():
    g = torch.Generator().manual_seed(2)
    w1, w2 = torch.randn(16, 64, generator=g), 4 * torch.randn(16, 64, generator=g)
    p1, p2 = quant.quantize_nvfp4(w1), quant.quantize_nvfp4(w2)
    assert p1[2] != p2[2]
    w, s, gm = quant.merge_nvfp4_parts([p1[0], p2[0]], [p1[1], p2[1]], [p1[2], p2[2]])
    assert gm == max(p1[2], p2[2])
    merged = quant.Nvfp4Linear(w, s, gm).reference_weight()
    ref = torch.cat([quant.Nvfp4Linear(*p1).reference_weight(),
                     quant.Nvfp4Linear(*p2).reference_weight()])
    assert torch.equal(merged[16:], ref[16:])  # the part that owns the largest global
    rel = ((merged - ref).abs() / ref.abs().clamp_min(1e-3)).max().item()
    assert rel < 0.07, rel


TP_CFG = ModelConfig(arch="llama", hidden_size=256, num_layers=1, num_heads=4, num_kv_heads=2,
                     head_dim=64, intermediate_size=512, vocab_size=512, rope_theta=10000.0,
                     rms_eps=1e-5, max_position=512)


def _tp_shard_body(rank, world, path, out):
    from vllm_sm70_b200.parallel import state

    state.init(tp_size=world, backend="gloo", timeout_s=120)
    llm = LLM(path, tensor_parallel_size=world, load_format="safetensors", **KW)
    L = llm.model.layers[0]
    torch.save({"qkv": L["qkv"].reference_weight(), "o": L["o"].reference_weight(),
                "gate_up": L["gate_up"].lin.reference_weight(),
                "down": L["down"].reference_weight()}, f"{out}.{rank}")
    llm.shutdown()
    state.shutdown()


@pytest.mark.parametrize("fmt", ["awq", "nvfp4"])
def test_quantized_tp2_shards(tmp_path, fmt):
    """TP2 shards of a quantised checkpoint (rows of q/k/v and gate/up, input
    columns of o / down, cut on the scale-block boundaries) are the matching
    slices of the TP1 weights."""
    from . import _mp

    a = LLM(TP_CFG, **KW)
    sd, want = _quantize_sd(a.model.hf_state_dict(), fmt)
    path = _write(tmp_path, _hf_config(TP_CFG, quantization_config=QCFG[fmt]), sd)
    _mp.run(_tp_shard_body, 2, args=(path, str(tmp_path / "w")), timeout=300)
    p = "model.layers.0."
    hd, I = 64, 512
    for r in range(2):
        got = torch.load(tmp_path / f"w.{r}")
        q = want[p + "self_attn.q_proj"][r * 2 * hd:(r + 1) * 2 * hd]
        k = want[p + "self_attn.k_proj"][r * hd:(r + 1) * hd]
        v = want[p + "self_attn.v_proj"][r * hd:(r + 1) * hd]
        assert torch.equal(got["qkv"], torch.cat([q, k, v]))
        assert torch.equal(got["o"], want[p + "self_attn.o_proj"][:, r * 2 * hd:(r + 1) * 2 * hd])
        rows = slice(r * I // 2, (r + 1) * I // 2)
        assert torch.equal(got["gate_up"], torch.cat([want[p + "mlp.gate_proj"][rows],
                                                      want[p + "mlp.up_proj"][rows]]))
        assert torch.equal(got["down"], want[p + "mlp.down_proj"][:, rows])
