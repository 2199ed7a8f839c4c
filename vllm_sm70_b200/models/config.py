"""Model configuration shared by the model families, HF ``config.json``
parsing, and the presets of the benchmark configurations (random-init
weights of these exact shapes)."""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path


@dataclass(frozen=True)
class ModelConfig:
    arch: str = "llama"               # llama | qwen3_moe | qwen3_next | flint
    hidden_size: int = 4096
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    vocab_size: int = 128256
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    rms_eps: float = 1e-5
    max_position: int = 131072
    tie_embeddings: bool = False
    qk_norm: bool = False
    # MoE
    num_experts: int = 0
    top_k: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    norm_topk_prob: bool = True
    # hybrid (gated DeltaNet) + attention output gate
    layer_types: tuple = ()           # per layer: "attention" | "linear_attention"
    linear_num_k_heads: int = 0
    linear_num_v_heads: int = 0
    linear_k_head_dim: int = 0
    linear_v_head_dim: int = 0
    linear_conv_kernel: int = 4
    attn_output_gate: bool = False
    partial_rotary_factor: float = 1.0
    num_mtp_layers: int = 0
    # quantisation of the linear / expert weights
    quant: str | None = None          # None | fp8 | awq | nvfp4
    quant_group: int = 128
    extra: dict = field(default_factory=dict)

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def to_dict(self) -> dict:
        d = asdict(self)
        d["layer_types"] = list(self.layer_types)
        return d

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)

    def param_count(self) -> int:
        h, L = self.hidden_size, self.num_layers
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        if self.num_experts:
            mlp = self.num_experts * 3 * h * self.moe_intermediate_size + h * self.num_experts
            if self.shared_expert_intermediate_size:
                mlp += 3 * h * self.shared_expert_intermediate_size
        else:
            mlp = 3 * h * self.intermediate_size
        emb = self.vocab_size * h * (1 if self.tie_embeddings else 2)
        return L * (attn + mlp) + emb

    @classmethod
    def from_hf(cls, cfg: dict | str | Path) -> "ModelConfig":
        if not isinstance(cfg, dict):
            p = Path(cfg)
            if p.is_dir():
                p = p / "config.json"
            cfg = json.loads(p.read_text())
        mt = cfg.get("model_type", "llama")
        h = cfg["hidden_size"]
        nh = cfg["num_attention_heads"]
        hd = cfg.get("head_dim") or h // nh
        base = dict(
            hidden_size=h, num_layers=cfg["num_hidden_layers"], num_heads=nh,
            num_kv_heads=cfg.get("num_key_value_heads", nh), head_dim=hd,
            intermediate_size=cfg.get("intermediate_size", 4 * h),
            vocab_size=cfg["vocab_size"], rope_theta=float(cfg.get("rope_theta", 10000.0)),
            rope_scaling=cfg.get("rope_scaling"), rms_eps=float(cfg.get("rms_norm_eps", 1e-6)),
            max_position=int(cfg.get("max_position_embeddings", 8192)),
            tie_embeddings=bool(cfg.get("tie_word_embeddings", False)),
        )
        q = cfg.get("quantization_config") or {}
        qm = q.get("quant_method")
        if qm == "fp8":
            base["quant"] = "fp8"
            base["quant_group"] = int((q.get("weight_block_size") or [128, 128])[0])
        elif qm == "awq":
            base["quant"] = "awq"
            base["quant_group"] = int(q.get("group_size", 128))
        elif qm in ("modelopt", "modelopt_fp4") or q.get("quant_algo") == "NVFP4":
            base["quant"] = "nvfp4"
            base["quant_group"] = 16
        if mt in ("qwen3_moe",):
            base.update(arch="qwen3_moe", qk_norm=True, num_experts=cfg["num_experts"],
                        top_k=cfg["num_experts_per_tok"],
                        moe_intermediate_size=cfg["moe_intermediate_size"],
                        norm_topk_prob=bool(cfg.get("norm_topk_prob", True)))
        elif mt in ("qwen3_next",):
            n = base["num_layers"]
            interval = int(cfg.get("full_attention_interval", 4))
            lt = cfg.get("layer_types") or [
                "attention" if (i + 1) % interval == 0 else "linear_attention" for i in range(n)]
            base.update(arch="qwen3_next", qk_norm=True, num_experts=cfg["num_experts"],
                        top_k=cfg["num_experts_per_tok"],
                        moe_intermediate_size=cfg["moe_intermediate_size"],
                        shared_expert_intermediate_size=cfg.get("shared_expert_intermediate_size", 0),
                        norm_topk_prob=bool(cfg.get("norm_topk_prob", True)),
                        layer_types=tuple(lt),
                        linear_num_k_heads=cfg["linear_num_key_heads"],
                        linear_num_v_heads=cfg["linear_num_value_heads"],
                        linear_k_head_dim=cfg["linear_key_head_dim"],
                        linear_v_head_dim=cfg["linear_value_head_dim"],
                        linear_conv_kernel=cfg.get("linear_conv_kernel_dim", 4),
                        attn_output_gate=True,
                        partial_rotary_factor=float(cfg.get("partial_rotary_factor", 0.25)),
                        num_mtp_layers=int(cfg.get("num_nextn_predict_layers", 1)))
        elif mt == "flint" or any("Flint" in a for a in cfg.get("architectures") or []):
            if cfg.get("attention_bias"):
                raise NotImplementedError("Flint with attention biases")
            if cfg.get("router_score_function", "sigmoid") != "sigmoid":
                raise ValueError("Flint routes with sigmoid scores")
            n = base["num_layers"]
            rp = cfg.get("rope_parameters") or {}
            by_type = {}
            if rp and all(isinstance(v, dict) for v in rp.values()):  # per layer type
                by_type = {k: float(v.get("rope_theta", base["rope_theta"])) for k, v in rp.items()}
            elif "rope_theta" in rp:
                base["rope_theta"] = float(rp["rope_theta"])
            base.update(arch="flint", qk_norm=True, num_experts=cfg["num_experts"],
                        top_k=cfg["num_experts_per_tok"],
                        moe_intermediate_size=cfg["moe_intermediate_size"],
                        shared_expert_intermediate_size=cfg.get("shared_expert_intermediate_size", 0),
                        norm_topk_prob=bool(cfg.get("norm_topk_prob", True)),
                        layer_types=tuple(cfg.get("layer_types") or ["full_attention"] * n),
                        extra={"sliding_window": int(cfg.get("sliding_window") or 0),
                               "no_rope_layers": list(cfg.get("no_rope_layer_indices") or []),
                               "mlp_only_layers": list(cfg.get("mlp_only_layers") or []),
                               "rope_theta_by_type": by_type})
        elif mt in ("qwen3", "qwen2"):
            base.update(arch="llama", qk_norm=(mt == "qwen3"))
        return cls(**base)


LLAMA31_ROPE_SCALING = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                        "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}


def llama31_8b() -> ModelConfig:
    """Llama-3.1-8B shapes (the headline benchmark model)."""
    return ModelConfig(arch="llama", hidden_size=4096, num_layers=32, num_heads=32,
                       num_kv_heads=8, head_dim=128, intermediate_size=14336, vocab_size=128256,
                       rope_theta=500000.0, rope_scaling=dict(LLAMA31_ROPE_SCALING), rms_eps=1e-5)


def llama31_70b_awq() -> ModelConfig:
    """Llama-3.1-70B shapes, AWQ int4 g128."""
    return ModelConfig(arch="llama", hidden_size=8192, num_layers=80, num_heads=64,
                       num_kv_heads=8, head_dim=128, intermediate_size=28672, vocab_size=128256,
                       rope_theta=500000.0, rope_scaling=dict(LLAMA31_ROPE_SCALING), rms_eps=1e-5,
                       quant="awq", quant_group=128)


def qwen3_30b_a3b_fp8() -> ModelConfig:
    """Qwen3-30B-A3B shapes, block-FP8 128x128."""
    return ModelConfig(arch="qwen3_moe", hidden_size=2048, num_layers=48, num_heads=32,
                       num_kv_heads=4, head_dim=128, intermediate_size=6144, vocab_size=151936,
                       rope_theta=1000000.0, rms_eps=1e-6, qk_norm=True, num_experts=128, top_k=8,
                       moe_intermediate_size=768, quant="fp8", quant_group=128)


def qwen3_next_80b_nvfp4() -> ModelConfig:
    """Qwen3-Next-80B-A3B shapes, NVFP4."""
    n = 48
    lt = tuple("attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(n))
    return ModelConfig(arch="qwen3_next", hidden_size=2048, num_layers=n, num_heads=16,
                       num_kv_heads=2, head_dim=256, intermediate_size=5120, vocab_size=151936,
                       rope_theta=10000000.0, rms_eps=1e-6, qk_norm=True, num_experts=512,
                       top_k=10, moe_intermediate_size=512, shared_expert_intermediate_size=512,
                       layer_types=lt, linear_num_k_heads=16, linear_num_v_heads=32,
                       linear_k_head_dim=128, linear_v_head_dim=128, attn_output_gate=True,
                       partial_rotary_factor=0.25, num_mtp_layers=1, quant="nvfp4",
                       quant_group=16)


PRESETS = {
    "llama-3.1-8b": llama31_8b,
    "llama-3.1-70b-awq": llama31_70b_awq,
    "qwen3-30b-a3b-fp8": qwen3_30b_a3b_fp8,
    "qwen3-next-80b-a3b-nvfp4": qwen3_next_80b_nvfp4,
}


def resolve(model) -> ModelConfig:
    if isinstance(model, ModelConfig):
        return model
    if isinstance(model, dict):
        return ModelConfig.from_hf(model)
    if isinstance(model, str) and model in PRESETS:
        return PRESETS[model]()
    return ModelConfig.from_hf(model)
