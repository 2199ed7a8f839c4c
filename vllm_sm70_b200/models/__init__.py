"""Model families: Llama-style dense decoders, Qwen3-MoE, Qwen3-Next hybrid,
Flint (sliding / full attention with sinks, sigmoid MoE)."""
from __future__ import annotations

import torch

from .config import ModelConfig, resolve  # noqa: F401


def build_model(cfg: ModelConfig, device: torch.device, dtype=torch.bfloat16, ps=None):
    if cfg.arch == "llama":
        from .llama import LlamaModel

        return LlamaModel(cfg, device, dtype, ps)
    if cfg.arch == "qwen3_moe":
        from .qwen3_moe import Qwen3MoeModel

        return Qwen3MoeModel(cfg, device, dtype, ps)
    if cfg.arch == "qwen3_next":
        from .qwen3_next import Qwen3NextModel

        return Qwen3NextModel(cfg, device, dtype, ps)
    if cfg.arch == "flint":
        from .flint import FlintModel

        return FlintModel(cfg, device, dtype, ps)
    raise ValueError(f"unknown architecture {cfg.arch}")
