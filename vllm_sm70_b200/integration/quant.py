"""Quantisation area: maps vLLM quantisation method names to this library's
weight-only linear / MoE implementations (FP8 128x128 block -> W8A16,
AWQ int4 g128 -> W4A16, ModelOpt NVFP4 -> W4A16). Reference parity:
``sm70/vllm_sm70/quant/configs.py:67-240``."""
from __future__ import annotations

SUPPORTED = {"fp8": "fp8", "awq": "awq", "modelopt_fp4": "nvfp4", "modelopt": "nvfp4"}


def method_for(quant_method: str | None) -> str | None:
    return SUPPORTED.get(quant_method) if quant_method else None


def register() -> None:
    return None
