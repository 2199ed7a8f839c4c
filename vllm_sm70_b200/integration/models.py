"""Model area: registers this library's model classes with vLLM's registry
when vLLM is importable (selected with ``--hf-overrides architectures``).
Reference parity: ``sm70/vllm_sm70/models/flint_sm70/__init__.py:63-82``."""
from __future__ import annotations

ARCHS = {
    "B200LlamaForCausalLM": "vllm_sm70_b200.models.llama:LlamaModel",
    "B200Qwen3MoeForCausalLM": "vllm_sm70_b200.models.qwen3_moe:Qwen3MoeModel",
    "B200Qwen3NextForCausalLM": "vllm_sm70_b200.models.qwen3_next:Qwen3NextModel",
    "B200FlintForCausalLM": "vllm_sm70_b200.models.flint:FlintModel",
}


def register() -> None:
    from . import hooks

    hooks.install()
    # The <think> / <tool_call> reasoning parser registers itself on import
    # ("glm47_b200").
    from . import reasoning  # noqa: F401
