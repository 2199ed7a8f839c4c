"""Model area: registers this library's vLLM model classes with vLLM's
``ModelRegistry`` (selected with ``--hf-overrides '{"architectures":
["B200LlamaForCausalLM"]}'`` and the like), installs the platform hook call
sites and the reasoning parser.

Registration uses vLLM's lazy ``"<module>:<class>"`` form, so plugin load
imports no model code, and is checked afterwards: when the registry does not
resolve an architecture to the registered target the area fails (and strict
mode turns that into a start-up error).

The engine-native model classes (``ENGINE_ARCHS``) serve this library's own
runtime (``vllm_sm70_b200.engine.LLM``); Flint has no vLLM model in the
installed vLLM, so it is served by that runtime only.

Reference parity: ``sm70/vllm_sm70/models/flint_sm70/__init__.py:63-82``.
"""
from __future__ import annotations

# vLLM architecture name -> lazy target of the vLLM model class.
VLLM_ARCHS = {
    "B200LlamaForCausalLM": "vllm_sm70_b200.integration.vllm_models:B200LlamaForCausalLM",
    "B200Qwen3MoeForCausalLM": "vllm_sm70_b200.integration.vllm_models:B200Qwen3MoeForCausalLM",
    "B200Qwen3NextForCausalLM":
        "vllm_sm70_b200.integration.vllm_models:B200Qwen3NextForCausalLM",
}
# Engine-native model classes (this library's runtime).
ENGINE_ARCHS = {
    "llama": "vllm_sm70_b200.models.llama:LlamaModel",
    "qwen3_moe": "vllm_sm70_b200.models.qwen3_moe:Qwen3MoeModel",
    "qwen3_next": "vllm_sm70_b200.models.qwen3_next:Qwen3NextModel",
    "flint": "vllm_sm70_b200.models.flint:FlintModel",
}
ARCHS = VLLM_ARCHS  # kept name

REGISTERED: dict[str, str] = {}


def register_models() -> dict[str, str]:
    """Register ``VLLM_ARCHS`` with vLLM (idempotent); raise when the registry
    does not resolve a name to its target afterwards."""
    from vllm.model_executor.models import ModelRegistry

    for arch, target in VLLM_ARCHS.items():
        if arch in REGISTERED:
            continue
        ModelRegistry.register_model(arch, target)
        entry = ModelRegistry.models.get(arch)
        module_name, _, class_name = target.partition(":")
        got = (getattr(entry, "module_name", None), getattr(entry, "class_name", None))
        if got != (module_name, class_name):
            raise RuntimeError(f"vllm_sm70_b200: {arch!r} resolves to {entry!r}, not {target}")
        REGISTERED[arch] = target
    return dict(REGISTERED)


def register() -> None:
    from . import hooks

    hooks.install()
    # The <think> / <tool_call> reasoning parser registers itself on import
    # ("glm47_b200").
    from . import reasoning  # noqa: F401

    try:
        import vllm.model_executor.models  # noqa: F401
    except Exception:  # noqa: BLE001 - no vLLM: nothing to register
        return
    register_models()
