"""CUDA-graph policy applied to a vLLM config before upstream sizing.

Capture sizes {1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256,
320, 384, 448, 512} capped by ``max_num_seqs`` and ``graph_max_batch``; with
speculative decoding the uniform-decode sizes are multiplied by (1 + k).
Only fills sizes the user did not set. Reference parity:
``sm70/vllm_sm70/graph_policy.py:64-240``.
"""
from __future__ import annotations

from ..engine.model_runner import default_capture_sizes


def capture_sizes(max_num_seqs: int, graph_max_batch: int = 512, spec_tokens: int = 0) -> list[int]:
    base = default_capture_sizes(max(1, min(max_num_seqs, graph_max_batch)))
    if spec_tokens > 0:
        q = 1 + spec_tokens
        base = sorted({s * q for s in base if s * q <= graph_max_batch * q})
    return base


def apply(vllm_config, cfg) -> None:
    if not cfg.cuda_graphs:
        return
    comp = getattr(vllm_config, "compilation_config", None)
    sched = getattr(vllm_config, "scheduler_config", None)
    if comp is None or sched is None:
        return
    if getattr(comp, "cudagraph_capture_sizes", None):
        return  # user-specified sizes win
    spec = getattr(vllm_config, "speculative_config", None)
    k = int(getattr(spec, "num_speculative_tokens", 0) or 0) if spec is not None else 0
    sizes = capture_sizes(int(getattr(sched, "max_num_seqs", 256)), cfg.graph_max_batch, k)
    try:
        comp.cudagraph_capture_sizes = sizes
    except Exception:  # noqa: BLE001 - frozen config variants: leave upstream sizing
        pass
