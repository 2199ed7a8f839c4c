"""NVTX ranges per model layer and engine phase (``VLLM_B200_NVTX=1``) so a
profiler's timeline groups kernels by layer / op; off by default, when the
calls cost one flag test.

    with tracing.nvtx("decode"):
        ...
    tracing.push("L3.attn"); ...; tracing.pop()

Reference parity: the profiling plan of the reference build notes (NVTX per
layer and op, CUDA-event device time); the reference itself ships none.
"""
from __future__ import annotations

import contextlib

from .. import envs

_state = {"on": None}


def enabled() -> bool:
    on = _state["on"]
    if on is None:
        on = bool(envs.get("VLLM_B200_NVTX"))
        try:
            import torch

            on = on and torch.cuda.is_available()
        except Exception:  # noqa: BLE001
            on = False
        _state["on"] = on
    return on


def set_enabled(on: bool | None) -> None:
    """Force on / off (None: re-read the environment on next use)."""
    _state["on"] = on


def push(name: str) -> None:
    if enabled():
        import torch

        torch.cuda.nvtx.range_push(name)


def pop() -> None:
    if enabled():
        import torch

        torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def nvtx(name: str):
    push(name)
    try:
        yield
    finally:
        pop()
