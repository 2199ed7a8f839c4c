"""Gated-DeltaNet area (Qwen3-Next linear attention): kernels in
``ops/gdn.py``; models use them directly."""


def register() -> None:
    return None
