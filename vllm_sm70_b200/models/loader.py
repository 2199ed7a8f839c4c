"""Checkpoint loading: HF-layout safetensors directories.

``load_checkpoint(model, path)`` opens every ``*.safetensors`` file under
``path`` (sharded checkpoints with ``model.safetensors.index.json`` or a
single ``model.safetensors``), indexes tensor names lazily and hands the
model a ``get_tensor(name)`` callable returning the full, unsharded CPU
tensor; the model cuts its tensor-parallel shard and builds its layers
(``load_hf_state``). Only the tensors a rank asks for are read.

Reference parity: weight loading goes through upstream vLLM's model loader
in the reference (its plugin only repacks quantised weights after loading,
``sm70/vllm_sm70/quant/*.py`` ``process_weights_after_loading``); this
runtime owns its models, so it owns the loader too.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch


class SafetensorsIndex:
    """name -> file map over a checkpoint directory with lazy tensor reads."""

    def __init__(self, path: str | Path):
        from safetensors import safe_open

        self._safe_open = safe_open
        root = Path(path)
        if root.is_file():
            files = [root]
            root = root.parent
        else:
            idx = root / "model.safetensors.index.json"
            if idx.exists():
                wm = json.loads(idx.read_text())["weight_map"]
                files = sorted({root / f for f in wm.values()})
            else:
                files = sorted(root.glob("*.safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files under {path}")
        self._where: dict[str, Path] = {}
        for f in files:
            with safe_open(str(f), framework="pt", device="cpu") as h:
                for k in h.keys():
                    self._where[k] = f
        self._open: dict[Path, object] = {}

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def names(self) -> list[str]:
        return sorted(self._where)

    def get(self, name: str) -> torch.Tensor:
        f = self._where.get(name)
        if f is None:
            raise KeyError(f"checkpoint has no tensor {name!r}")
        h = self._open.get(f)
        if h is None:
            h = self._safe_open(str(f), framework="pt", device="cpu")
            self._open[f] = h
        return h.get_tensor(name)


def load_checkpoint(model, path: str | Path) -> None:
    if not hasattr(model, "load_hf_state"):
        raise NotImplementedError(
            f"checkpoint loading is not implemented for {type(model).__name__}; "
            "use load_format='dummy'")
    index = SafetensorsIndex(path)
    model.load_hf_state(index.get, has=index.__contains__)
