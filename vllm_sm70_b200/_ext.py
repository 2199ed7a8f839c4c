"""Loader for the native kernel library ``_b200_C.so``.

Reference parity: ``sm70/vllm_sm70/_ext.py:15-61`` (import once, record the
failure, fingerprint = ABI version + sha256 of the ``.so`` for compile-cache
keys).

Policy: on a machine with a CUDA device the extension is REQUIRED -- every op
wrapper calls :func:`require` and raises if the ``.so`` did not load, so a GPU
test can never pass on a silent eager fallback. Without a GPU the wrappers use
their PyTorch reference implementations (the CPU oracles the tests compare
against).
"""
from __future__ import annotations

import hashlib
import os
import threading
from pathlib import Path

import torch

SO_PATH = Path(__file__).resolve().parent / "_b200_C.so"
_lock = threading.Lock()
_state: dict = {"loaded": False, "error": None, "fingerprint": None}


def load(build_if_missing: bool = False) -> bool:
    """Load the extension once. Returns True when the ops are registered."""
    with _lock:
        if _state["loaded"]:
            return True
        if os.environ.get("VLLM_B200_SKIP_EXT") == "1":
            _state["error"] = "disabled by VLLM_B200_SKIP_EXT=1"
            return False
        if not SO_PATH.exists() and build_if_missing:
            from . import build_ext

            build_ext.build()
        if not SO_PATH.exists():
            _state["error"] = f"{SO_PATH.name} not built (python -m vllm_sm70_b200.build_ext)"
            return False
        try:
            torch.ops.load_library(str(SO_PATH))
        except Exception as e:  # noqa: BLE001 - recorded and re-raised by require()
            _state["error"] = f"{type(e).__name__}: {e}"
            return False
        _state["loaded"] = True
        _state["error"] = None
        return True


def loaded() -> bool:
    return bool(_state["loaded"])


def error() -> str | None:
    return _state["error"]


def gpu_present() -> bool:
    return torch.cuda.is_available()


def require() -> None:
    """Raise unless the native library is loaded (used on every CUDA path)."""
    if not _state["loaded"] and not load():
        raise RuntimeError(f"vllm_sm70_b200 native library unavailable: {_state['error']}")


def has_op(name: str) -> bool:
    if not load():
        return False
    try:
        getattr(torch.ops._b200_C, name)
        return True
    except (AttributeError, RuntimeError):
        return False


def abi_version() -> int:
    require()
    return int(torch.ops._b200_C.abi_version())


def fingerprint() -> str:
    """``abi=<n>;so=<sha256>``; folded into compile / tuning cache keys."""
    if _state["fingerprint"] is None:
        if not load():
            _state["fingerprint"] = "abi=none;so=none"
        else:
            h = hashlib.sha256(SO_PATH.read_bytes()).hexdigest()[:16]
            _state["fingerprint"] = f"abi={abi_version()};so={h}"
    return _state["fingerprint"]


def ops():
    require()
    return torch.ops._b200_C
