"""Logger tree ``vllm.b200`` with log-once helpers.

Reference parity: the single ``vllm.sm70`` logger tree and the log-once-per-
reason pattern (``sm70/vllm_sm70/__init__.py:20``, ``_cuda_platform.py:329-338``,
``attention/__init__.py:98-102``).
"""
from __future__ import annotations

import logging
import threading

ROOT = "vllm.b200"
_seen: set = set()
_lock = threading.Lock()


def get_logger(name: str = "") -> logging.Logger:
    return logging.getLogger(ROOT + ("." + name if name else ""))


def log_once(logger: logging.Logger, level: int, key: str, msg: str, *args) -> bool:
    """Log ``msg`` the first time ``key`` is seen; returns True if logged."""
    with _lock:
        if key in _seen:
            return False
        _seen.add(key)
    logger.log(level, msg, *args)
    return True


def reset_once() -> None:
    with _lock:
        _seen.clear()
