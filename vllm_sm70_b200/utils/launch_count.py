"""Counts launches of this library's own kernels (not torch's) so a benchmark
can report how many native kernels ran in its timed region. Eager launches
are counted by the op wrappers; CUDA-graph replays add the per-graph count
recorded at capture time."""
from __future__ import annotations

import threading

_lock = threading.Lock()
_total = 0


def add(n: int = 1) -> None:
    global _total
    with _lock:
        _total += n


def total() -> int:
    return _total


def reset() -> None:
    global _total
    with _lock:
        _total = 0
