"""Composite Inductor post-grad pass.

vLLM exposes a single ``post_grad_custom_post_pass`` slot; this pass occupies
it and runs the registered patterns in order. Its uuid covers this source,
the pattern list and the native-library fingerprint, so vLLM's compile cache
invalidates when any of them changes. Reference parity:
``sm70/vllm_sm70/passes.py:37-115``.
"""
from __future__ import annotations

import hashlib
import inspect
import logging

logger = logging.getLogger("vllm.b200.passes")

_PATTERNS: list = []


def register_pattern(fn) -> None:
    """``fn(graph) -> int`` rewrites an FX graph in place, returns #rewrites."""
    if fn not in _PATTERNS:
        _PATTERNS.append(fn)


class CompositePass:
    def __init__(self, patterns=None):
        self.patterns = list(patterns if patterns is not None else _PATTERNS)

    def __call__(self, graph) -> None:
        for p in self.patterns:
            try:
                n = p(graph)
                if n:
                    logger.info("b200 pass %s rewrote %d sites", getattr(p, "__name__", p), n)
            except Exception as e:  # noqa: BLE001 - a failed rewrite keeps the graph unchanged
                logger.warning("b200 pass %s skipped: %s", getattr(p, "__name__", p), e)

    def uuid(self) -> str:
        from .. import _ext

        h = hashlib.sha256()
        h.update(inspect.getsource(CompositePass).encode())
        for p in self.patterns:
            try:
                h.update(inspect.getsource(p).encode())
            except (OSError, TypeError):
                h.update(repr(p).encode())
        h.update(_ext.fingerprint().encode())
        return h.hexdigest()


def install_composite_pass(vllm_config) -> bool:
    comp = getattr(vllm_config, "compilation_config", None)
    if comp is None:
        return False
    pc = getattr(comp, "pass_config", None)
    holder = comp
    slot = "post_grad_custom_post_pass"
    inductor = getattr(comp, "inductor_compile_config", None)
    if isinstance(inductor, dict):
        if inductor.get(slot) is not None and not isinstance(inductor.get(slot), CompositePass):
            logger.warning("post-grad pass slot taken; B200 patterns not installed")
            return False
        inductor[slot] = CompositePass()
        return True
    _ = (pc, holder)
    return False


def register() -> None:
    """Plugin area hook: register the built-in patterns."""
    from . import ar_norm_fusion

    register_pattern(ar_norm_fusion.fuse_all_reduce_add_rms_norm)
