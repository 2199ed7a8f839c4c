"""MoE router provider (platform hook U3).

``provider(runner)`` returns a route object for a vLLM ``MoERunner`` whose
gate this library can serve, or ``None`` to keep upstream routing. A route's
``try_route(hidden) -> (topk_weights fp32, topk_ids int32) | None`` defers
(None) under conditions it does not admit. Decisions are cached per layer
(including "no") and are rank-uniform.

Reference parity: ``sm70/vllm_sm70/router.py:123-339`` (K13 provider) and
``patches/0004-*:81-92`` (hook contract).
"""
from __future__ import annotations

import logging

logger = logging.getLogger("vllm.b200.router")
_decisions: dict = {}


def provider(runner):
    key = id(runner)
    if key in _decisions:
        return _decisions[key]
    route = None
    try:
        from ..ops import moe as moe_ops

        route = moe_ops.make_route_for_runner(runner)
    except Exception as e:  # noqa: BLE001 - not admitted: keep upstream routing
        logger.debug("fused router not admitted: %s", e)
        route = None
    _decisions[key] = route
    return route


def prepare_worker(worker) -> None:
    """Decide and allocate each MoE layer's route before graph capture."""
    model = getattr(worker, "get_model", lambda: None)()
    if model is None:
        return
    for mod in getattr(model, "modules", lambda: [])():
        runner = getattr(mod, "runner", None)
        if runner is not None:
            provider(runner)


def reset() -> None:
    _decisions.clear()
