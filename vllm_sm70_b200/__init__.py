"""vllm_sm70_b200: a Blackwell-native (B200, sm_100a) LLM-inference kernel
library, runtime and vLLM platform plugin.

Entry points (``pyproject.toml``):

* ``vllm.general_plugins: b200 = vllm_sm70_b200:register``
* ``vllm.platform_plugins: b200 = vllm_sm70_b200.platform:activate``

Reference parity: ``sm70/vllm_sm70/__init__.py:23-91`` -- idempotent
``register()`` that merges the env registry, loads the native library and
registers each plugin area in order, recording per-area failures so the
platform can fail fast (``failed_areas`` / ``retry_failed_areas``).
"""
from __future__ import annotations

import importlib
import logging
import threading

__version__ = "0.1.0"

logger = logging.getLogger("vllm.b200")

# Registration order matters: ops before the layers that use them.
AREAS = ("ops", "attention", "gdn", "fused_moe", "quant", "models", "passes")
_AREA_MODULES = {
    "ops": "vllm_sm70_b200.ops",
    "attention": "vllm_sm70_b200.integration.attention",
    "gdn": "vllm_sm70_b200.integration.gdn",
    "fused_moe": "vllm_sm70_b200.integration.fused_moe",
    "quant": "vllm_sm70_b200.integration.quant",
    "models": "vllm_sm70_b200.integration.models",
    "passes": "vllm_sm70_b200.integration.passes",
}

_lock = threading.Lock()
_registered = False
_area_status: dict[str, str | None] = {}


def _register_area(area: str) -> None:
    try:
        mod = importlib.import_module(_AREA_MODULES[area])
        hook = getattr(mod, "register", None)
        if hook is not None:
            hook()
        _area_status[area] = None
    except Exception as e:  # noqa: BLE001 - recorded; strict mode raises later
        _area_status[area] = f"{type(e).__name__}: {e}"
        logger.warning("vllm_sm70_b200: area %s failed to register: %s", area, e)


def register() -> None:
    """vLLM general-plugin hook (idempotent)."""
    global _registered
    with _lock:
        if _registered:
            return
        from . import _ext, envs

        envs.merge_into_vllm()
        _ext.load()
        for area in AREAS:
            _register_area(area)
        _registered = True


def failed_areas() -> dict[str, str]:
    return {a: e for a, e in _area_status.items() if e}


def retry_failed_areas() -> dict[str, str]:
    for area in list(failed_areas()):
        _register_area(area)
    return failed_areas()


def area_status() -> dict[str, str | None]:
    return dict(_area_status)


def _reset_for_tests() -> None:
    global _registered
    with _lock:
        _registered = False
        _area_status.clear()
