"""vLLM platform-plugin entry point (``vllm.platform_plugins``).

``activate()`` returns the qualified name of :class:`B200CudaPlatform` iff
every GPU visible to this process is a compute-capability 10.0 part (B200 /
GB200), and ``None`` otherwise so vLLM falls back to its own platform
resolution. It uses NVML only -- never CUDA -- so vLLM can still fork
workers afterwards. ``CUDA_VISIBLE_DEVICES`` entries may be indices or
``GPU-<uuid>`` strings.

Reference parity: ``sm70/vllm_sm70/platform.py:67-104`` (same contract for
cc 7.0).
"""
from __future__ import annotations

import logging
import os

logger = logging.getLogger("vllm.b200.platform")

PLATFORM_QUALNAME = "vllm_sm70_b200.integration.platform_impl.B200CudaPlatform"
TARGET_CC = (10, 0)


def _nvml():
    import pynvml  # nvidia-ml-py

    return pynvml


def _visible_handles(nv) -> list:
    count = nv.nvmlDeviceGetCount()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis is None:
        return [nv.nvmlDeviceGetHandleByIndex(i) for i in range(count)]
    vis = vis.strip()
    if vis == "":
        return []
    handles = []
    for tok in vis.split(","):
        tok = tok.strip()
        if not tok:
            continue
        if tok.startswith("GPU-") or tok.startswith("MIG-"):
            handles.append(nv.nvmlDeviceGetHandleByUUID(tok))
        else:
            idx = int(tok)
            if idx < 0:
                break  # CUDA stops enumerating at the first invalid index
            if idx >= count:
                break
            handles.append(nv.nvmlDeviceGetHandleByIndex(idx))
    return handles


def all_visible_gpus_are_b200(nv=None) -> bool:
    try:
        nv = nv or _nvml()
        nv.nvmlInit()
    except Exception as e:  # noqa: BLE001 - no NVML: not our platform
        logger.debug("NVML unavailable: %s", e)
        return False
    try:
        handles = _visible_handles(nv)
        if not handles:
            return False
        for h in handles:
            major, minor = nv.nvmlDeviceGetCudaComputeCapability(h)
            if (int(major), int(minor)) != TARGET_CC:
                return False
        return True
    except Exception as e:  # noqa: BLE001
        logger.debug("NVML query failed: %s", e)
        return False
    finally:
        try:
            nv.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass


def activate() -> str | None:
    """vLLM platform-plugin hook."""
    if os.environ.get("VLLM_B200_PLATFORM") == "0":
        return None
    if all_visible_gpus_are_b200():
        return PLATFORM_QUALNAME
    return None


def is_b200_ready() -> bool:
    """True when the platform would activate AND the native library loads."""
    from . import _ext

    return all_visible_gpus_are_b200() and _ext.load()
