"""vLLM IR-op providers backed by this library's kernels (ops area).

vLLM 0.22 dispatches RMSNorm through IR ops (``vllm.ir.ops.rms_norm`` and
``fused_add_rms_norm``) with a per-op provider priority list. This module
registers the provider ``"b200"`` for both, backed by
``_b200_C::rms_norm`` / ``_b200_C::fused_add_rms_norm`` (bf16 / fp16,
contiguous rows, no variance-size override), and
``B200CudaPlatform.get_default_ir_op_priority`` puts it first, so every
RMSNorm of a vLLM model runs the B200 kernel when the platform is active.
Other argument combinations fall through to the next provider.

Reference parity: the reference pins its IR-op priority in
``sm70/vllm_sm70/_cuda_platform.py`` (``get_default_ir_op_priority``).
"""
from __future__ import annotations

import torch
from torch import Tensor

PROVIDER = "b200"
_registered = False


def _rows_ok(x: Tensor) -> bool:
    return x.dim() >= 1 and x.is_contiguous() and x.shape[-1] % 8 == 0


def rms_supported(x, weight, epsilon, variance_size=None) -> bool:
    return (variance_size is None and weight is not None and x.is_cuda
            and x.dtype in (torch.bfloat16, torch.float16) and weight.dtype == x.dtype
            and _rows_ok(x) and weight.is_contiguous())


def add_rms_supported(x, x_residual, weight, epsilon, variance_size=None) -> bool:
    return (rms_supported(x, weight, epsilon, variance_size)
            and x_residual.dtype == x.dtype and x_residual.shape == x.shape
            and x_residual.is_contiguous())


def rms_norm(x: Tensor, weight: Tensor | None, epsilon: float,
             variance_size: int | None = None) -> Tensor:
    x2 = x.view(-1, x.shape[-1])
    out = torch.empty_like(x2)
    torch.ops._b200_C.rms_norm(out, x2, weight, float(epsilon))
    return out.view_as(x)


def fused_add_rms_norm(x: Tensor, x_residual: Tensor, weight: Tensor | None, epsilon: float,
                       variance_size: int | None = None) -> tuple[Tensor, Tensor]:
    torch.ops._b200_C.fused_add_rms_norm(x.view(-1, x.shape[-1]),
                                         x_residual.view(-1, x.shape[-1]), weight,
                                         float(epsilon))
    return x, x_residual


def register() -> bool:
    """Register the providers with vLLM's IR ops (idempotent). Returns False
    when vLLM's IR layer is not importable."""
    global _registered
    if _registered:
        return True
    try:
        from vllm import ir
    except Exception:  # noqa: BLE001 - vLLM without the IR layer
        return False
    from .. import _ext

    ok = _ext.loaded() and torch.cuda.is_available()
    if PROVIDER not in ir.ops.rms_norm.impls:
        ir.ops.rms_norm.register_impl(PROVIDER, supports_args=rms_supported,
                                      supported=ok)(rms_norm)
    if PROVIDER not in ir.ops.fused_add_rms_norm.impls:
        ir.ops.fused_add_rms_norm.register_impl(PROVIDER, supports_args=add_rms_supported,
                                                supported=ok, inplace=True)(fused_add_rms_norm)
    _registered = True
    return True


def with_b200_first(priority):
    """``IrOpPriorityConfig`` with ``"b200"`` put first for the two RMSNorm
    ops (other ops unchanged)."""
    import dataclasses

    changes = {}
    for name in ("rms_norm", "fused_add_rms_norm"):
        cur = list(getattr(priority, name, []) or [])
        if PROVIDER not in cur:
            changes[name] = [PROVIDER] + cur
    return dataclasses.replace(priority, **changes) if changes else priority
