"""Runtime installation of the platform hook call sites into the installed
vLLM (the reference adds them with its patch series: ``patches/0002-0005``).

* U1: ``dispatch_unquantized_gemm()`` consults
  ``current_platform.get_unquantized_gemm(linear_backend)`` first;
* U1: ``kernel_warmup(worker)`` calls ``current_platform.kernel_warmup``
  after upstream's warm-up.

Without a hook (or when the platform returns None) upstream behaviour is
unchanged. ``install()`` is idempotent.
"""
from __future__ import annotations

import logging

import torch

logger = logging.getLogger("vllm.b200.hooks")
_installed: dict = {}


def b200_unquantized_gemm(layer, x: torch.Tensor, weight: torch.Tensor,
                          bias: torch.Tensor | None = None) -> torch.Tensor:
    """U1 GEMM: bf16 2-D activations on the tcgen05 kernel, else torch."""
    from ..ops import linear

    if (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and weight.dim() == 2 and x.shape[-1] % 8 == 0 and weight.shape[0] % 8 == 0):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        y = linear.gemm(x2, weight)
        if bias is not None:
            y = y + bias
        return y.view(*x.shape[:-1], weight.shape[0])
    return torch.nn.functional.linear(x, weight, bias)


def install() -> dict:
    try:
        import vllm.model_executor.layers.utils as lu
        from vllm.platforms import current_platform
    except Exception as e:  # noqa: BLE001 - vLLM not importable
        return {"error": str(e)}
    if "u1_gemm" not in _installed and hasattr(lu, "dispatch_unquantized_gemm"):
        orig = lu.dispatch_unquantized_gemm

        def dispatch_unquantized_gemm(*a, **kw):
            hook = getattr(current_platform, "get_unquantized_gemm", None)
            fn = hook(kw.get("linear_backend")) if hook is not None else None
            return fn if fn is not None else orig(*a, **kw)

        lu.dispatch_unquantized_gemm = dispatch_unquantized_gemm
        _installed["u1_gemm"] = orig
    try:
        import vllm.model_executor.warmup.kernel_warmup as kw_mod
    except Exception:  # noqa: BLE001
        kw_mod = None
    if kw_mod is not None and "u1_warmup" not in _installed:
        orig_w = kw_mod.kernel_warmup

        def kernel_warmup(worker):
            orig_w(worker)
            hook = getattr(current_platform, "kernel_warmup", None)
            if hook is not None:
                hook(worker)

        kw_mod.kernel_warmup = kernel_warmup
        _installed["u1_warmup"] = orig_w
    return dict(_installed)
