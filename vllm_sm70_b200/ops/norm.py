"""RMSNorm / fused residual-add + RMSNorm wrappers.

The CPU reference mirrors the kernel's rounding: the residual sum is rounded
to the activation dtype first, the variance is taken from that rounded sum,
and the normalised value is rounded before the weight multiply.
"""
from __future__ import annotations

import torch

from .. import _ext
from ..utils import launch_count


def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return ((xf * inv).to(x.dtype).float() * w.float()).to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float,
             out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        _ext.require()
        torch.ops._b200_C.rms_norm(out, x, w, eps)
        launch_count.add(1)
    else:
        out.copy_(rms_norm_ref(x, w, eps))
    return out


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                       eps: float) -> None:
    """In place: ``residual <- x + residual``; ``x <- rmsnorm(residual) * w``."""
    if x.is_cuda:
        _ext.require()
        torch.ops._b200_C.fused_add_rms_norm(x, residual, w, eps)
        launch_count.add(1)
        return
    s = (x.float() + residual.float()).to(x.dtype)
    residual.copy_(s)
    x.copy_(rms_norm_ref(s, w, eps))
