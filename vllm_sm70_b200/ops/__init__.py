"""Op wrappers over ``torch.ops._b200_C`` with CPU reference implementations.

Reference parity: ``sm70/vllm_sm70/ops/__init__.py:28-46`` (area that imports
the wrapper modules and registers fakes).
"""
from __future__ import annotations

from . import attention, linear, norm, sampling  # noqa: F401
from .attention import paged_attention, rope_kv_write  # noqa: F401
from .linear import gemm, gemm_silu_mul, interleave_gate_up, silu_mul  # noqa: F401
from .norm import fused_add_rms_norm, rms_norm  # noqa: F401
from .sampling import argmax  # noqa: F401


def register() -> None:
    """Plugin area hook: load the library and register fake kernels."""
    from .. import _ext
    from . import _fakes

    if _ext.load():
        _fakes.register_all()
    # RMSNorm of vLLM models: the "b200" IR-op provider (first in the
    # platform's priority list).
    from ..integration import ir_ops

    ir_ops.register()
