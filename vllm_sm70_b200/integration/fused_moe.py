"""Fused-MoE area: bf16 routed experts of vLLM MoE layers run the grouped
tcgen05 expert GEMMs of ``ops/moe.py``.

When the B200 platform is active, vLLM's ``UnquantizedFusedMoEMethod`` is
replaced out of tree (``CustomOp.register_oot``) by
:class:`~vllm_sm70_b200.integration.vllm_models` ``B200MoEMethod``: the
expert-sorted permutation, the grouped gate/up GEMM, SiLU * up, the grouped
down GEMM and the weighted combine, all graph-capturable, with the route from
the U3 router hook (``models/router.py``) when it answers. Layers it cannot
serve (expert bias, non-SiLU activations, sizes off the 128-row tiles) keep
vLLM's kernels. Kill switch: ``VLLM_B200_MOE=0``.

Reference parity: the reference's fused-MoE area
(``sm70/vllm_sm70/fused_moe/method.py:56-416``), which routes vLLM's MoE
layers to its TurboMind MoE GEMMs.
"""
from __future__ import annotations

import logging

logger = logging.getLogger("vllm.b200.fused_moe")
INSTALLED: dict[str, type] = {}


def register() -> dict[str, type]:
    from .. import envs
    from .vllm_models import _b200_active, methods

    if INSTALLED or not envs.get("VLLM_B200_MOE"):
        return dict(INSTALLED)
    try:
        from vllm.model_executor.custom_op import CustomOp, op_registry_oot
    except Exception as e:  # noqa: BLE001 - no vLLM
        logger.debug("vLLM not importable: %s", e)
        return {}
    if not _b200_active():
        return {}
    _, B200MoEMethod = methods()
    name = "UnquantizedFusedMoEMethod"
    if name not in op_registry_oot:
        CustomOp.register_oot(name=name)(B200MoEMethod)
    INSTALLED[name] = B200MoEMethod
    return dict(INSTALLED)
