"""``B200CudaPlatform``: the vLLM platform class returned by ``activate()``.

Subclass of vLLM's CUDA platform with the hook surface of the reference
plugin (method names and contracts kept):

* U1 ``get_unquantized_gemm(linear_backend)`` -> callable or None, and
  ``kernel_warmup(worker)`` (pre-capture GEMM plan / tuning, router and
  sampler preparation, in that order);
* U2 ``b200_recurrent_bv(BV, V, NHV, device)`` (``sm70_recurrent_bv`` alias):
  block size for FLA's recurrent gated-delta decode;
* U3 ``get_moe_router_provider()`` -> provider(runner) -> route or None;
* U4 ``get_hidden_state_sampler()`` -> sampler with ``try_sample(...)``;
* ``get_attn_backend_cls`` (CUSTOM = B200 paged attention for bf16 decoder
  layers with head size 64/128/256; an explicit ``--attention-backend`` wins),
  ``apply_config_platform_defaults`` (graph policy), ``check_and_update_config``
  (fail-fast on failed plugin areas, composite pass install),
  ``get_default_ir_op_priority``.

The installed vLLM may lack the upstream call sites of U1-U4; ``hooks.install``
adds them by wrapping at plugin registration.

Reference parity: ``sm70/vllm_sm70/_cuda_platform.py:100-302``.
"""
from __future__ import annotations

import logging

from vllm.platforms.cuda import CudaPlatform

from .. import envs
from ..config import b200_config

logger = logging.getLogger("vllm.b200.platform")


def _enforce_strict() -> None:
    """Raise when a plugin area failed to register (unless strict is off)."""
    import vllm_sm70_b200 as pkg

    failed = pkg.retry_failed_areas()
    if failed and envs.get("VLLM_B200_PLUGIN_STRICT"):
        raise RuntimeError(f"vllm_sm70_b200: plugin areas failed to register: {failed}")


class B200CudaPlatform(CudaPlatform):
    device_name = "cuda"

    # ------------------------------------------------------------ kernels
    @classmethod
    def import_kernels(cls) -> None:
        super().import_kernels()
        from .. import _ext

        _ext.load()

    # ------------------------------------------------------------ attention
    @classmethod
    def get_attn_backend_cls(cls, selected_backend, attn_selector_config, *args, **kwargs):
        if selected_backend is None and b200_config().attention:
            from . import attention

            try:
                head = attn_selector_config.head_size
                dtype = attn_selector_config.dtype
            except AttributeError:
                head, dtype = None, None
            if head is not None and attention.select(head, dtype):
                logger.info("vllm_sm70_b200: using the B200 paged attention backend")
                return "vllm_sm70_b200.integration.attention.B200AttentionBackend"
        return super().get_attn_backend_cls(selected_backend, attn_selector_config, *args,
                                            **kwargs)

    # ------------------------------------------------------------ config
    @classmethod
    def apply_config_platform_defaults(cls, vllm_config) -> None:
        from . import graph_policy

        sup = getattr(super(), "apply_config_platform_defaults", None)
        if sup is not None:
            sup(vllm_config)
        graph_policy.apply(vllm_config, b200_config(vllm_config))

    @classmethod
    def check_and_update_config(cls, vllm_config) -> None:
        super().check_and_update_config(vllm_config)
        _enforce_strict()
        from . import passes

        passes.install_composite_pass(vllm_config)

    @classmethod
    def get_default_ir_op_priority(cls, vllm_config):
        """vLLM's CUDA defaults with the "b200" RMSNorm providers first
        (``integration/ir_ops.py``); kill switch ``VLLM_B200_RMSNORM=0``."""
        prio = super().get_default_ir_op_priority(vllm_config)
        if not envs.get("VLLM_B200_RMSNORM"):
            return prio
        from . import ir_ops

        ir_ops.register()
        return ir_ops.with_b200_first(prio)

    # ------------------------------------------------------------ U1
    @classmethod
    def get_unquantized_gemm(cls, linear_backend=None):
        """Return the tcgen05 GEMM for unquantized bf16 linears (None keeps
        upstream)."""
        if not b200_config().gemm:
            return None
        from . import hooks

        return hooks.b200_unquantized_gemm

    @classmethod
    def kernel_warmup(cls, worker) -> None:
        """Ordered pre-capture warm-up: (1) GEMM plans / tuning with TP
        agreement, (2) router preparation, (3) sampler preparation. A failure
        raises on every rank (a silent per-rank fallback would desynchronise
        collectives)."""
        from ..engine import warmup

        warmup.platform_warmup(worker)

    # ------------------------------------------------------------ U2
    @classmethod
    def b200_recurrent_bv(cls, BV: int, V: int, NHV: int, device=None) -> int:
        """Largest BV in {64, 32, 16, 8} (<= the caller's BV) that still gives
        at least two waves of CTAs over the SMs."""
        import torch

        sms = 148  # B200, when no GPU is visible (CPU-side planning)
        if torch.cuda.is_available():
            dev = device if device is not None else torch.cuda.current_device()
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
        for bv in (64, 32, 16, 8):
            if bv > BV:
                continue
            if NHV * ((V + bv - 1) // bv) >= 2 * sms:
                return bv
        return min(BV, 8)

    sm70_recurrent_bv = b200_recurrent_bv

    # ------------------------------------------------------------ U3
    @classmethod
    def get_moe_router_provider(cls):
        if not b200_config().fused_router:
            return None
        from ..models import router

        return router.provider

    # ------------------------------------------------------------ U4
    @classmethod
    def get_hidden_state_sampler(cls):
        if not b200_config().hidden_state_sampler:
            return None
        from ..engine import hidden_state_sampler

        return hidden_state_sampler.get()
