"""Quantisation area: vLLM quantisation configs whose linear methods run this
library's tcgen05 GEMMs.

Registered names (``register_quantization_config``, replacing vLLM's own
entries of the same name, as the reference plugin does for ``fp8`` and
``modelopt_fp4``):

* ``"fp8"`` -> :class:`B200Fp8Config`: checkpoints with ``weight_block_size``
  ``[128, 128]`` (e4m3 ``weight`` + fp32 ``weight_scale_inv``) run
  :class:`~vllm_sm70_b200.ops.quant.Fp8BlockLinear`;
* ``"awq"`` -> :class:`B200AWQConfig`: AutoAWQ int4, group 128, zero point
  (``qweight`` / ``qzeros`` / ``scales``) runs
  :class:`~vllm_sm70_b200.ops.quant.AwqLinear`;
* ``"modelopt_fp4"`` -> :class:`B200ModelOptNvFp4Config`: ModelOpt NVFP4
  (``weight`` e2m1 pairs, ``weight_scale`` e4m3 per 16, ``weight_scale_2``
  fp32) runs :class:`~vllm_sm70_b200.ops.quant.Nvfp4Linear`.

Each method keeps the upstream ``create_weights`` (so vLLM's loaders,
TP sharding and fused q/k/v, gate/up parameter layouts stay unchanged),
converts the loaded tensors once in ``process_weights_after_loading`` and
calls the B200 GEMM in ``apply``. Layers this library does not serve
(other block sizes, MoE experts, KV-cache scales) keep the upstream method,
and so does every layer when the B200 platform is not active (no cc 10.0
GPU), so registering on another machine changes nothing.

Reference parity: ``sm70/vllm_sm70/quant/configs.py:67-240`` (config
overrides, ``_register_all`` at :172-178), ``quant/fp8_linear.py``,
``quant/nvfp4_linear.py``.
"""
from __future__ import annotations

import logging

import torch

logger = logging.getLogger("vllm.b200.quant")

# vLLM quantisation method name -> this library's weight format.
SUPPORTED = {"fp8": "fp8", "awq": "awq", "modelopt_fp4": "nvfp4", "modelopt": "nvfp4"}
REGISTERED: dict[str, type] = {}


def method_for(quant_method: str | None) -> str | None:
    return SUPPORTED.get(quant_method) if quant_method else None


def _active() -> bool:
    """B200 linear methods run only when every visible GPU is cc 10.0 and the
    native library loaded (otherwise the upstream method is returned)."""
    from .. import _ext, platform

    return platform.is_b200_ready() and _ext.loaded()


def _apply_layer(layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None):
    lin = layer._b200_linear
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    y = lin.forward(x2)
    if bias is not None:
        y = y + bias
    return y.view(*x.shape[:-1], lin.out_features).to(x.dtype)


def _make_classes():
    """Build the config / method classes (vLLM imports happen here, not at
    plugin import, so a vLLM-less process can import this module)."""
    from vllm.model_executor.layers.linear import LinearBase
    from vllm.model_executor.layers.quantization.awq import AWQConfig, AWQLinearMethod
    from vllm.model_executor.layers.quantization.fp8 import Fp8Config, Fp8LinearMethod
    from vllm.model_executor.layers.quantization.modelopt import (
        ModelOptNvFp4Config, ModelOptNvFp4LinearMethod)

    from ..ops import quant as Q

    class B200Fp8LinearMethod(Fp8LinearMethod):
        """Block-FP8 (128 x 128) linear on the tcgen05 GEMM."""

        def process_weights_after_loading(self, layer) -> None:
            w = layer.weight.data
            if w.shape[0] != layer.output_size_per_partition:  # stored [K, N]
                w = w.t()
            layer._b200_linear = Q.Fp8BlockLinear(w.contiguous(), layer.weight_scale_inv.data)

        def apply(self, layer, x, bias=None):
            return _apply_layer(layer, x, bias)

    class B200AwqLinearMethod(AWQLinearMethod):
        """AWQ int4 g128 linear on the tcgen05 GEMM (dequantised in the producer)."""

        def process_weights_after_loading(self, layer) -> None:
            layer._b200_linear = Q.AwqLinear(layer.qweight.data, layer.qzeros.data,
                                             layer.scales.data, self.quant_config.group_size)

        def apply(self, layer, x, bias=None):
            return _apply_layer(layer, x, bias)

    class B200Nvfp4LinearMethod(ModelOptNvFp4LinearMethod):
        """ModelOpt NVFP4 linear on the tcgen05 GEMM."""

        def process_weights_after_loading(self, layer) -> None:
            g = float(layer.weight_scale_2.data.float().max())
            layer._b200_linear = Q.Nvfp4Linear(layer.weight.data.view(torch.uint8),
                                               layer.weight_scale.data, g)

        def apply(self, layer, x, bias=None):
            return _apply_layer(layer, x, bias)

    class B200Fp8Config(Fp8Config):
        def get_quant_method(self, layer, prefix):
            m = super().get_quant_method(layer, prefix)
            if (type(m) is Fp8LinearMethod and isinstance(layer, LinearBase)
                    and list(self.weight_block_size or []) == [128, 128] and _active()):
                return B200Fp8LinearMethod(self)
            return m

    class B200AWQConfig(AWQConfig):
        def get_quant_method(self, layer, prefix):
            m = super().get_quant_method(layer, prefix)
            if (type(m) is AWQLinearMethod and self.group_size == 128 and self.zero_point
                    and self.weight_bits == 4 and _active()):
                return B200AwqLinearMethod(self)
            return m

    class B200ModelOptNvFp4Config(ModelOptNvFp4Config):
        def get_quant_method(self, layer, prefix):
            m = super().get_quant_method(layer, prefix)
            if (isinstance(m, ModelOptNvFp4LinearMethod) and self.group_size == 16
                    and _active()):
                return B200Nvfp4LinearMethod(self)
            return m

    return {
        "fp8": B200Fp8Config, "awq": B200AWQConfig, "modelopt_fp4": B200ModelOptNvFp4Config,
    }, {
        "fp8": B200Fp8LinearMethod, "awq": B200AwqLinearMethod,
        "modelopt_fp4": B200Nvfp4LinearMethod,
    }


CONFIGS: dict[str, type] = {}
METHODS: dict[str, type] = {}


def register() -> dict[str, type]:
    """Register the three configs with vLLM (idempotent). Kill switches:
    ``VLLM_B200_FP8_GEMM`` / ``VLLM_B200_AWQ_GEMM`` / ``VLLM_B200_NVFP4_GEMM``."""
    from .. import envs

    if REGISTERED:
        return dict(REGISTERED)
    try:
        from vllm.model_executor.layers.quantization import register_quantization_config
    except Exception as e:  # noqa: BLE001 - vLLM not importable: nothing to register
        logger.debug("vLLM not importable, quant configs not registered: %s", e)
        return {}
    cfgs, meths = _make_classes()
    CONFIGS.update(cfgs)
    METHODS.update(meths)
    switch = {"fp8": "VLLM_B200_FP8_GEMM", "awq": "VLLM_B200_AWQ_GEMM",
              "modelopt_fp4": "VLLM_B200_NVFP4_GEMM"}
    for name, cls in cfgs.items():
        if not envs.get(switch[name]):
            continue
        register_quantization_config(name)(cls)
        REGISTERED[name] = cls
    return dict(REGISTERED)
