"""vLLM model classes that run this library's fused kernels.

Registered with vLLM's ``ModelRegistry`` by the models area
(``integration/models.py``) and selected with
``--hf-overrides '{"architectures": ["B200LlamaForCausalLM"]}'`` (or the
Qwen3 variants). Each class keeps vLLM's module tree, weight names and
loaders (so HF checkpoints, TP sharding and the quantisation configs work
unchanged) and swaps in the B200 pieces where the layer structure allows it:

* MLP (Llama, Qwen3-MoE dense layers): the merged ``gate_up_proj`` becomes
  ONE tcgen05 GEMM with SiLU(gate) * up fused into its epilogue
  (:class:`GateUpSiluMethod`: rows interleaved in 64-row gate / up blocks at
  load time, output width I instead of 2I), and the activation module is
  dropped;
* routed experts (Qwen3-MoE, Qwen3-Next, bf16): :class:`B200MoEMethod` runs
  the expert-sorted permutation, the grouped tcgen05 expert GEMMs, SiLU * up
  and the weighted combine of ``ops/moe.py`` instead of vLLM's fused-MoE
  kernels; routing goes through the U3 router hook;
* RMSNorm, attention, unquantised linears and the quantised linears come from
  the platform (IR-op provider, B200 attention backend, U1 GEMM hook, quant
  configs) and so apply to these classes as to any vLLM model.

Reference parity: ``sm70/vllm_sm70/models/flint_sm70/__init__.py:63-82``
(lazy ``"<module>:<class>"`` registration, checked after registering) and the
reference's model class ``flint_sm70/model.py``.
"""
from __future__ import annotations

import logging

import torch
from torch import nn

logger = logging.getLogger("vllm.b200.models")

GATE_UP_BLOCK = 64


def _b200_active() -> bool:
    from .. import _ext, platform

    return platform.is_b200_ready() and _ext.loaded()


def interleave_rows_inplace(w: torch.Tensor, block: int = GATE_UP_BLOCK) -> None:
    """[gate (I rows) | up (I rows)] -> [g0..g63, u0..u63, g64.., ...] in the
    same storage (so captured graphs and weight pointers stay valid)."""
    n2, k = w.shape
    n = n2 // 2
    g = w[:n].reshape(n // block, block, k)
    u = w[n:].reshape(n // block, block, k)
    w.copy_(torch.stack([g, u], dim=1).reshape(n2, k))


def _make_method_classes():
    from vllm.model_executor.layers.fused_moe.unquantized_fused_moe_method import (
        UnquantizedFusedMoEMethod)
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod

    from ..ops import linear as _lin
    from ..ops import moe as _moe

    class GateUpSiluMethod(UnquantizedLinearMethod):
        """Merged gate/up projection with SiLU(gate) * up in the GEMM epilogue."""

        def process_weights_after_loading(self, layer) -> None:
            super().process_weights_after_loading(layer)
            interleave_rows_inplace(layer.weight.data)
            layer._b200_interleaved = True

        def apply(self, layer, x, bias=None):
            assert bias is None
            x2 = x.reshape(-1, x.shape[-1])
            if not x2.is_contiguous():
                x2 = x2.contiguous()
            y = _lin.gemm_silu_mul(x2, layer.weight)
            return y.view(*x.shape[:-1], y.shape[-1])

    class B200MoEMethod(UnquantizedFusedMoEMethod):
        """bf16 routed experts on the grouped tcgen05 GEMMs (ops/moe.py)."""

        _b200 = True

        def _supported(self, layer) -> bool:
            moe = self.moe
            act = str(getattr(moe, "activation", "silu")).lower()
            return (not getattr(moe, "has_bias", False) and "silu" in act
                    and layer.w13_weight.dtype == torch.bfloat16
                    and layer.w13_weight.shape[1] % 256 == 0
                    and layer.w2_weight.shape[1] % 128 == 0)

        def process_weights_after_loading(self, layer) -> None:
            # vLLM's own backends may re-layout the expert weights; this method
            # reads them as loaded: w13 [E, 2I, H] ([gate | up] rows), w2 [E, H, I].
            # Layers it does not serve (bias, other activations, odd sizes) keep
            # vLLM's kernels.
            self._b200 = self._supported(layer)
            self._b200_ws = None
            if not self._b200:
                super().process_weights_after_loading(layer)

        @property
        def is_monolithic(self) -> bool:
            return False if self._b200 else super().is_monolithic

        def _workspace(self, layer, T: int, k: int, device):
            ws = self._b200_ws
            if ws is None or ws.max_tokens < T or ws.k != k:
                E, I2, H = layer.w13_weight.shape
                cap = max(T, 256)
                ws = _moe.MoEWorkspace(cap, k, E, H, I2 // 2, device)
                self._b200_ws = ws
            return ws

        def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
                  shared_experts_input=None):
            if not self._b200:
                return super().apply(layer, x, topk_weights, topk_ids, shared_experts,
                                     shared_experts_input)
            E, I2, H = layer.w13_weight.shape
            ew = _moe.ExpertWeights("bf16", E, H, I2 // 2,
                                    layer.w13_weight.data.view(E * I2, H),
                                    layer.w2_weight.data.view(E * H, I2 // 2))
            T, k = topk_ids.shape
            ws = self._workspace(layer, T, k, x.device)
            x2 = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
            e_base = getattr(self, "_b200_ebase", None)
            if e_base is None:
                # Expert-parallel layer: global ids of the local experts are
                # contiguous; the first local global id is the base. Read once
                # (the first call runs in vLLM's profiling pass, before capture).
                e_base = 0
                emap = getattr(layer, "expert_map", None)
                if emap is not None:
                    local = torch.nonzero(emap >= 0).flatten()
                    e_base = int(local[0]) if local.numel() else 0
                self._b200_ebase = e_base
            return _moe.experts_forward(x2.contiguous(), topk_weights.float().contiguous(),
                                        topk_ids.to(torch.int32).contiguous(), ew, ws,
                                        e_base=e_base).to(x.dtype)

    return GateUpSiluMethod, B200MoEMethod


_METHODS = None


def methods():
    global _METHODS
    if _METHODS is None:
        _METHODS = _make_method_classes()
    return _METHODS


def fuse_mlp(mlp: nn.Module, quant_config) -> bool:
    """Turn a vLLM ``gate_up_proj -> act_fn -> down_proj`` MLP into the fused
    form when it is unquantised bf16 SiLU with I a multiple of 64."""
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod

    GateUpSiluMethod, _ = methods()
    gu = getattr(mlp, "gate_up_proj", None)
    if gu is None or not isinstance(getattr(gu, "quant_method", None), UnquantizedLinearMethod):
        return False
    if getattr(gu, "bias", None) is not None or quant_config is not None:
        return False
    n2 = gu.weight.shape[0]
    if n2 % (2 * GATE_UP_BLOCK) != 0 or gu.weight.dtype != torch.bfloat16:
        return False
    gu.quant_method = GateUpSiluMethod()
    mlp.act_fn = nn.Identity()
    return True


def swap_moe_methods(model: nn.Module) -> int:
    """Replace vLLM's unquantised fused-MoE method of every routed-expert layer
    with :class:`B200MoEMethod`; returns the number of layers swapped."""
    from vllm.model_executor.layers.fused_moe.unquantized_fused_moe_method import (
        UnquantizedFusedMoEMethod)

    _, B200MoEMethod = methods()
    n = 0
    for mod in model.modules():
        qm = getattr(mod, "quant_method", None)
        if type(qm) is UnquantizedFusedMoEMethod and getattr(mod, "w13_weight", None) is not None:
            if mod.w13_weight.dtype != torch.bfloat16:
                continue
            mod.quant_method = B200MoEMethod(qm.moe)
            n += 1
    return n


def _classes():
    from vllm.model_executor.models.llama import LlamaDecoderLayer, LlamaForCausalLM
    from vllm.model_executor.models.qwen3_moe import Qwen3MoeForCausalLM

    class B200LlamaDecoderLayer(LlamaDecoderLayer):
        def __init__(self, vllm_config, prefix: str = "", config=None, **kw):
            super().__init__(vllm_config=vllm_config, prefix=prefix, config=config, **kw)
            if _b200_active():
                fuse_mlp(self.mlp, self.get_quant_config(vllm_config))

    class B200LlamaForCausalLM(LlamaForCausalLM):
        """Llama family on the B200 kernels (fused gate_up + SiLU epilogue)."""

        def __init__(self, *, vllm_config, prefix: str = ""):
            super().__init__(vllm_config=vllm_config, prefix=prefix,
                             layer_type=B200LlamaDecoderLayer)

    class B200Qwen3MoeForCausalLM(Qwen3MoeForCausalLM):
        """Qwen3-MoE on the B200 kernels (grouped expert GEMMs, fused dense MLPs)."""

        def __init__(self, *, vllm_config, prefix: str = ""):
            super().__init__(vllm_config=vllm_config, prefix=prefix)
            if _b200_active():
                qc = vllm_config.quant_config
                for layer in self.model.layers:
                    mlp = getattr(layer, "mlp", None)
                    if mlp is not None and hasattr(mlp, "gate_up_proj"):
                        fuse_mlp(mlp, qc)
                swap_moe_methods(self)

    out = {"B200LlamaForCausalLM": B200LlamaForCausalLM,
           "B200Qwen3MoeForCausalLM": B200Qwen3MoeForCausalLM}
    try:
        from vllm.model_executor.models.qwen3_next import Qwen3NextForCausalLM

        class B200Qwen3NextForCausalLM(Qwen3NextForCausalLM):
            """Qwen3-Next hybrid on the B200 kernels (grouped expert GEMMs; the
            gated-DeltaNet prefill runs the B200 op through the GDN area)."""

            def __init__(self, *, vllm_config, prefix: str = ""):
                super().__init__(vllm_config=vllm_config, prefix=prefix)
                if _b200_active():
                    swap_moe_methods(self)

        out["B200Qwen3NextForCausalLM"] = B200Qwen3NextForCausalLM
    except Exception as e:  # noqa: BLE001 - this vLLM has no Qwen3-Next
        logger.debug("Qwen3-Next not available in this vLLM: %s", e)
    return out


_CLASSES = None


def __getattr__(name: str):
    global _CLASSES
    if name in ("B200LlamaForCausalLM", "B200Qwen3MoeForCausalLM", "B200Qwen3NextForCausalLM"):
        if _CLASSES is None:
            _CLASSES = _classes()
        if name in _CLASSES:
            return _CLASSES[name]
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
