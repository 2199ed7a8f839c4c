"""Gated-DeltaNet area: vLLM's Qwen3-Next / Qwen3.5 linear-attention layers
run the gated delta rule on this library's kernels.

``QwenGatedDeltaNetAttention`` is a vLLM ``PluggableLayer``: registering an
out-of-tree subclass under its name makes every instance vLLM's model code
builds an instance of the subclass (no upstream file is touched). The
subclass overrides ``_forward_core`` -- causal conv1d + recurrence, between
the projections that vLLM keeps -- for the batches it can serve:

* prefill and mixed prefill / decode batches: vLLM's varlen causal conv1d,
  then the chunked tensor-core gated delta rule (``csrc/gdn/gdn_chunk.cu``:
  64-token WY/UT form, fp32 state in registers across chunks) straight on
  the raw gates ``a`` / ``b`` and the un-normalised q / k (gating, L2 norm
  and the q scale happen inside the kernel, so vLLM's post-conv preparation
  pass and its gather / scatter of the initial states disappear); sequences
  without an initial state start from zero through ``has_init``;
* pure decode batches: vLLM's conv1d state update, then the token-serial
  recurrence kernel (``csrc/gdn/gdn.cu``) on the slot-indexed state.

The kernels keep the state in fp32 and read it in place from vLLM's paged
state cache (slot stride = the cache's page stride), so the route needs
``mamba_ssm_cache_dtype="float32"``; a bf16 state, speculative rows in the
batch, head dims other than 64 / 128 (prefill: 128) or a state layout the
kernels cannot address keep the upstream path, as does the start-up warm-up
pass without metadata. Padding rows of a captured decode batch carry the
null block (0); they are mapped to "no state", so they neither read nor
write a slot. Kill switch: ``VLLM_B200_GDN=0``.

Reference parity: the reference's GDN layer subclass registered through
``PluggableLayer.register_oot`` (``sm70/vllm_sm70/gdn/layer.py:42-56``),
which routes non-speculative decode to its own recurrence kernel and keeps
upstream's conv1d; here prefill is routed as well.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Callable

import torch

logger = logging.getLogger("vllm.b200.gdn")
INSTALLED: dict[str, type] = {}
_NULL_BLOCK_ID = 0  # vLLM's reserved null block: state index of padding rows


@dataclass
class GdnDims:
    """The per-rank shape of one GDN layer."""
    HK: int
    HV: int
    DK: int
    DV: int

    @classmethod
    def of(cls, layer) -> "GdnDims":
        tp = max(int(getattr(layer, "tp_size", 1)), 1)
        return cls(layer.num_k_heads // tp, layer.num_v_heads // tp, layer.head_k_dim,
                   layer.head_v_dim)


def state_ok(ssm_state: torch.Tensor, d: GdnDims) -> bool:
    """Can the kernels address this state cache in place? fp32, [slots, HV,
    DV, DK] with each slot a dense 16-byte aligned block (slots may be padded
    apart, as pages of vLLM's hybrid cache are)."""
    if ssm_state.dtype != torch.float32 or ssm_state.dim() != 4:
        return False
    if tuple(ssm_state.shape[1:]) != (d.HV, d.DV, d.DK):
        return False
    return (ssm_state.stride(3) == 1 and ssm_state.stride(2) == d.DK
            and ssm_state.stride(1) == d.DV * d.DK and ssm_state.stride(0) >= d.HV * d.DV * d.DK
            and ssm_state.stride(0) % 4 == 0 and ssm_state.data_ptr() % 16 == 0)


def can_serve(md, ssm_state: torch.Tensor, d: GdnDims) -> bool:
    if md is None or getattr(md, "spec_sequence_masks", None) is not None:
        return False
    if md.num_prefills == 0 and md.num_decodes == 0:
        return False
    if d.HV % d.HK:
        return False
    if md.num_prefills > 0:
        if not (d.DK == d.DV == 128):  # the chunked kernel's head dims
            return False
    elif not (d.DK == d.DV and d.DK in (64, 128)):
        return False
    return state_ok(ssm_state, d)


def _capturing(t: torch.Tensor) -> bool:
    return t.is_cuda and torch.cuda.is_current_stream_capturing()


def _fp32(layer, name: str) -> torch.Tensor:
    """fp32 copy of a per-head gate parameter, refreshed when the parameter
    is rewritten (weight loading copies into it in place). Never stored while
    a CUDA graph is being captured: captured kernels do not run, so a cache
    filled then would hold garbage for later eager calls (the graph itself
    recomputes the cast on every replay)."""
    p = getattr(layer, name)
    if p.dtype == torch.float32:
        return p.detach()
    key = (p.data_ptr(), p._version)
    cache = layer.__dict__.setdefault("_b200_fp32", {})
    hit = cache.get(name)
    if hit is None or hit[0] != key:
        val = p.detach().float().contiguous()
        if _capturing(val):
            return val
        hit = (key, val)
        cache[name] = hit
    return hit[1]


def _rows(x: torch.Tensor) -> torch.Tensor:
    return x if x.stride(-1) == 1 else x.contiguous()


def _gates(a: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    if a.stride(-1) == 1 and b.stride(-1) == 1 and a.stride(0) == b.stride(0):
        return a, b
    return a.contiguous(), b.contiguous()


_CU: dict = {}


def _decode_cu(n: int, device) -> torch.Tensor:
    """[0, 1, ..., n] (one token per decode row), cached per device and sized
    past any captured decode batch (vLLM's eager warm-up pass before each
    capture fills it); under capture a missing cache is computed in the graph
    and not stored."""
    c = _CU.get(device)
    if c is None or c.numel() < n + 1:
        c = torch.arange(max(n + 1, 16384), dtype=torch.int32, device=device)
        if _capturing(c):
            return c[: n + 1]
        _CU[device] = c
    return c[: n + 1]


def gdn_core(layer, mixed_qkv: torch.Tensor, b: torch.Tensor, a: torch.Tensor,
             core_attn_out: torch.Tensor, md, conv_state: torch.Tensor,
             ssm_state: torch.Tensor, conv_prefill: Callable, conv_decode: Callable) -> bool:
    """The GDN core of one vLLM forward on this library's kernels.

    ``conv_prefill(x, md)`` / ``conv_decode(x, idx)`` run vLLM's causal
    conv1d (they own the conv-state layout). Returns False, having done
    nothing, when the batch is not one this route serves."""
    from ..ops import gdn as gdn_ops

    d = GdnDims.of(layer)
    if not can_serve(md, ssm_state, d):
        return False
    n = int(md.num_actual_tokens)
    kd = d.HK * d.DK
    a, b = _gates(a[:n], b[:n])
    A_log, dt_bias = _fp32(layer, "A_log"), _fp32(layer, "dt_bias")
    out = core_attn_out[:n].reshape(n, d.HV * d.DV)
    direct = out.data_ptr() == core_attn_out.data_ptr() and out.stride(-1) == 1
    o = out if direct else torch.empty(n, d.HV * d.DV, dtype=core_attn_out.dtype,
                                       device=core_attn_out.device)
    if md.num_prefills > 0:
        x = _rows(conv_prefill(mixed_qkv[:n], md))
        cu = md.non_spec_query_start_loc.to(torch.int32)
        slots = md.non_spec_state_indices_tensor.to(torch.int32)
        has_init = md.has_initial_state
        gdn_ops.gdn_recurrent(x[:, :kd], x[:, kd:2 * kd], x[:, 2 * kd:], a, b, A_log, dt_bias,
                              ssm_state, cu, slots, d.HK, d.HV, out=o, chunked=True,
                              has_init=None if has_init is None else has_init.contiguous())
    else:
        idx = md.non_spec_state_indices_tensor[:n]
        x = _rows(conv_decode(mixed_qkv[:n], idx))
        slots = torch.where(idx == _NULL_BLOCK_ID, -1, idx).to(torch.int32)
        gdn_ops.gdn_recurrent(x[:, :kd], x[:, kd:2 * kd], x[:, 2 * kd:], a, b, A_log, dt_bias,
                              ssm_state, _decode_cu(n, x.device), slots, d.HK, d.HV, out=o)
    if not direct:
        core_attn_out[:n].copy_(o.view(core_attn_out[:n].shape))
    return True


def _vllm_conv(layer, up, conv_state):
    w = layer.conv1d.weight
    w2 = w.view(w.size(0), w.size(2))

    def prefill(x, md):
        return up.causal_conv1d_fn(
            x.transpose(0, 1), w2, layer.conv1d.bias, activation=layer.activation,
            conv_states=conv_state, has_initial_state=md.has_initial_state,
            cache_indices=md.non_spec_state_indices_tensor,
            query_start_loc=md.non_spec_query_start_loc, metadata=md).transpose(0, 1)

    def decode(x, idx):
        return up.causal_conv1d_update(x, conv_state, w2, layer.conv1d.bias, layer.activation,
                                       conv_state_indices=idx, validate_data=False)

    return prefill, decode


def layer_class():
    """Build the subclass of vLLM's ``QwenGatedDeltaNetAttention`` (imports
    vLLM)."""
    from vllm.forward_context import get_forward_context
    from vllm.model_executor.layers.mamba.gdn import qwen_gdn_linear_attn as up

    class B200QwenGatedDeltaNetAttention(up.QwenGatedDeltaNetAttention):
        def _forward_core(self, mixed_qkv, b, a, core_attn_out):
            raw = get_forward_context().attn_metadata
            md = raw.get(self.prefix) if isinstance(raw, dict) else None
            if md is not None:
                conv_state = (self.kv_cache[0] if up.is_conv_state_dim_first()
                              else self.kv_cache[0].transpose(-1, -2))
                prefill, decode = _vllm_conv(self, up, conv_state)
                if gdn_core(self, mixed_qkv, b, a, core_attn_out, md, conv_state,
                            self.kv_cache[1], prefill, decode):
                    return None
            return super()._forward_core(mixed_qkv, b, a, core_attn_out)

    return B200QwenGatedDeltaNetAttention


def register() -> dict[str, type]:
    """Install the GDN layer subclass with vLLM's out-of-tree registry
    (idempotent). Returns the installed classes by upstream name."""
    from .. import envs
    from .vllm_models import _b200_active

    if INSTALLED or not envs.get("VLLM_B200_GDN"):
        return dict(INSTALLED)
    try:
        from vllm.model_executor.custom_op import PluggableLayer, op_registry_oot
    except Exception as e:  # noqa: BLE001 - no vLLM
        logger.debug("vLLM not importable: %s", e)
        return {}
    if not _b200_active():
        return {}
    name = "QwenGatedDeltaNetAttention"
    if name in op_registry_oot:
        logger.warning("another plugin already replaced %s; keeping it", name)
        return {}
    cls = layer_class()
    PluggableLayer.register_oot(name=name)(cls)
    INSTALLED[name] = cls
    return dict(INSTALLED)
