"""Flint: a sparse-MoE decoder with hybrid sliding / full attention.

Per layer (``layer_types``):
  * attention: q/k RMSNorm, GQA, a learned per-head sink logit (an extra
    softmax column with no value: ``self_attn.softmax_offset``), a sliding
    window on ``"sliding_attention"`` layers (key j visible from query i when
    i - window < j <= i), full causal on ``"full_attention"`` layers; RoPE
    with the layer type's theta, none on ``no_rope_layer_indices`` (an
    identity cos / sin table: the fused RoPE + KV-write kernel then only
    normalises and writes);
  * MLP: dense SwiGLU on ``mlp_only_layers``, else a routed MoE with sigmoid
    scores, top-k, optional renormalisation, plus an ungated shared expert.

Everything runs on the kernels of the other families: the paged attention
kernels take the window and the sinks, the router kernel the sigmoid mode,
and TP / EP follow ``Qwen3MoeModel`` (TP expert slices with the fused
all-reduce, or data-parallel attention with the all-to-all MoE).

Reference parity: ``FlintSm70ForCausalLM``
(``sm70/vllm_sm70/models/flint_sm70/model.py:145-560``: attention with
sinks / SWA / no-RoPE layers ``:260-420``, sigmoid MoE with a shared expert
``:190-250``, dense ``mlp_only_layers`` ``:440-460``). BF16 needs none of the
reference's FP16 range rescaling (``fp16_rescale.py``).
"""
from __future__ import annotations

import torch

from .. import ops
from .llama import LlamaModel, _shard
from .qwen3_moe import Qwen3MoeModel


class FlintModel(Qwen3MoeModel):
    def __init__(self, cfg, device, dtype=torch.bfloat16, ps=None):
        super().__init__(cfg, device, dtype, ps)
        ex = cfg.extra
        n = cfg.num_layers
        self.layer_kinds = tuple(cfg.layer_types) or ("full_attention",) * n
        self.window = int(ex.get("sliding_window") or 0)
        self.no_rope = set(int(i) for i in ex.get("no_rope_layers", ()))
        self.mlp_only = set(int(i) for i in ex.get("mlp_only_layers", ()))
        self.theta_by_kind = dict(ex.get("rope_theta_by_type") or {})
        self.router_sigmoid = True
        self.tables: dict = {}

    # ------------------------------------------------------------------ attention
    def _init_rope(self) -> None:
        rot = int(self.d * self.cfg.partial_rotary_factor)
        self.tables = {}
        for kind in set(self.layer_kinds):
            theta = float(self.theta_by_kind.get(kind, self.cfg.rope_theta))
            self.tables[kind] = ops.attention.rope_cos_sin(rot, self.cfg.max_position, theta,
                                                           self.cfg.rope_scaling,
                                                           device=self.device)
        ref = next(iter(self.tables.values()))
        half = ref.shape[1] // 2
        ident = torch.cat([torch.ones_like(ref[:, :half]), torch.zeros_like(ref[:, half:])], 1)
        self.tables["none"] = ident.contiguous()
        self.cos_sin = self.tables[self.layer_kinds[0]]

    def attn_params(self, li, L):
        kind = self.layer_kinds[li]
        cs = self.tables["none" if li in self.no_rope else kind]
        window = self.window if kind == "sliding_attention" else 0
        return cs, window, L.get("sinks")

    def _load_layer_extra(self, li, a, get_tensor, has, t) -> dict:
        """This rank's heads of the learned sink logits."""
        if not has(a + "softmax_offset"):
            return {}
        heads = _shard(self.cfg.num_heads, self.ps.tp_size, self.ps.tp_rank)
        return {"sinks": get_tensor(a + "softmax_offset").float()[heads].to(self.device)}

    # ------------------------------------------------------------------ MLP
    def init_layer_mlp_dummy(self, rnd, li: int) -> dict:
        if li in self.mlp_only:
            return LlamaModel.init_mlp_dummy(self, rnd)
        L = self.init_mlp_dummy(rnd)
        L.pop("shared_gate", None)  # Flint's shared expert is not gated
        return L

    def init_dummy(self, seed: int = 0, std: float = 0.02) -> None:
        super().init_dummy(seed, std)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 7919 + 31)
        heads = _shard(self.cfg.num_heads, self.ps.tp_size, self.ps.tp_rank)
        for L in self.layers:  # the same full sink vector on every rank, sliced
            full = torch.randn(self.cfg.num_heads, generator=g, device=self.device)
            L["sinks"] = full[heads].contiguous()

    def _load_layer_mlp(self, li, m, get_tensor, has, t, qfmt, linear) -> dict:
        if li in self.mlp_only:
            return LlamaModel._load_mlp(self, m, get_tensor, has, t, qfmt, linear)
        return self._load_mlp(m, get_tensor, has, t, qfmt, linear)

    def _mlp_state(self, m: str, L: dict) -> dict:
        if "experts" not in L:
            return LlamaModel._mlp_state(self, m, L)
        return super()._mlp_state(m, L)

    def hf_state_dict(self) -> dict:
        sd = super().hf_state_dict()
        for i, L in enumerate(self.layers):
            if "sinks" in L:
                sd[f"model.layers.{i}.self_attn.softmax_offset"] = L["sinks"].detach().cpu()
        return sd

    def mlp(self, li, L, x, out):
        if "experts" not in L:  # dense layer (row-parallel output)
            return LlamaModel.mlp(self, li, L, x, out)
        return super().mlp(li, L, x, out)

    def weight_bytes(self) -> int:
        n = self.embed.numel() * 2 + (0 if self.cfg.tie_embeddings else self.lm_head.numel() * 2)
        for L in self.layers:
            n += L["qkv"].weight_bytes() + L["o"].weight_bytes()
            if "experts" in L:
                n += L["experts"].bytes()
            else:
                n += L["gate_up"].weight_bytes() + L["down"].weight_bytes()
        return n
