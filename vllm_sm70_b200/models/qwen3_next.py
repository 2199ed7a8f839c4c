"""Qwen3-Next hybrid: 3:1 gated-DeltaNet linear-attention : gated full-
attention layers, a 512-expert top-10 MoE with a gated shared expert, zero-
centred RMSNorms, and a 1-layer MTP head for speculative decoding.

Full-attention layer: ``q_proj`` emits [q | gate] per head (D each); q/k
RMSNorm; partial RoPE (``partial_rotary_factor`` of the head dim); paged
attention; ``out = attn * sigmoid(gate)``; ``o_proj``.
Linear-attention layer (gated DeltaNet): ``in_proj_qkvz`` -> q, k (HK x DK),
v, z (HV x DV); ``in_proj_ba`` -> b, a (HV); causal conv1d + SiLU over
[q | k | v]; the gated delta rule with a per-sequence fp32 state; gated
RMSNorm with z; ``out_proj``.

Parallelism: attention heads, GDN heads and the shared expert are tensor-
parallel; routed experts are expert-parallel over the same group (see
``models/qwen3_moe.py``). KV cache exists only for the full-attention layers;
the GDN conv / recurrent states live in per-batch-slot buffers.

Reference parity: the Qwen GDN layer and hybrid model served by the
reference (``sm70/vllm_sm70/gdn/layer.py:42-164``, upstream Qwen3-Next), and
its DFlash2 draft for speculative decoding (replaced by the MTP head,
``models/mtp.py``).
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..ops import gdn as gdn_ops
from ..parallel import comm, state as pstate
from ..utils import launch_count
from .layers import AttnMeta, KVCache
from .qwen3_moe import Qwen3MoeModel


class Qwen3NextModel(Qwen3MoeModel):
    def __init__(self, cfg, device, dtype=torch.bfloat16, ps=None):
        super().__init__(cfg, device, dtype, ps)
        tp = self.ps.tp_size
        self.layer_types = list(cfg.layer_types) or [
            "attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(cfg.num_layers)]
        self.attn_layer_ids = [i for i, t in enumerate(self.layer_types) if t == "attention"]
        self.HK = cfg.linear_num_k_heads // tp
        self.HV = cfg.linear_num_v_heads // tp
        self.DK = cfg.linear_k_head_dim
        self.DV = cfg.linear_v_head_dim
        self.conv_dim = 2 * self.HK * self.DK + self.HV * self.DV
        self.conv_w = cfg.linear_conv_kernel
        self.rot = int(self.d * cfg.partial_rotary_factor)
        self.gdn_state = None
        self.conv_state = None
        self.max_slots = 0
        self._verify_saved: dict = {}

    # ------------------------------------------------------------------ state
    def allocate_states(self, max_slots: int) -> None:
        """Per-batch-slot GDN states: recurrent [L, slots, HV, DV, DK] fp32,
        conv [L, slots, conv_dim, W-1] fp32."""
        n_lin = sum(1 for t in self.layer_types if t == "linear_attention")
        self.max_slots = max_slots
        self.gdn_state = torch.zeros(n_lin, max_slots, self.HV, self.DV, self.DK,
                                     dtype=torch.float32, device=self.device)
        self.conv_state = torch.zeros(n_lin, max_slots, self.conv_dim, self.conv_w - 1,
                                      dtype=torch.float32, device=self.device)

    def reset_slots(self, slots: torch.Tensor) -> None:
        if self.gdn_state is not None and slots.numel():
            self.gdn_state.index_fill_(1, slots, 0.0)
            self.conv_state.index_fill_(1, slots, 0.0)

    def commit_spec(self, num_accepted: torch.Tensor, q_len: int, slots: torch.Tensor) -> None:
        """After a speculative verify of ``q_len`` tokens per row, advance the
        recurrent / conv states over the first ``num_accepted[row]`` tokens
        only (re-running the state kernels on the saved layer inputs)."""
        rows = num_accepted.shape[0]
        dev = num_accepted.device
        # Tokens of row r live at [r * q_len, r * q_len + q_len); take the first n_r.
        starts = torch.arange(rows, device=dev, dtype=torch.int64) * q_len
        n = num_accepted.to(torch.int64)
        idx_list = torch.arange(q_len, device=dev)[None, :] + starts[:, None]
        keep = torch.arange(q_len, device=dev)[None, :] < n[:, None]
        sel = idx_list[keep]
        cu = torch.zeros(rows + 1, dtype=torch.int32, device=dev)
        cu[1:] = torch.cumsum(n, 0).to(torch.int32)
        HK, HV, DK, DV = self.HK, self.HV, self.DK, self.DV
        lin = [i for i, t in enumerate(self.layer_types) if t == "linear_attention"]
        for lin_idx, li in enumerate(lin):
            if lin_idx not in self._verify_saved:
                continue
            L = self.layers[li]
            mixed, b, a = self._verify_saved[lin_idx]
            mixed_s = mixed.index_select(0, sel).contiguous()
            b_s = b.index_select(0, sel).contiguous()
            a_s = a.index_select(0, sel).contiguous()
            conv_out = gdn_ops.causal_conv1d(mixed_s, L["conv_w"], None, self.conv_state[lin_idx],
                                             cu, slots, True)
            q = conv_out[:, : HK * DK]
            k = conv_out[:, HK * DK: 2 * HK * DK]
            v = conv_out[:, 2 * HK * DK:]
            gdn_ops.gdn_recurrent(q, k, v, a_s, b_s, L["A_log"], L["dt_bias"],
                                  self.gdn_state[lin_idx], cu, slots, HK, HV)
        self._verify_saved.clear()

    # ------------------------------------------------------------------ weights
    def load_hf_state(self, get_tensor, has=None) -> None:
        """Load an HF Qwen3-Next checkpoint (bf16, or block-FP8 projections).

        Layouts converted here: the zero-centred RMSNorm weights (input /
        post-attention / final / q / k norms store ``w`` with effective weight
        ``1 + w``) become effective weights; the gated-DeltaNet ``in_proj_qkvz``
        rows, stored per key-head group as [q | k | v | z] (the group's value
        heads together), become [q (all local key heads) | k | v | z], and
        ``in_proj_ba`` ([b | a] per group) becomes [b | a]; ``conv1d.weight``
        [C, 1, W] channels are already [q | k | v]. This rank keeps its key-head
        groups (with their value heads), attention heads and MLP shards.
        Quantised GDN projections are dequantised, reordered and re-quantised
        per ``cfg.quant``.
        """
        cfg, dev, dt = self.cfg, self.device, self.dtype
        tp, r = self.ps.tp_size, self.ps.tp_rank
        has = has or (lambda name: True)
        t, qfmt, linear = self._loader_helpers(get_tensor, has)

        def zc(name):  # zero-centred norm -> effective weight
            return (1.0 + get_tensor(name).float()).to(device=dev, dtype=dt)

        def dense(prefix):  # full-precision weight of a projection (dequantised if stored so)
            return self._dense_weight(get_tensor, qfmt, prefix)

        h, d = cfg.hidden_size, self.d
        vs = slice(r * self.vocab_local, (r + 1) * self.vocab_local)
        emb = t("model.embed_tokens.weight")
        pad = self.vocab_local * tp - emb.shape[0]
        if pad:
            emb = torch.cat([emb, emb.new_zeros(pad, emb.shape[1])])
        self._set_embedding(emb)
        if cfg.tie_embeddings:
            self.lm_head = self.embed
        else:
            lm = t("lm_head.weight")
            if pad:
                lm = torch.cat([lm, lm.new_zeros(pad, lm.shape[1])])
            self.lm_head = lm[vs].contiguous()
        self.final_norm = zc("model.norm.weight")
        qg_rows, ks, o_cols = self.attn_shards()
        # gated DeltaNet: key-head groups [g0, g1) and their value heads
        HKa, HVa = cfg.linear_num_k_heads, cfg.linear_num_v_heads
        rat = HVa // HKa
        DK, DV = self.DK, self.DV
        S = 2 * DK + 2 * DV * rat
        g0, g1 = r * self.HK, (r + 1) * self.HK
        kd = HKa * DK
        self.layers = []
        for i, kind in enumerate(self.layer_types):
            p = f"model.layers.{i}."
            L = {"kind": kind, "in_norm": zc(p + "input_layernorm.weight"),
                 "post_norm": zc(p + "post_attention_layernorm.weight")}
            if kind == "attention":
                a = p + "self_attn."
                L["qkv"] = linear([(a + "q_proj", qg_rows), (a + "k_proj", ks), (a + "v_proj", ks)])
                L["o"] = linear([(a + "o_proj", None)], cols=o_cols)
                L["q_norm"] = zc(a + "q_norm.weight")
                L["k_norm"] = zc(a + "k_norm.weight")
            else:
                la = p + "linear_attn."
                W = dense(la + "in_proj_qkvz").view(HKa, S, h)[g0:g1]
                qkvz = torch.cat([W[:, :DK].reshape(-1, h), W[:, DK:2 * DK].reshape(-1, h),
                                  W[:, 2 * DK:2 * DK + DV * rat].reshape(-1, h),
                                  W[:, 2 * DK + DV * rat:].reshape(-1, h)])
                L["qkvz"] = self.make_linear(qkvz.to(dev))
                BA = dense(la + "in_proj_ba").view(HKa, 2 * rat, h)[g0:g1]
                L["ba_w"] = torch.cat([BA[:, :rat].reshape(-1, h),
                                       BA[:, rat:].reshape(-1, h)]).to(device=dev, dtype=dt)
                conv = get_tensor(la + "conv1d.weight").reshape(-1, get_tensor(
                    la + "conv1d.weight").shape[-1])
                L["conv_w"] = torch.cat([conv[g0 * DK:g1 * DK], conv[kd + g0 * DK:kd + g1 * DK],
                                         conv[2 * kd + g0 * rat * DV:2 * kd + g1 * rat * DV]]
                                        ).to(device=dev, dtype=dt)
                vh = slice(g0 * rat, g1 * rat)
                L["A_log"] = get_tensor(la + "A_log").float()[vh].to(dev)
                L["dt_bias"] = get_tensor(la + "dt_bias").float()[vh].to(dev)
                L["gnorm"] = t(la + "norm.weight")
                L["out"] = linear([(la + "out_proj", None)],
                                  cols=slice(g0 * rat * DV, g1 * rat * DV))
            L.update(self._load_mlp(p + "mlp.", get_tensor, has, t, qfmt, linear))
            self.layers.append(L)
        self._init_rope()

    def attn_shards(self) -> tuple[slice, slice, slice]:
        """This rank's rows of a gated-attention q_proj ([q | gate] per head,
        2d rows each) and of k_proj / v_proj, and its columns of o_proj."""
        cfg, d = self.cfg, self.d
        tp, r = self.ps.tp_size, self.ps.tp_rank
        qg_rows = slice(r * self.hq * 2 * d, (r + 1) * self.hq * 2 * d)
        o_cols = slice(r * self.hq * d, (r + 1) * self.hq * d)
        if self.kv_replicated:
            kvh = r * cfg.num_kv_heads // tp
            ks = slice(kvh * d, (kvh + 1) * d)
        else:
            ks = slice(r * self.hkv * d, (r + 1) * self.hkv * d)
        return qg_rows, ks, o_cols

    def hf_state_dict(self) -> dict:
        """This (TP = 1, bf16) model's weights under HF Qwen3-Next names and
        layouts: the inverse of ``load_hf_state``."""
        assert self.ps.tp_size == 1, "export from a single-rank model"
        cfg, d, h = self.cfg, self.d, self.cfg.hidden_size
        hq, hkv = self.hq, self.hkv
        HK, HV, DK, DV = self.HK, self.HV, self.DK, self.DV
        rat = HV // HK

        def unzc(w):
            return (w.float() - 1.0).to(w.dtype)

        sd = {"model.embed_tokens.weight": self.embed[: cfg.vocab_size],
              "model.norm.weight": unzc(self.final_norm)}
        if not cfg.tie_embeddings:
            sd["lm_head.weight"] = self.lm_head[: cfg.vocab_size]
        for i, L in enumerate(self.layers):
            p = f"model.layers.{i}."
            sd[p + "input_layernorm.weight"] = unzc(L["in_norm"])
            sd[p + "post_attention_layernorm.weight"] = unzc(L["post_norm"])
            if L["kind"] == "attention":
                a = p + "self_attn."
                qg, k, v = torch.split(L["qkv"].w, [2 * hq * d, hkv * d, hkv * d])
                sd.update({a + "q_proj.weight": qg, a + "k_proj.weight": k, a + "v_proj.weight": v,
                           a + "o_proj.weight": L["o"].w, a + "q_norm.weight": unzc(L["q_norm"]),
                           a + "k_norm.weight": unzc(L["k_norm"])})
            else:
                la = p + "linear_attn."
                q, k, v, z = torch.split(L["qkvz"].w, [HK * DK, HK * DK, HV * DV, HV * DV])
                W = torch.cat([q.view(HK, DK, h), k.view(HK, DK, h), v.view(HK, rat * DV, h),
                               z.view(HK, rat * DV, h)], 1).reshape(-1, h)
                b, a_ = torch.split(L["ba_w"], [HV, HV])
                BA = torch.cat([b.view(HK, rat, h), a_.view(HK, rat, h)], 1).reshape(-1, h)
                sd.update({la + "in_proj_qkvz.weight": W, la + "in_proj_ba.weight": BA,
                           la + "conv1d.weight": L["conv_w"].unsqueeze(1),
                           la + "A_log": L["A_log"], la + "dt_bias": L["dt_bias"],
                           la + "norm.weight": L["gnorm"], la + "out_proj.weight": L["out"].w})
            sd.update(self._mlp_state(p + "mlp.", L))
        return {k: v.detach().contiguous().cpu() for k, v in sd.items()}

    def init_dummy(self, seed: int = 0, std: float = 0.02) -> None:
        cfg, dev, dt = self.cfg, self.device, self.dtype
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 7919 + self.ps.tp_rank)

        def rnd(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std

        h = cfg.hidden_size
        self._set_embedding(self._dummy_embedding(seed, std))
        self.lm_head = self.embed if cfg.tie_embeddings else rnd(self.vocab_local, h).to(dt)
        # zero-centred norms: effective weight = 1 + w (w = 0 at init)
        self.final_norm = torch.ones(h, device=dev, dtype=dt)
        self.layers = []
        for li, kind in enumerate(self.layer_types):
            L = {"kind": kind, "in_norm": torch.ones(h, device=dev, dtype=dt),
                 "post_norm": torch.ones(h, device=dev, dtype=dt)}
            if kind == "attention":
                qkv_out = (2 * self.hq + 2 * self.hkv) * self.d  # [q | gate] per head, k, v
                L["qkv"] = self.make_linear(rnd(qkv_out, h))
                L["o"] = self.make_linear(rnd(h, self.hq * self.d))
                L["q_norm"] = torch.ones(self.d, device=dev, dtype=dt)
                L["k_norm"] = torch.ones(self.d, device=dev, dtype=dt)
            else:
                qkvz = 2 * self.HK * self.DK + 2 * self.HV * self.DV
                L["qkvz"] = self.make_linear(rnd(qkvz, h))
                L["ba_w"] = rnd(2 * self.HV, h).to(dt)  # tiny: kept bf16
                L["conv_w"] = (rnd(self.conv_dim, self.conv_w) * 10).to(dt)
                L["A_log"] = torch.log(torch.rand(self.HV, generator=g, device=dev) * 15 + 1)
                L["dt_bias"] = torch.ones(self.HV, device=dev)
                L["gnorm"] = torch.ones(self.DV, device=dev, dtype=dt)
                L["out"] = self.make_linear(rnd(h, self.HV * self.DV))
            L.update(self.init_mlp_dummy(rnd))
            self.layers.append(L)
        self._init_rope()

    def _init_rope(self) -> None:
        self.cos_sin = ops.attention.rope_cos_sin(self.rot, self.cfg.max_position,
                                                  self.cfg.rope_theta, self.cfg.rope_scaling,
                                                  device=self.device)

    # ------------------------------------------------------------------ forward
    def _attention(self, li, L, x, meta: AttnMeta, kv: KVCache, T):
        d, hq, hkv = self.d, self.hq, self.hkv
        qkvg = L["qkv"].forward(x)                          # [T, (2hq + 2hkv) d]
        qg = qkvg[:, : 2 * hq * d].view(T, hq, 2, d)
        gate = qg[:, :, 1]
        # contiguous [q | k | v] for the fused RoPE + KV writer
        qkv = torch.cat([qg[:, :, 0].reshape(T, hq * d), qkvg[:, 2 * hq * d:]], 1).contiguous()
        ops.rope_kv_write(qkv, meta.positions, self.cos_sin, kv.k[li], kv.v[li],
                          meta.slot_mapping, hq, hkv, L["q_norm"], L["k_norm"], self.cfg.rms_eps)
        q = qkv.view(T, hq + 2 * hkv, d)[:, :hq]
        attn = torch.empty(T, hq, d, device=x.device, dtype=self.dtype)
        ops.paged_attention(attn, q, kv.k[li], kv.v[li], meta.block_table, meta.seq_lens,
                            meta.cu_q, meta.max_q_len, self.scale, 0, None, meta.decode,
                            meta.num_splits, meta.part_o, meta.part_ml)
        attn = (attn.float() * torch.sigmoid(gate.float())).to(self.dtype)
        return L["o"].forward(attn.view(T, hq * d), out=comm.row_parallel_out(T, x.shape[1]))

    def _linear_attention(self, li, L, x, meta: AttnMeta, T):
        HK, HV, DK, DV = self.HK, self.HV, self.DK, self.DV
        lin_idx = sum(1 for t in self.layer_types[:li] if t == "linear_attention")
        qkvz = L["qkvz"].forward(x)                         # [T, 2HK DK + 2HV DV]
        mixed = qkvz[:, : self.conv_dim]
        z = qkvz[:, self.conv_dim:]
        ba = ops.gemm(x, L["ba_w"]) if x.is_cuda else (x.float() @ L["ba_w"].float().t()).to(x.dtype)
        b, a = ba[:, :HV], ba[:, HV:]
        conv_out = torch.empty(T, self.conv_dim, device=x.device, dtype=self.dtype)
        slots = meta.state_slots
        write = not meta.spec_verify
        if meta.spec_verify:  # keep the inputs for the commit pass after acceptance
            self._verify_saved[lin_idx] = (mixed, b, a)
        gdn_ops.causal_conv1d(mixed, L["conv_w"], None, self.conv_state[lin_idx], meta.cu_q,
                              slots, True, out=conv_out, write_state=write)
        q = conv_out[:, : HK * DK]
        k = conv_out[:, HK * DK: 2 * HK * DK]
        v = conv_out[:, 2 * HK * DK:]
        o = gdn_ops.gdn_recurrent(q, k, v, a, b, L["A_log"], L["dt_bias"],
                                  self.gdn_state[lin_idx], meta.cu_q, slots, HK, HV,
                                  write_state=write, chunked=not meta.decode)
        gdn_ops.gated_rmsnorm(o, z, L["gnorm"], HV, self.cfg.rms_eps)
        return L["out"].forward(o, out=comm.row_parallel_out(T, x.shape[1]))

    def forward(self, ids: torch.Tensor, meta: AttnMeta, kv: KVCache) -> torch.Tensor:
        eps = self.cfg.rms_eps
        T = ids.shape[0]
        H = self.cfg.hidden_size
        residual = comm.adopt_residual(self.embed_tokens(ids))
        x = ops.rms_norm(residual, self.layers[0]["in_norm"], eps)
        for li, L in enumerate(self.layers):
            if li > 0:
                x, residual = comm.all_reduce_add_rms_norm(x, residual, L["in_norm"], eps)
            if L["kind"] == "attention":
                o = self._attention(li, L, x, meta, kv, T)
            else:
                o = self._linear_attention(li, L, x, meta, T)
            x, residual = comm.all_reduce_add_rms_norm(o, residual, L["post_norm"], eps)
            x = self.mlp(li, L, x, comm.row_parallel_out(T, H))
        x, residual = comm.all_reduce_add_rms_norm(x, residual, self.final_norm, eps)
        self.last_hidden = x
        return x

    def weight_bytes(self) -> int:
        n = self.embed.numel() * 2 + (0 if self.cfg.tie_embeddings else self.lm_head.numel() * 2)
        for L in self.layers:
            for key in ("qkv", "o", "qkvz", "out"):
                if key in L and L[key] is not None:
                    n += L[key].weight_bytes()
            n += L["experts"].bytes()
        return n
