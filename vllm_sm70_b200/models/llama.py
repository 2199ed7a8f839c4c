"""Llama-family dense decoder (Llama-3.x; Qwen3-dense with q/k-norm) on the
B200 kernels, tensor-parallel over the TP group.

Per layer (T tokens):
  x   = fused_add_rms_norm(x, residual)                  # residual += x
  qkv = gemm(x, Wqkv)                                     # tcgen05
  rope_kv_write(qkv -> q rotated in place, K/V -> paged cache)
  a   = paged_attention(q view of qkv)                    # GQA-packed
  o   = gemm(a, Wo)          -- TP: all-reduce fused with the next norm
  h   = gemm_silu_mul(norm(o + residual), Wgate_up)       # SiLU*up in epilogue
  x   = gemm(h, Wdown)       -- TP: all-reduce fused with the next norm

Reference parity: the reference's dense path is the Flint layer stack
(``sm70/vllm_sm70/models/flint_sm70/model.py:145-482``) through upstream
vLLM Column/RowParallel layers; here the model class owns its TP layers so
the row-parallel all-reduce can be fused with the residual add + RMSNorm
(the reference's K17, ``sm70/vllm_sm70/ar_rms_fusion.py:105-433``).
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..parallel import comm, state as pstate
from ..utils import launch_count, tracing
from .config import ModelConfig
from .layers import AttnMeta, DenseLinear, GateUpLinear, KVCache


class _QuantGateUp:
    """Quantised gate/up projection ([gate | up] rows) followed by SiLU*up."""

    def __init__(self, lin):
        self.lin = lin
        self.w = None  # no bf16 weight: the tuner skips this layer
        self.out_features = lin.out_features // 2
        self.in_features = lin.in_features

    def forward(self, x, out=None):
        h = self.lin.forward(x)
        return ops.silu_mul(h, out=out)

    def weight_bytes(self):
        return self.lin.weight_bytes()


CANDIDATES = 64  # per-shard candidate set of top-k / top-p sampling (kernel limit)


def _shard(n: int, tp: int, rank: int) -> slice:
    assert n % tp == 0, (n, tp)
    k = n // tp
    return slice(rank * k, (rank + 1) * k)


class LlamaModel:
    def __init__(self, cfg: ModelConfig, device: torch.device, dtype=torch.bfloat16,
                 ps: pstate.ParallelState | None = None):
        self.cfg = cfg
        self.device = device
        self.dtype = dtype
        self.ps = ps or pstate.get()
        tp = self.ps.tp_size
        assert cfg.num_heads % tp == 0, "num_heads must divide by TP"
        self.hq = cfg.num_heads // tp
        self.hkv = max(1, cfg.num_kv_heads // tp)
        self.kv_replicated = cfg.num_kv_heads < tp
        self.d = cfg.head_dim
        self.inter = cfg.intermediate_size // tp
        assert cfg.vocab_size % tp == 0 or True
        self.vocab_local = math.ceil(cfg.vocab_size / tp)
        self.vocab_start = self.ps.tp_rank * self.vocab_local
        self.layers: list[dict] = []
        self.scale = 1.0 / math.sqrt(self.d)
        self.cos_sin = None
        self.embed = None        # this rank's vocab shard (LM-head tie)
        self.embed_full = None   # the whole table, replicated: no collective on lookup
        self.lm_head = None
        self.final_norm = None

    # ------------------------------------------------------------------ weights
    def make_linear(self, w: torch.Tensor) -> "DenseLinear":
        """Dense bf16 or weight-only quantised linear per ``cfg.quant``."""
        if self.cfg.quant in ("fp8", "awq", "nvfp4"):
            from ..ops import quant

            return quant.make_linear(self.cfg.quant, w)
        return DenseLinear(w.to(self.dtype))

    def make_gate_up(self, wg: torch.Tensor, wu: torch.Tensor):
        if self.cfg.quant in ("fp8", "awq", "nvfp4"):
            from ..ops import quant

            return _QuantGateUp(quant.make_linear(self.cfg.quant, torch.cat([wg, wu], 0)))
        return GateUpLinear(wg.to(self.dtype), wu.to(self.dtype))

    def init_mlp_dummy(self, rnd) -> dict:
        h = self.cfg.hidden_size
        return {"gate_up": self.make_gate_up(rnd(self.inter, h), rnd(self.inter, h)),
                "down": self.make_linear(rnd(h, self.inter))}

    def init_layer_mlp_dummy(self, rnd, li: int) -> dict:
        """The MLP weights of layer ``li`` (every layer alike here)."""
        return self.init_mlp_dummy(rnd)

    def init_dummy(self, seed: int = 0, std: float = 0.02) -> None:
        """Random-init weights of the configured shapes (TP-local shards)."""
        cfg, dev, dt = self.cfg, self.device, self.dtype
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 7919 + self.ps.tp_rank)

        def rnd(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std

        h = cfg.hidden_size
        self._set_embedding(self._dummy_embedding(seed, std))
        self.lm_head = self.embed if cfg.tie_embeddings else rnd(self.vocab_local, h).to(dt)
        self.final_norm = torch.ones(h, device=dev, dtype=dt)
        qkv_out = (self.hq + 2 * self.hkv) * self.d
        self.layers = []
        for _ in range(cfg.num_layers):
            L = {
                "in_norm": torch.ones(h, device=dev, dtype=dt),
                "post_norm": torch.ones(h, device=dev, dtype=dt),
                "qkv": self.make_linear(rnd(qkv_out, h)),
                "o": self.make_linear(rnd(h, self.hq * self.d)),
            }
            L.update(self.init_layer_mlp_dummy(rnd, len(self.layers)))
            if cfg.qk_norm:
                L["q_norm"] = torch.ones(self.d, device=dev, dtype=dt)
                L["k_norm"] = torch.ones(self.d, device=dev, dtype=dt)
            self.layers.append(L)
        self._init_rope()

    def _loader_helpers(self, get_tensor, has):
        """(t, qfmt, linear) closures over a checkpoint: ``t(name)`` a tensor
        on this device in the compute dtype; ``qfmt(prefix)`` the storage
        format of that projection (``"fp8"`` block-FP8, ``"awq"`` AutoAWQ
        int4, ``"nvfp4"`` ModelOpt NVFP4, None for plain floats);
        ``linear(parts, cols)`` a linear layer from row slices of one or more
        projections in their format (shards stay aligned to the scale blocks:
        128 rows / columns for FP8, 8 output columns / 128 input rows for
        AWQ, 16 input columns for NVFP4)."""
        cfg, dev, dt = self.cfg, self.device, self.dtype
        from ..ops import quant

        def t(name):
            return get_tensor(name).to(device=dev, dtype=dt)

        def qfmt(prefix):
            if cfg.quant == "fp8" and has(prefix + ".weight_scale_inv"):
                return "fp8"
            if has(prefix + ".qweight"):
                return "awq"
            if has(prefix + ".weight_scale") and has(prefix + ".weight_scale_2"):
                return "nvfp4"
            return None

        def div(sl: slice, n: int, what: str) -> slice:
            assert sl.start % n == 0 and sl.stop % n == 0, f"{what} shard not aligned to {n}"
            return slice(sl.start // n, sl.stop // n)

        def fp8_part(pre, rows, cols):
            w = get_tensor(pre + ".weight")
            s = get_tensor(pre + ".weight_scale_inv").float()
            rows = rows or slice(0, w.shape[0])
            w, s = w[rows], s[div(rows, 128, "FP8")]
            if cols is not None:
                w, s = w[:, cols], s[:, div(cols, 128, "FP8")]
            return w, s

        def awq_part(pre, rows, cols):
            q, z, sc = (get_tensor(pre + n) for n in (".qweight", ".qzeros", ".scales"))
            rows = rows or slice(0, q.shape[1] * 8)
            q, z, sc = q[:, div(rows, 8, "AWQ")], z[:, div(rows, 8, "AWQ")], sc[:, rows]
            if cols is not None:
                g = div(cols, 128, "AWQ")
                q, z, sc = q[cols], z[g], sc[g]
            return q, z, sc

        def nvfp4_part(pre, rows, cols):
            w = get_tensor(pre + ".weight").view(torch.uint8)
            s = get_tensor(pre + ".weight_scale").view(torch.float8_e4m3fn)
            g = float(get_tensor(pre + ".weight_scale_2").float().max())
            rows = rows or slice(0, w.shape[0])
            w, s = w[rows], s[rows]
            if cols is not None:
                w, s = w[:, div(cols, 2, "NVFP4")], s[:, div(cols, 16, "NVFP4")]
            return w, s, g

        def linear(parts, cols=None):
            """Concatenate the row slices ``parts = [(prefix, rows)]`` (rows of
            each projection), optionally cutting input columns ``cols``."""
            fmts = {qfmt(pre) for pre, _ in parts}
            if fmts == {"fp8"}:
                ws, ss = zip(*(fp8_part(pre, rows, cols) for pre, rows in parts))
                return quant.Fp8BlockLinear(torch.cat(ws).to(dev), torch.cat(ss).to(dev))
            if fmts == {"awq"}:
                qs, zs, scs = zip(*(awq_part(pre, rows, cols) for pre, rows in parts))
                return quant.AwqLinear(torch.cat(qs, 1).to(dev), torch.cat(zs, 1).to(dev),
                                       torch.cat(scs, 1).to(dev), cfg.quant_group)
            if fmts == {"nvfp4"}:
                ws, ss, gs = zip(*(nvfp4_part(pre, rows, cols) for pre, rows in parts))
                w, s, g = quant.merge_nvfp4_parts(list(ws), list(ss), list(gs))
                return quant.Nvfp4Linear(w.to(dev), s.to(dev), g)
            ws = []
            for pre, rows in parts:
                w = (self._dense_weight(get_tensor, qfmt, pre).to(device=dev, dtype=dt)
                     if qfmt(pre) else t(pre + ".weight"))
                w = w[rows] if rows is not None else w
                ws.append(w[:, cols] if cols is not None else w)
            return DenseLinear(torch.cat(ws, 0))

        return t, qfmt, linear

    @staticmethod
    def _dense_weight(get_tensor, qfmt, prefix: str) -> torch.Tensor:
        """The full-precision (fp32, CPU) weight ``[N, K]`` of a projection in
        any stored format (quantised ones dequantised)."""
        from ..ops import quant

        fmt = qfmt(prefix)
        if fmt is None:
            return get_tensor(prefix + ".weight").float()
        if fmt == "fp8":
            w = get_tensor(prefix + ".weight")
            s = get_tensor(prefix + ".weight_scale_inv").float()
            s = s.repeat_interleave(128, 0)[: w.shape[0]].repeat_interleave(128, 1)[:, : w.shape[1]]
            return w.float() * s
        if fmt == "awq":
            lin = quant.AwqLinear(get_tensor(prefix + ".qweight"), get_tensor(prefix + ".qzeros"),
                                  get_tensor(prefix + ".scales"))
        else:
            lin = quant.Nvfp4Linear(get_tensor(prefix + ".weight").view(torch.uint8),
                                    get_tensor(prefix + ".weight_scale"),
                                    float(get_tensor(prefix + ".weight_scale_2").float().max()))
        return lin.reference_weight()

    def load_hf_state(self, get_tensor, has=None) -> None:
        """Load from an HF Llama / Qwen3-dense checkpoint: bf16 / fp16 weights,
        or block-FP8 (``weight`` e4m3 + ``weight_scale_inv`` per 128x128
        block, the HF "fp8" quantization_config layout). ``get_tensor(name)``
        returns the full (unsharded) tensor; this rank's shards are cut here
        (FP8 shards stay aligned to the 128-row / -column scale blocks)."""
        cfg = self.cfg
        tp, r = self.ps.tp_size, self.ps.tp_rank
        has = has or (lambda name: True)
        t, qfmt, linear = self._loader_helpers(get_tensor, has)
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
        self.final_norm = t("model.norm.weight")
        qs = _shard(cfg.num_heads * self.d, tp, r)
        if self.kv_replicated:
            kvh = r * cfg.num_kv_heads // tp
            ks = slice(kvh * self.d, (kvh + 1) * self.d)
        else:
            ks = _shard(cfg.num_kv_heads * self.d, tp, r)
        self.layers = []
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            a, m = p + "self_attn.", p + "mlp."
            L = {
                "in_norm": t(p + "input_layernorm.weight"),
                "post_norm": t(p + "post_attention_layernorm.weight"),
                "qkv": linear([(a + "q_proj", qs), (a + "k_proj", ks), (a + "v_proj", ks)]),
                "o": linear([(a + "o_proj", None)], cols=qs),
            }
            L.update(self._load_layer_mlp(i, m, get_tensor, has, t, qfmt, linear))
            if cfg.qk_norm:
                L["q_norm"] = t(a + "q_norm.weight")
                L["k_norm"] = t(a + "k_norm.weight")
            L.update(self._load_layer_extra(i, a, get_tensor, has, t))
            self.layers.append(L)
        self._init_rope()

    def hf_state_dict(self) -> dict:
        """This (TP = 1, bf16) model's weights under HF checkpoint names: the
        inverse of ``load_hf_state`` (used to write converted checkpoints)."""
        assert self.ps.tp_size == 1, "export from a single-rank model"
        cfg, hq, hkv, d = self.cfg, self.hq, self.hkv, self.d
        sd = {"model.embed_tokens.weight": self.embed[: cfg.vocab_size],
              "model.norm.weight": self.final_norm}
        if not cfg.tie_embeddings:
            sd["lm_head.weight"] = self.lm_head[: cfg.vocab_size]
        for i, L in enumerate(self.layers):
            p = f"model.layers.{i}."
            a = p + "self_attn."
            q, k, v = torch.split(L["qkv"].w, [hq * d, hkv * d, hkv * d])
            sd.update({p + "input_layernorm.weight": L["in_norm"],
                       p + "post_attention_layernorm.weight": L["post_norm"],
                       a + "q_proj.weight": q, a + "k_proj.weight": k, a + "v_proj.weight": v,
                       a + "o_proj.weight": L["o"].w})
            if cfg.qk_norm:
                sd[a + "q_norm.weight"] = L["q_norm"]
                sd[a + "k_norm.weight"] = L["k_norm"]
            sd.update(self._mlp_state(p + "mlp.", L))
        return {k: v.detach().contiguous().cpu() for k, v in sd.items()}

    def _mlp_state(self, m: str, L: dict) -> dict:
        g, u = ops.linear.deinterleave_gate_up(L["gate_up"].w)
        return {m + "gate_proj.weight": g, m + "up_proj.weight": u,
                m + "down_proj.weight": L["down"].w}

    def _load_layer_mlp(self, li: int, m: str, get_tensor, has, t, qfmt, linear) -> dict:
        """The MLP of layer ``li`` (every layer alike here)."""
        return self._load_mlp(m, get_tensor, has, t, qfmt, linear)

    def _load_layer_extra(self, li: int, a: str, get_tensor, has, t) -> dict:
        """Further attention tensors of layer ``li`` (none here)."""
        return {}

    def _load_mlp(self, m: str, get_tensor, has, t, qfmt, linear) -> dict:
        """Dense SwiGLU MLP at checkpoint prefix ``m`` (``...mlp.``)."""
        is_ = _shard(self.cfg.intermediate_size, self.ps.tp_size, self.ps.tp_rank)
        return self._load_swiglu(m, is_, t, qfmt, linear)

    @staticmethod
    def _load_swiglu(m: str, rows: slice, t, qfmt, linear) -> dict:
        out = {"down": linear([(m + "down_proj", None)], cols=rows)}
        gf = qfmt(m + "gate_proj")
        if gf is not None and gf == qfmt(m + "up_proj"):  # quantised [gate | up]
            out["gate_up"] = _QuantGateUp(linear([(m + "gate_proj", rows), (m + "up_proj", rows)]))
        else:
            out["gate_up"] = GateUpLinear(t(m + "gate_proj.weight")[rows],
                                          t(m + "up_proj.weight")[rows])
        return out

    def _init_rope(self) -> None:
        rot = int(self.d * self.cfg.partial_rotary_factor)
        self.cos_sin = ops.attention.rope_cos_sin(rot, self.cfg.max_position, self.cfg.rope_theta,
                                                  self.cfg.rope_scaling, device=self.device)

    def weight_bytes(self) -> int:
        n = self.embed.numel() * 2 + (0 if self.cfg.tie_embeddings else self.lm_head.numel() * 2)
        for L in self.layers:
            n += sum(L[k].weight_bytes() for k in ("qkv", "o", "gate_up", "down"))
        return n

    # ------------------------------------------------------------------ forward
    def _dummy_embedding(self, seed: int, std: float) -> torch.Tensor:
        """Random full (padded) embedding table, identical on every rank."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 7919 + 104723)
        n = self.vocab_local * self.ps.tp_size
        return (torch.randn(n, self.cfg.hidden_size, generator=g, device=self.device,
                            dtype=torch.float32) * std).to(self.dtype)

    def _set_embedding(self, full: torch.Tensor) -> None:
        """Keep the whole (padded) table on every rank -- one lookup, no
        all-reduce per step -- and this rank's vocab shard as a view of it
        (the LM head's rows when the embeddings are tied)."""
        r = self.ps.tp_rank
        self.embed_full = full.contiguous()
        self.embed = self.embed_full[r * self.vocab_local:(r + 1) * self.vocab_local]

    def embed_tokens(self, ids: torch.Tensor) -> torch.Tensor:
        out = torch.empty(ids.shape[0], self.cfg.hidden_size, device=ids.device, dtype=self.dtype)
        full = self.embed_full is not None
        table, start = (self.embed_full, 0) if full else (self.embed, self.vocab_start)
        if ids.is_cuda:
            torch.ops._b200_C.embedding(out, ids, table, start)
            launch_count.add(1)
        else:
            loc = ids - start
            ok = (loc >= 0) & (loc < table.shape[0])
            out.copy_(table[loc.clamp(0, table.shape[0] - 1)] * ok[:, None])
        if self.ps.tp_size > 1 and not full:
            pstate.tp_all_reduce(out)
        return out

    def forward(self, ids: torch.Tensor, meta: AttnMeta, kv: KVCache) -> torch.Tensor:
        cfg = self.cfg
        eps = cfg.rms_eps
        T = ids.shape[0]
        H = cfg.hidden_size
        residual = comm.adopt_residual(self.embed_tokens(ids))
        x = ops.rms_norm(residual, self.layers[0]["in_norm"], eps)
        attn_out = torch.empty(T, self.hq, self.d, device=ids.device, dtype=self.dtype)
        n_layers = len(self.layers)
        for li, L in enumerate(self.layers):
            tracing.push(f"layer{li}")
            cos_sin, window, sinks = self.attn_params(li, L)
            qkv = L["qkv"].forward(x)
            ops.rope_kv_write(qkv, meta.positions, cos_sin, kv.k[li], kv.v[li],
                              meta.slot_mapping, self.hq, self.hkv, L.get("q_norm"),
                              L.get("k_norm"), eps)
            q = qkv.view(T, self.hq + 2 * self.hkv, self.d)[:, : self.hq]
            ops.paged_attention(attn_out, q, kv.k[li], kv.v[li], meta.block_table,
                                meta.seq_lens, meta.cu_q, meta.max_q_len, self.scale, window,
                                sinks, meta.decode, meta.num_splits, meta.part_o, meta.part_ml)
            x, residual = comm.linear_all_reduce_add_rms_norm(
                L["o"], attn_out.view(T, self.hq * self.d), residual, L["post_norm"], eps)
            nxt = self.layers[li + 1]["in_norm"] if li + 1 < n_layers else self.final_norm
            x, residual = self.mlp_ar(li, L, x, residual, nxt, eps)
            tracing.pop()
        return x

    def attn_params(self, li: int, L: dict):
        """(RoPE cos/sin table, sliding window (0 = none), sink logits or
        None) of attention layer ``li``."""
        return self.cos_sin, 0, None

    def mlp_ar(self, li: int, L: dict, x: torch.Tensor, residual: torch.Tensor,
               norm_w: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
        """MLP, then the TP all-reduce + residual add + RMSNorm with ``norm_w``
        (the next layer's input norm, or the final norm). The dense SwiGLU's
        down projection can run fused with the collective in one kernel."""
        T, H = x.shape[0], self.cfg.hidden_size
        if type(self).mlp is LlamaModel.mlp:
            h = L["gate_up"].forward(x)
            return comm.linear_all_reduce_add_rms_norm(L["down"], h, residual, norm_w, eps)
        out = self.mlp(li, L, x, comm.row_parallel_out(T, H))
        return comm.all_reduce_add_rms_norm(out, residual, norm_w, eps)

    def mlp(self, li: int, L: dict, x: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
        """Dense SwiGLU MLP (row-parallel output, reduced by the caller)."""
        h = L["gate_up"].forward(x)
        return L["down"].forward(h, out=out)

    def greedy(self, hidden: torch.Tensor) -> torch.Tensor:
        """Vocab-parallel greedy sampling: local LM-head GEMM + argmax, then a
        rank-order merge of (value, id) pairs. Returns int32 ids ``[rows]``."""
        logits = ops.gemm(hidden, self.lm_head)
        if self.ps.tp_size == 1:
            ids, _ = ops.argmax(logits[:, : self.cfg.vocab_size])
            return ids
        # Padded vocab rows (vocab not divisible by TP) are excluded.
        nvalid = max(1, min(self.vocab_local, self.cfg.vocab_size - self.vocab_start))
        ids, vals = ops.argmax(logits[:, :nvalid], id_offset=self.vocab_start)
        return comm.greedy_merge(vals, ids)

    def sample(self, hidden: torch.Tensor, temperature: torch.Tensor, seeds: torch.Tensor,
               row_offsets: torch.Tensor | None = None, offset: int = 0) -> torch.Tensor:
        """Per-row temperature sampling (T <= 0: greedy) from the vocab-
        parallel LM head: local Gumbel-max per rank, rank-order merge of the
        perturbed (value, id) pairs -- exact, one tiny all-gather."""
        logits = ops.gemm(hidden, self.lm_head)
        nvalid = max(1, min(self.vocab_local, self.cfg.vocab_size - self.vocab_start))
        ids, vals = ops.sampling.gumbel_sample(logits[:, :nvalid], temperature, seeds, offset,
                                               self.vocab_start, row_offsets)
        if self.ps.tp_size == 1:
            return ids
        return comm.greedy_merge(vals, ids)

    def sample_filtered(self, hidden: torch.Tensor, temperature: torch.Tensor,
                        top_k: torch.Tensor, top_p: torch.Tensor,
                        seeds: torch.Tensor, penalize=None) -> torch.Tensor:
        """Per-row temperature + top-k + top-p sampling: the local top-64
        candidates of each vocab shard, all-gathered over TP, then one
        sampling kernel over the merged set (top-k is bounded by the
        candidate count and top-p is taken over the candidates). ``seeds``
        must already differ per step. ``penalize(logits, vocab_start)``
        (optional) rewrites this rank's fp32 logit shard first (sampling
        penalties)."""
        logits = ops.gemm(hidden, self.lm_head)
        nvalid = max(1, min(self.vocab_local, self.cfg.vocab_size - self.vocab_start))
        C = min(CANDIDATES, nvalid)
        lg = logits[:, :nvalid]
        if penalize is not None:
            lg = penalize(lg.float(), self.vocab_start).contiguous()
        v, i = ops.sampling.topk_candidates(lg, C, self.vocab_start)
        if self.ps.tp_size > 1:
            v, i = comm.gather_candidates(v, i)
        return ops.sampling.sample_candidates(v, i, temperature, top_k, top_p, seeds, 0)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        lg = ops.gemm(hidden, self.lm_head)
        if self.ps.tp_size > 1:
            lg = pstate.tp_all_gather(lg, dim=1)
        return lg[:, : self.cfg.vocab_size]
