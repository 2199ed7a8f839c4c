"""Multi-token-prediction (MTP) draft head for speculative decoding.

One extra decoder layer that predicts the token after next from the target
model's last hidden state and the embedding of the token just sampled:

    e = rmsnorm_e(embed(tok));  h = rmsnorm_h(hidden)
    x = fc([e | h])             (2H -> H)
    x = decoder_layer(x)        (full attention over the head's own KV cache + MLP/MoE)
    hidden' = rmsnorm(x);  logits = lm_head(hidden')   (embedding / LM head shared)

Drafting k tokens runs the head k times, feeding each draft and the head's
own output hidden state back in. The head keeps one paged KV cache layer,
indexed by the same block table as the target.

Reference parity: the reference's DFlash2 draft (``sm70/vllm_sm70/models/
qwen/dflash_sm70.py``) serves the same role for Qwen3.8; Qwen3-Next ships an
MTP layer (``num_nextn_predict_layers``), used with k=3 draft tokens.
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..parallel import comm
from .layers import AttnMeta, DenseLinear, KVCache


class MTPHead:
    def __init__(self, target, seed: int = 1, std: float = 0.02):
        self.t = target
        cfg, dev, dt = target.cfg, target.device, target.dtype
        h = cfg.hidden_size
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 104729 + target.ps.tp_rank)

        def rnd(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std

        self.norm_e = torch.ones(h, device=dev, dtype=dt)
        self.norm_h = torch.ones(h, device=dev, dtype=dt)
        self.fc = DenseLinear(rnd(h, 2 * h).to(dt))  # replicated (not sharded)
        self.final_norm = torch.ones(h, device=dev, dtype=dt)
        hq, hkv, d = target.hq, target.hkv, target.d
        # gated attention (Qwen3-Next): q_proj emits [q | gate] per head
        self.gated = bool(cfg.attn_output_gate) and hasattr(target, "_attention")
        qkv_rows = ((2 if self.gated else 1) * hq + 2 * hkv) * d
        L = {"in_norm": torch.ones(h, device=dev, dtype=dt),
             "post_norm": torch.ones(h, device=dev, dtype=dt),
             "qkv": target.make_linear(rnd(qkv_rows, h)),
             "o": target.make_linear(rnd(h, hq * d))}
        if cfg.qk_norm or self.gated:
            L["q_norm"] = torch.ones(d, device=dev, dtype=dt)
            L["k_norm"] = torch.ones(d, device=dev, dtype=dt)
        L.update(target.init_mlp_dummy(rnd))
        self.layer = L
        self.kv: KVCache | None = None
        self.scale = 1.0 / math.sqrt(d)

    def allocate_cache(self, num_blocks: int, block_size: int) -> None:
        t = self.t
        self.kv = KVCache.allocate(1, num_blocks, t.hkv, block_size, t.d, dtype=t.dtype,
                                   device=t.device)

    def forward(self, ids: torch.Tensor, hidden: torch.Tensor, meta: AttnMeta) -> torch.Tensor:
        """One draft position per row: returns the head's normalised hidden."""
        t = self.t
        eps = t.cfg.rms_eps
        T = ids.shape[0]
        H = t.cfg.hidden_size
        e = ops.rms_norm(t.embed_tokens(ids), self.norm_e, eps)
        hn = ops.rms_norm(hidden.contiguous(), self.norm_h, eps)
        x = self.fc.forward(torch.cat([e, hn], 1).contiguous())
        residual = comm.adopt_residual(x)
        L = self.layer
        xn = ops.rms_norm(residual, L["in_norm"], eps)
        if self.gated:
            o = t._attention(0, L, xn, meta, self.kv, T)
            return self._finish(L, o, residual, T, H, eps)
        qkv = L["qkv"].forward(xn)
        ops.rope_kv_write(qkv, meta.positions, t.cos_sin, self.kv.k[0], self.kv.v[0],
                          meta.slot_mapping, t.hq, t.hkv, L.get("q_norm"), L.get("k_norm"), eps)
        q = qkv.view(T, t.hq + 2 * t.hkv, t.d)[:, : t.hq]
        attn = torch.empty(T, t.hq, t.d, device=ids.device, dtype=t.dtype)
        ops.paged_attention(attn, q, self.kv.k[0], self.kv.v[0], meta.block_table, meta.seq_lens,
                            meta.cu_q, meta.max_q_len, self.scale, 0, None, meta.decode,
                            meta.num_splits, meta.part_o, meta.part_ml)
        o = L["o"].forward(attn.view(T, t.hq * t.d), out=comm.row_parallel_out(T, H))
        return self._finish(L, o, residual, T, H, eps)

    def _finish(self, L, o, residual, T, H, eps):
        t = self.t
        x, residual = comm.all_reduce_add_rms_norm(o, residual, L["post_norm"], eps)
        x = t.mlp(-1, L, x, comm.row_parallel_out(T, H))
        x, residual = comm.all_reduce_add_rms_norm(x, residual, self.final_norm, eps)
        return x

    # ------------------------------------------------------------------ checkpoints
    def load_hf_state(self, get_tensor, has=None, prefix: str = "mtp.") -> None:
        """Qwen3-Next MTP weights (``mtp.*``): zero-centred RMSNorms (stored
        ``w``, effective ``1 + w``), ``fc`` over [norm(embedding) | norm(hidden)],
        one gated-attention decoder layer with the target's MoE MLP."""
        t = self.t
        assert self.gated, "checkpoint MTP weights are the Qwen3-Next (gated attention) layout"
        has = has or (lambda name: True)
        tt, qfmt, linear = t._loader_helpers(get_tensor, has)

        def zc(name):
            return (1.0 + get_tensor(name).float()).to(device=t.device, dtype=t.dtype)

        self.norm_e = zc(prefix + "pre_fc_norm_embedding.weight")
        self.norm_h = zc(prefix + "pre_fc_norm_hidden.weight")
        self.fc = DenseLinear(tt(prefix + "fc.weight"))
        self.final_norm = zc(prefix + "norm.weight")
        p = prefix + "layers.0."
        a = p + "self_attn."
        qg_rows, ks, o_cols = t.attn_shards()
        L = {"in_norm": zc(p + "input_layernorm.weight"),
             "post_norm": zc(p + "post_attention_layernorm.weight"),
             "qkv": linear([(a + "q_proj", qg_rows), (a + "k_proj", ks), (a + "v_proj", ks)]),
             "o": linear([(a + "o_proj", None)], cols=o_cols),
             "q_norm": zc(a + "q_norm.weight"), "k_norm": zc(a + "k_norm.weight")}
        L.update(t._load_mlp(p + "mlp.", get_tensor, has, tt, qfmt, linear))
        self.layer = L

    def hf_state_dict(self, prefix: str = "mtp.") -> dict:
        """Inverse of ``load_hf_state`` (TP = 1, bf16)."""
        t, L = self.t, self.layer
        hq, hkv, d = t.hq, t.hkv, t.d

        def unzc(w):
            return (w.float() - 1.0).to(w.dtype)

        p = prefix + "layers.0."
        a = p + "self_attn."
        qg, k, v = torch.split(L["qkv"].w, [2 * hq * d, hkv * d, hkv * d])
        sd = {prefix + "pre_fc_norm_embedding.weight": unzc(self.norm_e),
              prefix + "pre_fc_norm_hidden.weight": unzc(self.norm_h),
              prefix + "fc.weight": self.fc.w, prefix + "norm.weight": unzc(self.final_norm),
              p + "input_layernorm.weight": unzc(L["in_norm"]),
              p + "post_attention_layernorm.weight": unzc(L["post_norm"]),
              a + "q_proj.weight": qg, a + "k_proj.weight": k, a + "v_proj.weight": v,
              a + "o_proj.weight": L["o"].w, a + "q_norm.weight": unzc(L["q_norm"]),
              a + "k_norm.weight": unzc(L["k_norm"])}
        sd.update(t._mlp_state(p + "mlp.", L))
        return {k_: v_.detach().contiguous().cpu() for k_, v_ in sd.items()}
