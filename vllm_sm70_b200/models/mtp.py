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
        L = {"in_norm": torch.ones(h, device=dev, dtype=dt),
             "post_norm": torch.ones(h, device=dev, dtype=dt),
             "qkv": target.make_linear(rnd((hq + 2 * hkv) * d, h)),
             "o": target.make_linear(rnd(h, hq * d))}
        if cfg.qk_norm:
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
        qkv = L["qkv"].forward(xn)
        ops.rope_kv_write(qkv, meta.positions, t.cos_sin, self.kv.k[0], self.kv.v[0],
                          meta.slot_mapping, t.hq, t.hkv, L.get("q_norm"), L.get("k_norm"), eps)
        q = qkv.view(T, t.hq + 2 * t.hkv, t.d)[:, : t.hq]
        attn = torch.empty(T, t.hq, t.d, device=ids.device, dtype=t.dtype)
        ops.paged_attention(attn, q, self.kv.k[0], self.kv.v[0], meta.block_table, meta.seq_lens,
                            meta.cu_q, meta.max_q_len, self.scale, 0, None, meta.decode,
                            meta.num_splits, meta.part_o, meta.part_ml)
        o = L["o"].forward(attn.view(T, t.hq * t.d), out=comm.row_parallel_out(T, H))
        x, residual = comm.all_reduce_add_rms_norm(o, residual, L["post_norm"], eps)
        x = t.mlp(-1, L, x, comm.row_parallel_out(T, H))
        x, residual = comm.all_reduce_add_rms_norm(x, residual, self.final_norm, eps)
        return x
