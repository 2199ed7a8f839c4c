"""Independent dense (non-paged) fp32 forward of a Flint model, read back
from a ``FlintModel``'s weights and driven by its ``ModelConfig`` alone:
per-layer RoPE theta / no RoPE, sliding-window masks, sink logits, dense or
sigmoid-routed MoE layers with an ungated shared expert."""
import math

import torch

from vllm_sm70_b200.ops import attention as A
from vllm_sm70_b200.ops.linear import deinterleave_gate_up

from ._llama_ref import _rms, _rope


def _swiglu(h, gate_up_w, down_w):
    wg, wu = deinterleave_gate_up(gate_up_w.float())
    g, u = h @ wg.t(), h @ wu.t()
    return (g * torch.sigmoid(g) * u) @ down_w.float().t()


def flint_logits(model, ids: torch.Tensor) -> torch.Tensor:
    cfg = model.cfg
    ex = cfg.extra
    f = lambda t: t.float().cpu()  # noqa: E731
    L = ids.numel()
    hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    pos = torch.arange(L)
    x = f(model.embed)[ids]
    for li, Ly in enumerate(model.layers):
        kind = cfg.layer_types[li]
        h = _rms(x, f(Ly["in_norm"]), cfg.rms_eps)
        qkv = h @ f(Ly["qkv"].w).t()
        q = qkv[:, : hq * d].view(L, hq, d)
        k = qkv[:, hq * d: (hq + hkv) * d].view(L, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(L, hkv, d)
        q = _rms(q, f(Ly["q_norm"]), cfg.rms_eps)
        k = _rms(k, f(Ly["k_norm"]), cfg.rms_eps)
        if li not in ex["no_rope_layers"]:
            theta = ex["rope_theta_by_type"].get(kind, cfg.rope_theta)
            cs = A.rope_cos_sin(d, max(L, 8), theta)
            q, k = _rope(q, cs, pos), _rope(k, cs, pos)
        window = ex["sliding_window"] if kind == "sliding_attention" else 0
        a = A.attention_ref(q, k, v, 1 / math.sqrt(d), window, f(Ly["sinks"]))
        x = x + a.reshape(L, hq * d) @ f(Ly["o"].w).t()
        h = _rms(x, f(Ly["post_norm"]), cfg.rms_eps)
        if li in ex["mlp_only_layers"]:
            x = x + _swiglu(h, Ly["gate_up"].w, f(Ly["down"].w))
            continue
        scores = torch.sigmoid(h @ f(Ly["router"]).t())
        w, e = scores.topk(cfg.top_k, dim=-1)
        if cfg.norm_topk_prob:
            w = w / w.sum(-1, keepdim=True)
        w13, w2 = Ly["experts"].dense_ref()
        I = cfg.moe_intermediate_size
        y = torch.zeros_like(x)
        for t in range(L):
            for j in range(cfg.top_k):
                hh = w13[int(e[t, j])] @ h[t]
                g, u = hh[:I], hh[I:]
                act = (g * torch.sigmoid(g) * u).to(torch.bfloat16).float()
                y[t] += w[t, j] * (w2[int(e[t, j])] @ act)
        if "shared_gate_up" in Ly:
            y = y + _swiglu(h, Ly["shared_gate_up"].w, f(Ly["shared_down"].w))
        x = x + y
    x = _rms(x, f(model.final_norm), cfg.rms_eps)
    return x @ f(model.lm_head).t()


def greedy_reference(model, prompt: torch.Tensor, n: int) -> list[int]:
    ids = prompt.clone()
    out = []
    for _ in range(n):
        nxt = int(flint_logits(model, ids)[-1].argmax())
        out.append(nxt)
        ids = torch.cat([ids, torch.tensor([nxt])])
    return out
