"""Independent dense (non-paged) fp32 Llama forward used as the oracle for
model-level tests. Weights are read back from a ``LlamaModel``."""
import math

import torch

from vllm_sm70_b200.ops import attention as A
from vllm_sm70_b200.ops.linear import deinterleave_gate_up


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, cs, pos):
    half = cs.shape[1] // 2
    c, s = cs[pos, :half][:, None], cs[pos, half:][:, None]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def llama_logits(model, ids: torch.Tensor) -> torch.Tensor:
    """Full-sequence causal forward; returns fp32 logits [L, vocab]."""
    cfg = model.cfg
    f = lambda t: t.float().cpu()  # noqa: E731
    L = ids.numel()
    hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    cs = A.rope_cos_sin(d, max(L, 8), cfg.rope_theta, cfg.rope_scaling)
    pos = torch.arange(L)
    x = f(model.embed)[ids]
    for Ly in model.layers:
        h = _rms(x, f(Ly["in_norm"]), cfg.rms_eps)
        qkv = h @ f(Ly["qkv"].w).t()
        q = qkv[:, : hq * d].view(L, hq, d)
        k = qkv[:, hq * d: (hq + hkv) * d].view(L, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(L, hkv, d)
        if cfg.qk_norm:
            q = _rms(q, f(Ly["q_norm"]), cfg.rms_eps)
            k = _rms(k, f(Ly["k_norm"]), cfg.rms_eps)
        q, k = _rope(q, cs, pos), _rope(k, cs, pos)
        a = A.attention_ref(q, k, v, 1 / math.sqrt(d))
        x = x + a.reshape(L, hq * d) @ f(Ly["o"].w).t()
        h = _rms(x, f(Ly["post_norm"]), cfg.rms_eps)
        wg, wu = deinterleave_gate_up(f(Ly["gate_up"].w))
        g, u = h @ wg.t(), h @ wu.t()
        x = x + (g * torch.sigmoid(g) * u) @ f(Ly["down"].w).t()
    x = _rms(x, f(model.final_norm), cfg.rms_eps)
    return x @ f(model.lm_head).t()


def greedy_reference(model, prompt: torch.Tensor, n: int) -> list[int]:
    ids = prompt.clone()
    out = []
    for _ in range(n):
        nxt = int(llama_logits(model, ids)[-1].argmax())
        out.append(nxt)
        ids = torch.cat([ids, torch.tensor([nxt])])
    return out
