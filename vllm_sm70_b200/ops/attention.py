"""Paged attention, RoPE + KV-cache write wrappers and their CPU oracles.

Cache layout: ``k_cache / v_cache [num_blocks, Hkv, block_size, D]`` -- one
(block, kv-head) is a contiguous ``block_size x D`` tile, so a decode CTA that
serves one KV head streams contiguous 4 KiB runs (block 16, D 128).

Reference parity: Flash-V100 ops ``fv100_decode_paged{,_sinks,_xqa,_fused}``,
``fv100_prefill_paged{,_sinks}``, ``fv100_decode_verify``
(``sm70/csrc/flash_v100/fv100_ops.cpp:208-272``) and the CPU stand-ins used by
the reference tests (``sm70/tests/attention/_fv100_ref.py:17-60``:
``paged_kv``, ``decode_reference``, ``prefill_reference``).
"""
from __future__ import annotations

import math

import torch

from .. import _ext, envs
from ..utils import launch_count


# --------------------------------------------------------------------------
# Paged-KV construction and the dense oracles (CPU or GPU, fp32 math)
# --------------------------------------------------------------------------
def build_paged_kv(k: list[torch.Tensor], v: list[torch.Tensor], block_size: int,
                   num_blocks: int | None = None, generator: torch.Generator | None = None,
                   garbage: float = float("nan")):
    """Scatter per-sequence ``k[i], v[i]: [L_i, Hkv, D]`` into a paged cache
    with randomly shuffled physical blocks. Unused slots hold ``garbage`` (NaN
    by default) so any read outside the valid context poisons the output.

    Returns ``(k_cache, v_cache, block_table[int32], seq_lens[int32])``.
    """
    n = len(k)
    hkv, d = k[0].shape[1], k[0].shape[2]
    lens = [int(t.shape[0]) for t in k]
    nblk_per = [max(1, math.ceil(L / block_size)) for L in lens]
    total = sum(nblk_per)
    num_blocks = num_blocks or total + 3
    perm = torch.randperm(num_blocks, generator=generator)[:total]
    dev, dt = k[0].device, k[0].dtype
    kc = torch.full((num_blocks, hkv, block_size, d), garbage, dtype=dt, device=dev)
    vc = torch.full((num_blocks, hkv, block_size, d), garbage, dtype=dt, device=dev)
    max_blocks = max(nblk_per)
    bt = torch.zeros(n, max_blocks, dtype=torch.int32)
    cur = 0
    for i in range(n):
        for b in range(nblk_per[i]):
            phys = int(perm[cur])
            cur += 1
            bt[i, b] = phys
            lo, hi = b * block_size, min((b + 1) * block_size, lens[i])
            if hi > lo:
                kc[phys, :, : hi - lo] = k[i][lo:hi].transpose(0, 1)
                vc[phys, :, : hi - lo] = v[i][lo:hi].transpose(0, 1)
    return kc, vc, bt.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev)


def gather_paged(kc: torch.Tensor, bt_row: torch.Tensor, L: int) -> torch.Tensor:
    """Inverse of :func:`build_paged_kv` for one sequence: ``[L, Hkv, D]``."""
    bs = kc.shape[2]
    nb = math.ceil(L / bs)
    blocks = kc[bt_row[:nb].long()]  # [nb, Hkv, bs, D]
    return blocks.transpose(1, 2).reshape(nb * bs, kc.shape[1], kc.shape[3])[:L]


def attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                  window: int = 0, sinks: torch.Tensor | None = None) -> torch.Tensor:
    """Dense causal GQA attention for ONE sequence, fp32 math.

    ``q [Lq, Hq, D]`` are the last ``Lq`` positions of a context of ``L =
    k.shape[0]`` tokens; returns ``[Lq, Hq, D]`` (fp32)."""
    lq, hq, d = q.shape
    L, hkv, _ = k.shape
    g = hq // hkv
    qf = q.float().transpose(0, 1)                                  # [Hq, Lq, D]
    kf = k.float().repeat_interleave(g, dim=1).transpose(0, 1)       # [Hq, L, D]
    vf = v.float().repeat_interleave(g, dim=1).transpose(0, 1)
    s = (qf @ kf.transpose(1, 2)) * scale                            # [Hq, Lq, L]
    qpos = torch.arange(L - lq, L, device=q.device)[:, None]
    kpos = torch.arange(L, device=q.device)[None, :]
    mask = kpos <= qpos
    if window > 0:
        mask &= kpos > qpos - window
    s = s.masked_fill(~mask[None], float("-inf"))
    if sinks is not None:
        sk = sinks.float()[:, None, None].expand(hq, lq, 1)
        s = torch.cat([s, sk], dim=-1)
        p = torch.softmax(s, dim=-1)[..., :-1]
    else:
        p = torch.softmax(s, dim=-1)
    return (p @ vf).transpose(0, 1)


def sdpa_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Same contract as :func:`attention_ref` (no window / sinks) through
    ``torch.nn.functional.scaled_dot_product_attention`` -- the dense SDPA
    reference of the CPU correctness config."""
    lq, hq, d = q.shape
    L, hkv, _ = k.shape
    g = hq // hkv
    qf = q.float().transpose(0, 1)[None]
    kf = k.float().repeat_interleave(g, dim=1).transpose(0, 1)[None]
    vf = v.float().repeat_interleave(g, dim=1).transpose(0, 1)[None]
    qpos = torch.arange(L - lq, L, device=q.device)[:, None]
    kpos = torch.arange(L, device=q.device)[None, :]
    mask = (kpos <= qpos)[None, None]
    o = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, attn_mask=mask, scale=scale)
    return o[0].transpose(0, 1)


def paged_attention_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        block_table: torch.Tensor, seq_lens: torch.Tensor, cu_q: torch.Tensor,
                        scale: float, window: int = 0,
                        sinks: torch.Tensor | None = None) -> torch.Tensor:
    """CPU/GPU oracle of the paged kernel contract (fp32 out, ``[T, Hq, D]``)."""
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    for s in range(seq_lens.numel()):
        q0, q1 = int(cu_q[s]), int(cu_q[s + 1])
        if q1 == q0:
            continue
        L = int(seq_lens[s])
        k = gather_paged(k_cache, block_table[s], L)
        v = gather_paged(v_cache, block_table[s], L)
        out[q0:q1] = attention_ref(q[q0:q1], k, v, scale, window, sinks)
    return out


# --------------------------------------------------------------------------
# Device ops
# --------------------------------------------------------------------------
def paged_attention(out: torch.Tensor, q: torch.Tensor, k_cache: torch.Tensor,
                    v_cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                    cu_q: torch.Tensor, max_q_len: int, scale: float, window: int = 0,
                    sinks: torch.Tensor | None = None, decode: bool = False,
                    num_splits: int = 1, part_o: torch.Tensor | None = None,
                    part_ml: torch.Tensor | None = None) -> torch.Tensor:
    """``out [T, Hq, D]`` <- paged causal attention of ``q [T, Hq, D]``
    (``q`` may be a strided view into the QKV projection output)."""
    if q.is_cuda and envs.get("VLLM_B200_ATTN"):
        _ext.require()
        torch.ops._b200_C.paged_attention(out, q, k_cache, v_cache, block_table, seq_lens, cu_q,
                                          max_q_len, scale, window, sinks, decode, num_splits,
                                          part_o, part_ml)
        launch_count.add(2 if (decode and num_splits > 1) else 1)
        return out
    out.copy_(paged_attention_ref(q, k_cache, v_cache, block_table, seq_lens, cu_q, scale,
                                  window, sinks).to(out.dtype))
    return out


def rope_cos_sin(rot_dim: int, max_pos: int, theta: float, scaling: dict | None = None,
                 device=None) -> torch.Tensor:
    """``[max_pos, rot_dim]`` fp32: cos in the first half, sin in the second.
    Supports Llama-3 frequency scaling (``rope_type == "llama3"``)."""
    inv = 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim))
    if scaling and scaling.get("rope_type", scaling.get("type")) == "llama3":
        factor = scaling["factor"]
        lo, hi = scaling["low_freq_factor"], scaling["high_freq_factor"]
        old = scaling["original_max_position_embeddings"]
        lo_wl, hi_wl = old / lo, old / hi
        wl = 2 * math.pi / inv
        smooth = (old / wl - lo) / (hi - lo)
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).float().to(device)


def rope_kv_write_ref(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                      k_cache: torch.Tensor, v_cache: torch.Tensor, slots: torch.Tensor,
                      hq: int, hkv: int, q_norm=None, k_norm=None, eps: float = 1e-6) -> None:
    d = k_cache.shape[3]
    bs = k_cache.shape[2]
    t = qkv.shape[0]
    x = qkv.view(t, hq + 2 * hkv, d).float()
    rot = cos_sin.shape[1]
    half = rot // 2
    cs = cos_sin[positions.long()]
    c, s = cs[:, None, :half], cs[:, None, half:]

    def norm(h, w):
        inv = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
        return (h * inv).to(qkv.dtype).float() * w.float()

    q = x[:, :hq]
    k = x[:, hq:hq + hkv]
    if q_norm is not None:
        q = norm(q, q_norm)
    if k_norm is not None:
        k = norm(k, k_norm)

    def rope(h):
        h = h.clone()
        x1, x2 = h[..., :half].clone(), h[..., half:rot].clone()
        h[..., :half] = x1 * c - x2 * s
        h[..., half:rot] = x2 * c + x1 * s
        return h

    q, k = rope(q), rope(k)
    qkv.view(t, hq + 2 * hkv, d)[:, :hq] = q.to(qkv.dtype)
    qkv.view(t, hq + 2 * hkv, d)[:, hq:hq + hkv] = k.to(qkv.dtype)
    v = x[:, hq + hkv:]
    for i in range(t):
        sl = int(slots[i])
        if sl < 0:
            continue
        b, o = sl // bs, sl % bs
        k_cache[b, :, o] = k[i].to(k_cache.dtype)
        v_cache[b, :, o] = v[i].to(v_cache.dtype)


def rope_kv_write(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                  k_cache: torch.Tensor, v_cache: torch.Tensor, slots: torch.Tensor,
                  hq: int, hkv: int, q_norm=None, k_norm=None, eps: float = 1e-6) -> None:
    if qkv.is_cuda and envs.get("VLLM_B200_ROPE_KV"):
        _ext.require()
        torch.ops._b200_C.rope_kv_write(qkv, positions, cos_sin, k_cache, v_cache, slots, hq, hkv,
                                        q_norm, k_norm, eps)
        launch_count.add(1)
        return
    rope_kv_write_ref(qkv, positions, cos_sin, k_cache, v_cache, slots, hq, hkv, q_norm, k_norm,
                      eps)
