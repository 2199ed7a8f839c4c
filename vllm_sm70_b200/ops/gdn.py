"""Gated DeltaNet ops (Qwen3-Next linear-attention layers) and their fp32
torch oracles.

Layer math (per sequence, per v-head h, k-head h // (HV / HK)):
  conv:   x = silu(causal_conv1d([q | k | v]))         (kernel 4, rolling state)
  gates:  g_t = -exp(A_log[h]) * softplus(a_t + dt_bias[h]),  beta_t = sigmoid(b_t)
  norm:   q_t, k_t L2-normalised, q_t *= dk^-1/2
  rule:   S <- exp(g_t) S ;  S <- S + beta_t (v_t - S k_t) k_t^T ;  o_t = S q_t
  out:    o <- rmsnorm(o) * w * silu(z)  per head

Reference parity: ``sm70/vllm_sm70/gdn/kernels.py:201-498`` (FlashQLA route)
and ``sm70/csrc/gdn/gdn_forward.cu`` (varlen token-serial recurrence, decode
with slot-indexed state); the reference's test oracle
``sm70/tests/gdn/_gdn_ref.py``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _ext, envs
from ..utils import launch_count


def causal_conv1d_ref(x, w, bias, state, cu, slots, silu=True):
    """x [T, C], w [C, W], state [slots, C, W-1] (updated in place)."""
    T, C = x.shape
    W = w.shape[1]
    y = torch.empty(T, C, dtype=torch.float32, device=x.device)
    for s in range(len(slots)):
        t0, t1 = int(cu[s]), int(cu[s + 1])
        slot = int(slots[s])
        hist = state[slot].clone() if slot >= 0 else torch.zeros(C, W - 1, device=x.device)
        xs = torch.cat([hist, x[t0:t1].float().t()], dim=1)  # [C, W-1+L]
        for t in range(t1 - t0):
            acc = (xs[:, t:t + W] * w.float()).sum(1)
            if bias is not None:
                acc = acc + bias.float()
            y[t0 + t] = F.silu(acc) if silu else acc
        if slot >= 0:
            state[slot] = xs[:, -(W - 1):]
    return y


def gdn_recurrent_ref(q, k, v, a, b, A_log, dt_bias, state, cu, slots, HK, HV,
                      reset_state=False, has_init=None):
    T = q.shape[0]
    DK = q.shape[1] // HK
    DV = v.shape[1] // HV
    o = torch.empty(T, HV * DV, dtype=torch.float32, device=q.device)
    for s in range(len(slots)):
        t0, t1 = int(cu[s]), int(cu[s + 1])
        slot = int(slots[s])
        fresh = reset_state or (has_init is not None and not bool(has_init[s]))
        for h in range(HV):
            hk = h // (HV // HK)
            S = (torch.zeros(DV, DK, device=q.device) if (slot < 0 or fresh)
                 else state[slot, h].clone())
            for t in range(t0, t1):
                qt = q[t, hk * DK:(hk + 1) * DK].float()
                kt = k[t, hk * DK:(hk + 1) * DK].float()
                qt = qt / (qt.norm() ** 2 + 1e-6).sqrt() * DK ** -0.5
                kt = kt / (kt.norm() ** 2 + 1e-6).sqrt()
                g = -torch.exp(A_log[h]) * F.softplus(a[t, h].float() + dt_bias[h])
                beta = torch.sigmoid(b[t, h].float())
                S = S * torch.exp(g)
                vt = v[t, h * DV:(h + 1) * DV].float()
                S = S + beta * torch.outer(vt - S @ kt, kt)
                o[t, h * DV:(h + 1) * DV] = S @ qt
            if slot >= 0:
                state[slot, h] = S
    return o


def gated_rmsnorm_ref(o, z, w, H, eps):
    T = o.shape[0]
    D = w.numel()
    of = o.float().view(T, H, D)
    inv = torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps)
    n = (of * inv).to(torch.bfloat16).float() * w.float()
    zf = z.float().view(T, H, D)
    return (n * F.silu(zf)).view(T, H * D)


def causal_conv1d(x, w, bias, state, cu, slots, silu=True, out=None, write_state=True):
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        _ext.require()
        torch.ops._b200_C.causal_conv1d(out, x, w, bias, state, cu, slots, silu, write_state)
        launch_count.add(1)
    else:
        st = state if write_state else state.clone()
        out.copy_(causal_conv1d_ref(x, w, bias, st, cu, slots, silu).to(out.dtype))
    return out


def chunk_ok(q, v, HK, HV) -> bool:
    """The chunked (64-token WY/UT) prefill kernel takes head dims 128."""
    return (q.is_cuda and envs.get("VLLM_B200_GDN_CHUNK") and q.shape[1] // HK == 128
            and v.shape[1] // HV == 128)


def gdn_recurrent(q, k, v, a, b, A_log, dt_bias, state, cu, slots, HK, HV, reset_state=False,
                  out=None, write_state=True, chunked=False, has_init=None):
    """Gated delta rule over varlen sequences. ``chunked``: prefill through the
    chunked tensor-core kernel when it takes the shape (same state semantics);
    decode / verify steps stay token-serial.

    ``state`` [slots, HV, DV, DK] fp32 may have padded slots (each slot's block
    dense, as in a paged state cache); ``has_init`` [nseq] bool: sequences with
    False start from a zero state (and still store their final state)."""
    if out is None:
        out = torch.empty(q.shape[0], v.shape[1], dtype=torch.bfloat16, device=q.device)
    if q.is_cuda:
        _ext.require()
        torch.ops._b200_C.gdn_recurrent(out, q, k, v, a, b, A_log, dt_bias, state, cu, slots,
                                        HK, HV, reset_state, write_state,
                                        bool(chunked) and chunk_ok(q, v, HK, HV), has_init)
        launch_count.add(1)
    else:
        st = state if write_state else state.clone()
        out.copy_(gdn_recurrent_ref(q, k, v, a, b, A_log, dt_bias, st, cu, slots, HK, HV,
                                    reset_state, has_init).to(out.dtype))
    return out


def gated_rmsnorm(o, z, w, H, eps):
    """In place on ``o [T, H*D]``."""
    if o.is_cuda:
        _ext.require()
        torch.ops._b200_C.gated_rmsnorm(o, z, w, H, eps)
        launch_count.add(1)
    else:
        o.copy_(gated_rmsnorm_ref(o, z, w, H, eps).to(o.dtype))
    return o
