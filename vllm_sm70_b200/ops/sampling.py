"""Greedy (argmax) sampling and the vocab-parallel top-1 merge.

Tie order (shared by the kernel, this oracle and the rank merge): NaN first,
then the larger value, then the lower token id. Reference parity:
``sm70/vllm_sm70/sample_greedy.py:74-328`` (per-rank argmax -> all-gather of
(value, id) pairs) and ``sm70/csrc/custom_ar/top1_custom_ar.cu:52-101``.
"""
from __future__ import annotations

import torch

from .. import _ext
from ..utils import launch_count


def argmax_ref(logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    x = logits.float()
    nan = torch.isnan(x)
    has_nan = nan.any(-1)
    # First NaN index for rows with NaN; else the first max index.
    first_nan = torch.where(nan, torch.arange(x.shape[-1], device=x.device), x.shape[-1]).min(-1)
    mx = torch.where(nan, torch.full_like(x, float("-inf")), x).max(-1)
    is_max = torch.where(nan, False, x == mx.values[:, None])
    first_max = torch.where(is_max, torch.arange(x.shape[-1], device=x.device),
                            x.shape[-1]).min(-1).values
    ids = torch.where(has_nan, first_nan.values, first_max).to(torch.int32)
    vals = torch.where(has_nan, torch.full_like(mx.values, float("nan")), mx.values)
    return ids, vals


def argmax(logits: torch.Tensor, id_offset: int = 0,
           ids: torch.Tensor | None = None,
           vals: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    rows = logits.shape[0]
    if ids is None:
        ids = torch.empty(rows, dtype=torch.int32, device=logits.device)
    if vals is None:
        vals = torch.empty(rows, dtype=torch.float32, device=logits.device)
    if logits.is_cuda:
        _ext.require()
        torch.ops._b200_C.argmax(ids, vals, logits, id_offset)
        launch_count.add(1)
    else:
        i, v = argmax_ref(logits)
        ids.copy_(i + id_offset)
        vals.copy_(v)
    return ids, vals


def merge_rank_top1(vals: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """``vals/ids [world, rows]`` (rank order) -> global greedy ids ``[rows]``
    under the same tie order (NaN first, max value, lowest id)."""
    v = vals.float()
    nan = torch.isnan(v)
    key_nan = torch.where(nan, ids.to(torch.int64), torch.iinfo(torch.int64).max)
    any_nan = nan.any(0)
    nan_pick = key_nan.min(0).values
    vm = torch.where(nan, torch.full_like(v, float("-inf")), v)
    mx = vm.max(0).values
    cand = torch.where((vm == mx[None]) & ~nan, ids.to(torch.int64), torch.iinfo(torch.int64).max)
    pick = cand.min(0).values
    return torch.where(any_nan, nan_pick, pick).to(torch.int32)


# ------------------------------------------------------------------ random sampling
def gumbel_sample(logits: torch.Tensor, temperature: torch.Tensor, seeds: torch.Tensor,
                  offset: int, id_offset: int = 0, row_offsets: torch.Tensor | None = None):
    """Exact sample from softmax(logits / T) per row (Gumbel-max with Philox
    noise keyed by (seed, global token id)); T <= 0 rows are greedy. Returns
    (ids int32, perturbed max value) so vocab shards merge with
    :func:`merge_rank_top1`."""
    rows = logits.shape[0]
    ids = torch.empty(rows, dtype=torch.int32, device=logits.device)
    vals = torch.empty(rows, dtype=torch.float32, device=logits.device)
    if not logits.is_cuda:
        # noise keyed like the kernel's: per row by (seed, output position,
        # offset), per column by the GLOBAL token id -- so a request's samples
        # do not depend on its batch row, and vocab shards merge exactly
        x = logits.float()
        t = temperature.float()[:, None]
        V = x.shape[1]
        u = torch.empty_like(x)
        for r in range(rows):
            pos = int(row_offsets[r]) if row_offsets is not None else 0
            key = (int(seeds[r]) * 1000003 + pos * 7919 + int(offset)) & 0x7FFFFFFFFFFFFFFF
            g = torch.Generator().manual_seed(key)
            u[r] = torch.rand(id_offset + V, generator=g)[id_offset:]
        u = u.clamp(1e-12, 1 - 1e-7)
        pert = torch.where(t > 0, x / t.clamp_min(1e-6) - torch.log(-torch.log(u)), x)
        vals.copy_(pert.max(-1).values)
        ids.copy_(pert.argmax(-1).to(torch.int32) + id_offset)
        return ids, vals
    _ext.require()
    torch.ops._b200_C.gumbel_argmax(ids, vals, logits, temperature, seeds, offset, id_offset,
                                    row_offsets)
    launch_count.add(1)
    return ids, vals


def topk_candidates(logits: torch.Tensor, K: int, id_offset: int = 0):
    """Per-row top-K (value desc, id asc) of a logit shard: (vals fp32, ids int32)."""
    rows = logits.shape[0]
    if not logits.is_cuda:
        x = logits.float().nan_to_num(nan=float("-inf"))
        order = torch.sort(-x, dim=-1, stable=True).indices[:, :K]
        return torch.gather(x, 1, order), (order + id_offset).to(torch.int32)
    vals = torch.empty(rows, K, dtype=torch.float32, device=logits.device)
    ids = torch.empty(rows, K, dtype=torch.int32, device=logits.device)
    _ext.require()
    torch.ops._b200_C.topk_candidates(vals, ids, logits, K, id_offset)
    launch_count.add(1)
    return vals, ids


def sample_candidates(cand_v: torch.Tensor, cand_i: torch.Tensor, temperature: torch.Tensor,
                      top_k: torch.Tensor, top_p: torch.Tensor, seeds: torch.Tensor,
                      offset: int) -> torch.Tensor:
    """Temperature / top-k / top-p sampling over merged candidate sets."""
    if not cand_v.is_cuda:
        return sample_candidates_ref(cand_v, cand_i, temperature, top_k, top_p, seeds, offset)
    out = torch.empty(cand_v.shape[0], dtype=torch.int32, device=cand_v.device)
    _ext.require()
    torch.ops._b200_C.sample_candidates(out, cand_v.contiguous(), cand_i.contiguous(),
                                        temperature, top_k, top_p, seeds, offset)
    launch_count.add(1)
    return out


def sample_candidates_ref(cand_v, cand_i, temperature, top_k, top_p, seeds, offset):
    """CPU oracle of :func:`sample_candidates` with the kernel's rules:
    candidates with id < 0 are absent; order by (value desc, id asc);
    T <= 0 -> the first candidate; keep the first ``top_k`` (> 0), then the
    shortest prefix whose softmax(v / T) mass reaches ``top_p``; pick
    argmax p_j / E_j with E_j ~ Exp(1) (torch RNG keyed by (seed, offset)
    instead of Philox)."""
    rows = cand_v.shape[0]
    out = torch.empty(rows, dtype=torch.int32)
    for r in range(rows):
        v = cand_v[r].float()
        ids = cand_i[r].to(torch.int64)
        ok = ids >= 0
        v, ids = v[ok], ids[ok]
        if ids.numel() == 0:
            out[r] = -1
            continue
        order = sorted(range(ids.numel()), key=lambda j: (-float(v[j]), int(ids[j])))
        v, ids = v[order], ids[order]
        t = float(temperature[r])
        if t <= 0:
            out[r] = int(ids[0])
            continue
        k = int(top_k[r])
        kk = min(k, ids.numel()) if k > 0 else ids.numel()
        p = torch.exp((v[:kk] - v[0]) / t)
        csum = torch.cumsum(p, 0)
        hit = (csum >= float(top_p[r]) * float(csum[-1])).nonzero()
        keep = int(hit[0]) + 1 if hit.numel() else kk
        g = torch.Generator().manual_seed((int(seeds[r]) * 1000003 + int(offset)) & 0x7FFFFFFFFFFFFFFF)
        e = torch.empty(keep).exponential_(generator=g)
        out[r] = int(ids[int(torch.argmax(p[:keep] / e))])
    return out.to(cand_v.device)


def rejection_sample(target_logits: torch.Tensor, draft_logits: torch.Tensor,
                     draft_ids: torch.Tensor, temperature: torch.Tensor, seeds: torch.Tensor,
                     offset: int):
    """Verify ``k`` draft tokens per row. Returns (out_tokens [rows, k+1] with
    -1 padding, num_out [rows]) -- accepted drafts plus one corrected / bonus
    token."""
    rows, k = draft_ids.shape
    if not target_logits.is_cuda:
        return rejection_sample_ref(target_logits, draft_logits, draft_ids, temperature, seeds,
                                    offset)
    out = torch.empty(rows, k + 1, dtype=torch.int32, device=draft_ids.device)
    n = torch.empty(rows, dtype=torch.int32, device=draft_ids.device)
    _ext.require()
    torch.ops._b200_C.rejection_sample(out, n, target_logits.contiguous(),
                                       draft_logits.contiguous(), draft_ids.contiguous(),
                                       temperature, seeds, offset)
    launch_count.add(1)
    return out, n


def rejection_sample_ref(target_logits, draft_logits, draft_ids, temperature, seeds, offset):
    """CPU oracle with the same acceptance rule (torch RNG instead of Philox)."""
    rows, k = draft_ids.shape
    out = torch.full((rows, k + 1), -1, dtype=torch.int32)
    n = torch.zeros(rows, dtype=torch.int32)
    for r in range(rows):
        T = float(temperature[r])
        g = torch.Generator().manual_seed((int(seeds[r]) * 1000003 + int(offset)) % (1 << 63))
        e = 0
        for i in range(k + 1):
            tl = target_logits[r, i].float()
            if T <= 0:
                am = int(tl.argmax())
                out[r, e] = am
                e += 1
                if i == k or am != int(draft_ids[r, i]):
                    break
                continue
            p = torch.softmax(tl / T, -1)
            if i == k:
                out[r, e] = int(torch.multinomial(p, 1, generator=g))
                e += 1
                break
            q = torch.softmax(draft_logits[r, i].float() / T, -1)
            d = int(draft_ids[r, i])
            if float(torch.rand(1, generator=g)) * float(q[d]) <= float(p[d]):
                out[r, e] = d
                e += 1
                continue
            res = (p - q).clamp_min(0)
            out[r, e] = int(torch.multinomial(res / res.sum(), 1, generator=g)) if res.sum() > 0 else d
            e += 1
            break
        n[r] = e
    return out, n
