"""Qwen3-MoE (e.g. Qwen3-30B-A3B): the Llama-style attention block with q/k
RMSNorm and a routed-expert MLP (softmax top-k, renormalised), block-FP8
weights when the checkpoint is FP8.

Parallelism, two layouts:

* TP (the default at TP > 1): attention is tensor-parallel; experts are
  expert-parallel over the same group (rank r owns experts
  [r*E/W, (r+1)*E/W)). Every rank holds every token after the attention
  all-reduce, so the MoE block needs no all-to-all: each rank runs its local
  experts for all tokens and the partial sums ride the fused all-reduce +
  residual + RMSNorm that follows.
* DP attention + EP (``LLM(data_parallel_size=W, enable_expert_parallel=
  True)``): every rank holds the whole attention / dense part and serves its
  own requests; the experts are split over the EP group and the MoE block
  dispatches tokens to the ranks that own their experts and combines the
  results (``parallel/ep.py``).

Reference parity: the Flint MoE block (``sm70/vllm_sm70/models/flint_sm70/
model.py:200-300``) with its fused router and MoE methods; Qwen3-MoE is one
of the supported model families.
"""
from __future__ import annotations

import torch

from ..ops import linear as linear_ops
from ..ops import moe as moe_ops
from .llama import LlamaModel


class Qwen3MoeModel(LlamaModel):
    def __init__(self, cfg, device, dtype=torch.bfloat16, ps=None):
        super().__init__(cfg, device, dtype, ps)
        ps = self.ps
        self.ep_a2a = None
        if ps.ep_size > 1:  # data-parallel attention (TP inside each replica), EP over all ranks
            from ..parallel.ep import EPAllToAll

            self.ep_a2a = EPAllToAll(ps, cfg.num_experts, cfg.top_k)
            n, r = ps.ep_size, ps.ep_rank
        else:
            n, r = ps.tp_size, ps.tp_rank
        assert cfg.num_experts % n == 0, "experts must divide across the EP group"
        self.E_local = cfg.num_experts // n
        self.e_base = r * self.E_local
        self.moe_ws = None
        self.router_sigmoid = False  # softmax top-k scores (sigmoid: Flint)

    def init_mlp_dummy(self, rnd) -> dict:
        cfg = self.cfg
        h, I, E = cfg.hidden_size, cfg.moe_intermediate_size, self.E_local
        fmt = cfg.quant if cfg.quant in ("fp8", "awq", "nvfp4") else "bf16"
        w13 = rnd(E, 2 * I, h)
        w2 = rnd(E, h, I)
        L = {"router": rnd(cfg.num_experts, h).to(self.dtype),
             "experts": moe_ops.ExpertWeights.from_dense(fmt, w13, w2)}
        if cfg.shared_expert_intermediate_size:
            Is = cfg.shared_expert_intermediate_size // self.ps.tp_size
            L["shared_gate_up"] = self.make_gate_up(rnd(Is, h), rnd(Is, h))
            L["shared_down"] = self.make_linear(rnd(h, Is))
            L["shared_gate"] = rnd(1, h).to(self.dtype)
        return L

    def _load_mlp(self, m: str, get_tensor, has, t, qfmt, linear) -> dict:
        """Router ``mlp.gate``, this rank's experts ``mlp.experts.{e}.*`` (bf16,
        block-FP8, AWQ int4 or ModelOpt NVFP4, stacked as loaded) and the
        optional shared expert."""
        cfg = self.cfg
        E, e0 = self.E_local, self.e_base
        L = {"router": t(m + "gate.weight")}
        ex = [f"{m}experts.{e0 + j}." for j in range(E)]
        fmts = {qfmt(x + pr) for x in ex for pr in ("gate_proj", "up_proj", "down_proj")}
        H, I = cfg.hidden_size, cfg.moe_intermediate_size
        if fmts == {"fp8"}:
            def cat(names, scale):
                suffix = ".weight_scale_inv" if scale else ".weight"
                v = [get_tensor(n + suffix) for n in names]
                return torch.cat([x.float() if scale else x for x in v]).to(self.device)

            w13 = cat([x + pr for x in ex for pr in ("gate_proj", "up_proj")], False)
            s13 = cat([x + pr for x in ex for pr in ("gate_proj", "up_proj")], True)
            w2 = cat([x + "down_proj" for x in ex], False)
            s2 = cat([x + "down_proj" for x in ex], True)
            L["experts"] = moe_ops.ExpertWeights(
                "fp8", E, H, I, w13.contiguous().view(torch.uint8),
                w2.contiguous().view(torch.uint8), s13.contiguous(), s2.contiguous())
        elif fmts in ({"awq"}, {"nvfp4"}):
            # per expert: [gate | up] and down as quantised linears, then stacked by rows
            l13 = [linear([(x + "gate_proj", None), (x + "up_proj", None)]) for x in ex]
            l2 = [linear([(x + "down_proj", None)]) for x in ex]
            fmt = fmts.pop()
            if fmt == "awq":
                L["experts"] = moe_ops.ExpertWeights(
                    "awq", E, H, I, torch.cat([a.raw for a in l13]), torch.cat([a.raw for a in l2]),
                    torch.cat([a.scales for a in l13]), torch.cat([a.scales for a in l2]))
            else:
                from ..ops import quant

                w13, s13, g13 = quant.merge_nvfp4_parts([a.raw for a in l13],
                                                        [a.scales for a in l13],
                                                        [a.out_scale for a in l13])
                w2, s2, g2 = quant.merge_nvfp4_parts([a.raw for a in l2], [a.scales for a in l2],
                                                     [a.out_scale for a in l2])
                L["experts"] = moe_ops.ExpertWeights("nvfp4", E, H, I, w13, w2,
                                                     s13.view(torch.uint8), s2.view(torch.uint8),
                                                     g13, g2)
        else:
            w13 = torch.stack([torch.cat([t(x + "gate_proj.weight"), t(x + "up_proj.weight")])
                               for x in ex])
            w2 = torch.stack([t(x + "down_proj.weight") for x in ex])
            L["experts"] = moe_ops.ExpertWeights.from_dense("bf16", w13, w2)
        if cfg.shared_expert_intermediate_size:
            from .llama import _shard

            rows = _shard(cfg.shared_expert_intermediate_size, self.ps.tp_size, self.ps.tp_rank)
            sh = self._load_swiglu(m + "shared_expert.", rows, t, qfmt, linear)
            L["shared_gate_up"], L["shared_down"] = sh["gate_up"], sh["down"]
            if has(m + "shared_expert_gate.weight"):
                L["shared_gate"] = t(m + "shared_expert_gate.weight")
        return L

    def _mlp_state(self, m: str, L: dict) -> dict:
        cfg = self.cfg
        ew = L["experts"]
        assert ew.fmt == "bf16", "export of quantised experts is not supported"
        I, H = cfg.moe_intermediate_size, cfg.hidden_size
        w13 = ew.w13.view(ew.E, 2 * I, H)
        w2 = ew.w2.view(ew.E, H, I)
        sd = {m + "gate.weight": L["router"]}
        for e in range(ew.E):
            x = f"{m}experts.{e}."
            sd[x + "gate_proj.weight"] = w13[e, :I]
            sd[x + "up_proj.weight"] = w13[e, I:]
            sd[x + "down_proj.weight"] = w2[e]
        if "shared_gate_up" in L:
            g, u = linear_ops.deinterleave_gate_up(L["shared_gate_up"].w)
            sd.update({m + "shared_expert.gate_proj.weight": g,
                       m + "shared_expert.up_proj.weight": u,
                       m + "shared_expert.down_proj.weight": L["shared_down"].w})
            if "shared_gate" in L:
                sd[m + "shared_expert_gate.weight"] = L["shared_gate"]
        return sd

    def _ws(self, T: int):
        cfg = self.cfg
        if self.moe_ws is None or self.moe_ws.max_tokens < T:
            n = max(T, 256)
            self.moe_ws = moe_ops.MoEWorkspace(n, cfg.top_k, self.E_local, cfg.hidden_size,
                                               cfg.moe_intermediate_size, self.device)
        return self.moe_ws

    def reserve_workspace(self, max_tokens: int) -> None:
        self._ws(max_tokens)
        if self.ep_a2a is not None:
            self.ep_a2a.reserve(max_tokens, self.cfg.hidden_size)

    def mlp(self, li, L, x, out):
        cfg = self.cfg
        T = x.shape[0]
        ws = self._ws(T) if x.is_cuda else None
        w, ids = moe_ops.route(x, L["router"], cfg.top_k, use_sigmoid=self.router_sigmoid,
                               renorm=cfg.norm_topk_prob, ws=ws)
        shared = None
        if "shared_gate_up" in L:
            sh = L["shared_down"].forward(L["shared_gate_up"].forward(x))
            if "shared_gate" in L:  # sigmoid-gated shared expert (Qwen3-Next)
                gate = torch.sigmoid((x.float() @ L["shared_gate"].float().t()))
                shared = (sh.float() * gate).to(x.dtype)
            else:
                shared = sh
        if self.ep_a2a is not None:
            return self._ep_moe(L, x, w, ids, shared, out)
        return moe_ops.experts_forward(x, w, ids, L["experts"], ws, self.e_base, shared, out)

    # ------------------------------------------------------------------ DP + EP
    def _ep_moe(self, L, x, w, ids, shared, out):
        """Dispatch -> local experts -> combine (data-parallel attention). Rows
        travel in the model dtype on every rank (the idle pass's too), so the
        byte counts of the exchange agree whatever dtype a layer hands in.

        With TP inside the replica (TP x EP), the tokens are replicated over the
        TP group: TP rank r dispatches only its slice [T r / tp, T (r+1) / tp)
        and writes the routed result into those rows of an output that holds
        this rank's shared-expert partial sum (or zero) everywhere; the TP
        all-reduce that follows the block then sums the disjoint slices and the
        shared-expert partials -- it doubles as the all-gather."""
        ep = self.ep_a2a
        dt = x.dtype
        tp, r = self.ps.tp_size, self.ps.tp_rank
        if tp > 1:
            T = x.shape[0]
            lo, hi = T * r // tp, T * (r + 1) // tp
            y = self._ep_exchange(L, x[lo:hi], w[lo:hi], ids[lo:hi], None, None)
            full = out if out is not None else torch.empty(T, self.cfg.hidden_size, dtype=dt,
                                                           device=x.device)
            if shared is not None:
                full.copy_(shared)
            else:
                full.zero_()
            if hi > lo:
                full[lo:hi] += y.to(dt)
            return full
        res = self._ep_exchange(L, x, w, ids, shared, out)
        return res if res.dtype == dt else res.to(dt)

    def _ep_exchange(self, L, x, w, ids, shared, out):
        ep = self.ep_a2a
        xr, wr, idr, plan = ep.dispatch(x.to(self.dtype), w, ids)
        yr = xr.new_empty(xr.shape[0], self.cfg.hidden_size)
        if xr.shape[0]:
            ws = self._ws(xr.shape[0]) if xr.is_cuda else None
            moe_ops.experts_forward(xr, wr, idr, L["experts"], ws, self.e_base, None, yr)
        return ep.combine(yr, plan, shared, out)

    def ep_idle_pass(self) -> None:
        """A forward without local tokens: every MoE block still serves the
        rows the other ranks dispatch to this rank's experts."""
        H, k = self.cfg.hidden_size, self.cfg.top_k
        x = torch.empty(0, H, device=self.device, dtype=self.dtype)
        w = torch.empty(0, k, device=self.device, dtype=torch.float32)
        ids = torch.empty(0, k, device=self.device, dtype=torch.int32)
        for L in self.layers:
            if "experts" in L:
                self._ep_moe(L, x, w, ids, None, None)

    def ep_drain(self) -> None:
        """Keep serving idle passes until no rank of the group has work."""
        if self.ep_a2a is None:
            return
        while self.ep_a2a.step(False) > 0:
            self.ep_idle_pass()

    def weight_bytes(self) -> int:
        n = self.embed.numel() * 2 + (0 if self.cfg.tie_embeddings else self.lm_head.numel() * 2)
        for L in self.layers:
            n += L["qkv"].weight_bytes() + L["o"].weight_bytes() + L["experts"].bytes()
        return n
