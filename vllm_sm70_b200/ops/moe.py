"""Mixture-of-experts: router top-k, expert-sorted permutation, grouped
tcgen05 expert GEMMs (bf16 or weight-only FP8 / AWQ / NVFP4 with the
dequantisation fused in the producer), SiLU*up, weighted combine.

Expert parallelism: a rank owns experts ``[e_base, e_base + E_local)``; every
rank holds every token (attention is tensor-parallel), so the rank computes
its local experts for all tokens and the partial outputs are summed by the
row-parallel all-reduce that the model already fuses with the next residual
add + RMSNorm. Nothing in the data path depends on host-side counts, so the
whole block is CUDA-graph capturable.

Reference parity: MoE methods and routing runtime
(``sm70/vllm_sm70/fused_moe/method.py:56-416``), FP8 / NVFP4 MoE methods
(``quant/fp8_moe.py``, ``quant/nvfp4_moe.py``), the fused router (K13,
``router.py``) and the decode MoE kernels (K12). The reference refuses EP
(``method.py:357-358``); here EP over the TP group is the default at TP > 1.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _ext, envs
from ..utils import launch_count
from . import linear as _lin
from . import quant as _q

FMT = {"bf16": 0, "fp8": 1, "awq": 2, "nvfp4": 3}


def topk_ref(logits: torch.Tensor, k: int, use_sigmoid: bool = False, renorm: bool = True):
    x = logits.float().nan_to_num(nan=float("-inf"))
    sc = torch.sigmoid(x) if use_sigmoid else torch.softmax(x, -1)
    sc = sc.nan_to_num(nan=0.0)
    # ties -> lower expert id: stable sort on (-score, id)
    order = torch.sort(-sc, dim=-1, stable=True).indices[:, :k]
    w = torch.gather(sc, 1, order)
    if renorm:
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-20)
    return w, order.to(torch.int32)


def topk(logits: torch.Tensor, k: int, use_sigmoid: bool = False, renorm: bool = True,
         bias: torch.Tensor | None = None, w: torch.Tensor | None = None,
         ids: torch.Tensor | None = None):
    T = logits.shape[0]
    if w is None:
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    if ids is None:
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        _ext.require()
        torch.ops._b200_C.moe_topk(w, ids, logits, k, use_sigmoid, renorm, bias)
        launch_count.add(1)
    else:
        ww, ii = topk_ref(logits if bias is None else logits, k, use_sigmoid, renorm)
        w.copy_(ww)
        ids.copy_(ii)
    return w, ids


def router_ref(x: torch.Tensor, wr: torch.Tensor, k: int, use_sigmoid: bool = False,
               renorm: bool = True):
    """fp32 router logits and the top-k selection (oracle of :func:`route`)."""
    return topk_ref(x.float() @ wr.float().t(), k, use_sigmoid, renorm)


def route(x: torch.Tensor, wr: torch.Tensor, k: int, use_sigmoid: bool = False,
          renorm: bool = True, ws: "MoEWorkspace | None" = None):
    """Router logits ``x @ wr^T`` and the top-k experts per token: (weights
    fp32 [T, k], ids int32 [T, k]). Up to ``VLLM_B200_FUSED_ROUTER_MAX_TOKENS``
    tokens (decode steps) one fused kernel computes fp32 logits and selects;
    larger batches run the tcgen05 GEMM (bf16 logits) and the top-k kernel.
    Reference parity: the fused router (``sm70/csrc/router/flint_router.cuh:
    1-186``)."""
    T = x.shape[0]
    w = ws.w[:T] if ws is not None else None
    ids = ws.ids[:T] if ws is not None else None
    if not x.is_cuda:
        ww, ii = router_ref(x, wr, k, use_sigmoid, renorm)
        return ww, ii
    if (ws is not None and envs.get("VLLM_B200_FUSED_ROUTER")
            and 0 < T <= envs.get("VLLM_B200_FUSED_ROUTER_MAX_TOKENS") and T <= ws.max_tokens
            and x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.shape[1] * 16 <= 96 * 1024):
        _ext.require()
        lg, ctr = ws.router_buffers(wr.shape[0])
        torch.ops._b200_C.moe_router(w, ids, x, wr.contiguous(), k, use_sigmoid, renorm, None,
                                     lg, ctr)
        launch_count.add(1)
        return w, ids
    logits = _lin.gemm(x, wr)
    return topk(logits, k, use_sigmoid=use_sigmoid, renorm=renorm, w=w, ids=ids)


@dataclass
class ExpertWeights:
    """Stacked per-expert weights: w13 [E*2I, H] ([gate | up] rows per expert)
    and w2 [E*H, I], bf16 or raw quantised bytes with stacked scales."""
    fmt: str
    E: int
    H: int
    I: int
    w13: torch.Tensor
    w2: torch.Tensor
    s13: torch.Tensor | None = None
    s2: torch.Tensor | None = None
    g13: float = 1.0
    g2: float = 1.0

    @classmethod
    def from_dense(cls, fmt: str, w13: torch.Tensor, w2: torch.Tensor):
        """w13 [E, 2I, H], w2 [E, H, I] dense (fp32/bf16) -> stacked format."""
        E, I2, H = w13.shape
        I = I2 // 2
        if fmt == "bf16":
            return cls(fmt, E, H, I, w13.reshape(E * I2, H).to(torch.bfloat16).contiguous(),
                       w2.reshape(E * H, I).to(torch.bfloat16).contiguous())
        l13 = _q.make_linear(fmt, w13.reshape(E * I2, H))
        l2 = _q.make_linear(fmt, w2.reshape(E * H, I))
        return cls(fmt, E, H, I, l13.raw, l2.raw, l13.scales, l2.scales, l13.out_scale,
                   l2.out_scale)

    def dense_ref(self) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 [E, 2I, H], [E, H, I] of what the kernels compute with."""
        if self.fmt == "bf16":
            return (self.w13.float().view(self.E, 2 * self.I, self.H),
                    self.w2.float().view(self.E, self.H, self.I))
        a = _wrap(self.fmt, self.w13, self.s13, self.g13, self.E * 2 * self.I, self.H)
        b = _wrap(self.fmt, self.w2, self.s2, self.g2, self.E * self.H, self.I)
        return (a.reference_weight().view(self.E, 2 * self.I, self.H),
                b.reference_weight().view(self.E, self.H, self.I))

    def nvfp4_atoms(self):
        """Block scales of w13 / w2 in the tensor-core atom order (cached; not
        stored while a CUDA graph is captured -- captured kernels do not run,
        so such a cache would be garbage for later eager calls)."""
        if getattr(self, "_atoms", None) is None:
            atoms = (_q.nvfp4_sf_atoms(self.s13.view(torch.uint8)),
                     _q.nvfp4_sf_atoms(self.s2.view(torch.uint8)))
            if self.s13.is_cuda and torch.cuda.is_current_stream_capturing():
                return atoms
            self._atoms = atoms
        return self._atoms

    def bytes(self) -> int:
        n = self.w13.numel() * self.w13.element_size() + self.w2.numel() * self.w2.element_size()
        for s in (self.s13, self.s2):
            if s is not None:
                n += s.numel() * s.element_size()
        return n


def _w4a4(ew) -> bool:
    return (ew.fmt == "nvfp4" and _q.w4a4_enabled() and ew.H % 256 == 0 and ew.I % 256 == 0
            and (2 * ew.I) % 128 == 0 and ew.H % 128 == 0)


def _wrap(fmt, raw, scales, gscale, N, K):
    obj = object.__new__({"fp8": _q.Fp8BlockLinear, "awq": _q.AwqLinear,
                          "nvfp4": _q.Nvfp4Linear}[fmt])
    obj.raw, obj.scales, obj.out_scale = raw, scales, gscale
    obj.out_features, obj.in_features = N, K
    return obj


class MoEWorkspace:
    """Persistent per-forward buffers sized for ``max_tokens`` (graph-safe)."""

    def __init__(self, max_tokens: int, k: int, E_local: int, H: int, I: int, device):
        P = max_tokens * k
        i32 = dict(dtype=torch.int32, device=device)
        self.max_tokens, self.k = max_tokens, k
        self.w = torch.empty(max_tokens, k, dtype=torch.float32, device=device)
        self.ids = torch.empty(max_tokens, k, **i32)
        self.counts = torch.empty(E_local, **i32)
        self.offsets = torch.empty(E_local + 1, **i32)
        self.tile_off = torch.empty(E_local + 1, **i32)
        self.rank = torch.empty(P, **i32)
        self.pos = torch.empty(max_tokens, k, **i32)
        self.src = torch.empty(P, **i32)
        self.x_perm = torch.empty(P, H, dtype=torch.bfloat16, device=device)
        self.h = torch.empty(P, 2 * I, dtype=torch.bfloat16, device=device)
        self.act = torch.empty(P, I, dtype=torch.bfloat16, device=device)
        self.y = torch.empty(P, H, dtype=torch.bfloat16, device=device)
        self.P, self.H, self.I = P, H, I
        self.E_local = E_local
        self._fp8 = None
        self._fp4 = None

    def router_buffers(self, E: int):
        """fp32 logits scratch [max_tokens, E] and the per-tile arrival
        counters of the fused router (zero; the kernel leaves them zero)."""
        if getattr(self, "_rt", None) is None or self._rt[0].shape[1] != E:
            dev = self.w.device
            self._rt = (torch.empty(self.max_tokens, E, dtype=torch.float32, device=dev),
                        torch.zeros((self.max_tokens + 7) // 8, dtype=torch.int32, device=dev))
        return self._rt

    def nvfp4_buffers(self):
        """Padded-permutation buffers for the W4A4 grouped GEMMs (every expert's
        rows start at a multiple of 128): rows P + E * 127."""
        if self._fp4 is None:
            dev = self.x_perm.device
            Pp = self.P + self.E_local * 127
            H, I = self.H, self.I
            bf = dict(dtype=torch.bfloat16, device=dev)
            u8 = dict(dtype=torch.uint8, device=dev)
            f32 = dict(dtype=torch.float32, device=dev)
            self._fp4 = dict(
                Pp=Pp, x=torch.empty(Pp, H, **bf), h=torch.empty(Pp, 2 * I, **bf),
                act=torch.empty(Pp, I, **bf), y=torch.empty(Pp, H, **bf),
                src=torch.empty(Pp, dtype=torch.int32, device=dev),
                xq=torch.empty(Pp, H // 2, **u8),
                xsf=torch.empty((Pp + 127) // 128 * (H // 64) * 512, **u8),
                xrs=torch.empty(Pp, **f32),
                aq=torch.empty(Pp, I // 2, **u8),
                asf=torch.empty((Pp + 127) // 128 * (I // 64) * 512, **u8),
                ars=torch.empty(Pp, **f32))
        return self._fp4

    def fp8_buffers(self):
        """e4m3 activation rows and their K-group-major scales for the W8A8
        expert GEMMs (allocated on first use, kept for later forwards)."""
        if self._fp8 is None:
            dev = self.x_perm.device
            ld = max(4, (self.P + 3) // 4 * 4)
            self._fp8 = (torch.empty(self.P, self.H, dtype=torch.uint8, device=dev),
                         torch.empty((self.H + 127) // 128, ld, dtype=torch.float32, device=dev),
                         torch.empty(self.P, self.I, dtype=torch.uint8, device=dev),
                         torch.empty((self.I + 127) // 128, ld, dtype=torch.float32, device=dev))
        return self._fp8


def experts_forward_ref(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, ew: ExpertWeights,
                        e_base: int = 0) -> torch.Tensor:
    """fp32 oracle of the routed experts (local experts only)."""
    w13, w2 = ew.dense_ref()
    T, k = ids.shape
    out = torch.zeros(T, ew.H, dtype=torch.float32, device=x.device)
    if _w4a4(ew):
        # W4A4: exact e2m1 x e4m3 weights times the global scales, and both GEMM
        # inputs through the per-token NVFP4 activation quantisation.
        w13 = (_wrap("nvfp4", ew.w13, ew.s13, 1.0, ew.E * 2 * ew.I, ew.H).exact_weight()
               * ew.g13).view(ew.E, 2 * ew.I, ew.H)
        w2 = (_wrap("nvfp4", ew.w2, ew.s2, 1.0, ew.E * ew.H, ew.I).exact_weight()
              * ew.g2).view(ew.E, ew.H, ew.I)
        xf = _q.nvfp4_act_dequant_ref(x)
        for t in range(T):
            for j in range(k):
                e = int(ids[t, j]) - e_base
                if e < 0 or e >= ew.E:
                    continue
                # The kernels round h to bf16 before SiLU*up (the GEMM output).
                h = (w13[e] @ xf[t]).to(torch.bfloat16).float()
                g, u = h[: ew.I], h[ew.I:]
                a = (g * torch.sigmoid(g) * u).to(torch.bfloat16)
                out[t] += float(w[t, j]) * (w2[e] @ _q.nvfp4_act_dequant_ref(a[None])[0])
        return out
    w8a8 = ew.fmt == "fp8" and _q.w8a8_enabled()
    if w8a8:
        # W8A8: exact dequantised weights, and both GEMM inputs go through the
        # per-token, 128-group e4m3 activation quantisation.
        w13 = _wrap("fp8", ew.w13, ew.s13, 1.0, ew.E * 2 * ew.I, ew.H).exact_weight()
        w13 = w13.view(ew.E, 2 * ew.I, ew.H)
        w2 = _wrap("fp8", ew.w2, ew.s2, 1.0, ew.E * ew.H, ew.I).exact_weight()
        w2 = w2.view(ew.E, ew.H, ew.I)
        xf = _q.fp8_act_dequant_ref(x)
    else:
        xf = x.float()
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j]) - e_base
            if e < 0 or e >= ew.E:
                continue
            h = w13[e] @ xf[t]
            g, u = h[: ew.I], h[ew.I:]
            a = (g * torch.sigmoid(g) * u).to(torch.bfloat16)
            a = _q.fp8_act_dequant_ref(a[None])[0] if w8a8 else a.float()
            out[t] += float(w[t, j]) * (w2[e] @ a)
    return out


def experts_forward(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, ew: ExpertWeights,
                    ws: MoEWorkspace, e_base: int = 0, shared: torch.Tensor | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts for tokens ``x [T, H]`` with routing ``(w, ids) [T, k]``;
    only experts ``[e_base, e_base + ew.E)`` are computed here. ``shared``
    (same shape as the output) is added in the combine."""
    T, k = ids.shape
    if out is None:
        out = torch.empty(T, ew.H, dtype=x.dtype, device=x.device)
    if not x.is_cuda:
        r = experts_forward_ref(x, w, ids, ew, e_base)
        if shared is not None:
            r = r + shared.float()
        out.copy_(r.to(out.dtype))
        return out
    _ext.require()
    ops = torch.ops._b200_C
    P = T * k
    xp, h, act, y = ws.x_perm[:P], ws.h[:P], ws.act[:P], ws.y[:P]
    pos = ws.pos[:T]
    ops.moe_permute(ids, ew.E, e_base, x, xp, ws.counts, ws.offsets, ws.rank, pos, ws.src)
    fmt = FMT[ew.fmt]
    if _w4a4(ew):
        # W4A4 grouped GEMMs on kind::mxf4nvf4: a padded permutation (expert
        # blocks start at multiples of 128 rows) so the activation scale atoms
        # of a 128-row token tile belong to one expert.
        b = ws.nvfp4_buffers()
        Pp = P + ew.E * 127
        xpp, hp, ap, yp = b["x"][:Pp], b["h"][:Pp], b["act"][:Pp], b["y"][:Pp]
        ops.moe_permute(ids, ew.E, e_base, x, xpp, ws.counts, ws.offsets, ws.rank, pos,
                        b["src"][:Pp], 128)
        s13, s2 = ew.nvfp4_atoms()
        used = ws.offsets[ew.E:ew.E + 1]  # padded rows in use (device)
        ops.quant_nvfp4_act(xpp, b["xq"][:Pp], b["xsf"], b["xrs"], used)
        ops.gemm_nvfp4_grouped_out(hp, b["xq"][:Pp], b["xsf"], b["xrs"], ew.w13, s13, ew.g13,
                                   ew.E, 2 * ew.I, ws.offsets, ws.tile_off)
        ops.silu_mul(ap, hp, 0, used)
        ops.quant_nvfp4_act(ap, b["aq"][:Pp], b["asf"], b["ars"], used)
        ops.gemm_nvfp4_grouped_out(yp, b["aq"][:Pp], b["asf"], b["ars"], ew.w2, s2, ew.g2,
                                   ew.E, ew.H, ws.offsets, ws.tile_off)
        ops.moe_combine(out, yp, pos, w, shared, 1.0)
        launch_count.add(9)
        return out
    if ew.fmt == "fp8" and _q.w8a8_enabled():
        # W8A8 grouped GEMMs on kind::f8f6f4 with per-K-block scale promotion.
        xq, sa1, aq, sa2 = ws.fp8_buffers()
        ops.quant_fp8_act(xp, xq[:P], sa1)
        ops.gemm_fp8_grouped_out(h, xq[:P], sa1, ew.w13, ew.s13, ew.E, 2 * ew.I, ws.offsets,
                                 ws.tile_off, 0)
        ops.silu_mul(act, h)
        ops.quant_fp8_act(act, aq[:P], sa2)
        ops.gemm_fp8_grouped_out(y, aq[:P], sa2, ew.w2, ew.s2, ew.E, ew.H, ws.offsets,
                                 ws.tile_off, 0)
        launch_count.add(2)
    else:
        ops.gemm_grouped_out(h, xp, ew.w13, ew.E, 2 * ew.I, ws.offsets, ws.tile_off, fmt,
                             ew.s13, ew.g13, 0)
        ops.silu_mul(act, h)
        ops.gemm_grouped_out(y, act, ew.w2, ew.E, ew.H, ws.offsets, ws.tile_off, fmt, ew.s2,
                             ew.g2, 0)
    ops.moe_combine(out, y, pos, w, shared, 1.0)
    launch_count.add(8)  # count, offsets, scatter, 2x(tiles + GEMM), silu, combine
    return out


class TopKRoute:
    """Route of one vLLM MoE layer on the B200 top-k kernel: softmax or
    sigmoid scores, optional per-expert correction bias, top-k with ties to
    the lower expert id, optional renormalisation (``moe_topk``)."""

    def __init__(self, top_k: int, renorm: bool, use_sigmoid: bool, bias=None):
        self.top_k, self.renorm, self.use_sigmoid, self.bias = top_k, renorm, use_sigmoid, bias

    def try_route(self, hidden_states, router_logits=None):
        if router_logits is None or not router_logits.is_cuda or router_logits.dim() != 2:
            return None
        lg = router_logits
        if lg.dtype not in (torch.float32, torch.bfloat16):
            lg = lg.float()
        return topk(lg.contiguous(), self.top_k, self.use_sigmoid, self.renorm, self.bias)


def make_route_for_runner(runner):
    """U3 provider hook: a :class:`TopKRoute` for a vLLM ``MoERunner`` whose
    router is plain (fused) top-k over softmax / sigmoid scores without EPLB,
    grouped top-k or custom routing; ``None`` keeps vLLM's routing. Layers of
    this library's own models carry ``b200_route`` already."""
    if getattr(runner, "b200_route", None) is not None:
        return runner.b200_route
    router = getattr(runner, "router", None)
    if router is None or type(router).__name__ not in ("FusedTopKRouter", "FusedTopKBiasRouter"):
        return None
    if getattr(router, "eplb_state", None) is not None and getattr(
            router.eplb_state, "logical_to_physical_map", None) is not None:
        return None
    scoring = str(getattr(router, "scoring_func", "softmax"))
    if scoring not in ("softmax", "sigmoid"):
        return None
    k = int(getattr(router, "top_k", 0))
    if not 1 <= k <= 16:
        return None
    bias = getattr(router, "e_score_correction_bias", None)
    if bias is not None:
        bias = bias.float().contiguous()
    return TopKRoute(k, bool(getattr(router, "renormalize", True)), scoring == "sigmoid", bias)
