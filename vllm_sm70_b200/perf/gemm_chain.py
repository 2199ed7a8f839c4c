"""Decode-GEMM chain benchmark.

A decode step runs each GEMM shape once per layer, back to back, with every
layer's weights streaming from HBM and the launches replayed from a CUDA graph.
A single flushed launch timed with events charges the kernel for its launch
and start-up in full; inside the chain the next kernel's prologue overlaps the
previous kernel's tail (programmatic dependent launch), so the per-GEMM cost a
decode step actually pays can differ. This tool measures that cost:

* one chain per GEMM kind (``L`` launches of the same shape, a distinct weight
  tensor per launch), captured in one CUDA graph and replayed;
* the mixed layer chain (qkv, o_proj, gate_up + SiLU*up, down per layer);
* each for the tcgen05 kernels (planner or tuned plans, or explicit plans
  given with ``--plan kind=cfg:splits``) and for the vendor library
  (``torch.mm``, gate_up without the SiLU) on the same buffers.

Shapes default to Llama-3.1-8B at TP1 (hidden 4096, 32 q / 8 kv heads of 128,
intermediate 14336). Prints one JSON line per measurement: microseconds per
GEMM (chain time / L) and the weight-stream rate.

    python -m vllm_sm70_b200.perf.gemm_chain --M 256 [--layers 32] [--sweep kind]
"""
from __future__ import annotations

import argparse
import json

import torch

KINDS = ("qkv", "o", "gate_up", "down")


def shapes(hidden: int = 4096, heads: int = 32, kv_heads: int = 8, head_dim: int = 128,
           inter: int = 14336) -> dict[str, tuple[int, int]]:
    """(N, K) per GEMM kind; gate_up's N counts both halves (interleaved)."""
    return {"qkv": ((heads + 2 * kv_heads) * head_dim, hidden),
            "o": (heads * head_dim, hidden),
            "gate_up": (2 * inter, hidden),
            "down": (hidden, inter)}


class Chain:
    def __init__(self, M: int, layers: int, kinds=KINDS, dev=None, **shape_kw):
        self.M, self.L = M, layers
        self.dev = dev or torch.device("cuda", torch.cuda.current_device())
        self.shp = shapes(**shape_kw)
        self.kinds = kinds
        g = torch.Generator(device=self.dev).manual_seed(0)
        self.w = {k: [torch.randn(*self.shp[k], device=self.dev, dtype=torch.bfloat16,
                                  generator=g).mul_(0.02) for _ in range(layers)]
                  for k in kinds}
        self.x = {k: torch.randn(M, self.shp[k][1], device=self.dev, dtype=torch.bfloat16,
                                 generator=g) for k in kinds}
        self.y = {k: torch.empty(M, self.shp[k][0] // (2 if k == "gate_up" else 1),
                                 device=self.dev, dtype=torch.bfloat16) for k in kinds}
        self.gu = torch.empty(M, self.shp["gate_up"][0], device=self.dev, dtype=torch.bfloat16) \
            if "gate_up" in kinds else None

    def call(self, kind: str, i: int, impl: str, plan=None):
        from ..ops import linear

        x, w, y = self.x[kind], self.w[kind][i], self.y[kind]
        cfg, sp = plan if plan else (-1, 0)
        if impl == "library":
            torch.mm(x, w.t(), out=self.gu if kind == "gate_up" else y)
        elif kind == "gate_up":
            linear.gemm_silu_mul(x, w, out=y, cfg=cfg)
        else:
            linear.gemm(x, w, out=y, cfg=cfg, splits=sp)

    def time(self, kinds, impl: str, plans=None, reps: int = 5) -> float:
        """Microseconds per layer for the chain of ``kinds`` (graph replay)."""
        plans = plans or {}

        def body():
            for i in range(self.L):
                for k in kinds:
                    self.call(k, i, impl, plans.get(k))

        body()
        torch.cuda.synchronize()
        s0 = torch.cuda.Stream()
        s0.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s0):
            body()
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s0):
                body()
        torch.cuda.synchronize()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            g.replay()
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1e3 / reps / self.L
        del g
        return us


def _parse_plans(items) -> dict:
    out = {}
    for it in items or []:
        k, v = it.split("=")
        c, s = v.split(":")
        out[k] = (int(c), int(s))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=256)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--kinds", default=",".join(KINDS))
    ap.add_argument("--plan", action="append", help="kind=cfg:splits (tcgen05 plan override)")
    ap.add_argument("--sweep", default="", help="kind: time every cfg:splits in --cands")
    ap.add_argument("--cands", default="", help="comma list of cfg:splits for --sweep")
    ap.add_argument("--tune", action="store_true", help="run the warm-up tuner on the shapes first")
    ap.add_argument("--no-library", action="store_true")
    args = ap.parse_args()

    from .. import _ext
    from ..ops import linear

    _ext.require()
    dev = torch.cuda.current_device()
    torch.ops._b200_C.init_device(dev)
    linear.configure_workspace(dev)
    kinds = tuple(k for k in args.kinds.split(",") if k)
    ch = Chain(args.M, args.layers, kinds)
    plans = _parse_plans(args.plan)
    if args.tune:
        from ..engine import warmup

        warmup.tune_shapes([(args.M, *ch.shp[k], 1 if k == "gate_up" else 0) for k in kinds])
    peaks_note = {}
    for k in kinds:
        p = plans.get(k)
        N, K = ch.shp[k]
        auto = linear.plan(args.M, N, K, 1 if k == "gate_up" else 0)
        peaks_note[k] = p or auto
    wbytes = {k: ch.shp[k][0] * ch.shp[k][1] * 2 for k in kinds}

    def emit(**r):
        print(json.dumps(r), flush=True)

    if args.sweep:
        k = args.sweep
        for c in args.cands.split(","):
            cfg, sp = (int(v) for v in c.split(":"))
            try:
                us = ch.time((k,), "ours", {k: (cfg, sp)})
            except RuntimeError as ex:  # a plan the shape cannot take
                emit(kind=k, cfg=cfg, splits=sp, error=str(ex)[:120])
                continue
            emit(kind=k, M=args.M, cfg=cfg, splits=sp, us=round(us, 2),
                 weight_gbs=round(wbytes[k] / us / 1e3, 1))
        return
    for impl in ("ours",) + (() if args.no_library else ("library",)):
        tot = 0.0
        for k in kinds:
            us = ch.time((k,), impl, plans)
            tot += us
            emit(impl=impl, kind=k, M=args.M, N=ch.shp[k][0], K=ch.shp[k][1], us=round(us, 2),
                 weight_gbs=round(wbytes[k] / us / 1e3, 1),
                 plan=list(peaks_note[k]) if impl == "ours" else None)
        us = ch.time(kinds, impl, plans)
        emit(impl=impl, kind="layer", M=args.M, us=round(us, 2), sum_of_kinds=round(tot, 2),
             weight_gbs=round(sum(wbytes.values()) / us / 1e3, 1))


if __name__ == "__main__":
    main()
