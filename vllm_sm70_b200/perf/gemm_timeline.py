"""Per-CTA timeline of tcgen05 GEMM launches (profiling aid).

Installs a device buffer with ``_b200_C::gemm_set_timeline``; the kernel then
stamps %globaltimer at up to sixteen points per CTA (see STAMPS), one row per
CTA and launch (``TL_CTAS`` launch counters, then ``TL_SEQS`` x ``TL_CTAS``
rows). Single launch: prints, relative to the earliest CTA entry, the median /
max over CTAs of each stamp, and the kernel duration measured with CUDA events
around the same launch. ``--chain L``: L back-to-back launches of the same
shape, each with its own weight tensor (as the layers of a decode step), and
per launch the span from its first CTA entry to its last CTA exit, the gap to
the previous launch's last exit (negative: overlapped by programmatic
dependent launch) and the median stamps relative to the launch's first entry.

    python -m vllm_sm70_b200.perf.gemm_timeline --M 256 --N 4096 --K 4096 --cfg 1 --splits 2
    python -m vllm_sm70_b200.perf.gemm_timeline --M 256 --N 6144 --K 4096 --chain 8
"""
from __future__ import annotations

import argparse
import json

import torch

STAMPS = ["entry", "setup", "first_tma", "first_stage", "last_mma", "first_acc", "epi_done",
          "exit", "partial_written", "fenced", "staged", "stored", "splits_arrived",
          "bulk_received"]
SLOTS = 16
TL_CTAS = 256
TL_SEQS = 64


def _setup(M, N, K, layers):
    from .. import _ext
    from ..ops import linear

    _ext.require()
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.ops._b200_C.init_device(dev.index)
    linear.configure_workspace(dev.index)
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    ws = [torch.randn(N, K, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    buf = torch.zeros(TL_CTAS + TL_SEQS * TL_CTAS * SLOTS, dtype=torch.int64, device=dev)
    return linear, a, ws, out, buf


def _rows(buf: torch.Tensor, seq: int) -> torch.Tensor:
    t = buf[TL_CTAS:].view(TL_SEQS, TL_CTAS, SLOTS)[seq].cpu()
    return t[t[:, 0] > 0]


def _stamps(t: torch.Tensor, base: int) -> dict:
    res = {}
    rel = (t - base).double() / 1e3  # us
    for i, name in enumerate(STAMPS):
        col = rel[:, i][t[:, i] > 0]
        if col.numel():
            res[name] = [round(float(col.median()), 2), round(float(col.max()), 2)]
    return res


def run(M: int, N: int, K: int, cfg: int, splits: int, flush: bool = True) -> dict:
    linear, a, ws, out, buf = _setup(M, N, K, 1)
    w = ws[0]
    for _ in range(3):
        linear.gemm(a, w, out=out, cfg=cfg, splits=splits)
    fl = torch.empty(256 << 20, dtype=torch.uint8, device=a.device) if flush else None
    if fl is not None:
        fl.fill_(1)
        fl.sum()
    torch.cuda.synchronize()
    torch.ops._b200_C.gemm_set_timeline(buf)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    linear.gemm(a, w, out=out, cfg=cfg, splits=splits)
    e.record()
    torch.cuda.synchronize()
    torch.ops._b200_C.gemm_set_timeline(None)
    t = _rows(buf, 0)
    res = {"M": M, "N": N, "K": K, "cfg": cfg, "splits": splits, "ctas": int(t.shape[0]),
           "event_us": round(s.elapsed_time(e) * 1e3, 2)}
    res.update(_stamps(t, int(t[:, 0].min())))
    return res


def run_chain(M: int, N: int, K: int, cfg: int, splits: int, layers: int) -> dict:
    layers = min(layers, TL_SEQS)
    linear, a, ws, out, buf = _setup(M, N, K, layers)
    for w in ws:
        linear.gemm(a, w, out=out, cfg=cfg, splits=splits)
    torch.cuda.synchronize()
    torch.ops._b200_C.gemm_set_timeline(buf)
    torch.cuda._sleep(200_000)  # the host enqueues the whole chain before it starts
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for w in ws:
        linear.gemm(a, w, out=out, cfg=cfg, splits=splits)
    e.record()
    torch.cuda.synchronize()
    torch.ops._b200_C.gemm_set_timeline(None)
    launches = []
    prev_end = None
    for q in range(layers):
        t = _rows(buf, q)
        if not t.shape[0]:
            continue
        start = int(t[:, 0].min())
        end = int(t[:, 7].max())
        d = {"launch": q, "ctas": int(t.shape[0]), "span_us": round((end - start) / 1e3, 2),
             "gap_us": None if prev_end is None else round((start - prev_end) / 1e3, 2)}
        d.update(_stamps(t, start))
        launches.append(d)
        prev_end = end
    steady = launches[1:] or launches
    med = lambda xs: sorted(xs)[len(xs) // 2]  # noqa: E731
    return {"M": M, "N": N, "K": K, "cfg": cfg, "splits": splits, "layers": layers,
            "event_us_per_launch": round(s.elapsed_time(e) * 1e3 / layers, 2),
            "span_us_median": med([x["span_us"] for x in steady]),
            "gap_us_median": med([x["gap_us"] for x in steady if x["gap_us"] is not None] or [0]),
            "launches": launches}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=256)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--cfg", type=int, default=-1)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--no-flush", action="store_true")
    ap.add_argument("--chain", type=int, default=0, help="launches in a back-to-back chain")
    ap.add_argument("--brief", action="store_true", help="chain: launches 1-3 only")
    args = ap.parse_args(argv)
    if args.chain:
        r = run_chain(args.M, args.N, args.K, args.cfg, args.splits, args.chain)
        if args.brief:
            r["launches"] = r["launches"][1:4]
        print(json.dumps(r))
    else:
        print(json.dumps(run(args.M, args.N, args.K, args.cfg, args.splits, not args.no_flush)))


if __name__ == "__main__":
    main()
