"""Per-CTA timeline of one tcgen05 GEMM launch (profiling aid).

Installs a device buffer with ``_b200_C::gemm_set_timeline``; the kernel then
stamps %globaltimer at up to sixteen points per CTA (see STAMPS). Prints, relative to the earliest
CTA entry, the median / max over CTAs of each stamp, and the kernel duration
measured with CUDA events around the same launch.

    python -m vllm_sm70_b200.perf.gemm_timeline --M 256 --N 4096 --K 4096 --cfg 1 --splits 2
"""
from __future__ import annotations

import argparse
import json

import torch

STAMPS = ["entry", "setup", "first_tma", "first_stage", "last_mma", "first_acc", "epi_done",
          "exit", "partial_written", "fenced", "staged", "stored", "splits_arrived",
          "bulk_received"]
SLOTS = 16


def run(M: int, N: int, K: int, cfg: int, splits: int, flush: bool = True) -> dict:
    from .. import _ext
    from ..ops import linear

    _ext.require()
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.ops._b200_C.init_device(dev.index)
    linear.configure_workspace(dev.index)
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    buf = torch.zeros(SLOTS * 2 * sms, dtype=torch.int64, device=dev)
    for _ in range(3):
        linear.gemm(a, w, out=out, cfg=cfg, splits=splits)
    fl = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if flush else None
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
    t = buf.view(-1, SLOTS).cpu()
    t = t[t[:, 0] > 0]
    base = int(t[:, 0].min())
    rel = (t - base).double() / 1e3  # us
    res = {"M": M, "N": N, "K": K, "cfg": cfg, "splits": splits, "ctas": int(t.shape[0]),
           "event_us": round(s.elapsed_time(e) * 1e3, 2)}
    for i, name in enumerate(STAMPS):
        col = rel[:, i]
        col = col[t[:, i] > 0]
        if col.numel():
            res[name] = [round(float(col.median()), 2), round(float(col.max()), 2)]
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=256)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--cfg", type=int, default=-1)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--no-flush", action="store_true")
    args = ap.parse_args(argv)
    print(json.dumps(run(args.M, args.N, args.K, args.cfg, args.splits, not args.no_flush)))


if __name__ == "__main__":
    main()
