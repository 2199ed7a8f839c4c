"""Per-CTA timeline of the tcgen05 prefill attention kernel (profiling aid).

Installs a device buffer with ``_b200_C::attn_fa_set_timeline``; every CTA
stamps %globaltimer at entry, set-up done, Q landed (MMA warp), first S
ready (softmax), softmax loop done, O complete, epilogue done and exit
(slots 0-7). Prints the median CTA phase durations, the CTA lifetime split
by key tiles, and how busy the SMs are over the kernel's span.

    python -m vllm_sm70_b200.perf.fa_timeline --seqs 16 --len 1024
"""
from __future__ import annotations

import argparse
import json

import torch

PHASES = [("setup", 0, 1), ("q_landed", 1, 2), ("first_s", 2, 3), ("softmax_loop", 3, 4),
          ("o_done", 4, 5), ("epilogue", 5, 6), ("exit", 6, 7)]


def run(seqs: int, length: int, hq: int = 32, hkv: int = 8, bs: int = 16) -> dict:
    from .. import _ext
    from ..ops import attention as A

    _ext.require()
    dev = torch.device("cuda", torch.cuda.current_device())
    d = 128
    nb_seq = (length + bs - 1) // bs
    nb = seqs * nb_seq
    kc = torch.randn(nb, hkv, bs, d, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.randperm(nb, device=dev, dtype=torch.int32).view(seqs, nb_seq)
    sl = torch.full((seqs,), length, device=dev, dtype=torch.int32)
    cu = torch.arange(seqs + 1, device=dev, dtype=torch.int32) * length
    q = torch.randn(seqs * length, hq, d, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    for _ in range(3):
        A.paged_attention(out, q, kc, vc, bt, sl, cu, length, 0.088, decode=False)
    G = hq // hkv
    n_qt = (length * G + 127) // 128
    ctas = n_qt * seqs * hkv
    buf = torch.zeros(ctas * 64, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    torch.ops._b200_C.attn_fa_set_timeline(buf)
    torch.cuda._sleep(100_000)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    A.paged_attention(out, q, kc, vc, bt, sl, cu, length, 0.088, decode=False)
    e.record()
    torch.cuda.synchronize()
    torch.ops._b200_C.attn_fa_set_timeline(None)
    t = buf.view(ctas, 64).cpu().double()
    t = t[t[:, 0] > 0]
    base = float(t[:, 0].min())
    span = float(t[:, 7].max()) - base
    res = {"seqs": seqs, "len": length, "ctas": int(t.shape[0]),
           "event_us": round(s.elapsed_time(e) * 1e3, 1), "span_us": round(span / 1e3, 1)}
    for name, a, b in PHASES:
        dd = (t[:, b] - t[:, a]) / 1e3
        dd = dd[(t[:, a] > 0) & (t[:, b] > 0)]
        if dd.numel():
            res[name + "_us"] = round(float(dd.median()), 2)
    life = (t[:, 7] - t[:, 0]) / 1e3
    res["cta_life_us_median"] = round(float(life.median()), 2)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    res["sm_busy_frac"] = round(float(life.sum()) / (sms * span / 1e3), 3)
    # Per key tile j < 8 (slot 8 + 7 j + k): k = 2 S issued, 3 PV issued,
    # 4 softmax start (S ready), 5 P buffer free, 6 softmax done.
    def tile(k):
        return t[:, 8 + k::7][:, :8]

    def med(x, ok):
        x = x[ok]
        return round(float(x.median()) / 1e3, 3) if x.numel() else None

    st, en, si, pi = tile(4), tile(6), tile(2), tile(3)
    res["tile_period_us_median"] = med(st[:, 1:] - st[:, :-1], (st[:, 1:] > 0) & (st[:, :-1] > 0))
    # softmax busy per tile, and its wait for the next S (tensor core / loads)
    res["softmax_busy_us"] = med(en - st, (en > 0) & (st > 0))
    res["softmax_wait_next_s_us"] = med(st[:, 1:] - en[:, :-1], (st[:, 1:] > 0) & (en[:, :-1] > 0))
    # MMA issuer: S_j issue -> softmax j start (S latency on the tensor core)
    res["s_issue_to_ready_us"] = med(st - si, (st > 0) & (si > 0))
    # softmax j done -> PV_j issued
    res["p_ready_to_pv_issue_us"] = med(pi - en, (pi > 0) & (en > 0))
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--seqs", type=int, default=16)
    ap.add_argument("--len", type=int, default=1024)
    args = ap.parse_args(argv)
    print(json.dumps(run(args.seqs, args.len)))


if __name__ == "__main__":
    main()
