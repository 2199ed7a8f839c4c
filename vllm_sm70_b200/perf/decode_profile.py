"""Decode-step (or prefill-chunk) driver for a per-kernel breakdown of the serving loop.

Builds the engine on random-init Llama-3.1-8B weights, prefills ``--requests``
prompts of ``--prompt-len`` tokens and runs ``--decode-steps`` batched decode
steps inside an NVTX range named ``decode`` (eager launches, so a profiler sees
every kernel of the step as its own launch); every prefill chunk runs inside a
range named ``prefill``. Prints the decode milliseconds per step measured with
CUDA events. Under a one-metric launch list:

    ncu --nvtx --nvtx-include "decode/" --metrics gpu__time_duration.sum \\
        --clock-control none --csv --log-file launches.csv \\
        python -m vllm_sm70_b200.perf.decode_profile

then ``python -m vllm_sm70_b200.perf.decode_profile --summarize launches.csv``
groups the captured launches by kernel and prints each one's share. With
``--nvtx-include "prefill/"`` (and ``--summarize ... --per prefill-chunks``
set to the number of chunks captured) the same list covers prefill chunks.
"""
from __future__ import annotations

import argparse
import csv
import json
import re
from collections import defaultdict


def summarize(path: str, steps: int) -> list[dict]:
    rows = []
    with open(path) as f:
        lines = [ln for ln in f if ln.startswith('"')]
    for r in csv.DictReader(lines):
        if r.get("Metric Name") != "gpu__time_duration.sum":
            continue
        v = float(r["Metric Value"].replace(",", ""))
        unit = r.get("Metric Unit", "ns")
        us = v / 1e3 if unit == "nsecond" or unit == "ns" else v if unit == "usecond" else v * 1e3
        name = r["Kernel Name"]
        name = re.sub(r"\(.*", "", name)
        name = re.sub(r"^void ", "", name)
        rows.append((name, us))
    agg = defaultdict(lambda: [0, 0.0])
    for n, us in rows:
        agg[n][0] += 1
        agg[n][1] += us
    total = sum(v[1] for v in agg.values())
    out = []
    for n, (c, us) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        out.append({"kernel": n[:110], "launches_per_step": round(c / steps, 1),
                    "us_per_step": round(us / steps, 1), "share": round(us / total, 4)})
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--decode-steps", type=int, default=2)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--summarize", default=None, help="launch-list CSV to group by kernel")
    args = ap.parse_args(argv)
    if args.summarize:
        for r in summarize(args.summarize, args.decode_steps):
            print(json.dumps(r))
        return

    import torch

    from ..engine import LLM, SamplingParams

    R, P, S = args.requests, args.prompt_len, args.decode_steps
    llm = LLM("llama-3.1-8b", max_num_seqs=R, max_model_len=P + S + 1,
              block_size=args.block_size, max_num_batched_tokens=16384, load_format="dummy",
              seed=0, enforce_eager=True)
    runner = llm.runner
    inner = runner.decode
    inner_pf = runner.prefill

    def decode(n_rows, steps):
        torch.cuda.nvtx.range_push("decode")
        inner(n_rows, steps)
        torch.cuda.nvtx.range_pop()

    def prefill(pieces):
        torch.cuda.nvtx.range_push("prefill")
        inner_pf(pieces)
        torch.cuda.nvtx.range_pop()

    runner.decode = decode
    runner.prefill = prefill
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(0, 128000, (R, P), generator=g)
    sp = SamplingParams(max_tokens=S + 1, temperature=0.0, ignore_eos=True)
    llm.generate(prompts, sp)
    st = llm.last_stats
    print(json.dumps({"requests": R, "prompt_len": P, "decode_steps": S,
                      "decode_ms_per_step": round(st.decode_ms / max(1, S), 3),
                      "prefill_ms": round(st.prefill_ms, 1)}))
    llm.shutdown()


if __name__ == "__main__":
    main()
