"""Headline benchmark: output tokens/s of the Llama-3.1-8B-shaped workload.

Workload: Llama-3.1-8B shapes, random-init bf16 weights
(std 0.02), 256 requests with uniform-random prompt ids of length 1024, 256
greedy output tokens each (ignore EOS), tensor-parallel over N GPUs of one
node. One bench "step" is the whole workload: prefill of all 256 prompts and
255 decode steps, through the public ``LLM.generate`` API.

    python bench.py --gpus 1 --steps 3 --warmup 3
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference ...   # upstream vLLM + the reference plugin

``value`` is device time (CUDA events on the launching stream, barrier +
synchronize on both sides, max over ranks); ``e2e`` is the host wall clock of
the same ``generate`` calls (pinned prompt upload + output download included).
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = "output tok/s (box, max over ranks) at 1/2/4/8 B200; p50 TTFT/TPOT"
MODEL = "Llama-3.1-8B-shaped (32L, h4096, 32q/8kv, d128, ffn14336, vocab128256)"
N_REQ, PROMPT, OUT = 256, 1024, 256  # the headline workload; --requests/--prompt-len/
# --output-len exist only for profiling runs and mark the JSON line "profiling"
BASELINE_VALUE = None  # no published number exists for this config
PRESET, TEMPERATURE, SPEC_K = "llama-3.1-8b", 0.0, 0
PROFILING = False  # set by --requests / --prompt-len / --output-len

# The other benchmark configurations of this project (--config): preset, workload, sampling.
WORKLOADS = {
    "llama-3.1-8b": dict(preset="llama-3.1-8b", model=MODEL, requests=256, prompt=1024,
                         output=256, temperature=0.0, spec_k=0),
    "qwen3-30b-a3b-fp8": dict(
        preset="qwen3-30b-a3b-fp8", requests=512, prompt=2048, output=256, temperature=0.0,
        spec_k=0, model="Qwen3-30B-A3B-shaped (48L, h2048, 32q/4kv, d128, 128 experts top-8, "
                        "expert ffn 768, vocab151936), block-FP8 weights"),
    "llama-3.1-70b-awq": dict(
        preset="llama-3.1-70b-awq", requests=128, prompt=4096, output=512, temperature=0.0,
        spec_k=0, model="Llama-3.1-70B-shaped (80L, h8192, 64q/8kv, d128, ffn28672), AWQ int4 g128"),
    "qwen3-next-80b-a3b-nvfp4": dict(
        preset="qwen3-next-80b-a3b-nvfp4", requests=256, prompt=8192, output=256,
        temperature=0.7, spec_k=3,
        model="Qwen3-Next-80B-A3B-shaped (48L hybrid 3:1 gated-DeltaNet / gated attention, "
              "512 experts top-10 + shared, MTP k=3), NVFP4 weights"),
}


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", ",".join(map(str, self.gpus))],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001 - clocks are best-effort metadata
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        load = [s for s in sm if s > 500] or sm
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist_setup():
    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    return world, rank


def _max_over_ranks(x: float) -> float:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def _sum_over_ranks(x: float) -> float:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        return float(t.item())
    return x


def _barrier():
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def make_prompts(seed: int = 1234):
    """Fresh uniform-random prompt ids. Every warm-up and timed step uses a new
    seed, so no step can be served from a prefix cache of an earlier one."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 128000, (N_REQ, PROMPT), generator=g, dtype=torch.int64)


# ----------------------------------------------------------------------------- ours
def run_ours(args) -> dict:
    sys.path.insert(0, str(ROOT))
    from vllm_sm70_b200.engine import LLM, SamplingParams
    from vllm_sm70_b200.parallel import state as pstate
    from vllm_sm70_b200.utils import launch_count

    world, rank = _dist_setup()
    dp = args.layout == "dp-ep" and world > 1  # each replica serves its share of the requests
    tp_in = args.tp if dp else 1  # dp-ep: TP ranks inside a replica (the TP x EP layout)
    if dp and world % tp_in:
        raise SystemExit(f"--tp {tp_in} does not divide the world size {world}")
    n_rep = world // tp_in if dp else 1
    if dp:
        ps = pstate.init(tp_size=tp_in, ep_size=world)
    else:
        ps = pstate.init(tp_size=args.gpus if world > 1 else 1)
    rep = rank // tp_in  # contiguous ranks form a replica and pass the same prompts
    share = (lambda p: p[rep::n_rep].contiguous()) if dp else (lambda p: p)
    llm = LLM(PRESET, tensor_parallel_size=ps.tp_size,
              max_num_seqs=(N_REQ + n_rep - 1) // n_rep if dp else N_REQ,
              max_model_len=PROMPT + OUT + (SPEC_K + 1 if SPEC_K else 0),
              block_size=args.block_size, max_num_batched_tokens=args.chunk,
              load_format="dummy", seed=0, speculative_k=SPEC_K,
              data_parallel_size=n_rep if dp else 1, enable_expert_parallel=dp)
    warm = [share(make_prompts(1000 + i)).pin_memory() for i in range(args.warmup)]
    timed = [share(make_prompts(2000 + i)).pin_memory() for i in range(args.steps)]
    prompts = timed[0]
    sp = SamplingParams(max_tokens=OUT, temperature=TEMPERATURE, ignore_eos=True)
    for w in warm:
        llm.generate(w, sp)
    torch.cuda.synchronize()
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    launch_count.reset()
    _barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    ev0.record()
    ttft, tpot = [], []
    pre_ms = dec_ms = 0.0
    outs = None
    for i in range(args.steps):
        outs = llm.generate(timed[i], sp)
        st = llm.last_stats
        ttft += st.ttft_ms
        tpot += st.tpot_ms
        pre_ms += st.prefill_ms
        dec_ms += st.decode_ms
    ev1.record()
    torch.cuda.synchronize()
    _barrier()
    wall = time.perf_counter() - w0
    dev_ms = ev0.elapsed_time(ev1)
    launches = launch_count.total()
    clocks = sampler.stop() if sampler else None
    dev_ms = _max_over_ranks(dev_ms)
    wall = _max_over_ranks(wall)
    n_out = sum(len(o.output_token_ids) for o in outs) * args.steps
    if dp:  # every replica served its own share: the job's tokens are the sum
        n_out = int(_sum_over_ranks(float(n_out) if rank % tp_in == 0 else 0.0))
    value = n_out / (dev_ms / 1e3)
    e2e = n_out / wall
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 2),
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 3),
        "dtype": "bf16", "data": "synthetic (uniform-random prompt ids, random-init weights std 0.02)",
        "config": {"model": MODEL, "global_batch": N_REQ, "seq_len": PROMPT,
                   "output_len": OUT,
                   "parallelism": (f"dp{n_rep}-tp{tp_in}-ep{world}" if tp_in > 1 else
                                   f"dp{world}-ep{world}") if dp else f"tp{args.gpus}",
                   "temperature": TEMPERATURE, "speculative_k": SPEC_K,
                   "l2": "inputs larger than L2 (16 GB of weights streamed per step)",
                   "block_size": args.block_size, "prefill_chunk_tokens": args.chunk},
        "p50_ttft_ms": round(statistics.median(ttft), 1) if ttft else None,
        "p50_tpot_ms": round(statistics.median(tpot), 3) if tpot else None,
        "phase_ms_per_step": {"prefill": round(pre_ms / args.steps, 1),
                              "decode": round(dec_ms / args.steps, 1)},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s",
                "h2d_bytes_per_step": int(prompts.numel() * prompts.element_size()),
                "d2h_bytes_per_step": int(N_REQ * OUT * 4)},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if PROFILING:
        res["profiling"] = True
    if rank == 0:
        print(json.dumps(res), flush=True)
    llm.shutdown()
    pstate.shutdown()
    return res


def run_online(args) -> dict:
    """Serving under load (one GPU): requests arrive as a Poisson process of
    ``--arrival-rate`` per second (seeded) into the continuous-batching engine
    loop; per-request TTFT / TPOT from host clocks (arrival to first token,
    first to last token). Not the headline metric."""
    import random

    sys.path.insert(0, str(ROOT))
    from vllm_sm70_b200.engine import LLM, SamplingParams

    world, _ = _dist_setup()
    if world > 1:
        raise SystemExit("--arrival-rate runs on one GPU")
    llm = LLM(PRESET, max_num_seqs=N_REQ, max_model_len=PROMPT + OUT + (SPEC_K + 1 if SPEC_K else 0),
              block_size=args.block_size, max_num_batched_tokens=args.chunk,
              load_format="dummy", seed=0, speculative_k=SPEC_K)
    sp = SamplingParams(max_tokens=OUT, temperature=TEMPERATURE, ignore_eos=True)
    for i in range(args.warmup):  # warm-up: a short plain batch
        llm.generate(make_prompts(1000 + i)[:8], sp)
    prompts = make_prompts(3000)
    rng = random.Random(7)
    arrivals, t = [], 0.0
    for _ in range(N_REQ):
        t += rng.expovariate(args.arrival_rate)
        arrivals.append(t)
    t0 = time.perf_counter()
    nxt, first, last, done = 0, {}, {}, {}

    def feed(block):
        nonlocal nxt
        if nxt >= N_REQ:
            return None
        now = time.perf_counter() - t0
        if block and arrivals[nxt] > now:
            time.sleep(arrivals[nxt] - now)
            now = arrivals[nxt]
        out = []
        while nxt < N_REQ and arrivals[nxt] <= now:
            out.append((nxt, prompts[nxt], sp))
            nxt += 1
        return out

    def on_tokens(rid, ids, fin):
        if ids:
            tt = time.perf_counter() - t0
            first.setdefault(rid, tt)
            last[rid] = tt

    llm.generate([], feed=feed, on_tokens=on_tokens,
                 on_finish=lambda o: done.__setitem__(o.request_id, len(o.output_token_ids)))
    wall = time.perf_counter() - t0
    ttft = sorted(first[i] - arrivals[i] for i in done)
    tpot = sorted((last[i] - first[i]) / (done[i] - 1) for i in done if done[i] > 1)

    def pct(v, q):
        return round(v[min(len(v) - 1, int(q * len(v)))] * 1e3, 2) if v else None

    res = {"metric": "online serving: output tok/s and p50 / p90 TTFT, TPOT (host clock)",
           "value": round(sum(done.values()) / wall, 1), "unit": "tok/s",
           "arrival_rate_per_s": args.arrival_rate, "requests": N_REQ,
           "p50_ttft_ms": pct(ttft, 0.5), "p90_ttft_ms": pct(ttft, 0.9),
           "p50_tpot_ms": pct(tpot, 0.5), "p90_tpot_ms": pct(tpot, 0.9),
           "config": {"model": MODEL, "seq_len": PROMPT, "output_len": OUT},
           "profiling": True}
    print(json.dumps(res), flush=True)
    llm.shutdown()
    return res


# ----------------------------------------------------------------------------- reference
def _write_hf_config(d: Path):
    cfg = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
        "intermediate_size": 14336, "num_attention_heads": 32, "num_key_value_heads": 8,
        "num_hidden_layers": 32, "head_dim": 128, "vocab_size": 128256, "rms_norm_eps": 1e-5,
        "rope_theta": 500000.0, "max_position_embeddings": 131072, "torch_dtype": "bfloat16",
        "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                         "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
        "bos_token_id": 128000, "eos_token_id": 128001, "tie_word_embeddings": False,
        "hidden_act": "silu", "initializer_range": 0.02,
    }
    (d / "config.json").write_text(json.dumps(cfg))


def run_reference(args) -> dict:
    world, rank = _dist_setup()
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "vllm_sm70").exists():
        line = {"impl": "reference", "unavailable": "baseline/_ref not installed"}
        print(json.dumps(line))
        return line
    sys.path.insert(0, str(ref))
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    try:
        import vllm_sm70  # noqa: F401  (the reference plugin; inert unless every GPU is sm_70)
        from vllm import LLM, SamplingParams
        from vllm.inputs import TokensPrompt
    except Exception as e:  # noqa: BLE001
        line = {"impl": "reference", "unavailable": f"import failed: {type(e).__name__}: {e}"}
        print(json.dumps(line))
        return line
    d = Path(tempfile.mkdtemp(prefix="ref_llama8b_"))
    _write_hf_config(d)
    kw = dict(model=str(d), load_format="dummy", dtype="bfloat16", skip_tokenizer_init=True,
              max_num_seqs=N_REQ, max_model_len=PROMPT + OUT, seed=0,
              tensor_parallel_size=args.gpus, gpu_memory_utilization=0.85)
    if world > 1:
        kw["distributed_executor_backend"] = "external_launcher"
    llm = LLM(**kw)
    def tp(seed):
        return [TokensPrompt(prompt_token_ids=row.tolist()) for row in make_prompts(seed)]

    warm = [tp(1000 + i) for i in range(args.warmup)]
    timed = [tp(2000 + i) for i in range(args.steps)]
    sp = SamplingParams(max_tokens=OUT, temperature=0.0, ignore_eos=True)
    for w in warm:
        llm.generate(w, sp, use_tqdm=False)
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    _barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    ev0.record()
    ttft, tpot = [], []
    n_out = 0
    for i in range(args.steps):
        outs = llm.generate(timed[i], sp, use_tqdm=False)
        for o in outs:
            n_out += len(o.outputs[0].token_ids)
            m = getattr(o, "metrics", None)
            if m is not None and getattr(m, "first_token_latency", None) is not None:
                ttft.append(m.first_token_latency * 1e3)
    ev1.record()
    torch.cuda.synchronize()
    _barrier()
    wall = time.perf_counter() - w0
    dev_ms = _max_over_ranks(ev0.elapsed_time(ev1))
    wall = _max_over_ranks(wall)
    clocks = sampler.stop() if sampler else None
    value = n_out / (dev_ms / 1e3)
    res = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random prompt ids, dummy weights)",
        "config": {"model": MODEL, "global_batch": N_REQ, "seq_len": PROMPT, "output_len": OUT,
                   "parallelism": f"tp{args.gpus}",
                   "stack": "upstream vLLM (image) + vllm_sm70 plugin from baseline/_ref"},
        "p50_ttft_ms": round(statistics.median(ttft), 1) if ttft else None,
        "e2e": {"value": round(n_out / wall, 1), "unit": "tok/s",
                "h2d_bytes_per_step": N_REQ * PROMPT * 8, "d2h_bytes_per_step": N_REQ * OUT * 4},
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(res), flush=True)
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--chunk", type=int, default=16384, help="prefill tokens per chunk")
    ap.add_argument("--requests", type=int, default=None, help="profiling only")
    ap.add_argument("--prompt-len", type=int, default=None, help="profiling only")
    ap.add_argument("--output-len", type=int, default=None, help="profiling only")
    ap.add_argument("--verbose", action="store_true", help="log engine set-up (GEMM plans)")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="llama-3.1-8b",
                    help="benchmark configuration (default: the headline Llama-3.1-8B workload)")
    ap.add_argument("--arrival-rate", type=float, default=None,
                    help="serving under load instead of the headline batch: Poisson "
                         "arrivals per second into the continuous-batching loop (1 GPU)")
    ap.add_argument("--layout", choices=["tp", "dp-ep"], default="tp",
                    help="N > 1: tensor parallel (MoE experts sliced over the TP group), or "
                         "data-parallel attention with all-to-all expert parallelism")
    ap.add_argument("--tp", type=int, default=1,
                    help="dp-ep only: tensor-parallel ranks inside each data-parallel replica "
                         "(TP x EP: experts over all ranks, attention and dense GEMMs over TP)")
    args = ap.parse_args(argv)
    if args.verbose:
        import logging
        logging.basicConfig(level=logging.INFO, stream=sys.stderr)
    global N_REQ, PROMPT, OUT, MODEL, PRESET, TEMPERATURE, SPEC_K, PROFILING
    wl = WORKLOADS[args.config]
    N_REQ, PROMPT, OUT, MODEL = wl["requests"], wl["prompt"], wl["output"], wl["model"]
    PRESET, TEMPERATURE, SPEC_K = wl["preset"], wl["temperature"], wl["spec_k"]
    if args.impl == "reference" and args.config != "llama-3.1-8b":
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference arm is wired for the headline Llama-3.1-8B config only"}))
        return
    if args.requests or args.prompt_len or args.output_len:
        N_REQ = args.requests or N_REQ
        PROMPT = args.prompt_len or PROMPT
        OUT = args.output_len or OUT
        PROFILING = True
        print("warning: non-default workload; the JSON line is for profiling only",
              file=sys.stderr)
    if args.warmup < 3:
        print("warning: --warmup < 3 does not meet the timing rules", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    elif args.arrival_rate:
        run_online(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
