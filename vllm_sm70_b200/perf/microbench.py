"""Kernel microbenchmarks (CUDA-event timed, after warm-up).

    python -m vllm_sm70_b200.perf.microbench gemm --M 256 --N 6144 --K 4096
    python -m vllm_sm70_b200.perf.microbench decode-attn --batch 256 --ctx 1152
    python -m vllm_sm70_b200.perf.microbench prefill-attn --seqs 16 --len 1024
    python -m vllm_sm70_b200.perf.microbench all

Each case prints one JSON line with the device time per launch and the
achieved fraction of the measured roofline (``MEASURED_PEAKS.json`` when
present: HBM GB/s for bandwidth-bound kernels, bf16 TFLOP/s for GEMMs).
Inputs are sized above the 126 MB L2 where the case allows, or the L2 is
flushed between iterations (``--flush``).

Reference parity: ``sm70/tools/bench_fv100_capture.py`` (attention
microbench) and the reference's per-kernel GB/s tables.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


_FLUSH = None


def flush_l2():
    """Evict L2 by READING a 256 MB buffer (a write-based flush leaves L2 full
    of dirty lines whose write-back would be charged to the timed kernel)."""
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    _FLUSH.sum()


GRAPH = False  # --graph: time CUDA-graph replays (no host launch work in the timed region)


def time_fn(fn, iters: int = 20, warmup: int = 3, flush: bool = False) -> float:
    """Mean device ms per call (CUDA events on the current stream)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if GRAPH:
        s0 = torch.cuda.Stream()
        s0.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s0):
            fn()  # warm on the capture stream
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s0):
                fn()
        torch.cuda.synchronize()
        fn = g.replay
    if not flush:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / iters
    tot = 0.0
    for _ in range(iters):
        flush_l2()
        torch.cuda._sleep(100_000)  # GPU busy while the host enqueues the timed launch
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        tot += s.elapsed_time(e)
    return tot / iters


def _setup():
    from .. import _ext
    from ..ops import linear

    _ext.require()
    dev = torch.cuda.current_device()
    torch.ops._b200_C.init_device(dev)
    linear.configure_workspace(dev)


def bench_gemm(M, N, K, cfg=-1, splits=0, iters=20, flush=False, cublas=True, epi=0):
    """epi 1: fused SiLU(gate)*up epilogue (N interleaved gate/up rows, N/2 outputs)."""
    from ..ops import linear

    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(M, N // 2 if epi else N, device="cuda", dtype=torch.bfloat16)
    if epi:
        if cfg >= 0 and splits > 0:  # the SiLU op takes its split from the plan table
            torch.ops._b200_C.gemm_set_plan(M, N, K, 1, cfg, splits)
            cfg = -1
        fn = lambda: torch.ops._b200_C.gemm_bf16_silu_mul_out(out, a, w, cfg)  # noqa: E731
    else:
        fn = lambda: linear.gemm(a, w, out=out, cfg=cfg, splits=splits)  # noqa: E731
    ms = time_fn(fn, iters, flush=flush)
    pk = peaks()
    flops = 2.0 * M * N * K
    byts = 2.0 * (M * K + N * K + M * N)
    res = {"kernel": "gemm_bf16_silu" if epi else "gemm_bf16", "M": M, "N": N, "K": K,
           "plan": linear.plan(M, N, K, epi),
           "ms": round(ms, 5), "tflops": round(flops / ms / 1e9, 1),
           "gbs": round(byts / ms / 1e6, 1),
           "frac_tensor": round(flops / ms / 1e9 / pk["bf16_tflops"], 3),
           "frac_hbm": round(byts / ms / 1e6 / pk["hbm_gbs"], 3), "peaks": pk["src"]}
    if cublas:
        full = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms2 = time_fn(lambda: torch.matmul(a, w.t(), out=full), iters, flush=flush)
        res["cublas_ms"] = round(ms2, 5)
        res["vs_cublas"] = round(ms2 / ms, 3)
    return res


def bench_gemm_fp8(M, N, K, bn=0, iters=20, flush=False):
    """W8A8 block-FP8 GEMM (kind::f8f6f4 + scale promotion) on pre-quantised
    activations, plus the activation quantiser, vs the bf16 tcgen05 GEMM of
    the same shape."""
    from ..ops import linear, quant

    w = torch.randn(N, K, device="cuda") * 0.05
    lin = quant.make_linear("fp8", w)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    xq, sa = quant.quant_fp8_act(x)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ms = time_fn(lambda: torch.ops._b200_C.gemm_fp8_out(out, xq, sa, lin.raw, lin.scales, bn),
                 iters, flush=flush)
    ms_q = time_fn(lambda: torch.ops._b200_C.quant_fp8_act(x, xq, sa), iters, flush=flush)
    wb = w.to(torch.bfloat16)
    ms_bf16 = time_fn(lambda: linear.gemm(x, wb, out=out), iters, flush=flush)
    pk = peaks()
    flops = 2.0 * M * N * K
    byts = M * K + N * K + 2.0 * M * N
    return {"kernel": "gemm_fp8_w8a8", "M": M, "N": N, "K": K, "bn": bn, "ms": round(ms, 5),
            "tflops": round(flops / ms / 1e9, 1), "gbs": round(byts / ms / 1e6, 1),
            "frac_hbm": round(byts / ms / 1e6 / pk["hbm_gbs"], 3),
            "quant_ms": round(ms_q, 5), "bf16_gemm_ms": round(ms_bf16, 5), "peaks": pk["src"]}


def bench_gemm_nvfp4(M, N, K, iters=20, flush=False):
    """NVFP4 W4A4 GEMM (kind::mxf4nvf4, block-16 e4m3 scales in TMEM) on
    pre-quantised activations, plus the activation quantiser, vs the bf16
    tcgen05 GEMM of the same shape."""
    from ..ops import linear, quant

    w = torch.randn(N, K, device="cuda") * 0.02
    lin = quant.make_linear("nvfp4", w)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    xq, sf, rs = quant.quant_nvfp4_act(x)
    atoms = lin.sf_atoms()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ms = time_fn(lambda: torch.ops._b200_C.gemm_nvfp4_out(out, xq, sf, rs, lin.raw, atoms,
                                                          lin.out_scale, -1), iters, flush=flush)
    ms_q = time_fn(lambda: torch.ops._b200_C.quant_nvfp4_act(x, xq, sf, rs), iters, flush=flush)
    wb = w.to(torch.bfloat16)
    ms_bf16 = time_fn(lambda: linear.gemm(x, wb, out=out), iters, flush=flush)
    pk = peaks()
    flops = 2.0 * M * N * K
    byts = M * K / 2 + N * K / 2 + 2.0 * M * N
    return {"kernel": "gemm_nvfp4_w4a4", "M": M, "N": N, "K": K, "ms": round(ms, 5),
            "tflops": round(flops / ms / 1e9, 1), "gbs": round(byts / ms / 1e6, 1),
            "frac_hbm": round(byts / ms / 1e6 / pk["hbm_gbs"], 3),
            "quant_ms": round(ms_q, 5), "bf16_gemm_ms": round(ms_bf16, 5), "peaks": pk["src"]}


def bench_gdn_chunk(nseq=4, length=8192, hk=16, hv=32, d=128, iters=5, serial=True):
    """Gated-DeltaNet prefill: the 64-token chunked WY/UT kernel vs the
    token-serial recurrence on the same inputs (Qwen3-Next head shape)."""
    from ..ops import gdn

    T = nseq * length
    cu = torch.arange(nseq + 1, device="cuda", dtype=torch.int32) * length
    slots = torch.arange(nseq, device="cuda", dtype=torch.int32)
    q = torch.randn(T, hk * d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, hk * d, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, hv * d, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(T, hv, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(T, hv, device="cuda", dtype=torch.bfloat16)
    A_log = torch.randn(hv, device="cuda") * 0.5
    dt = torch.randn(hv, device="cuda") * 0.5
    st = torch.zeros(nseq, hv, d, d, device="cuda")
    out = torch.empty(T, hv * d, device="cuda", dtype=torch.bfloat16)

    def run(chunked):
        gdn.gdn_recurrent(q, k, v, a, b, A_log, dt, st, cu, slots, hk, hv, True, out, True,
                          chunked)

    ms = time_fn(lambda: run(True), iters)
    r = {"kernel": "gdn_chunk", "nseq": nseq, "len": length, "hk": hk, "hv": hv, "d": d,
         "ms": round(ms, 4)}
    if serial:
        r["serial_ms"] = round(time_fn(lambda: run(False), max(1, iters // 2)), 4)
    return r


def bench_moe(T=16384, E=128, k=8, H=2048, I=768, fmt="fp8", iters=10):
    """One MoE expert layer (top-k routing, permutation, grouped expert GEMMs,
    SiLU*up, weighted combine) on Qwen3-30B-A3B shapes, random routing."""
    from ..ops import moe

    g = torch.Generator(device="cuda").manual_seed(1)
    w13 = torch.randn(E, 2 * I, H, device="cuda", generator=g) * 0.05
    w2 = torch.randn(E, H, I, device="cuda", generator=g) * 0.05
    ew = moe.ExpertWeights.from_dense(fmt, w13, w2)
    del w13, w2
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w, ids = moe.topk(torch.randn(T, E, device="cuda"), k)
    ws = moe.MoEWorkspace(T, k, E, H, I, "cuda")
    ms = time_fn(lambda: moe.experts_forward(x, w, ids, ew, ws), iters, flush=True)
    flops = 2.0 * T * k * (2 * I * H + H * I)
    return {"kernel": "moe_experts", "fmt": fmt, "T": T, "E": E, "k": k, "H": H, "I": I,
            "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1)}


def bench_rope_kv(T=16384, hq=32, hkv=8, d=128, bs=16, iters=20):
    """Fused RoPE + paged KV write on a [T, (hq + 2 hkv) d] QKV tensor."""
    from ..ops import attention as A

    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(T, device="cuda") % 4096
    nb = (T + bs - 1) // bs
    slots = torch.arange(T, device="cuda")
    cs = A.rope_cos_sin(d, 4096, 5e5, device="cuda")
    kc = torch.empty(nb, hkv, bs, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.empty_like(kc)
    ms = time_fn(lambda: A.rope_kv_write(qkv, pos, cs, kc, vc, slots, hq, hkv), iters, flush=True)
    byts = T * (hq + 2 * hkv) * d * 2 + T * (hq + hkv) * d * 2 + 2 * T * hkv * d * 2
    pk = peaks()
    return {"kernel": "rope_kv", "T": T, "ms": round(ms, 5), "gbs": round(byts / ms / 1e6, 1),
            "frac_hbm": round(byts / ms / 1e6 / pk["hbm_gbs"], 3), "peaks": pk["src"]}


def bench_rms_norm(T=16384, H=4096, iters=20):
    """Fused residual add + RMSNorm (in place) on [T, H] bf16 rows."""
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    ms = time_fn(lambda: torch.ops._b200_C.fused_add_rms_norm(x, r, w, 1e-5), iters, flush=True)
    byts = 4.0 * T * H * 2
    pk = peaks()
    return {"kernel": "fused_add_rms_norm", "T": T, "H": H, "ms": round(ms, 5),
            "gbs": round(byts / ms / 1e6, 1), "frac_hbm": round(byts / ms / 1e6 / pk["hbm_gbs"], 3),
            "peaks": pk["src"]}


def bench_decode_attn(batch=256, ctx=1152, hq=32, hkv=8, d=128, bs=16, splits=1, iters=20,
                      seq_blocks=False):
    from ..ops import attention as A

    nb = batch * math.ceil(ctx / bs)
    kc = torch.randn(nb, hkv, bs, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = (torch.arange(nb, device="cuda", dtype=torch.int32) if seq_blocks
          else torch.randperm(nb, device="cuda", dtype=torch.int32)).view(batch, -1)
    sl = torch.full((batch,), ctx, device="cuda", dtype=torch.int32)
    cu = torch.arange(batch + 1, device="cuda", dtype=torch.int32)
    q = torch.randn(batch, hq, d, device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(q)
    po = pml = None
    if splits > 1:
        po = torch.empty(splits, batch, hq, d, device="cuda")
        pml = torch.empty(splits, batch, hq, 2, device="cuda")
    ms = time_fn(lambda: A.paged_attention(o, q, kc, vc, bt, sl, cu, 1, d ** -0.5, decode=True,
                                           num_splits=splits, part_o=po, part_ml=pml), iters)
    byts = batch * ctx * hkv * d * 2 * 2
    pk = peaks()
    return {"kernel": "paged_attention_decode", "batch": batch, "ctx": ctx, "hq": hq, "hkv": hkv,
            "d": d, "block": bs, "splits": splits, "blocks": "sequential" if seq_blocks else "random",
            "ms": round(ms, 5),
            "gbs": round(byts / ms / 1e6, 1), "frac_hbm": round(byts / ms / 1e6 / pk["hbm_gbs"], 3),
            "peaks": pk["src"]}


def bench_prefill_attn(seqs=16, length=1024, hq=32, hkv=8, d=128, bs=16, iters=10):
    from ..ops import attention as A

    nb = seqs * length // bs
    kc = torch.randn(nb, hkv, bs, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.arange(nb, device="cuda", dtype=torch.int32).view(seqs, -1)
    sl = torch.full((seqs,), length, device="cuda", dtype=torch.int32)
    cu = torch.arange(seqs + 1, device="cuda", dtype=torch.int32) * length
    q = torch.randn(seqs * length, hq, d, device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(q)
    ms = time_fn(lambda: A.paged_attention(o, q, kc, vc, bt, sl, cu, length, d ** -0.5), iters)
    flops = seqs * hq * length * length * d * 2.0  # causal: 2 GEMMs x L^2/2 x 2 flop
    pk = peaks()
    return {"kernel": "paged_attention_prefill", "seqs": seqs, "len": length, "hq": hq, "hkv": hkv,
            "d": d, "block": bs, "ms": round(ms, 5), "tflops": round(flops / ms / 1e9, 1),
            "frac_tensor": round(flops / ms / 1e9 / pk["bf16_tflops"], 3), "peaks": pk["src"]}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "gemm-cublas", "gemm-fp8", "gemm-nvfp4",
                                     "decode-attn", "prefill-attn", "gdn-chunk", "rope-kv",
                                     "rms-norm", "moe", "all"])
    ap.add_argument("--M", type=int, default=256)
    ap.add_argument("--N", type=int, default=6144)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--cfg", type=int, default=-1)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=1152)
    ap.add_argument("--seqs", type=int, default=16)
    ap.add_argument("--len", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--flush", action="store_true")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="gemm: time every (cfg, splits)")
    ap.add_argument("--epi", type=int, default=0, help="gemm: 1 = fused SiLU*up epilogue")
    ap.add_argument("--graph", action="store_true", help="time CUDA-graph replays")
    ap.add_argument("--block", type=int, default=16, help="attention: KV-cache block size")
    ap.add_argument("--d", type=int, default=128, help="attention: head dim")
    ap.add_argument("--hq", type=int, default=32, help="attention: query heads")
    ap.add_argument("--hkv", type=int, default=8, help="attention: KV heads")
    ap.add_argument("--fmt", default="fp8", help="moe: expert weight format")
    ap.add_argument("--seq-blocks", action="store_true",
                    help="decode-attn: sequential block table (default: random permutation)")
    args = ap.parse_args(argv)
    global GRAPH
    GRAPH = args.graph
    _setup()
    out = []
    if args.case == "gemm" and args.sweep:
        from ..engine import warmup

        for cfg, sp in warmup.candidates(args.M, args.N, args.K, args.epi):
            r = bench_gemm(args.M, args.N, args.K, cfg, sp, args.iters, args.flush, False,
                           args.epi)
            r["cfg"], r["splits"] = cfg, sp
            out.append(r)
        torch.ops._b200_C.gemm_clear_plans()
        out.append(bench_gemm(args.M, args.N, args.K, -1, 0, args.iters, args.flush, True,
                              args.epi))
    elif args.case == "gemm":
        out.append(bench_gemm(args.M, args.N, args.K, args.cfg, args.splits, args.iters,
                              args.flush, not args.no_cublas, args.epi))
    elif args.case == "gemm-fp8":
        out.append(bench_gemm_fp8(args.M, args.N, args.K, max(0, args.cfg), args.iters,
                                  args.flush))
    elif args.case == "gemm-nvfp4":
        out.append(bench_gemm_nvfp4(args.M, args.N, args.K, args.iters, args.flush))
    elif args.case == "gdn-chunk":
        out.append(bench_gdn_chunk(args.seqs, args.len, iters=args.iters,
                                   serial=not args.no_cublas))
    elif args.case == "rope-kv":
        out.append(bench_rope_kv(args.M, args.hq, args.hkv, args.d, args.block, args.iters))
    elif args.case == "moe":
        out.append(bench_moe(args.M, fmt=args.fmt, iters=args.iters))
    elif args.case == "rms-norm":
        out.append(bench_rms_norm(args.M, args.K, args.iters))
    elif args.case == "gemm-cublas":
        a = torch.randn(args.M, args.K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(args.N, args.K, device="cuda", dtype=torch.bfloat16)
        o = torch.empty(args.M, args.N, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: torch.matmul(a, w.t(), out=o), args.iters, flush=args.flush)
        out.append({"kernel": "cublas_bf16", "M": args.M, "N": args.N, "K": args.K,
                    "ms": round(ms, 5), "tflops": round(2.0 * args.M * args.N * args.K / ms / 1e9, 1)})
    elif args.case == "decode-attn":
        out.append(bench_decode_attn(args.batch, args.ctx, hq=args.hq, hkv=args.hkv, d=args.d,
                                     bs=args.block,
                                     splits=max(1, args.splits), iters=args.iters,
                                     seq_blocks=args.seq_blocks))
    elif args.case == "prefill-attn":
        out.append(bench_prefill_attn(args.seqs, args.len, hq=args.hq, hkv=args.hkv, d=args.d,
                                      bs=args.block, iters=args.iters))
    else:
        for (M, N, K) in [(16384, 6144, 4096), (16384, 4096, 4096), (16384, 28672, 4096),
                          (16384, 4096, 14336), (256, 6144, 4096), (256, 4096, 4096),
                          (256, 28672, 4096), (256, 4096, 14336), (256, 128256, 4096),
                          (1, 4096, 4096), (16, 6144, 4096), (64, 28672, 4096)]:
            out.append(bench_gemm(M, N, K, iters=args.iters, flush=M <= 256))
        out.append(bench_decode_attn(256, 1152))
        out.append(bench_decode_attn(1, 8192, splits=16))
        out.append(bench_prefill_attn(16, 1024))
    for r in out:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
