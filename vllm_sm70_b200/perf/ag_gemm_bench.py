"""All-gather -> GEMM timing at TP W (one process per GPU).

Times, on every rank with CUDA events, and reports the max over ranks: the
fused kernel (``parallel.symm.AgGemm``), and the baseline NCCL all-gather
followed by the same tcgen05 GEMM. Roofline: the slower of the GEMM at the
measured bf16 burst and the bytes each rank receives over NVLink ((W - 1) / W
of the gathered activations) at the measured 770 GB/s per direction.

    torchrun --nproc-per-node 2 -m vllm_sm70_b200.perf.ag_gemm_bench --T 16384 --N 3072 --K 4096
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, default=16384)
    ap.add_argument("--N", type=int, default=3072)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)

    from .. import _ext
    from ..ops import linear
    from ..parallel import state, symm
    from .microbench import peaks

    _ext.require()
    ps = state.init(timeout_s=120)
    dev = ps.device
    torch.ops._b200_C.init_device(dev.index)
    linear.configure_workspace(dev.index)
    W = ps.tp_size
    T, N, K = args.T, args.N, args.K
    ag = symm.AgGemm(ps, T, K)
    shard = torch.randn(T // W, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
    out = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
    gathered = torch.empty(T, K, device=dev, dtype=torch.bfloat16)

    def fused():
        ag(shard, w, out=out)

    def baseline():
        dist.all_gather_into_tensor(gathered, shard, group=ps.tp_group)
        linear.gemm(gathered, w, out=out)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / args.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ps.tp_group)
        return float(t.item())

    ms_f = timed(fused)
    ms_b = timed(baseline)
    ms_g = timed(lambda: linear.gemm(gathered, w, out=out))
    pk = peaks()
    flops = 2.0 * T * N * K
    nvlink = (W - 1) / W * T * K * 2  # bytes each rank receives
    bound_ms = max(flops / (pk["bf16_tflops"] * 1e9), nvlink / 770e6)
    if ps.tp_rank == 0:
        print(json.dumps({"kernel": "all_gather_gemm", "W": W, "T": T, "N": N, "K": K,
                          "fused_ms": round(ms_f, 4), "nccl_then_gemm_ms": round(ms_b, 4),
                          "gemm_only_ms": round(ms_g, 4), "roofline_ms": round(bound_ms, 4),
                          "frac_of_roofline": round(bound_ms / ms_f, 3), "peaks": pk["src"]}))
    del ag
    torch.cuda.synchronize()
    dist.barrier(group=ps.cpu_group)
    state.shutdown()


if __name__ == "__main__":
    main()
