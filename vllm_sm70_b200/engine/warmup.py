"""Pre-capture warm-up: GEMM tile / split-K tuning with TP agreement and a
LUT file with a manifest.

For every GEMM shape the model will run at the CUDA-graph batch sizes, the
tuner times each admissible (tile config, split-K) pair with CUDA events
(L2 flushed between launches, as in the model where each layer's weights are
cold) and installs the fastest in the native dispatch table
(``_b200_C::gemm_set_plan``). Under TP, rank 0 tunes and the table is
broadcast over the gloo CPU group, so every rank runs identical plans (graph
capture and collective shapes stay rank-uniform). Failures are shared before
anyone raises.

LUT files: JSON ``{"manifest": {...}, "plans": [[M, N, K, epi, cfg, splits], ...]}``;
the manifest records the library fingerprint and GPU name, and a strict import
(``VLLM_B200_GEMM_LUT_STRICT=1``) refuses a mismatch.

Reference parity: the TP-coordinated TurboMind warm-up and dispatch-cache
export/import (``sm70/vllm_sm70/warmup/__init__.py``, ``plan.py``,
``coord.py:16-223``, ``cache.py:1-356``; ops ``sm70_gemm_import_cache`` /
``sm70_gemm_export_cache``, ``gemm_runtime.cpp:832-872``).
"""
from __future__ import annotations

import json
import logging
from pathlib import Path

import torch

from .. import _ext, envs
from ..ops import linear as _lin

logger = logging.getLogger("vllm.b200.warmup")

EPI_NONE, EPI_SILU = 0, 1
# cfg id -> (BN, swap, BM); BM 256 = tall tile (two M=128 accumulators)
CFGS = {0: (256, False, 128), 1: (128, False, 128), 2: (16, True, 128), 3: (32, True, 128),
        4: (64, True, 128), 5: (192, False, 128), 6: (96, False, 128), 7: (64, False, 128),
        8: (128, True, 128), 9: (256, False, 256), 10: (224, False, 256), 11: (128, False, 256),
        12: (112, False, 256), 13: (64, False, 256),
        # CTA pairs (cta_group::2): 256-row tiles over two SMs
        19: (256, False, 256), 20: (128, False, 256), 21: (192, False, 256), 22: (64, False, 256),
        23: (96, False, 256)}
# cluster split-K configs (the K slices of a tile reduce through distributed
# shared memory): cfg id -> (BN, BM); only tried with splits >= 2
CLUSTER_CFGS = {14: (256, 128), 15: (128, 128), 16: (128, 256), 17: (112, 256), 18: (64, 256)}
SILU_CFGS = (0, 1, 9, 11, 14, 16, 19, 20)
SPLITS = (1, 2, 3, 4, 6, 8)


def candidates(M: int, N: int, K: int, epi: int) -> list[tuple[int, int]]:
    out = []
    nkb = (K + 63) // 64
    for cfg, (bn, swap, bm) in CFGS.items():
        if epi == EPI_SILU and cfg not in SILU_CFGS:
            continue
        if swap and (M > 256 or bn < min(M, 128) // 2 or (bn > 16 and bn // 2 >= M)):
            continue
        if not swap and M <= 16:
            continue
        if bm == 256 and M <= 128:
            continue
        for s in SPLITS:
            if s > 1 and (nkb + s - 1) // s < 4:
                continue
            out.append((cfg, s))
    if M <= 512:
        for cfg, (bn, bm) in CLUSTER_CFGS.items():
            if epi == EPI_SILU and cfg not in SILU_CFGS:
                continue
            if M <= 16 or (bm == 256 and M <= 128):
                continue
            for s in SPLITS:
                if s > 1 and (nkb + s - 1) // s >= 4:
                    out.append((cfg, s))
    return out


def _time(fn, iters: int, flush_buf: torch.Tensor) -> float:
    """Median device ms of ``fn`` over ``iters`` launches, each after an L2
    flush; two untimed calls first (module load, library heuristics)."""
    fn()
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush_buf.sum()  # read-based L2 eviction (no dirty lines left behind)
        # Keep the GPU busy while the host enqueues the timed launch, so host
        # launch overhead never shows up as device time.
        torch.cuda._sleep(100_000)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    return ts[len(ts) // 2]


def tune_shapes(shapes: list[tuple[int, int, int, int]], iters: int = 5,
                device: torch.device | None = None, library: bool | None = None) -> list[list[int]]:
    """Time candidates for each (M, N, K, epi); install and return the winners.
    ``library``: also time cuBLAS for plain GEMMs (cfg -2 in the returned plans
    marks a shape routed to it); default VLLM_B200_GEMM_LIBRARY."""
    if library is None:
        library = envs.get("VLLM_B200_GEMM_LIBRARY")
    _ext.require()
    ops = torch.ops._b200_C
    dev = device or torch.device("cuda", torch.cuda.current_device())
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    if library:
        # First library call of the process (handle, workspace, kernel load)
        # stays out of every timed region.
        x = torch.randn(256, 256, device=dev, dtype=torch.bfloat16)
        torch.mm(x, x.t())
        torch.cuda.synchronize()
    plans = []
    cache: dict = {}
    for (M, N, K, epi) in shapes:
        key = (M, N, K, epi)
        if key in cache:
            continue
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        w = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        out = torch.empty(M, N // 2 if epi == EPI_SILU else N, device=dev, dtype=torch.bfloat16)
        best = None
        for cfg, sp in candidates(M, N, K, epi):
            if epi == EPI_SILU:
                ops.gemm_set_plan(M, N, K, epi, cfg, sp)
                fn = lambda: ops.gemm_bf16_silu_mul_out(out, a, w, -1)  # noqa: E731
            else:
                fn = lambda c=cfg, s_=sp: ops.gemm_bf16_out(out, a, w, c, s_)  # noqa: E731
            try:
                ms = _time(fn, iters, flush)
            except RuntimeError as e:  # a config the launcher rejects for this shape
                logger.debug("tune %s cfg=%d s=%d rejected: %s", key, cfg, sp, e)
                continue
            if best is None or ms < best[0]:
                best = (ms, cfg, sp)
        if best is not None and library:
            # The vendor library is a candidate too (kept only when it beats the
            # best tcgen05 plan by more than noise): the plain GEMM, or for
            # gate_up the GEMM on the interleaved weights + the SiLU*up kernel.
            if epi == EPI_NONE:
                fn = lambda: torch.mm(a, w.t(), out=out)  # noqa: E731
            else:
                gu = torch.empty(M, N, device=dev, dtype=torch.bfloat16)

                def fn():
                    torch.mm(a, w.t(), out=gu)
                    ops.silu_mul(out, gu, _lin.GATE_UP_BLOCK)
            ms = _time(fn, iters, flush)
            if ms < best[0] * 0.97:
                best = (ms, _lin.LIBRARY_CFG, 0)
        if best is not None:
            if best[1] == _lin.LIBRARY_CFG:
                _lin.set_library(M, N, K, True, epi)
                ops.gemm_set_plan(M, N, K, epi, -1, 0)
            else:
                _lin.set_library(M, N, K, False, epi)
                ops.gemm_set_plan(M, N, K, epi, best[1], best[2])
            plans.append([M, N, K, epi, best[1], best[2]])
            cache[key] = best
            logger.info("gemm plan M=%d N=%d K=%d epi=%d -> cfg=%d splits=%d (%.1f us)",
                        M, N, K, epi, best[1], best[2], best[0] * 1e3)
        del a, w, out
    return plans


def install_plans(plans) -> None:
    _ext.require()
    for p in plans:
        M, N, K, epi, cfg, sp = [int(x) for x in p]
        if cfg == _lin.LIBRARY_CFG:
            _lin.set_library(M, N, K, True, epi)
            torch.ops._b200_C.gemm_set_plan(M, N, K, epi, -1, 0)
        else:
            _lin.set_library(M, N, K, False, epi)
            torch.ops._b200_C.gemm_set_plan(M, N, K, epi, cfg, sp)


def export_plans() -> list[list[int]]:
    _ext.require()
    flat = list(torch.ops._b200_C.gemm_export_plans())
    plans = [flat[i:i + 6] for i in range(0, len(flat), 6)]
    return (plans + [[M, N, K, EPI_NONE, _lin.LIBRARY_CFG, 0] for (M, N, K) in _lin.library_shapes()]
            + [[M, N, K, EPI_SILU, _lin.LIBRARY_CFG, 0] for (M, N, K) in _lin.library_shapes(1)])


def manifest() -> dict:
    return {"fingerprint": _ext.fingerprint(),
            "gpu": torch.cuda.get_device_name() if torch.cuda.is_available() else "none",
            "torch": torch.__version__, "format": 1}


def save_lut(path: str | Path, plans=None) -> None:
    plans = export_plans() if plans is None else plans
    Path(path).write_text(json.dumps({"manifest": manifest(), "plans": plans}))


def load_lut(path: str | Path, strict: bool | None = None) -> int:
    strict = envs.get("VLLM_B200_GEMM_LUT_STRICT") if strict is None else strict
    d = json.loads(Path(path).read_text())
    man = d.get("manifest", {})
    mine = manifest()
    if man.get("fingerprint") != mine["fingerprint"] or man.get("gpu") != mine["gpu"]:
        msg = f"GEMM LUT {path} was made for {man}, this build is {mine}"
        if strict:
            raise RuntimeError(msg)
        logger.warning("%s; importing anyway (non-strict)", msg)
    install_plans(d.get("plans", []))
    return len(d.get("plans", []))


def agree(plans: list | None, ps) -> list:
    """Broadcast rank 0's plans to every TP rank over the CPU group; a failure
    on any rank is shared first so no rank is left inside a collective."""
    import torch.distributed as dist

    if ps is None or ps.world_size <= 1:
        return plans or []
    ok = plans is not None or ps.rank != 0
    flags = [None] * ps.world_size
    dist.all_gather_object(flags, bool(ok), group=ps.cpu_group)
    if not all(flags):
        raise RuntimeError(f"GEMM warm-up failed on ranks {[i for i, f in enumerate(flags) if not f]}")
    box = [plans if ps.rank == 0 else None]
    dist.broadcast_object_list(box, src=0, group=ps.cpu_group)
    if ps.rank != 0:
        install_plans(box[0])
    return box[0]


def model_gemm_shapes(model, Ms: list[int],
                      lm_ms: list[int] | None = None) -> list[tuple[int, int, int, int]]:
    """(M, N, K, epi) of every distinct GEMM the model runs at each M; the LM
    head only at ``lm_ms`` (it sees one sampled row per sequence, so the
    prefill chunk size never reaches it). ``lm_ms`` None: every M."""
    shapes = []
    seen = set()
    for L in model.layers:
        for name, lin in L.items():
            w = getattr(lin, "w", None)
            if not isinstance(w, torch.Tensor) or not hasattr(lin, "forward"):
                continue
            if w.dtype != torch.bfloat16:
                continue
            epi = EPI_SILU if type(lin).__name__ == "GateUpLinear" else EPI_NONE
            nk = (w.shape[0], w.shape[1], epi)
            if nk in seen:
                continue
            seen.add(nk)
    lm = getattr(model, "lm_head", None)
    lm_nk = (lm.shape[0], lm.shape[1], EPI_NONE) if lm is not None else None
    lm_set = set(Ms if lm_ms is None else lm_ms)
    for M in Ms:
        for (N, K, epi) in sorted(seen):
            shapes.append((M, N, K, epi))
        if lm_nk is not None and lm_nk not in seen and M in lm_set:
            shapes.append((M,) + lm_nk)
    return shapes


def engine_warmup(model, ps, Ms: list[int], lut_path: str | None = None,
                  lm_ms: list[int] | None = None) -> None:
    """Tune (or import) the plans for the decode batch sizes before capture."""
    if not envs.get("VLLM_B200_WARMUP"):
        return
    path = lut_path or envs.get("VLLM_B200_GEMM_LUT_PATH")
    if path and Path(path).exists():
        n = load_lut(path)
        logger.info("imported %d GEMM plans from %s", n, path)
        return
    plans = None
    if ps is None or ps.rank == 0:
        try:
            plans = tune_shapes(model_gemm_shapes(model, Ms, lm_ms))
        except Exception as e:  # noqa: BLE001 - shared with the other ranks by agree()
            logger.error("GEMM tuning failed: %s", e)
            plans = None
            if ps is None or ps.world_size <= 1:
                raise
    plans = agree(plans, ps)
    out = envs.get("VLLM_B200_GEMM_LUT_EXPORT_PATH")
    if out and (ps is None or ps.rank == 0):
        save_lut(out, plans)


def platform_warmup(worker) -> None:
    """vLLM ``kernel_warmup`` hook (U1): router and sampler preparation and
    GEMM planning for vLLM-owned linears go through the same tables."""
    from ..integration import ar_norm_fusion
    from ..models import router
    from . import hidden_state_sampler

    router.prepare_worker(worker)
    hidden_state_sampler.prepare_worker(worker)
    ar_norm_fusion.install_for_worker(worker)
