"""TP/EP communication entry points used by the models.

Each entry point has two paths:

* fused -- one kernel over symmetric (peer-mapped) memory that performs the
  collective and the following compute (``parallel/symm.py`` +
  ``csrc/comm/*``), selected when the symmetric workspace is set up and the
  kill switch is on;
* baseline -- NCCL through ``torch.distributed`` followed by the unfused op.

The path choice depends only on rank-uniform inputs (config, env, shapes),
so every rank enters the same collective -- the reference's rule
(``sm70/vllm_sm70/sample.py:230-271``, ``sample_greedy.py:171-205``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import envs, ops
from . import state as pstate

_fused = {"ar_rmsnorm": None, "tp_exchange": None, "local_gemm_norm": None}


def set_local_gemm_norm(impl) -> None:
    """Install the TP1 GEMM + residual add + RMSNorm kernel path (a
    ``parallel.symm.LocalAddRmsNorm`` or None)."""
    _fused["local_gemm_norm"] = impl


def local_gemm_norm():
    impl = _fused["local_gemm_norm"]
    if impl is None or not envs.get("VLLM_B200_FUSED_GEMM_NORM"):
        return None
    return impl


def set_tp_exchange(impl) -> None:
    """Install the sampler exchange over peer memory (a
    ``parallel.symm.TpExchange`` or None)."""
    _fused["tp_exchange"] = impl


def tp_exchange():
    impl = _fused["tp_exchange"]
    if impl is None or not envs.get("VLLM_B200_FUSED_SAMPLER_XCHG"):
        return None
    return impl


def set_fused_ar_rmsnorm(impl) -> None:
    """Install the fused all-reduce + add + RMSNorm implementation (a
    ``parallel.symm.FusedArRmsNorm`` or None)."""
    _fused["ar_rmsnorm"] = impl


def fused_ar_rmsnorm():
    impl = _fused["ar_rmsnorm"]
    if impl is None or not envs.get("VLLM_B200_FUSED_AR_RMSNORM"):
        return None
    return impl


def row_parallel_out(T: int, H: int, dtype=torch.bfloat16, device=None) -> torch.Tensor | None:
    """Output buffer for a row-parallel GEMM whose result feeds
    :func:`all_reduce_add_rms_norm`: the fused path's peer-visible stage
    buffer (so the GEMM writes the collective's input directly), else None."""
    impl = fused_ar_rmsnorm()
    if impl is not None and impl.admits(T) and impl.H == H:
        return impl.stage_view(T)
    return None


def adopt_residual(residual: torch.Tensor) -> torch.Tensor:
    """Move the residual stream into the fused path's symmetric buffer (once
    per forward) so the fused kernel updates it in place on every rank."""
    impl = fused_ar_rmsnorm() if pstate.get().tp_size > 1 else local_gemm_norm()
    T = residual.shape[0]
    if impl is not None and impl.admits(T) and impl.H == residual.shape[1]:
        rv = impl.res_view(T)
        rv.copy_(residual)
        return rv
    return residual


def all_reduce_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                            eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """``x <- allreduce_tp(x)``; ``residual += x``; ``x <- rmsnorm(residual) w``.
    Returns ``(x, residual)`` (views of symmetric buffers on the fused path,
    the updated inputs otherwise)."""
    st = pstate.get()
    if st.tp_size > 1:
        impl = fused_ar_rmsnorm()
        if impl is not None:
            r = impl(x, residual, w, eps)
            if r is not None:
                return r
        dist.all_reduce(x, group=st.tp_group)
    ops.fused_add_rms_norm(x, residual, w, eps)
    return x, residual


def linear_all_reduce_add_rms_norm(lin, x: torch.Tensor, residual: torch.Tensor,
                                   w: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Row-parallel linear followed by :func:`all_reduce_add_rms_norm`. With
    TP > 1, a bf16 dense weight and the fused workspace up, the GEMM and the
    collective run as ONE kernel (``VLLM_B200_FUSED_GEMM_AR``, from
    ``VLLM_B200_FUSED_GEMM_AR_MIN_TOKENS`` tokens up -- a rank-uniform choice);
    otherwise the GEMM writes the stage and the collective follows."""
    st = pstate.get()
    T, H = x.shape[0], getattr(lin, "out_features", None)
    if st.tp_size == 1:
        impl = local_gemm_norm()
        lw = getattr(lin, "w", None)
        if (impl is not None and type(lin).__name__ == "DenseLinear" and lw is not None
                and lw.dtype == torch.bfloat16 and x.is_cuda and x.stride(1) == 1
                and residual.is_cuda):
            r = impl.gemm(x, lw, residual, w, eps)
            if r is not None:
                return r
    if (st.tp_size > 1 and envs.get("VLLM_B200_FUSED_GEMM_AR")
            and T >= envs.get("VLLM_B200_FUSED_GEMM_AR_MIN_TOKENS")):
        impl = fused_ar_rmsnorm()
        lw = getattr(lin, "w", None)
        if (impl is not None and type(lin).__name__ == "DenseLinear" and lw is not None
                and lw.dtype == torch.bfloat16 and x.is_cuda and x.stride(1) == 1):
            r = impl.gemm(x, lw, residual, w, eps)
            if r is not None:
                return r
    out = lin.forward(x, out=row_parallel_out(T, H) if H is not None else None)
    return all_reduce_add_rms_norm(out, residual, w, eps)


def greedy_merge(vals: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """Gather per-rank (max value, id) pairs and pick the global top-1 in rank
    order with the shared tie rule: one peer-memory kernel when the sampler
    exchange is installed (rows within its capacity), else an NCCL all-gather
    and the merge kernel. Reference parity: F12 greedy
    (``sm70/vllm_sm70/sample_greedy.py:293-328``) and the P2P top-1 exchange
    (``sm70/csrc/custom_ar/top1_custom_ar.cu:52-101``)."""
    st = pstate.get()
    if st.tp_size == 1:
        return ids
    impl = tp_exchange()
    if impl is not None and ids.is_cuda:
        out = impl.top1(vals, ids)
        if out is not None:
            return out
    rows = ids.shape[0]
    packed = torch.stack([vals.float(), ids.float()], 0)  # ids < 2^24 are exact in fp32
    allp = torch.empty(st.tp_size * 2, rows, dtype=torch.float32, device=ids.device)
    dist.all_gather_into_tensor(allp, packed.contiguous(), group=st.tp_group)
    allp = allp.view(st.tp_size, 2, rows)
    return ops.sampling.merge_rank_top1(allp[:, 0], allp[:, 1].to(torch.int64))


def gather_candidates(v: torch.Tensor, i: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The ranks' per-row candidate lists ``[rows, C]`` concatenated in rank
    order along the candidate dimension: one peer-memory kernel when the
    sampler exchange is installed, else two NCCL all-gathers. Reference
    parity: the candidate gather (``sm70/vllm_sm70/sample.py:308-309``)."""
    st = pstate.get()
    if st.tp_size == 1:
        return v, i
    impl = tp_exchange()
    if impl is not None and v.is_cuda:
        r = impl.gather(v, i)
        if r is not None:
            return r
    return pstate.tp_all_gather(v, dim=1), pstate.tp_all_gather(i, dim=1)
