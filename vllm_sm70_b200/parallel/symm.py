"""Symmetric (peer-mapped) workspaces for the fused TP collectives.

Buffers come from ``torch.distributed._symmetric_memory`` (allocation and
the handle exchange are the plumbing; every kernel that touches them is this
library's own, with plain NVLink loads/stores -- no library kernel is ever
handed a peer's memory). Allocation and rendezvous happen once at start-up,
before any CUDA-graph capture, so captured kernels carry fixed peer
addresses (the reference's R5 lesson: register at init, never graph
operands).

``FusedArRmsNorm`` owns three [T_max, H] bf16 buffers per rank (stage =
row-parallel GEMM output, residual, normalised output) and a signal pad; it
implements ``all_reduce_add_rms_norm`` for ``T <= T_max`` (rank-uniform
admission), else defers to NCCL.
"""
from __future__ import annotations

import logging

import torch
import torch.distributed as dist

from .. import envs
from ..utils import launch_count

logger = logging.getLogger("vllm.b200.symm")

SIGNAL_WORDS = 64  # uint32 words per rank: ready[W], done[W], epoch, done_target, arrive


def nvls_min_ranks() -> int:
    return int(envs.get("VLLM_B200_NVLS_MIN_RANKS"))


class FusedArRmsNorm:
    def __init__(self, ps, max_tokens: int, hidden: int, dtype=torch.bfloat16,
                 grid_cap: int | None = None):
        import torch.distributed._symmetric_memory as symm_mem

        assert ps.tp_size in (2, 4, 8), ps.tp_size
        self.ps = ps
        self.T_max = max_tokens
        self.H = hidden
        dev = ps.device
        # One CTA per SM at most (the whole grid must be resident: it spins on
        # peer flags).
        self.grid_cap = grid_cap or (torch.cuda.get_device_properties(dev).multi_processor_count
                                     if dev.type == "cuda" else 148)
        group = ps.tp_group

        def alloc(n, dt):
            t = symm_mem.empty(n, dtype=dt, device=dev)
            h = symm_mem.rendezvous(t, group)
            return t, h

        self.stage, hs = alloc(max_tokens * hidden, dtype)
        self.res, hr = alloc(max_tokens * hidden, dtype)
        self.out, ho = alloc(max_tokens * hidden, dtype)
        self.flags, hf = alloc(SIGNAL_WORDS, torch.int32)
        self.flags.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
        self.stage_ptrs = [int(p) for p in hs.buffer_ptrs]
        self.res_ptrs = [int(p) for p in hr.buffer_ptrs]
        self.out_ptrs = [int(p) for p in ho.buffer_ptrs]
        self.flag_ptrs = [int(p) for p in hf.buffer_ptrs]
        self._handles = (hs, hr, ho, hf)
        # NVLS: multicast addresses of the three data buffers when the fabric
        # offers them (NVSwitch) and VLLM_B200_NVLS=1; the decision must be
        # rank-uniform, so it is agreed over the CPU group.
        self.mc_ptrs: list[int] = []
        want = bool(envs.get("VLLM_B200_NVLS")) and ps.tp_size >= nvls_min_ranks()
        ok = False
        if want and dev.type == "cuda":
            try:
                ok = bool(symm_mem._SymmetricMemory.has_multicast_support(
                    symm_mem.DeviceType.CUDA, dev.index)) and all(
                        int(h.multicast_ptr) != 0 for h in (hs, hr, ho))
            except (AttributeError, RuntimeError):
                ok = False
        vote = torch.tensor([1 if ok else 0], dtype=torch.int32)
        dist.all_reduce(vote, op=dist.ReduceOp.MIN, group=ps.cpu_group)
        if int(vote.item()) == 1:
            self.mc_ptrs = [int(hs.multicast_ptr), int(hr.multicast_ptr), int(ho.multicast_ptr)]
            logger.info("fused all-reduce + RMSNorm: NVLS multicast (W=%d)", ps.tp_size)
        self.timeout_ms = int(envs.get("VLLM_B200_COMM_TIMEOUT_MS"))
        self.calls = 0

    # Views handed to the model -------------------------------------------------
    def stage_view(self, T: int) -> torch.Tensor:
        return self.stage[: T * self.H].view(T, self.H)

    def res_view(self, T: int) -> torch.Tensor:
        return self.res[: T * self.H].view(T, self.H)

    def out_view(self, T: int) -> torch.Tensor:
        return self.out[: T * self.H].view(T, self.H)

    def admits(self, T: int) -> bool:
        return 0 < T <= self.T_max

    def grid(self, T: int) -> int:
        rows = (T + self.ps.tp_size - 1) // self.ps.tp_size
        return max(1, min(self.grid_cap, rows))

    def __call__(self, x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
        """Returns (normalised x, residual) as views of the symmetric buffers,
        or None when not admitted (caller uses NCCL)."""
        T = x.shape[0]
        if not self.admits(T) or x.shape[1] != self.H:
            return None
        st = self.stage_view(T)
        if x.data_ptr() != st.data_ptr():
            st.copy_(x)
        rv = self.res_view(T)
        if residual.data_ptr() != rv.data_ptr():
            rv.copy_(residual)
        torch.ops._b200_C.ar_rmsnorm(self.stage_ptrs, self.res_ptrs, self.out_ptrs,
                                     self.flag_ptrs, self.ps.tp_rank, T, self.H, w, eps,
                                     self.timeout_ms, self.grid(T), self.mc_ptrs)
        launch_count.add(1)
        self.calls += 1
        return self.out_view(T), rv

    def gemm(self, x: torch.Tensor, lin_w: torch.Tensor, residual: torch.Tensor,
             w: torch.Tensor, eps: float, cfg: int = -1, splits: int = 0):
        """Row-parallel ``x @ lin_w^T`` fused with the all-reduce + residual
        add + RMSNorm in ONE kernel (the tcgen05 GEMM writes this rank's stage,
        then its CTAs run the collective over NVLink). Returns (normalised x,
        residual) as views of the symmetric buffers, or None when not taken."""
        T = x.shape[0]
        if not self.admits(T) or lin_w.shape[0] != self.H:
            return None
        rv = self.res_view(T)
        if residual.data_ptr() != rv.data_ptr():
            rv.copy_(residual)
        ok = torch.ops._b200_C.gemm_ar_rmsnorm(x, lin_w, self.stage_ptrs, self.res_ptrs,
                                               self.out_ptrs, self.flag_ptrs, self.ps.tp_rank,
                                               w, eps, self.timeout_ms, cfg, splits,
                                               self.mc_ptrs)
        if not ok:
            return None
        launch_count.add(1)
        self.calls += 1
        return self.out_view(T), rv


class TpExchange:
    """Symmetric buffers of the vocab-parallel sampler exchange
    (``_b200_C::tp_exchange``): per rank a receive buffer of two halves x W
    slots of ``cap`` bytes and a signal pad. One kernel stores this rank's
    (value, id) pairs or top-C candidate lists into every rank's slot and
    merges (greedy) or concatenates (candidates) in rank order on every rank.
    ``rows_max`` bounds the rows per call (larger calls use NCCL)."""

    def __init__(self, ps, rows_max: int, cands: int):
        import torch.distributed._symmetric_memory as symm_mem

        assert ps.tp_size in (2, 4, 8), ps.tp_size
        self.ps = ps
        self.rows_max = rows_max
        self.cands = cands
        self.cap = ((rows_max * max(1, cands) * 8 + 15) // 16) * 16
        W = ps.tp_size
        dev = ps.device
        self.recv = symm_mem.empty(2 * W * self.cap, dtype=torch.uint8, device=dev)
        hr = symm_mem.rendezvous(self.recv, ps.tp_group)
        self.pad = symm_mem.empty(16, dtype=torch.int32, device=dev)
        hp = symm_mem.rendezvous(self.pad, ps.tp_group)
        self.pad.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
        self.bufs = []
        for q in range(W):
            self.bufs += [int(hr.buffer_ptrs[q]), int(hp.buffer_ptrs[q])]
        self._handles = (hr, hp)
        self.timeout_ms = int(envs.get("VLLM_B200_COMM_TIMEOUT_MS"))

    def top1(self, vals: torch.Tensor, ids: torch.Tensor) -> torch.Tensor | None:
        """Global greedy ids [rows] int32 from this rank's (value, id) pairs."""
        rows = ids.shape[0]
        if rows > self.rows_max or rows * 8 > self.cap:
            return None
        out = torch.empty(rows, dtype=torch.int32, device=ids.device)
        torch.ops._b200_C.tp_exchange(self.bufs, self.ps.tp_rank, self.cap, 0,
                                      vals.float().contiguous(), ids.int().contiguous(), out,
                                      None, self.timeout_ms)
        launch_count.add(1)
        return out

    def gather(self, v: torch.Tensor, i: torch.Tensor):
        """(values [rows, W*C] fp32, ids [rows, W*C] int32): the ranks'
        candidate lists [rows, C] concatenated in rank order."""
        rows, C = v.shape
        if rows * C * 8 > self.cap:
            return None
        W = self.ps.tp_size
        ov = torch.empty(rows, W * C, dtype=torch.float32, device=v.device)
        oi = torch.empty(rows, W * C, dtype=torch.int32, device=v.device)
        torch.ops._b200_C.tp_exchange(self.bufs, self.ps.tp_rank, self.cap, 1,
                                      v.float().contiguous(), i.int().contiguous(), ov, oi,
                                      self.timeout_ms)
        launch_count.add(1)
        return ov, oi


class AgGemm:
    """Column-parallel all-gather -> GEMM (``_b200_C::gemm_ag``): each rank
    holds a row shard ``[T / W, K]`` of the input; one kernel per rank copies
    its shard into every rank's symmetric gather buffer (two halves of
    ``t_max`` rows used by alternate epochs) and multiplies the gathered rows
    by its weight shard, each tile starting as soon as the ranks it reads from
    have published their rows. Reference parity: the per-tile flag-publish /
    peer-load pattern of the reference's dormant tile all-reduce epilogue
    (``sm70/csrc/turbomind/lmdeploy/src/turbomind/kernels/gemm/epilogue.h:347-560``)."""

    def __init__(self, ps, t_max: int, K: int, dtype=torch.bfloat16):
        import torch.distributed._symmetric_memory as symm_mem

        assert ps.tp_size in (2, 4, 8), ps.tp_size
        self.ps, self.t_max, self.K = ps, t_max, K
        dev = ps.device
        self.xfull = symm_mem.empty(2 * t_max * K, dtype=dtype, device=dev)
        hx = symm_mem.rendezvous(self.xfull, ps.tp_group)
        self.pad = symm_mem.empty(16, dtype=torch.int32, device=dev)
        hp = symm_mem.rendezvous(self.pad, ps.tp_group)
        self.pad.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
        self.xfull_ptrs = [int(p) for p in hx.buffer_ptrs]
        self.pad_ptrs = [int(p) for p in hp.buffer_ptrs]
        self._handles = (hx, hp)
        self.timeout_ms = int(envs.get("VLLM_B200_COMM_TIMEOUT_MS"))

    def admits(self, T: int, K: int) -> bool:
        return K == self.K and 0 < T <= self.t_max and T % self.ps.tp_size == 0

    def __call__(self, shard: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
                 cfg: int = -1, splits: int = 0) -> torch.Tensor:
        T = shard.shape[0] * self.ps.tp_size
        if out is None:
            out = torch.empty(T, w.shape[0], dtype=shard.dtype, device=shard.device)
        torch.ops._b200_C.gemm_ag(w, out, shard.contiguous(), self.xfull_ptrs, self.pad_ptrs,
                                  self.ps.tp_rank, self.t_max, cfg, splits, self.timeout_ms)
        launch_count.add(1)
        return out


class LocalAddRmsNorm:
    """TP1: a row GEMM (o_proj, down_proj) fused with the residual add and
    RMSNorm that follow it, in one kernel -- the fused all-reduce epilogue of
    :class:`FusedArRmsNorm` with a single rank: every CTA stores its tiles
    into the stage, the CTAs meet at a grid-wide flag barrier (the grid is
    resident) and then add the residual and normalise the rows. Plain device
    buffers (no peers); the same interface as FusedArRmsNorm's GEMM path, and
    the same bits as the GEMM followed by ``fused_add_rms_norm``."""

    def __init__(self, device, max_tokens: int, hidden: int, dtype=torch.bfloat16):
        self.T_max, self.H = max_tokens, hidden
        self.stage = torch.empty(max_tokens * hidden, dtype=dtype, device=device)
        self.res = torch.empty(max_tokens * hidden, dtype=dtype, device=device)
        self.out = torch.empty(max_tokens * hidden, dtype=dtype, device=device)
        self.flags = torch.zeros(SIGNAL_WORDS, dtype=torch.int32, device=device)
        self.stage_ptrs = [self.stage.data_ptr()]
        self.res_ptrs = [self.res.data_ptr()]
        self.out_ptrs = [self.out.data_ptr()]
        self.flag_ptrs = [self.flags.data_ptr()]
        self.timeout_ms = int(envs.get("VLLM_B200_COMM_TIMEOUT_MS"))
        self.calls = 0

    def admits(self, T: int) -> bool:
        return 0 < T <= self.T_max

    def res_view(self, T: int) -> torch.Tensor:
        return self.res[: T * self.H].view(T, self.H)

    def out_view(self, T: int) -> torch.Tensor:
        return self.out[: T * self.H].view(T, self.H)

    def gemm(self, x: torch.Tensor, lin_w: torch.Tensor, residual: torch.Tensor,
             w: torch.Tensor, eps: float, cfg: int = -1, splits: int = 0):
        """(normalised rows, new residual) as views of the buffers, or None
        when not taken (the caller runs the GEMM and fused_add_rms_norm)."""
        T = x.shape[0]
        if not self.admits(T) or lin_w.shape[0] != self.H:
            return None
        rv = self.res_view(T)
        if residual.data_ptr() != rv.data_ptr():
            rv.copy_(residual)
        ok = torch.ops._b200_C.gemm_ar_rmsnorm(x, lin_w, self.stage_ptrs, self.res_ptrs,
                                               self.out_ptrs, self.flag_ptrs, 0, w, eps,
                                               self.timeout_ms, cfg, splits, [])
        if not ok:
            return None
        launch_count.add(1)
        self.calls += 1
        return self.out_view(T), rv
