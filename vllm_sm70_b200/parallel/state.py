"""Process-group plumbing: one process per GPU, ``torch.distributed`` over NCCL
(plus a gloo CPU group for control-plane agreement), tensor- and
expert-parallel groups.

Reference parity: upstream vLLM's ``GroupCoordinator`` as used by the
reference (``sm70/vllm_sm70/ar_rms_fusion.py:178-185``,
``sample_greedy.py:159-168``, gloo ``cpu_group`` in ``warmup/coord.py:54-60``).
The reference supports TP in {1, 2}; this runtime supports TP and EP of
1/2/4/8 and TPxEP hybrids on one node.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    world_size: int = 1
    rank: int = 0
    local_rank: int = 0
    tp_size: int = 1
    tp_rank: int = 0
    ep_size: int = 1
    ep_rank: int = 0
    device: torch.device = torch.device("cpu")
    tp_group: object = None
    ep_group: object = None
    cpu_group: object = None
    backend: str = "none"

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1


_STATE: ParallelState | None = None


def get() -> ParallelState:
    global _STATE
    if _STATE is None:
        _STATE = ParallelState(device=torch.device("cuda", 0) if torch.cuda.is_available()
                               else torch.device("cpu"))
    return _STATE


def init(tp_size: int | None = None, ep_size: int = 1, backend: str | None = None,
         timeout_s: float = 120.0) -> ParallelState:
    """Initialise from the torchrun environment (RANK/WORLD_SIZE/LOCAL_RANK/
    MASTER_*). Single process when WORLD_SIZE is unset or 1."""
    global _STATE
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
        if dev.type == "cuda":
            torch.cuda.set_device(dev)
        _STATE = ParallelState(device=dev, tp_size=1, ep_size=1)
        return _STATE
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    use_cuda = torch.cuda.is_available()
    if backend is None:
        backend = "nccl" if use_cuda else "gloo"
    if use_cuda:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    if not dist.is_initialized():
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = dev
        dist.init_process_group(**kw)
    tp = tp_size or world
    assert world % tp == 0, (world, tp)
    # Contiguous ranks form a TP group; EP spans the whole world by default.
    tp_group = None
    my_tp = None
    for start in range(0, world, tp):
        ranks = list(range(start, start + tp))
        g = dist.new_group(ranks) if tp < world else dist.group.WORLD
        if rank in ranks:
            my_tp = g
    tp_group = my_tp
    ep = ep_size if ep_size > 1 else 1
    ep_group = dist.group.WORLD if ep == world else (None if ep == 1 else dist.new_group(
        list(range(rank - rank % ep, rank - rank % ep + ep))))
    cpu_group = dist.new_group(backend="gloo") if backend != "gloo" else dist.group.WORLD
    _STATE = ParallelState(world_size=world, rank=rank, local_rank=local, tp_size=tp,
                           tp_rank=rank % tp, ep_size=ep, ep_rank=rank % ep, device=dev,
                           tp_group=tp_group, ep_group=ep_group, cpu_group=cpu_group,
                           backend=backend)
    return _STATE


def shutdown() -> None:
    global _STATE
    if dist.is_initialized():
        dist.destroy_process_group()
    _STATE = None


# -- NCCL baseline collectives (the fused kernels fall back to these) ----------
def tp_all_reduce(x: torch.Tensor) -> torch.Tensor:
    st = get()
    if st.tp_size > 1:
        dist.all_reduce(x, group=st.tp_group)
    return x


def tp_all_gather(x: torch.Tensor, dim: int = 0) -> torch.Tensor:
    st = get()
    if st.tp_size == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(st.tp_size)]
    dist.all_gather(parts, x.contiguous(), group=st.tp_group)
    return torch.cat(parts, dim=dim)


def tp_all_gather_into(out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """``out [tp * n, ...]`` <- concat over ranks of ``x [n, ...]``."""
    st = get()
    if st.tp_size == 1:
        out.copy_(x)
        return out
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def barrier() -> None:
    st = get()
    if st.world_size > 1:
        dist.barrier(group=st.cpu_group)
