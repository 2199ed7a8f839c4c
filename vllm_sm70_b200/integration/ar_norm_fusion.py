"""TP all-reduce + residual add + RMSNorm fusion in vLLM's compiled graph.

The rewrite (a pattern of the composite post-grad pass): a
``vllm.all_reduce(x, group)`` whose only user is
``vllm_ir.fused_add_rms_norm(ar, residual, weight, eps)`` becomes ONE call
of ``vllm_b200.all_reduce_fused_add_rms_norm(x, residual, weight, eps,
group)``. Matching is structural (op identity and def-use edges on the FX
graph), so it sees exactly the node pair vLLM's decoder layers emit after
every row-parallel projection; an all-reduce with other users (its output is
needed elsewhere) is left alone.

The fused op decides at run time with rank-uniform inputs only (the
installed implementation, the kill switch, the token count): the installed
fused route -- one kernel over symmetric NVLink buffers that reduces, adds
the residual and normalises (``csrc/comm/ar_rmsnorm.cu``) -- or the exact
unfused pair it replaced. Without an installed route (CPU, TP = 1, or
``VLLM_B200_FUSED_AR_RMSNORM=0``) the result is the unfused computation.

Reference parity: the K17 pattern and its runtime gate
(``sm70/vllm_sm70/ar_rms_fusion.py:105-433``: ``fused_add_rms_norm(
all_reduce(x), residual)`` -> ``tp2_all_reduce_fused_add_rms_norm``).
"""
from __future__ import annotations

import logging

import torch

logger = logging.getLogger("vllm.b200.passes")

OP = "vllm_b200::all_reduce_fused_add_rms_norm"

# Installed fused route: fn(x, residual, weight, eps) -> (out, residual) or None
# to decline (the op then runs the unfused pair). Set by the worker when its
# symmetric workspace is up.
_route = {"fn": None}


def install_fused_route(fn) -> None:
    _route["fn"] = fn


def install_for_worker(worker) -> bool:
    """Inside a vLLM worker (``kernel_warmup``, before graph capture):
    allocate the symmetric workspace over vLLM's TP group and install the
    fused route. Every rank decides from rank-uniform facts and the ranks
    agree over the CPU group before the collective allocation, so either all
    of them install it or none does. Returns whether it was installed."""
    from types import SimpleNamespace

    import torch.distributed as dist

    from .. import envs

    try:
        from vllm.distributed import get_tp_group

        g = get_tp_group()
    except Exception:  # noqa: BLE001 - no vLLM distributed state: nothing to fuse
        return False
    ok = (bool(envs.get("VLLM_B200_FUSED_AR_RMSNORM")) and torch.cuda.is_available()
          and g.world_size in (2, 4, 8))
    cfg = getattr(worker, "vllm_config", None)
    if ok and cfg is not None:
        H = int(cfg.model_config.get_hidden_size())
        T = int(cfg.scheduler_config.max_num_batched_tokens)
        ok = cfg.model_config.dtype == torch.bfloat16 and H % 8 == 0
    else:
        ok = False
    if g.world_size > 1:
        flags = [None] * g.world_size
        dist.all_gather_object(flags, ok, group=g.cpu_group)
        ok = all(flags)
    if not ok:
        return False
    from ..parallel.symm import FusedArRmsNorm

    ps = SimpleNamespace(tp_size=g.world_size, tp_rank=g.rank_in_group,
                         device=torch.device("cuda", torch.cuda.current_device()),
                         tp_group=g.device_group, cpu_group=g.cpu_group)
    impl = FusedArRmsNorm(ps, T, H)

    def route(x, residual, weight, eps):
        if (x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous()
                or residual.shape != x.shape or weight.dtype != torch.bfloat16):
            return None
        return impl(x, residual, weight, eps)

    install_fused_route(route)
    logger.info("fused all-reduce + RMSNorm route installed (TP %d, %d tokens)", g.world_size, T)
    return True


def _unfused(x, residual, weight, eps, group_name):
    ar = torch.ops.vllm.all_reduce(x, group_name)
    return torch.ops.vllm_ir.fused_add_rms_norm(ar, residual, weight, eps)


@torch.library.custom_op(OP, mutates_args=())
def all_reduce_fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor,
                                  weight: torch.Tensor | None, eps: float,
                                  group_name: str) -> tuple[torch.Tensor, torch.Tensor]:
    from .. import envs

    fn = _route["fn"]
    if fn is not None and weight is not None and envs.get("VLLM_B200_FUSED_AR_RMSNORM"):
        r = fn(x, residual, weight, eps)
        if r is not None:
            return r[0].clone(), r[1].clone()
    out, res = _unfused(x, residual, weight, eps, group_name)
    return out, res


@all_reduce_fused_add_rms_norm.register_fake
def _(x, residual, weight, eps, group_name):
    return torch.empty_like(x), torch.empty_like(residual)


def _targets():
    """(all_reduce, fused_add_rms_norm) op overloads, or None when vLLM's ops
    are not registered in this process."""
    try:
        return (torch.ops.vllm.all_reduce.default,
                torch.ops.vllm_ir.fused_add_rms_norm.default)
    except (AttributeError, RuntimeError):
        return None


def fuse_all_reduce_add_rms_norm(graph, targets=None) -> int:
    """Rewrite every (all-reduce -> fused add + RMSNorm) pair of ``graph``
    (a ``torch.fx.Graph`` or ``GraphModule``) in place; returns the count."""
    g = getattr(graph, "graph", graph)
    targets = targets or _targets()
    if targets is None:
        return 0
    ar_t, rms_t = targets
    fused = torch.ops.vllm_b200.all_reduce_fused_add_rms_norm.default
    n = 0
    for node in list(g.nodes):
        if node.op != "call_function" or node.target is not rms_t:
            continue
        args = list(node.args) + [None] * (4 - len(node.args))
        kw = dict(node.kwargs)
        x = kw.get("x", args[0])
        residual = kw.get("x_residual", args[1])
        weight = kw.get("weight", args[2])
        eps = kw.get("epsilon", args[3])
        if kw.get("variance_size") is not None or len(node.args) > 4:
            continue  # partial-width variance: not the layer pattern
        if (not isinstance(x, torch.fx.Node) or x.op != "call_function" or x.target is not ar_t
                or len(x.users) != 1):
            continue
        src, group = (list(x.args) + [x.kwargs.get("group_name")])[:2]
        if "group_name" in x.kwargs:
            group = x.kwargs["group_name"]
        with g.inserting_before(node):
            new = g.call_function(fused, (src, residual, weight, eps, group))
        new.meta.update(node.meta)
        node.replace_all_uses_with(new)
        g.erase_node(node)
        g.erase_node(x)
        n += 1
    if n:
        g.lint()
        if hasattr(graph, "recompile"):
            graph.recompile()
    return n
