"""Fake (meta) kernels for ``_b200_C`` ops so they trace under
``torch.compile`` / FakeTensor mode.

Every op that returns nothing (it writes its ``Tensor(a!)`` outputs in place)
gets a no-op fake, found from the registered schemas so a new op cannot be
missed; ops that return tensors get shape rules. Host-side control and query
ops (device set-up, plan tables, status words, the NVLink collectives' pointer
lists) never appear inside a traced region: they are listed in ``NO_FAKE``
with the reason.

Reference parity: the ``register_fake`` blocks in ``sm70/vllm_sm70/ops/tm.py``
and ``ops/fv100.py:60-131`` and the reference's ``NO_FAKE_OPS`` list
(``ops/tm.py:2301``).
"""
from __future__ import annotations

import torch

LIB = "_b200_C"

# op -> why it has no fake
NO_FAKE = {
    "abi_version": "host query",
    "read_status": "host query of the device status word",
    "init_device": "device set-up",
    "gemm_configure_workspace": "device set-up",
    "gemm_set_plan": "plan table (host)",
    "gemm_clear_plans": "plan table (host)",
    "gemm_export_plans": "plan table (host)",
    "gemm_bf16_plan": "plan query (host)",
    "gemm_bf16_config": "plan query (host)",
    "gemm_set_timeline": "profiling hook",
    "attn_fa_set_timeline": "profiling hook",
    "build_prefill_meta": "host-side metadata builder (CPU tensors, data-dependent sizes)",
    "ar_rmsnorm": "NVLink collective over peer pointers (eager / CUDA-graph only)",
    "gemm_ar_rmsnorm": "GEMM + NVLink collective over peer pointers (eager / CUDA-graph only)",
    "ep_dispatch": "expert-parallel exchange over peer pointers (eager only)",
    "ep_receive": "expert-parallel exchange over peer pointers (eager only)",
    "ep_return": "expert-parallel exchange over peer pointers (eager only)",
    "ep_finish": "expert-parallel exchange over peer pointers (eager only)",
    "tp_exchange": "peer-memory collective (raw pointer lists)",
    "gemm_ag": "all-gather -> GEMM over peer memory (raw pointer lists)",
}

_done = False


def _schemas():
    return [s for s in torch._C._jit_get_all_schemas() if s.name.startswith(LIB + "::")]


def register_all() -> None:
    global _done
    if _done:
        return

    @torch.library.register_fake(f"{LIB}::gemm_bf16")
    def _gemm(a, w, cfg=-1):
        return a.new_empty(a.shape[0], w.shape[0])

    explicit = {"gemm_bf16"}
    for s in _schemas():
        name = s.name.split("::", 1)[1]
        if name in explicit or name in NO_FAKE:
            continue
        if len(s.returns) == 0:
            torch.library.register_fake(f"{LIB}::{name}")(lambda *a, **k: None)
    _done = True


def missing() -> list[str]:
    """Ops with neither a fake nor a NO_FAKE entry (must stay empty)."""
    from torch._library.simple_registry import singleton

    out = []
    for s in _schemas():
        name = s.name.split("::", 1)[1]
        if name in NO_FAKE:
            continue
        entry = singleton.find(s.name)
        if entry.fake_impl.kernel is None:
            out.append(name)
    return sorted(out)
