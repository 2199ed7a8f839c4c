"""Fake (meta) kernels for ``_b200_C`` ops so they trace under
``torch.compile`` / FakeTensor mode. Reference parity: the ``register_fake``
blocks in ``sm70/vllm_sm70/ops/tm.py`` and ``ops/fv100.py:60-131``."""
from __future__ import annotations

import torch

_done = False


def register_all() -> None:
    global _done
    if _done:
        return
    lib = "_b200_C"

    @torch.library.register_fake(f"{lib}::gemm_bf16")
    def _gemm(a, w, cfg=-1):
        return a.new_empty(a.shape[0], w.shape[0])

    for name in ("gemm_bf16_out", "gemm_bf16_silu_mul_out", "rms_norm", "fused_add_rms_norm",
                 "rope_kv_write", "paged_attention", "argmax", "silu_mul", "embedding"):
        torch.library.register_fake(f"{lib}::{name}")(lambda *a, **k: None)
    _done = True
