"""Typed runtime policy ``B200Config``.

Read from vLLM's ``additional_config["b200"]`` (``"sm70"`` is accepted as an
alias so reference deployments keep working) or constructed directly. Frozen,
``extra="forbid"``: unknown keys are an error. Kill switches in the
environment (``envs.py``, kind ``kill``) can only turn a field OFF; the
environment can never enable something the config disabled. Only the
``GRAPH_FIELDS`` change captured graphs / compiled code and feed
:meth:`compute_hash`.

Reference parity: ``sm70/vllm_sm70/config/__init__.py:42-454`` (``Sm70Config``,
``GRAPH_FIELDS``, ``sm70_config()`` cached per ``VllmConfig``, frozen
``CONSTANTS``).
"""
from __future__ import annotations

import hashlib
import json
import weakref

from pydantic import BaseModel, ConfigDict, Field

from .. import envs

# Frozen tuning constants (not user knobs).
CONSTANTS = {
    "gemm_block_m": 128,
    "gemm_block_k": 64,
    "gemm_workspace_bytes": 64 << 20,
    "gemm_workspace_counters": 16384,
    "attn_decode_key_tile": 64,
    "attn_prefill_key_tile": 64,
    "decode_split_target_waves": 2,
    "comm_wait_timeout_ms": 2000,
    "moe_gate_up_block": 64,
}

# Kill switch env var -> field it can disable.
_KILL_MAP = {
    "VLLM_B200_GEMM": "gemm",
    "VLLM_B200_GEMM_SILU_EPILOGUE": "gemm_silu_epilogue",
    "VLLM_B200_ATTN": "attention",
    "VLLM_B200_ROPE_KV": "rope_kv_fusion",
    "VLLM_B200_FP8_GEMM": "fp8_gemm",
    "VLLM_B200_AWQ_GEMM": "awq_gemm",
    "VLLM_B200_NVFP4_GEMM": "nvfp4_gemm",
    "VLLM_B200_MOE": "moe",
    "VLLM_B200_ROUTER": "fused_router",
    "VLLM_B200_SAMPLER": "hidden_state_sampler",
    "VLLM_B200_GREEDY_FASTPATH": "greedy_fastpath",
    "VLLM_B200_GDN": "gdn",
    "VLLM_B200_FUSED_AR_RMSNORM": "fused_ar_rmsnorm",
    "VLLM_B200_FUSED_GEMM_RS": "fused_gemm_rs",
    "VLLM_B200_FUSED_AG_GEMM": "fused_ag_gemm",
    "VLLM_B200_FUSED_EP_A2A": "fused_ep_a2a",
    "VLLM_B200_CUDA_GRAPHS": "cuda_graphs",
    "VLLM_B200_WARMUP": "warmup",
}

GRAPH_FIELDS = ("gemm", "gemm_silu_epilogue", "attention", "rope_kv_fusion", "fp8_gemm",
                "awq_gemm", "nvfp4_gemm", "moe", "fused_router", "gdn", "fused_ar_rmsnorm",
                "fused_gemm_rs", "fused_ag_gemm", "fused_ep_a2a", "cuda_graphs",
                "graph_max_batch", "block_size")


class B200Config(BaseModel):
    model_config = ConfigDict(frozen=True, extra="forbid")

    gemm: bool = True
    gemm_silu_epilogue: bool = True
    attention: bool = True
    rope_kv_fusion: bool = True
    fp8_gemm: bool = True
    awq_gemm: bool = True
    nvfp4_gemm: bool = True
    moe: bool = True
    fused_router: bool = True
    hidden_state_sampler: bool = True
    greedy_fastpath: bool = True
    gdn: bool = True
    fused_ar_rmsnorm: bool = True
    fused_gemm_rs: bool = True
    fused_ag_gemm: bool = True
    fused_ep_a2a: bool = True
    cuda_graphs: bool = True
    warmup: bool = True
    graph_max_batch: int = Field(512, ge=1, le=4096)
    block_size: int = Field(16, ge=8, le=1024)
    gemm_lut_path: str | None = None
    strict: bool = True

    def with_env(self) -> "B200Config":
        """Apply kill switches: only turns fields OFF."""
        off = {f: False for var, f in _KILL_MAP.items() if not envs.get(var)}
        upd = {k: v for k, v in off.items() if getattr(self, k)}
        if not envs.get("VLLM_B200_PLUGIN_STRICT"):
            upd["strict"] = False
        return self.model_copy(update=upd) if upd else self

    def compute_hash(self) -> str:
        d = {f: getattr(self, f) for f in GRAPH_FIELDS}
        return hashlib.sha256(json.dumps(d, sort_keys=True).encode()).hexdigest()[:16]


_cache: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()
_default: B200Config | None = None


def _raw_from_vllm(vllm_config) -> dict:
    add = getattr(vllm_config, "additional_config", None) or {}
    if isinstance(add, dict):
        for key in ("b200", "sm70"):
            if key in add and isinstance(add[key], dict):
                return dict(add[key])
    return {}


def b200_config(vllm_config=None) -> B200Config:
    """Typed policy for a ``VllmConfig`` (cached per object) or the default."""
    global _default
    if vllm_config is None:
        if _default is None:
            _default = B200Config().with_env()
        return _default
    try:
        hit = _cache.get(vllm_config)
    except TypeError:
        hit = None
    if hit is not None:
        return hit
    cfg = B200Config(**_raw_from_vllm(vllm_config)).with_env()
    try:
        _cache[vllm_config] = cfg
    except TypeError:
        pass
    return cfg
