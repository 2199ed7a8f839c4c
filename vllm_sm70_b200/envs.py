"""Single registry of ``VLLM_B200_*`` environment variables.

Reference parity: ``sm70/vllm_sm70/envs.py:34-115`` (getter kinds) and
``:118-396`` (sections), ``:410-420`` (merge into ``vllm.envs``).

Getter kinds (same semantics as the reference):

* kill switch -- only ``"0"`` acts (turns a fused path OFF); any other value,
  or unset, leaves the default. The environment can never ENABLE something
  the typed config disabled.
* opt-in      -- only ``"1"`` acts (turns an experimental path ON).
* debug       -- ``"1"`` enables extra logging / checks.
* tuning      -- free-form string passed through to the native library.
* path        -- a filesystem path or unset.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable


@dataclass(frozen=True)
class EnvVar:
    name: str
    kind: str  # kill | optin | debug | tuning | path | int
    default: object
    section: str
    doc: str

    def get(self):
        raw = os.environ.get(self.name)
        if self.kind == "kill":
            return False if raw == "0" else bool(self.default)
        if self.kind == "optin":
            return True if raw == "1" else bool(self.default)
        if self.kind == "debug":
            return raw == "1"
        if self.kind == "int":
            try:
                return int(raw) if raw is not None else self.default
            except ValueError:
                return self.default
        return raw if raw is not None else self.default


_REGISTRY: dict[str, EnvVar] = {}


def _reg(name, kind, default, section, doc):
    _REGISTRY[name] = EnvVar(name, kind, default, section, doc)


# -- plugin ---------------------------------------------------------------
_reg("VLLM_B200_PLUGIN_STRICT", "kill", True, "plugin",
     "Fail fast when a plugin area fails to register (0 = warn only).")
_reg("VLLM_B200_PLUGIN_DEBUG", "debug", False, "plugin", "Verbose plugin logging.")
_reg("VLLM_B200_SKIP_EXT", "optin", False, "plugin",
     "Do not load _b200_C (CPU-only tests).")
# -- kernels (kill switches back to the baseline path) --------------------
_reg("VLLM_B200_GEMM", "kill", True, "kernels", "tcgen05 BF16 GEMM (0 = torch.matmul).")
_reg("VLLM_B200_GEMM_SILU_EPILOGUE", "kill", True, "kernels",
     "Fuse SiLU*up into the gate_up GEMM epilogue.")
# Read by the native library (std::getenv, once per process):
_reg("VLLM_B200_ATTN_DECODE_TMA", "kill", True, "kernels",
     "TMA-fed paged decode / spec-verify attention (0 = the cp.async kernel).")
_reg("VLLM_B200_ATTN_PREFILL_TC", "kill", True, "kernels",
     "tcgen05 prefill attention (0 = the mma.sync kernel).")
_reg("VLLM_B200_ATTN_EXP2_SPLIT", "int", 1, "kernels",
     "Ping-pong prefill attention: share of the softmax exponentials of mask-free tiles "
     "computed on the FMA pipe (0 none, 1 a quarter, 2 half; measured at 4 x 8192: 2.41 / "
     "2.22 / 2.36 ms).")
_reg("VLLM_B200_ATTN_PINGPONG", "kill", True, "kernels",
     "tcgen05 prefill attention, head_dim 128: two 128-row Q tiles per CTA with one softmax "
     "warpgroup each (0 = one Q tile per CTA).")
_reg("VLLM_B200_GEMM_EXT_REDUCE", "optin", False, "kernels",
     "Split-K GEMMs write fp32 partials to a [split][M][N] workspace and a reduction kernel "
     "sums them (measured slower than the in-kernel reduction at decode sizes).")
_reg("VLLM_B200_GEMM_SERIAL_SPLIT", "optin", False, "kernels",
     "Split-K GEMMs: the last split to arrive sums each tile and the others exit early "
     "(measured slower in decode-step chains than the shared reduction).")
_reg("VLLM_B200_GEMM_TMA_BOX", "int", 0, "kernels",
     "Rows per TMA box of the bf16 GEMM operands (0 = one box per tile; profiling aid).")
_reg("VLLM_B200_FUSED_ROUTER", "kill", True, "kernels",
     "MoE router logits (fp32) and top-k in one kernel for small batches (0 = router GEMM "
     "+ top-k kernel).")
_reg("VLLM_B200_FUSED_ROUTER_MAX_TOKENS", "int", 1024, "kernels",
     "Largest token count routed by the fused router kernel.")
_reg("VLLM_B200_RMSNORM", "kill", True, "kernels",
     "RMSNorm / fused add + RMSNorm kernels as vLLM's first IR-op provider.")
_reg("VLLM_B200_ATTN", "kill", True, "kernels", "Paged attention kernels (0 = SDPA reference).")
_reg("VLLM_B200_ROPE_KV", "kill", True, "kernels", "Fused RoPE + KV-cache write kernel.")
_reg("VLLM_B200_FP8_GEMM", "kill", True, "kernels", "Block-FP8 tcgen05 GEMM.")
_reg("VLLM_B200_FP8_W8A8", "kill", True, "kernels",
     "Block-FP8 weights run W8A8: activations quantised per token and 128-wide K group to e4m3, "
     "kind::f8f6f4 tensor-core MMAs with exact fp32 scale promotion per K block. 0 = W8A16 "
     "(weights dequantised to bf16 in the GEMM producer).")
_reg("VLLM_B200_AWQ_GEMM", "kill", True, "kernels", "AWQ int4 GEMM.")
_reg("VLLM_B200_NVFP4_GEMM", "kill", True, "kernels", "NVFP4 GEMM.")
_reg("VLLM_B200_NVFP4_W4A4", "kill", True, "kernels",
     "NVFP4 weights run W4A4: activations quantised per token (fp32 row scale) and 16-element "
     "block (e4m3 scale) to e2m1, kind::mxf4nvf4 tensor-core MMAs with the block scales in TMEM. "
     "0 = W4A16 (weights dequantised to bf16 in the GEMM producer).")
_reg("VLLM_B200_MOE", "kill", True, "kernels", "Grouped expert GEMM + router kernels.")
_reg("VLLM_B200_ROUTER", "kill", True, "kernels", "Fused MoE router (U3 provider).")
_reg("VLLM_B200_SAMPLER", "kill", True, "kernels", "Hidden-state sampler (U4 provider).")
_reg("VLLM_B200_GREEDY_FASTPATH", "kill", True, "kernels", "Vocab-parallel greedy top-1.")
_reg("VLLM_B200_GDN", "kill", True, "kernels", "Gated-DeltaNet kernels.")
_reg("VLLM_B200_GDN_CHUNK", "kill", True, "kernels",
     "Gated-DeltaNet prefill in 64-token chunks (WY/UT form on the tensor cores) instead of "
     "the token-serial recurrence (head dims 128).")
# -- collectives ----------------------------------------------------------
_reg("VLLM_B200_FUSED_AR_RMSNORM", "kill", True, "comm",
     "Fused all-reduce + residual + RMSNorm over NVLink peer memory (0 = NCCL + norm).")
_reg("VLLM_B200_FUSED_GEMM_RS", "kill", True, "comm", "Fused GEMM -> reduce-scatter.")
_reg("VLLM_B200_FUSED_AG_GEMM", "kill", True, "comm", "Fused all-gather -> GEMM.")
_reg("VLLM_B200_FUSED_EP_A2A", "kill", True, "comm", "Fused EP dispatch / combine.")
_reg("VLLM_B200_FUSED_SAMPLER_XCHG", "kill", True, "comm",
     "Vocab-parallel sampling at TP > 1: exchange the greedy (value, id) pairs / top-k "
     "candidates over NVLink peer memory in one kernel (0 = NCCL all-gather + merge).")
_reg("VLLM_B200_NVLS", "optin", False, "comm",
     "Fused all-reduce + RMSNorm through NVLS: multimem.ld_reduce sums each owned row in the "
     "NVSwitch (fp32 accumulation, order unspecified: not bitwise equal to the rank-order sum) "
     "and multimem.st writes every rank's copy, when the symmetric buffers have multicast "
     "addresses and TP >= VLLM_B200_NVLS_MIN_RANKS.")
_reg("VLLM_B200_NVLS_MIN_RANKS", "int", 4, "comm",
     "Smallest TP size that takes the NVLS all-reduce (VLLM_B200_NVLS=1).")
_reg("VLLM_B200_COMM_TIMEOUT_MS", "int", 2000, "comm",
     "Bound (ms) for every device-side flag wait in fused collectives.")
# -- runtime --------------------------------------------------------------
_reg("VLLM_B200_CUDA_GRAPHS", "kill", True, "runtime", "Capture decode steps in CUDA graphs.")
_reg("VLLM_B200_GRAPH_MAX_BS", "int", 512, "runtime", "Largest captured decode batch.")
_reg("VLLM_B200_WARMUP", "kill", True, "runtime", "Pre-capture GEMM warm-up / tuning.")
_reg("VLLM_B200_STRUCTURED_ANY_WHITESPACE", "kill", True, "runtime",
     "JSON grammars of structured outputs allow optional whitespace (0 = compact JSON for "
     "every request, like a request's disable_any_whitespace).")
_reg("VLLM_B200_STOP_CHECK_STEPS", "int", 16, "runtime",
     "Longest decode burst while a running request can end on a stop token: its new "
     "tokens are checked after each burst and a stopped request retires (0 = run "
     "every request to max_tokens and cut the output at the stop afterwards).")
_reg("VLLM_B200_GEMM_LIBRARY", "optin", False, "runtime",
     "Baseline switch, off by default: let the warm-up tuner route a plain bf16 GEMM shape to "
     "the vendor library (cuBLAS) when it measures faster than every tcgen05 plan. With it off "
     "every GEMM of the models runs the tcgen05 kernels.")
_reg("VLLM_B200_FUSED_GEMM_AR", "kill", True, "comm",
     "TP > 1: run each row-parallel GEMM (o_proj, down_proj) and the following all-reduce + "
     "residual + RMSNorm as one kernel (tcgen05 tiles, then the collective over NVLink peer "
     "memory) instead of a GEMM followed by the collective kernel, for token counts of at "
     "least VLLM_B200_FUSED_GEMM_AR_MIN_TOKENS.")
_reg("VLLM_B200_FUSED_GEMM_NORM", "optin", False, "kernels",
     "TP1: run each row GEMM (o_proj, down_proj) and the residual add + RMSNorm after it as one "
     "kernel (the fused all-reduce epilogue with one rank). Off: measured slower on the "
     "headline (9,383 vs 10,233 tok/s, same box) -- the fused launcher is limited to non-pair "
     "tiles and its grid barrier costs more than the norm kernel it removes.")
_reg("VLLM_B200_FUSED_GEMM_AR_MIN_TOKENS", "int", 1, "comm",
     "Smallest token count that takes the fused GEMM + all-reduce kernel (measured at TP2 on "
     "Llama-3.1-8B shapes with every GEMM on the tcgen05 kernels: the fused kernel is as fast or "
     "faster at 256-row decode steps and 16384-token prefill chunks).")
_reg("VLLM_B200_PREFIX_CACHING", "optin", False, "runtime",
     "Reuse the KV of full prompt blocks across requests with the same token prefix "
     "(LLM(enable_prefix_caching=...) overrides).")
_reg("VLLM_B200_PREFIX_HOST_BLOCKS", "int", 0, "runtime",
     "Prefix caching: KV blocks kept in pinned host memory after eviction from the device "
     "(0 = no host tier).")
_reg("VLLM_B200_PREFIX_DISK_DIR", "path", None, "runtime",
     "Prefix caching: directory of a persistent KV tier (every cached prompt block is also "
     "written there, one file per block, and found again by later engine processes of the "
     "same model / layout / rank). Unset = no disk tier.")
_reg("VLLM_B200_PREFIX_DISK_BLOCKS", "int", 65536, "runtime",
     "Prefix caching: blocks kept in the disk tier (least recently used files deleted).")
_reg("VLLM_B200_NVTX", "optin", False, "runtime",
     "Emit NVTX ranges per layer and engine phase for profiler timelines.")
_reg("VLLM_B200_WATCHDOG_S", "int", 0, "runtime",
     "Seconds a prefill chunk / decode burst may stay pending on the GPU before the engine "
     "raises (0 = no watchdog).")
_reg("VLLM_B200_PDL", "kill", True, "runtime",
     "Launch the decode-path kernels with programmatic dependent launch (read by the native "
     "library at load).")
_reg("VLLM_B200_GEMM_LUT_PATH", "path", None, "runtime", "Tuned GEMM config table to import.")
_reg("VLLM_B200_GEMM_LUT_EXPORT_PATH", "path", None, "runtime", "Where to export the table.")
_reg("VLLM_B200_GEMM_LUT_STRICT", "optin", False, "runtime",
     "Refuse a LUT whose manifest does not match this build / GPU.")


def get(name: str):
    return _REGISTRY[name].get()


def registry() -> dict[str, EnvVar]:
    return dict(_REGISTRY)


def sections() -> dict[str, list[str]]:
    out: dict[str, list[str]] = {}
    for v in _REGISTRY.values():
        out.setdefault(v.section, []).append(v.name)
    return out


def compile_factors() -> dict[str, object]:
    """Values that change generated code / graphs; hashed into cache keys."""
    return {k: v.get() for k, v in sorted(_REGISTRY.items()) if v.kind in ("kill", "optin")}


def merge_into_vllm() -> int:
    """Expose the getters through ``vllm.envs`` (when vLLM is importable) so
    its environment validation and compile hashing see them. Returns the
    number of names merged (0 without vLLM)."""
    try:
        import vllm.envs as venvs  # type: ignore
    except Exception:  # noqa: BLE001 - vLLM is optional for the core library
        return 0
    table = getattr(venvs, "environment_variables", None)
    if not isinstance(table, dict):
        return 0
    n = 0
    for name, var in _REGISTRY.items():
        if name not in table:
            table[name] = _getter(var)
            n += 1
    return n


def _getter(var: EnvVar) -> Callable[[], object]:
    return lambda: var.get()
