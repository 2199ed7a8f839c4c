"""BF16 GEMM wrappers over the tcgen05 kernel (``_b200_C::gemm_bf16*``).

Reference parity: the TurboMind f16 ops ``sm70_f16_gemm{,_out}`` and the
gated-SiLU epilogue (``sm70/csrc/turbomind/ops/tm_f16_sm70.cu:351-365``,
wrappers ``sm70/vllm_sm70/ops/tm.py:35-50``). On B200 the weight needs no
repack for the plain GEMM (the kernel TMA-loads K-major rows directly); the
fused SiLU epilogue wants the gate/up rows interleaved in 64-row blocks,
produced once at load time by :func:`interleave_gate_up`.
"""
from __future__ import annotations

import torch

from .. import _ext, envs
from ..utils import launch_count

GATE_UP_BLOCK = 64


def _use_native(t: torch.Tensor) -> bool:
    if not t.is_cuda:
        return False
    if not envs.get("VLLM_B200_GEMM"):
        return False
    _ext.require()
    return True


DEFAULT_WS_BYTES = 64 << 20
DEFAULT_WS_COUNTERS = 16384
_ws_configured: set = set()


def configure_workspace(device: int, ws_bytes: int = DEFAULT_WS_BYTES,
                        n_counters: int = DEFAULT_WS_COUNTERS) -> None:
    """Allocate the per-device split-K workspace (fp32 partial tiles + arrival
    counters). Call once at start-up, before any CUDA-graph capture; GEMMs
    planned with split-K fall back to one split when it is absent or too small.
    Reference parity: ``sm70_gemm_configure_workspace``
    (``sm70/csrc/turbomind/ops/gemm_runtime.cpp:825-897``)."""
    _ext.require()
    torch.ops._b200_C.gemm_configure_workspace(device, ws_bytes, n_counters)
    _ws_configured.add(device)


def plan(M: int, N: int, K: int, epi: int = 0, num_sm: int | None = None) -> tuple[int, int]:
    """(tile config, split-K) chosen by the native planner (for the current
    device's SM count unless ``num_sm`` is given)."""
    _ext.require()
    if num_sm is None:
        num_sm = (torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
                  if torch.cuda.is_available() else 148)
    c, s = torch.ops._b200_C.gemm_bf16_plan(M, N, K, epi, num_sm)
    return int(c), int(s)


# Plain bf16 GEMM shapes (M, N, K) for which the warm-up tuner measured the
# vendor library (cuBLAS through torch.mm) faster than every tcgen05 plan;
# fused, quantised and grouped GEMMs always run the tcgen05 kernels.
LIBRARY_CFG = -2
_LIBRARY: set = set()
_LIBRARY_SILU: set = set()  # gate_up shapes: library GEMM + interleaved SiLU kernel


def set_library(M: int, N: int, K: int, on: bool = True, epi: int = 0) -> None:
    target = _LIBRARY_SILU if epi else _LIBRARY
    (target.add if on else target.discard)((int(M), int(N), int(K)))


def clear_library() -> None:
    _LIBRARY.clear()
    _LIBRARY_SILU.clear()


def library_shapes(epi: int = 0) -> list[tuple[int, int, int]]:
    return sorted(_LIBRARY_SILU if epi else _LIBRARY)


def gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
         cfg: int = -1, splits: int = 0) -> torch.Tensor:
    """``x[M, K] @ w[N, K].T`` in bf16 with fp32 accumulation."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    if (cfg < 0 and splits <= 0 and _LIBRARY and x.is_cuda
            and (x.shape[0], w.shape[0], x.shape[1]) in _LIBRARY):
        torch.mm(x, w.t(), out=out)
        return out
    if _use_native(x):
        torch.ops._b200_C.gemm_bf16_out(out, x, w, cfg, splits)
        launch_count.add(1)
    else:
        out.copy_((x.float() @ w.float().t()).to(out.dtype))
    return out


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """Stack gate/up rows as [g0..g63, u0..u63, g64..g127, u64..u127, ...]."""
    n, k = w_gate.shape
    assert w_up.shape == (n, k) and n % GATE_UP_BLOCK == 0, (w_gate.shape, w_up.shape)
    g = w_gate.reshape(n // GATE_UP_BLOCK, GATE_UP_BLOCK, k)
    u = w_up.reshape(n // GATE_UP_BLOCK, GATE_UP_BLOCK, k)
    return torch.stack([g, u], dim=1).reshape(2 * n, k).contiguous()


def deinterleave_gate_up(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    n2, k = w.shape
    v = w.reshape(n2 // (2 * GATE_UP_BLOCK), 2, GATE_UP_BLOCK, k)
    return v[:, 0].reshape(n2 // 2, k), v[:, 1].reshape(n2 // 2, k)


def silu_mul_ref(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    g = gate.float()
    return (g * torch.sigmoid(g) * up.float()).to(gate.dtype)


def gemm_silu_mul(x: torch.Tensor, w_interleaved: torch.Tensor,
                  out: torch.Tensor | None = None, cfg: int = -1) -> torch.Tensor:
    """``silu(x @ w_gate.T) * (x @ w_up.T)`` with the activation fused in the
    GEMM epilogue. ``w_interleaved`` comes from :func:`interleave_gate_up`."""
    n = w_interleaved.shape[0] // 2
    if out is None:
        out = torch.empty(x.shape[0], n, dtype=x.dtype, device=x.device)
    M, K = x.shape
    if (cfg < 0 and _LIBRARY_SILU and x.is_cuda
            and (M, w_interleaved.shape[0], K) in _LIBRARY_SILU):
        # Tuner's choice for this shape: vendor GEMM on the interleaved weights,
        # then the interleaved SiLU*up kernel.
        gu = torch.mm(x, w_interleaved.t())
        torch.ops._b200_C.silu_mul(out, gu, GATE_UP_BLOCK)
        launch_count.add(1)
        return out
    if _use_native(x) and envs.get("VLLM_B200_GEMM_SILU_EPILOGUE"):
        torch.ops._b200_C.gemm_bf16_silu_mul_out(out, x, w_interleaved, cfg)
        launch_count.add(1)
        return out
    wg, wu = deinterleave_gate_up(w_interleaved)
    if _use_native(x):
        gu = torch.empty(x.shape[0], 2 * n, dtype=x.dtype, device=x.device)
        gemm(x, torch.cat([wg, wu], 0), out=gu)
        torch.ops._b200_C.silu_mul(out, gu)
        launch_count.add(1)
        return out
    g = x.float() @ wg.float().t()
    u = x.float() @ wu.float().t()
    out.copy_((g * torch.sigmoid(g) * u).to(out.dtype))
    return out


def silu_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x = [gate | up]`` -> ``silu(gate) * up``."""
    n = x.shape[-1] // 2
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    if x.is_cuda:
        _ext.require()
        torch.ops._b200_C.silu_mul(out, x)
        launch_count.add(1)
    else:
        out.copy_(silu_mul_ref(x[..., :n], x[..., n:]))
    return out
