"""Runtime installation of the platform hook call sites into the installed
vLLM (the reference adds them with its patch series: ``patches/0002-0005``).

* U1: ``dispatch_unquantized_gemm()`` consults
  ``current_platform.get_unquantized_gemm(linear_backend)`` first;
* U1: ``kernel_warmup(worker)`` calls ``current_platform.kernel_warmup``
  after upstream's warm-up;
* U3: ``MoERunner._apply_quant_method`` asks
  ``current_platform.get_moe_router_provider()(runner)`` for a route; a route
  whose ``try_route(hidden_states, router_logits)`` answers replaces
  ``router.select_experts`` for that call (the reference's patch 0004 hooks
  the same runner step);
* U4: ``GPUModelRunner.execute_model`` lets
  ``current_platform.get_hidden_state_sampler()`` sample from the final hidden
  states in place of ``compute_logits`` + the upstream sampler when the batch
  has no speculative tokens and no structured output; ``_sample`` then
  returns that output (the reference's patch 0005 adds the same branch).

Without a hook (or when the platform returns None) upstream behaviour is
unchanged. ``install()`` is idempotent.
"""
from __future__ import annotations

import logging

import torch

logger = logging.getLogger("vllm.b200.hooks")
_installed: dict = {}


def b200_unquantized_gemm(layer, x: torch.Tensor, weight: torch.Tensor,
                          bias: torch.Tensor | None = None) -> torch.Tensor:
    """U1 GEMM: bf16 2-D activations on the tcgen05 kernel, else torch."""
    from ..ops import linear

    if (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and weight.dim() == 2 and x.shape[-1] % 8 == 0 and weight.shape[0] % 8 == 0):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        y = linear.gemm(x2, weight)
        if bias is not None:
            y = y + bias
        return y.view(*x.shape[:-1], weight.shape[0])
    return torch.nn.functional.linear(x, weight, bias)


def install() -> dict:
    try:
        import vllm.model_executor.layers.utils as lu
        from vllm.platforms import current_platform
    except Exception as e:  # noqa: BLE001 - vLLM not importable
        return {"error": str(e)}
    if "u1_gemm" not in _installed and hasattr(lu, "dispatch_unquantized_gemm"):
        orig = lu.dispatch_unquantized_gemm

        def dispatch_unquantized_gemm(*a, **kw):
            hook = getattr(current_platform, "get_unquantized_gemm", None)
            fn = hook(kw.get("linear_backend")) if hook is not None else None
            return fn if fn is not None else orig(*a, **kw)

        lu.dispatch_unquantized_gemm = dispatch_unquantized_gemm
        _installed["u1_gemm"] = orig
    try:
        import vllm.model_executor.warmup.kernel_warmup as kw_mod
    except Exception:  # noqa: BLE001
        kw_mod = None
    if kw_mod is not None and "u1_warmup" not in _installed:
        orig_w = kw_mod.kernel_warmup

        def kernel_warmup(worker):
            orig_w(worker)
            hook = getattr(current_platform, "kernel_warmup", None)
            if hook is not None:
                hook(worker)

        kw_mod.kernel_warmup = kernel_warmup
        _installed["u1_warmup"] = orig_w
    _install_u3(current_platform)
    _install_u4(current_platform)
    return dict(_installed)


def _install_u3(current_platform, MoERunner=None, key: str = "u3_router") -> None:
    """Wrap ``MoERunner._apply_quant_method`` (``MoERunner`` is vLLM's class
    unless a test passes another)."""
    if key in _installed:
        return
    if MoERunner is None:
        try:
            from vllm.model_executor.layers.fused_moe.runner.moe_runner import MoERunner
        except Exception:  # noqa: BLE001 - this vLLM has no MoE runner
            return
    orig = MoERunner._apply_quant_method

    def _apply_quant_method(self, layer, hidden_states, router_logits, shared_experts_input,
                            input_ids=None):
        hook = getattr(current_platform, "get_moe_router_provider", None)
        provider = hook() if hook is not None else None
        route = provider(self) if provider is not None else None
        pre = None
        if route is not None and not self._quant_method.is_monolithic:
            pre = route.try_route(hidden_states, router_logits)
        if pre is None:
            return orig(self, layer, hidden_states, router_logits, shared_experts_input,
                        input_ids)
        router = self.router
        router.select_experts = lambda *a, **k: pre  # this call only
        try:
            return orig(self, layer, hidden_states, router_logits, shared_experts_input,
                        input_ids)
        finally:
            del router.select_experts

    MoERunner._apply_quant_method = _apply_quant_method
    _installed[key] = orig


def u4_admits(scheduler_output) -> bool:
    """Batches the hidden-state sampler may take: no speculative tokens, no
    structured output (the runner applies grammar bitmasks to logits)."""
    if getattr(scheduler_output, "has_structured_output_requests", False):
        return False
    spec = getattr(scheduler_output, "scheduled_spec_decode_tokens", None)
    return not spec


def _install_u4(current_platform, GPUModelRunner=None, key: str = "u4_sampler") -> None:
    """Wrap ``GPUModelRunner.execute_model`` / ``_sample`` (vLLM's class unless
    a test passes another)."""
    if key in _installed:
        return
    if GPUModelRunner is None:
        try:
            from vllm.v1.worker.gpu_model_runner import GPUModelRunner
        except Exception:  # noqa: BLE001
            return
    orig_exec = GPUModelRunner.execute_model
    orig_sample = GPUModelRunner._sample

    def _wrap_compute_logits(runner, sampler):
        model = runner.model
        orig_cl = model.compute_logits

        def compute_logits(hidden_states, *a, **kw):
            scheduler_output = getattr(runner, "_b200_u4_ctx", None)
            if scheduler_output is not None and not a and not kw:
                out = sampler.try_sample(model, hidden_states,
                                         runner.input_batch.sampling_metadata,
                                         scheduler_output, None)
                if out is not None:
                    runner._b200_sampler_output = out
                    # Placeholder: no logits are materialised on this path.
                    return hidden_states.new_empty((hidden_states.shape[0], 0))
            return orig_cl(hidden_states, *a, **kw)

        model.compute_logits = compute_logits
        runner._b200_u4_wrapped = model

    def execute_model(self, scheduler_output, *a, **kw):
        hook = getattr(current_platform, "get_hidden_state_sampler", None)
        sampler = hook() if hook is not None else None
        if sampler is None or getattr(self, "is_pooling_model", False):
            return orig_exec(self, scheduler_output, *a, **kw)
        if getattr(self, "_b200_u4_wrapped", None) is not self.model:
            _wrap_compute_logits(self, sampler)
        self._b200_u4_ctx = scheduler_output if u4_admits(scheduler_output) else None
        try:
            return orig_exec(self, scheduler_output, *a, **kw)
        finally:
            self._b200_u4_ctx = None

    def _sample(self, logits, spec_decode_metadata):
        out = getattr(self, "_b200_sampler_output", None)
        if out is not None and spec_decode_metadata is None:
            self._b200_sampler_output = None
            self.input_batch.update_async_output_token_ids()
            return out
        return orig_sample(self, logits, spec_decode_metadata)

    GPUModelRunner.execute_model = execute_model
    GPUModelRunner._sample = _sample
    _installed[key] = (orig_exec, orig_sample)
