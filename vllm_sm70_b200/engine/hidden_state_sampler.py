"""Hidden-state sampler (platform hook U4).

``get()`` returns an object whose ``try_sample(model, hidden_states,
sampling_metadata, scheduler_output, spec_decode_metadata)`` samples directly
from the final hidden states -- greedy through the vocab-parallel LM-head
argmax (per-rank GEMM + argmax, rank-order (value, id) merge), random
sampling through the top-k candidate sampler -- or returns ``None`` to defer
to the upstream ``compute_logits`` + sampler path. Rejection reasons are
logged once each.

Reference parity: ``sm70/vllm_sm70/sample_v1.py:95-255``,
``sample_greedy.py:74-328``, ``sample.py:57-446``.
"""
from __future__ import annotations

import logging

from ..utils.logging import log_once

logger = logging.getLogger("vllm.b200.sampler")


class HiddenStateSampler:
    def __init__(self):
        self.prepared = False

    def _reject(self, reason: str):
        log_once(logger, logging.INFO, "reject:" + reason, "hidden-state sampler deferred: %s",
                 reason)
        return None

    def try_sample(self, model, sample_hidden_states, sampling_metadata, scheduler_output=None,
                   spec_decode_metadata=None):
        if spec_decode_metadata is not None:
            return self._reject("speculative decoding")
        if not self.prepared:
            return self._reject("worker not prepared")
        lm = getattr(model, "b200_greedy", None)
        if lm is None:
            return self._reject("model has no fused LM head")
        if not getattr(sampling_metadata, "all_greedy", False):
            return self._reject("non-greedy requests")
        return lm(sample_hidden_states)


_SAMPLER = HiddenStateSampler()


def get() -> HiddenStateSampler:
    return _SAMPLER


def prepare_worker(worker) -> None:
    _SAMPLER.prepared = True
