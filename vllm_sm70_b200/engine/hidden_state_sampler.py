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
        md = sampling_metadata
        if not getattr(md, "all_greedy", False):
            return self._reject("non-greedy requests")
        if getattr(md, "max_num_logprobs", None) is not None:
            return self._reject("log-probabilities requested")
        if not getattr(md, "no_penalties", True):
            return self._reject("sampling penalties")
        if getattr(md, "allowed_token_ids_mask", None) is not None or getattr(
                md, "bad_words_token_ids", None):
            return self._reject("allowed / bad token lists")
        lp = getattr(md, "logitsprocs", None)
        if lp is not None and list(getattr(lp, "non_argmax_invariant", []) or []):
            return self._reject("logits processors that change the argmax")
        lm = getattr(model, "b200_greedy", None)
        if lm is not None:
            return lm(sample_hidden_states)
        head = vllm_lm_head(model)
        if head is None:
            return self._reject("LM head not served (bias, soft cap, scale, quantised)")
        return greedy_sample(head, sample_hidden_states)


def vllm_lm_head(model):
    """(weight rows of this rank's original-vocabulary shard, first global id,
    TP group or None) of a vLLM causal LM whose logits are a plain bf16
    ``hidden @ W^T`` (no bias, no soft cap, scale 1, unquantised), else None."""
    import torch

    head = getattr(model, "lm_head", None)
    lp = getattr(model, "logits_processor", None)
    w = getattr(head, "weight", None)
    if w is None or lp is None or not isinstance(w, torch.Tensor) or w.dtype != torch.bfloat16:
        return None
    if getattr(head, "bias", None) is not None or getattr(lp, "soft_cap", None) is not None:
        return None
    if float(getattr(lp, "scale", 1.0)) != 1.0:
        return None
    si = getattr(head, "shard_indices", None)
    if si is None:
        return None
    start, end = int(si.org_vocab_start_index), int(si.org_vocab_end_index)
    rows = w[: end - start]
    tp = getattr(head, "tp_size", 1)
    return rows, start, tp


def greedy_sample(head, hidden):
    """Greedy tokens from the final hidden states: this rank's LM-head shard
    on the tcgen05 GEMM, the B200 argmax kernel (NaN first, max, lowest id),
    and under TP a rank-order merge of the (value, id) pairs gathered over the
    TP group -- the logits never leave the rank."""
    import torch
    from vllm.v1.outputs import SamplerOutput

    from ..ops import linear, sampling

    rows, start, tp = head
    h = hidden if hidden.dtype == torch.bfloat16 else hidden.to(torch.bfloat16)
    logits = linear.gemm(h.contiguous(), rows)
    ids, vals = sampling.argmax(logits, start)
    if tp > 1:
        from vllm.distributed import tensor_model_parallel_all_gather

        pairs = torch.stack([vals, ids.to(torch.float32)], 0)  # ids < 2^24 exact in fp32
        g = tensor_model_parallel_all_gather(pairs.unsqueeze(0), dim=0)  # [tp, 2, rows]
        ids = sampling.merge_rank_top1(g[:, 0], g[:, 1].to(torch.int32)).to(torch.int32)
    return SamplerOutput(sampled_token_ids=ids.view(-1, 1).to(torch.int32), logprobs_tensors=None)


_SAMPLER = HiddenStateSampler()


def get() -> HiddenStateSampler:
    return _SAMPLER


def prepare_worker(worker) -> None:
    _SAMPLER.prepared = True
