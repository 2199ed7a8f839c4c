"""Beam search over the engine's public API (vLLM's ``LLM.beam_search``).

Every step runs one ``generate`` call over all live beams of all prompts with
``max_tokens=1`` and ``logprobs=2 * beam_width``: the teacher-forced
log-probabilities of each beam's next token (the raw distribution) give the
candidate extensions. Per prompt, candidates that end in the tokenizer's EOS
(unless ``ignore_eos``) move to the finished list, the others are ranked by
their score and the best ``beam_width`` continue. At the end the finished and
live beams are ranked together. The score is vLLM's: cumulative log-prob
divided by ``len(tokens) ** length_penalty``, with ``tokens`` the prompt plus
the output and a final EOS not counted. With prefix caching on, each step's
prefill reuses the beams' cached prompt blocks.

Reference parity: the reference serves beam search through upstream vLLM
(``vllm/entrypoints/llm.py`` ``LLM.beam_search``); this is the same request
surface on the in-repo engine.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .sampling_params import SamplingParams


@dataclass
class BeamSearchParams:
    beam_width: int
    max_tokens: int
    ignore_eos: bool = False
    temperature: float = 0.0
    length_penalty: float = 1.0


@dataclass
class BeamSearchSequence:
    tokens: list[int]                 # prompt + output
    cum_logprob: float = 0.0
    logprobs: list = field(default_factory=list)  # {token id: log-prob} per output token
    text: str | None = None
    finished: bool = False


@dataclass
class BeamSearchOutput:
    sequences: list[BeamSearchSequence]


def beam_score(tokens: list[int], cum_logprob: float, eos: int | None,
               length_penalty: float) -> float:
    n = len(tokens) - (1 if eos is not None and tokens and tokens[-1] == eos else 0)
    return cum_logprob / (max(n, 1) ** length_penalty)


def beam_search(llm, prompts, params: BeamSearchParams) -> list[BeamSearchOutput]:
    """``prompts``: token-id lists / tensors, strings (needs a tokenizer) or
    vLLM's prompt dicts."""
    W = int(params.beam_width)
    if W < 1 or params.max_tokens < 1:
        raise ValueError("beam_width and max_tokens must be >= 1")
    tok = llm.tokenizer
    eos = None if params.ignore_eos or tok is None else getattr(tok, "eos_token_id", None)
    starts = [[int(t) for t in llm._prompt_ids(p)] for p in prompts]
    beams = [[BeamSearchSequence(list(s))] for s in starts]
    done: list[list[BeamSearchSequence]] = [[] for _ in starts]
    sp = SamplingParams(max_tokens=1, logprobs=2 * W, temperature=params.temperature,
                        ignore_eos=True)

    def key(b):
        return beam_score(b.tokens, b.cum_logprob, eos, params.length_penalty)

    for _ in range(params.max_tokens):
        flat = [(i, b) for i, bs in enumerate(beams) for b in bs]
        if not flat:
            break
        outs = llm.generate([b.tokens for _, b in flat], sp, collect_stats=False)
        cands: list[list[BeamSearchSequence]] = [[] for _ in starts]
        for (i, b), o in zip(flat, outs):
            for t, lp in o.logprobs[0].items():
                nb = BeamSearchSequence(b.tokens + [int(t)], b.cum_logprob + float(lp),
                                        b.logprobs + [o.logprobs[0]])
                if eos is not None and int(t) == eos:
                    nb.finished = True
                    done[i].append(nb)
                else:
                    cands[i].append(nb)
        beams = [sorted(c, key=key, reverse=True)[:W] for c in cands]
    results = []
    for i, s in enumerate(starts):
        best = sorted(done[i] + beams[i], key=key, reverse=True)[:W]
        if tok is not None:
            for b in best:
                b.text = tok.decode(b.tokens[len(s):], skip_special_tokens=True)
        results.append(BeamSearchOutput(best))
    return results
