"""Structured outputs: grammar-constrained decoding for the in-repo engine.

A request with ``SamplingParams(structured_outputs=StructuredOutputsParams(...))``
samples only tokens its grammar allows. The request forms are vLLM's
(``json`` schema, ``regex``, ``choice``, EBNF ``grammar``, ``json_object``);
grammars are compiled by xgrammar against the engine's tokenizer, the same
library vLLM uses by default. Per request, an xgrammar matcher tracks the
output so far and writes the next token's allow-list as a bitmask row (bit
``t % 32`` of word ``t // 32`` set = token ``t`` allowed). The model runner
applies that row to each rank's fp32 logit shard on the candidate-sampling
path (disallowed tokens to -inf) before ``allowed_token_ids``, ``logit_bias``
and the penalties. After every sampled token the scheduler feeds the new
tokens to the matcher and uploads the next row, so a constrained request
decodes one step per burst; a matcher that reaches its grammar's end retires
the request (finish reason "stop").

Reference parity: the reference serves structured outputs through upstream
vLLM and refuses them in its own hidden-state sampler
(``sm70/vllm_sm70/sample_v1.py:95-255``); this module gives the standalone
engine the same request surface.
"""
from __future__ import annotations

import json as _json
import re
from collections import OrderedDict
from dataclasses import dataclass

import torch


@dataclass
class StructuredOutputsParams:
    """vLLM's structured-output request (exactly one field set)."""
    json: dict | str | None = None        # JSON schema (dict or its JSON text)
    regex: str | None = None
    choice: list[str] | None = None       # the output is one of these strings
    grammar: str | None = None            # EBNF (xgrammar / GBNF syntax)
    json_object: bool | None = None       # any JSON object
    disable_any_whitespace: bool = False  # JSON without optional whitespace

    def key(self) -> tuple:
        """(kind, canonical text, compact JSON): one compiled grammar per key."""
        set_ = [(k, v) for k, v in (("json", self.json), ("regex", self.regex),
                                    ("choice", self.choice), ("grammar", self.grammar),
                                    ("json_object", self.json_object)) if v not in (None, False)]
        if len(set_) != 1:
            raise ValueError("structured_outputs needs exactly one of json, regex, choice, "
                             "grammar, json_object")
        kind, v = set_[0]
        compact = bool(self.disable_any_whitespace) or not _any_whitespace()
        if kind == "json":
            return kind, v if isinstance(v, str) else _json.dumps(v, sort_keys=True), compact
        if kind == "choice":
            if not v:
                raise ValueError("structured_outputs.choice is empty")
            return kind, "|".join(re.escape(str(c)) for c in v), compact
        return kind, "" if kind == "json_object" else str(v), compact


def _any_whitespace() -> bool:
    from .. import envs

    return bool(envs.get("VLLM_B200_STRUCTURED_ANY_WHITESPACE"))


def bitmask_words(vocab_size: int) -> int:
    return (vocab_size + 31) // 32


class GrammarCompiler:
    """Compiles and caches grammars for one tokenizer and model vocabulary."""

    def __init__(self, tokenizer, vocab_size: int, cache_size: int = 64):
        try:
            import xgrammar as xgr
        except ImportError as e:  # pragma: no cover - xgrammar ships with vLLM
            raise RuntimeError("structured outputs need the xgrammar package") from e
        self._xgr = xgr
        self.vocab_size = int(vocab_size)
        info = xgr.TokenizerInfo.from_huggingface(tokenizer, vocab_size=self.vocab_size)
        self._compiler = xgr.GrammarCompiler(info)
        self._cache: OrderedDict = OrderedDict()
        self._cache_size = cache_size

    def compile(self, so: StructuredOutputsParams):
        key = so.key()
        g = self._cache.get(key)
        if g is not None:
            self._cache.move_to_end(key)
            return g
        kind, text, compact = key
        c = self._compiler
        try:
            if kind == "json":
                g = c.compile_json_schema(text, any_whitespace=not compact)
            elif kind in ("regex", "choice"):
                g = c.compile_regex(text)
            elif kind == "grammar":
                g = c.compile_grammar(text)
            elif compact:  # any JSON object, no optional whitespace
                g = c.compile_json_schema('{"type": "object"}', any_whitespace=False)
            else:
                g = c.compile_builtin_json_grammar()
        except Exception as e:  # noqa: BLE001 - xgrammar raises several types
            raise ValueError(f"invalid structured_outputs.{kind}: {e}") from e
        self._cache[key] = g
        if len(self._cache) > self._cache_size:
            self._cache.popitem(last=False)
        return g

    def matcher(self, so: StructuredOutputsParams) -> "Guide":
        return Guide(self._xgr.GrammarMatcher(self.compile(so)), self.vocab_size)


class Guide:
    """One request's grammar state: tokens accepted so far and the bitmask
    row of the next token."""

    def __init__(self, matcher, vocab_size: int):
        self.m = matcher
        self.row = torch.full((1, bitmask_words(vocab_size)), -1, dtype=torch.int32)
        self.accepted = 0          # output tokens fed to the matcher
        self.failed = False        # a token the grammar does not allow was sampled

    def next_row(self) -> torch.Tensor:
        """The allow-list of the next token ([1, words] int32)."""
        self.m.fill_next_token_bitmask(self.row, 0)
        return self.row

    def advance(self, tokens: list[int]) -> None:
        """Feed newly sampled tokens (after the last accepted one)."""
        for t in tokens:
            if self.done:
                break
            if not self.m.accept_token(int(t)):
                self.failed = True
                break
            self.accepted += 1

    @property
    def done(self) -> bool:
        """The grammar is complete (its stop token accepted) or was violated."""
        return self.failed or self.m.is_terminated()


def mask_logits(lg: torch.Tensor, rows_bits: torch.Tensor, vocab_start: int) -> torch.Tensor:
    """``lg`` [b, V] (the shard of token ids [vocab_start, vocab_start + V))
    with every token whose bit is clear in ``rows_bits`` [b, words] set to
    -inf."""
    V = lg.shape[1]
    idx = torch.arange(vocab_start, vocab_start + V, device=lg.device)
    words = rows_bits.index_select(1, idx // 32)
    bit = torch.bitwise_and(torch.bitwise_right_shift(words, (idx % 32).to(torch.int32)), 1)
    return torch.where(bit == 0, torch.full_like(lg, float("-inf")), lg)
