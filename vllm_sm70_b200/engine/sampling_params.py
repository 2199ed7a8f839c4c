"""Sampling parameters and request outputs (the ``vllm.SamplingParams`` /
``RequestOutput`` subset this runtime serves)."""
from __future__ import annotations

from dataclasses import dataclass, field

from .structured import StructuredOutputsParams


@dataclass
class SamplingParams:
    max_tokens: int = 16
    n: int = 1                            # samples per prompt (LLM.generate)
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    seed: int | None = None
    ignore_eos: bool = False
    stop_token_ids: list[int] = field(default_factory=list)
    stop: list[str] = field(default_factory=list)   # stop strings (needs a tokenizer)
    include_stop_str_in_output: bool = False
    min_tokens: int = 0                              # stop tokens / strings ignored before
    min_p: float = 0.0                   # drop tokens below min_p x the top probability
    repetition_penalty: float = 1.0      # > 1 discourages prompt / output tokens
    presence_penalty: float = 0.0        # subtracted once per token present in the output
    frequency_penalty: float = 0.0       # subtracted per occurrence in the output
    logit_bias: dict[int, float] | None = None   # {token id: added to its logit}
    allowed_token_ids: list[int] | None = None   # only these tokens can be sampled
    structured_outputs: StructuredOutputsParams | None = None  # grammar-constrained output
    bad_words: list[str] | None = None   # words whose last token is banned after their prefix
    truncate_prompt_tokens: int | None = None  # keep only the prompt's last k tokens
    detokenize: bool = True              # fill RequestOutput.text (needs a tokenizer)
    skip_special_tokens: bool = True     # ... without special tokens
    # vLLM's per-request ``priority`` (lower = sooner) under
    # LLM(scheduling_policy="priority"); generate(priority=[...]) sets it
    priority: int = 0
    logprobs: int | None = None          # per output token: its log-prob + the top-N
    prompt_logprobs: int | None = None   # per prompt token (the first has none) + top-N

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0 or self.top_k == 1


@dataclass
class CompletionOutput:
    """vLLM's per-sample view (``RequestOutput.outputs[i]``)."""
    index: int
    text: str | None
    token_ids: list[int]
    logprobs: list | None = None
    finish_reason: str | None = None
    stop_reason: int | str | None = None


@dataclass
class RequestOutput:
    request_id: int
    prompt_token_ids: list[int]
    output_token_ids: list[int]
    finished: bool = True
    ttft_s: float | None = None
    tpot_s: float | None = None
    error: str | None = None       # set when the request could not be served
    # {token id: log-prob} per output / prompt token (the chosen token and the
    # top-N of the model's raw distribution); None when not requested
    logprobs: list | None = None
    prompt_logprobs: list | None = None
    text: str | None = None        # the decoded output, when the engine has a tokenizer
    more: list | None = None       # samples 2..n (RequestOutput each) when n > 1
    # vLLM's reasons: "stop" (a stop token or string ended the output; stop_reason
    # is that token id or string) or "length" (max_tokens reached)
    finish_reason: str | None = None
    stop_reason: int | str | None = None

    @property
    def outputs(self) -> list[CompletionOutput]:
        """vLLM's shape: ``outputs[i].text`` / ``outputs[i].token_ids``, one
        entry per sample."""
        out = []
        for i, o in enumerate([self] + list(self.more or [])):
            reason = "abort" if o.error == "aborted" else ("error" if o.error else o.finish_reason)
            out.append(CompletionOutput(i, o.text, o.output_token_ids, o.logprobs, reason,
                                        None if o.error else o.stop_reason))
        return out
