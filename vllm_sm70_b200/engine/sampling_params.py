"""Sampling parameters and request outputs (the ``vllm.SamplingParams`` /
``RequestOutput`` subset this runtime serves)."""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    seed: int | None = None
    ignore_eos: bool = False
    stop_token_ids: list[int] = field(default_factory=list)

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0 or self.top_k == 1


@dataclass
class RequestOutput:
    request_id: int
    prompt_token_ids: list[int]
    output_token_ids: list[int]
    finished: bool = True
    ttft_s: float | None = None
    tpot_s: float | None = None
    error: str | None = None       # set when the request could not be served
