"""Inference runtime: ``LLM`` entry point, scheduler, model runner, KV blocks."""
from .llm import LLM  # noqa: F401
from .sampling_params import CompletionOutput, RequestOutput, SamplingParams  # noqa: F401
from .structured import StructuredOutputsParams  # noqa: F401
from .beam_search import BeamSearchOutput, BeamSearchParams  # noqa: F401
