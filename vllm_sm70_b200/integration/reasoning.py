"""Reasoning parser for ``<think>`` / ``<tool_call>`` output (GLM-4.7 style),
registered with vLLM as ``glm47_b200``.

Two chat-template layouts are handled:

* the generation prompt leaves ``<think>`` open: the output begins inside the
  reasoning block, and ``enable_thinking=False`` / ``thinking=False`` in the
  chat-template kwargs switch extraction off (the template then closes the
  block inside the prompt);
* the generation prompt stops at ``<|assistant|>``: the model writes
  ``<think>`` itself when it reasons, so output without it is plain content
  and the thinking switches do not matter.

In both, ``</think>`` (dropped) or ``<tool_call>`` (kept, it starts the text the
tool parser reads) ends the reasoning; everything after is content. A
``</think>`` with no open block is dropped. Reasoning is returned with trailing
whitespace removed; the streaming path holds whitespace back so its pieces join
to the same text. Marker text counts as a marker in streaming only when the
marker's own token was generated. Token-level queries look at the current turn
only (after the last turn-opening special token).

The splitting logic (``ThinkSplitter``, ``ThinkTokens``) needs no tokenizer and
no vLLM; ``Glm47B200ReasoningParser`` adapts it to vLLM's ``ReasoningParser``
interface when vLLM is importable. Usage with vLLM:
``--reasoning-parser-plugin vllm_sm70_b200.integration.reasoning
--reasoning-parser glm47_b200``.

Reference parity: the ``glm47_sm70`` parser (``sm70/vllm_sm70/reasoning.py:1-328``),
component RP1; same observable behaviour, written as a state machine here.
"""
from __future__ import annotations

from collections.abc import Iterable, Sequence
from dataclasses import dataclass

THINK_OPEN = "<think>"
THINK_CLOSE = "</think>"
TOOL_OPEN = "<tool_call>"
MARKERS = (THINK_OPEN, THINK_CLOSE, TOOL_OPEN)
# Special tokens that open a turn in a rendered conversation.
TURN_TOKENS = ("<|system|>", "<|developer|>", "<|user|>", "<|assistant|>", "<|observation|>")


def template_opens_think(chat_template) -> bool | None:
    """Does the template's generation prompt leave ``<think>`` open?

    Looks at the template text after its last ``add_generation_prompt``; an
    empty ``<think></think>`` pair (thinking switched off) does not count.
    ``None`` when the template is missing or has no generation prompt.
    """
    if isinstance(chat_template, dict):
        chat_template = chat_template.get("default")
    if not isinstance(chat_template, str):
        return None
    at = chat_template.rfind("add_generation_prompt")
    if at < 0:
        return None
    return THINK_OPEN in chat_template[at:].replace(THINK_OPEN + THINK_CLOSE, "")


@dataclass
class ThinkSplitter:
    """Text-level state machine: feed text pieces in order, get each piece's
    (reasoning, content) split."""

    inside: bool          # currently inside a reasoning block
    finished: bool = False  # reasoning has ended; the rest is content

    def feed(self, text: str, allowed: Iterable[str] = MARKERS) -> tuple[str, str]:
        allowed = tuple(m for m in MARKERS if m in set(allowed))
        reasoning, content = [], []
        pos = 0
        while not self.finished and pos < len(text):
            hit, marker = len(text), ""
            for m in allowed:
                k = text.find(m, pos)
                if 0 <= k < hit:
                    hit, marker = k, m
            (reasoning if self.inside else content).append(text[pos:hit])
            pos = hit + len(marker)
            if marker == THINK_OPEN:
                self.inside = True
            elif marker:
                self.inside, self.finished = False, True
                if marker == TOOL_OPEN:
                    content.append(marker)
        if self.finished and pos < len(text):
            content.append(text[pos:])
        return "".join(reasoning), "".join(content)


class ThinkTokens:
    """Token-level queries over generated / prompt ids."""

    def __init__(self, open_id: int, close_id: int, tool_id: int | None,
                 turn_ids: Iterable[int], starts_inside: bool):
        self.open_id, self.close_id, self.tool_id = open_id, close_id, tool_id
        self.enders = {close_id} | ({tool_id} if tool_id is not None else set())
        self.turn_ids = set(turn_ids)
        self.starts_inside = starts_inside

    def turn_start(self, ids: Sequence[int]) -> int:
        for k in range(len(ids) - 1, -1, -1):
            if ids[k] in self.turn_ids:
                return k + 1
        return 0

    def reasoning_ended(self, ids: Sequence[int]) -> bool:
        """Scanning back through the current turn: an end marker before any
        ``<think>`` or turn boundary means the reasoning is over."""
        for k in range(len(ids) - 1, -1, -1):
            t = ids[k]
            if t in self.enders:
                return True
            if t == self.open_id or t in self.turn_ids:
                return False
        return False

    def content_ids(self, ids: list[int]) -> list[int]:
        start = self.turn_start(ids)
        inside = self.starts_inside
        for k in range(start, len(ids)):
            t = ids[k]
            if t == self.close_id:
                return ids[k + 1:]
            if t == self.tool_id:
                return ids[k:]
            if t == self.open_id:
                inside = True
        return [] if inside else ids[start:]

    def count_reasoning(self, ids: Sequence[int]) -> int:
        n, inside = 0, self.starts_inside
        for t in ids:
            if t in self.enders:
                break
            if t == self.open_id:
                inside = True
            elif inside:
                n += 1
        return n


def thinking_policy(chat_template, chat_kwargs: dict | None) -> tuple[bool, bool]:
    """(extraction enabled, output starts inside reasoning) for a request."""
    opens = template_opens_think(chat_template)
    model_opens = opens is False
    kw = chat_kwargs or {}
    t, e = kw.get("thinking"), kw.get("enable_thinking")
    enabled = model_opens or (t is None and e is None) or bool(t) or bool(e)
    return enabled, enabled and not model_opens


def _delta_message_cls():
    for mod in ("vllm.entrypoints.openai.engine.protocol", "vllm.entrypoints.openai.protocol",
                "vllm.entrypoints.generate.base.protocol"):
        try:
            m = __import__(mod, fromlist=["DeltaMessage"])
            return m.DeltaMessage
        except (ImportError, AttributeError):
            continue
    return None


try:  # the vLLM adapter (optional: the logic above needs no vLLM)
    from vllm.reasoning.abs_reasoning_parsers import ReasoningParser, ReasoningParserManager
except Exception:  # noqa: BLE001 - vLLM absent or incompatible
    ReasoningParser = None
    ReasoningParserManager = None

if ReasoningParser is not None:

    class Glm47B200ReasoningParser(ReasoningParser):
        """vLLM ``ReasoningParser`` over ``ThinkSplitter`` / ``ThinkTokens``."""

        def __init__(self, tokenizer, *args, **kwargs):
            super().__init__(tokenizer, *args, **kwargs)
            vocab = self.vocab
            if THINK_OPEN not in vocab or THINK_CLOSE not in vocab:
                raise RuntimeError("glm47_b200: the tokenizer has no <think> / </think> tokens")
            self.enabled, self.starts_inside = thinking_policy(
                getattr(tokenizer, "chat_template", None), kwargs.get("chat_template_kwargs"))
            self.tokens = ThinkTokens(vocab[THINK_OPEN], vocab[THINK_CLOSE], vocab.get(TOOL_OPEN),
                                      [vocab[t] for t in TURN_TOKENS if t in vocab],
                                      self.starts_inside)
            self._marker_ids = {m: vocab.get(m) for m in MARKERS}
            self._delta = _delta_message_cls()
            self._stream = ThinkSplitter(self.starts_inside)
            self._held = ""

        def adjust_request(self, request):
            request.skip_special_tokens = False  # markers must reach the parser as text
            return request

        @property
        def reasoning_start_str(self) -> str:
            return THINK_OPEN

        @property
        def reasoning_end_str(self) -> str:
            return THINK_CLOSE

        def is_reasoning_end(self, input_ids) -> bool:
            return True if not self.enabled else self.tokens.reasoning_ended(input_ids)

        def is_reasoning_end_streaming(self, input_ids, delta_ids) -> bool:
            return True if not self.enabled else any(t in self.tokens.enders for t in delta_ids)

        def extract_content_ids(self, input_ids):
            return input_ids if not self.enabled else self.tokens.content_ids(list(input_ids))

        def count_reasoning_tokens(self, token_ids) -> int:
            return 0 if not self.enabled else self.tokens.count_reasoning(token_ids)

        def extract_reasoning(self, model_output, request):
            if not self.enabled:
                return None, model_output
            r, c = ThinkSplitter(self.starts_inside).feed(model_output)
            return r.rstrip() or None, c or None

        def extract_reasoning_streaming(self, previous_text, current_text, delta_text,
                                        previous_token_ids, current_token_ids, delta_token_ids):
            if not previous_text and not previous_token_ids:
                self._stream, self._held = ThinkSplitter(self.starts_inside), ""
            if not self.enabled or self._stream.finished:
                return self._delta(content=delta_text) if delta_text else None
            allowed = MARKERS
            if delta_token_ids:
                ids = set(delta_token_ids)
                allowed = [m for m, i in self._marker_ids.items() if i is not None and i in ids]
            r, c = self._stream.feed(delta_text, allowed)
            if r:
                r = self._held + r
                kept = r.rstrip()
                self._held, r = r[len(kept):], kept
            if self._stream.finished:
                self._held = ""
            if not r and not c:
                return None
            return self._delta(reasoning=r or None, content=c or None)

    try:
        ReasoningParserManager.register_module("glm47_b200", module=Glm47B200ReasoningParser)
    except Exception:  # noqa: BLE001 - registry API differs; the class is still importable
        pass
