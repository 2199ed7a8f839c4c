"""Reasoning parser (``<think>`` / ``<tool_call>``): both chat-template layouts,
streaming vs one-shot agreement, token-level queries. CPU only."""
import pytest

from vllm_sm70_b200.integration import reasoning as R

OPENS = "{% if add_generation_prompt %}<|assistant|><think>{% endif %}"
STOPS = "{% if add_generation_prompt %}<|assistant|>{% endif %}"
OFF = "{% if add_generation_prompt %}<|assistant|><think></think>{% endif %}"


def test_template_detection():
    assert R.template_opens_think(OPENS) is True
    assert R.template_opens_think(STOPS) is False
    assert R.template_opens_think(OFF) is False
    assert R.template_opens_think({"default": OPENS}) is True
    assert R.template_opens_think(None) is None
    assert R.template_opens_think("no prompt here") is None


def test_policy():
    assert R.thinking_policy(OPENS, None) == (True, True)
    assert R.thinking_policy(OPENS, {"enable_thinking": False}) == (False, False)
    # the model opens <think> itself: switches do not matter, output starts as content
    assert R.thinking_policy(STOPS, {"enable_thinking": False}) == (True, False)
    assert R.thinking_policy(None, None) == (True, True)


@pytest.mark.parametrize("inside,text,want", [
    (True, "plan it</think>answer", ("plan it", "answer")),
    (True, "plan  \n</think>answer", ("plan  \n", "answer")),
    (False, "just an answer", ("", "just an answer")),
    (False, "<think>hmm</think>ok", ("hmm", "ok")),
    (True, "look up<tool_call>{\"n\":1}</tool_call>", ("look up", "<tool_call>{\"n\":1}</tool_call>")),
    (False, "stray</think>rest", ("", "strayrest")),
    (True, "a</think>b</think>c", ("a", "b</think>c")),
])
def test_splitter(inside, text, want):
    assert R.ThinkSplitter(inside).feed(text) == want


def test_streaming_matches_one_shot():
    text = "<think>step one\n\nstep two  \n</think>\nfinal <think>not markup"
    whole = R.ThinkSplitter(False).feed(text)
    for cut in range(1, 7):
        sp = R.ThinkSplitter(False)
        r = c = ""
        # split at marker boundaries so each marker arrives whole (as one token would)
        pieces = ["<think>", "step one\n", "\nstep two  \n", "</think>", "\nfinal ", "<think>not markup"]
        for p in pieces[:cut] + ["".join(pieces[cut:])]:
            a, b = sp.feed(p)
            r, c = r + a, c + b
        assert (r, c) == whole


def test_marker_text_without_its_token_is_plain():
    sp = R.ThinkSplitter(True)
    assert sp.feed("quoting </think> literally", allowed=()) == ("quoting </think> literally", "")
    assert not sp.finished


def _toks():
    # ids: <think>=1 </think>=2 <tool_call>=3 <|user|>=4 <|assistant|>=5, text tokens >= 10
    return R.ThinkTokens(1, 2, 3, [4, 5], starts_inside=True)


def test_token_queries():
    t = _toks()
    # an earlier turn's </think> does not end the current turn's reasoning
    assert not t.reasoning_ended([4, 10, 2, 11, 5, 12, 13])
    assert t.reasoning_ended([5, 12, 13, 2])
    assert t.reasoning_ended([5, 12, 3])
    assert not t.reasoning_ended([5, 1, 12])
    assert t.content_ids([5, 12, 13, 2, 20, 21]) == [20, 21]
    assert t.content_ids([5, 12, 3, 30]) == [3, 30]
    assert t.content_ids([5, 12, 13]) == []
    assert t.count_reasoning([12, 13, 14, 2, 20]) == 3
    t2 = R.ThinkTokens(1, 2, 3, [4, 5], starts_inside=False)
    assert t2.content_ids([5, 12, 13]) == [12, 13]
    assert t2.count_reasoning([12, 1, 13, 14, 2]) == 2


def test_vllm_adapter_registered():
    if R.ReasoningParser is None:
        pytest.skip("vLLM reasoning API not importable")

    class Tok:
        chat_template = STOPS

        def get_vocab(self):
            return {"<think>": 1, "</think>": 2, "<tool_call>": 3, "<|user|>": 4,
                    "<|assistant|>": 5, "a": 10}

    p = R.Glm47B200ReasoningParser(Tok())
    assert p.extract_reasoning("<think>why  </think>because", None) == ("why", "because")
    assert p.extract_reasoning("plain", None) == (None, "plain")
    d1 = p.extract_reasoning_streaming("", "<think>x ", "<think>x ", [], [1, 10], [1, 10])
    assert d1.reasoning == "x"
    d2 = p.extract_reasoning_streaming("<think>x ", "<think>x y", "y", [1, 10], [1, 10, 10], [10])
    assert d2.reasoning == " y"
