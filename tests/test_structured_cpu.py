"""Structured outputs on CPU: greedy decoding under a grammar equals a dense
reference that masks the logits with an independent xgrammar matcher; every
output is accepted by its grammar (choice, regex, JSON schema, EBNF, JSON
object); requests without a grammar in the same batch are unchanged; a
completed grammar retires the request; bad grammars are refused."""
import json

import pytest
import torch

from vllm_sm70_b200.engine import LLM, SamplingParams, StructuredOutputsParams

from ._llama_ref import llama_logits
from .test_engine_cpu import TINY

xgr = pytest.importorskip("xgrammar")


def _tokenizer():
    """Byte-level tokenizer of the tiny model's 512-token vocabulary: the 256
    bytes, an end-of-sequence token (256) and unused specials."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    chars = sorted(pre_tokenizers.ByteLevel.alphabet())
    tk = Tokenizer(models.BPE(vocab={c: i for i, c in enumerate(chars)}, merges=[]))
    tk.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tk.decoder = decoders.ByteLevel()
    tk.add_special_tokens(["<eos>"] + [f"<x{i}>" for i in range(512 - 257)])
    return PreTrainedTokenizerFast(tokenizer_object=tk, eos_token="<eos>")


TOK = _tokenizer()


def _llm():
    return LLM(TINY, max_num_seqs=4, max_model_len=160, block_size=16, dtype=torch.float32,
               enforce_eager=True, max_num_batched_tokens=64, tokenizer=TOK)


def _dense_guided(llm, prompt, so, n):
    """Greedy decoding with the grammar's mask applied to a dense forward."""
    g = llm._grammars().compile(so)
    m = xgr.GrammarMatcher(g)
    bm = xgr.allocate_token_bitmask(1, TINY.vocab_size)
    ids, out = prompt.clone(), []
    for _ in range(n):
        m.fill_next_token_bitmask(bm, 0)
        lg = llama_logits(llm.model, ids)[-1].clone()
        for t in range(lg.numel()):
            if not (int(bm[0, t // 32]) >> (t % 32)) & 1:
                lg[t] = float("-inf")
        t = int(lg.argmax())
        out.append(t)
        assert m.accept_token(t)
        ids = torch.cat([ids, torch.tensor([t])])
        if m.is_terminated():
            break
    return out


def _prompt(n=9, seed=5):
    return torch.randint(0, 256, (n,), generator=torch.Generator().manual_seed(seed))


def test_guided_greedy_equals_dense_reference():
    llm = _llm()
    p = _prompt()
    eos = TOK.eos_token_id
    so = StructuredOutputsParams(choice=["alpha", "beta", "gamma"])
    plain = llm.generate([p], SamplingParams(max_tokens=10, ignore_eos=True))[0]
    got = llm.generate([p, p], [SamplingParams(max_tokens=20, structured_outputs=so),
                                SamplingParams(max_tokens=10, ignore_eos=True)])
    want = _dense_guided(llm, p, so, 20)
    assert got[0].output_token_ids == want and want[-1] == eos
    assert got[0].outputs[0].text in ("alpha", "beta", "gamma")
    assert got[0].outputs[0].finish_reason == "stop"
    assert got[1].output_token_ids == plain.output_token_ids


@pytest.mark.parametrize("so,check", [
    (StructuredOutputsParams(regex=r"[0-9]{3}-[a-z]{2}"),
     lambda t: len(t) == 6 and t[:3].isdigit() and t[3] == "-" and t[4:].isalpha()),
    (StructuredOutputsParams(json={"type": "object", "properties": {
        "ok": {"type": "boolean"}, "n": {"type": "integer", "minimum": 0, "maximum": 9}},
        "required": ["ok", "n"], "additionalProperties": False}),
     lambda t: set(json.loads(t)) == {"ok", "n"} and isinstance(json.loads(t)["ok"], bool)),
    (StructuredOutputsParams(grammar='root ::= ("yes" | "no") " " [0-9]'),
     lambda t: t.split(" ")[0] in ("yes", "no") and t[-1].isdigit()),
])
def test_outputs_follow_their_grammar(so, check):
    """Sampled (temperature 1) outputs complete and satisfy the grammar."""
    llm = _llm()
    sp = SamplingParams(max_tokens=60, temperature=1.0, seed=3, structured_outputs=so,
                        stop_token_ids=[TOK.eos_token_id])
    for o in llm.generate([_prompt(7, s) for s in range(3)], sp):
        assert o.outputs[0].finish_reason == "stop", o.outputs[0].text
        assert check(o.outputs[0].text), o.outputs[0].text
        m = xgr.GrammarMatcher(llm._grammars().compile(so))
        assert all(m.accept_token(t) for t in o.output_token_ids) and m.is_terminated()


def test_json_object_and_refusals():
    llm = _llm()
    so = StructuredOutputsParams(json_object=True)
    o = llm.generate([_prompt()], SamplingParams(max_tokens=100, structured_outputs=so))[0]
    m = xgr.GrammarMatcher(llm._grammars().compile(so))
    assert all(m.accept_token(t) for t in o.output_token_ids)  # a prefix of a JSON object
    assert o.outputs[0].text.startswith("{")
    for bad in (StructuredOutputsParams(), StructuredOutputsParams(regex="a", choice=["b"]),
                StructuredOutputsParams(json="{not json"), StructuredOutputsParams(choice=[])):
        with pytest.raises(ValueError):
            llm.generate([_prompt()], SamplingParams(max_tokens=4, structured_outputs=bad))
    no_tok = LLM(TINY, max_num_seqs=2, max_model_len=64, dtype=torch.float32, enforce_eager=True)
    with pytest.raises(ValueError, match="tokenizer"):
        no_tok.generate([_prompt()], SamplingParams(max_tokens=4, structured_outputs=so))


def test_online_mode_guided_requests():
    """Continuous batching (requests arrive through a feed, prefill chunks
    interleave with decode): a grammar request gives the offline tokens; an
    invalid grammar fails that request alone."""
    llm = _llm()
    so = StructuredOutputsParams(choice=["alpha", "beta", "gamma"])
    sp = SamplingParams(max_tokens=20, structured_outputs=so)
    p = _prompt()
    offline = llm.generate([p], sp)[0].output_token_ids
    items = [[(0, p, sp), (1, _prompt(70, 2), SamplingParams(max_tokens=6, ignore_eos=True)),
              (2, p, SamplingParams(max_tokens=4, structured_outputs=StructuredOutputsParams(
                  json="{bad")))]]
    done = {}

    def feed(block):
        return items.pop(0) if items else None

    llm.generate([], feed=feed, on_finish=lambda o: done.__setitem__(o.request_id, o))
    assert done[0].output_token_ids == offline and done[0].error is None
    assert len(done[1].output_token_ids) == 6
    assert done[2].error and "structured_outputs" in done[2].error


def test_server_response_format_and_forced_tool_choice(monkeypatch):
    """Through the OpenAI chat endpoint: ``response_format`` json_schema
    replies parse against the schema; a named ``tool_choice`` returns that
    function's call with schema-valid arguments; "required" returns a
    non-empty list of calls of offered functions."""
    from fastapi.testclient import TestClient

    from vllm_sm70_b200.entrypoints.openai_server import build_app

    # compact JSON: a random-weight model would otherwise emit whitespace forever
    monkeypatch.setenv("VLLM_B200_STRUCTURED_ANY_WHITESPACE", "0")
    tok = _tokenizer()
    tok.chat_template = "{% for m in messages %}{{ m['content'] }}{% endfor %}"
    llm = LLM(TINY, max_num_seqs=4, max_model_len=200, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=64)
    schema = {"type": "object", "properties": {"city": {"type": "string", "enum": ["Paris", "Rome"]},
                                               "days": {"type": "integer", "minimum": 1,
                                                        "maximum": 7}},
              "required": ["city", "days"], "additionalProperties": False}
    tools = [{"type": "function", "function": {"name": "forecast", "parameters": schema}},
             {"type": "function", "function": {"name": "ping", "parameters": {
                 "type": "object", "properties": {}, "additionalProperties": False}}}]
    body = {"messages": [{"role": "user", "content": "weather?"}], "max_tokens": 80,
            "temperature": 0.0}
    with TestClient(build_app(llm, tok, "tiny")) as c:
        r = c.post("/v1/chat/completions", json={**body, "response_format": {
            "type": "json_schema", "json_schema": {"name": "w", "schema": schema}}}).json()
        obj = json.loads(r["choices"][0]["message"]["content"])
        assert obj["city"] in ("Paris", "Rome") and 1 <= obj["days"] <= 7
        r = c.post("/v1/chat/completions", json={**body, "tools": tools, "tool_choice": {
            "type": "function", "function": {"name": "forecast"}}}).json()["choices"][0]
        call = r["message"]["tool_calls"][0]["function"]
        assert r["message"]["content"] is None and call["name"] == "forecast"
        assert json.loads(call["arguments"])["city"] in ("Paris", "Rome")
        r = c.post("/v1/chat/completions", json={**body, "max_tokens": 150, "tools": tools,
                                                 "tool_choice": "required"}).json()["choices"][0]
        calls = r["message"]["tool_calls"]
        assert calls and all(x["function"]["name"] in ("forecast", "ping") for x in calls)
        bad = c.post("/v1/chat/completions", json={**body, "tools": tools, "tool_choice": {
            "type": "function", "function": {"name": "nope"}}})
        assert bad.status_code == 400


def test_llm_chat_template_options():
    """LLM.chat takes vLLM's chat_template, add_generation_prompt and
    continue_final_message (the reply extends the last assistant message)."""
    llm = _llm()
    tpl = ("{% for m in messages %}<{{ m['role'] }}>{{ m['content'] }}{% endfor %}"
           "{% if add_generation_prompt %}<assistant>{% endif %}")
    sp = SamplingParams(max_tokens=2, ignore_eos=True)
    msgs = [{"role": "user", "content": "hi"}]
    enc = lambda t: TOK.encode(t, add_special_tokens=False)  # noqa: E731
    o = llm.chat(msgs, sp, chat_template=tpl)[0]
    assert o.prompt_token_ids == enc("<user>hi<assistant>")
    o = llm.chat(msgs, sp, chat_template=tpl, add_generation_prompt=False)[0]
    assert o.prompt_token_ids == enc("<user>hi")
    cont = msgs + [{"role": "assistant", "content": "Sure"}]
    o = llm.chat(cont, sp, chat_template=tpl, add_generation_prompt=False,
                 continue_final_message=True)[0]
    assert o.prompt_token_ids == enc("<user>hi<assistant>Sure")
    with pytest.raises(ValueError):
        llm.chat(cont, sp, chat_template=tpl, continue_final_message=True)
