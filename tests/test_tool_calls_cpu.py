"""Tool-call extraction (JSON and GLM-4.x block bodies, unterminated and
malformed blocks) and its use by the chat endpoint when tools are offered."""
import json

import torch

from vllm_sm70_b200.integration.tool_calls import parse_tool_calls


def test_json_and_glm_blocks():
    text = ('Let me check.<tool_call>{"name": "get_weather", "arguments": {"city": "Paris"}}'
            '</tool_call>\n<tool_call>search\n<arg_key>query</arg_key>\n<arg_value>b200 '
            'specs</arg_value>\n<arg_key>top_k</arg_key>\n<arg_value>3</arg_value>\n</tool_call>')
    content, calls = parse_tool_calls(text)
    assert content == "Let me check."
    assert [c["function"]["name"] for c in calls] == ["get_weather", "search"]
    assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Paris"}
    assert json.loads(calls[1]["function"]["arguments"]) == {"query": "b200 specs", "top_k": 3}
    assert all(c["type"] == "function" and c["id"].startswith("call_") for c in calls)


def test_unterminated_and_malformed():
    content, calls = parse_tool_calls('<tool_call>{"name": "f", "arguments": {}}')
    assert content is None and calls[0]["function"]["name"] == "f"
    bad = "text <tool_call>{not json</tool_call> tail"
    content, calls = parse_tool_calls(bad)
    assert calls == [] and content == bad
    assert parse_tool_calls("no calls here") == ("no calls here", [])


def test_chat_endpoint_returns_tool_calls():
    from fastapi.testclient import TestClient

    from vllm_sm70_b200.engine import LLM
    from vllm_sm70_b200.entrypoints.openai_server import build_app

    from .test_openai_server_cpu import TINY, Tok

    reply = '<tool_call>{"name": "lookup", "arguments": {"id": 7}}</tool_call>'
    seen = {}

    class ToolTok(Tok):
        chat_template = "{% if add_generation_prompt %}<|assistant|>{% endif %}"

        def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=True, **kw):
            seen.update(kw)
            return super().apply_chat_template(messages, add_generation_prompt, tokenize)

        def decode(self, ids, skip_special_tokens=True):
            return reply  # what the model "said"

    llm = LLM(TINY, max_num_seqs=2, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=64)
    tools = [{"type": "function", "function": {"name": "lookup", "parameters": {}}}]
    with TestClient(build_app(llm, ToolTok(), "tiny")) as c:
        body = {"messages": [{"role": "user", "content": "x"}], "max_tokens": 2,
                "temperature": 0.0, "ignore_eos": True}
        r = c.post("/v1/chat/completions", json={**body, "tools": tools}).json()["choices"][0]
        assert seen.get("tools") == tools
        assert r["finish_reason"] == "tool_calls" and r["message"]["content"] is None
        fn = r["message"]["tool_calls"][0]["function"]
        assert fn["name"] == "lookup" and json.loads(fn["arguments"]) == {"id": 7}
        plain = c.post("/v1/chat/completions", json=body).json()["choices"][0]
        assert "tool_calls" not in plain["message"] and plain["message"]["content"] == reply
