"""Tool-call extraction for chat replies (OpenAI ``tool_calls``).

The reasoning split leaves ``<tool_call>`` blocks in the content (they end
the reasoning); this parser turns each block into one OpenAI tool call. Two
block bodies are understood:

* JSON (Hermes / Qwen style)::

      <tool_call>{"name": "get_weather", "arguments": {"city": "Paris"}}</tool_call>

* GLM-4.x style: the function name on the first line, then key / value
  pairs, each value JSON when it parses as JSON, else a string::

      <tool_call>get_weather
      <arg_key>city</arg_key>
      <arg_value>Paris</arg_value>
      </tool_call>

A block left open at the end of the reply (generation stopped inside it) is
parsed up to the end. Text outside the blocks stays the message content. A
block that does not parse stays in the content, untouched.

Reference parity: the ``<tool_call>`` handling of the reference's GLM-4.7
reasoning parser, which hands tool-call blocks to vLLM's tool parser
(``sm70/vllm_sm70/reasoning.py:28-60``).
"""
from __future__ import annotations

import json
import re
import uuid

OPEN, CLOSE = "<tool_call>", "</tool_call>"
_ARG = re.compile(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", re.S)


def _value(v: str):
    try:
        return json.loads(v)
    except (ValueError, TypeError):
        return v


def _parse_block(body: str) -> dict | None:
    body = body.strip()
    if not body:
        return None
    if body.startswith("{"):
        try:
            d = json.loads(body)
        except ValueError:
            return None
        name = d.get("name") if isinstance(d, dict) else None
        if not isinstance(name, str):
            return None
        args = d.get("arguments", d.get("parameters", {}))
        return {"name": name, "arguments": args if isinstance(args, str) else json.dumps(args)}
    head, _, rest = body.partition("\n")
    name = head.strip()
    if not name or "<" in name or " " in name:
        return None
    args = {k.strip(): _value(v.strip()) for k, v in _ARG.findall(rest)}
    return {"name": name, "arguments": json.dumps(args)}


def parse_tool_calls(text: str) -> tuple[str | None, list[dict]]:
    """(content without the parsed blocks -- None if nothing is left --,
    OpenAI ``tool_calls`` list)."""
    calls, keep, pos = [], [], 0
    while True:
        i = text.find(OPEN, pos)
        if i < 0:
            keep.append(text[pos:])
            break
        j = text.find(CLOSE, i + len(OPEN))
        end = len(text) if j < 0 else j + len(CLOSE)
        body = text[i + len(OPEN): len(text) if j < 0 else j]
        fn = _parse_block(body)
        keep.append(text[pos:i])
        if fn is None:
            keep.append(text[i:end])
        else:
            calls.append({"id": f"call_{uuid.uuid4().hex[:24]}", "type": "function",
                          "function": fn})
        pos = end
        if j < 0:
            break
    content = "".join(keep).strip()
    return (content or None), calls


def forced_tool_calls(forced, text: str) -> list[dict]:
    """OpenAI ``tool_calls`` of a reply generated under a forced
    ``tool_choice`` (the grammar made it the call's JSON): a named function's
    arguments object, or the "required" array of {"name", "parameters"}.
    Empty when the text is not complete JSON (the reply hit ``max_tokens``)."""
    kind, _schema = forced
    try:
        obj = json.loads(text)
    except ValueError:
        return []

    def call(name, args):
        return {"id": f"call_{uuid.uuid4().hex[:24]}", "type": "function",
                "function": {"name": name, "arguments": json.dumps(args)}}

    if kind == "required":
        return [call(c["name"], c.get("parameters", {})) for c in obj]
    return [call(kind[1], obj)]
