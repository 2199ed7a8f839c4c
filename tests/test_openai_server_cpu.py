"""OpenAI-compatible server over the engine (CPU engine, tiny model, a fake
tokenizer): completions from token ids and text, batching of concurrent
requests, stop tokens / strings, chat with the reasoning split, streamed
(server-sent events) completions and chat equal to the unstreamed replies,
and the 400s for what is not served."""
import json
import threading

import pytest
import torch

from vllm_sm70_b200.engine import LLM, SamplingParams
from vllm_sm70_b200.entrypoints.openai_server import build_app
from vllm_sm70_b200.models.config import ModelConfig

TINY = ModelConfig(arch="llama", hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                   head_dim=32, intermediate_size=256, vocab_size=512, rope_theta=10000.0,
                   rms_eps=1e-5, max_position=512)


class Tok:
    """Characters <-> ids 1..255; a few special tokens above."""
    eos_token_id = 300
    eos_token = "</s>"
    chat_template = "{% if add_generation_prompt %}<|assistant|><think>{% endif %}"
    special = {301: "<think>", 302: "</think>", 300: "</s>"}

    def encode(self, text):
        return [min(255, max(1, ord(c))) for c in text]

    def decode(self, ids, skip_special_tokens=True):
        out = []
        for i in ids:
            if i in self.special:
                if not skip_special_tokens:
                    out.append(self.special[i])
            elif 0 < i < 256:
                out.append(chr(i))
            else:
                out.append("?")
        return "".join(out)

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=True, **kw):
        text = "".join(f"<{m['role']}>{m['content']}" for m in messages)
        return self.encode(text) + [301]


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient

    llm = LLM(TINY, max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=64)
    app = build_app(llm, Tok(), "tiny", reasoning_parser="glm47_b200", max_batch=4)
    with TestClient(app) as c:
        c.llm = llm
        c.app_ = app
        yield c


def test_models_and_health(client):
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"


def test_completion_token_ids_match_engine(client):
    ids = list(range(10, 30))
    r = client.post("/v1/completions", json={"prompt": ids, "max_tokens": 6,
                                              "temperature": 0.0, "ignore_eos": True}).json()
    want = client.llm.generate([torch.tensor(ids)], SamplingParams(max_tokens=6))[0]
    assert r["choices"][0]["token_ids"] == want.output_token_ids
    assert r["usage"] == {"prompt_tokens": 20, "completion_tokens": 6, "total_tokens": 26}
    assert r["choices"][0]["finish_reason"] == "length"


def test_text_prompt_batch_and_concurrency(client):
    r = client.post("/v1/completions", json={"prompt": ["hello", "world!!"], "max_tokens": 4,
                                              "temperature": 0.0, "ignore_eos": True}).json()
    assert [c["index"] for c in r["choices"]] == [0, 1]
    assert all(len(c["token_ids"]) == 4 and isinstance(c["text"], str) for c in r["choices"])
    # concurrent requests are served (batched by the worker)
    res = []

    def go(i):
        res.append(client.post("/v1/completions", json={
            "prompt": list(range(5 + i, 25 + i)), "max_tokens": 3, "temperature": 0.0,
            "ignore_eos": True}).status_code)

    th = [threading.Thread(target=go, args=(i,)) for i in range(6)]
    [t.start() for t in th]
    [t.join() for t in th]
    assert res == [200] * 6


def test_stop_string_and_unsupported(client):
    r = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 8, "temperature": 0.0,
                                              "ignore_eos": True, "stop": ["\\u0000"]})
    assert r.status_code == 200
    for bad in ({"n": 17}, {"logprobs": 21},
                {"logprobs": 1, "stream": True},
                {"stream": True, "prompt": ["a", "b"]}):
        body = {"prompt": [1, 2, 3], "max_tokens": 2, **bad}
        assert client.post("/v1/completions", json=body).status_code == 400


def test_chat_reasoning_split(client):
    r = client.post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "hi"}], "max_tokens": 5, "temperature": 0.0,
        "ignore_eos": True}).json()
    msg = r["choices"][0]["message"]
    assert msg["role"] == "assistant" and "content" in msg
    # the template opens <think>: everything before </think> is reasoning
    assert "reasoning_content" in msg


def test_stop_token_truncates_engine_output():
    from vllm_sm70_b200.engine.llm import _truncate_at_stop

    sp = SamplingParams(max_tokens=8, stop_token_ids=[7])
    assert _truncate_at_stop([1, 2, 7, 9, 7], sp) == [1, 2, 7]
    assert _truncate_at_stop([1, 2, 3], sp) == [1, 2, 3]
    sp2 = SamplingParams(max_tokens=8, stop_token_ids=[7], ignore_eos=True)
    assert _truncate_at_stop([1, 7, 3], sp2) == [1, 7, 3]


def _events(client, url, body):
    """The JSON payloads of a server-sent event stream (``[DONE]`` last)."""
    out = []
    with client.stream("POST", url, json=body) as r:
        assert r.status_code == 200
        assert r.headers["content-type"].startswith("text/event-stream")
        for line in r.iter_lines():
            if line.startswith("data: "):
                data = line[len("data: "):]
                out.append(data if data == "[DONE]" else json.loads(data))
    assert out and out[-1] == "[DONE]"
    return out[:-1]


def test_stream_completion_equals_unstreamed(client):
    body = {"prompt": "streaming!", "max_tokens": 19, "temperature": 0.0, "ignore_eos": True}
    whole = client.post("/v1/completions", json=body).json()["choices"][0]
    ev = _events(client, "/v1/completions", {**body, "stream": True})
    assert len(ev) >= 3  # several bursts of at most STREAM_INTERVAL tokens
    ids = [t for e in ev for t in e["choices"][0]["token_ids"]]
    text = "".join(e["choices"][0]["text"] for e in ev)
    assert ids == whole["token_ids"] and text == whole["text"]
    assert [e["choices"][0]["finish_reason"] for e in ev][-1] == "length"
    assert all(e["choices"][0]["finish_reason"] is None for e in ev[:-1])


def test_stream_chat_equals_unstreamed(client):
    body = {"messages": [{"role": "user", "content": "hey"}], "max_tokens": 12,
            "temperature": 0.0, "ignore_eos": True}
    whole = client.post("/v1/chat/completions", json=body).json()["choices"][0]["message"]
    ev = _events(client, "/v1/chat/completions", {**body, "stream": True})
    assert ev[0]["choices"][0]["delta"] == {"role": "assistant"}
    deltas = [e["choices"][0]["delta"] for e in ev[1:]]
    reasoning = "".join(d.get("reasoning_content", "") for d in deltas)
    content = "".join(d.get("content", "") for d in deltas)
    assert (reasoning.rstrip() or None) == whole["reasoning_content"]
    assert content == whole["content"]
    assert ev[-1]["choices"][0]["finish_reason"] == "length"


def test_tokenize_detokenize_and_metrics(client):
    t = client.post("/tokenize", json={"prompt": "hey"}).json()
    assert t["tokens"] == [ord("h"), ord("e"), ord("y")] and t["count"] == 3
    c = client.post("/tokenize", json={"messages": [{"role": "user", "content": "x"}]}).json()
    assert c["tokens"][-1] == 301  # the template opens <think>
    assert client.post("/detokenize", json={"tokens": t["tokens"]}).json()["prompt"] == "hey"
    before = client.get("/metrics").text
    client.post("/v1/completions", json={"prompt": list(range(10, 17)), "max_tokens": 4,
                                         "temperature": 0.0, "ignore_eos": True})
    text = client.get("/metrics").text

    def value(body, name):
        for line in body.splitlines():
            if line.startswith(name + "{") or line.startswith(name + " "):
                return float(line.rsplit(" ", 1)[1])
        return 0.0
    assert value(text, "vllm:prompt_tokens_total") - value(before, "vllm:prompt_tokens_total") == 7
    assert (value(text, "vllm:generation_tokens_total")
            - value(before, "vllm:generation_tokens_total")) == 4
    assert "vllm:time_to_first_token_seconds_bucket" in text
    assert 'finished_reason="length"' in text


def test_continuous_batching_late_short_request_overtakes():
    """A short request submitted while a long one is decoding joins the
    running batch and finishes first (it does not wait for the long one);
    both equal their stand-alone results."""
    import threading

    from vllm_sm70_b200.entrypoints.openai_server import Batcher

    llm = LLM(TINY, max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=64)
    long_p, short_p = list(range(10, 30)), list(range(40, 50))
    want_long = llm.generate([torch.tensor(long_p)], SamplingParams(max_tokens=60))[0]
    want_short = llm.generate([torch.tensor(short_p)], SamplingParams(max_tokens=3))[0]
    b = Batcher(llm, max_batch=4)
    order = []
    started = threading.Event()
    f_long = b.submit(long_p, SamplingParams(max_tokens=60),
                      stream=lambda ids, fin: started.set())
    assert started.wait(30)  # the long request is decoding
    f_short = b.submit(short_p, SamplingParams(max_tokens=3))
    f_short.add_done_callback(lambda f: order.append("short"))
    f_long.add_done_callback(lambda f: order.append("long"))
    assert f_short.result(60).output_token_ids == want_short.output_token_ids
    assert f_long.result(60).output_token_ids == want_long.output_token_ids
    assert order == ["short", "long"] and b.batches >= 2
    b.close()
    assert not b.thread.is_alive()


def test_completion_logprobs_and_echo(client):
    """``logprobs`` / ``echo`` follow OpenAI's legacy completions format and
    equal the engine's teacher-forced scores; ``max_tokens: 0`` with ``echo``
    scores the prompt alone (what loglikelihood evaluations send)."""
    ids = list(range(60, 72))
    r = client.post("/v1/completions", json={"prompt": ids, "max_tokens": 4, "temperature": 0.0,
                                             "ignore_eos": True, "logprobs": 2}).json()
    lp = r["choices"][0]["logprobs"]
    out = r["choices"][0]["token_ids"]
    assert len(lp["tokens"]) == 4 and len(lp["token_logprobs"]) == 4
    assert all(len(t) >= 2 for t in lp["top_logprobs"])
    seq = torch.tensor(ids + out)
    ref = client.llm.score([seq])[0]
    assert all(abs(a - float(b)) < 1e-4 for a, b in zip(lp["token_logprobs"], ref[len(ids) - 1:]))
    e = client.post("/v1/completions", json={"prompt": ids, "max_tokens": 0, "echo": True,
                                             "logprobs": 0}).json()["choices"][0]
    assert e["token_ids"] == [] and e["logprobs"]["token_logprobs"][0] is None
    ref_p = client.llm.score([torch.tensor(ids)])[0]
    got = e["logprobs"]["token_logprobs"][1:]
    assert len(got) == len(ids) - 1 and all(abs(a - float(b)) < 1e-4 for a, b in zip(got, ref_p))


def test_chat_logprobs(client):
    r = client.post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "temperature": 0.0,
        "ignore_eos": True, "logprobs": True, "top_logprobs": 2}).json()
    content = r["choices"][0]["logprobs"]["content"]
    assert len(content) == 3
    for c in content:
        assert c["logprob"] <= 0 and 1 <= len(c["top_logprobs"]) <= 2
        assert c["top_logprobs"][0]["logprob"] >= c["logprob"] - 1e-6  # greedy = top-1


def test_n_samples(client):
    """``n`` samples per prompt: greedy ones agree, seeded temperature ones
    differ from one another and repeat with the same seed."""
    body = {"prompt": list(range(20, 30)), "max_tokens": 6, "ignore_eos": True, "n": 3}
    g = client.post("/v1/completions", json={**body, "temperature": 0.0}).json()["choices"]
    assert [c["index"] for c in g] == [0, 1, 2]
    assert g[0]["token_ids"] == g[1]["token_ids"] == g[2]["token_ids"]
    t = {**body, "temperature": 1.5, "seed": 7}
    a = [c["token_ids"] for c in client.post("/v1/completions", json=t).json()["choices"]]
    b = [c["token_ids"] for c in client.post("/v1/completions", json=t).json()["choices"]]
    assert a == b and len({tuple(x) for x in a}) > 1
    c = client.post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "yo"}], "max_tokens": 3, "temperature": 0.0,
        "ignore_eos": True, "n": 2}).json()
    assert [ch["index"] for ch in c["choices"]] == [0, 1]
    assert c["usage"]["completion_tokens"] == 6


def test_cli_builds_engine_and_app(tmp_path, monkeypatch):
    """``python -m vllm_sm70_b200.entrypoints.openai_server`` flags reach the
    engine (here: dummy weights of a checkpoint config, prefix cache with a
    disk tier, eager) and the app is handed to uvicorn."""
    import json as _json

    import uvicorn

    from vllm_sm70_b200.entrypoints import openai_server as srv

    from .test_loader_cpu import _hf_config

    (tmp_path / "config.json").write_text(_json.dumps(_hf_config(TINY)))
    seen = {}
    monkeypatch.setattr(uvicorn, "run", lambda app, host, port: seen.update(app=app, port=port))
    built = {}
    real = srv.build_app

    def spy(llm, *a, **k):
        built["llm"] = llm
        return real(llm, *a, **k)
    monkeypatch.setattr(srv, "build_app", spy)
    srv.main(["--model", str(tmp_path), "--load-format", "dummy", "--port", "8123",
              "--max-num-seqs", "2", "--max-model-len", "64", "--enforce-eager",
              "--prefix-cache-dir", str(tmp_path / "kv"), "--max-num-batched-tokens", "64"])
    llm = built["llm"]
    assert seen["port"] == 8123 and llm.prefix_cache is not None
    assert llm.prefix_cache.disk is not None and not llm.runner.use_graphs
    seen["app"].state.batcher.close()


def test_continuous_batching_with_speculative_decoding():
    """The online engine loop with an MTP draft head (Qwen3-Next, k = 2):
    requests submitted while others run give the plain greedy tokens."""
    import threading

    from vllm_sm70_b200.entrypoints.openai_server import Batcher
    from vllm_sm70_b200.models.config import ModelConfig

    from .test_ep_cpu import NEXT_HF

    cfg = ModelConfig.from_hf({**NEXT_HF, "num_nextn_predict_layers": 1})
    kw = dict(max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=32)
    plain = LLM(cfg, **kw)
    spec = LLM(cfg, speculative_k=2, **kw)
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (9, 30, 5)]
    want = [o.output_token_ids for o in plain.generate(prompts, SamplingParams(max_tokens=7))]
    b = Batcher(spec, max_batch=4)
    first = threading.Event()
    futs = [b.submit(prompts[0], SamplingParams(max_tokens=7), stream=lambda i, f: first.set())]
    assert first.wait(60)
    futs += [b.submit(p, SamplingParams(max_tokens=7)) for p in prompts[1:]]
    assert [f.result(120).output_token_ids for f in futs] == want
    b.close()


def test_abort_running_and_queued_requests():
    """``Batcher.abort``: a decoding request leaves the batch at the next
    iteration with the tokens it has (its future fails with "aborted"), a
    request still queued never runs, and the others are unaffected."""
    import threading

    from vllm_sm70_b200.entrypoints.openai_server import Batcher

    llm = LLM(TINY, max_num_seqs=2, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=64)
    other = list(range(50, 60))
    want = llm.generate([torch.tensor(other)], SamplingParams(max_tokens=5))[0]
    b = Batcher(llm, max_batch=2)
    started = threading.Event()
    f_long = b.submit(list(range(10, 30)), SamplingParams(max_tokens=100),
                      stream=lambda ids, fin: started.set())
    assert started.wait(30)
    b.abort(f_long.rid)
    with pytest.raises(ValueError, match="aborted"):
        f_long.result(30)
    f_ok = b.submit(other, SamplingParams(max_tokens=5))
    assert f_ok.result(30).output_token_ids == want.output_token_ids
    b.close()


def test_stream_client_disconnect_aborts(client, monkeypatch):
    """A streaming client that goes away after the first chunk (an ASGI
    ``http.disconnect``): its request is aborted instead of running to
    max_tokens. Decode bursts are slowed so that the request cannot finish on
    its own in the meantime."""
    import asyncio
    import json as _json
    import time as _t

    b = client.app_.state.batcher
    runner = client.llm.runner
    real = runner.decode
    monkeypatch.setattr(runner, "decode", lambda *a, **k: (_t.sleep(0.2), real(*a, **k))[1])
    before = b.aborted
    body = _json.dumps({"prompt": list(range(5, 15)), "max_tokens": 100, "temperature": 0.0,
                        "ignore_eos": True, "stream": True}).encode()

    async def drive():
        first = asyncio.Event()
        sent_request = False

        async def receive():
            nonlocal sent_request
            if not sent_request:
                sent_request = True
                return {"type": "http.request", "body": body, "more_body": False}
            await first.wait()
            return {"type": "http.disconnect"}

        async def send(m):
            if m["type"] == "http.response.body" and b"data: {" in m.get("body", b""):
                first.set()

        scope = {"type": "http", "asgi": {"version": "3.0"}, "http_version": "1.1",
                 "method": "POST", "scheme": "http", "path": "/v1/completions", "raw_path":
                 b"/v1/completions", "query_string": b"", "root_path": "",
                 "headers": [(b"content-type", b"application/json")],
                 "client": ("test", 1), "server": ("test", 80)}
        await asyncio.wait_for(client.app_(scope, receive, send), 60)

    asyncio.run(drive())
    deadline = _t.time() + 30
    while b.inflight and _t.time() < deadline:
        _t.sleep(0.05)
    assert not b.inflight and b.aborted == before + 1


def test_embeddings(client):
    """``/v1/embeddings`` and ``LLM.embed``: unit vectors of the last token's
    final hidden state; the same input gives the same vector whether sent as
    text or ids, and equals the engine's own call."""
    r = client.post("/v1/embeddings", json={"input": ["hey", "there!"]}).json()
    vs = [torch.tensor(d["embedding"]) for d in r["data"]]
    assert len(vs) == 2 and all(abs(float(v.norm()) - 1) < 1e-5 for v in vs)
    ids = [ord(c) for c in "hey"]
    r2 = client.post("/v1/embeddings", json={"input": ids}).json()
    assert torch.allclose(torch.tensor(r2["data"][0]["embedding"]), vs[0], atol=1e-6)
    direct = client.llm.embed([ids])[0]
    assert torch.allclose(direct, vs[0], atol=1e-6) and r["usage"]["prompt_tokens"] == 9


def test_stream_usage_and_max_completion_tokens(client):
    ev = _events(client, "/v1/completions", {
        "prompt": list(range(7, 17)), "max_tokens": 5, "temperature": 0.0, "ignore_eos": True,
        "stream": True, "stream_options": {"include_usage": True}})
    assert ev[-1]["choices"] == [] and ev[-1]["usage"] == {
        "prompt_tokens": 10, "completion_tokens": 5, "total_tokens": 15}
    ev = _events(client, "/v1/chat/completions", {
        "messages": [{"role": "user", "content": "q"}], "max_completion_tokens": 3,
        "temperature": 0.0, "ignore_eos": True, "stream": True,
        "stream_options": {"include_usage": True}})
    assert ev[-1]["usage"]["completion_tokens"] == 3


def test_health_reports_a_dead_engine():
    """/health turns 503 once the engine loop stopped on an error; pending and
    new requests fail instead of hanging; ``LLM`` is a context manager."""
    from fastapi.testclient import TestClient

    with LLM(TINY, max_num_seqs=2, max_model_len=64, block_size=16, dtype=torch.float32,
             enforce_eager=True, max_num_batched_tokens=32) as llm:
        def boom(*a, **k):
            raise RuntimeError("device lost")
        llm.runner.prefill = boom
        with TestClient(build_app(llm, None, "tiny"), raise_server_exceptions=False) as c:
            assert c.get("/health").status_code == 200
            assert c.get("/v1/models").json()["data"][0]["max_model_len"] == 64
            r = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 2})
            assert r.status_code == 500
            h = c.get("/health")
            assert h.status_code == 503 and "device lost" in h.json()["error"]


def test_logit_bias_request_fields():
    """OpenAI ``logit_bias`` (string token ids, bias clamped to [-100, 100])
    and vLLM's ``allowed_token_ids`` reach the sampling parameters."""
    from vllm_sm70_b200.entrypoints.openai_server import _params

    sp = _params({"logit_bias": {"5": 3.5, "9": -250}, "allowed_token_ids": [5, 9, 11]}, None)
    assert sp.logit_bias == {5: 3.5, 9: -100.0}
    assert sp.allowed_token_ids == [5, 9, 11]
    sp = _params({}, None)
    assert sp.logit_bias is None and sp.allowed_token_ids is None and sp.min_tokens == 0
    assert _params({"min_tokens": 3}, None).min_tokens == 3


def test_structured_output_request_fields():
    """response_format (json_object / json_schema), vLLM's structured_outputs
    object and the guided_* fields become StructuredOutputsParams."""
    from vllm_sm70_b200.entrypoints.openai_server import _params

    schema = {"type": "object", "properties": {"a": {"type": "integer"}}}
    so = _params({"response_format": {"type": "json_schema",
                                      "json_schema": {"name": "x", "schema": schema}}}, None)
    assert so.structured_outputs.json == schema
    assert _params({"response_format": {"type": "json_object"}},
                   None).structured_outputs.json_object is True
    assert _params({"response_format": {"type": "text"}}, None).structured_outputs is None
    assert _params({"structured_outputs": {"choice": ["a", "b"]}},
                   None).structured_outputs.choice == ["a", "b"]
    assert _params({"guided_regex": "[0-9]+"}, None).structured_outputs.regex == "[0-9]+"
    with pytest.raises(ValueError):
        _params({"response_format": {"type": "json_schema", "json_schema": {}}}, None)


def test_stream_completion_n_samples(client):
    """``n`` > 1 streams every sample as chunks tagged with its choice index;
    each sample's tokens equal the unstreamed n-sample reply's."""
    body = {"prompt": "many", "max_tokens": 11, "temperature": 1.0, "seed": 5, "n": 3,
            "ignore_eos": True}
    whole = client.post("/v1/completions", json=body).json()["choices"]
    ev = _events(client, "/v1/completions", {**body, "stream": True})
    got = {}
    for e in ev:
        c = e["choices"][0]
        got.setdefault(c["index"], []).extend(c["token_ids"])
    assert sorted(got) == [0, 1, 2]
    assert [got[k] for k in range(3)] == [c["token_ids"] for c in whole]
    assert sum(e["choices"][0]["finish_reason"] == "length" for e in ev) == 3
