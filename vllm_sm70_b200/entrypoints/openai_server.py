"""OpenAI-compatible HTTP server over the engine (``LLM``).

    python -m vllm_sm70_b200.entrypoints.openai_server --model /path/to/hf-checkpoint \\
        --port 8000 [--max-num-seqs 256] [--max-model-len 4096]
    (TP: one process per GPU under torchrun; rank 0 serves HTTP, every rank runs the engine)

Endpoints: ``GET /health``, ``GET /v1/models``, ``POST /v1/completions``,
``POST /v1/chat/completions``, ``POST /tokenize``, ``POST /detokenize`` and
``GET /metrics`` (Prometheus, vLLM's metric names: ``entrypoints/metrics.py``).
Requests are continuously batched: one engine thread runs a long-lived
``LLM.generate`` that admits each request as it arrives, next to the running
ones, after the current decode burst; each handler awaits its own result. With a tokenizer, text prompts and chat
messages (through the checkpoint's chat template) are accepted and the
``<think>`` / ``<tool_call>`` reasoning split is applied to chat replies
(``--reasoning-parser glm47_b200``); when a chat request offers ``tools``,
they reach the chat template and ``<tool_call>`` blocks in the reply become
OpenAI ``tool_calls`` (``integration/tool_calls.py``). Token-id prompts work
without a tokenizer.

Streaming (``"stream": true``): server-sent events, one chunk per decode
burst of at most ``STREAM_INTERVAL`` steps (text deltas from the cumulative
decode, so multi-token characters are not split), then ``data: [DONE]``.

Log-probabilities: completions ``logprobs`` (top-N, up to 20) and ``echo``
(prompt log-probs too, also with ``max_tokens: 0`` for scoring); chat
``logprobs`` / ``top_logprobs``. They are the model's raw distribution, from
a teacher-forced pass when the request finishes, and are not streamed.

Scope: ``n`` samples per prompt (up to 16; one when streaming); sampling is greedy, temperature (Gumbel-max, seeded) or temperature with
top-k / top-p (over the top-64 candidates of each vocab shard).

Reference parity: the reference is served through ``vllm serve`` with its
plugin; this is the same OpenAI surface for the standalone runtime.
"""
from __future__ import annotations

import argparse
import asyncio
import concurrent.futures
import json
import queue
import threading
import time
import uuid

from ..engine.llm import chat_token_ids
from ..engine.sampling_params import SamplingParams

STREAM_INTERVAL = 8  # decode steps per streamed chunk
HEARTBEAT_S = 1.0    # longest idle wait of rank 0 while other ranks wait on it


class Batcher:
    """Continuous batching: one engine thread runs a single long-lived
    ``LLM.generate`` whose ``feed`` hands it the requests queued since its
    last scheduler iteration, so a request that arrives while others decode
    joins them after the current burst (at most ``STREAM_INTERVAL`` steps)
    instead of waiting for them to finish. Under TP, rank 0's feed broadcasts
    each iteration's new requests over the CPU group and the other ranks'
    ``follower_loop`` feeds the same ones to their engines."""

    def __init__(self, llm, max_batch: int = 256, group=None, metrics=None):
        self.llm = llm
        self.max_batch = max_batch
        self.group = group
        self.metrics = metrics
        self.q: queue.Queue = queue.Queue()
        self.aborts: queue.Queue = queue.Queue()
        self.calls: queue.Queue = queue.Queue()
        self._stop = False
        self._dead: BaseException | None = None
        self._lock = threading.Lock()
        self._next = 0
        self.inflight: dict[int, dict] = {}
        self.batches = 0  # scheduler iterations that admitted new requests
        self.aborted = 0  # requests that ended by abort
        if metrics is not None:
            llm.spec_hook = metrics.spec_step
        self.thread = threading.Thread(target=self._run, name="b200-engine", daemon=True)
        self.thread.start()

    def submit(self, prompt_ids: list[int], params: SamplingParams,
               stream=None) -> concurrent.futures.Future:
        """Queue one request. ``stream(new_ids, finished)`` (optional) is called
        from the engine thread as tokens are produced; ``new_ids`` is None if
        the request failed."""
        fut: concurrent.futures.Future = concurrent.futures.Future()
        if self._dead is not None:
            fut.set_exception(RuntimeError(f"engine stopped: {self._dead}"))
            return fut
        with self._lock:
            rid = self._next
            self._next += 1
        fut.rid = rid
        self.q.put((rid, list(prompt_ids), params, fut, stream))
        return fut

    def call(self, fn) -> concurrent.futures.Future:
        """Run ``fn()`` on the engine thread when the loop is idle -- no request
        queued, prefilling or decoding, so every batch slot is free (engine
        calls such as embeddings use slot 0); single-rank deployments only."""
        fut: concurrent.futures.Future = concurrent.futures.Future()
        if self.group is not None:
            fut.set_exception(RuntimeError("engine calls are served on one rank only"))
            return fut
        self.calls.put((fn, fut))
        return fut

    def _run_calls(self) -> None:
        while True:
            try:
                fn, fut = self.calls.get_nowait()
            except queue.Empty:
                return
            try:
                fut.set_result(fn())
            except Exception as e:  # noqa: BLE001 - reported to the caller
                fut.set_exception(e)

    def abort(self, rid: int) -> None:
        """Cancel a request (e.g. its client went away): it leaves the batch at
        the next scheduler iteration; its future fails with "aborted"."""
        self.aborts.put(rid)

    def _take_aborts(self) -> list:
        out = []
        while True:
            try:
                out.append(("abort", self.aborts.get_nowait()))
            except queue.Empty:
                return out

    # -- engine-thread callbacks ---------------------------------------------
    def _bcast(self, obj):
        if self.group is not None:
            import torch.distributed as dist

            dist.broadcast_object_list([obj], src=0, group=self.group)
        return obj

    def _feed(self, block: bool):
        items = []
        try:
            if block:
                # idle (every batch slot free): engine calls run now; then wait for a
                # request, at most HEARTBEAT_S when other ranks wait on this one in a
                # collective (they must not reach the group's timeout)
                self._run_calls()
                until = time.perf_counter() + (HEARTBEAT_S if self.group is not None else 1e9)
                while not self._stop and not items and time.perf_counter() < until:
                    try:
                        items.append(self.q.get(timeout=0.05))
                    except queue.Empty:
                        self._run_calls()
            while len(items) < self.max_batch:
                items.append(self.q.get_nowait())
        except queue.Empty:
            pass
        if self._stop and not items:
            return self._bcast(None)
        now = time.perf_counter()
        for rid, ids, sp, fut, cb in items:
            self.inflight[rid] = {"fut": fut, "stream": cb, "sp": sp, "n_prompt": len(ids),
                                  "t0": now, "t_first": None, "t_last": None}
        if items:
            self.batches += 1
        if self.metrics is not None:
            self.metrics.gauges(len(self.inflight), self.q.qsize())
        return self._bcast([(rid, ids, sp) for rid, ids, sp, _, _ in items]
                           + self._take_aborts())

    def _on_tokens(self, rid, ids, fin):
        e = self.inflight.get(rid)
        if e is None:
            return
        if ids:
            t = time.perf_counter()
            e["t_first"] = e["t_first"] or t
            e["t_last"] = t
        if e["stream"] is not None:
            try:
                e["stream"](ids, fin)
            except Exception:  # noqa: BLE001 - the consumer is gone: drop only this request
                e["stream"] = None
                self.abort(rid)

    def _on_finish(self, out):
        e = self.inflight.pop(out.request_id, None)
        if e is None:
            return
        if out.error is not None:
            self.aborted += out.error == "aborted"
            if e["stream"] is not None:
                try:
                    e["stream"](None, True)
                except Exception:  # noqa: BLE001 - the consumer is gone
                    pass
            e["fut"].set_exception(ValueError(out.error))
            return
        if self.metrics is not None:
            n = len(out.output_token_ids)
            ttft = e["t_first"] - e["t0"] if e["t_first"] else None
            tpot = ((e["t_last"] - e["t_first"]) / (n - 1)
                    if e["t_first"] and e["t_last"] and n > 1 else None)
            self.metrics.request_finished(self.llm, e["n_prompt"], out, e["sp"], ttft, tpot)
            self.metrics.gauges(len(self.inflight), self.q.qsize())
        e["fut"].set_result(out)

    def _run(self) -> None:
        try:
            self.llm.generate([], feed=self._feed, on_tokens=self._on_tokens,
                              on_finish=self._on_finish, stream_interval=STREAM_INTERVAL)
        except BaseException as exc:  # noqa: BLE001 - reported to every waiting request
            self._dead = exc
            pending = list(self.inflight.values())
            self.inflight.clear()
            while True:
                try:
                    _, _, _, fut, cb = self.q.get_nowait()
                except queue.Empty:
                    break
                pending.append({"fut": fut, "stream": cb})
            for e in pending:
                if e["stream"] is not None:
                    try:
                        e["stream"](None, True)
                    except Exception:  # noqa: BLE001 - the consumer is gone
                        pass
                if not e["fut"].done():
                    e["fut"].set_exception(exc)

    def close(self) -> None:
        """Finish the running requests, then end the engine loop (under TP
        this also releases the followers)."""
        self._stop = True
        self.thread.join(timeout=60.0)


class DPBatcher(Batcher):
    """Data-parallel serving (each rank a whole replica, optionally with
    all-to-all expert parallelism): rank 0 takes the HTTP requests and hands
    each to a rank; every rank runs its own engine loop. Each scheduler
    iteration is a lock-step unit over the CPU group: (1) serve the other
    ranks' expert traffic until every rank is idle (``ep_drain``), (2) gather
    the followers' streamed tokens and finished outputs to rank 0, (3) rank 0
    assigns the new requests (to the least-loaded rank) and broadcasts them.
    The loop is closed only once no rank has work, so all ranks leave it
    together."""

    def __init__(self, llm, max_batch: int = 256, group=None, metrics=None):
        import torch.distributed as dist

        self.world = dist.get_world_size(group)
        self.load = [0] * self.world          # requests in flight per rank
        self.assigned = [0] * self.world      # requests handed to each rank so far
        self.owner: dict[int, int] = {}
        super().__init__(llm, max_batch, group, metrics)

    def _feed(self, block: bool):
        import torch.distributed as dist

        self.llm.model_ep_drain()
        gathered = [None] * self.world
        dist.all_gather_object(gathered, (not block, []), group=self.group)
        any_busy = any(b for b, _ in gathered)
        for r in range(1, self.world):
            for ev in gathered[r][1]:
                self._event(ev)
        items = []
        try:
            if not any_busy and not self.inflight:
                until = time.perf_counter() + HEARTBEAT_S
                while not self._stop and not items and time.perf_counter() < until:
                    try:
                        items.append(self.q.get(timeout=0.05))
                    except queue.Empty:
                        pass
            while len(items) < self.max_batch:
                items.append(self.q.get_nowait())
        except queue.Empty:
            pass
        if self._stop and not items and not any_busy and not self.inflight:
            dist.broadcast_object_list([None], src=0, group=self.group)
            return None
        now = time.perf_counter()
        shares = [[] for _ in range(self.world)]
        for rid, ids, sp, fut, cb in items:
            rank = min(range(self.world), key=lambda r: self.load[r])
            self.load[rank] += 1
            self.assigned[rank] += 1
            self.owner[rid] = rank
            self.inflight[rid] = {"fut": fut, "stream": cb, "sp": sp, "n_prompt": len(ids),
                                  "t0": now, "t_first": None, "t_last": None}
            shares[rank].append((rid, ids, sp))
        for ab in self._take_aborts():
            if ab[1] in self.owner:
                shares[self.owner[ab[1]]].append(ab)
        if items:
            self.batches += 1
        if self.metrics is not None:
            self.metrics.gauges(len(self.inflight), self.q.qsize())
        dist.broadcast_object_list([shares], src=0, group=self.group)
        return shares[0]

    def _event(self, ev) -> None:
        if ev[0] == "tok":
            self._on_tokens(ev[1], ev[2], ev[3])
        else:
            self._on_finish(ev[1])

    def _on_finish(self, out):
        r = self.owner.pop(out.request_id, None)
        if r is not None:
            self.load[r] -= 1
        super()._on_finish(out)


def dp_follower_loop(llm, group) -> None:
    """Ranks > 0 of data-parallel serving: run this rank's engine loop on the
    requests rank 0 assigns to it, in the lock step of :class:`DPBatcher`."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    events: list = []

    def feed(block):
        llm.model_ep_drain()
        dist.all_gather_object([None] * world, (not block, list(events)), group=group)
        events.clear()
        obj = [None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return None if obj[0] is None else obj[0][rank]

    llm.generate([], feed=feed, stream_interval=STREAM_INTERVAL,
                 on_tokens=lambda rid, ids, fin: events.append(("tok", rid, ids, fin)),
                 on_finish=lambda out: events.append(("fin", out)))


def follower_loop(llm, group) -> None:
    """Ranks > 0 under TP: run rank 0's engine loop in lock step -- every
    scheduler iteration takes the requests rank 0 broadcasts -- until rank 0
    closes it."""
    import torch.distributed as dist

    def feed(_block):
        obj = [None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return obj[0]

    llm.generate([], feed=feed, stream_interval=STREAM_INTERVAL)


MAX_LOGPROBS = 20
MAX_N = 16


def _samples(sp: SamplingParams, n: int) -> list[SamplingParams]:
    """The ``n`` requests of one prompt: distinct sampling seeds (the given
    seed + i, or the engine's per-request default)."""
    import dataclasses

    if n == 1:
        return [sp]
    return [dataclasses.replace(sp, seed=None if sp.seed is None else int(sp.seed) + i)
            for i in range(n)]


def _params(body: dict, tokenizer, chat: bool = False) -> SamplingParams:
    """SamplingParams of a request body. Log-probs: completions take
    ``logprobs`` (top-N, OpenAI's legacy form) and ``echo`` (the prompt's
    too); chat takes ``logprobs: true`` with ``top_logprobs``."""
    n = int(body.get("n", 1))
    if not 1 <= n <= MAX_N:
        raise ValueError(f"n must be in [1, {MAX_N}]")
    if n > 1 and body.get("stream") and chat:
        raise ValueError("chat streaming serves n = 1")
    if chat:
        n_lp = int(body.get("top_logprobs") or 0) if body.get("logprobs") else None
        prompt_lp = None
    else:
        n_lp = body.get("logprobs")
        n_lp = None if n_lp is None or n_lp is False else int(n_lp)
        prompt_lp = (n_lp or 0) if body.get("echo") else None
    if n_lp is not None and not 0 <= n_lp <= MAX_LOGPROBS:
        raise ValueError(f"logprobs must be in [0, {MAX_LOGPROBS}]")
    if (n_lp is not None or prompt_lp is not None) and body.get("stream"):
        raise ValueError("log-probabilities are not streamed")
    stop_ids = list(body.get("stop_token_ids") or [])
    ignore_eos = bool(body.get("ignore_eos", False))
    eos = getattr(tokenizer, "eos_token_id", None) if tokenizer is not None else None
    if eos is not None and not ignore_eos:
        stop_ids.append(int(eos))
    top_k = body.get("top_k")
    mt = body.get("max_completion_tokens", body.get("max_tokens"))
    bias = body.get("logit_bias")
    if bias is not None:  # OpenAI: {"token id": bias in [-100, 100]}
        bias = {int(t): min(100.0, max(-100.0, float(v))) for t, v in dict(bias).items()}
    allowed = body.get("allowed_token_ids")  # vLLM's extra field
    guided = _structured(body)
    return SamplingParams(max_tokens=16 if mt is None else int(mt),
                          logprobs=n_lp, prompt_logprobs=prompt_lp,
                          temperature=float(body.get("temperature", 1.0)),
                          top_k=int(top_k) if top_k is not None else -1,
                          top_p=float(body.get("top_p", 1.0)),
                          repetition_penalty=float(body.get("repetition_penalty", 1.0)),
                          min_p=float(body.get("min_p", 0.0)),
                          presence_penalty=float(body.get("presence_penalty", 0.0)),
                          frequency_penalty=float(body.get("frequency_penalty", 0.0)),
                          seed=body.get("seed"), ignore_eos=ignore_eos, stop_token_ids=stop_ids,
                          min_tokens=int(body.get("min_tokens", 0)), logit_bias=bias or None,
                          allowed_token_ids=None if allowed is None else [int(t) for t in allowed],
                          structured_outputs=guided,
                          bad_words=list(body["bad_words"]) if body.get("bad_words") else None,
                          truncate_prompt_tokens=body.get("truncate_prompt_tokens"),
                          skip_special_tokens=bool(body.get("skip_special_tokens", True)),
                          priority=int(body.get("priority", 0)))


def _forced_tool_schema(body: dict):
    """(kind, JSON schema) of the reply a forced ``tool_choice`` demands, as
    vLLM builds it: a named function -> its ``parameters`` object; "required"
    -> a non-empty array of {"name", "parameters"} over the offered tools;
    None for "auto" / "none" / no tools."""
    choice = body.get("tool_choice")
    tools = [t.get("function", t) for t in body.get("tools") or []]
    if not tools or choice in (None, "auto", "none"):
        return None
    params = lambda f: f.get("parameters") or {"type": "object"}  # noqa: E731
    if choice == "required":
        return "required", {"type": "array", "minItems": 1, "items": {"anyOf": [
            {"type": "object", "properties": {"name": {"type": "string", "enum": [f["name"]]},
                                              "parameters": params(f)},
             "required": ["name", "parameters"]} for f in tools]}}
    if isinstance(choice, dict):
        name = (choice.get("function") or {}).get("name")
        for f in tools:
            if f.get("name") == name:
                return ("named", name), params(f)
        raise ValueError(f"tool_choice names an unknown function: {name}")
    raise ValueError(f"tool_choice {choice!r} is not supported")


def _structured(body: dict):
    """Structured-output request of a body: OpenAI ``response_format``
    (``json_object``, or ``json_schema`` with its ``schema``), vLLM's
    ``structured_outputs`` object (json / regex / choice / grammar /
    json_object) and its older ``guided_json`` / ``guided_regex`` /
    ``guided_choice`` / ``guided_grammar`` fields; None when there is none."""
    from ..engine.structured import StructuredOutputsParams

    so = body.get("structured_outputs")
    if so:
        keys = ("json", "regex", "choice", "grammar", "json_object", "disable_any_whitespace")
        return StructuredOutputsParams(**{k: so[k] for k in keys if k in so})
    for field, kw in (("guided_json", "json"), ("guided_regex", "regex"),
                      ("guided_choice", "choice"), ("guided_grammar", "grammar")):
        if body.get(field) is not None:
            return StructuredOutputsParams(**{kw: body[field]})
    rf = body.get("response_format") or {}
    if rf.get("type") == "json_object":
        return StructuredOutputsParams(json_object=True)
    if rf.get("type") == "json_schema":
        js = rf.get("json_schema") or {}
        schema = js.get("schema", js.get("json_schema"))
        if schema is None:
            raise ValueError("response_format json_schema needs a schema")
        return StructuredOutputsParams(json=schema)
    return None


def _apply_stop_strings(text: str, stop) -> tuple[str, bool]:
    if not stop:
        return text, False
    stops = [stop] if isinstance(stop, str) else list(stop)
    cut = min((text.find(s) for s in stops if s and text.find(s) >= 0), default=-1)
    return (text[:cut], True) if cut >= 0 else (text, False)


class _TextStream:
    """Token ids -> text deltas by decoding the cumulative ids (a trailing
    incomplete character is held back until the next piece completes it)."""

    def __init__(self, decode):
        self.decode = decode
        self.ids: list[int] = []
        self.sent = ""

    def push(self, ids: list[int], final: bool) -> str:
        self.ids += ids
        full = self.decode(self.ids)
        if (not final and full.endswith("\ufffd")) or not full.startswith(self.sent):
            return ""
        delta, self.sent = full[len(self.sent):], full
        return delta


def _sse(obj) -> str:
    return f"data: {json.dumps(obj)}\n\n"


def build_app(llm, tokenizer=None, model_name: str = "model", reasoning_parser: str | None = None,
              max_batch: int = 256, group=None):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import StreamingResponse

    from ..integration import reasoning as rp

    import contextlib

    from .metrics import ServerMetrics

    metrics = ServerMetrics(model_name)
    if tokenizer is not None and hasattr(llm, "set_tokenizer") and llm.tokenizer is None:
        llm.set_tokenizer(tokenizer)  # structured-output grammars need it too
    ps = getattr(llm, "ps", None)
    dp = ps is not None and ps.world_size > 1 and ps.tp_size == 1
    batcher = (DPBatcher(llm, max_batch, ps.cpu_group, metrics) if dp
               else Batcher(llm, max_batch, group, metrics))

    @contextlib.asynccontextmanager
    async def lifespan(_app):
        yield
        batcher.close()

    app = FastAPI(title="vllm-b200", lifespan=lifespan)
    app.state.batcher = batcher
    created = int(time.time())

    def encode(prompt):
        if isinstance(prompt, list) and all(isinstance(t, int) for t in prompt):
            return list(prompt)
        if isinstance(prompt, str):
            if tokenizer is None:
                raise HTTPException(400, "text prompts need a tokenizer; send token ids")
            return list(tokenizer.encode(prompt))
        raise HTTPException(400, "prompt must be a string or a list of token ids")

    def decode(ids):
        return tokenizer.decode(ids, skip_special_tokens=True) if tokenizer is not None else None

    def tok_str(i: int) -> str:
        return (tokenizer.decode([i], skip_special_tokens=False) if tokenizer is not None
                else f"token_id:{i}")

    def completion_logprobs(ids, entries, offset0: int) -> dict:
        """OpenAI's legacy completions ``logprobs`` object for token ``ids``
        with engine entries ``{id: log-prob}`` (None for a first prompt token)."""
        toks, lps, tops, offs = [], [], [], []
        off = offset0
        for i, d in zip(ids, entries):
            s_ = tok_str(i)
            toks.append(s_)
            offs.append(off)
            off += len(s_)
            lps.append(None if d is None else d[i])
            tops.append(None if d is None else {tok_str(k): v for k, v in d.items()})
        return {"tokens": toks, "token_logprobs": lps, "top_logprobs": tops, "text_offset": offs}

    async def run(prompt_ids, sp):
        fut = batcher.submit(prompt_ids, sp)
        return await asyncio.wrap_future(fut)

    def start_stream(prompt_ids, sp, q=None, tag=None) -> asyncio.Queue:
        """Submit a streamed request; its (new ids, finished) pieces arrive on
        the returned queue -- ``q`` if given, as (tag, new ids, finished) when
        a ``tag`` is given (several samples on one queue)."""
        loop = asyncio.get_running_loop()
        q = asyncio.Queue() if q is None else q
        item = (lambda ids, fin: (ids, fin)) if tag is None else (lambda ids, fin: (tag, ids, fin))
        fut = batcher.submit(prompt_ids, sp, lambda ids, fin: loop.call_soon_threadsafe(
            q.put_nowait, item(ids, fin)))
        q.rid = getattr(fut, "rid", None)
        q.rids = getattr(q, "rids", []) + [q.rid]
        return q

    async def guarded(gen, q):
        """Pass the stream through; if the client goes away before it ends,
        abort the request so it stops holding a batch slot."""
        done = False
        try:
            async for item in gen:
                yield item
            done = True
        finally:
            for rid in (getattr(q, "rids", None) or [q.rid]) if not done else []:
                if rid is not None:
                    batcher.abort(rid)

    def stream_completion(prompt_ids, sp, stop, usage=False, n=1):
        """Server-sent events of one prompt's ``n`` samples; each chunk is
        one sample's new tokens, tagged with the sample's choice index."""
        q: asyncio.Queue = asyncio.Queue()
        for k, spk in enumerate(_samples(sp, n)):
            start_stream(prompt_ids, spk, q, k)
        rid, made = f"cmpl-{uuid.uuid4().hex}", int(time.time())

        async def events():
            ts = [_TextStream(decode) if tokenizer is not None else None for _ in range(n)]
            hit, stopped = [False] * n, [False] * n
            n_gen, open_ = 0, n
            while open_:
                k, ids, fin = await q.get()
                if ids is None:
                    yield _sse({"error": {"message": "generation failed"}})
                    break
                if ids and ids[-1] in sp.stop_token_ids:
                    stopped[k] = True
                text = None
                if ts[k] is not None:
                    text = "" if hit[k] else ts[k].push(ids, fin)
                    if not hit[k] and stop:
                        cut, hit[k] = _apply_stop_strings(ts[k].sent, stop)
                        if hit[k]:  # drop what follows the stop string
                            text = text[: max(0, len(text) - (len(ts[k].sent) - len(cut)))]
                choice = {"index": k, "text": text, "token_ids": ids,
                          "finish_reason": ("stop" if (stopped[k] or hit[k]) else "length")
                          if fin else None}
                yield _sse({"id": rid, "object": "text_completion", "created": made,
                            "model": model_name, "choices": [choice]})
                n_gen += len(ids)
                open_ -= bool(fin)
            if usage:
                yield _sse({"id": rid, "object": "text_completion", "created": made,
                            "model": model_name, "choices": [],
                            "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": n_gen,
                                      "total_tokens": len(prompt_ids) + n_gen}})
            yield "data: [DONE]\n\n"

        return StreamingResponse(guarded(events(), q), media_type="text/event-stream")

    @app.get("/health")
    async def health():
        """200 while the engine loop runs; 503 once it has stopped on an error
        (an orchestrator should restart the server)."""
        if batcher._dead is not None or not batcher.thread.is_alive():
            from fastapi.responses import JSONResponse

            return JSONResponse({"status": "engine stopped", "error": str(batcher._dead)},
                                status_code=503)
        return {"status": "ok"}

    @app.get("/metrics")
    async def prometheus():
        from fastapi.responses import Response
        from prometheus_client import CONTENT_TYPE_LATEST

        return Response(metrics.exposition(), media_type=CONTENT_TYPE_LATEST)

    @app.post("/v1/embeddings")
    async def embeddings(body: dict):
        """Last-token embeddings of the inputs (run on the engine thread between
        its scheduler iterations)."""
        inp = body.get("input")
        batch = inp if isinstance(inp, list) and inp and not isinstance(inp[0], int) else [inp]
        ids = [encode(x) for x in batch]
        fut = batcher.call(lambda: llm.embed(ids))
        vecs = await asyncio.wrap_future(fut)
        return {"object": "list", "model": model_name,
                "data": [{"object": "embedding", "index": i, "embedding": v.tolist()}
                         for i, v in enumerate(vecs)],
                "usage": {"prompt_tokens": sum(len(x) for x in ids),
                          "total_tokens": sum(len(x) for x in ids)}}

    @app.post("/tokenize")
    async def tokenize(body: dict):
        if "messages" in body:
            if tokenizer is None or not hasattr(tokenizer, "apply_chat_template"):
                raise HTTPException(400, "chat needs a tokenizer with a chat template")
            ids = chat_token_ids(
                tokenizer, body["messages"],
                add_generation_prompt=bool(body.get("add_generation_prompt", True)),
                **(body.get("chat_template_kwargs") or {}))
        else:
            ids = encode(body.get("prompt"))
        return {"tokens": ids, "count": len(ids), "max_model_len": llm.runner.max_model_len}

    @app.post("/detokenize")
    async def detokenize(body: dict):
        if tokenizer is None:
            raise HTTPException(400, "detokenize needs a tokenizer")
        return {"prompt": decode(list(body.get("tokens") or []))}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model",
                                            "created": created, "owned_by": "vllm-b200",
                                            "max_model_len": llm.runner.max_model_len}]}

    @app.post("/v1/completions")
    async def completions(body: dict):
        try:
            sp = _params(body, tokenizer)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        prompts = body.get("prompt")
        batch = (prompts if isinstance(prompts, list) and prompts
                 and not all(isinstance(t, int) for t in prompts) else [prompts])
        ids = [encode(p) for p in batch]
        if body.get("stream"):
            if len(ids) != 1:
                raise HTTPException(400, "streaming serves one prompt per request")
            return stream_completion(ids[0], sp, body.get("stop"),
                                     bool((body.get("stream_options") or {}).get("include_usage")),
                                     int(body.get("n", 1)))
        n = int(body.get("n", 1))
        jobs = [(pi, spj) for pi in range(len(ids)) for spj in _samples(sp, n)]
        try:
            outs = await asyncio.gather(*[run(ids[pi], spj) for pi, spj in jobs])
        except ValueError as e:  # a request the engine could not serve
            raise HTTPException(400, str(e)) from e
        echo = bool(body.get("echo"))
        choices, n_out = [], 0
        for k, ((i, _), o) in enumerate(zip(jobs, outs)):
            text = decode(o.output_token_ids)
            last = o.output_token_ids[-1] if o.output_token_ids else None
            stopped = last is not None and last in sp.stop_token_ids
            if text is not None:
                text, hit = _apply_stop_strings(text, body.get("stop"))
                stopped = stopped or hit
            n_out += len(o.output_token_ids)
            ch = {"index": k, "text": text, "token_ids": o.output_token_ids,
                  "finish_reason": "stop" if stopped else "length", "logprobs": None}
            if echo:
                ptext = decode(ids[i])
                ch["text"] = (ptext or "") + (text or "") if tokenizer is not None else None
                ch["prompt_token_ids"] = ids[i]
            if sp.logprobs is not None or echo and sp.prompt_logprobs is not None:
                lp_ids, lp_entries = [], []
                if echo:
                    lp_ids += ids[i]
                    lp_entries += o.prompt_logprobs or [None] * len(ids[i])
                if sp.logprobs is not None:
                    lp_ids += o.output_token_ids
                    lp_entries += o.logprobs or []
                ch["logprobs"] = completion_logprobs(lp_ids, lp_entries, 0)
            choices.append(ch)
        return {"id": f"cmpl-{uuid.uuid4().hex}", "object": "text_completion", "created":
                int(time.time()), "model": model_name, "choices": choices,
                "usage": {"prompt_tokens": sum(len(p) for p in ids), "completion_tokens": n_out,
                          "total_tokens": sum(len(p) for p in ids) + n_out}}

    def stream_chat(prompt_ids, sp, kwargs, stop, usage=False):
        q = start_stream(prompt_ids, sp)
        rid, made = f"chatcmpl-{uuid.uuid4().hex}", int(time.time())
        splitter = None
        if reasoning_parser == "glm47_b200":
            enabled, inside = rp.thinking_policy(getattr(tokenizer, "chat_template", None), kwargs)
            splitter = rp.ThinkSplitter(inside) if enabled else None
        stops = set(sp.stop_token_ids)
        # special tokens are kept (the reasoning markers); stop tokens are not text
        ts = _TextStream(lambda ids: tokenizer.decode([t for t in ids if t not in stops],
                                                      skip_special_tokens=False))

        def chunk(delta, finish=None):
            return _sse({"id": rid, "object": "chat.completion.chunk", "created": made,
                         "model": model_name,
                         "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]})

        async def events():
            yield chunk({"role": "assistant"})
            stopped = hit = False
            n_gen = 0
            content_sent = ""
            while True:
                ids, fin = await q.get()
                if ids is None:
                    yield _sse({"error": {"message": "generation failed"}})
                    break
                if ids and ids[-1] in stops:
                    stopped = True
                text = ts.push(ids, fin)
                delta = {}
                if text and not hit:
                    r, c = splitter.feed(text) if splitter is not None else ("", text)
                    if r:
                        delta["reasoning_content"] = r
                    if c and stop:
                        cut, hit = _apply_stop_strings(content_sent + c, stop)
                        c = cut[len(content_sent):] if hit else c
                    if c:
                        delta["content"] = c
                        content_sent += c
                if delta:
                    yield chunk(delta)
                n_gen += len(ids)
                if fin:
                    yield chunk({}, "stop" if (stopped or hit) else "length")
                    break
            if usage:
                yield _sse({"id": rid, "object": "chat.completion.chunk", "created": made,
                            "model": model_name, "choices": [],
                            "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": n_gen,
                                      "total_tokens": len(prompt_ids) + n_gen}})
            yield "data: [DONE]\n\n"

        return StreamingResponse(guarded(events(), q), media_type="text/event-stream")

    @app.post("/v1/chat/completions")
    async def chat(body: dict):
        if tokenizer is None or not hasattr(tokenizer, "apply_chat_template"):
            raise HTTPException(400, "chat needs a tokenizer with a chat template")
        try:
            sp = _params(body, tokenizer, chat=True)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        try:
            forced = _forced_tool_schema(body)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        if forced is not None:  # the reply is the call's JSON, constrained by its schema
            import dataclasses

            from ..engine.structured import StructuredOutputsParams

            if body.get("stream"):
                raise HTTPException(400, "a forced tool_choice is served without streaming")
            sp = dataclasses.replace(sp, structured_outputs=StructuredOutputsParams(
                json=forced[1]))
        kwargs = body.get("chat_template_kwargs") or {}
        tools = body.get("tools") if body.get("tool_choice", "auto") != "none" else None
        tpl = dict(kwargs, tools=tools) if tools else kwargs
        ids = chat_token_ids(tokenizer, body["messages"], add_generation_prompt=True, **tpl)
        if body.get("stream"):
            return stream_chat(ids, sp, kwargs, body.get("stop"),
                               bool((body.get("stream_options") or {}).get("include_usage")))
        try:
            outs = await asyncio.gather(*[run(ids, spj)
                                          for spj in _samples(sp, int(body.get("n", 1)))])
        except ValueError as e:  # a request the engine could not serve
            raise HTTPException(400, str(e)) from e
        choices = [chat_choice(k, o, sp, kwargs, body.get("stop"), bool(tools), forced)
                   for k, o in enumerate(outs)]
        n_out = sum(len(o.output_token_ids) for o in outs)
        return {"id": f"chatcmpl-{uuid.uuid4().hex}", "object": "chat.completion",
                "created": int(time.time()), "model": model_name, "choices": choices,
                "usage": {"prompt_tokens": len(ids), "completion_tokens": n_out,
                          "total_tokens": len(ids) + n_out}}

    def chat_choice(index, o, sp, kwargs, stop, tools=False, forced=None) -> dict:
        raw = tokenizer.decode(o.output_token_ids, skip_special_tokens=False)
        last = o.output_token_ids[-1] if o.output_token_ids else None
        stopped = last is not None and last in sp.stop_token_ids
        msg = {"role": "assistant"}
        if reasoning_parser == "glm47_b200":
            enabled, inside = rp.thinking_policy(getattr(tokenizer, "chat_template", None), kwargs)
            if enabled:
                r, c = rp.ThinkSplitter(inside).feed(raw)
                msg["reasoning_content"] = r.rstrip() or None
                raw = c
        content = raw
        eos_text = getattr(tokenizer, "eos_token", None)
        if eos_text and content.endswith(eos_text):
            content = content[: -len(eos_text)]
        content, hit = _apply_stop_strings(content, stop)
        msg["content"] = content
        finish = "stop" if (stopped or hit) else "length"
        if forced is not None and not o.error:
            from ..integration.tool_calls import forced_tool_calls

            calls = forced_tool_calls(forced, content)
            if calls:
                msg["content"], msg["tool_calls"] = None, calls
        elif tools:  # the request offered tools: <tool_call> blocks become tool_calls
            from ..integration.tool_calls import parse_tool_calls

            rest, calls = parse_tool_calls(content)
            if calls:
                msg["content"], msg["tool_calls"] = rest, calls
                finish = "tool_calls"
        logprobs = None
        if sp.logprobs is not None:
            def item(tok, lp):
                s_ = tok_str(tok)
                return {"token": s_, "logprob": lp, "bytes": list(s_.encode())}
            logprobs = {"content": [
                dict(item(t, d[t]), top_logprobs=[item(k, v) for k, v in sorted(
                    d.items(), key=lambda kv: -kv[1])[: sp.logprobs]])
                for t, d in zip(o.output_token_ids, o.logprobs or [])]}
        return {"index": index, "message": msg, "logprobs": logprobs, "finish_reason": finish}

    return app


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True, help="HF checkpoint directory or preset name")
    ap.add_argument("--load-format", default="safetensors", choices=["safetensors", "dummy"])
    ap.add_argument("--served-model-name", default=None)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--tensor-parallel-size", type=int, default=1)
    ap.add_argument("--data-parallel-size", type=int, default=1,
                    help="replicas (one per rank under torchrun); rank 0 serves HTTP")
    ap.add_argument("--enable-expert-parallel", action="store_true",
                    help="data-parallel MoE: experts split over the ranks, all-to-all tokens")
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--max-model-len", type=int, default=4096)
    ap.add_argument("--max-num-batched-tokens", type=int, default=16384)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--enable-prefix-caching", action="store_true")
    ap.add_argument("--prefix-cache-dir", default=None,
                    help="persistent KV tier of the prefix cache (implies prefix caching)")
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.90)
    ap.add_argument("--enforce-eager", action="store_true", help="no CUDA-graph decode")
    ap.add_argument("--speculative-k", type=int, default=0,
                    help="draft tokens per step from the model's MTP head (0 = off)")
    ap.add_argument("--seed", type=int, default=0, help="dummy-weight seed")
    ap.add_argument("--gemm-lut", default=None, help="tuned GEMM plan table to import")
    ap.add_argument("--tokenizer", default=None, help="tokenizer directory (default: --model)")
    ap.add_argument("--reasoning-parser", default=None, choices=[None, "glm47_b200"])
    args = ap.parse_args(argv)

    from ..engine import LLM
    from ..parallel import state as pstate

    llm = LLM(args.model, tensor_parallel_size=args.tensor_parallel_size,
              max_num_seqs=args.max_num_seqs, max_model_len=args.max_model_len,
              max_num_batched_tokens=args.max_num_batched_tokens, block_size=args.block_size,
              load_format=args.load_format,
              enable_prefix_caching=args.enable_prefix_caching or bool(args.prefix_cache_dir),
              prefix_cache_dir=args.prefix_cache_dir,
              gpu_memory_utilization=args.gpu_memory_utilization,
              enforce_eager=args.enforce_eager, speculative_k=args.speculative_k,
              seed=args.seed, gemm_lut_path=args.gemm_lut,
              data_parallel_size=args.data_parallel_size,
              enable_expert_parallel=args.enable_expert_parallel)
    tok = None
    if args.load_format == "safetensors" or args.tokenizer:
        try:
            from transformers import AutoTokenizer

            tok = AutoTokenizer.from_pretrained(args.tokenizer or args.model)
        except Exception:  # noqa: BLE001 - token-id prompts still work
            tok = None
    if tok is not None:  # every rank compiles structured-output grammars against it
        llm.set_tokenizer(tok)
    ps = pstate.get()
    group = ps.cpu_group if ps.tp_size > 1 else None
    if ps.tp_size > 1 and ps.tp_rank != 0:
        follower_loop(llm, group)
        return
    if ps.world_size > 1 and ps.tp_size == 1 and ps.rank != 0:  # data-parallel replicas
        dp_follower_loop(llm, ps.cpu_group)
        return
    import uvicorn

    app = build_app(llm, tok, args.served_model_name or args.model,
                    reasoning_parser=args.reasoning_parser, max_batch=args.max_num_seqs,
                    group=group)
    uvicorn.run(app, host=args.host, port=args.port)


if __name__ == "__main__":
    main()
