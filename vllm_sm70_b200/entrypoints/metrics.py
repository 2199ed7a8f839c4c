"""Prometheus metrics of the OpenAI server, under vLLM's metric names so
dashboards and scripts written against ``vllm serve``'s ``/metrics`` keep
working: request / token counters, time-to-first-token and
time-per-output-token histograms, running / waiting gauges, prefix-cache
queries and hits, and speculative-decoding acceptance counters.

Each server owns its own ``CollectorRegistry`` (several apps can live in one
process, e.g. in tests). Request times are host clock from submission to the
first / last token of the continuous-batching engine loop.

Reference parity: serving metrics are read from upstream vLLM's Prometheus
``/metrics`` by the reference's checks (``scripts/check6-lmcache-reaper.py``
parses the text exposition; acceptance from ``vllm:spec_decode_*``).
"""
from __future__ import annotations

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest

_TTFT_BUCKETS = (0.001, 0.005, 0.01, 0.02, 0.04, 0.06, 0.08, 0.1, 0.25, 0.5, 0.75, 1.0, 2.5,
                 5.0, 7.5, 10.0, 20.0, 40.0, 80.0)
_TPOT_BUCKETS = (0.001, 0.0025, 0.005, 0.0075, 0.01, 0.015, 0.02, 0.025, 0.03, 0.04, 0.05,
                 0.075, 0.1, 0.15, 0.2, 0.3, 0.4, 0.5, 0.75, 1.0, 2.5)


class ServerMetrics:
    def __init__(self, model_name: str):
        self.registry = CollectorRegistry()
        r, lab = self.registry, {"model_name": model_name}
        names = ["model_name"]

        def counter(name, doc):
            return Counter(name, doc, names, registry=r).labels(**lab)

        def gauge(name, doc):
            return Gauge(name, doc, names, registry=r).labels(**lab)

        self.requests = Counter("vllm:request_success", "Finished requests.",
                                names + ["finished_reason"], registry=r)
        self.model_name = model_name
        self.prompt_tokens = counter("vllm:prompt_tokens", "Prefill tokens processed.")
        self.generation_tokens = counter("vllm:generation_tokens", "Generated tokens.")
        self.running = gauge("vllm:num_requests_running", "Requests in the running batch.")
        self.waiting = gauge("vllm:num_requests_waiting", "Requests queued for a batch.")
        self.ttft = Histogram("vllm:time_to_first_token_seconds", "Time to first token.",
                              names, buckets=_TTFT_BUCKETS, registry=r).labels(**lab)
        self.tpot = Histogram("vllm:time_per_output_token_seconds", "Time per output token.",
                              names, buckets=_TPOT_BUCKETS, registry=r).labels(**lab)
        self.prefix_queries = counter("vllm:gpu_prefix_cache_queries",
                                      "Prompt tokens looked up in the prefix cache.")
        self.prefix_hits = counter("vllm:gpu_prefix_cache_hits",
                                   "Prompt tokens served from the prefix cache.")
        self.spec_drafts = counter("vllm:spec_decode_num_drafts", "Speculative steps x rows.")
        self.spec_accepted = counter("vllm:spec_decode_num_accepted_tokens",
                                     "Draft tokens accepted (emitted minus one per step).")
        self.spec_emitted = counter("vllm:spec_decode_num_emitted_tokens",
                                    "Tokens emitted by speculative steps.")
        self._pc_seen = (0, 0)

    def gauges(self, running: int, waiting: int) -> None:
        self.running.set(running)
        self.waiting.set(waiting)

    def request_finished(self, llm, n_prompt: int, out, sp, ttft_s, tpot_s) -> None:
        """Account one finished request (times: host clock from submission)."""
        toks = out.output_token_ids
        self.prompt_tokens.inc(n_prompt)
        self.generation_tokens.inc(len(toks))
        stopped = bool(toks) and toks[-1] in set(sp.stop_token_ids) and not sp.ignore_eos
        self.requests.labels(model_name=self.model_name,
                             finished_reason="stop" if stopped else "length").inc()
        if ttft_s is not None:
            self.ttft.observe(ttft_s)
        if tpot_s is not None:
            self.tpot.observe(tpot_s)
        pc = getattr(llm, "prefix_cache", None)
        if pc is not None:  # the cache counts blocks; export tokens
            q, h = pc.queries * pc.bs, pc.hits * pc.bs
            q0, h0 = self._pc_seen
            self.prefix_queries.inc(max(0, q - q0))
            self.prefix_hits.inc(max(0, h - h0))
            self._pc_seen = (q, h)

    def spec_step(self, rows: int, emitted: int) -> None:
        """Speculative decoding: ``rows`` rows stepped, ``emitted`` tokens."""
        self.spec_drafts.inc(rows)
        self.spec_emitted.inc(emitted)
        self.spec_accepted.inc(max(0, emitted - rows))

    def exposition(self) -> bytes:
        return generate_latest(self.registry)
