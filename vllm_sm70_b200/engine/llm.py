"""``LLM``: the offline-inference entry point of the runtime.

    llm = LLM("llama-3.1-8b", tensor_parallel_size=1, load_format="dummy")
    outs = llm.generate(prompt_token_ids, SamplingParams(max_tokens=256, ignore_eos=True))

Scheduling: requests are admitted while a batch slot and the KV blocks for
``prompt + max_tokens`` are free; admitted prompts are prefilled in chunks
of at most ``max_num_batched_tokens`` tokens (long prompts are split across
chunks, the attention kernel reads the cached prefix), then all running
requests decode together in CUDA-graph steps until the next request
finishes; finished requests release their slot and blocks and waiting ones
are admitted. Under ``torchrun`` every rank constructs the same ``LLM`` and
runs the same schedule (decisions depend only on rank-uniform inputs).

Data parallelism (``data_parallel_size`` replicas of ``tensor_parallel_size``
ranks each, world = dp x tp; contiguous ranks form a replica): the ranks of a
replica hold its TP shards and ``generate`` serves that replica's prompts (the
replica's ranks pass the same prompts). TP > 1 inside a replica is the MoE
TP x EP layout. With ``enable_expert_parallel`` an MoE model splits its experts over
the ranks and exchanges tokens in every MoE block (``parallel/ep.py``); each
forward is then preceded by a vote over the ranks, and a rank that runs out
of work keeps serving idle passes until every rank is done, so all ranks take
the same collective steps. That mode runs eager (the all-to-all split sizes
are host values).

Reference parity: the reference serves through upstream vLLM ``LLM`` /
``vllm serve``; this in-repo runner is the engine the B200
kernels and fused collectives run under (also exposed to vLLM through the
platform plugin, ``vllm_sm70_b200.integration``).
"""
from __future__ import annotations

import math
import time
from collections import deque
from dataclasses import dataclass, field

import torch

from .. import envs
from ..models import build_model
from ..models.config import ModelConfig, resolve
from ..parallel import state as pstate
from ..utils import tracing
from ..utils.watchdog import StreamWatchdog
from .model_runner import ModelRunner
from .prefix_cache import DiskKVTier, HostKVTier, PrefixCache
from .sampling_params import RequestOutput, SamplingParams


@dataclass
class _Req:
    rid: int
    prompt: torch.Tensor           # int64 CPU
    params: SamplingParams
    slot: int = -1
    blocks: torch.Tensor | None = None
    prefilled: int = 0
    generated: int = 0
    done: bool = False
    out: list = field(default_factory=list)
    t_first: float | None = None
    t_last: float | None = None
    streamed: int = 0              # output tokens already handed to the stream callback
    logprobs: list | None = None
    prompt_logprobs: list | None = None
    stream_stopped: bool = False   # a stop token was streamed: nothing more follows
    aborted: bool = False          # cancelled by the caller (online mode)
    scanned: int = 0               # output tokens already searched for a stop token
    guide: object = None           # structured outputs: the grammar state (structured.Guide)
    stop_hit: bool = False         # a stop token was generated: retire at the burst's end


@dataclass
class GenerateStats:
    prefill_ms: float = 0.0
    decode_ms: float = 0.0
    total_ms: float = 0.0
    decode_steps: int = 0
    ttft_ms: list = field(default_factory=list)
    tpot_ms: list = field(default_factory=list)
    spec_tokens: int = 0   # tokens emitted by speculative steps
    spec_slots: int = 0    # (row, step) pairs; spec_tokens / spec_slots = tokens per step


def _penalized(p: SamplingParams, spec: bool = False) -> bool:
    """Whether the request rewrites its logits before sampling. ``min_tokens``
    masks the stop tokens until that many tokens exist (vLLM's rule), except
    under speculative decoding, where stops before ``min_tokens`` are only
    ignored."""
    return (p.repetition_penalty != 1.0 or p.presence_penalty != 0.0
            or p.frequency_penalty != 0.0 or p.min_p > 0.0 or bool(p.logit_bias)
            or p.allowed_token_ids is not None or p.structured_outputs is not None
            or bool(p.bad_words)
            or (not spec and p.min_tokens > 0 and _can_stop(p)))


def _check_token_ids(p: SamplingParams, vocab: int) -> None:
    """vLLM's argument checks of the token-id fields of a request."""
    if p.allowed_token_ids is not None:
        if not p.allowed_token_ids:
            raise ValueError("allowed_token_ids is empty")
        if any(not 0 <= int(t) < vocab for t in p.allowed_token_ids):
            raise ValueError(f"allowed_token_ids out of the vocabulary [0, {vocab})")
    if p.logit_bias and any(not 0 <= int(t) < vocab for t in p.logit_bias):
        raise ValueError(f"logit_bias token id out of the vocabulary [0, {vocab})")


def _filters(p: SamplingParams, spec: bool = False) -> bool:
    """Whether the request needs the candidate sampling path (top-k / top-p,
    sampling penalties, min_p, logit_bias, allowed_token_ids or a grammar)."""
    return p.top_k not in (-1, 0) or p.top_p < 1.0 or _penalized(p, spec)


def chat_token_ids(tokenizer, messages, **kw) -> list[int]:
    """Token ids of ``tokenizer.apply_chat_template(messages, tokenize=True,
    **kw)``. Newer transformers return a mapping with ``input_ids`` (one
    conversation) instead of the id list."""
    out = tokenizer.apply_chat_template(messages, tokenize=True, **kw)
    if hasattr(out, "keys"):
        out = out["input_ids"]
    return [int(t) for t in out]


def _can_stop(p: SamplingParams) -> bool:
    """Whether a stop token can end the request before ``max_tokens``."""
    return not p.ignore_eos and bool(p.stop_token_ids)


def _stop_index(tokens, p: SamplingParams, start: int = 0) -> int | None:
    """Index of the first stop token at or after ``start`` that may end the
    output (its count exceeds ``min_tokens``), or None."""
    if not _can_stop(p):
        return None
    stops = set(p.stop_token_ids)
    for i in range(max(start, p.min_tokens), len(tokens)):
        if tokens[i] in stops:
            return i
    return None


def _truncate_at_stop(tokens: list[int], p: SamplingParams) -> list[int]:
    """Cut the output after the first stop token (kept, like vLLM's token ids)
    unless the request ignores EOS. Decode runs whole bursts on the device, so
    tokens of the burst past a stop are computed and dropped here."""
    i = _stop_index(tokens, p)
    return tokens if i is None else tokens[: i + 1]


def _finish_reason(tokens: list[int], p: SamplingParams, text_cut: str | None):
    """vLLM's (finish_reason, stop_reason) of a complete output: ("stop", the
    stop token id or the stop string) when a stop ended it, else ("length",
    None)."""
    if text_cut is not None:
        return "stop", text_cut
    if tokens and _can_stop(p) and len(tokens) > p.min_tokens \
            and tokens[-1] in set(p.stop_token_ids):
        return "stop", int(tokens[-1])
    return "length", None


def _cut_at_stop_string(tokens: list[int], p: SamplingParams, decode) -> tuple[list[int], str]:
    """(tokens, text) cut at the first stop string that ends after
    ``min_tokens`` tokens: the tokens up to the one that completes it, the
    text up to its start (or its end with ``include_stop_str_in_output``)."""
    return _match_stop_string(tokens, p, decode)[:2]


def _match_stop_string(tokens: list[int], p: SamplingParams, decode):
    """:func:`_cut_at_stop_string` plus the stop string that matched (None
    when none did)."""
    text = decode(tokens)
    if not p.stop:
        return tokens, text, None
    best = None
    for st in p.stop:
        at = text.find(st) if st else -1
        while at >= 0:
            end = at + len(st)
            # the first token count whose decoded prefix covers the stop string
            # (decoded length grows with the count: bisect)
            lo, hi = 1, len(tokens)
            while lo < hi:
                mid = (lo + hi) // 2
                if len(decode(tokens[:mid])) >= end:
                    hi = mid
                else:
                    lo = mid + 1
            k = lo
            if k > p.min_tokens:
                if best is None or at < best[0]:
                    best = (at, end, k, st)
                break
            at = text.find(st, at + 1)
    if best is None:
        return tokens, text, None
    at, end, k, st = best
    return tokens[:k], text[: end if p.include_stop_str_in_output else at], st


class LLM:
    def __init__(self, model: str | ModelConfig | dict = "llama-3.1-8b",
                 tensor_parallel_size: int | None = None, max_num_seqs: int = 256,
                 max_model_len: int = 4096, block_size: int = 16,
                 max_num_batched_tokens: int = 16384, gpu_memory_utilization: float = 0.90,
                 load_format: str = "dummy", seed: int = 0, enforce_eager: bool = False,
                 dtype=torch.bfloat16, num_kv_blocks: int | None = None,
                 tune_gemm: bool = True, gemm_lut_path: str | None = None,
                 speculative_k: int = 0, enable_prefix_caching: bool | None = None,
                 data_parallel_size: int = 1, enable_expert_parallel: bool = False,
                 prefix_cache_dir: str | None = None, tokenizer=None,
                 scheduling_policy: str = "fcfs"):
        self.cfg: ModelConfig = resolve(model)
        # tokenizer: an object with encode / decode (/ apply_chat_template), a
        # directory for transformers.AutoTokenizer, or None (then the checkpoint
        # directory's tokenizer is tried on first use)
        self._tokenizer = tokenizer
        self._grammar_compiler = None  # structured outputs (built on first use)
        if scheduling_policy not in ("fcfs", "priority"):
            raise ValueError(f"scheduling_policy must be fcfs or priority, not {scheduling_policy}")
        # priority: waiting requests are admitted lowest priority value first
        # (ties in arrival order); running requests are never preempted
        self.scheduling_policy = scheduling_policy
        self._tokenizer_src = None  # a checkpoint directory that ships tokenizer files
        if isinstance(model, str):
            from pathlib import Path

            d = Path(model)
            if d.is_dir() and any((d / f).exists() for f in ("tokenizer.json",
                                                              "tokenizer_config.json",
                                                              "tokenizer.model")):
                self._tokenizer_src = str(d)
        ps = pstate.get() if pstate._STATE is not None else None
        dp = int(data_parallel_size)
        if dp > 1:
            tp = int(tensor_parallel_size or 1)
            if tp > 1 and not enable_expert_parallel:
                raise NotImplementedError("data parallelism with TP > 1 inside each replica is "
                                          "the MoE TP x EP layout (enable_expert_parallel)")
            world = dp * tp
            ep = world if enable_expert_parallel else 1
            if ps is None or ps.tp_size != tp or ps.world_size != world or ps.ep_size != ep:
                ps = pstate.init(tp_size=tp, ep_size=ep)
            if ps.world_size != world:
                raise ValueError(f"data_parallel_size {dp} x tensor_parallel_size {tp} != "
                                 f"world size {ps.world_size}")
        elif ps is None or (tensor_parallel_size and ps.tp_size != tensor_parallel_size):
            ps = pstate.init(tp_size=tensor_parallel_size)
        self.ps = ps
        self.device = ps.device
        self.max_num_batched_tokens = max_num_batched_tokens
        self.model = build_model(self.cfg, self.device, dtype, ps)
        if load_format == "dummy":
            self.model.init_dummy(seed=seed)
        else:
            from ..models.loader import load_checkpoint

            load_checkpoint(self.model, model)
        if self.device.type == "cuda":
            from .. import _ext

            _ext.require()
            from ..ops import linear as _linear

            torch.ops._b200_C.init_device(self.device.index or 0)
            _linear.configure_workspace(self.device.index or 0)
            torch.cuda.synchronize()
        if num_kv_blocks is None:
            num_kv_blocks = self._size_kv(max_num_seqs, max_model_len, block_size,
                                          gpu_memory_utilization)
        num_sms = (torch.cuda.get_device_properties(self.device).multi_processor_count
                   if self.device.type == "cuda" else 148)
        self.ep = getattr(self.model, "ep_a2a", None)  # DP attention + all-to-all MoE
        self.runner = ModelRunner(self.model, max_num_seqs, max_model_len, block_size,
                                  num_kv_blocks, self.device,
                                  use_graphs=not enforce_eager and self.ep is None,
                                  num_sms=num_sms)
        if (self.device.type == "cuda" and ps.tp_size == 1 and self.ep is None
                and envs.get("VLLM_B200_FUSED_GEMM_NORM")):
            from ..parallel import comm, symm

            # Held by the engine too: its captured graphs bake in these buffers.
            self._local_norm = symm.LocalAddRmsNorm(
                self.device, max(max_num_batched_tokens, max_num_seqs), self.cfg.hidden_size)
            comm.set_local_gemm_norm(self._local_norm)
        if self.device.type == "cuda" and ps.tp_size > 1:
            from ..parallel import comm, symm

            comm.set_fused_ar_rmsnorm(symm.FusedArRmsNorm(
                ps, max(max_num_batched_tokens, max_num_seqs), self.cfg.hidden_size))
            # Sampler rows: decode rows, or (1 + k) verify rows per sequence.
            comm.set_tp_exchange(symm.TpExchange(ps, max_num_seqs * (1 + max(3, int(speculative_k))),
                                                 64))
        self.spec_k = int(speculative_k)
        if self.spec_k > 0 and self.ep is not None:
            raise NotImplementedError("speculative decoding with the all-to-all EP layout")
        if self.spec_k > 0:
            from ..models.mtp import MTPHead

            head = MTPHead(self.model, seed=seed + 1)
            if load_format != "dummy" and head.gated:
                from ..models.loader import SafetensorsIndex

                index = SafetensorsIndex(model)
                if "mtp.fc.weight" in index:  # the checkpoint ships its MTP layer
                    head.load_hf_state(index.get, has=index.__contains__)
            self.runner.enable_spec(head, self.spec_k)
        if self.device.type == "cuda" and tune_gemm:
            from . import warmup

            # decode batch sizes plus the full prefill chunk
            tune_ms = sorted(set(self.runner.capture_sizes) | {self.max_num_batched_tokens})
            warmup.engine_warmup(self.model, ps, tune_ms, gemm_lut_path,
                                 lm_ms=list(self.runner.capture_sizes))
        if self.spec_k == 0:
            self.runner.capture()
        self.last_stats: GenerateStats | None = None
        self.spec_hook = None  # spec_hook(rows, emitted tokens) after each speculative step
        # Prefix caching: content-addressed reuse of full prompt KV blocks. Not
        # for models with recurrent state or with a speculative draft head
        # (neither state is cached with the blocks).
        if enable_prefix_caching is None:
            enable_prefix_caching = bool(envs.get("VLLM_B200_PREFIX_CACHING"))
        hybrid = hasattr(self.model, "reset_slots")
        self.prefix_cache = None
        if enable_prefix_caching and not hybrid and self.spec_k == 0:
            host_blocks = int(envs.get("VLLM_B200_PREFIX_HOST_BLOCKS"))
            host = HostKVTier(self.runner.kv, host_blocks) if host_blocks > 0 else None
            disk = None
            disk_dir = prefix_cache_dir or envs.get("VLLM_B200_PREFIX_DISK_DIR")
            if disk_dir:
                disk = DiskKVTier(self.runner.kv, disk_dir,
                                  self._kv_namespace(model, load_format, seed, dtype),
                                  int(envs.get("VLLM_B200_PREFIX_DISK_BLOCKS")))
            self.prefix_cache = PrefixCache(self.runner.alloc, self.runner.block_size, host, disk)
        wd = int(envs.get("VLLM_B200_WATCHDOG_S"))
        self.watchdog = (StreamWatchdog(wd) if wd > 0 and self.device.type == "cuda" else None)

    def _kv_namespace(self, model, load_format: str, seed: int, dtype) -> str:
        """Name of this engine's KV bytes: model shapes, weight source, dtype,
        cache layout and TP position (the disk tier's directory)."""
        import hashlib
        import json
        from pathlib import Path

        src = model if isinstance(model, str) else None
        if src is not None and Path(src).exists():
            files = sorted(Path(src).glob("*.safetensors")) if Path(src).is_dir() else [Path(src)]
            src = [str(Path(src).resolve())] + [(f.name, f.stat().st_size, int(f.stat().st_mtime))
                                               for f in files]
        ident = {"cfg": self.cfg.to_dict(), "src": src, "format": load_format,
                 "seed": seed if load_format == "dummy" else None, "dtype": str(dtype),
                 "block": self.runner.block_size, "hkv": self.model.hkv, "d": self.model.d,
                 "tp": [self.ps.tp_size, self.ps.tp_rank]}
        blob = json.dumps(ident, sort_keys=True, default=str).encode()
        return hashlib.sha256(blob).hexdigest()[:20]

    def __enter__(self) -> "LLM":
        return self

    def __exit__(self, *exc) -> None:
        self.shutdown()

    def shutdown(self) -> None:
        """Release CUDA graphs (they may hold NCCL work) before the process
        group is destroyed."""
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        self.runner.release_graphs()
        from ..parallel import comm

        comm.set_fused_ar_rmsnorm(None)
        if getattr(self, "watchdog", None) is not None:
            self.watchdog.close()
            self.watchdog = None

    def _size_kv(self, max_num_seqs, max_model_len, block_size, util) -> int:
        m = self.model
        n_attn = len(getattr(m, "attn_layer_ids", range(self.cfg.num_layers)))
        per_block = 2 * n_attn * m.hkv * block_size * m.d * 2
        need = max_num_seqs * math.ceil(max_model_len / block_size) + 1
        if self.device.type != "cuda":
            return min(need, 4096)
        free, total = torch.cuda.mem_get_info(self.device)
        T = self.max_num_batched_tokens
        h = self.cfg.hidden_size
        act = T * (2 * h + 3 * max(self.cfg.intermediate_size, 1) // max(self.ps.tp_size, 1)
                   + (m.hq + 2 * m.hkv) * m.d * 2) * 2 * 2
        reserve = act + (4 << 30) + int((1 - util) * total)
        budget = max(0, free - reserve)
        return int(max(2, min(need, budget // per_block)))

    # ------------------------------------------------------------------ API
    # ------------------------------------------------------------------ text
    @property
    def tokenizer(self):
        """The tokenizer (loaded on first use), or None when there is none."""
        if isinstance(self._tokenizer, str) or (self._tokenizer is None and self._tokenizer_src):
            src = self._tokenizer if isinstance(self._tokenizer, str) else self._tokenizer_src
            self._tokenizer_src = None
            try:
                from transformers import AutoTokenizer

                self._tokenizer = AutoTokenizer.from_pretrained(src)
            except Exception:  # noqa: BLE001 - presets and bare configs have none
                self._tokenizer = None
        return self._tokenizer

    def _encode(self, text: str) -> list[int]:
        tok = self.tokenizer
        if tok is None:
            raise ValueError("text prompts need a tokenizer (LLM(..., tokenizer=...))")
        return list(tok.encode(text))

    def chat(self, messages, sampling_params: SamplingParams | None = None,
             chat_template_kwargs: dict | None = None, tools=None, use_tqdm: bool = False,
             chat_template: str | None = None, add_generation_prompt: bool = True,
             continue_final_message: bool = False) -> list[RequestOutput]:
        """vLLM's ``LLM.chat``: one conversation (a list of ``{"role",
        "content"}`` messages) or a list of them, through the tokenizer's
        chat template with the generation prompt appended."""
        tok = self.tokenizer
        if tok is None or not hasattr(tok, "apply_chat_template"):
            raise ValueError("chat needs a tokenizer with a chat template")
        convs = [messages] if messages and isinstance(messages[0], dict) else list(messages)
        kw = dict(chat_template_kwargs or {})
        if tools:
            kw["tools"] = tools
        if chat_template is not None:
            kw["chat_template"] = chat_template
        if continue_final_message:  # the reply extends the last (assistant) message
            if add_generation_prompt:
                raise ValueError("continue_final_message needs add_generation_prompt=False")
            kw["continue_final_message"] = True
        ids = [chat_token_ids(tok, c, add_generation_prompt=add_generation_prompt, **kw)
               for c in convs]
        return self.generate(ids, sampling_params)

    def score(self, prompt_token_ids, logits_rows: int = 1024) -> list[torch.Tensor]:
        """Teacher-forced log-probabilities (vLLM's ``prompt_logprobs``): for
        each prompt ``x`` of length L, ``lp[i] = log p(x[i+1] | x[:i+1])``
        for i < L - 1 (fp32, on the host). The prompt is prefilled in chunks
        of ``max_num_batched_tokens`` into scratch blocks; the LM head and
        log-softmax run on at most ``logits_rows`` rows at a time (the full
        vocabulary row of every token is not held at once). Call between
        ``generate`` calls (it uses batch slot 0)."""
        if isinstance(prompt_token_ids, torch.Tensor):
            prompts = [row for row in prompt_token_ids.to(torch.int64)]
        else:
            prompts = [torch.as_tensor(p, dtype=torch.int64) for p in prompt_token_ids]
        out = []
        for p in prompts:
            if p.numel() > self.runner.max_model_len:
                raise ValueError(f"prompt of {p.numel()} tokens > max_model_len")
            out.append(self._score_seq(0, p, 0, logits_rows)[0])
        if self.ep is not None:
            self.model.ep_drain()
        return out

    def embed(self, prompts, normalize: bool = True) -> list[torch.Tensor]:
        """vLLM's ``LLM.embed`` for a decoder: the final (normed) hidden state
        of each prompt's last token (last-token pooling), L2-normalised unless
        ``normalize`` is False; fp32 on the host. Text prompts need a
        tokenizer. Call between ``generate`` calls (it uses batch slot 0)."""
        if isinstance(prompts, str) or (isinstance(prompts, (list, tuple)) and prompts
                                        and isinstance(prompts[0], int)):
            prompts = [prompts]
        runner = self.runner
        out = []
        for p in prompts:
            seq = torch.as_tensor(self._encode(p) if isinstance(p, str) else p, dtype=torch.int64)
            L = seq.numel()
            if L > runner.max_model_len:
                raise ValueError(f"prompt of {L} tokens > max_model_len")
            nblk = math.ceil(L / runner.block_size)
            if runner.alloc.num_free() < nblk and self.prefix_cache is not None:
                self.prefix_cache.evict(nblk)
            blocks = runner.alloc.allocate(nblk)
            runner.set_block_row(0, blocks)
            try:
                pos, h = 0, None
                while pos < L:
                    n = min(self.max_num_batched_tokens, L - pos)
                    h = runner.prefill_hidden([(0, seq[pos:pos + n], pos, False, L)])
                    pos += n
                v = h[-1].float().cpu()
            finally:
                runner.alloc.free(blocks)
                runner.deactivate([0])
            out.append(torch.nn.functional.normalize(v, dim=0) if normalize else v)
        if self.ep is not None:
            self.model.ep_drain()
        return out

    def _score_seq(self, slot: int, seq: torch.Tensor, top_n: int = 0,
                   logits_rows: int = 1024):
        """Teacher-forced pass over ``seq`` through batch slot ``slot`` (which
        must be idle) on freshly allocated blocks, so no block another request
        or the prefix cache holds is rewritten. Returns (lp ``[L-1]``, top ids
        ``[L-1, top_n]``, top log-probs) -- the last two None when top_n is
        0 -- of the model's raw distribution (no temperature / top-k)."""
        runner = self.runner
        L = seq.numel()
        nblk = math.ceil(L / runner.block_size)
        if runner.alloc.num_free() < nblk and self.prefix_cache is not None:
            self.prefix_cache.evict(nblk)
        if runner.alloc.num_free() < nblk:
            raise RuntimeError("KV cache too small to score the sequence")
        blocks = runner.alloc.allocate(nblk)
        runner.set_block_row(slot, blocks)
        lp = torch.empty(max(L - 1, 0), dtype=torch.float32)
        tids = torch.empty(max(L - 1, 0), top_n, dtype=torch.int64) if top_n else None
        tlp = torch.empty(max(L - 1, 0), top_n, dtype=torch.float32) if top_n else None
        try:
            pos = 0
            while pos < L:
                n = min(self.max_num_batched_tokens, L - pos)
                h = runner.prefill_hidden([(slot, seq[pos:pos + n], pos, False, L)])
                m = min(n, L - 1 - pos)  # rows that predict a token of seq
                for a in range(0, m, logits_rows):
                    e = min(m, a + logits_rows)
                    lg = self.model.logits(h[a:e]).float()
                    lsm = lg - torch.logsumexp(lg, 1, keepdim=True)
                    tgt = seq[pos + a + 1:pos + e + 1].to(lg.device)
                    lp[pos + a:pos + e] = lsm.gather(1, tgt[:, None]).squeeze(1).cpu()
                    if top_n:
                        v, i = lsm.topk(top_n, dim=1)
                        tids[pos + a:pos + e] = i.cpu()
                        tlp[pos + a:pos + e] = v.cpu()
                pos += n
        finally:
            runner.alloc.free(blocks)
            runner.deactivate([slot])
        return lp, tids, tlp

    def model_ep_drain(self) -> None:
        """Serve the other ranks' expert traffic until every rank is idle (the
        all-to-all EP layout); a no-op otherwise."""
        if self.ep is not None:
            self.model.ep_drain()

    @staticmethod
    def _output(r: "_Req") -> RequestOutput:
        o = RequestOutput(r.rid, r.prompt.tolist(), r.out, True, logprobs=r.logprobs,
                          prompt_logprobs=r.prompt_logprobs)
        o.finish_reason, o.stop_reason = _finish_reason(r.out, r.params, None)
        if r.guide is not None and r.guide.done and not r.guide.failed \
                and o.finish_reason == "length":
            o.finish_reason = "stop"  # the grammar ended on its own stop token
        if r.guide is not None and r.guide.failed:
            o.error = "structured output: a sampled token broke the grammar"
        return o

    def _grammars(self):
        """The structured-output grammar compiler (built on first use)."""
        if self._grammar_compiler is None:
            tok = self.tokenizer
            if tok is None:
                raise ValueError("structured outputs need a tokenizer (LLM(..., tokenizer=...))")
            from .structured import GrammarCompiler

            try:
                self._grammar_compiler = GrammarCompiler(tok, self.cfg.vocab_size)
            except Exception as e:  # noqa: BLE001 - xgrammar cannot read this tokenizer
                raise ValueError(f"structured outputs: unsupported tokenizer ({e})") from e
        return self._grammar_compiler

    def _prompt_ids(self, p):
        """Token ids of one prompt: ids, text, or vLLM's prompt dicts
        (``TokensPrompt`` {"prompt_token_ids": ...} / ``TextPrompt``
        {"prompt": ...})."""
        if isinstance(p, dict):
            if "prompt_token_ids" in p:
                return list(p["prompt_token_ids"])
            if "prompt" in p:
                return self._encode(p["prompt"])
            raise ValueError("a prompt dict needs prompt_token_ids or prompt")
        return self._encode(p) if isinstance(p, str) else p

    def beam_search(self, prompts, params):
        """vLLM's ``LLM.beam_search``: ``params`` a ``BeamSearchParams``;
        one ``BeamSearchOutput`` (best ``beam_width`` sequences) per prompt."""
        from .beam_search import beam_search

        return beam_search(self, prompts, params)

    def get_tokenizer(self):
        """vLLM's ``LLM.get_tokenizer``."""
        return self.tokenizer

    def set_tokenizer(self, tokenizer) -> None:
        """vLLM's ``LLM.set_tokenizer``: text prompts, output text, stop
        strings and structured-output grammars use ``tokenizer`` from now on."""
        self._tokenizer, self._tokenizer_src = tokenizer, None
        self._grammar_compiler = None

    def _check_request(self, p: SamplingParams) -> None:
        """Argument checks of one request (ValueError): token ids in the
        vocabulary, and a structured-output grammar that compiles."""
        _check_token_ids(p, self.cfg.vocab_size)
        if p.structured_outputs is not None:
            self._grammars().compile(p.structured_outputs)
        self._bad_word_ids(p)

    def _bad_word_ids(self, p: SamplingParams) -> list[list[int]]:
        """Token sequences of a request's ``bad_words``, vLLM's way: each word
        as it starts the text and, when the tokenizer gives it a different
        first token of the same length, as it follows a space."""
        if not p.bad_words:
            return []
        tok = self.tokenizer
        if tok is None:
            raise ValueError("bad_words need a tokenizer (LLM(..., tokenizer=...))")

        def enc(text):
            try:
                return [int(t) for t in tok.encode(text, add_special_tokens=False)]
            except TypeError:  # tokenizers without the keyword
                return [int(t) for t in tok.encode(text)]

        out = []
        for w in p.bad_words:
            bare = enc(w.lstrip())
            if not bare:
                continue
            out.append(bare)
            spaced = enc(" " + w.lstrip())
            if spaced and spaced[0] != bare[0] and len(spaced) == len(bare):
                out.append(spaced)
        if any(not 0 <= t < self.cfg.vocab_size for w in out for t in w):
            raise ValueError(f"bad_words encode to ids outside the vocabulary [0, "
                             f"{self.cfg.vocab_size})")
        return out

    def _logprobs_of(self, r: "_Req") -> tuple[list | None, list | None]:
        """(output, prompt) log-prob lists of a finished request that asked
        for them: one ``{token id: log-prob}`` per token with the chosen token
        and the top-N."""
        sp = r.params
        top = max(sp.logprobs or 0, sp.prompt_logprobs or 0)
        seq = torch.cat([r.prompt, torch.tensor(r.out, dtype=torch.int64)])
        lp, tids, tlp = self._score_seq(r.slot, seq, top)
        Lp = r.prompt.numel()

        def entry(i: int, n: int) -> dict:  # token seq[i + 1]
            d = {int(seq[i + 1]): float(lp[i])}
            for j in range(n):
                d.setdefault(int(tids[i, j]), float(tlp[i, j]))
            return d

        out = None
        if sp.logprobs is not None:
            out = [entry(Lp - 1 + k, sp.logprobs) for k in range(len(r.out))]
        prompt = None
        if sp.prompt_logprobs is not None:
            prompt = [None] + [entry(i, sp.prompt_logprobs) for i in range(Lp - 1)]
        return out, prompt

    def generate(self, prompt_token_ids, sampling_params: SamplingParams | list | None = None,
                 collect_stats: bool = True, on_tokens=None,
                 stream_interval: int = 0, feed=None, on_finish=None,
                 use_tqdm: bool = False, priority: list[int] | None = None) -> list[RequestOutput]:
        """Serve the prompts to completion; returns one output per prompt.

        Streaming: ``on_tokens(request_index, new_token_ids, finished)`` is
        called with each request's new tokens after its prefill and after
        every decode burst (at most ``stream_interval`` steps per burst when
        > 0), and once with ``finished=True``; tokens after a stop token are
        not streamed. Under TP every rank must pass the same
        ``stream_interval`` (it sets the burst boundaries).

        Continuous batching (``feed``): ``feed(block)`` is called once per
        scheduler iteration and returns new requests ``[(request_id, prompt
        ids, SamplingParams)]`` (or ``("abort", request_id)`` to cancel one) to admit alongside the running ones (waiting
        for at least one when ``block`` is true: nothing runs), or None to
        finish once the running requests are done. Finished requests go to
        ``on_finish(RequestOutput)`` instead of the return value; a request
        that cannot be served (longer than ``max_model_len``, larger than the
        KV cache) finishes with ``error`` set while the others carry on.
        Bursts are at most ``stream_interval`` (default 8) steps, so arrivals
        join within a few steps. Under TP every rank's ``feed`` must return
        the same requests in the same calls (rank 0 broadcasts them)."""
        if sampling_params is None:
            sampling_params = SamplingParams()
        if isinstance(prompt_token_ids, (str, dict)) or (
                isinstance(prompt_token_ids, (list, tuple)) and prompt_token_ids
                and isinstance(prompt_token_ids[0], int)):
            prompt_token_ids = [prompt_token_ids]  # one prompt (text, token ids or a dict)
        if isinstance(prompt_token_ids, torch.Tensor):
            prompts = [row for row in prompt_token_ids.to(torch.int64)]
        else:
            prompts = [torch.as_tensor(self._prompt_ids(p), dtype=torch.int64)
                       for p in prompt_token_ids]
        params = (sampling_params if isinstance(sampling_params, list)
                  else [sampling_params] * len(prompts))
        if priority is not None:
            import dataclasses

            if self.scheduling_policy != "priority":
                raise ValueError("priority needs LLM(scheduling_policy='priority')")
            if len(priority) != len(prompts):
                raise ValueError("one priority per prompt")
            params = [dataclasses.replace(sp, priority=int(q)) for sp, q in zip(params, priority)]
        prompts = [p[-sp.truncate_prompt_tokens:] if sp.truncate_prompt_tokens
                   and sp.truncate_prompt_tokens > 0 else p for p, sp in zip(prompts, params)]
        if any(p.n > 1 for p in params) and feed is None:
            return self._generate_n(prompts, params, collect_stats, on_tokens, stream_interval)
        for p in params:
            self._check_request(p)
        spec = bool(self.spec_k)
        filtering = any(_filters(p, spec) for p in params)
        if filtering and self.spec_k:
            raise NotImplementedError("top-k / top-p / penalties / logit_bias / "
                                      "allowed_token_ids with speculative decoding")
        reqs = [_Req(i, prompts[i], params[i]) for i in range(len(prompts))]
        runner = self.runner
        runner.filtering = filtering
        runner.penalties = any(_penalized(p, spec) for p in params)
        try:
            return self._generate(reqs, on_tokens, int(stream_interval), feed, on_finish)
        finally:
            runner.filtering = False
            runner.penalties = False

    def _generate_n(self, prompts, params, collect_stats, on_tokens, stream_interval):
        """``n`` samples per prompt: each sample is its own request (distinct
        seeds: the given one + i, or the per-request default), run in one
        batch; sample i > 0 goes to the first sample's ``more``."""
        import dataclasses

        if on_tokens is not None:
            # A flat sample index is not a prompt index, and one callback stream
            # per prompt cannot carry several samples' tokens apart.
            raise ValueError("on_tokens streaming supports n = 1 per prompt only")
        flat_p, flat_sp, owner = [], [], []
        for i, (p, sp) in enumerate(zip(prompts, params)):
            for j in range(max(1, sp.n)):
                flat_p.append(p)
                flat_sp.append(dataclasses.replace(
                    sp, n=1, seed=None if sp.seed is None else int(sp.seed) + j))
                owner.append(i)
        outs = self.generate(flat_p, flat_sp, collect_stats, on_tokens, stream_interval)
        merged: list[RequestOutput] = []
        for i, o in zip(owner, outs):
            o.request_id = i  # every sample reports its prompt's index
            if i == len(merged):
                merged.append(o)
            else:
                merged[i].more = (merged[i].more or []) + [o]
        return merged

    def _generate(self, reqs: list[_Req], on_tokens=None, stream_interval: int = 0,
                  feed=None, on_finish=None) -> list[RequestOutput]:
        runner = self.runner
        online = feed is not None
        if online and on_finish is None:
            on_finish = lambda out: None  # noqa: E731 - e.g. TP followers
        if online and stream_interval <= 0:
            stream_interval = 8  # bounded bursts: arrivals join within a few steps
        # Online, models without recurrent state: one prefill chunk per scheduler
        # iteration, so the running requests decode between a long prompt's
        # chunks. The prompt's device block row is published only when its prefill
        # completes; until then its decode rows are padding (scratch block 0).
        # (Decode steps update every row's recurrent state, so hybrid models finish
        # a prompt's prefill before decoding.)
        interleave = online and not hasattr(self.model, "reset_slots")
        prefilling: deque = deque()

        def emit(rs, rows_h=None, final=False):
            """Hand each request's not-yet-streamed tokens to ``on_tokens``."""
            if on_tokens is None or not rs:
                return
            if rows_h is None:
                idx = torch.tensor([r.slot for r in rs], device=self.device)
                rows_h = runner.out_tokens.index_select(0, idx).cpu()
            for r, row in zip(rs, rows_h):
                upto = min(r.generated, r.params.max_tokens)
                new = [] if r.stream_stopped else row[r.streamed:upto].tolist()
                if new:
                    j = _stop_index(row[:upto].tolist(), r.params, r.streamed)
                    if j is not None:
                        new, r.stream_stopped = new[: j + 1 - r.streamed], True
                r.streamed = upto
                if new or final:
                    on_tokens(r.rid, new, final)

        bs = runner.block_size
        waiting = deque(reqs)
        running: list[_Req] = []
        free_slots = list(range(runner.B - 1, -1, -1))
        stats = GenerateStats()
        cuda = self.device.type == "cuda"
        ev = (lambda: torch.cuda.Event(enable_timing=True)) if cuda else None
        t0 = ev() if cuda else None
        if cuda:
            t0.record()
        wall0 = time.perf_counter()
        pending_first: list[tuple[object, list[_Req]]] = []
        decode_events: list[tuple[object, list[_Req], int]] = []
        prefill_spans: list[tuple[object, object]] = []
        stop_every = max(0, int(envs.get("VLLM_B200_STOP_CHECK_STEPS")))

        def scan_stops(rs) -> None:
            """Search the not-yet-scanned output tokens of requests that can
            end on a stop token (one device-to-host copy of the new columns);
            a hit retires the request now instead of at ``max_tokens``, which
            frees its slot and KV blocks for waiting requests. Every rank sees
            the same tokens, so TP ranks decide alike."""
            rs = [r for r in rs if not r.stop_hit and _can_stop(r.params)
                  and r.scanned < min(r.generated, r.params.max_tokens)]
            if not stop_every or not rs:
                return
            lo = min(r.scanned for r in rs)
            hi = max(min(r.generated, r.params.max_tokens) for r in rs)
            idx = torch.tensor([r.slot for r in rs], device=self.device)
            cols = runner.out_tokens.index_select(0, idx)[:, lo:hi].cpu()
            for r, row in zip(rs, cols):
                upto = min(r.generated, r.params.max_tokens)
                first = max(r.scanned, r.params.min_tokens)
                stops = set(r.params.stop_token_ids)
                if any(int(t) in stops for t in row[first - lo:upto - lo].tolist()):
                    r.stop_hit = True
                r.scanned = upto

        def advance_guides(rs) -> None:
            """Feed the new tokens of structured-output requests to their
            grammar matchers and upload each one's next allow-list row; a
            matcher that reached its grammar's end retires the request."""
            rs = [r for r in rs if r.guide is not None and not r.guide.done
                  and r.guide.accepted < min(r.generated, r.params.max_tokens)]
            if not rs:
                return
            lo = min(r.guide.accepted for r in rs)
            hi = max(min(r.generated, r.params.max_tokens) for r in rs)
            idx = torch.tensor([r.slot for r in rs], device=self.device)
            cols = runner.out_tokens.index_select(0, idx)[:, lo:hi].cpu()
            for r, row in zip(rs, cols):
                upto = min(r.generated, r.params.max_tokens)
                r.guide.advance(row[r.guide.accepted - lo:upto - lo].tolist())
                if r.guide.done:
                    r.stop_hit = True
                else:
                    runner.set_guide_row(r.slot, r.guide.next_row())

        def finished(r) -> bool:
            return r.generated >= r.params.max_tokens or r.aborted or r.stop_hit

        def cancel(rid) -> None:
            """Abort a request wherever it is: queued, mid-prefill or decoding
            (a decoding one finishes at the end of the current burst with the
            tokens it has)."""
            for r in list(waiting):
                if r.rid == rid:
                    waiting.remove(r)
                    on_finish(RequestOutput(r.rid, r.prompt.tolist(), [], True, error="aborted"))
            for r in list(prefilling):
                if r.rid == rid:
                    prefilling.remove(r)
                    runner.deactivate([r.slot])
                    runner.alloc.free(r.blocks)
                    free_slots.append(r.slot)
                    on_finish(RequestOutput(r.rid, r.prompt.tolist(), [], True, error="aborted"))
            for r in running:
                if r.rid == rid and not r.done:
                    r.aborted = True

        def pull() -> bool:
            """Queue the feed's new requests; False once it is closed."""
            items = feed(not waiting and not running and not prefilling)
            if items is None:
                return False
            for item in items:
                if item[0] == "abort":  # ("abort", request id)
                    cancel(item[1])
                    continue
                rid, ids, sp = item
                try:
                    self._check_request(sp)
                except ValueError as e:  # fail this request alone
                    on_finish(RequestOutput(rid, list(ids), [], True, error=str(e)))
                    continue
                if _filters(sp, bool(self.spec_k)):
                    if self.spec_k:
                        raise NotImplementedError("top-k / top-p / penalties / logit_bias / "
                                                  "allowed_token_ids with speculative decoding")
                    runner.filtering = True
                    runner.penalties = runner.penalties or _penalized(sp, bool(self.spec_k))
                ids = torch.as_tensor(ids, dtype=torch.int64)
                if sp.truncate_prompt_tokens and sp.truncate_prompt_tokens > 0:
                    ids = ids[-sp.truncate_prompt_tokens:]
                waiting.append(_Req(rid, ids, sp))
            return True

        feed_open = online
        while waiting or running or prefilling or feed_open:
            if feed_open:
                feed_open = pull()
                if not (waiting or running or prefilling):
                    continue
            # ---- admission
            admitted: list[_Req] = []
            if self.scheduling_policy == "priority" and len(waiting) > 1:
                order = sorted(waiting, key=lambda q: q.params.priority)  # stable: arrival ties
                waiting.clear()
                waiting.extend(order)
            while waiting and free_slots:
                r = waiting[0]
                L = r.prompt.numel()
                total = L + r.params.max_tokens + (self.spec_k + 1 if self.spec_k else 0)
                if total > runner.max_model_len:
                    msg = f"request {r.rid}: {total} tokens > max_model_len"
                    if not online:
                        raise ValueError(msg)
                    waiting.popleft()  # fail this request, keep serving the others
                    on_finish(RequestOutput(r.rid, r.prompt.tolist(), [], True, error=msg))
                    continue
                nblk = math.ceil(total / bs)
                pc = self.prefix_cache
                hit = pc.lookup(r.prompt)[1] if pc is not None else []
                need = nblk - len(hit)
                if pc is not None and runner.alloc.num_free() < need:
                    pc.evict(need)
                if runner.alloc.num_free() < need:
                    if hit:  # give the prefix references back
                        runner.alloc.free(torch.tensor(hit, dtype=torch.int32))
                    break
                waiting.popleft()
                r.slot = free_slots.pop()
                r.blocks = torch.cat([torch.tensor(hit, dtype=torch.int32),
                                      runner.alloc.allocate(need)])
                r.prefilled = len(hit) * bs  # cached KV: prefill starts after it
                runner.set_block_row(r.slot, r.blocks, device=not interleave)
                seed = r.params.seed if r.params.seed is not None else 0x9E3779B97F4A7C15 ^ r.rid
                sp = r.params
                runner.set_sampling(r.slot, 0.0 if sp.greedy else sp.temperature,
                                    seed & 0x7FFFFFFFFFFFFFFF, sp.top_k, sp.top_p,
                                    sp.repetition_penalty, sp.presence_penalty,
                                    sp.frequency_penalty,
                                    r.prompt if runner.penalties else None, sp.min_p,
                                    sp.logit_bias, sp.allowed_token_ids,
                                    sp.min_tokens if _can_stop(sp) and not self.spec_k else 0,
                                    sp.stop_token_ids)
                runner.set_bad_words(r.slot, self._bad_word_ids(sp))
                if sp.structured_outputs is not None:
                    r.guide = self._grammars().matcher(sp.structured_outputs)
                    runner.set_guide_row(r.slot, r.guide.next_row())
                else:
                    runner.set_guide_row(r.slot, None)
                admitted.append(r)
            if not admitted and not running and not prefilling:
                if not waiting:  # (online) every new request was refused above
                    continue
                if not online:
                    raise RuntimeError("cannot admit any request: KV cache too small")
                r = waiting.popleft()
                on_finish(RequestOutput(r.rid, r.prompt.tolist(), [], True,
                                        error="KV cache too small for this request"))
                continue
            # ---- chunked prefill of the admitted prompts
            if interleave:
                queue = prefilling
                queue.extend(admitted)
            else:
                queue = deque(admitted)
            while queue:
                budget = self.max_num_batched_tokens
                pieces, finishing = [], []
                while queue and budget > 0:
                    r = queue[0]
                    n = min(budget, r.prompt.numel() - r.prefilled)
                    last = r.prefilled + n == r.prompt.numel()
                    pieces.append((r.slot, r.prompt[r.prefilled:r.prefilled + n], r.prefilled,
                                   last, r.prompt.numel()))
                    r.prefilled += n
                    budget -= n
                    if last:
                        queue.popleft()
                        finishing.append(r)
                if self.watchdog is not None:
                    self.watchdog.check()
                if cuda:
                    e_pre = ev()
                    e_pre.record()
                tracing.push("prefill")
                runner.prefill(pieces)
                tracing.pop()
                if cuda:
                    e_post = ev()
                    e_post.record()
                    prefill_spans.append((e_pre, e_post))
                    if self.watchdog is not None:
                        self.watchdog.arm(e_post, "prefill chunk")
                for r in finishing:
                    r.generated = 1
                    if self.prefix_cache is not None:
                        self.prefix_cache.insert(r.prompt, r.blocks)
                if cuda and finishing:
                    e = ev()
                    e.record()
                    pending_first.append((e, finishing))
                if interleave and finishing:
                    runner.publish_rows([r.slot for r in finishing])
                emit([r for r in finishing if r.params.max_tokens > 1])
                running.extend(finishing)
                if interleave:
                    break  # one chunk, then a decode burst of the running requests
            # ---- decode until the next request finishes
            live = [r for r in running if not r.done]
            advance_guides(live)
            scan_stops(live)  # a first token (from prefill) may already stop
            finished_now = [r for r in live if finished(r)]
            if not live:
                continue  # (interleaved) only prompts mid-prefill
            if not finished_now and self.spec_k:
                n_rows = max(r.slot for r in live) + 1
                n = runner.spec_step(n_rows).cpu()
                stats.decode_steps += 1
                for r in live:
                    r.generated += int(n[r.slot])
                    stats.spec_tokens += int(n[r.slot])
                stats.spec_slots += len(live)
                if self.spec_hook is not None:
                    self.spec_hook(len(live), sum(int(n[r.slot]) for r in live))
                advance_guides(live)
                scan_stops(live)
                finished_now = [r for r in live if finished(r)]
                if cuda and finished_now:
                    e = ev()
                    e.record()
                    decode_events.append((e, finished_now, 1))
            elif not finished_now:
                steps = min(r.params.max_tokens - r.generated for r in live)
                if stream_interval > 0:
                    steps = min(steps, stream_interval)
                if stop_every and any(_can_stop(r.params) for r in live):
                    steps = min(steps, stop_every)
                if any(r.guide is not None for r in live):
                    steps = 1  # the next allow-list depends on this step's token
                n_rows = max(r.slot for r in live) + 1
                if self.watchdog is not None:
                    self.watchdog.check()
                tracing.push("decode")
                runner.decode(n_rows, steps)
                tracing.pop()
                stats.decode_steps += steps
                for r in live:
                    r.generated += steps
                advance_guides(live)
                scan_stops(live)
                finished_now = [r for r in live if finished(r)]
                if cuda:
                    e = ev()
                    e.record()
                    decode_events.append((e, finished_now, steps))
                    if self.watchdog is not None:
                        self.watchdog.arm(e, f"decode burst of {steps} steps")
            emit([r for r in live if r.generated < r.params.max_tokens])
            # ---- retire
            if finished_now:
                slots = [r.slot for r in finished_now]
                runner.deactivate(slots)
                outs = runner.out_tokens[torch.tensor(slots, device=self.device)]
                outs_h = outs.to("cpu", non_blocking=False)
                emit(finished_now, outs_h, final=True)
                for r, row in zip(finished_now, outs_h):
                    n_out = min(r.generated, r.params.max_tokens)
                    if r.guide is not None and r.guide.done:
                        n_out = min(n_out, r.guide.accepted + int(r.guide.failed))
                    r.out = _truncate_at_stop(row[:n_out].tolist(), r.params)
                    r.done = True
                    runner.alloc.free(r.blocks)
                    if r.params.logprobs is not None or r.params.prompt_logprobs is not None:
                        r.logprobs, r.prompt_logprobs = self._logprobs_of(r)
                    free_slots.append(r.slot)
                    if on_finish is not None:
                        o = self._output(r)
                        o.error = "aborted" if r.aborted else None
                        on_finish(o)
                running = [r for r in running if not r.done]
                if online:  # a long-lived session keeps no per-request records
                    pending_first.clear()
                    decode_events.clear()
                    prefill_spans.clear()
        if self.ep is not None:  # serve the other ranks' MoE traffic until all are done
            self.model.ep_drain()
        if cuda:
            t_end = ev()
            t_end.record()
            t_end.synchronize()
            for e, rs in pending_first:
                ms = t0.elapsed_time(e)
                for r in rs:
                    r.t_first = ms
            for e, rs, _ in decode_events:
                ms = t0.elapsed_time(e)
                for r in rs:
                    r.t_last = ms
            stats.total_ms = t0.elapsed_time(t_end)
            stats.prefill_ms = sum(a.elapsed_time(b) for a, b in prefill_spans)
            stats.decode_ms = stats.total_ms - stats.prefill_ms
        else:
            stats.total_ms = (time.perf_counter() - wall0) * 1e3
        outs = []
        for r in reqs:
            if r.t_first is not None:
                stats.ttft_ms.append(r.t_first)
                if r.t_last is not None and len(r.out) > 1:
                    stats.tpot_ms.append((r.t_last - r.t_first) / (len(r.out) - 1))
            o = self._output(r)
            o.ttft_s = None if r.t_first is None else r.t_first / 1e3
            o.tpot_s = None if not stats.tpot_ms else stats.tpot_ms[-1] / 1e3
            outs.append(o)
        self.last_stats = stats
        tok = self.tokenizer if outs else None
        if tok is not None:  # vLLM's RequestOutput.text (and stop strings)
            for o, r in zip(outs, reqs):
                sp = r.params
                if not sp.detokenize and not sp.stop:
                    continue
                dec = lambda ids, skip=sp.skip_special_tokens: tok.decode(  # noqa: E731
                    ids, skip_special_tokens=skip)
                o.output_token_ids, o.text, hit = _match_stop_string(o.output_token_ids, sp, dec)
                if not sp.detokenize:
                    o.text = None
                if hit is not None:
                    o.finish_reason, o.stop_reason = "stop", hit
        elif any(r.params.stop for r in reqs):
            raise ValueError("stop strings need a tokenizer (LLM(..., tokenizer=...))")
        return outs
