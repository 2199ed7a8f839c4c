"""Model runner: paged KV cache, device-resident decode state, chunked
prefill, and CUDA-graph-captured decode steps.

Decode metadata never leaves the device. Per batch slot the runner keeps
``seq_lens``, ``active``, the block-table row, the next input id and the
output cursor; a decode step derives positions / slot mappings from them,
runs the model, samples, appends the token to ``out_tokens`` and advances
the counters -- all inside one CUDA graph, so a step costs one graph launch
and no host<->device traffic. Blocks for ``prompt + max_tokens`` are
reserved at admission, so the block table is static while a request decodes.
Padded graph rows (``active == 0``) read and write only the reserved scratch
block 0.

Reference parity: upstream vLLM ``GPUModelRunner`` + the reference's graph
policy (``sm70/vllm_sm70/graph_policy.py:64-110``: capture sizes, decode-only
FULL graphs) and its lesson that host metadata building becomes the
bottleneck (``docs/history/sm70_flint_tp2_pcie.md:716-730``).
"""
from __future__ import annotations

import math

import torch

from .. import envs
from ..utils import launch_count
from ..models.layers import AttnMeta, KVCache
from .block_manager import build_prefill_meta, make_allocator
from .structured import mask_logits


def default_capture_sizes(max_bs: int) -> list[int]:
    sizes = [1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512]
    out = [s for s in sizes if s < max_bs] + [max_bs]
    return sorted(set(out))


class ModelRunner:
    def __init__(self, model, max_num_seqs: int, max_model_len: int, block_size: int,
                 num_blocks: int, device: torch.device, use_graphs: bool = True,
                 num_sms: int = 148):
        self.model = model
        self.cfg = model.cfg
        self.device = device
        self.B = max_num_seqs
        self.block_size = block_size
        self.max_model_len = max_model_len
        self.max_blocks = math.ceil(max_model_len / block_size)
        self.num_blocks = num_blocks
        self.num_sms = num_sms
        self.kv = KVCache.allocate(self.cfg.num_layers, num_blocks, model.hkv, block_size,
                                   model.d, dtype=model.dtype, device=device,
                                   layers=getattr(model, "attn_layer_ids", None))
        self.alloc = make_allocator(num_blocks, reserved=1)
        B, dev = self.B, device
        self.ids = torch.zeros(B, dtype=torch.int64, device=dev)
        self.seq_lens = torch.ones(B, dtype=torch.int32, device=dev)
        self.active = torch.zeros(B, dtype=torch.int32, device=dev)
        self.block_table = torch.zeros(B, self.max_blocks, dtype=torch.int32, device=dev)
        self.cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
        self.out_cap = max_model_len
        self.out_tokens = torch.zeros(B, self.out_cap, dtype=torch.int32, device=dev)
        self.out_pos = torch.zeros(B, dtype=torch.int64, device=dev)
        self.row_base = torch.arange(B, dtype=torch.int64, device=dev) * self.out_cap
        self.bt_host = torch.zeros(B, self.max_blocks, dtype=torch.int32).pin_memory() \
            if dev.type == "cuda" else torch.zeros(B, self.max_blocks, dtype=torch.int32)
        self.slot_ids = torch.arange(B, dtype=torch.int32, device=dev)
        self.temperature = torch.zeros(B, dtype=torch.float32, device=dev)
        self.seeds = torch.zeros(B, dtype=torch.int64, device=dev)
        self.top_k = torch.full((B,), -1, dtype=torch.int32, device=dev)
        self.top_p = torch.ones(B, dtype=torch.float32, device=dev)
        # sampling penalties (vLLM semantics), applied on the candidate path
        self.rep_pen = torch.ones(B, dtype=torch.float32, device=dev)
        self.pres_pen = torch.zeros(B, dtype=torch.float32, device=dev)
        self.freq_pen = torch.zeros(B, dtype=torch.float32, device=dev)
        self.min_p = torch.zeros(B, dtype=torch.float32, device=dev)
        self.prompt_ids: torch.Tensor | None = None  # [B, max_model_len], -1 padded
        # logit_bias / allowed_token_ids: per-slot sparse rows (token id, -1 =
        # unused), allocated on first use and widened to the longest request
        self.bias_ids: torch.Tensor | None = None    # [B, nb] int64
        self.bias_vals: torch.Tensor | None = None   # [B, nb] fp32
        self.allow_ids: torch.Tensor | None = None   # [B, na] int64; a row of -1 = no limit
        # min_tokens: the stop tokens are masked while fewer tokens exist
        self.min_tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.stop_ids: torch.Tensor | None = None    # [B, ns] int64
        # structured outputs: per-slot allow-list bitmask of the next token
        # (engine/structured.py), allocated on first use; -1 rows allow all
        self.guide: torch.Tensor | None = None       # [B, ceil(vocab / 32)] int32
        # bad_words: per slot, token sequences right-aligned in [B, words, L]
        # (-1 pads the front and unused words): the last token of a word is
        # banned when the output ends with the rest of it
        self.bad_words: torch.Tensor | None = None
        self.penalties = False
        # Decode graphs always sample through the temperature path: rows with
        # T <= 0 reduce to the exact greedy argmax.
        self.sampling = True
        # Top-k / top-p requests in flight: candidate sampling, eager decode
        # (the captured graphs hold the temperature path).
        self.filtering = False
        if hasattr(model, "allocate_states"):
            model.allocate_states(B)
        if hasattr(model, "reserve_workspace"):
            model.reserve_workspace(B)
        self.use_graphs = use_graphs and dev.type == "cuda" and envs.get("VLLM_B200_CUDA_GRAPHS")
        self.capture_sizes = default_capture_sizes(B)
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: dict[int, int] = {}
        self.split_bufs: dict[int, tuple] = {}
        self.pool = None
        # DP attention + all-to-all MoE: every forward starts with the ranks' vote
        self.ep = getattr(model, "ep_a2a", None)

    # ------------------------------------------------------------ block tables
    def set_block_row(self, slot: int, blocks: torch.Tensor, device: bool = True) -> None:
        """Host block-table row of ``slot`` (prefill metadata reads it) and,
        unless ``device`` is False, the device row decode steps read. A slot
        whose device row stays zero is decode padding: its decode rows read
        and write only the reserved scratch block 0 (see :meth:`publish_rows`)."""
        n = blocks.numel()
        self.bt_host[slot].zero_()
        self.bt_host[slot, :n] = blocks
        if device:
            self.block_table[slot].copy_(self.bt_host[slot], non_blocking=True)

    def publish_rows(self, slots: list[int]) -> None:
        """Copy the host block-table rows of ``slots`` to the device (a request
        whose prefill has completed joins the decode batch)."""
        for s in slots:
            self.block_table[s].copy_(self.bt_host[s], non_blocking=True)

    # ------------------------------------------------------------ decode
    def _splits_for(self, b: int) -> int:
        work = b * self.model.hkv
        return max(1, min(16, math.ceil(2 * self.num_sms / max(work, 1))))

    def _split_buffers(self, b: int):
        if b not in self.split_bufs:
            ns = self._splits_for(b)
            if ns > 1:
                po = torch.empty(ns, b, self.model.hq, self.model.d, device=self.device)
                pml = torch.empty(ns, b, self.model.hq, 2, device=self.device)
            else:
                po = pml = None
            self.split_bufs[b] = (ns, po, pml)
        return self.split_bufs[b]

    def _decode_body(self, b: int) -> None:
        bs = self.block_size
        sl = self.seq_lens[:b]
        pos = sl.to(torch.int64) - 1
        bt = self.block_table[:b]
        blk = torch.gather(bt, 1, (pos // bs).unsqueeze(1)).squeeze(1).to(torch.int64)
        slots = blk * bs + pos % bs
        ns, po, pml = self._split_buffers(b)
        meta = AttnMeta(positions=pos, slot_mapping=slots, block_table=bt, seq_lens=sl,
                        cu_q=self.cu_q[: b + 1], max_q_len=1, decode=True, num_splits=ns,
                        part_o=po, part_ml=pml, state_slots=self.slot_ids[:b])
        if self.ep is not None:
            self.ep.step(True, b)
        h = self.model.forward(self.ids[:b], meta, self.kv)
        if self.filtering:
            nxt = self.model.sample_filtered(h, self.temperature[:b], self.top_k[:b],
                                             self.top_p[:b], self._step_seeds(self.seeds[:b],
                                                                              self.out_pos[:b]),
                                             self._penalizer(self.slot_ids[:b].long()))
        elif self.sampling:
            nxt = self.model.sample(h, self.temperature[:b], self.seeds[:b], self.out_pos[:b])
        else:
            nxt = self.model.greedy(h)
        self.ids[:b].copy_(nxt)
        self.out_tokens.view(-1).index_copy_(0, self.row_base[:b] + self.out_pos[:b], nxt)
        act = self.active[:b]
        self.out_pos[:b] += act
        self.seq_lens[:b] += act

    def _penalizer(self, rows: torch.Tensor):
        """Logit rewrite for batch slots ``rows`` (None when no request in
        flight needs one), in vLLM's order: the structured-output grammar's
        allow-list and ``allowed_token_ids`` (every other
        token to -inf), ``logit_bias`` (added), the stop tokens to -inf while
        fewer than ``min_tokens`` tokens exist, then the penalties --
        repetition over prompt and output tokens (divide positive logits,
        multiply negative ones), presence and frequency over output tokens
        (subtract per occurrence) -- and last the ``min_p`` cut."""
        if not self.penalties:
            return None

        def sparse(ids_t, vals, vs, V):
            """Dense [b, V] sum of per-row (token id, value) pairs that fall
            in this rank's vocab shard [vs, vs + V)."""
            ids = ids_t.index_select(0, rows)
            loc = ids - vs
            ok = (ids >= 0) & (loc >= 0) & (loc < V)
            out = torch.zeros(ids.shape[0], V, device=ids.device)
            out.scatter_add_(1, loc.clamp(0, V - 1), torch.where(ok, vals, torch.zeros_like(vals)))
            return out

        def apply(lg: torch.Tensor, vs: int) -> torch.Tensor:
            b, V = lg.shape
            if self.guide is not None:
                lg = mask_logits(lg, self.guide.index_select(0, rows), vs)
            if self.bad_words is not None:
                lg = self._ban_bad_words(lg, rows, vs)
            if self.allow_ids is not None:
                a = self.allow_ids.index_select(0, rows)
                keep = sparse(self.allow_ids, torch.ones(a.shape, device=lg.device), vs, V) > 0
                limited = (a >= 0).any(1)
                lg = torch.where(limited[:, None] & ~keep, torch.full_like(lg, float("-inf")), lg)
            if self.bias_ids is not None:
                lg = lg + sparse(self.bias_ids, self.bias_vals.index_select(0, rows), vs, V)
            if self.stop_ids is not None:
                early = self.out_pos.index_select(0, rows) < self.min_tokens.index_select(0, rows)
                st = self.stop_ids.index_select(0, rows)
                hit = sparse(self.stop_ids, torch.ones(st.shape, device=lg.device), vs, V) > 0
                lg = torch.where(early[:, None] & hit, torch.full_like(lg, float("-inf")), lg)
            outs = self.out_tokens.index_select(0, rows).long()
            pos = self.out_pos.index_select(0, rows)
            ok = torch.arange(outs.shape[1], device=lg.device)[None, :] < pos[:, None]
            loc = outs - vs
            ok &= (loc >= 0) & (loc < V)
            counts = torch.zeros(b, V, device=lg.device)
            counts.scatter_add_(1, loc.clamp(0, V - 1), ok.float())
            pr = self.prompt_ids.index_select(0, rows)
            ploc = pr - vs
            pok = (pr >= 0) & (ploc >= 0) & (ploc < V)
            pseen = torch.zeros(b, V, device=lg.device)
            pseen.scatter_add_(1, ploc.clamp(0, V - 1), pok.float())
            seen = counts > 0
            rp = self.rep_pen.index_select(0, rows)[:, None]
            lg = torch.where(seen | (pseen > 0), torch.where(lg > 0, lg / rp, lg * rp), lg)
            lg = (lg - self.freq_pen.index_select(0, rows)[:, None] * counts
                  - self.pres_pen.index_select(0, rows)[:, None] * seen.float())
            mp = self.min_p.index_select(0, rows)
            if bool((mp > 0).any()):
                # p_i >= min_p * p_max  <=>  logit_i >= max logit + T * log(min_p),
                # with the row maximum over every vocab shard
                mx = lg.max(1).values
                from ..parallel import state as pstate

                if pstate.get().tp_size > 1:
                    import torch.distributed as dist

                    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=pstate.get().tp_group)
                t = self.temperature.index_select(0, rows).clamp_min(1e-6)
                cut = mx + t * torch.log(mp.clamp_min(1e-30))
                lg = torch.where((mp[:, None] > 0) & (lg < cut[:, None]),
                                 torch.full_like(lg, float("-inf")), lg)
            return lg
        return apply

    @staticmethod
    def _step_seeds(seeds: torch.Tensor, out_pos: torch.Tensor) -> torch.Tensor:
        """Per-row sampling key of the token at ``out_pos`` (fresh noise every
        step without a host-side counter)."""
        return seeds ^ (out_pos * 0x100000001)

    def bucket(self, n_rows: int) -> int:
        for s in self.capture_sizes:
            if s >= n_rows:
                return s
        raise ValueError(f"batch {n_rows} exceeds max_num_seqs {self.B}")

    def capture(self, sizes: list[int] | None = None) -> None:
        """Capture decode graphs (call at start-up, with no active requests)."""
        if not self.use_graphs:
            return
        sizes = sizes or self.capture_sizes
        assert int(self.active.sum()) == 0, "capture needs an idle runner"
        torch.cuda.synchronize()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for b in sizes:
                self._decode_body(b)  # warm-up: allocators, GEMM attributes
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        for b in sorted(sizes, reverse=True):
            g = torch.cuda.CUDAGraph()
            before = launch_count.total()
            with torch.cuda.graph(g, pool=self.pool):
                self._decode_body(b)
            self.graph_launches[b] = launch_count.total() - before
            self.graphs[b] = g
        torch.cuda.synchronize()
        # Capture/warm-up touched padded rows only; reset their counters.
        self.out_pos.zero_()
        self.seq_lens.fill_(1)

    def decode(self, n_rows: int, steps: int) -> None:
        b = self.bucket(n_rows)
        g = None if self.filtering else self.graphs.get(b)
        for _ in range(steps):
            if g is not None:
                g.replay()
            else:
                self._decode_body(b)
        if g is not None:
            launch_count.add(self.graph_launches[b] * steps)

    def release_graphs(self) -> None:
        self.graphs.clear()
        self.pool = None

    # ------------------------------------------------------------ prefill
    def set_sampling(self, slot: int, temperature: float, seed: int, top_k: int = -1,
                     top_p: float = 1.0, repetition_penalty: float = 1.0,
                     presence_penalty: float = 0.0, frequency_penalty: float = 0.0,
                     prompt: torch.Tensor | None = None, min_p: float = 0.0,
                     logit_bias: dict | None = None,
                     allowed_token_ids: list | None = None, min_tokens: int = 0,
                     stop_token_ids: list | None = None) -> None:
        self.temperature[slot] = float(temperature)
        self.seeds[slot] = int(seed)
        self.top_k[slot] = int(top_k) if top_k > 0 else -1
        self.top_p[slot] = float(top_p)
        self.rep_pen[slot] = float(repetition_penalty)
        self.pres_pen[slot] = float(presence_penalty)
        self.freq_pen[slot] = float(frequency_penalty)
        self.min_p[slot] = float(min_p)
        bias = sorted((int(t), float(v)) for t, v in (logit_bias or {}).items())
        self.bias_ids, self.bias_vals = self._sparse_row(
            self.bias_ids, self.bias_vals, slot, [t for t, _ in bias], [v for _, v in bias])
        self.allow_ids, _ = self._sparse_row(self.allow_ids, None, slot,
                                             sorted({int(t) for t in allowed_token_ids or []}))
        self.min_tokens[slot] = int(min_tokens)
        self.stop_ids, _ = self._sparse_row(
            self.stop_ids, None, slot,
            sorted({int(t) for t in stop_token_ids or []}) if min_tokens > 0 else [])
        if prompt is not None:  # the prompt's tokens count for the repetition penalty
            if self.prompt_ids is None:
                self.prompt_ids = torch.full((self.B, self.max_model_len), -1, dtype=torch.int64,
                                             device=self.device)
            self.prompt_ids[slot].fill_(-1)
            self.prompt_ids[slot, : prompt.numel()] = prompt.to(self.device)

    def _ban_bad_words(self, lg: torch.Tensor, rows: torch.Tensor, vs: int) -> torch.Tensor:
        """-inf for the last token of every bad word whose preceding tokens
        are the last output tokens of the row (vLLM's rule; output tokens
        only, so a word longer than the output so far + 1 cannot match)."""
        b, V = lg.shape
        bw = self.bad_words.index_select(0, rows)                  # [b, W, L]
        L = bw.shape[2]
        last = bw[:, :, L - 1]
        hit = last >= 0
        if L > 1:
            pos = self.out_pos.index_select(0, rows)
            idx = pos[:, None] - (L - 1) + torch.arange(L - 1, device=lg.device)[None, :]
            tail = self.out_tokens.index_select(0, rows).long().gather(1, idx.clamp_min(0))
            tail = torch.where(idx >= 0, tail, torch.full_like(tail, -2))   # [b, L-1]
            pref = bw[:, :, : L - 1]
            hit &= ((pref < 0) | (pref == tail[:, None, :])).all(2)
        loc = last - vs
        hit &= (loc >= 0) & (loc < V)
        ban = torch.zeros(b, V, device=lg.device)
        ban.scatter_add_(1, loc.clamp(0, V - 1), hit.float())
        return torch.where(ban > 0, torch.full_like(lg, float("-inf")), lg)

    def set_bad_words(self, slot: int, words: list[list[int]] | None) -> None:
        """Token sequences of ``slot``'s bad words (None / empty: none)."""
        words = [list(w) for w in words or [] if w]
        if self.bad_words is None and not words:
            return
        W = max(len(words), 1 if self.bad_words is None else self.bad_words.shape[1])
        L = max([len(w) for w in words] + [1 if self.bad_words is None else
                                           self.bad_words.shape[2]])
        if self.bad_words is None or self.bad_words.shape[1:] != (W, L):
            t = torch.full((self.B, W, L), -1, dtype=torch.int64, device=self.device)
            if self.bad_words is not None:
                _, w0, l0 = self.bad_words.shape
                t[:, :w0, L - l0:] = self.bad_words
            self.bad_words = t
        row = torch.full((W, L), -1, dtype=torch.int64)
        for i, w in enumerate(words):
            row[i, L - len(w):] = torch.tensor(w, dtype=torch.int64)
        self.bad_words[slot].copy_(row.to(self.device))

    def set_guide_row(self, slot: int, row: torch.Tensor | None) -> None:
        """Allow-list bitmask of ``slot``'s next token ([1, words] int32, from
        the request's grammar matcher), or None to lift the limit."""
        if row is None:
            if self.guide is not None:
                self.guide[slot].fill_(-1)
            return
        if self.guide is None:
            self.guide = torch.full((self.B, row.shape[-1]), -1, dtype=torch.int32,
                                    device=self.device)
        self.guide[slot].copy_(row.reshape(-1), non_blocking=False)

    def _sparse_row(self, ids_t, vals_t, slot: int, ids: list, vals: list | None = None):
        """Write ``slot``'s row of a per-slot sparse table (ids padded with -1,
        values with 0), allocating the table on first use and widening it to
        the longest row; a slot without entries only clears its row."""
        n = len(ids)
        if ids_t is None and n == 0:
            return ids_t, vals_t
        if ids_t is None or ids_t.shape[1] < n:
            w = max(n, 2 * (0 if ids_t is None else ids_t.shape[1]), 8)
            new_ids = torch.full((self.B, w), -1, dtype=torch.int64, device=self.device)
            new_vals = torch.zeros(self.B, w, dtype=torch.float32, device=self.device)
            if ids_t is not None:
                new_ids[:, : ids_t.shape[1]] = ids_t
                if vals_t is not None:
                    new_vals[:, : vals_t.shape[1]] = vals_t
            ids_t, vals_t = new_ids, (new_vals if vals is not None else None)
        ids_t[slot].fill_(-1)
        if n:
            ids_t[slot, :n] = torch.tensor(ids, dtype=torch.int64).to(self.device)
        if vals_t is not None:
            vals_t[slot].zero_()
            if n:
                vals_t[slot, :n] = torch.tensor(vals, dtype=torch.float32).to(self.device)
        return ids_t, vals_t

    def prefill(self, pieces: list[tuple[int, torch.Tensor, int, bool, int]]) -> None:
        """``pieces``: (slot, token ids [n] int64 CPU, ctx_start, is_last, total_len)."""
        h, cu, h2d = self._prefill_forward(pieces)
        self._sample_last(pieces, h, cu, h2d)

    def prefill_hidden(self, pieces) -> torch.Tensor:
        """The forward of :meth:`prefill` without sampling: the final hidden
        states of every token of the chunk (``[sum n, H]``)."""
        return self._prefill_forward(pieces)[0]

    def _prefill_forward(self, pieces):
        dev = self.device
        S = len(pieces)
        toks = torch.cat([p[1] for p in pieces])
        q_len = torch.tensor([p[1].numel() for p in pieces], dtype=torch.int32)
        ctx = torch.tensor([p[2] for p in pieces], dtype=torch.int32)
        slots_idx = [p[0] for p in pieces]
        bt_rows = self.bt_host[slots_idx]
        pos, slot_map = build_prefill_meta(bt_rows, ctx, q_len, self.block_size)
        seq_lens = ctx + q_len
        cu = torch.zeros(S + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(q_len, 0)
        pin = dev.type == "cuda"

        def h2d(t):
            return (t.pin_memory() if pin else t).to(dev, non_blocking=True)

        ids_d = h2d(toks)
        state_slots = h2d(torch.tensor(slots_idx, dtype=torch.int32))
        fresh = [p[0] for p in pieces if p[2] == 0]
        if fresh and hasattr(self.model, "reset_slots"):
            self.model.reset_slots(h2d(torch.tensor(fresh, dtype=torch.int64)))
        meta = AttnMeta(positions=h2d(pos), slot_mapping=h2d(slot_map),
                        block_table=h2d(bt_rows), seq_lens=h2d(seq_lens), cu_q=h2d(cu),
                        max_q_len=int(q_len.max()), decode=False, state_slots=state_slots)
        if self.ep is not None:
            self.ep.step(True, int(toks.numel()))
        return self.model.forward(ids_d, meta, self.kv), cu, h2d

    def _sample_last(self, pieces, h, cu, h2d) -> None:
        """First output token of every piece that completes its prompt."""
        last = [i for i, p in enumerate(pieces) if p[3]]
        if not last:
            return
        rows = h2d(torch.tensor([int(cu[i + 1]) - 1 for i in last], dtype=torch.int64))
        h_last = h.index_select(0, rows)
        sidx = h2d(torch.tensor([pieces[i][0] for i in last], dtype=torch.int64))
        if self.filtering:  # first output token: out_pos 0
            nxt = self.model.sample_filtered(h_last, self.temperature.index_select(0, sidx),
                                             self.top_k.index_select(0, sidx),
                                             self.top_p.index_select(0, sidx),
                                             self.seeds.index_select(0, sidx),
                                             self._penalizer(sidx))
        elif self.sampling:
            nxt = self.model.sample(h_last, self.temperature.index_select(0, sidx),
                                    self.seeds.index_select(0, sidx), None, offset=0)
        else:
            nxt = self.model.greedy(h_last)
        total = h2d(torch.tensor([pieces[i][4] + 1 for i in last], dtype=torch.int32))
        self.ids.index_copy_(0, sidx, nxt.to(torch.int64))
        self.seq_lens.index_copy_(0, sidx, total)
        self.out_tokens.view(-1).index_copy_(0, self.row_base.index_select(0, sidx), nxt)
        self.out_pos.index_fill_(0, sidx, 1)
        self.active.index_fill_(0, sidx, 1)
        if getattr(self, "spec_k", 0):
            self.last_hidden.index_copy_(0, sidx, h_last)

    # ------------------------------------------------------------ speculative decoding
    def enable_spec(self, mtp, k: int) -> None:
        """Attach an MTP draft head drafting ``k`` tokens per step."""
        self.mtp = mtp
        self.spec_k = k
        mtp.allocate_cache(self.num_blocks, self.block_size)
        H = self.cfg.hidden_size
        self.last_hidden = torch.zeros(self.B, H, dtype=self.model.dtype, device=self.device)
        self.spec_offset = 0

    def _meta_for(self, b: int, q_len: int, start_pos: torch.Tensor, decode: bool = True,
                  spec_verify: bool = False) -> AttnMeta:
        """Metadata for ``q_len`` consecutive tokens per row starting at
        ``start_pos[row]`` (rows 0..b-1 of the batch)."""
        bs = self.block_size
        dev = self.device
        pos = (start_pos.to(torch.int64)[:, None] + torch.arange(q_len, device=dev)[None, :])
        bt = self.block_table[:b]
        blk = torch.gather(bt, 1, (pos // bs)).to(torch.int64)
        slots = (blk * bs + pos % bs).reshape(-1)
        seq_lens = (start_pos + q_len).to(torch.int32)
        cu = torch.arange(b + 1, device=dev, dtype=torch.int32) * q_len
        return AttnMeta(positions=pos.reshape(-1), slot_mapping=slots, block_table=bt,
                        seq_lens=seq_lens, cu_q=cu, max_q_len=q_len, decode=decode,
                        state_slots=self.slot_ids[:b], spec_verify=spec_verify)

    def spec_step(self, b: int) -> torch.Tensor:
        """One draft (MTP, k tokens) + verify (target, k+1 tokens) + rejection
        step over rows 0..b-1. Returns the number of tokens emitted per row
        (device int32; 0 for inactive rows)."""
        from ..ops import sampling

        k = self.spec_k
        m = self.model
        act = self.active[:b]
        sl = self.seq_lens[:b]               # context incl. ids[row] (at position sl - 1)
        base = sl.to(torch.int64) - 1
        tok = self.ids[:b]
        hid = self.last_hidden[:b]
        temp, seeds = self.temperature[:b], self.seeds[:b]
        d_ids, d_logits = [], []
        for j in range(k):
            meta = self._meta_for(b, 1, base + j)
            hid = self.mtp.forward(tok, hid, meta)
            lg = m.logits(hid)
            nxt, _ = sampling.gumbel_sample(lg, temp, seeds, self.spec_offset * 64 + j)
            tok = nxt.to(torch.int64)
            d_ids.append(nxt)
            d_logits.append(lg if not lg.is_cuda else lg.to(torch.bfloat16))
        draft_ids = torch.stack(d_ids, 1).contiguous()                  # [b, k] int32
        toks = torch.cat([self.ids[:b, None], draft_ids.to(torch.int64)], 1).reshape(-1)
        meta = self._meta_for(b, k + 1, base, decode=True, spec_verify=True)
        hidden = m.forward(toks, meta, self.kv)                          # [b*(k+1), H]
        tl = m.logits(hidden)
        tl = (tl.to(torch.bfloat16) if tl.is_cuda else tl).view(b, k + 1, -1)
        out, n = sampling.rejection_sample(tl, torch.stack(d_logits, 1), draft_ids, temp, seeds,
                                           self.spec_offset * 64 + 63)
        self.spec_offset += 1
        n = n * act
        if hasattr(m, "commit_spec"):
            m.commit_spec(n, k + 1, self.slot_ids[:b])
        # commit: emitted tokens, counters, next input id and hidden
        nl = n.to(torch.int64)
        last = torch.gather(out.to(torch.int64), 1, (nl - 1).clamp(min=0)[:, None]).squeeze(1)
        self.ids[:b] = torch.where(nl > 0, last, self.ids[:b])
        hv = hidden.view(b, k + 1, -1)
        hsel = torch.gather(hv, 1, (nl - 1).clamp(min=0)[:, None, None].expand(b, 1, hv.shape[2]))
        self.last_hidden[:b] = torch.where((nl > 0)[:, None], hsel.squeeze(1), self.last_hidden[:b])
        cols = self.out_pos[:b, None] + torch.arange(k + 1, device=self.device)[None, :]
        valid = torch.arange(k + 1, device=self.device)[None, :] < nl[:, None]
        flat_idx = (self.row_base[:b, None] + cols.clamp(max=self.out_cap - 1))[valid]
        self.out_tokens.view(-1).index_copy_(0, flat_idx, out[valid])
        self.out_pos[:b] += nl
        self.seq_lens[:b] += n
        return n

    def deactivate(self, slots: list[int]) -> None:
        if not slots:
            return
        idx = torch.tensor(slots, dtype=torch.int64, device=self.device)
        self.active.index_fill_(0, idx, 0)
        self.seq_lens.index_fill_(0, idx, 1)
        self.out_pos.index_fill_(0, idx, 0)
        self.block_table.index_fill_(0, idx, 0)
        for s in slots:
            self.bt_host[s].zero_()
