"""Expert parallelism with data-parallel attention: each rank serves its own
requests (attention, dense layers and the LM head are replicated, no TP
collective), and the MoE blocks exchange tokens with the ranks that own
their experts.

Per MoE block, on every rank of the EP group:

  dispatch  for each local token, one row per destination rank that owns at
            least one of its top-k experts (rank d owns experts
            ``[d*E/W, (d+1)*E/W)``); rows are ordered by (destination, token).
            Each row carries the hidden vector and the token's full routing
            (k ids + k weights), so the receiver needs no other state: its
            grouped expert GEMMs compute only the ids it owns.
  experts   the received rows through the local experts (one bf16 partial
            sum per row over the experts of this rank).
  combine   the partial rows go back to their source rank, which sums them
            in rank order in fp32 (deterministic, independent of arrival
            order) and rounds once -- the same arithmetic as the TP
            expert-slice path, whose all-reduce sums the bf16 partials in
            rank order.

Transport (this module): ``torch.distributed.all_to_all_single`` over the EP
group -- NCCL on GPUs, gloo on CPU -- after a count exchange, with the row
payload (hidden bytes + routing) packed into one tensor so a block costs
three collectives (counts, dispatch, combine). This is the baseline path;
the split sizes live on the host, so the MoE block is not graph-captured in
this mode.

Lock-step: every forward on every rank is preceded by one ``step()`` vote
over the CPU group. A rank with no work of its own votes "idle" and runs
``idle_pass`` -- every MoE block with zero local tokens, which still serves
the tokens other ranks send to its experts -- until a vote finds no rank
active. So all ranks enter the same collectives in the same order.

Reference parity: the reference refuses expert parallelism
(``sm70/vllm_sm70/fused_moe/method.py:357-358``); the mode follows upstream
vLLM's ``--data-parallel-size N --enable-expert-parallel`` serving layout
(data-parallel attention, all-to-all MoE).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DispatchPlan:
    T: int                   # local tokens
    t_idx: torch.Tensor      # [n_send] token of each sent row, (destination, token) order
    send: list[int]          # rows sent to each rank
    recv: list[int]          # rows received from each rank


class EPAllToAll:
    def __init__(self, ps, num_experts: int, top_k: int):
        assert ps.ep_size > 1 and num_experts % ps.ep_size == 0, (ps.ep_size, num_experts)
        self.W = ps.ep_size
        self.rank = ps.ep_rank
        self.group = ps.ep_group
        self.cpu_group = ps.cpu_group
        self.E_local = num_experts // ps.ep_size
        self.k = top_k
        self.sent_rows = 0       # rows dispatched by this rank (statistics)
        self.recv_rows = 0       # rows served by this rank's experts

    # -------------------------------------------------------------- lock-step
    def step(self, active: bool) -> int:
        """Vote before a forward; returns how many ranks are active in it."""
        t = torch.tensor([1 if active else 0], dtype=torch.int64)
        dist.all_reduce(t, group=self.cpu_group)
        return int(t.item())

    # -------------------------------------------------------------- transport
    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits) -> None:
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                               input_split_sizes=in_splits, group=self.group)

    def dispatch(self, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor):
        """``x [T, H]``, routing ``w [T, k]`` fp32 / ``ids [T, k]`` int32 ->
        (received rows ``[N, H]``, their weights ``[N, k]``, ids ``[N, k]``,
        plan)."""
        T, H = x.shape
        k = self.k
        dev = x.device
        dest = ids.to(torch.int64) // self.E_local                      # [T, k]
        mask = torch.zeros(T, self.W, dtype=torch.bool, device=dev)
        if T:
            mask.scatter_(1, dest, True)
        nz = mask.t().nonzero()                                          # (d, t), d-major
        t_idx = nz[:, 1]
        send_counts = mask.sum(0).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        send, recv = send_counts.tolist(), recv_counts.tolist()
        # one packed row per (token, destination): hidden bytes | ids | weight bits
        xb = x.index_select(0, t_idx).contiguous().view(torch.uint8)
        meta = torch.cat([ids.index_select(0, t_idx),
                          w.index_select(0, t_idx).contiguous().view(torch.int32)], 1)
        payload = torch.cat([xb, meta.contiguous().view(torch.uint8)], 1)
        hb = H * x.element_size()
        got = torch.empty(sum(recv), hb + 8 * k, dtype=torch.uint8, device=dev)
        self._a2a(got, payload, recv, send)
        xr = got[:, :hb].contiguous().view(x.dtype)
        mr = got[:, hb:].contiguous().view(torch.int32)
        idr = mr[:, :k].contiguous()
        wr = mr[:, k:].contiguous().view(torch.float32)
        self.sent_rows += len(t_idx)
        self.recv_rows += xr.shape[0]
        return xr, wr, idr, DispatchPlan(T, t_idx, send, recv)

    def combine(self, yr: torch.Tensor, plan: DispatchPlan, shared: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Partial outputs of the received rows back to their source ranks;
        ``out[t] = round(sum over destinations in rank order + shared)``."""
        H = yr.shape[1]
        ys = torch.empty(sum(plan.send), H, dtype=yr.dtype, device=yr.device)
        self._a2a(ys, yr.contiguous(), plan.send, plan.recv)
        acc = torch.zeros(plan.T, H, dtype=torch.float32, device=yr.device)
        off = 0
        for n in plan.send:  # rank order; indices are unique within one source
            if n:
                acc.index_add_(0, plan.t_idx[off:off + n], ys[off:off + n].float())
            off += n
        if shared is not None:
            acc += shared.float()
        if out is None:
            out = torch.empty(plan.T, H, dtype=yr.dtype, device=yr.device)
        out.copy_(acc)
        return out
