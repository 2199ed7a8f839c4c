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

Transport: on GPUs, ``EPPeer`` -- this library's own kernels storing the rows
straight into the owners' symmetric buffers over NVLink and the partial rows
back into their sources' (csrc/comm/ep_a2a.cu: no host round trip, no NCCL
call inside the block; bit-identical results to the baseline). Otherwise
``torch.distributed.all_to_all_single`` over the EP group -- NCCL on GPUs,
gloo on CPU -- after a count exchange, with the row payload (hidden bytes +
routing) packed into one tensor so a block costs three collectives (counts,
dispatch, combine): the baseline path (``VLLM_B200_FUSED_EP_A2A=0``), whose
split sizes live on the host.

Lock-step: every forward on every rank is preceded by one ``step()`` vote
over the CPU group (which also shares every rank's token count: the peer
path sizes its receive buffers from their sum). A rank with no work of its own votes "idle" and runs
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

from ..utils import launch_count


@dataclass
class DispatchPlan:
    T: int                   # local tokens
    t_idx: torch.Tensor      # [n_send] token of each sent row, (destination, token) order
    send: list[int]          # rows sent to each rank
    recv: list[int]          # rows received from each rank


@dataclass
class PeerPlan:
    T: int                   # local tokens
    n_max: int               # rows of the compacted receive buffers


class EPPeer:
    """Token exchange over peer memory (kernels in csrc/comm/ep_a2a.cu).

    Symmetric buffers over the EP group, allocated once (a collective: every
    rank constructs this with the same sizes): recv rows / routing / returned
    partial rows for ``T_cap`` tokens per source rank, plus a signal pad.
    Peer addresses come from the symmetric-memory rendezvous; only this
    library's kernels touch them, with plain NVLink loads and stores."""

    def __init__(self, ps, E_local: int, top_k: int, hidden: int, T_cap: int):
        import torch.distributed._symmetric_memory as symm_mem

        from .. import envs

        self.W, self.rank, self.E_local, self.k, self.H = ps.ep_size, ps.ep_rank, E_local, top_k, hidden
        self.T_cap = T_cap
        dev = ps.device
        W = self.W

        def alloc(n, dt):
            t = symm_mem.empty(n, dtype=dt, device=dev)
            return t, symm_mem.rendezvous(t, ps.ep_group)

        self.recv_x, hx = alloc(W * T_cap * hidden, torch.bfloat16)
        self.recv_meta, hm = alloc(W * T_cap * 2 * top_k, torch.int32)
        self.back_y, hy = alloc(W * T_cap * hidden, torch.bfloat16)
        self.pad, hp = alloc(64, torch.int32)
        self.pad.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=ps.cpu_group)
        self._handles = (hx, hm, hy, hp)
        self.bufs = []
        for r in range(W):
            self.bufs += [int(hx.buffer_ptrs[r]), int(hm.buffer_ptrs[r]), int(hy.buffer_ptrs[r]),
                          int(hp.buffer_ptrs[r])]
        self.timeout_ms = int(envs.get("VLLM_B200_COMM_TIMEOUT_MS"))
        self.slot = torch.empty(T_cap * W, dtype=torch.int32, device=dev)
        self.send_count = torch.empty(W, dtype=torch.int32, device=dev)
        self.n_rows = torch.zeros(1, dtype=torch.int32, device=dev)
        self._recv = None

    def _recv_buffers(self, n_max: int, device):
        if self._recv is None or self._recv[0].shape[0] < n_max:
            n = max(n_max, 64)
            self._recv = (torch.empty(n, self.H, dtype=torch.bfloat16, device=device),
                          torch.empty(n, self.k, dtype=torch.int32, device=device),
                          torch.empty(n, self.k, dtype=torch.float32, device=device),
                          torch.empty(n, dtype=torch.int32, device=device))
        return tuple(b[:n_max] for b in self._recv)

    def _args(self):
        return (self.bufs, self.rank, self.E_local, self.T_cap, self.timeout_ms)

    def dispatch(self, x, w, ids, n_max: int):
        ops = torch.ops._b200_C
        T = x.shape[0]
        ops.ep_dispatch(*self._args(), x.contiguous(), ids.to(torch.int32).contiguous(),
                        w.float().contiguous(), self.slot, self.send_count)
        xc, idc, wc, rs = self._recv_buffers(n_max, x.device)
        ops.ep_receive(*self._args(), xc, idc, wc, rs, self.n_rows)
        self._row_src = rs
        launch_count.add(3)
        return xc, wc, idc, PeerPlan(T, n_max)

    def combine(self, yr, plan: PeerPlan, shared=None, out=None):
        ops = torch.ops._b200_C
        if out is None:
            out = torch.empty(plan.T, self.H, dtype=yr.dtype, device=yr.device)
        ops.ep_return(*self._args(), self.k, yr.contiguous(), self._row_src, self.n_rows)
        sh = shared.contiguous() if shared is not None else None
        ops.ep_finish(*self._args(), self.k, self.slot, sh, out)
        launch_count.add(2)
        return out


class EPAllToAll:
    def __init__(self, ps, num_experts: int, top_k: int):
        assert ps.ep_size > 1 and num_experts % ps.ep_size == 0, (ps.ep_size, num_experts)
        self.ps = ps
        self.W = ps.ep_size
        self.rank = ps.ep_rank
        self.group = ps.ep_group
        self.cpu_group = ps.cpu_group
        self.E_local = num_experts // ps.ep_size
        self.k = top_k
        self.sent_rows = 0       # rows dispatched by this rank (statistics)
        self.recv_rows = 0       # rows served by this rank's experts
        self.peer: EPPeer | None = None
        self.t_sum = 0           # tokens of all ranks in the current forward
        self.t_max = 0

    def reserve(self, max_tokens: int, hidden: int) -> None:
        """Allocate the peer-memory transport for up to ``max_tokens`` tokens per
        rank and forward (collective: every rank calls it with the same size)."""
        from .. import envs

        if (self.peer is None and torch.cuda.is_available() and self.ps.device.type == "cuda"
                and envs.get("VLLM_B200_FUSED_EP_A2A")):
            self.peer = EPPeer(self.ps, self.E_local, self.k, hidden, max_tokens)

    # -------------------------------------------------------------- lock-step
    def step(self, active: bool, tokens: int = 0) -> int:
        """Vote before a forward; returns how many ranks are active in it, and
        records the sum / maximum of the ranks' token counts."""
        t = torch.tensor([1 if active else 0, int(tokens)], dtype=torch.int64)
        got = [torch.zeros_like(t) for _ in range(self.W)]
        dist.all_gather(got, t, group=self.cpu_group)
        self.t_sum = sum(int(g[1]) for g in got)
        self.t_max = max(int(g[1]) for g in got)
        return sum(int(g[0]) for g in got)

    def _use_peer(self, x) -> bool:
        return self.peer is not None and x.is_cuda and self.t_max <= self.peer.T_cap

    # -------------------------------------------------------------- transport
    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits) -> None:
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                               input_split_sizes=in_splits, group=self.group)

    def dispatch(self, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor):
        """``x [T, H]``, routing ``w [T, k]`` fp32 / ``ids [T, k]`` int32 ->
        (received rows ``[N, H]``, their weights ``[N, k]``, ids ``[N, k]``,
        plan). On the peer path N is an upper bound (the vote's token sum);
        rows past the received ones carry expert id -1 (no expert)."""
        if self._use_peer(x):
            n_max = max(1, min(self.t_sum, self.W * self.peer.T_cap))
            return self.peer.dispatch(x, w, ids, n_max)
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
        if isinstance(plan, PeerPlan):
            return self.peer.combine(yr, plan, shared, out)
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
