"""Building blocks shared by the model families: linear layers (BF16 and the
quantised weight formats behind one ``forward`` interface), the paged KV
cache and the per-step attention metadata."""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .. import ops


class Linear:
    """``y = x @ W^T`` for a TP-local weight shard. Subclasses hold quantised
    weights; all share ``forward(x, out=None)``."""

    out_features: int
    in_features: int

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        raise NotImplementedError

    def weight_bytes(self) -> int:
        raise NotImplementedError


class DenseLinear(Linear):
    def __init__(self, w: torch.Tensor):
        self.w = w.contiguous()
        self.out_features, self.in_features = self.w.shape

    def forward(self, x, out=None):
        return ops.gemm(x, self.w, out=out)

    def weight_bytes(self):
        return self.w.numel() * self.w.element_size()


class GateUpLinear(Linear):
    """Gate/up projection with the SiLU*up activation fused in the GEMM
    epilogue; ``w`` is stored 64-row interleaved (``interleave_gate_up``)."""

    def __init__(self, w_gate: torch.Tensor, w_up: torch.Tensor):
        self.w = ops.interleave_gate_up(w_gate, w_up)
        self.out_features = w_gate.shape[0]  # after the activation
        self.in_features = w_gate.shape[1]

    def forward(self, x, out=None):
        return ops.gemm_silu_mul(x, self.w, out=out)

    def weight_bytes(self):
        return self.w.numel() * self.w.element_size()


@dataclass
class AttnMeta:
    """Per-step attention metadata (device tensors)."""
    positions: torch.Tensor      # [T] int64
    slot_mapping: torch.Tensor   # [T] int64
    block_table: torch.Tensor    # [S, max_blocks] int32
    seq_lens: torch.Tensor       # [S] int32 (context incl. this step's tokens)
    cu_q: torch.Tensor           # [S + 1] int32
    max_q_len: int
    decode: bool
    num_splits: int = 1
    part_o: torch.Tensor | None = None
    part_ml: torch.Tensor | None = None
    last_token_idx: torch.Tensor | None = None  # [S] int64 rows whose logits are needed
    state_slots: torch.Tensor | None = None     # [S] int32 recurrent-state slot per sequence
    spec_verify: bool = False                   # recurrent states are read, not advanced


@dataclass
class KVCache:
    """Per-layer paged caches ``[num_blocks, Hkv_local, block_size, D]``."""
    k: list = field(default_factory=list)
    v: list = field(default_factory=list)
    block_size: int = 16
    num_blocks: int = 0

    @classmethod
    def allocate(cls, num_layers: int, num_blocks: int, hkv: int, block_size: int, d: int,
                 dtype=torch.bfloat16, device="cuda", layers: list[int] | None = None):
        c = cls(block_size=block_size, num_blocks=num_blocks)
        idx = layers if layers is not None else list(range(num_layers))
        c.k = [None] * num_layers
        c.v = [None] * num_layers
        for i in idx:
            c.k[i] = torch.zeros(num_blocks, hkv, block_size, d, dtype=dtype, device=device)
            c.v[i] = torch.zeros(num_blocks, hkv, block_size, d, dtype=dtype, device=device)
        return c

    @staticmethod
    def bytes_per_block(num_attn_layers: int, hkv: int, block_size: int, d: int,
                        dtype=torch.bfloat16) -> int:
        return 2 * num_attn_layers * hkv * block_size * d * torch.tensor([], dtype=dtype).element_size()
