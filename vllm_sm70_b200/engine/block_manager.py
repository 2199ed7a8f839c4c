"""KV block manager: the native allocator (``torch.classes._b200_C.
BlockAllocator``) with a pure-Python twin for machines without the library.
Block ids below ``reserved`` are never handed out; block 0 is the scratch
block that padded CUDA-graph rows write into."""
from __future__ import annotations

import torch

from .. import _ext


class _PyAllocator:
    def __init__(self, num_blocks: int, reserved: int):
        assert num_blocks > reserved >= 0
        self._free = list(range(num_blocks - 1, reserved - 1, -1))
        self._ref = [0] * num_blocks
        self._reserved = reserved

    def num_free(self):
        return len(self._free)

    def num_total(self):
        return len(self._ref)

    def allocate(self, n):
        if len(self._free) < n:
            raise RuntimeError(f"BlockAllocator: out of KV blocks (need {n}, free {len(self._free)})")
        out = []
        for _ in range(n):
            b = self._free.pop()
            self._ref[b] = 1
            out.append(b)
        return torch.tensor(out, dtype=torch.int32)

    def incref(self, blocks):
        for b in blocks.tolist():
            assert self._ref[b] > 0
            self._ref[b] += 1

    def free(self, blocks):
        for b in blocks.tolist():
            assert b >= self._reserved and self._ref[b] > 0, f"double free of block {b}"
            self._ref[b] -= 1
            if self._ref[b] == 0:
                self._free.append(b)

    def block_refcount(self, b):
        return self._ref[b]


def make_allocator(num_blocks: int, reserved: int = 1):
    if _ext.load():
        return torch.classes._b200_C.BlockAllocator(num_blocks, reserved)
    return _PyAllocator(num_blocks, reserved)


def build_prefill_meta(block_table: torch.Tensor, ctx_start: torch.Tensor, q_len: torch.Tensor,
                       block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    if _ext.load():
        return torch.ops._b200_C.build_prefill_meta(block_table, ctx_start, q_len, block_size)
    pos, slots = [], []
    for s in range(q_len.numel()):
        c0, n = int(ctx_start[s]), int(q_len[s])
        p = torch.arange(c0, c0 + n, dtype=torch.int64)
        blk = block_table[s].long()[p // block_size]
        pos.append(p)
        slots.append(blk * block_size + p % block_size)
    return torch.cat(pos), torch.cat(slots)
