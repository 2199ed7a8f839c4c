"""Prefix caching of KV blocks: full prompt blocks are content-addressed so
a later request that starts with the same tokens reuses their KV instead of
prefilling them again.

A block's key is a hash of its tokens chained with its parent block's key
(so equal tokens at different positions or after different prefixes never
collide into the same entry). The cache holds one reference on every block it
indexes (through the engine's refcounting allocator); a request that reuses a
block takes its own reference. When an allocation runs short, entries that
only the cache still references are evicted least-recently-used first -- into
an optional host-memory tier (``HostKVTier``) from which a later hit copies
them back.

Hybrid models with recurrent state (gated DeltaNet) cannot skip prefill on a
KV hit -- the state is not cached -- so the engine does not enable this for
them.

Reference parity: vLLM's automatic prefix caching, which the reference's
deployment keeps on (``sm70/nix/module.nix:241``).
"""
from __future__ import annotations

from collections import OrderedDict

import torch

_MASK = (1 << 61) - 1


def block_keys(tokens: torch.Tensor, block_size: int, n_blocks: int) -> list[int]:
    """Chained keys of the first ``n_blocks`` full blocks of ``tokens``."""
    keys, parent = [], 0x51F15E
    t = tokens[: n_blocks * block_size].tolist()
    for b in range(n_blocks):
        h = hash((parent, tuple(t[b * block_size:(b + 1) * block_size]))) & _MASK
        keys.append(h)
        parent = h
    return keys


class HostKVTier:
    """Second tier of the prefix cache in (pinned) host memory: blocks evicted
    from the device are copied here under their key and copied back into a
    fresh device block on a later hit, so the reusable prefix set is not
    bounded by the KV pool. Each rank keeps its own KV shard; the decisions
    depend only on keys and the allocator state, so they are rank-uniform."""

    def __init__(self, kv, capacity_blocks: int, pin: bool = True):
        self.kv = kv
        self.layers = [i for i, t in enumerate(kv.k) if t is not None]
        ref = kv.k[self.layers[0]]
        shape = (capacity_blocks,) + tuple(ref.shape[1:])
        pin = pin and ref.is_cuda
        self.hk = {i: torch.empty(shape, dtype=ref.dtype, pin_memory=pin) for i in self.layers}
        self.hv = {i: torch.empty(shape, dtype=ref.dtype, pin_memory=pin) for i in self.layers}
        self.slots: OrderedDict[int, int] = OrderedDict()  # key -> host slot (LRU order)
        self.free = list(range(capacity_blocks - 1, -1, -1))
        self.saved = 0
        self.restored = 0

    def save(self, key: int, block: int) -> None:
        if key in self.slots:
            self.slots.move_to_end(key)
            return
        if not self.free:  # drop the least recently used host copy
            _, s = self.slots.popitem(last=False)
            self.free.append(s)
        s = self.free.pop()
        for i in self.layers:  # stream-ordered after the kernels that wrote the block
            self.hk[i][s].copy_(self.kv.k[i][block])
            self.hv[i][s].copy_(self.kv.v[i][block])
        self.slots[key] = s
        self.saved += 1

    def restore(self, key: int, block: int) -> bool:
        s = self.slots.get(key)
        if s is None:
            return False
        self.slots.move_to_end(key)
        for i in self.layers:  # stream-ordered before the prefill that reads it
            self.kv.k[i][block].copy_(self.hk[i][s], non_blocking=True)
            self.kv.v[i][block].copy_(self.hv[i][s], non_blocking=True)
        self.restored += 1
        return True


class PrefixCache:
    def __init__(self, alloc, block_size: int, host: HostKVTier | None = None):
        self.alloc = alloc
        self.bs = block_size
        self.host = host
        self.entries: OrderedDict[int, int] = OrderedDict()  # key -> block id (LRU order)
        self.hits = 0      # blocks served from the cache (either tier)
        self.queries = 0   # full blocks looked up

    def lookup(self, prompt: torch.Tensor) -> tuple[list[int], list[int]]:
        """Longest cached prefix of ``prompt``'s full blocks, leaving at least
        one prompt token to prefill (its logits start the generation).
        Returns (keys, block ids); the caller owns a new reference on each."""
        n_full = (prompt.numel() - 1) // self.bs
        if n_full <= 0:
            return [], []
        keys = block_keys(prompt, self.bs, n_full)
        self.queries += n_full
        blocks = []
        for k in keys:
            b = self.entries.get(k)
            if b is not None:
                self.entries.move_to_end(k)
                self.alloc.incref(torch.tensor([b], dtype=torch.int32))
                blocks.append(b)
                continue
            # host tier: back into a fresh device block (the cache keeps a reference),
            # making room by pushing other cache-only blocks to the host first
            if self.host is None or k not in self.host.slots:
                break
            if self.alloc.num_free() < 1:
                self.evict(1)
            if self.alloc.num_free() < 1:
                break
            b = int(self.alloc.allocate(1)[0])
            self.host.restore(k, b)
            self.entries[k] = b
            self.alloc.incref(torch.tensor([b], dtype=torch.int32))
            blocks.append(b)
        self.hits += len(blocks)
        return keys[: len(blocks)], blocks

    def insert(self, prompt: torch.Tensor, blocks: torch.Tensor) -> None:
        """Index the full prompt blocks of a request whose prefill finished
        (``blocks`` is its block list in order)."""
        n_full = prompt.numel() // self.bs
        if n_full <= 0:
            return
        keys = block_keys(prompt, self.bs, n_full)
        new = []
        for k, b in zip(keys, blocks[:n_full].tolist()):
            if k in self.entries:
                self.entries.move_to_end(k)
                continue
            self.entries[k] = b
            new.append(b)
        if new:
            self.alloc.incref(torch.tensor(new, dtype=torch.int32))

    def evict(self, need: int) -> int:
        """Free least-recently-used entries held only by the cache until
        ``need`` blocks are free (or nothing is evictable). Returns the number
        of blocks freed."""
        freed = 0
        for k in list(self.entries.keys()):
            if self.alloc.num_free() >= need:
                break
            b = self.entries[k]
            if self.alloc.block_refcount(b) == 1:
                del self.entries[k]
                if self.host is not None:
                    self.host.save(k, b)
                self.alloc.free(torch.tensor([b], dtype=torch.int32))
                freed += 1
        return freed

    def clear(self) -> None:
        if self.entries:
            self.alloc.free(torch.tensor(list(self.entries.values()), dtype=torch.int32))
        self.entries.clear()
