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

A third, persistent tier (``DiskKVTier``) writes every indexed block
through to files named by its key, so a later engine process with the same
model, layout and rank -- after a restart, or another replica on the same
host -- starts with those prefixes cached.

Hybrid models with recurrent state (gated DeltaNet) cannot skip prefill on a
KV hit -- the state is not cached -- so the engine does not enable this for
them.

Reference parity: vLLM's automatic prefix caching, which the reference's
deployment keeps on (``sm70/nix/module.nix:241``).
"""
from __future__ import annotations

import io
import os
from collections import OrderedDict
from pathlib import Path

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


class DiskKVTier:
    """Persistent tier: one file per block under ``root/namespace``, named by
    the block's chained key (keys are deterministic across processes: they
    hash token ids only). ``namespace`` must identify everything that makes
    KV bytes differ -- model, weights, dtype, block size, TP rank -- so
    tiers of different engines never mix. Files are written atomically
    (temporary name + rename); the least recently used ones beyond
    ``capacity_blocks`` are deleted. Reads check the tensor shapes."""

    def __init__(self, kv, root: str | Path, namespace: str, capacity_blocks: int):
        self.kv = kv
        self.layers = [i for i, t in enumerate(kv.k) if t is not None]
        self.dir = Path(root) / namespace
        self.dir.mkdir(parents=True, exist_ok=True)
        self.capacity = int(capacity_blocks)
        self.saved = 0
        self.restored = 0
        self._size: int | None = None  # bytes of one block file (a shorter file is damaged)

    def _path(self, key: int) -> Path:
        return self.dir / f"{key:016x}.kv"

    def has(self, key: int) -> bool:
        return self._path(key).exists()

    def save(self, key: int, block: int) -> None:
        p = self._path(key)
        if self._size is not None and p.exists() and p.stat().st_size == self._size:
            os.utime(p)  # already there (and whole): refresh its LRU time
            return
        k = torch.stack([self.kv.k[i][block] for i in self.layers]).cpu()
        v = torch.stack([self.kv.v[i][block] for i in self.layers]).cpu()
        buf = io.BytesIO()
        torch.save({"k": k, "v": v}, buf)
        blob = buf.getvalue()
        self._size = len(blob)  # every block of a namespace serialises to this size
        if p.exists() and p.stat().st_size == self._size:
            os.utime(p)
            return
        tmp = p.with_name(f"{p.name}.{os.getpid()}.tmp")
        tmp.write_bytes(blob)
        os.replace(tmp, p)
        self.saved += 1
        self._trim()

    def restore(self, key: int, block: int) -> bool:
        p = self._path(key)
        try:
            d = torch.load(p, map_location="cpu", weights_only=True)
        except FileNotFoundError:
            return False
        except Exception:  # noqa: BLE001 - damaged file: drop it, the block is prefilled
            p.unlink(missing_ok=True)
            return False
        ref = self.kv.k[self.layers[0]][block]
        if (not isinstance(d, dict) or "k" not in d or "v" not in d
                or d["k"].shape != (len(self.layers),) + tuple(ref.shape)
                or d["k"].dtype != ref.dtype or d["v"].shape != d["k"].shape):
            p.unlink(missing_ok=True)
            return False
        for j, i in enumerate(self.layers):
            self.kv.k[i][block].copy_(d["k"][j])
            self.kv.v[i][block].copy_(d["v"][j])
        os.utime(p)
        self.restored += 1
        return True

    def _trim(self) -> None:
        files = list(self.dir.glob("*.kv"))
        if len(files) <= self.capacity:
            return
        files.sort(key=lambda f: f.stat().st_mtime)
        for f in files[: len(files) - self.capacity]:
            try:
                f.unlink()
            except FileNotFoundError:
                pass


class PrefixCache:
    def __init__(self, alloc, block_size: int, host: HostKVTier | None = None,
                 disk: DiskKVTier | None = None):
        self.alloc = alloc
        self.bs = block_size
        self.host = host
        self.disk = disk
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
            # host or disk tier: back into a fresh device block (the cache keeps a
            # reference), making room by pushing other cache-only blocks out first
            in_host = self.host is not None and k in self.host.slots
            if not in_host and (self.disk is None or not self.disk.has(k)):
                break
            if self.alloc.num_free() < 1:
                self.evict(1)
            if self.alloc.num_free() < 1:
                break
            b = int(self.alloc.allocate(1)[0])
            if not (self.host.restore(k, b) if in_host else self.disk.restore(k, b)):
                self.alloc.free(torch.tensor([b], dtype=torch.int32))
                break
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
            if self.disk is not None:  # write through: persists past this process
                self.disk.save(k, b)
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
