"""L0 (HBM) page pool with a content-addressed prefix cache.

Pages are 16-token blocks of the page-first KV arena. A full block is
identified by the chain hash ``sha256(parent || u32-LE tokens)`` (the same
chain the reference computes in python/lake/engine/agents/grpc_skeleton.py:28-42
and go/router/prefixhash.go:16-39, so router, pool and engine agree on block
identity). Cached blocks whose reference count drops to zero stay resident in
an LRU list and are evicted only when a fresh page is needed.
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict
from typing import Iterable, Sequence


def chain_block_hashes(token_ids: Sequence[int], block_size: int, parent: bytes = b"",
                       full_only: bool = False) -> list[bytes]:
    """Chain hash per block of ``block_size`` tokens (the trailing partial block included unless full_only)."""
    out: list[bytes] = []
    n = len(token_ids)
    end = n - (n % block_size) if full_only else n
    for i in range(0, end, block_size):
        chunk = token_ids[i:i + block_size]
        h = hashlib.sha256()
        h.update(parent)
        h.update(b"".join(int(t).to_bytes(4, "little", signed=False) for t in chunk))
        parent = h.digest()
        out.append(parent)
    return out


class NoFreeBlocks(RuntimeError):
    pass


class BlockPool:
    def __init__(self, num_blocks: int, block_size: int = 16, enable_prefix_cache: bool = True):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.enable_prefix_cache = enable_prefix_cache
        self.free: list[int] = list(range(num_blocks - 1, -1, -1))
        self.ref = [0] * num_blocks
        self.hash_of: dict[int, bytes] = {}
        self.block_of: dict[bytes, int] = {}
        self.evictable: OrderedDict[int, None] = OrderedDict()
        self.stats = {"hits": 0, "queries": 0, "evictions": 0}
        self.on_evict = None  # callback(block, hash) before a cached page is handed out again

    # -------------------------------------------------------------- queries
    @property
    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def can_alloc(self, n: int) -> bool:
        return self.num_free >= n

    # -------------------------------------------------------------- alloc
    def alloc(self, n: int) -> list[int]:
        if n > self.num_free:
            raise NoFreeBlocks(f"need {n} blocks, {self.num_free} free")
        out = []
        for _ in range(n):
            if self.free:
                b = self.free.pop()
            else:
                b, _ = self.evictable.popitem(last=False)
                h = self.hash_of.pop(b, None)
                if h is not None and self.block_of.get(h) == b:
                    del self.block_of[h]
                if h is not None and self.on_evict is not None:
                    self.on_evict(b, h)
                self.stats["evictions"] += 1
            self.ref[b] = 1
            out.append(b)
        return out

    def release(self, blocks: Iterable[int]) -> None:
        for b in blocks:
            self.ref[b] -= 1
            assert self.ref[b] >= 0, f"block {b} released too often"
            if self.ref[b] == 0:
                if b in self.hash_of and self.enable_prefix_cache:
                    self.evictable[b] = None
                    self.evictable.move_to_end(b)
                else:
                    self.hash_of.pop(b, None)
                    self.free.append(b)

    # -------------------------------------------------------------- prefix cache
    def lookup(self, hashes: Sequence[bytes]) -> list[int]:
        """Longest cached prefix of `hashes`; each returned block gets a reference."""
        self.stats["queries"] += 1
        if not self.enable_prefix_cache:
            return []
        out = []
        for h in hashes:
            b = self.block_of.get(h)
            if b is None:
                break
            if self.ref[b] == 0:
                self.evictable.pop(b, None)
            self.ref[b] += 1
            out.append(b)
        if out:
            self.stats["hits"] += len(out)
        return out

    def peek(self, hashes: Sequence[bytes]) -> int:
        """Number of leading hashes resident (no references taken)."""
        n = 0
        for h in hashes:
            if h not in self.block_of:
                break
            n += 1
        return n

    def register(self, block: int, h: bytes) -> None:
        if not self.enable_prefix_cache:
            return
        if h in self.block_of and self.block_of[h] != block:
            return  # another copy already canonical
        self.hash_of[block] = h
        self.block_of[h] = block

    def residency(self) -> dict:
        return {"free": len(self.free), "cached_idle": len(self.evictable), "total": self.num_blocks,
                "used": self.num_blocks - len(self.free) - len(self.evictable)}
