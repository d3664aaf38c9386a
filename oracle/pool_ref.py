"""The reference PagedKVPool on CPU tensors (TEST ORACLE, see oracle/__init__.py).

Restates multi_turn/cache/paged.py:40-131 over ``radix_ref``: data movement is the reference's own torch
calls — ``kv.index_select(2, idx)`` for gather (paged.py:113), a view for one contiguous run (:108-111),
``kv.index_copy_(2, idx, new)`` for write (:116) — so it is the bit-exact oracle for the sm_100a kernels,
and the timed CPU baseline. ``page_size > 1`` follows the product's paged mode (whole-page allocation,
page-aligned keys).
"""

from __future__ import annotations

import threading
from array import array
from dataclasses import dataclass

import numpy as np
import torch

from oracle.radix_ref import Allocator, Clock, RadixCache


@dataclass
class PoolStats:
    lookups: int = 0
    hit_tokens: int = 0
    miss_tokens: int = 0
    inserted_tokens: int = 0
    evicted_tokens: int = 0
    contiguous_views: int = 0
    gathers: int = 0


class Match:
    def __init__(self, pool, length, indices, node):
        self.pool, self.length, self.indices, self.node = pool, length, indices, node

    def release(self) -> None:
        if self.node is not None:
            self.pool.tree.dec_lock_ref(self.node)
            self.node = None


def _key(vids) -> list:
    if isinstance(vids, array):
        return list(vids)
    return np.ascontiguousarray(vids, dtype=np.int64).reshape(-1).tolist()


class RefPagedKVPool:
    def __init__(self, name, layers, heads, head_dim, budget_bytes, dtype, device="cpu", extra_dim=0, page_size=1,
                 allocate=True, clock_resolution=1):
        elem = torch.empty((), dtype=dtype).element_size()
        per_token = layers * 2 * heads * head_dim * elem + extra_dim * elem
        self.name = name
        self.page_size = page_size
        capacity = max(int(budget_bytes // per_token), 1)
        self.capacity = max(capacity // page_size, 1) * page_size
        self.layers, self.heads, self.head_dim = layers, heads, head_dim
        rows = self.capacity + page_size
        self.kv = torch.empty(layers, 2, rows, heads, head_dim, dtype=dtype, device=device) if allocate else None
        self.extra = torch.empty(rows, extra_dim, dtype=dtype, device=device) if (extra_dim and allocate) else None
        self.allocator = Allocator(self.capacity, page_size)
        self.tree = RadixCache(self.allocator, page_size, Clock(clock_resolution))
        self.stats = PoolStats()
        self.lock = threading.RLock()

    def match(self, vids) -> Match:
        key = _key(vids)
        with self.lock:
            self.stats.lookups += 1
            value, node = self.tree.match_prefix(key)
            length = len(value)
            if length:
                self.tree.inc_lock_ref(node)
                indices = torch.from_numpy(value.copy())
            else:
                node, indices = None, None
            self.stats.hit_tokens += length
            self.stats.miss_tokens += len(key) - length
            return Match(self, length, indices, node)

    def alloc(self, n: int):
        with self.lock:
            if n > self.capacity:
                return None
            need_tokens = -(-n // self.page_size) * self.page_size
            if self.allocator.available_size() < need_tokens:
                self.stats.evicted_tokens += self.tree.evict(need_tokens - self.allocator.available_size())
            out = self.allocator.alloc(n)
            return None if out is None else torch.from_numpy(out)

    def insert(self, vids, indices: torch.Tensor, owned_from: int) -> None:
        key = _key(vids)
        slots = indices.to(torch.int64).numpy()
        with self.lock:
            present = self.tree.insert(key, slots)
            aligned = len(key) // self.page_size * self.page_size
            if present > owned_from:
                self.allocator.free(slots[owned_from:present])
            tail = max(aligned, owned_from)
            if tail < len(key):
                self.allocator.free(slots[tail:])
            self.stats.inserted_tokens += max(aligned - max(present, owned_from), 0)

    def gather(self, indices: torch.Tensor) -> torch.Tensor:
        n = indices.numel()
        first = int(indices[0]) if n else 0
        if n and int(indices[-1]) - first == n - 1 and (n == 1 or bool((indices[1:] - indices[:-1] == 1).all())):
            self.stats.contiguous_views += 1
            return self.kv[:, :, first:first + n]
        self.stats.gathers += 1
        return self.kv.index_select(2, indices)

    def write(self, indices: torch.Tensor, kv: torch.Tensor) -> None:
        self.kv.index_copy_(2, indices, kv.to(self.kv.dtype))

    def usage(self) -> dict:
        with self.lock:
            return dict(capacity=self.capacity, free=self.allocator.available_size(),
                        evictable=self.tree.evictable_size(), protected=self.tree.protected_size(),
                        **self.stats.__dict__)

    def clear(self) -> None:
        with self.lock:
            self.tree.reset()
            self.allocator.clear()
