"""Restatement of SGLang's RadixCache + TokenToKVPoolAllocator (TEST ORACLE, see oracle/__init__.py).

Follows the behaviour QwenEdit's PagedKVPool relies on (multi_turn/cache/paged.py:52-131):
* ``TokenToKVPoolAllocator(size, need_sort=True)`` (paged.py:52-54): free slots 1..size in a sorted list;
  ``alloc(n)`` takes the head, merging and sorting the release list first when the head is short;
  ``free`` appends to the release list.
* ``RadixCache.create_simulated(page_size=1)`` (paged.py:55): children keyed by first token; match /
  insert split nodes; every node on a walk gets the walk's access time; ``evict`` heapifies leaves on
  last-access time and pops unlocked ones, pushing a parent that loses its last child; lock refs walk to
  the root moving tokens between evictable and protected.
* time.monotonic() is a logical clock: one tick per walk and per node construction. ``Clock(resolution=k)``
  gives every k consecutive reads the same value instead: a wall clock too coarse to separate some reads, under
  which leaves can tie on last-access time and the heap's layout decides between them (``evict`` then records
  ``tie_seen``).

Written in plain Python with dicts, lists and heapq so it reads like the original design; the product
(libqeb200's C++ prefix index) is checked against it operation for operation.
"""

from __future__ import annotations

import heapq
import itertools

import numpy as np


class Clock:
    def __init__(self, resolution: int = 1):
        self._t = itertools.count(0)
        self.resolution = resolution

    def __call__(self) -> int:
        return 1 + next(self._t) // self.resolution


class TreeNode:
    def __init__(self, clock: Clock):
        self.children: dict = {}
        self.parent: TreeNode | None = None
        self.key: list[int] = []
        self.value: np.ndarray = np.empty(0, np.int64)
        self.lock_ref = 0
        self.last_access_time = clock()

    def __lt__(self, other: "TreeNode") -> bool:
        return self.last_access_time < other.last_access_time


class Allocator:
    """TokenToKVPoolAllocator (need_sort=True); page_size > 1 hands out whole pages (paged allocator)."""

    def __init__(self, size_tokens: int, page_size: int = 1):
        self.page_size = page_size
        self.num_pages = size_tokens // page_size
        self.clear()

    def clear(self) -> None:
        self.free_pages = list(range(1, self.num_pages + 1))
        self.release_pages: list[int] = []

    def available_size(self) -> int:
        return (len(self.free_pages) + len(self.release_pages)) * self.page_size

    def merge_and_sort_free(self) -> None:
        if self.release_pages:
            self.free_pages = sorted(self.free_pages + self.release_pages)
            self.release_pages = []

    def alloc(self, need_size: int) -> np.ndarray | None:
        P = self.page_size
        units = -(-need_size // P)
        if units > len(self.free_pages):
            self.merge_and_sort_free()
        if units > len(self.free_pages):
            return None
        pages, self.free_pages = self.free_pages[:units], self.free_pages[units:]
        if P == 1:
            return np.asarray(pages, np.int64)
        t = np.arange(need_size, dtype=np.int64)
        return np.asarray(pages, np.int64)[t // P] * P + t % P

    def free(self, free_index) -> None:
        free_index = np.asarray(free_index, np.int64)
        if free_index.size == 0:
            return
        if self.page_size == 1:
            self.release_pages.extend(int(x) for x in free_index)
        else:
            self.release_pages.extend(int(x) for x in np.unique(free_index // self.page_size))


class RadixCache:
    def __init__(self, allocator: Allocator, page_size: int = 1, clock: Clock | None = None):
        self.allocator = allocator
        self.page_size = page_size
        self.clock = clock if clock is not None else Clock()
        self.tie_seen = False  # an eviction chose between leaves of equal last-access time
        self.reset()

    # -- keys
    def _child_key(self, key) -> tuple:
        return tuple(key[: self.page_size])

    def _key_match(self, a, b) -> int:
        P = self.page_size
        n = min(len(a), len(b))
        i = 0
        if P == 1:
            while i < n and a[i] == b[i]:
                i += 1
            return i
        while i + P <= n and a[i:i + P] == b[i:i + P]:
            i += P
        return i

    def reset(self) -> None:
        self.root_node = TreeNode(self.clock)
        self.root_node.lock_ref = 1
        self.evictable_size_ = 0
        self.protected_size_ = 0

    def _aligned(self, key: list) -> list:
        return key if self.page_size == 1 else key[: len(key) // self.page_size * self.page_size]

    # -- match
    def match_prefix(self, key: list) -> tuple[np.ndarray, TreeNode]:
        key = self._aligned(key)
        if len(key) == 0:
            return np.empty(0, np.int64), self.root_node
        access = self.clock()
        node = self.root_node
        node.last_access_time = access
        value = []
        while len(key) > 0 and self._child_key(key) in node.children:
            child = node.children[self._child_key(key)]
            child.last_access_time = access
            plen = self._key_match(child.key, key)
            if plen < len(child.key):
                new_node = self._split_node(child, plen)
                value.append(new_node.value)
                node = new_node
                break
            value.append(child.value)
            node = child
            key = key[plen:]
        return (np.concatenate(value) if value else np.empty(0, np.int64)), node

    def _split_node(self, child: TreeNode, split_len: int) -> TreeNode:
        new_node = TreeNode(self.clock)
        new_node.children = {self._child_key(child.key[split_len:]): child}
        new_node.parent = child.parent
        new_node.lock_ref = child.lock_ref
        new_node.key = child.key[:split_len]
        new_node.value = child.value[:split_len]
        child.parent = new_node
        child.key = child.key[split_len:]
        child.value = child.value[split_len:]
        new_node.parent.children[self._child_key(new_node.key)] = new_node
        return new_node

    # -- insert
    def insert(self, key: list, value: np.ndarray) -> int:
        key = self._aligned(key)
        value = value[: len(key)]
        access = self.clock()
        node = self.root_node
        node.last_access_time = access
        if len(key) == 0:
            return 0
        total = 0
        while len(key) > 0 and self._child_key(key) in node.children:
            node = node.children[self._child_key(key)]
            node.last_access_time = access
            plen = self._key_match(node.key, key)
            total += plen
            key = key[plen:]
            value = value[plen:]
            if plen < len(node.key):
                node = self._split_node(node, plen)
        if len(key):
            new_node = TreeNode(self.clock)
            new_node.parent = node
            new_node.key = list(key)
            new_node.value = np.asarray(value, np.int64).copy()
            node.children[self._child_key(key)] = new_node
            self.evictable_size_ += len(key)
        return total

    # -- locks
    def inc_lock_ref(self, node: TreeNode) -> None:
        while node is not self.root_node:
            if node.lock_ref == 0:
                self.evictable_size_ -= len(node.key)
                self.protected_size_ += len(node.key)
            node.lock_ref += 1
            node = node.parent

    def dec_lock_ref(self, node: TreeNode) -> None:
        while node is not self.root_node:
            if node.lock_ref == 1:
                self.evictable_size_ += len(node.key)
                self.protected_size_ -= len(node.key)
            node.lock_ref -= 1
            node = node.parent

    # -- eviction
    def _collect_leaves(self) -> list[TreeNode]:
        out, stack = [], [self.root_node]
        while stack:
            cur = stack.pop()
            if len(cur.children) == 0:
                out.append(cur)
            else:
                stack.extend(cur.children.values())
        return out

    def evict(self, num_tokens: int) -> int:
        heap = [(n.last_access_time, n) for n in self._collect_leaves()]
        heapq.heapify(heap)
        evicted = 0
        while evicted < num_tokens and heap:
            t, x = heapq.heappop(heap)
            if heap and heap[0][0] == t:
                self.tie_seen = True
            if x is self.root_node:
                break
            if x.lock_ref > 0:
                continue
            self.allocator.free(x.value)
            evicted += len(x.value)
            for k, v in list(x.parent.children.items()):
                if v is x:
                    del x.parent.children[k]
                    break
            self.evictable_size_ -= len(x.key)
            if len(x.parent.children) == 0:
                heapq.heappush(heap, (x.parent.last_access_time, x.parent))
        return evicted

    def evictable_size(self) -> int:
        return self.evictable_size_

    def protected_size(self) -> int:
        return self.protected_size_

    def node_count(self) -> int:
        n, stack = 0, [self.root_node]
        while stack:
            cur = stack.pop()
            n += len(cur.children)
            stack.extend(cur.children.values())
        return n
