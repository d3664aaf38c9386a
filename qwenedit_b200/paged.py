"""Paged prefix K/V pool: drop-in for QwenEdit's ``multi_turn.cache.paged`` (paged.py:18-131).

Same constructor, methods, attributes, statistics and error behaviour as the reference ``PagedKVPool``:

* ``match(vids) -> Match`` (paged.py:72-85), ``alloc(n) -> Tensor | None`` (:87-95, never raises on
  exhaustion), ``insert(vids, indices, owned_from)`` (:97-103), ``gather(indices)`` (:106-113, a view of
  the pool when the slots are one contiguous run), ``write(indices, kv)`` (:115-116), ``usage()`` (:118-126),
  ``clear()`` (:128-131); ``Match.release()`` is idempotent (:34-37).
* ``.kv`` is ``[L, 2, rows, H, D]`` with row 0 (page 0) as padding, ``.extra`` ``[rows, extra_dim]``.

What is different underneath:

* the radix tree, LRU eviction and slot allocator are the native prefix index of libqeb200 (host C++,
  one call per operation) instead of SGLang's Python ``RadixCache`` / ``TokenToKVPoolAllocator``;
* gather and write are single sm_100a kernel launches over all layers and K/V (``index_select`` /
  ``index_copy_`` are not used), on the caller's current CUDA stream;
* slot tensors handed out by ``match`` / ``alloc`` carry a host mirror, so the contiguity test of
  ``gather`` needs no device-to-host sync (the reference reads three scalars back, paged.py:108-109);
* ``page_size > 1`` (an addition) allocates and matches whole pages; gathers then walk a block table.
  ``page_size=1`` reproduces the reference's token-granular behaviour.

No path runs on the CPU: gather / write require CUDA tensors and raise otherwise.
"""

from __future__ import annotations

import ctypes
import logging
import threading
from array import array
from dataclasses import dataclass

import numpy as np
import torch

from qwenedit_b200 import _lib

logger = logging.getLogger(__name__)


@dataclass
class PoolStats:
    """Counters with the reference's names (paged.py:18-26)."""

    lookups: int = 0
    hit_tokens: int = 0
    miss_tokens: int = 0
    inserted_tokens: int = 0
    evicted_tokens: int = 0
    contiguous_views: int = 0
    gathers: int = 0


def _as_key(vids) -> np.ndarray:
    if isinstance(vids, array):
        if vids.typecode != "q":
            raise TypeError("vids array must have typecode 'q'")
        return np.frombuffer(vids, dtype=np.int64) if len(vids) else np.empty(0, np.int64)
    return np.ascontiguousarray(vids, dtype=np.int64).reshape(-1)


class PrefixIndex:
    """Owning wrapper of a native ``qe_index`` (radix tree + allocator + LRU)."""

    def __init__(self, capacity_tokens: int, page_size: int):
        handle = ctypes.c_void_p()
        _lib.call("qe_index_create", capacity_tokens, page_size, ctypes.byref(handle))
        self._h = handle
        self.page_size = page_size

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().qe_index_destroy(h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def match(self, key: np.ndarray) -> tuple[int, np.ndarray, int]:
        n = len(key)
        out = np.empty(max(n, 1), np.int64)
        length, node = ctypes.c_int64(), ctypes.c_uint64()
        _lib.call("qe_index_match", self._h, _lib.ptr64(key), n, ctypes.byref(length), _lib.ptr64(out),
                  ctypes.byref(node))
        return length.value, out[: length.value], node.value

    def lock(self, node: int) -> None:
        _lib.call("qe_index_lock", self._h, node)

    def unlock(self, node: int) -> None:
        _lib.call("qe_index_unlock", self._h, node)

    def insert(self, key: np.ndarray, slots: np.ndarray) -> int:
        present = ctypes.c_int64()
        _lib.call("qe_index_insert", self._h, _lib.ptr64(key), _lib.ptr64(slots), len(key), ctypes.byref(present))
        return present.value

    def evict(self, num_tokens: int) -> int:
        out = ctypes.c_int64()
        _lib.call("qe_index_evict", self._h, num_tokens, ctypes.byref(out))
        return out.value

    def alloc(self, n: int) -> np.ndarray | None:
        out = np.empty(max(n, 1), np.int64)
        ok = ctypes.c_int32()
        _lib.call("qe_index_alloc", self._h, n, _lib.ptr64(out), ctypes.byref(ok))
        return out[:n] if ok.value else None

    def free(self, slots: np.ndarray) -> None:
        slots = np.ascontiguousarray(slots, dtype=np.int64)
        _lib.call("qe_index_free", self._h, _lib.ptr64(slots), len(slots))

    def usage(self) -> dict:
        out = np.zeros(4, np.int64)
        _lib.call("qe_index_usage", self._h, _lib.ptr64(out))
        return dict(free=int(out[0]), evictable=int(out[1]), protected=int(out[2]), nodes=int(out[3]))

    def clear(self) -> None:
        _lib.call("qe_index_clear", self._h)

    def shuffle_free(self, seed: int) -> None:
        _lib.call("qe_index_shuffle_free", self._h, seed)


class Match:
    """A locked prefix hit (paged.py:29-37): ``length``, device ``indices`` (None when 0), ``release()``."""

    def __init__(self, pool: "PagedKVPool", length: int, indices: torch.Tensor | None, node: int | None):
        self.pool, self.length, self.indices, self.node = pool, length, indices, node

    def release(self) -> None:
        if self.node is not None:
            self.pool._unlock(self.node)
            self.node = None


def _slots_tensor(host: np.ndarray, pool: "PagedKVPool") -> torch.Tensor:
    """Device int64 slot tensor with its host mirror attached (no sync needed to inspect it later)."""
    cpu = torch.from_numpy(host)
    if pool.device.type == "cuda":
        t = cpu.pin_memory().to(pool.device, non_blocking=True)
        pool.h2d_bytes += host.nbytes
    else:
        t = cpu.to(pool.device)
    t._qe_host = host
    return t


COPY_MODES = {"auto": 0, "warp": 1, "bulk": 2, "warp_row": 3, "warp16": 4}


def set_copy_mode(mode: str) -> None:
    """Select the paged copy kernel process-wide: "auto", "warp" (vectorised LDG/STG, short rows several per warp
    pass, 256-bit vectors on 32-byte aligned planes), "bulk" (TMA bulk copies), "warp_row" (the warp kernel, one
    row per warp pass) or "warp16" (the warp kernel and the head-major gather with 16-byte vectors only)."""
    _lib.call("qe_set_paged_copy_mode", COPY_MODES[mode])


def cat_slots(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``torch.cat([a, b])`` of slot tensors, keeping the host mirror when both carry one."""
    out = torch.cat([a, b])
    ha, hb = getattr(a, "_qe_host", None), getattr(b, "_qe_host", None)
    if ha is not None and hb is not None:
        out._qe_host = np.concatenate([ha, hb])
    return out


def pool_geometry(layers, heads, head_dim, budget_bytes, dtype, extra_dim=0, page_size=1) -> tuple[int, int, int]:
    """(capacity tokens, rows, bytes per token) of a pool: capacity = budget // bytes per token rounded down to
    whole pages (paged.py:44-47), plus one padding page of rows."""
    if page_size < 1:
        raise ValueError("page_size must be >= 1")
    elem = torch.empty((), dtype=dtype).element_size()
    per_token = layers * 2 * heads * head_dim * elem + extra_dim * elem
    capacity = max(int(budget_bytes // per_token), 1)
    capacity = max(capacity // page_size, 1) * page_size
    return capacity, capacity + page_size, per_token


class PagedKVPool:
    """Paged K/V prefix pool on one GPU (paged.py:40-131)."""

    def __init__(self, name, layers, heads, head_dim, budget_bytes, dtype, device, extra_dim=0, page_size=1,
                 kv=None):
        """`kv` (an addition): storage for the [L, 2, rows, H, D] pool allocated by the caller (the head-sharded
        pools pass memory that other processes can map); by default the pool allocates it."""
        self.capacity, self.rows, per_token = pool_geometry(layers, heads, head_dim, budget_bytes, dtype, extra_dim,
                                                            page_size)
        self.name = name
        self.page_size = int(page_size)
        self.layers, self.heads, self.head_dim = layers, heads, head_dim
        self.extra_dim = extra_dim
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        shape = (layers, 2, self.rows, heads, head_dim)
        if kv is None:
            kv = torch.empty(shape, dtype=dtype, device=self.device)
        elif tuple(kv.shape) != shape or kv.dtype != dtype or kv.device != self.device or not kv.is_contiguous():
            raise ValueError(f"kv storage must be a contiguous {list(shape)} {dtype} tensor on {self.device}")
        self.kv = kv
        self.extra = (
            torch.empty(self.rows, extra_dim, dtype=dtype, device=self.device) if extra_dim else None
        )
        self.index = PrefixIndex(self.capacity, self.page_size)
        self.stats = PoolStats()
        self.lock = threading.RLock()
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device) if self.device.type == "cuda" else None
        self.h2d_bytes = 0  # host-to-device bytes this pool has copied (slot lists, block tables, pointer tables)
        logger.info(
            "qwenedit_b200: %s pool: %d tokens (page %d), %.1f GiB (%d B/token)",
            name, self.capacity, self.page_size, self.capacity * per_token / (1 << 30), per_token,
        )

    # ---- prefix index ------------------------------------------------------------------------
    def match(self, vids) -> Match:
        key = _as_key(vids)
        with self.lock:
            self.stats.lookups += 1
            length, slots, node = self.index.match(key)
            if length:
                self.index.lock(node)
                indices = _slots_tensor(slots.copy(), self)
            else:
                node, indices = None, None
            self.stats.hit_tokens += length
            self.stats.miss_tokens += len(key) - length
            return Match(self, length, indices, node)

    def _unlock(self, node: int) -> None:
        with self.lock:
            self.index.unlock(node)

    def alloc(self, n: int) -> torch.Tensor | None:
        n = int(n)
        with self.lock:
            if n > self.capacity or n < 0:
                return None
            need_tokens = -(-n // self.page_size) * self.page_size
            free = self.index.usage()["free"]
            if free < need_tokens:
                self.stats.evicted_tokens += self.index.evict(need_tokens - free)
            slots = self.index.alloc(n)
            if slots is None:
                return None
            return _slots_tensor(slots.copy(), self)

    def insert(self, vids, indices: torch.Tensor, owned_from: int) -> None:
        key = _as_key(vids)
        slots = self._host_slots(indices)
        if len(slots) != len(key):
            raise ValueError(f"insert: {len(key)} ids but {len(slots)} slots")
        owned_from = int(owned_from)
        with self.lock:
            present = self.index.insert(key, slots)
            aligned = len(key) // self.page_size * self.page_size
            if present > owned_from:
                self.index.free(slots[owned_from:present])
            tail = max(aligned, owned_from)
            if tail < len(key):  # page mode: the owned partial last page is not cached
                self.index.free(slots[tail:])
            self.stats.inserted_tokens += max(aligned - max(present, owned_from), 0)

    # ---- data movement -----------------------------------------------------------------------
    def _host_slots(self, indices: torch.Tensor) -> np.ndarray:
        host = getattr(indices, "_qe_host", None)
        if host is None:
            host = indices.detach().to("cpu", torch.int64).numpy().reshape(-1)
            indices._qe_host = host
        return host

    def _row_bytes(self, t: torch.Tensor) -> int:
        return self.heads * self.head_dim * t.element_size()

    def _stream(self) -> int:
        return _lib.stream_of(self.device)

    def _block_table(self, indices: torch.Tensor, host: np.ndarray) -> torch.Tensor | None:
        """Device int32 page table when the slots are whole-page runs (page mode), else None."""
        if self.page_size == 1:
            return None
        cached = getattr(indices, "_qe_pages", None)
        if cached is not None:
            return cached
        P = self.page_size
        n = len(host)
        pages = host[::P] // P
        offsets = np.arange(n, dtype=np.int64)
        if n == 0 or not np.array_equal(host, pages[offsets // P] * P + offsets % P):
            return None
        bt = torch.from_numpy(pages.astype(np.int32))
        bt = bt.pin_memory().to(self.device, non_blocking=True)
        self.h2d_bytes += bt.numel() * 4
        indices._qe_pages = bt
        return bt

    def _require_cuda(self, *tensors: torch.Tensor) -> None:
        if self.device.type != "cuda":
            raise RuntimeError("PagedKVPool data movement runs only on CUDA devices (no CPU path)")
        for t in tensors:
            if t.device != self.device:
                raise ValueError(f"tensor on {t.device}, pool on {self.device}")

    def gather(self, indices: torch.Tensor) -> torch.Tensor:
        """K/V of `indices` as [L, 2, n, H, D]: a view when the slots are one run, else one gather launch."""
        host = self._host_slots(indices)
        n = len(host)
        if n and int(host[-1]) - int(host[0]) == n - 1 and (n == 1 or bool((np.diff(host) == 1).all())):
            self.stats.contiguous_views += 1
            first = int(host[0])
            return self.kv[:, :, first : first + n]
        self.stats.gathers += 1
        out = torch.empty(self.layers, 2, n, self.heads, self.head_dim, dtype=self.kv.dtype, device=self.device)
        if n:
            self._require_cuda(indices)
            self._copy("gather", self.kv, out, indices, host, n_planes=2 * self.layers)
        return out

    def gather_into(self, indices: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """``gather`` into a caller buffer [L, 2, n, H, D] (always a copy; never a view)."""
        host = self._host_slots(indices)
        self._require_cuda(indices, out)
        self._check_kv_shape(out, len(host))
        if out.dtype != self.kv.dtype or out.stride(4) != 1 or out.stride(3) != self.head_dim or \
                out.stride(2) != self.heads * self.head_dim:
            raise ValueError("gather_into needs a pool-dtype output with contiguous [n, H, D] rows")
        if len(host):
            self._copy("gather", self.kv, out, indices, host, n_planes=2 * self.layers)
        return out

    def gather_heads(self, indices: torch.Tensor, length: int | None = None) -> torch.Tensor:
        """K/V of `indices` head-major with room for a tail: [L, 2, H, length, D] (length >= n, default n), the
        first n positions filled from the pool, the rest left for the caller. For the text encoder's partial hit
        (encoder.py:173-182): write layer l's tail K/V into ``buf[l, :, :, m:]`` and attend over ``buf[l, 0][None]``
        / ``buf[l, 1][None]`` instead of transposing and concatenating the prefix every layer. One launch."""
        host = self._host_slots(indices)
        n = len(host)
        length = n if length is None else int(length)
        if length < n:
            raise ValueError(f"length {length} is shorter than the {n} gathered tokens")
        out = torch.empty(self.layers, 2, self.heads, length, self.head_dim, dtype=self.kv.dtype, device=self.device)
        if n:
            self._require_cuda(indices)
            e = self.kv.element_size()
            pool = _lib.planes(self.kv.data_ptr(), self.kv.stride(0) * e, self.kv.stride(1) * e, 2)
            oth = _lib.planes(out.data_ptr(), out.stride(0) * e, out.stride(1) * e, 2)
            slots = indices if indices.dtype == torch.int64 else indices.to(torch.int64)
            slots = slots.contiguous()
            with _lib.on_device(self.device):
                _lib.call("qe_gather_slots_heads", pool, self.rows, oth, 2 * self.layers, self._row_bytes(self.kv),
                          self.head_dim * e, out.stride(2) * e, out.stride(3) * e, slots.data_ptr(), n,
                          self._err.data_ptr(), self._stream())
        return out

    def write(self, indices: torch.Tensor, kv: torch.Tensor) -> None:
        """Scatter kv [L, 2, n, H, D] into pool rows `indices` (index_copy_ along dim 2)."""
        if kv.dtype != self.kv.dtype:
            kv = kv.to(self.kv.dtype)
        n = indices.numel()
        self._check_kv_shape(kv, n)
        if n == 0:
            return
        self._require_cuda(indices, kv)
        if kv.stride(4) != 1 or kv.stride(3) != self.head_dim or kv.stride(2) != self.heads * self.head_dim:
            kv = kv.contiguous()
        host = getattr(indices, "_qe_host", None)
        self._copy("append", self.kv, kv, indices, host, n_planes=2 * self.layers)

    def write_layers(self, indices: torch.Tensor, keys: list[torch.Tensor], values: list[torch.Tensor]) -> None:
        """``_store_computed``'s per-layer copies (hooks.py:136-138) in one launch: pool.kv[l, 0, idx] = keys[l]."""
        n = indices.numel()
        if len(keys) != self.layers or len(values) != self.layers:
            raise ValueError("write_layers needs one key and one value tensor per layer")
        if n == 0:
            return
        self._require_cuda(indices)
        ptrs = []
        srcs = []
        for k, v in zip(keys, values):
            for t in (k, v):
                if t.dtype != self.kv.dtype:
                    t = t.to(self.kv.dtype)
                if tuple(t.shape) != (n, self.heads, self.head_dim):
                    raise ValueError(f"layer K/V must be [{n}, {self.heads}, {self.head_dim}], got {tuple(t.shape)}")
                t = t.contiguous()
                self._require_cuda(t)
                if t.data_ptr() % 16:
                    t = t.clone()
                srcs.append(t)
                ptrs.append(t.data_ptr())
        table = torch.tensor(ptrs, dtype=torch.int64).pin_memory().to(self.device, non_blocking=True)
        self.h2d_bytes += 8 * len(ptrs)
        row = self._row_bytes(self.kv)
        e = self.kv.element_size()
        pool = _lib.planes(self.kv.data_ptr(), self.kv.stride(0) * e, self.kv.stride(1) * e, 2)
        slots = indices if indices.dtype == torch.int64 else indices.to(torch.int64)
        with _lib.on_device(self.device):
            _lib.call("qe_append_slots_ptrs", pool, self.rows, table.data_ptr(), 2 * self.layers, row,
                      slots.data_ptr(), n, self._err.data_ptr(), self._stream())
        # keep the sources and the pointer table alive until the launch has consumed them
        stream = torch.cuda.current_stream(self.device)
        for t in srcs:
            t.record_stream(stream)
        table.record_stream(stream)

    def gather_extra(self, indices: torch.Tensor) -> torch.Tensor:
        """``extra.index_select(0, indices)`` (encoder.py:114) as one gather launch."""
        if self.extra is None:
            raise RuntimeError("pool has no extra rows")
        host = self._host_slots(indices)
        out = torch.empty(len(host), self.extra_dim, dtype=self.extra.dtype, device=self.device)
        if len(host):
            self._require_cuda(indices)
            self._copy_extra("gather", out, indices, host)
        return out

    def write_extra(self, indices: torch.Tensor, rows: torch.Tensor) -> None:
        """``extra.index_copy_(0, indices, rows)`` (encoder.py:135) as one append launch."""
        if self.extra is None:
            raise RuntimeError("pool has no extra rows")
        rows = rows.to(self.extra.dtype).contiguous()
        n = indices.numel()
        if tuple(rows.shape) != (n, self.extra_dim):
            raise ValueError(f"extra rows must be [{n}, {self.extra_dim}]")
        if n:
            self._require_cuda(indices, rows)
            self._copy_extra("append", rows, indices, getattr(indices, "_qe_host", None))

    def _check_kv_shape(self, t: torch.Tensor, n: int) -> None:
        want = (self.layers, 2, n, self.heads, self.head_dim)
        if tuple(t.shape) != want:
            raise ValueError(f"K/V tensor must be {list(want)}, got {list(t.shape)}")

    def _copy(self, kind: str, pool_t: torch.Tensor, other: torch.Tensor, indices: torch.Tensor,
              host: np.ndarray | None, n_planes: int) -> None:
        e = pool_t.element_size()
        row = self._row_bytes(pool_t)
        pool = _lib.planes(pool_t.data_ptr(), pool_t.stride(0) * e, pool_t.stride(1) * e, 2)
        oth = _lib.planes(other.data_ptr(), other.stride(0) * e, other.stride(1) * e, 2)
        n = indices.numel()
        bt = self._block_table(indices, host) if host is not None else None
        with _lib.on_device(self.device):
            if bt is not None:
                _lib.call(f"qe_{kind}_pages", pool, self.rows, oth, n_planes, row, bt.data_ptr(), self.page_size, n,
                          self._err.data_ptr(), self._stream())
            else:
                slots = indices if indices.dtype == torch.int64 else indices.to(torch.int64)
                slots = slots.contiguous()
                _lib.call(f"qe_{kind}_slots", pool, self.rows, oth, n_planes, row, slots.data_ptr(), n,
                          self._err.data_ptr(), self._stream())

    def _copy_extra(self, kind: str, other: torch.Tensor, indices: torch.Tensor, host) -> None:
        e = self.extra.element_size()
        row = self.extra_dim * e
        pool = _lib.planes(self.extra.data_ptr(), 0, 0, 1)
        oth = _lib.planes(other.data_ptr(), 0, 0, 1)
        slots = indices if indices.dtype == torch.int64 else indices.to(torch.int64)
        slots = slots.contiguous()
        with _lib.on_device(self.device):
            _lib.call(f"qe_{kind}_slots", pool, self.rows, oth, 1, row, slots.data_ptr(), indices.numel(),
                      self._err.data_ptr(), self._stream())

    def device_errors(self) -> int:
        """Non-zero when a kernel skipped an out-of-range slot since the last call (reads the device flag)."""
        if self._err is None:
            return 0
        value = int(self._err.item())
        self._err.zero_()
        return value

    # ---- metrics -----------------------------------------------------------------------------
    def usage(self) -> dict:
        with self.lock:
            u = self.index.usage()
            return dict(
                capacity=self.capacity,
                free=u["free"],
                evictable=u["evictable"],
                protected=u["protected"],
                **self.stats.__dict__,
            )

    def clear(self) -> None:
        with self.lock:
            self.index.clear()
