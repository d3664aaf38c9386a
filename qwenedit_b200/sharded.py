"""Head-sharded prefix K/V pools over the GPUs of one node (one process per GPU).

QwenEdit keeps a session's whole-prefix K/V on one GPU and switches its pools off under tensor or sequence
parallelism (multi_turn/pipeline/encoding.py:214-220: "the pool holds whole-prefix K/V on one GPU; TP/SP shard
or exchange it"). ``HeadShardedKVPool`` is that shard-or-exchange: one logical pool spread over the ranks of a
process group by attention head. Rank r stores heads [r H/n, (r+1) H/n) of every pooled token.

* Index decisions (match / alloc / insert / LRU eviction) are replicated: every rank performs the same
  operations in the same order on its own native prefix index, so a token has the same slot on every rank and
  no slot list is ever sent. ``verify_replicas()`` compares a digest of the index state across ranks.
* ``gather`` / ``write`` move this rank's head slice only (tensor-parallel attention computes and reads its own
  heads): no communication.
* ``write_scatter`` takes K/V rows of a slice of the tokens with all heads (sequence parallel, before the
  attention all-to-all) and writes each head slice straight into its owner's pool through CUDA IPC peer
  mappings, in one kernel (``qe_append_scatter``): the all-to-all and the append are one pass over NVLink.
  ``barrier()`` (an all-reduce on the current stream) then makes the writes visible to every rank.

The pool memory of every rank is a plain device allocation exported with cudaIpcGetMemHandle and mapped by the
other ranks with cudaIpcOpenMemHandle; no multicast object and no waiting kernel is involved.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import logging
from ctypes import c_void_p

import torch
import torch.distributed as dist

from qwenedit_b200 import _lib
from qwenedit_b200.paged import PagedKVPool, pool_geometry

logger = logging.getLogger(__name__)

_IPC_HANDLE_BYTES = 64


class _DeviceMemory:
    """A device allocation seen as a flat uint8 tensor (own allocation, or another process's mapped in)."""

    def __init__(self, ptr: int, nbytes: int, device: torch.device, owner: bool):
        self.ptr, self.nbytes, self.device, self.owner = ptr, nbytes, device, owner
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}

    def tensor(self, dtype: torch.dtype, shape) -> torch.Tensor:
        flat = torch.as_tensor(self, device=self.device)  # zero-copy; keeps `self` alive
        return flat.view(dtype).view(shape)

    def close(self) -> None:
        if self.ptr:
            with torch.cuda.device(self.device):
                _lib.call("qe_ipc_free" if self.owner else "qe_ipc_close", self.ptr)
            self.ptr = 0


def _ipc_alloc(nbytes: int, device: torch.device) -> tuple[_DeviceMemory, bytes]:
    ptr = c_void_p()
    handle = (ctypes.c_uint8 * _IPC_HANDLE_BYTES)()
    with torch.cuda.device(device):
        _lib.call("qe_ipc_alloc", nbytes, ctypes.byref(ptr), ctypes.addressof(handle))
    return _DeviceMemory(ptr.value, nbytes, device, owner=True), bytes(handle)


def _ipc_open(handle: bytes, nbytes: int, device: torch.device) -> _DeviceMemory:
    buf = (ctypes.c_uint8 * _IPC_HANDLE_BYTES).from_buffer_copy(handle)
    ptr = c_void_p()
    with torch.cuda.device(device):
        _lib.call("qe_ipc_open", ctypes.addressof(buf), ctypes.byref(ptr))
    return _DeviceMemory(ptr.value, nbytes, device, owner=False)


def exchange(obj, group=None) -> list:
    """All ranks' `obj` in rank order (host objects, over the group's backend)."""
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


def index_digest(pool: PagedKVPool) -> str:
    """Digest of a pool's index state as every operation changes it: free / evictable / protected tokens and
    the lookup, insert and eviction counters."""
    return hashlib.blake2b(json.dumps(pool.usage(), sort_keys=True).encode(), digest_size=16).hexdigest()


def verify_replicas(pool: PagedKVPool, group=None) -> None:
    """Raise RuntimeError when the ranks' replicated index states differ (a rank skipped or reordered an
    operation); every rank raises, so none proceeds to a gather with slots that disagree."""
    digests = exchange(index_digest(pool), group)
    if len(set(digests)) != 1:
        raise RuntimeError(f"head-sharded pool {pool.name!r}: index replicas differ across ranks: {digests}")


class HeadShardedKVPool:
    """One prefix pool of [L, 2, tokens, H, D] spread over the ranks of `group` by head (see the module doc).

    `budget_bytes` is per rank. Same index API as ``PagedKVPool``; data movement on this rank's head slice.
    """

    def __init__(self, name, layers, heads, head_dim, budget_bytes, dtype, device, group=None, page_size=1):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if heads % self.world:
            raise ValueError(f"{heads} heads do not split over {self.world} ranks")
        if self.world > 8:
            raise ValueError("head-sharded pools span at most 8 ranks")
        self.heads = heads
        self.heads_local = heads // self.world
        self.head_start = self.rank * self.heads_local
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        _, rows, _ = pool_geometry(layers, self.heads_local, head_dim, budget_bytes, dtype, 0, page_size)
        elem = torch.empty((), dtype=dtype).element_size()
        nbytes = layers * 2 * rows * self.heads_local * head_dim * elem
        self._own, handle = _ipc_alloc(nbytes, self.device)
        kv = self._own.tensor(dtype, (layers, 2, rows, self.heads_local, head_dim))
        self.pool = PagedKVPool(name, layers, self.heads_local, head_dim, budget_bytes, dtype, self.device,
                                page_size=page_size, kv=kv)
        handles = exchange(handle, group)
        self._peers = [None if r == self.rank else _ipc_open(h, nbytes, self.device) for r, h in enumerate(handles)]
        bases = [self._own.ptr if m is None else m.ptr for m in self._peers]
        self._bases = (c_void_p * self.world)(*bases)
        self._barrier_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.nvlink_bytes = 0  # bytes this rank has written into other ranks' pools

    # ---- replicated index (same calls, same order, on every rank) -------------------------------
    @property
    def kv(self) -> torch.Tensor:
        return self.pool.kv

    @property
    def name(self) -> str:
        return self.pool.name

    def match(self, vids):
        return self.pool.match(vids)

    def alloc(self, n: int):
        return self.pool.alloc(n)

    def insert(self, vids, indices: torch.Tensor, owned_from: int) -> None:
        self.pool.insert(vids, indices, owned_from)

    def usage(self) -> dict:
        return self.pool.usage()

    def clear(self) -> None:
        self.pool.clear()

    def verify_replicas(self) -> None:
        verify_replicas(self.pool, self.group)

    # ---- data movement ---------------------------------------------------------------------------
    def gather(self, indices: torch.Tensor) -> torch.Tensor:
        """This rank's heads of `indices`: [L, 2, n, H/n, D] (local, no communication)."""
        return self.pool.gather(indices)

    def gather_into(self, indices: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        return self.pool.gather_into(indices, out)

    def write(self, indices: torch.Tensor, kv_local: torch.Tensor) -> None:
        """Write this rank's heads ([L, 2, n, H/n, D]) of the tokens at `indices` (tensor parallel)."""
        self.pool.write(indices, kv_local)

    def write_scatter(self, indices: torch.Tensor, kv: torch.Tensor) -> None:
        """Write K/V rows of this rank's tokens with ALL heads ([L, 2, n, H, D], `indices` their n slots) into
        every rank's pool: head slice r goes to rank r over NVLink, in one launch. Call ``barrier()`` on every
        rank before any rank reads the written rows."""
        pool = self.pool
        L, D = pool.layers, pool.head_dim
        if tuple(kv.shape) != (L, 2, indices.numel(), self.heads, D):
            raise ValueError(f"kv must be [{L}, 2, {indices.numel()}, {self.heads}, {D}], got {list(kv.shape)}")
        pool._require_cuda(kv, indices)
        if kv.dtype != pool.kv.dtype:
            kv = kv.to(pool.kv.dtype)
        if kv.stride(4) != 1 or kv.stride(3) != D or kv.stride(2) != self.heads * D:
            kv = kv.contiguous()
        slots = indices if indices.dtype == torch.int64 else indices.to(torch.int64)
        slots = slots.contiguous()
        e = pool.kv.element_size()
        geom = _lib.planes(0, pool.kv.stride(0) * e, pool.kv.stride(1) * e, 2)
        src = _lib.planes(kv.data_ptr(), kv.stride(0) * e, kv.stride(1) * e, 2)
        slice_bytes = self.heads_local * D * e
        n = slots.numel()
        with torch.cuda.device(self.device):
            _lib.call("qe_append_scatter", self._bases, self.world, geom, pool.rows, src, 2 * L, slice_bytes,
                      slots.data_ptr(), n, pool._err.data_ptr(), pool._stream())
        self.nvlink_bytes += (self.world - 1) * 2 * L * n * slice_bytes

    def barrier(self) -> None:
        """Stream-ordered barrier over the group: after it, every rank's earlier scatters are visible here."""
        dist.all_reduce(self._barrier_flag, group=self.group)

    def device_errors(self) -> int:
        return self.pool.device_errors()

    def close(self) -> None:
        """Unmap the peers' pools, then free this rank's (every rank must call it; collective). Tensors returned
        by ``gather`` as views of the pool are invalid afterwards."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for m in self._peers:
            if m is not None:
                m.close()
        self._peers = []
        dist.barrier(group=self.group)
        self.pool = None
        self._own.close()
        self._own = None

    def __del__(self):
        # releasing the memory needs the other ranks (they may still map it), so it is never done here: a pool
        # dropped without close() keeps its allocation until the process exits
        if getattr(self, "_own", None) is not None:
            logger.warning("HeadShardedKVPool %r dropped without close(); its device memory is held until exit",
                           getattr(self.pool, "name", "?"))


__all__ = ["HeadShardedKVPool", "exchange", "index_digest", "verify_replicas"]
