"""Session partitioning across the GPUs of one node (one process per GPU).

An edit session's prefix K/V lives only in the pools of the GPU that owns it, so the path shards by session
with no collective on the data path: ``owner(session_id, world)`` is a stable hash (BLAKE2b of the id, not
Python's salted ``hash``), identical in every process, and each rank serves only the sessions it owns.
The reference runs on one GPU and turns its pools off under TP/SP (pipeline/encoding.py:214-220); this
module is the multi-GPU layer it does not have.
"""

from __future__ import annotations

import hashlib
from collections.abc import Iterable


def owner(session_id: str, world: int) -> int:
    """Rank that owns `session_id` among `world` ranks (stable across processes and runs)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    digest = hashlib.blake2b(session_id.encode(), digest_size=8).digest()
    return int.from_bytes(digest, "little") % world


class SessionRouter:
    """This rank's view of the session partition."""

    def __init__(self, rank: int, world: int):
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        self.rank, self.world = rank, world

    def owns(self, session_id: str) -> bool:
        return owner(session_id, self.world) == self.rank

    def mine(self, session_ids: Iterable[str]) -> list[str]:
        return [s for s in session_ids if self.owns(s)]

    def partition(self, session_ids: Iterable[str]) -> dict[int, list[str]]:
        parts: dict[int, list[str]] = {r: [] for r in range(self.world)}
        for s in session_ids:
            parts[owner(s, self.world)].append(s)
        return parts
