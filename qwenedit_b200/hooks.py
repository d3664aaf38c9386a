"""Pool call sites of the DiT and text-encoder prefix caches, on the B200 pool.

Drop-in for the pool-facing parts of
  multi_turn/pipeline/encoding.py:34-49     MTCaches (per-request caches, vids, prefix lengths, held matches)
  multi_turn/pipeline/hooks.py:81-83        _set_caches       (per-layer views of a gathered prefix)
  multi_turn/pipeline/hooks.py:86-123       _fill_from_pool   (full hit / partial reuse / miss per sample)
  multi_turn/pipeline/hooks.py:126-139      _store_computed   (after a miss: 2*L index_copy_ -> ONE launch)
  multi_turn/cache/encoder.py:111-138       _encode's pool hit and _store (K/V planes + hidden-state rows)

The model compute that sits between them (the DiT tail prefill, cache/prefill.py:32-72, and the encoder
tail forward, cache/encoder.py:141-203) stays with the caller: ``fill_from_pool`` takes it as a callback.
Per-layer caches are any objects with ``update(key=..., value=...)`` and ``[...]`` access to "key" / "value",
as the SGLang DiT's joint-attention caches are.
"""

from __future__ import annotations

import logging
import time
from typing import Callable

import torch

from qwenedit_b200 import state
from qwenedit_b200.paged import Match, PagedKVPool, cat_slots

logger = logging.getLogger(__name__)


class MTCaches(list):
    """Per-request prefix caches (encoding.py:34-49): one list of per-layer caches per sample, the samples'
    virtual ids and prefix lengths, and the matches held until the request ends."""

    def __init__(self, caches, vids, prefix_lengths):
        super().__init__(caches)
        self.vids = vids
        self.prefix_lengths = prefix_lengths
        self.prepared = False
        self.matches: list[Match] = []
        # sample -> PagedPrefix: full hits served without a gather (fill_from_pool(paged=True)); the attention
        # reads them through qwenedit_b200.attention.paged_attention
        self.paged: dict = {}

    def release(self) -> None:
        for match in self.matches:
            match.release()
        self.matches.clear()

    def __del__(self):
        self.release()


def set_caches(caches, sample: int, kv: torch.Tensor) -> None:
    """Point each layer's joint-attention cache at its [1, n, H, D] K and V views of `kv` (no copy)."""
    for layer in range(kv.shape[0]):
        caches[sample][layer].update(key=kv[layer, 0][None], value=kv[layer, 1][None])


# prefill(sample, kv, start): fill kv[:, :, start:] ([L, 2, total, H, D]) for prefix positions start.. of `sample`
Prefill = Callable[[int, torch.Tensor, int], None]

FULL, PARTIAL, MISS = "full", "partial", "miss"


def classify(matched: int, total: int, can_prefill: bool) -> str:
    """How a sample's prefix is served given the matched length: the whole prefix cached (FULL); enough of it
    cached to be worth a tail prefill, at least MULTI_TURN_MIN_REUSE tokens, when the caller can prefill (PARTIAL);
    otherwise computed from scratch (MISS). The reference's branch rule (hooks.py:99-123)."""
    if matched == total:
        return FULL
    if can_prefill and matched >= state.MIN_REUSE:
        return PARTIAL
    return MISS


def _serve_full(pool: PagedKVPool, caches: MTCaches, sample: int, match: Match, paged: bool) -> None:
    # the gathered prefix (a view when its slots are one run), or the pages themselves, stay valid while the match
    # holds its lock
    if paged:
        from qwenedit_b200.attention import PagedPrefix

        caches.paged[sample] = PagedPrefix(pool, match.indices)
    else:
        set_caches(caches, sample, pool.gather(match.indices))
    caches.matches.append(match)


def _serve_partial(pool: PagedKVPool, caches: MTCaches, sample: int, match: Match, vids, total: int,
                   prefill: Prefill) -> None:
    m = match.length
    kv = torch.empty(pool.layers, 2, total, pool.heads, pool.head_dim, device=pool.kv.device, dtype=pool.kv.dtype)
    pool.gather_into(match.indices, kv[:, :, :m])
    prefill(sample, kv, m)
    set_caches(caches, sample, kv)
    tail = pool.alloc(total - m)
    if tail is not None:  # pool full of locked prefixes: serve this request, cache nothing
        pool.write(tail, kv[:, :, m:])
        pool.insert(vids, cat_slots(match.indices, tail), owned_from=m)
    match.release()  # the fresh buffer owns the data now


def fill_from_pool(pool: PagedKVPool, caches: MTCaches, prefill: Prefill | None = None, paged: bool = False) -> list[int]:
    """Serve each sample's prefix from the pool (hooks.py:86-123); returns the samples that missed, to be stored
    after the forward by `store_computed`.

    FULL: the prefix is gathered once and its match kept locked until the request ends (with `paged`, on a
    page-mode pool: not gathered at all; `caches.paged[sample]` is a PagedPrefix the attention reads the pages
    through); PARTIAL: the cached head goes into a fresh [L, 2, total, H, D] buffer, `prefill` computes the tail
    into it, and the tail is appended and inserted (owned from the match); MISS: nothing reused."""
    if paged and pool.page_size == 1:
        raise ValueError("paged serving needs a page-mode pool (page_size 8 or more)")
    pending = []
    for sample, vids in enumerate(caches.vids):
        if vids is None:
            continue
        t0 = time.perf_counter()
        total = caches.prefix_lengths[sample]
        match = pool.match(vids)
        kind = classify(match.length, total, prefill is not None)
        reused = match.length if kind != MISS else 0
        if kind == FULL:
            _serve_full(pool, caches, sample, match, paged)
        elif kind == PARTIAL:
            _serve_partial(pool, caches, sample, match, vids, total, prefill)
        else:
            match.release()
            pending.append(sample)
        if state.DEBUG:
            logger.info("qwenedit_b200: dit sample %d (%s) reused %d/%d prefix tokens in %.1f ms", sample, kind,
                        reused, total, (time.perf_counter() - t0) * 1e3)
    return pending


def store_computed(pool: PagedKVPool, caches: MTCaches, pending: list[int]) -> None:
    """After a miss, copy every layer's freshly computed prefix K/V into the pool in one launch and insert it."""
    for sample in pending:
        layers = caches[sample]
        if not layers[0]:
            continue
        total = caches.prefix_lengths[sample]
        slots = pool.alloc(total)
        if slots is None:
            continue
        pool.write_layers(slots, [layer["key"][0] for layer in layers], [layer["value"][0] for layer in layers])
        pool.insert(caches.vids[sample], slots, owned_from=0)


# ---- text encoder ------------------------------------------------------------------------------
def encoder_hit(pool: PagedKVPool, match: Match, total: int) -> torch.Tensor | None:
    """The full-hit branch of encoder.py:113-114: the cached hidden states of all `total` tokens, else None."""
    if match.length != total or match.indices is None:
        return None
    return pool.gather_extra(match.indices)


def encoder_store(pool: PagedKVPool, vids, match: Match | None, kv_new: torch.Tensor, hidden_new: torch.Tensor,
                  m: int) -> bool:
    """encoder.py:131-138: store the new tokens' K/V planes [L, 2, n, H, D] and hidden rows [n, hidden].
    Returns False (nothing stored) when the pool cannot make room."""
    slots = pool.alloc(kv_new.shape[2])
    if slots is None:
        return False
    pool.write(slots, kv_new)
    pool.write_extra(slots, hidden_new)
    indices = cat_slots(match.indices, slots) if m else slots
    pool.insert(vids, indices, owned_from=m)
    return True


# ---- stored output versions ---------------------------------------------------------------------
def compose(spec: dict, crop_latents: torch.Tensor, crop_grid: tuple[int, int]) -> bool:
    """``_compose`` (pipeline/hooks.py:232-247): store, as version ``spec["as"]``, the latents of version
    ``spec["base"]`` with the cells of ``spec["box"]`` replaced by ``crop_latents`` — one launch
    (``latents.compose``) instead of clone + slice assignment. Same checks and warnings; returns False when
    nothing was stored (missing base, or a box that does not match the crop grid)."""
    from qwenedit_b200 import latents

    base = state.OUTPUT_LATENTS.get(spec.get("base"))
    base_grid = state.OUTPUT_GRID.get(spec.get("base"))
    if base is None or base_grid is None:
        logger.warning("qwenedit_b200: compose base %s missing; the new version has no stored latents",
                       spec.get("base"))
        return False
    x0, y0, x1, y1 = (int(v) for v in spec["box"])
    if (y1 - y0, x1 - x0) != tuple(crop_grid):
        logger.warning("qwenedit_b200: compose box %s does not match the crop grid %s", spec["box"], crop_grid)
        return False
    state.OUTPUT_LATENTS.put(spec["as"], latents.compose(base, base_grid, crop_latents, (x0, y0, x1, y1)))
    state.OUTPUT_GRID[spec["as"]] = base_grid
    return True


__all__ = ["MTCaches", "set_caches", "classify", "fill_from_pool", "store_computed", "encoder_hit", "encoder_store",
           "compose"]
