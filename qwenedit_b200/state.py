"""Process-wide cache state: drop-in for ``multi_turn.state`` (reference: multi_turn/state.py:19-136).

What callers see is the reference's module surface: the flags ``PREFIX_CACHE``, ``ENCODER_CACHE``, ``DEBUG``,
``MIN_REUSE``, ``ENC_MIN_REUSE``; the latent stores ``OUTPUT_LATENTS`` / ``VAE_LATENTS`` (``LRU``) and
``OUTPUT_GRID``; ``stored_latents``; the lazily built pools ``dit_pool(model)`` / ``encoder_pool(encoder,
device)``; the key roots ``dit_root`` / ``encoder_root``; ``usage()`` and ``reset()``.

How it is organised here: one frozen ``Settings`` record read from the environment at import (same variable
names and defaults as the reference, plus the page sizes of the two pools), a ``PoolRegistry`` that owns the
pools by kind and builds each on first use, and an ``LRU`` kept as a plain insertion-ordered dict in which a
touched key is moved to the end by re-insertion.

Environment: MULTI_TURN_PREFIX_CACHE (1), MULTI_TURN_ENCODER_CACHE (1), MULTI_TURN_DEBUG (0),
MULTI_TURN_MIN_REUSE (256), MULTI_TURN_ENC_MIN_REUSE (128), MULTI_TURN_LATENT_SLOTS (512),
MULTI_TURN_KV_GPU_GIB (24), MULTI_TURN_ENC_GPU_GIB (4); additions: MULTI_TURN_KV_PAGE / MULTI_TURN_ENC_PAGE
(page size of the DiT / encoder pool; 1 = the reference's token-granular slots).
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Callable

import torch

from qwenedit_b200 import keys

logger = logging.getLogger(__name__)
GIB = 1 << 30


@dataclass(frozen=True)
class Settings:
    """Switches and sizes of the multi-turn caches, as the environment gives them."""

    prefix_cache: bool = True
    encoder_cache: bool = True
    debug: bool = False
    min_reuse: int = 256
    enc_min_reuse: int = 128
    latent_slots: int = 512
    dit_pool_gib: float = 24.0
    encoder_pool_gib: float = 4.0
    dit_page: int = 1
    encoder_page: int = 1

    @classmethod
    def from_env(cls, env=None) -> "Settings":
        env = os.environ if env is None else env

        def flag(name, default):
            return env.get(name, default) == "1"

        return cls(
            prefix_cache=flag("MULTI_TURN_PREFIX_CACHE", "1"),
            encoder_cache=flag("MULTI_TURN_ENCODER_CACHE", "1"),
            debug=flag("MULTI_TURN_DEBUG", "0"),
            min_reuse=int(env.get("MULTI_TURN_MIN_REUSE", 256)),
            enc_min_reuse=int(env.get("MULTI_TURN_ENC_MIN_REUSE", 128)),
            latent_slots=int(env.get("MULTI_TURN_LATENT_SLOTS", 512)),
            dit_pool_gib=float(env.get("MULTI_TURN_KV_GPU_GIB", 24)),
            encoder_pool_gib=float(env.get("MULTI_TURN_ENC_GPU_GIB", 4)),
            dit_page=int(env.get("MULTI_TURN_KV_PAGE", 1)),
            encoder_page=int(env.get("MULTI_TURN_ENC_PAGE", 1)),
        )


SETTINGS = Settings.from_env()
PREFIX_CACHE = SETTINGS.prefix_cache
ENCODER_CACHE = SETTINGS.encoder_cache
DEBUG = SETTINGS.debug
MIN_REUSE = SETTINGS.min_reuse
ENC_MIN_REUSE = SETTINGS.enc_min_reuse
KV_PAGE = SETTINGS.dit_page
ENC_PAGE = SETTINGS.encoder_page


class LRU:
    """A bounded map that drops its least recently used entry (reference rules, state.py:26-42): ``get`` of a
    present key and every ``put`` make that key the most recent; a ``put`` past ``capacity`` drops the oldest.
    ``items`` iterates oldest first."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self.items: dict = {}

    def _touch(self, key, value) -> None:
        self.items.pop(key, None)
        self.items[key] = value  # re-insertion puts the key last: dicts keep insertion order

    def get(self, key):
        value = self.items.get(key)
        if value is not None:
            self._touch(key, value)
        return value

    def put(self, key, value) -> None:
        self._touch(key, value)
        while len(self.items) > self.capacity:
            del self.items[next(iter(self.items))]


OUTPUT_LATENTS = LRU(SETTINGS.latent_slots)
OUTPUT_GRID: dict[str, tuple[int, int]] = {}
VAE_LATENTS = LRU(SETTINGS.latent_slots)


def _box_inside(box, grid) -> bool:
    x0, y0, x1, y1 = box
    rows, cols = grid
    return 0 <= x0 < x1 <= cols and 0 <= y0 < y1 <= rows


def stored_latents(latent_id, crop=None):
    """A previous turn's output latents [1, h*w, C], or the (x0, y0, x1, y1) box of them as [1, box cells, C]
    (a view when the box rows are contiguous). None when the id is unknown, the grid was never recorded or the
    box leaves the grid (reference: state.py:51-62)."""
    latents = OUTPUT_LATENTS.get(latent_id) if latent_id else None
    if latents is None or crop is None:
        return latents
    grid = OUTPUT_GRID.get(latent_id)
    if grid is None or not _box_inside(crop, grid):
        return None
    x0, y0, x1, y1 = crop
    cells = latents.view(1, grid[0], grid[1], -1)[:, y0:y1, x0:x1]
    return cells.reshape(1, (y1 - y0) * (x1 - x0), -1)


def kv_geometry(model) -> tuple[int, int, int]:
    """(layers, heads, head_dim) of a Qwen-Image DiT (reference: cache/prefill.py:14-16)."""
    blocks = model.transformer_blocks
    return len(blocks), blocks[0].attn.heads, blocks[0].attn.head_dim


def encoder_geometry(encoder) -> tuple[int, int, int, int]:
    """(layers, kv_heads, head_dim, hidden) of the Qwen-VL text encoder (reference: cache/encoder.py:62-65)."""
    lm = encoder.model.language_model
    first = lm.layers[0].self_attn
    return len(lm.layers), first.num_key_value_heads, first.head_dim, lm.config.hidden_size


class PoolRegistry:
    """The process's prefix pools by kind ("dit", "encoder"), each built on first request and kept for the
    life of the process (the reference's module globals, state.py:65-95)."""

    def __init__(self):
        self._pools: dict[str, object] = {}

    def get(self, kind: str):
        return self._pools.get(kind)

    def get_or_build(self, kind: str, build: Callable[[], object]):
        pool = self._pools.get(kind)
        if pool is None:
            pool = self._pools[kind] = build()
        return pool

    def usage(self, kind: str):
        pool = self._pools.get(kind)
        return pool.usage() if pool is not None else None

    def clear_all(self) -> None:
        for pool in self._pools.values():
            pool.clear()


POOLS = PoolRegistry()


def dit_pool(model):
    """The DiT prefix pool, sized by MULTI_TURN_KV_GPU_GIB on the device of the model's weights (state.py:68-80)."""

    def build():
        from qwenedit_b200.paged import PagedKVPool

        layers, heads, head_dim = kv_geometry(model)
        budget = int(SETTINGS.dit_pool_gib * GIB)
        return PagedKVPool("dit", layers, heads, head_dim, budget, torch.bfloat16, model.img_in.weight.device,
                           page_size=SETTINGS.dit_page)

    return POOLS.get_or_build("dit", build)


def encoder_pool(encoder, device):
    """The text-encoder prefix pool with the hidden-state rows as `extra` (state.py:83-95)."""

    def build():
        from qwenedit_b200.paged import PagedKVPool

        layers, kv_heads, head_dim, hidden = encoder_geometry(encoder)
        budget = int(SETTINGS.encoder_pool_gib * GIB)
        return PagedKVPool("encoder", layers, kv_heads, head_dim, budget, torch.bfloat16, device, extra_dim=hidden,
                           page_size=SETTINGS.encoder_page)

    return POOLS.get_or_build("encoder", build)


def _weights_epoch():
    """SGLang's conditioning-weights epoch when that runtime is present, else None (state.py:98-104)."""
    try:
        from sglang.multimodal_gen.runtime.cache.conditioning import conditioning_weights_epoch
    except Exception:
        return None
    try:
        return conditioning_weights_epoch()
    except Exception:
        return None


def encoder_root(stage) -> bytes:
    """Key root of the encoder pool: the encoder's checkpoint name (or class name) and the weights epoch."""
    encoder = stage.text_encoder
    name = getattr(getattr(encoder, "config", None), "_name_or_path", None) or type(encoder).__name__
    return keys.root_key("encoder", name, _weights_epoch())


def dit_root(server_args) -> bytes:
    """Key root of the DiT pool: model path, both quantisation settings and the weights epoch."""
    parts = (server_args.model_path, getattr(server_args, "component_quantizations", None),
             getattr(server_args, "transformer_quantization", None), _weights_epoch())
    return keys.root_key("dit", *parts)


def usage() -> dict:
    """Pool statistics and latent-store sizes (state.py:123-129)."""
    return {"dit": POOLS.usage("dit"), "encoder": POOLS.usage("encoder"),
            "output_latents": len(OUTPUT_LATENTS.items), "vae_latents": len(VAE_LATENTS.items)}


def reset() -> None:
    """Empty both pools (keeping their memory) and both latent stores (state.py:132-136)."""
    POOLS.clear_all()
    OUTPUT_LATENTS.items.clear()
    VAE_LATENTS.items.clear()
