"""Process-wide pools, key roots and latent LRUs: drop-in for ``multi_turn.state`` (state.py:19-136).

Same environment variables and defaults as the reference (read at import):
MULTI_TURN_PREFIX_CACHE, MULTI_TURN_ENCODER_CACHE, MULTI_TURN_DEBUG, MULTI_TURN_MIN_REUSE (256),
MULTI_TURN_ENC_MIN_REUSE (128), MULTI_TURN_LATENT_SLOTS (512), MULTI_TURN_KV_GPU_GIB (24),
MULTI_TURN_ENC_GPU_GIB (4); plus MULTI_TURN_KV_PAGE / MULTI_TURN_ENC_PAGE (page size of the DiT /
encoder pool, default 1 = the reference's token-granular slots).
"""

from __future__ import annotations

import logging
import os
from collections import OrderedDict

import torch

from qwenedit_b200 import keys

logger = logging.getLogger(__name__)
GIB = 1 << 30


def _env_float(name: str, default: float) -> float:
    return float(os.environ.get(name, default))


PREFIX_CACHE = os.environ.get("MULTI_TURN_PREFIX_CACHE", "1") == "1"
ENCODER_CACHE = os.environ.get("MULTI_TURN_ENCODER_CACHE", "1") == "1"
DEBUG = os.environ.get("MULTI_TURN_DEBUG", "0") == "1"
MIN_REUSE = int(os.environ.get("MULTI_TURN_MIN_REUSE", 256))
ENC_MIN_REUSE = int(os.environ.get("MULTI_TURN_ENC_MIN_REUSE", 128))
KV_PAGE = int(os.environ.get("MULTI_TURN_KV_PAGE", 1))
ENC_PAGE = int(os.environ.get("MULTI_TURN_ENC_PAGE", 1))


class LRU:
    """Bounded mapping that forgets the least recently used entry (state.py:26-42)."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self.items: OrderedDict = OrderedDict()

    def get(self, key):
        value = self.items.get(key)
        if value is not None:
            self.items.move_to_end(key)
        return value

    def put(self, key, value) -> None:
        self.items[key] = value
        self.items.move_to_end(key)
        while len(self.items) > self.capacity:
            self.items.popitem(last=False)


_slots = int(os.environ.get("MULTI_TURN_LATENT_SLOTS", 512))
OUTPUT_LATENTS = LRU(_slots)
OUTPUT_GRID: dict[str, tuple[int, int]] = {}
VAE_LATENTS = LRU(_slots)


def stored_latents(latent_id, crop=None):
    """Output latents of a previous turn, optionally cropped to (x0, y0, x1, y1) latent cells (state.py:51-62)."""
    latents = OUTPUT_LATENTS.get(latent_id) if latent_id else None
    if latents is None or crop is None:
        return latents
    grid = OUTPUT_GRID.get(latent_id)
    if grid is None:
        return None
    x0, y0, x1, y1 = crop
    h, w = grid
    if not (0 <= x0 < x1 <= w and 0 <= y0 < y1 <= h):
        return None
    return latents.view(1, h, w, -1)[:, y0:y1, x0:x1].reshape(1, (y1 - y0) * (x1 - x0), -1)


_dit_pool = None
_encoder_pool = None


def kv_geometry(model) -> tuple[int, int, int]:
    """(layers, heads, head_dim) of a Qwen-Image DiT (cache/prefill.py:14-16)."""
    attn = model.transformer_blocks[0].attn
    return len(model.transformer_blocks), attn.heads, attn.head_dim


def encoder_geometry(encoder) -> tuple[int, int, int, int]:
    """(layers, kv_heads, head_dim, hidden) of the Qwen-VL text encoder (cache/encoder.py:62-65)."""
    lm = encoder.model.language_model
    attn = lm.layers[0].self_attn
    return len(lm.layers), attn.num_key_value_heads, attn.head_dim, lm.config.hidden_size


def dit_pool(model):
    global _dit_pool
    if _dit_pool is None:
        from qwenedit_b200.paged import PagedKVPool

        layers, heads, head_dim = kv_geometry(model)
        _dit_pool = PagedKVPool(
            "dit", layers, heads, head_dim, int(_env_float("MULTI_TURN_KV_GPU_GIB", 24) * GIB), torch.bfloat16,
            model.img_in.weight.device, page_size=KV_PAGE,
        )
    return _dit_pool


def encoder_pool(encoder, device):
    global _encoder_pool
    if _encoder_pool is None:
        from qwenedit_b200.paged import PagedKVPool

        layers, kv_heads, head_dim, hidden = encoder_geometry(encoder)
        _encoder_pool = PagedKVPool(
            "encoder", layers, kv_heads, head_dim, int(_env_float("MULTI_TURN_ENC_GPU_GIB", 4) * GIB),
            torch.bfloat16, device, extra_dim=hidden, page_size=ENC_PAGE,
        )
    return _encoder_pool


def _weights_epoch():
    try:
        from sglang.multimodal_gen.runtime.cache.conditioning import conditioning_weights_epoch

        return conditioning_weights_epoch()
    except Exception:
        return None


def encoder_root(stage) -> bytes:
    config = getattr(stage.text_encoder, "config", None)
    name = getattr(config, "_name_or_path", None) or type(stage.text_encoder).__name__
    return keys.root_key("encoder", name, _weights_epoch())


def dit_root(server_args) -> bytes:
    return keys.root_key(
        "dit",
        server_args.model_path,
        getattr(server_args, "component_quantizations", None),
        getattr(server_args, "transformer_quantization", None),
        _weights_epoch(),
    )


def usage() -> dict:
    return {
        "dit": _dit_pool.usage() if _dit_pool else None,
        "encoder": _encoder_pool.usage() if _encoder_pool else None,
        "output_latents": len(OUTPUT_LATENTS.items),
        "vae_latents": len(VAE_LATENTS.items),
    }


def reset() -> None:
    for pool in (_dit_pool, _encoder_pool):
        if pool is not None:
            pool.clear()
    OUTPUT_LATENTS.items.clear()
    VAE_LATENTS.items.clear()
