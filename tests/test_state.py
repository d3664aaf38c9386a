"""Process-wide state (drop-in for multi_turn/state.py): the latent LRU's recency rule and the cropped
stored-latents lookup (state.py:26-62), on CPU."""

import torch

from qwenedit_b200 import state


def test_lru_forgets_least_recently_used():
    lru = state.LRU(2)
    lru.put("a", 1)
    lru.put("b", 2)
    assert lru.get("a") == 1  # a is now the most recent
    lru.put("c", 3)
    assert lru.get("b") is None and lru.get("a") == 1 and lru.get("c") == 3
    lru.put("a", 4)  # re-put refreshes and replaces
    lru.put("d", 5)
    assert list(lru.items) == ["a", "d"]
    assert lru.get("c") is None and lru.get("a") == 4 and list(lru.items) == ["d", "a"]


def test_stored_latents_crop_rules():
    lat = torch.arange(4 * 6 * 2, dtype=torch.float32).view(1, 24, 2)
    state.OUTPUT_LATENTS.put("v1", lat)
    state.OUTPUT_GRID["v1"] = (4, 6)
    assert state.stored_latents("v1") is lat
    assert state.stored_latents(None) is None and state.stored_latents("missing") is None
    crop = state.stored_latents("v1", (1, 1, 4, 3))
    want = lat.view(1, 4, 6, 2)[:, 1:3, 1:4].reshape(1, 6, 2)
    assert torch.equal(crop, want)
    full_width = state.stored_latents("v1", (0, 2, 6, 4))
    assert full_width.data_ptr() == lat.view(1, 4, 6, 2)[:, 2:4].data_ptr()  # a view, as reshape gives
    for bad in ((0, 0, 7, 1), (2, 1, 2, 2), (0, 3, 1, 5)):
        assert state.stored_latents("v1", bad) is None
    state.OUTPUT_LATENTS.put("nogrid", lat)
    assert state.stored_latents("nogrid", (0, 0, 1, 1)) is None


def test_environment_defaults():
    assert state.MIN_REUSE == 256 and state.ENC_MIN_REUSE == 128
    assert state.KV_PAGE >= 1 and state.ENC_PAGE >= 1
    assert state.OUTPUT_LATENTS.capacity == 512
