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


def test_settings_read_the_reference_variables():
    env = {"MULTI_TURN_PREFIX_CACHE": "0", "MULTI_TURN_DEBUG": "1", "MULTI_TURN_MIN_REUSE": "64",
           "MULTI_TURN_ENC_MIN_REUSE": "32", "MULTI_TURN_LATENT_SLOTS": "7", "MULTI_TURN_KV_GPU_GIB": "1.5",
           "MULTI_TURN_ENC_GPU_GIB": "0.25", "MULTI_TURN_KV_PAGE": "64"}
    s = state.Settings.from_env(env)
    assert (s.prefix_cache, s.encoder_cache, s.debug) == (False, True, True)
    assert (s.min_reuse, s.enc_min_reuse, s.latent_slots) == (64, 32, 7)
    assert (s.dit_pool_gib, s.encoder_pool_gib, s.dit_page, s.encoder_page) == (1.5, 0.25, 64, 1)
    assert state.Settings.from_env({}) == state.Settings()


def test_pool_registry_builds_once_and_resets():
    class FakePool:
        def __init__(self):
            self.cleared = 0

        def usage(self):
            return {"cleared": self.cleared}

        def clear(self):
            self.cleared += 1

    reg = state.PoolRegistry()
    built = []
    first = reg.get_or_build("dit", lambda: built.append(1) or FakePool())
    again = reg.get_or_build("dit", lambda: built.append(1) or FakePool())
    assert first is again and built == [1]
    assert reg.usage("encoder") is None and reg.usage("dit") == {"cleared": 0}
    reg.clear_all()
    assert reg.usage("dit") == {"cleared": 1}


def test_key_roots_are_the_reference_tuples():
    from types import SimpleNamespace

    from qwenedit_b200 import keys

    args = SimpleNamespace(model_path="/m", component_quantizations={"t": "fp4"}, transformer_quantization="fp4")
    assert state.dit_root(args) == keys.root_key("dit", "/m", {"t": "fp4"}, "fp4", None)
    enc = SimpleNamespace(text_encoder=SimpleNamespace(config=SimpleNamespace(_name_or_path="qwen-vl")))
    assert state.encoder_root(enc) == keys.root_key("encoder", "qwen-vl", None)
    u = state.usage()
    assert set(u) == {"dit", "encoder", "output_latents", "vae_latents"}
