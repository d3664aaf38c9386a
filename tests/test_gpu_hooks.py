"""Pool call sites (hooks.py:81-139, encoder.py:111-138) on the B200 pool: miss -> store -> full hit -> partial,
checked value for value against the tensors the DiT / encoder produced."""

import numpy as np
import pytest
import torch

from qwenedit_b200 import hooks, state
from qwenedit_b200.paged import PagedKVPool

pytestmark = pytest.mark.gpu
DEV = "cuda"
L, H, D = 6, 24, 128


class LayerCache(dict):
    """Stands in for the DiT's joint-attention layer cache: update(key=, value=) and ["key"] / ["value"]."""


def _pool(tokens, page=1):
    return PagedKVPool("dit", L, H, D, tokens * L * 2 * H * D * 2, torch.bfloat16, DEV, page_size=page)


def _computed(total, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [LayerCache(key=torch.randn(1, total, H, D, generator=g, device=DEV).bfloat16(),
                       value=torch.randn(1, total, H, D, generator=g, device=DEV).bfloat16()) for _ in range(L)]


@pytest.mark.parametrize("page", [1, 16])
def test_miss_store_hit_partial(page):
    pool = _pool(4000, page)
    total = 640
    vids = np.arange(1, total + 1, dtype=np.int64)
    # request 1: miss; the DiT computed every layer's K/V; store it in one launch
    layers = _computed(total, 0)
    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [vids], [total])
    assert hooks.fill_from_pool(pool, caches) == [0]
    caches[0] = layers
    hooks.store_computed(pool, caches, [0])
    caches.release()
    # request 2: full hit -> per-layer views equal what was computed
    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [vids], [total])
    assert hooks.fill_from_pool(pool, caches) == []
    for i in range(L):
        assert torch.equal(caches[0][i]["key"], layers[i]["key"])
        assert torch.equal(caches[0][i]["value"], layers[i]["value"])
    assert len(caches.matches) == 1 and pool.usage()["protected"] == total
    caches.release()
    assert pool.usage()["protected"] == 0
    # request 3: shares the first 512 tokens (>= MIN_REUSE) then diverges; prefill fills the tail
    vids3 = np.concatenate([vids[:512], np.arange(10_000, 10_192, dtype=np.int64)])  # page-aligned total
    total3 = len(vids3)
    tail_seen = {}

    def prefill(sample, kv, start):
        tail_seen["start"] = start
        kv[:, :, start:] = float(sample + 7)

    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [vids3], [total3])
    assert hooks.fill_from_pool(pool, caches, prefill) == []
    assert tail_seen["start"] == 512 >= state.MIN_REUSE
    for i in range(L):
        assert torch.equal(caches[0][i]["key"][0, :512], layers[i]["key"][0, :512])
        assert torch.all(caches[0][i]["key"][0, 512:] == 7.0)
    # request 4: now a full hit of the partial's prefix, served from the pool
    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [vids3], [total3])
    assert hooks.fill_from_pool(pool, caches) == []
    got = torch.cat([caches[0][i]["value"] for i in range(L)])
    assert torch.all(got[:, 512:] == 7.0)
    assert torch.equal(got[:, :512], torch.cat([layers[i]["value"][:, :512] for i in range(L)]))
    caches.release()
    assert pool.device_errors() == 0


def test_short_match_is_a_miss():
    pool = _pool(2000)
    vids = np.arange(1, 400, dtype=np.int64)
    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [vids], [len(vids)])
    hooks.fill_from_pool(pool, caches)
    caches[0] = _computed(len(vids), 1)
    hooks.store_computed(pool, caches, [0])
    short = np.concatenate([vids[:100], [999_999]])  # 100 < MIN_REUSE shared tokens
    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [short], [len(short)])
    assert hooks.fill_from_pool(pool, caches, prefill=lambda *a: None) == [0]
    assert pool.usage()["protected"] == 0


def test_encoder_store_and_hit():
    enc = PagedKVPool("encoder", 28, 4, 128, 3000 * (28 * 2 * 4 * 128 + 3584) * 2, torch.bfloat16, DEV,
                      extra_dim=3584)
    vids = np.arange(5, 305, dtype=np.int64)
    g = torch.Generator(device=DEV).manual_seed(3)
    kv = torch.randn(28, 2, 300, 4, 128, generator=g, device=DEV).bfloat16()
    hidden = torch.randn(300, 3584, generator=g, device=DEV).bfloat16()
    m = enc.match(vids)
    assert hooks.encoder_hit(enc, m, len(vids)) is None
    assert hooks.encoder_store(enc, vids, m, kv, hidden, 0)
    m.release()
    m = enc.match(vids)
    assert torch.equal(hooks.encoder_hit(enc, m, len(vids)), hidden)
    assert torch.equal(enc.gather(m.indices), kv)
    m.release()
    # a longer prompt sharing the first 300 tokens: store only the new 50 (owned from the match)
    longer = np.concatenate([vids, np.arange(7000, 7050, dtype=np.int64)])
    m = enc.match(longer)
    assert m.length == 300
    kv2 = torch.randn(28, 2, 50, 4, 128, generator=g, device=DEV).bfloat16()
    h2 = torch.randn(50, 3584, generator=g, device=DEV).bfloat16()
    assert hooks.encoder_store(enc, longer, m, kv2, h2, m.length)
    m.release()
    m = enc.match(longer)
    assert m.length == 350
    assert torch.equal(hooks.encoder_hit(enc, m, 350), torch.cat([hidden, h2]))
    m.release()


def test_full_hit_served_as_pages_feeds_the_paged_attention():
    """fill_from_pool(paged=True) on a page-mode pool: a full hit is not gathered; the attention over the
    PagedPrefix equals the attention over the per-layer caches the gathered path would have set."""
    import math

    from qwenedit_b200.attention import paged_attention

    pool = _pool(4000, 64)
    total = 640
    vids = np.arange(1, total + 1, dtype=np.int64)
    layers = _computed(total, 5)
    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [vids], [total])
    assert hooks.fill_from_pool(pool, caches, paged=True) == [0]
    caches[0] = layers
    hooks.store_computed(pool, caches, [0])
    caches.release()
    gathers = pool.stats.gathers
    caches = hooks.MTCaches([[LayerCache() for _ in range(L)]], [vids], [total])
    assert hooks.fill_from_pool(pool, caches, paged=True) == []
    assert pool.stats.gathers == gathers and pool.stats.contiguous_views == 0  # nothing gathered
    prefix = caches.paged[0]
    g = torch.Generator(device=DEV).manual_seed(6)
    q, k, v = (torch.randn(256, H, D, generator=g, device=DEV).bfloat16() for _ in range(3))
    for layer in (0, L - 1):
        out = paged_attention(q, prefix, layer, k, v)
        keys = torch.cat([layers[layer]["key"][0], k]).float().transpose(0, 1)
        values = torch.cat([layers[layer]["value"][0], v]).float().transpose(0, 1)
        s = q.float().transpose(0, 1) @ keys.transpose(1, 2) / math.sqrt(D)
        ref = (torch.softmax(s, dim=-1) @ values).transpose(0, 1)
        assert (out.float() - ref).abs().max().item() < 2e-2
    caches.release()
    assert pool.usage()["protected"] == 0
    with pytest.raises(ValueError, match="page-mode"):
        hooks.fill_from_pool(_pool(100), hooks.MTCaches([[LayerCache()]], [vids[:10]], [10]), paged=True)
