"""Host logic of the pool call sites (qwenedit_b200.hooks) on CPU, over the oracle's reference-semantics pool.

The reference's `_fill_from_pool` / `_store_computed` (multi_turn/pipeline/hooks.py:86-139) and the encoder pool
branches (multi_turn/cache/encoder.py:111-138) decide per sample between a full hit (gather, keep the lock), a
partial hit of at least MULTI_TURN_MIN_REUSE tokens (gather the head, prefill the tail, append it, release), and a
miss (release, recompute, store after the forward). These tests drive the product's hooks through every branch
with `oracle.pool_ref.RefPagedKVPool` (the reference pool's behaviour, CPU tensors) standing in for the device
pool; the adapter below adds the two entry points the product's pool has beyond the reference's (`gather_into`,
`write_layers`) with the reference's own torch calls. The kernels behind them are checked on the GPU elsewhere.
"""

import torch

from oracle.pool_ref import RefPagedKVPool
from qwenedit_b200 import hooks, state

L, H, D = 2, 2, 4


class _Pool(RefPagedKVPool):
    """Reference pool plus the product pool's extra entry points, each as the reference's own torch calls."""

    def gather_into(self, indices, out):
        out.copy_(self.gather(indices))

    def write_layers(self, slots, keys, values):  # hooks.py:136-138, one index_copy_ per layer and K/V
        for index, (k, v) in enumerate(zip(keys, values)):
            self.kv[index, 0].index_copy_(0, slots, k)
            self.kv[index, 1].index_copy_(0, slots, v)

    def gather_extra(self, indices):  # encoder.py:114
        return self.extra.index_select(0, indices)

    def write_extra(self, slots, hidden):  # encoder.py:136
        self.extra.index_copy_(0, slots, hidden.to(self.extra.dtype))


def _pool(tokens=200, extra=0):
    per_token = (L * 2 * H * D + extra) * 4
    pool = _Pool("dit", L, H, D, tokens * per_token, torch.float32, extra_dim=extra)
    pool.kv.zero_()
    return pool


def _vids(n, base=1000):
    return torch.arange(base, base + n, dtype=torch.int64).numpy()


def _request(vids_list):
    """MTCaches with one dict per layer (a per-layer cache: `update(key=, value=)` and ["key"] / ["value"])."""
    caches = [[{} for _ in range(L)] for _ in vids_list]
    lengths = [0 if v is None else len(v) for v in vids_list]
    return hooks.MTCaches(caches, vids_list, lengths)


def _forward(caches, sample, seed):
    """What the DiT forward leaves in the caches after a miss: per layer [1, n, H, D] K and V."""
    g = torch.Generator().manual_seed(seed)
    n = caches.prefix_lengths[sample]
    for layer in caches[sample]:
        layer.update(key=torch.randn(1, n, H, D, generator=g), value=torch.randn(1, n, H, D, generator=g))


def _stacked(caches, sample):
    """[L, 2, n, H, D] of what the caches of `sample` point at."""
    return torch.stack([torch.stack([c["key"][0], c["value"][0]]) for c in caches[sample]])


def test_miss_then_store_then_full_hit(monkeypatch):
    monkeypatch.setattr(state, "MIN_REUSE", 8)
    pool, a = _pool(), _vids(40)
    req = _request([a, None])
    assert hooks.fill_from_pool(pool, req) == [0]  # a miss; the None sample is skipped
    assert req.matches == [] and pool.usage()["protected"] == 0
    _forward(req, 0, seed=1)
    stored = _stacked(req, 0)
    hooks.store_computed(pool, req, [0])
    assert pool.usage()["inserted_tokens"] == 40

    hit = _request([a])
    assert hooks.fill_from_pool(pool, hit) == []
    assert torch.equal(_stacked(hit, 0), stored)
    assert len(hit.matches) == 1 and pool.usage()["protected"] == 40  # the hit keeps its lock for the request
    hit.release()
    hit.release()  # idempotent
    assert hit.matches == [] and pool.usage()["protected"] == 0


def test_partial_hit_prefills_the_tail_and_stores_it(monkeypatch):
    monkeypatch.setattr(state, "MIN_REUSE", 8)
    pool, a = _pool(), _vids(40)
    req = _request([a])
    hooks.fill_from_pool(pool, req)
    _forward(req, 0, seed=2)
    head = _stacked(req, 0)
    hooks.store_computed(pool, req, [0])

    b = _vids(55)  # the same 40-token head, 15 new tokens
    tail = torch.randn(L, 2, 15, H, D, generator=torch.Generator().manual_seed(3))
    calls = []

    def prefill(sample, kv, start):
        calls.append((sample, kv.shape, start))
        assert torch.equal(kv[:, :, :start], head)  # the head was gathered before the tail is computed
        kv[:, :, start:] = tail

    part = _request([b])
    assert hooks.fill_from_pool(pool, part, prefill) == []
    assert calls == [(0, (L, 2, 55, H, D), 40)]
    assert torch.equal(_stacked(part, 0), torch.cat([head, tail], dim=2))
    assert part.matches == [] and pool.usage()["protected"] == 0  # released after the append
    assert pool.usage()["inserted_tokens"] == 55

    again = _request([b])  # the whole prefix is now a full hit with the same values
    assert hooks.fill_from_pool(pool, again) == []
    assert torch.equal(_stacked(again, 0), torch.cat([head, tail], dim=2))
    again.release()


def test_short_match_or_no_prefill_is_a_miss(monkeypatch):
    pool, a = _pool(), _vids(40)
    monkeypatch.setattr(state, "MIN_REUSE", 8)
    req = _request([a])
    hooks.fill_from_pool(pool, req)
    _forward(req, 0, seed=4)
    hooks.store_computed(pool, req, [0])

    monkeypatch.setattr(state, "MIN_REUSE", 64)  # a 40-token head is too short to reuse
    short = _request([_vids(60)])
    assert hooks.fill_from_pool(pool, short, lambda *a: None) == [0]
    assert pool.usage()["protected"] == 0

    monkeypatch.setattr(state, "MIN_REUSE", 8)  # long enough, but no tail prefill to run
    assert hooks.fill_from_pool(pool, _request([_vids(60)]), None) == [0]
    assert pool.usage()["protected"] == 0


def test_store_skips_empty_caches_and_a_full_pool(monkeypatch):
    monkeypatch.setattr(state, "MIN_REUSE", 8)
    pool = _pool(tokens=64)
    req = _request([_vids(40), _vids(30, base=5000)])
    assert hooks.fill_from_pool(pool, req) == [0, 1]
    _forward(req, 0, seed=5)  # sample 1 was never computed: its caches stay empty
    hooks.store_computed(pool, req, [0, 1])
    assert pool.usage()["inserted_tokens"] == 40

    held = _request([_vids(40)])  # lock the 40 stored tokens so nothing can be evicted
    hooks.fill_from_pool(pool, held)
    big = _request([_vids(30, base=9000)])
    hooks.fill_from_pool(pool, big)
    _forward(big, 0, seed=6)
    hooks.store_computed(pool, big, [0])  # 24 free tokens for 30: alloc returns None, nothing raises
    assert pool.usage()["inserted_tokens"] == 40
    held.release()


def test_encoder_store_and_hit():
    hidden = 6
    pool = _Pool("encoder", L, H, D, 100 * (L * 2 * H * D + hidden) * 4, torch.float32, extra_dim=hidden)
    pool.kv.zero_()
    pool.extra.zero_()
    v = _vids(12)
    first = pool.match(v)
    assert hooks.encoder_hit(pool, first, 12) is None
    kv = torch.randn(L, 2, 12, H, D, generator=torch.Generator().manual_seed(7))
    rows = torch.randn(12, hidden, generator=torch.Generator().manual_seed(8))
    first.release()
    assert hooks.encoder_store(pool, v, None, kv, rows, 0)
    m = pool.match(v)
    assert torch.equal(hooks.encoder_hit(pool, m, 12), rows)
    assert torch.equal(pool.gather(m.indices), kv)
    m.release()

    longer = _vids(16)  # a partial hit: the 4 new tokens are appended after the 12 cached ones
    m = pool.match(longer)
    assert m.length == 12 and hooks.encoder_hit(pool, m, 16) is None
    kv4 = torch.randn(L, 2, 4, H, D, generator=torch.Generator().manual_seed(9))
    rows4 = torch.randn(4, hidden, generator=torch.Generator().manual_seed(10))
    assert hooks.encoder_store(pool, longer, m, kv4, rows4, 12)
    m.release()
    full = pool.match(longer)
    assert torch.equal(hooks.encoder_hit(pool, full, 16), torch.cat([rows, rows4]))
    full.release()
