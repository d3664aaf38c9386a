"""The 2K multi-turn workload under memory pressure, at full token counts: 8 sessions x 5 turns of a
16,384 + 512-token DiT prefix in a 24 GiB pool (room for two prefixes), plus 1,024-token prompts in a 4 GiB
encoder pool. Forced LRU eviction; the native index must make the same decisions as the oracle restatement
(match lengths, evicted token counts, allocated slots, usage) at every step. Index-only (meta device), CPU."""

import numpy as np
import pytest
import torch

from oracle.pool_ref import RefPagedKVPool
from qwenedit_b200.paged import PagedKVPool

GIB = 1 << 30
DIT = dict(layers=60, heads=24, head_dim=128)
ENC = dict(layers=28, heads=4, head_dim=128, extra=3584)


def _pools(kind, page):
    if kind == "dit":
        args = ("dit", DIT["layers"], DIT["heads"], DIT["head_dim"], 24 * GIB, torch.bfloat16)
        extra = 0
    else:
        args = ("encoder", ENC["layers"], ENC["heads"], ENC["head_dim"], 4 * GIB, torch.bfloat16)
        extra = ENC["extra"]
    ours = PagedKVPool(*args, "meta", extra_dim=extra, page_size=page)
    ref = RefPagedKVPool(*args, extra_dim=extra, page_size=page, allocate=False)
    return ours, ref


def _slots(t):
    return t._qe_host if hasattr(t, "_qe_host") else t.numpy()


def _turn(pool, vids):
    """One request through the pool: match, allocate the uncached tail, insert, release (hooks.py:95-112)."""
    m = pool.match(vids)
    n = len(vids) - m.length
    slots = pool.alloc(n)
    if slots is not None:
        idx = np.concatenate([_slots(m.indices), _slots(slots)]) if m.length else _slots(slots)
        t = torch.from_numpy(idx.copy())
        t._qe_host = t.numpy()
        pool.insert(vids, t, owned_from=m.length)
    m.release()
    return m.length, None if slots is None else _slots(slots).copy()


def _sessions(seed, text, image, turns, sessions):
    """Per session: a shared text header then a new conditioning image per turn (the previous output)."""
    rng = np.random.default_rng(seed)
    out = []
    for s in range(sessions):
        header = rng.integers(1, 1 << 62, size=text)
        out.append([np.concatenate([header, rng.integers(1, 1 << 62, size=image)]) for _ in range(turns)])
    return out


@pytest.mark.parametrize("page", [1, 64])
def test_dit_pool_2k_sessions_evict_identically(page):
    ours, ref = _pools("dit", page)
    assert ours.capacity == ref.capacity
    assert ours.capacity // (16384 + 512) == 2  # only two 2K prefixes fit: every turn evicts
    sess = _sessions(7, 512, 16384, 5, 8)
    rng = np.random.default_rng(3)
    order = [(s, t) for t in range(5) for s in rng.permutation(8)]
    for step, (s, t) in enumerate(order):
        a, b = _turn(ours, sess[s][t]), _turn(ref, sess[s][t])
        assert a[0] == b[0], step
        assert (a[1] is None) == (b[1] is None), step
        if a[1] is not None:
            np.testing.assert_array_equal(a[1], b[1])
        assert ours.usage() == ref.usage(), step
    assert ours.usage()["evicted_tokens"] > 30 * (16384 + 512) * 0.9
    # which prefixes survived: identical
    for s in range(8):
        for t in range(5):
            mo, mr = ours.match(sess[s][t]), ref.match(sess[s][t])
            assert mo.length == mr.length
            mo.release()
            mr.release()


@pytest.mark.parametrize("page", [1, 16])
def test_encoder_pool_prompts_identically(page):
    ours, ref = _pools("encoder", page)
    rng = np.random.default_rng(11)
    system = rng.integers(1, 1 << 62, size=180)  # shared system template
    prompts = [np.concatenate([system, rng.integers(1, 1 << 62, size=1024 - 180)]) for _ in range(80)]
    # 8 sessions x 5 turns, each turn re-sends its session's previous prompt plus edits (partial reuse)
    for step in range(120):
        p = prompts[int(rng.integers(len(prompts)))]
        if rng.random() < 0.3:
            p = np.concatenate([p[: int(rng.integers(200, 1000))], rng.integers(1, 1 << 62, size=64)])
        a, b = _turn(ours, p), _turn(ref, p)
        assert a[0] == b[0], step
        if a[1] is not None:
            np.testing.assert_array_equal(a[1], b[1])
        assert ours.usage() == ref.usage(), step
