"""The native prefix index (radix tree + allocator + LRU eviction, host C++) against the oracle restatement,
operation for operation, through the pool API the reference callers use (paged.py:72-131). CPU only: the
pools are created on the meta device, so only the host index runs."""

import numpy as np
import pytest
import torch

from oracle.pool_ref import RefPagedKVPool
from qwenedit_b200.paged import PagedKVPool

L, H, D = 2, 1, 4
PER_TOKEN = L * 2 * H * D * 2  # bf16


def pools(tokens, page=1):
    ours = PagedKVPool("t", L, H, D, tokens * PER_TOKEN, torch.bfloat16, "meta", page_size=page)
    ref = RefPagedKVPool("t", L, H, D, tokens * PER_TOKEN, torch.bfloat16, page_size=page, allocate=False)
    return ours, ref


def slots_of(t):
    return t._qe_host if hasattr(t, "_qe_host") else t.numpy()


def same_usage(ours, ref):
    u, r = ours.usage(), ref.usage()
    assert u == r, (u, r)


def fill(pool, vids, owned_from_zero=False):
    """The reference callers' flow (tests/test_paged.py:21-29, hooks.py:108-111): match, alloc the tail,
    insert, release. With owned_from_zero the caller allocates the whole prefix (hooks.py:133-139)."""
    match = pool.match(vids)
    m = match.length
    if owned_from_zero:
        slots = pool.alloc(len(vids))
        if slots is not None:
            pool.insert(vids, slots, owned_from=0)
    else:
        slots = pool.alloc(len(vids) - m)
        if slots is not None:
            idx = np.concatenate([slots_of(match.indices), slots_of(slots)]) if m else slots_of(slots)
            t = torch.from_numpy(idx.copy())
            t._qe_host = t.numpy()
            pool.insert(vids, t, owned_from=m)
    match.release()
    return m, (None if slots is None else slots_of(slots))


def test_reference_scenario_match_extends():
    """tests/test_paged.py:28-42 at the index level."""
    for pool in pools(64):
        a = np.arange(1, 9, dtype=np.int64)
        fill(pool, a)
        b = np.concatenate([a[:5], [100, 101]])
        m = pool.match(b)
        assert m.length == 5
        m.release()
        fill(pool, b)
        m = pool.match(b)
        assert m.length == 7
        m.release()


def test_reference_scenario_eviction_respects_locks():
    """tests/test_paged.py:45-55: a held match blocks eviction; after release a new fill evicts >= 6 tokens."""
    for pool in pools(16):
        a = np.arange(1, 11, dtype=np.int64)
        fill(pool, a)
        held = pool.match(a)
        assert pool.alloc(10) is None or pool.match(a).length == 10
        held.release()
        fill(pool, np.arange(1000, 1012, dtype=np.int64))
        m = pool.match(a)
        assert m.length < 10
        m.release()
        assert pool.usage()["evicted_tokens"] >= 6


def test_alloc_returns_none_never_raises():
    ours, ref = pools(32)
    for pool in (ours, ref):
        assert pool.alloc(33) is None
        assert pool.alloc(32) is not None
        assert pool.alloc(1) is None
    same_usage(ours, ref)


@pytest.mark.parametrize("page", [1, 4, 16])
@pytest.mark.parametrize("seed", range(6))
def test_random_sessions_match_oracle(page, seed):
    rng = np.random.default_rng(seed * 7 + page)
    cap = int(rng.integers(200, 600)) // page * page
    ours, ref = pools(cap, page)
    sessions = [list(rng.integers(1, 1 << 40, size=int(rng.integers(20, 120)))) for _ in range(6)]
    held = []
    for step in range(250):
        s = int(rng.integers(len(sessions)))
        base = sessions[s]
        kind = rng.random()
        if kind < 0.35:  # a new turn extends the session
            base = base + list(rng.integers(1, 1 << 40, size=int(rng.integers(1, 60))))
            sessions[s] = base
            vids = np.asarray(base, np.int64)
        elif kind < 0.55:  # an edit diverges part way
            cut = int(rng.integers(1, len(base)))
            vids = np.asarray(base[:cut] + list(rng.integers(1, 1 << 40, size=int(rng.integers(1, 40)))), np.int64)
        else:
            vids = np.asarray(base, np.int64)
        op = rng.random()
        if op < 0.12 and len(held) < 4:  # hold a lock across later operations
            mo, mr = ours.match(vids), ref.match(vids)
            assert mo.length == mr.length
            if mo.length:
                np.testing.assert_array_equal(mo.indices._qe_host, mr.indices.numpy())
            held.append((mo, mr))
        elif op < 0.2 and held:
            mo, mr = held.pop(int(rng.integers(len(held))))
            mo.release(), mr.release()
            mo.release(), mr.release()  # idempotent
        else:
            zero = op > 0.9
            ro = fill(ours, vids, zero)
            rr = fill(ref, vids, zero)
            assert ro[0] == rr[0], step
            if ro[1] is None or rr[1] is None:
                assert ro[1] is None and rr[1] is None, step
            else:
                np.testing.assert_array_equal(ro[1], rr[1])
        same_usage(ours, ref)
        if step % 50 == 0:
            assert ours.index.usage()["nodes"] == ref.tree.node_count()
    for mo, mr in held:
        mo.release(), mr.release()
    same_usage(ours, ref)
    assert ours.usage()["protected"] == 0


def _ref_pool(tokens, resolution):
    return RefPagedKVPool("t", L, H, D, tokens * PER_TOKEN, torch.bfloat16, allocate=False,
                          clock_resolution=resolution)


def _lockstep(resolution, seed):
    """The oracle with a logical and with a coarse clock on one workload: the step at which their results first
    differ (None if never), and whether an eviction of the coarse one chose between tied leaves before that."""
    rng = np.random.default_rng(100 + seed)
    cap = int(rng.integers(150, 400))
    logical, coarse = _ref_pool(cap, 1), _ref_pool(cap, resolution)
    sessions = [list(rng.integers(1, 1 << 40, size=int(rng.integers(20, 90)))) for _ in range(6)]
    for step in range(300):
        s = int(rng.integers(len(sessions)))
        if rng.random() < 0.4:
            sessions[s] = sessions[s] + list(rng.integers(1, 1 << 40, size=int(rng.integers(1, 50))))
        vids = np.asarray(sessions[s], np.int64)
        a, b = fill(logical, vids), fill(coarse, vids)
        same = a[0] == b[0] and (a[1] is None) == (b[1] is None) and (a[1] is None or np.array_equal(a[1], b[1]))
        if not same or logical.usage() != coarse.usage():
            return step, coarse.tree.tie_seen
    assert not logical.tree.tie_seen  # the logical clock never ties two leaves
    return None, coarse.tree.tie_seen


@pytest.mark.parametrize("resolution", [2, 7, 50])
@pytest.mark.parametrize("seed", range(4))
def test_coarse_clock_diverges_only_through_ties(resolution, seed):
    """SGLang stamps nodes with time.monotonic(); the oracle and the native index use a logical clock (every read a
    new tick). Under a clock too coarse to separate reads, leaves can tie on last-access time and the eviction heap's
    layout (heapq's sift order) picks the victim. The two agree at every operation until an eviction has had to
    choose between tied leaves."""
    step, tied = _lockstep(resolution, seed)
    if step is not None:
        assert tied, f"diverged at step {step} without a tied eviction"


def test_coarse_clock_does_change_eviction_order():
    """The divergence is real: with 7 or 50 reads per clock value every workload above diverges (after a tie),
    so eviction order matches SGLang's only while its clock separates the reads, which the logical clock assumes."""
    for resolution in (7, 50):
        for seed in range(4):
            step, tied = _lockstep(resolution, seed)
            assert step is not None and tied


def test_page_mode_truncates_and_frees_tail_pages():
    ours, ref = pools(64, page=16)
    for pool in (ours, ref):
        vids = np.arange(1, 41, dtype=np.int64)  # 2 whole pages + 8 tokens
        m, slots = fill(pool, vids)
        assert m == 0 and len(slots) == 40
        assert pool.usage()["free"] == 64 - 32  # the partial third page went back
        mm = pool.match(vids)
        assert mm.length == 32
        mm.release()
        mm = pool.match(vids[:20])
        assert mm.length == 16
        mm.release()
    same_usage(ours, ref)


def test_misuse_raises():
    ours, _ = pools(32)
    m = ours.match(np.arange(1, 5))
    assert m.length == 0 and m.indices is None and m.node is None
    fill(ours, np.arange(1, 5))
    m = ours.match(np.arange(1, 5))
    m.release()
    with pytest.raises(ValueError):
        ours.index.unlock(12345)
    with pytest.raises(Exception, match="out of range or already free"):
        ours.index.free(np.array([999999], np.int64))
    before = ours.usage()
    for bad in (0, -3, 33, 999999):  # slot 0 is padding; this pool's slots are 1 .. 32
        with pytest.raises(ValueError, match="outside"):
            ours.index.insert(np.arange(100, 104), np.array([5, 6, bad, 7], np.int64))
    assert ours.usage() == before and ours.match(np.arange(100, 104)).length == 0


def test_clear_resets_everything():
    ours, ref = pools(64)
    for pool in (ours, ref):
        fill(pool, np.arange(1, 30))
        pool.clear()
        assert pool.usage()["free"] == 64 and pool.usage()["evictable"] == 0
        assert pool.match(np.arange(1, 30)).length == 0
