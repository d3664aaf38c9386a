"""Session partition across ranks (the multi-GPU layout), exercised as 2 gloo ranks on CPU: every session is
served by exactly one rank, every rank computes the same partition, and each rank's pool only ever holds its
own sessions' prefixes (index-only pools on the meta device)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwenedit_b200.sessions import SessionRouter, owner


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qwenedit_b200.paged import PagedKVPool

        router = SessionRouter(rank, world)
        sessions = [f"session-{i}" for i in range(64)]
        mine = router.mine(sessions)
        pool = PagedKVPool("dit", 2, 1, 4, 4096 * 16, torch.bfloat16, "meta")
        rng = np.random.default_rng(0)  # same stream on every rank: the request sequence is global
        served = 0
        for _ in range(200):
            sid = sessions[int(rng.integers(len(sessions)))]
            vids = np.frombuffer(sid.encode().ljust(16, b"_"), dtype=np.int64).copy()
            vids = np.concatenate([vids, np.arange(1, 20, dtype=np.int64)])
            if not router.owns(sid):
                continue
            m = pool.match(vids)
            slots = pool.alloc(len(vids) - m.length)
            if slots is not None:
                import torch as _t

                idx = np.concatenate([m.indices._qe_host, slots._qe_host]) if m.length else slots._qe_host
                t = _t.from_numpy(idx.copy())
                t._qe_host = t.numpy()
                pool.insert(vids, t, owned_from=m.length)
            m.release()
            served += 1
        counts = [None] * world
        dist.all_gather_object(counts, {"rank": rank, "mine": mine, "served": served,
                                        "partition": router.partition(sessions)})
        if rank == 0:
            result_q.put(counts)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_ranks_partition_sessions_without_overlap():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    counts = q.get(timeout=100)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    mine = [set(c["mine"]) for c in counts]
    assert mine[0].isdisjoint(mine[1])
    assert mine[0] | mine[1] == {f"session-{i}" for i in range(64)}
    assert counts[0]["partition"] == counts[1]["partition"]  # same partition computed on both ranks
    assert sum(c["served"] for c in counts) == 200
    assert all(len(m) > 10 for m in mine)  # the hash spreads sessions


def test_owner_is_stable_and_in_range():
    assert owner("abc", 1) == 0
    assert all(0 <= owner(f"s{i}", 8) < 8 for i in range(100))
    assert owner("session-17", 8) == owner("session-17", 8)
    with pytest.raises(ValueError):
        owner("x", 0)
