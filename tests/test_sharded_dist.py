"""Head-sharded pools, host side, as 2 gloo ranks on CPU: the replicated prefix index gives every rank the same
slots for the same operation sequence, `verify_replicas` passes then, and fails on every rank as soon as one
rank performs an operation the other did not (the failure is raised on the host before any data moves)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ops(pool, rng, rounds):
    """A session's turns: match the prefix, allocate the new tokens, insert; the same on every rank."""
    slots_seen = []
    base = rng.integers(1, 1 << 62, size=64)
    for t in range(rounds):
        vids = np.concatenate([base, rng.integers(1, 1 << 62, size=int(rng.integers(8, 40)))])
        m = pool.match(vids)
        new = pool.alloc(len(vids) - m.length)
        if new is not None:
            idx = np.concatenate([m.indices._qe_host, new._qe_host]) if m.length else new._qe_host
            ti = torch.from_numpy(idx.copy())
            ti._qe_host = ti.numpy()
            pool.insert(vids, ti, owned_from=m.length)
            slots_seen.append(idx.tolist())
        m.release()
    return slots_seen


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qwenedit_b200.paged import PagedKVPool
        from qwenedit_b200.sharded import exchange, verify_replicas

        # each rank's share of a 24-head pool: 12 heads, small budget so that eviction runs
        pool = PagedKVPool("dit-shard", 2, 24 // world, 8, 600 * 2 * 2 * (24 // world) * 8 * 2, torch.bfloat16,
                           "meta", page_size=4)
        rng = np.random.default_rng(7)  # the request stream is global: same on every rank
        slots = _ops(pool, rng, 40)
        verify_replicas(pool)  # must pass
        all_slots = exchange(slots)
        same = all(s == all_slots[0] for s in all_slots)
        # rank 1 performs one extra operation: every rank must see the divergence
        if rank == 1:
            pool.alloc(4)
        try:
            verify_replicas(pool)
            diverged = False
        except RuntimeError:
            diverged = True
        result_q.put({"rank": rank, "same_slots": same, "evicted": pool.usage()["evicted_tokens"],
                      "diverged_detected": diverged})
    finally:
        dist.destroy_process_group()


def test_replicated_index_and_divergence_detection():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r["same_slots"] for r in results)
    assert all(r["evicted"] > 0 for r in results)  # the op stream ran the LRU eviction
    assert all(r["diverged_detected"] for r in results)


if __name__ == "__main__":
    pytest.main([__file__, "-q"])
