"""Head-sharded pools on 2 GPUs (one process per GPU, NCCL): the fused scatter-append writes each rank's token
slice into every owner's pool over NVLink, and every rank's local gather then returns exactly its heads of the
full K/V (bit-exact against the same rows computed on the host). Also the tensor-parallel form (each rank writes
its own heads) and the out-of-range slot flag. Skipped on a box with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_kv(L, n, H, D, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(L, 2, n, H, D, generator=g).bfloat16()


def _worker(rank, world, port, page_size, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    out = {"rank": rank}
    try:
        import numpy as np

        from qwenedit_b200.sharded import HeadShardedKVPool

        L, H, D, n = 4, 8, 64, 1000
        dev = torch.device("cuda", rank)
        pool = HeadShardedKVPool("shard", L, H, D, 16 << 20, torch.bfloat16, dev, page_size=page_size)
        pool.pool.index.shuffle_free(3)  # scattered slots (same seed on every rank: replicated decisions)
        vids = np.arange(1, n + 1, dtype=np.int64)
        slots = pool.alloc(n)
        full = _full_kv(L, n, H, D, seed=11)
        hs = slice(pool.head_start, pool.head_start + pool.heads_local)
        # sequence parallel: rank r holds tokens [r n/2, (r+1) n/2) with all heads
        lo, hi = rank * n // world, (rank + 1) * n // world
        pool.write_scatter(slots[lo:hi], full[:, :, lo:hi].to(dev))
        pool.barrier()
        pool.insert(vids, slots, owned_from=0)
        pool.verify_replicas()
        m = pool.match(vids)
        cached = n // page_size * page_size  # page mode keeps whole pages only
        got = pool.gather(m.indices).cpu()
        out["scatter_exact"] = m.length == cached and bool(torch.equal(got, full[:, :, :cached, hs]))
        m.release()
        out["errors_clean"] = pool.device_errors() == 0
        # tensor parallel: each rank writes its own heads of a second prefix
        vids2 = np.arange(5000, 5000 + 300, dtype=np.int64)
        slots2 = pool.alloc(300)
        full2 = _full_kv(L, 300, H, D, seed=12)
        pool.write(slots2, full2[:, :, :, hs].contiguous().to(dev))
        pool.insert(vids2, slots2, owned_from=0)
        m2 = pool.match(vids2)
        c2 = 300 // page_size * page_size
        out["local_exact"] = m2.length == c2 and bool(torch.equal(pool.gather(m2.indices).cpu(), full2[:, :, :c2, hs]))
        m2.release()
        # an out-of-range slot is skipped and flagged, not written
        bad = torch.tensor([pool.pool.rows + 5], dtype=torch.int64, device=dev)
        pool.write_scatter(bad, full[:, :, :1].to(dev))
        pool.barrier()
        out["bad_slot_flagged"] = pool.device_errors() != 0
        out["nvlink_bytes"] = pool.nvlink_bytes
        pool.close()
    except Exception as exc:  # reported to the parent; every rank still leaves the group
        out["error"] = repr(exc)
    finally:
        dist.destroy_process_group()
        result_q.put(out)


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("page_size", [1, 64])
def test_head_sharded_scatter_and_gather(page_size):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, page_size, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=300) for _ in procs), key=lambda r: r["rank"])
    for p in procs:
        p.join(timeout=60)
    for r in results:
        assert "error" not in r, r
        assert r["scatter_exact"] and r["local_exact"] and r["errors_clean"] and r["bad_slot_flagged"], r
        # each rank sent the other rank's half of its token slice: L * 2 * (n/2) * (H/2) * D * 2 bytes
        assert r["nvlink_bytes"] == 4 * 2 * 500 * 4 * 64 * 2 + 4 * 2 * 1 * 4 * 64 * 2
