"""Paged K/V gather / append on the GPU against the oracle (the reference's index_select / index_copy_ on CPU),
bit for bit; the reference's own pool tests (tests/test_paged.py:28-65) replayed on CUDA; the CPU
round-trip config; and size-independent properties at the 1K-edit shapes."""

import numpy as np
import pytest
import torch

from oracle.pool_ref import RefPagedKVPool
from qwenedit_b200.paged import PagedKVPool
from tests.golden import inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True, params=["warp", "warp_row", "warp16", "bulk"])
def copy_kernel(request):
    """Run every test with every paged-copy kernel (vectorised warp copy with 256-bit vectors where aligned,
    several short rows per warp pass or one row per pass, 16-byte vectors only, TMA bulk pipeline)."""
    from qwenedit_b200.paged import set_copy_mode

    set_copy_mode(request.param)
    yield request.param
    set_copy_mode("auto")


def _pool(L, H, D, tokens, dtype, page=1, extra=0, seed=0):
    elem = torch.empty((), dtype=dtype).element_size()
    budget = tokens * (L * 2 * H * D + extra) * elem
    pool = PagedKVPool("t", L, H, D, budget, dtype, DEV, extra_dim=extra, page_size=page)
    pool.kv.copy_(inputs.f32(seed, tuple(pool.kv.shape)).to(dtype))
    if extra:
        pool.extra.copy_(inputs.f32(seed + 9, tuple(pool.extra.shape)).to(dtype))
    return pool


def _slots(seed, n, rows, start=1):
    return torch.from_numpy(inputs.permutation(seed, rows - start)[:n] + start)


@pytest.mark.parametrize("L,H,D,dtype", [(2, 2, 8, torch.float32), (4, 24, 128, torch.float32),
                                         (3, 4, 128, torch.bfloat16), (5, 3, 5, torch.bfloat16),
                                         (2, 1, 2, torch.float32)])
def test_gather_slots_bit_exact(L, H, D, dtype):
    pool = _pool(L, H, D, 700, dtype, seed=L * 100 + H)
    idx = _slots(7, 500, pool.rows, start=0)
    got = pool.gather(idx.to(DEV))
    ref = pool.kv.cpu().index_select(2, idx)
    assert got.shape == ref.shape and torch.equal(got.cpu(), ref)
    assert pool.stats.gathers == 1 and pool.device_errors() == 0


@pytest.mark.parametrize("page", [4, 16, 64])
def test_gather_through_block_table_bit_exact(page):
    pool = _pool(3, 24, 128, 64 * 40, torch.bfloat16, page=page, seed=page)
    pool.index.shuffle_free(page)  # scattered pages: a real gather, not the contiguous-run view
    m = pool.match(np.arange(1, 10))
    assert m.length == 0
    n = page * 23 + page // 2  # a partial last page
    slots = pool.alloc(n)
    host = slots._qe_host
    assert np.array_equal(host[page:2 * page] // page, np.full(page, host[page] // page))
    out = pool.gather(slots)
    assert getattr(slots, "_qe_pages", None) is not None  # the block-table kernel ran
    ref = pool.kv.cpu().index_select(2, torch.from_numpy(host))
    assert torch.equal(out.cpu(), ref)


@pytest.mark.parametrize("H,page", [(3, 64), (6, 64), (12, 16), (4, 1), (1, 1), (24, 64)])
def test_short_rows_gather_and_append(H, page):
    """Row sizes of the head-sharded DiT pools (3 / 6 / 12 of 24 heads: 768 B - 3 KiB), the encoder (4 heads, 1 KiB)
    and tiny rows, through block tables and slot lists, with a token count that is no multiple of the rows moved
    per warp pass."""
    L, D = 3, 128
    pool = _pool(L, H, D, 64 * 30, torch.bfloat16, page=page, seed=H * 7 + page)
    pool.index.shuffle_free(H + page)
    n = 64 * 11 + 37
    slots = pool.alloc(n)
    new = inputs.f32(H + 3, (L, 2, n, H, D)).to(torch.bfloat16)
    pool.write(slots, new.to(DEV))
    ref = pool.kv.cpu().clone()
    ref.index_copy_(2, torch.from_numpy(slots._qe_host), new)
    assert torch.equal(pool.kv.cpu(), ref)
    out = pool.gather(slots)
    assert torch.equal(out.cpu(), new) and pool.device_errors() == 0


@pytest.mark.parametrize("H,D,page", [(4, 128, 1), (24, 128, 64), (3, 64, 1), (1, 8, 4)])
def test_gather_heads_is_transposed_gather_with_room(H, D, page):
    """gather_heads == index_select then [L, 2, H, n, D] with `length - n` free positions; and the encoder's
    per-layer transpose + cat of the prefix with a tail (encoder.py:178-180) equals the buffer with the tail
    written in place."""
    L = 3
    pool = _pool(L, H, D, 64 * 20, torch.bfloat16, page=page, seed=H + D)
    pool.index.shuffle_free(H * D)
    m, n = 333, 45
    idx = pool.alloc(m)
    buf = pool.gather_heads(idx, m + n)
    assert buf.shape == (L, 2, H, m + n, D) and pool.device_errors() == 0
    ref = pool.kv.cpu().index_select(2, torch.from_numpy(idx._qe_host)).permute(0, 1, 3, 2, 4)
    assert torch.equal(buf[:, :, :, :m].cpu(), ref)
    cached = pool.gather(idx)
    for layer in range(L):
        k = inputs.f32(layer, (1, H, n, D)).to(torch.bfloat16).to(DEV)
        want = torch.cat([cached[layer, 0].transpose(0, 1)[None], k], dim=2)
        buf[layer, 0, :, m:] = k[0]
        assert torch.equal(buf[layer, 0][None], want)


def test_contiguous_run_is_a_view():
    """tests/test_paged.py:58-65."""
    pool = PagedKVPool("t", 2, 1, 4, 64 * 32, torch.bfloat16, DEV)
    a = np.arange(1, 9, dtype=np.int64)
    _fill(pool, a, 1.0)
    m = pool.match(a)
    view = pool.gather(m.indices)
    assert view.data_ptr() == pool.kv[:, :, int(m.indices[0])].data_ptr()
    assert pool.stats.contiguous_views == 1
    m.release()


def _fill(pool, vids, value):
    match = pool.match(vids)
    n = len(vids) - match.length
    slots = pool.alloc(n)
    pool.write(slots, torch.full((2, 2, n, 1, 4), value, dtype=torch.bfloat16, device=DEV))
    idx = torch.cat([match.indices, slots]) if match.length else slots
    pool.insert(vids, idx, owned_from=match.length)
    match.release()


def test_reference_match_extends_and_reads_back():
    """tests/test_paged.py:28-42 on CUDA."""
    pool = PagedKVPool("t", 2, 1, 4, 64 * 32, torch.bfloat16, DEV)
    a = np.arange(1, 9, dtype=np.int64)
    _fill(pool, a, 1.0)
    b = np.concatenate([a[:5], [100, 101]])
    m = pool.match(b)
    assert m.length == 5 and torch.all(pool.gather(m.indices) == 1.0)
    m.release()
    _fill(pool, b, 2.0)
    m = pool.match(b)
    assert m.length == 7
    got = pool.gather(m.indices)
    assert torch.all(got[:, :, :5] == 1.0) and torch.all(got[:, :, 5:] == 2.0)
    m.release()


def test_reference_eviction_respects_locks():
    """tests/test_paged.py:45-55 on CUDA."""
    pool = PagedKVPool("t", 2, 1, 4, 16 * 32, torch.bfloat16, DEV)
    a = np.arange(1, 11, dtype=np.int64)
    _fill(pool, a, 1.0)
    held = pool.match(a)
    assert pool.alloc(10) is None or pool.match(a).length == 10
    held.release()
    _fill(pool, np.arange(1000, 1012, dtype=np.int64), 3.0)
    assert pool.match(a).length < 10
    assert pool.usage()["evicted_tokens"] >= 6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_write_bit_exact_with_strided_source(dtype):
    L, H, D = 4, 6, 64
    pool = _pool(L, H, D, 900, dtype, seed=3)
    ref = pool.kv.cpu().clone()
    total, m = 700, 180
    big = inputs.f32(5, (L, 2, total, H, D)).to(dtype).to(DEV)
    src = big[:, :, m:]  # hooks.py:110 writes kv[:, :, m:] of a larger tensor
    idx = _slots(11, total - m, pool.rows)
    pool.write(idx.to(DEV), src)
    ref.index_copy_(2, idx, src.cpu())
    assert torch.equal(pool.kv.cpu(), ref)
    # dtype conversion on the way in (paged.py:116 kv.to(self.kv.dtype))
    pool.write(idx.to(DEV), src.float() if dtype == torch.bfloat16 else src.double())
    assert torch.equal(pool.kv.cpu(), ref)


@pytest.mark.parametrize("page", [1, 64])
def test_write_through_block_table(page):
    pool = _pool(3, 24, 128, 64 * 30, torch.bfloat16, page=page, seed=4)
    n = 64 * 7 + 13
    slots = pool.alloc(n)
    new = inputs.f32(6, (3, 2, n, 24, 128)).bfloat16().to(DEV)
    ref = pool.kv.cpu().clone()
    pool._block_table(slots, slots._qe_host)
    pool.write(slots, new)
    ref.index_copy_(2, torch.from_numpy(slots._qe_host), new.cpu())
    assert torch.equal(pool.kv.cpu(), ref)


def test_write_layers_matches_per_layer_index_copy():
    """hooks.py:136-138 (2*L index_copy_) as one launch."""
    L, H, D = 6, 24, 128
    pool = _pool(L, H, D, 1000, torch.bfloat16, seed=8)
    n = 333
    idx = _slots(12, n, pool.rows)
    keys = [inputs.f32(100 + i, (n, H, D)).bfloat16().to(DEV) for i in range(L)]
    values = [inputs.f32(200 + i, (n, H, D)).bfloat16().to(DEV) for i in range(L)]
    ref = pool.kv.cpu().clone()
    pool.write_layers(idx.to(DEV), keys, values)
    for i in range(L):
        ref[i, 0].index_copy_(0, idx, keys[i].cpu())
        ref[i, 1].index_copy_(0, idx, values[i].cpu())
    torch.cuda.synchronize()
    assert torch.equal(pool.kv.cpu(), ref)


def test_pointer_append_skips_and_flags_a_misaligned_source():
    """qe_append_slots_ptrs through the C ABI with one source plane starting 2 bytes past a 16-byte boundary:
    the kernel sets bit 4 of the error flag and leaves that plane's pool rows untouched instead of issuing
    misaligned vector loads; every other plane equals the per-layer index_copy_."""
    from qwenedit_b200 import _lib

    L, H, D = 3, 24, 128
    pool = _pool(L, H, D, 600, torch.bfloat16, seed=31)
    n = 111
    idx = _slots(32, n, pool.rows)
    srcs = [inputs.f32(300 + i, (n, H, D)).bfloat16().to(DEV) for i in range(2 * L)]
    bad = 3  # layer 1, V
    buf = torch.empty(n * H * D + 1, dtype=torch.bfloat16, device=DEV)
    shifted = buf[1:].view(n, H, D)
    shifted.copy_(srcs[bad])
    assert shifted.data_ptr() % 16 == 2
    ptrs = [t.data_ptr() for t in srcs]
    ptrs[bad] = shifted.data_ptr()
    table = torch.tensor(ptrs, dtype=torch.int64, device=DEV)
    ref = pool.kv.cpu().clone()
    for p in range(2 * L):
        if p != bad:
            ref[p // 2, p % 2].index_copy_(0, idx, srcs[p].cpu())
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kv = pool.kv
    planes = _lib.planes(kv.data_ptr(), kv.stride(0) * 2, kv.stride(1) * 2, 2)
    _lib.call("qe_append_slots_ptrs", planes, pool.rows, table.data_ptr(), 2 * L, H * D * 2,
              idx.to(DEV).data_ptr(), n, err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert err.item() & 4
    assert torch.equal(pool.kv.cpu(), ref)


def test_encoder_extra_rows():
    """encoder.py:114 (extra.index_select) and :135 (extra.index_copy_); encoder geometry 28 x 4 x 128 + 3584."""
    pool = _pool(28, 4, 128, 300, torch.bfloat16, extra=3584, seed=9)
    idx = _slots(13, 200, pool.rows)
    got = pool.gather_extra(idx.to(DEV))
    assert torch.equal(got.cpu(), pool.extra.cpu().index_select(0, idx))
    rows = inputs.f32(14, (200, 3584)).bfloat16().to(DEV)
    ref = pool.extra.cpu().clone()
    pool.write_extra(idx.to(DEV), rows)
    ref.index_copy_(0, idx, rows.cpu())
    assert torch.equal(pool.extra.cpu(), ref)


def test_empty_and_single():
    pool = _pool(2, 2, 8, 50, torch.float32)
    out = pool.gather(torch.empty(0, dtype=torch.int64, device=DEV))
    assert out.shape == (2, 2, 0, 2, 8)
    one = pool.gather(torch.tensor([7], device=DEV))
    assert one.data_ptr() == pool.kv[:, :, 7].data_ptr()
    pool.write(torch.empty(0, dtype=torch.int64, device=DEV), torch.empty(2, 2, 0, 2, 8, device=DEV))


def test_out_of_range_slot_is_skipped_and_reported():
    pool = _pool(2, 2, 8, 50, torch.float32)
    bad = torch.tensor([3, pool.rows + 5, 4], device=DEV)
    out = pool.gather(bad)
    torch.cuda.synchronize()
    assert pool.device_errors() != 0
    assert torch.equal(out[:, :, 0].cpu(), pool.kv[:, :, 3].cpu())
    assert torch.equal(out[:, :, 2].cpu(), pool.kv[:, :, 4].cpu())
    assert pool.device_errors() == 0  # reading clears the flag


def _randn(seed, shape):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g)


def test_cpu_round_trip_config():
    """The CPU-sized round-trip workload (4 layers, 24 x 128, fp32 ~N(0,1), page 64, 512 pages; 3 sessions of 4096 image +
    256 text tokens; append one 4096-token turn each; gather each session) vs the oracle pool, bit-exact."""
    L, H, D, P = 4, 24, 128, 64
    budget = 512 * P * L * 2 * H * D * 4
    ours = PagedKVPool("c1", L, H, D, budget, torch.float32, DEV, page_size=P)
    ref = RefPagedKVPool("c1", L, H, D, budget, torch.float32, page_size=P)
    ours.kv.normal_(generator=torch.Generator(device=DEV).manual_seed(77))
    ref.kv.copy_(ours.kv.cpu())
    for s in range(3):
        prefix = np.arange(1, 4096 + 256 + 1, dtype=np.int64) + s * 10_000_000
        turn = np.concatenate([prefix, np.arange(1, 4097, dtype=np.int64) + s * 10_000_000 + 5_000_000])
        for vids, seed in ((prefix, 1000 + s), (turn, 2000 + s)):
            for pool in (ours, ref):
                m = pool.match(vids)
                n = len(vids) - m.length
                slots = pool.alloc(n)
                new = _randn(seed, (L, 2, n, H, D))
                pool.write(slots, new.to(DEV) if pool is ours else new)
                idx = torch.cat([m.indices.cpu(), slots.cpu()]) if m.length else slots.cpu()
                pool.insert(vids, idx, owned_from=m.length)
                m.release()
        got_m, want_m = ours.match(turn), ref.match(turn)
        assert got_m.length == want_m.length == len(turn) // P * P
        assert torch.equal(ours.gather(got_m.indices).cpu(), ref.gather(want_m.indices))
        got_m.release()
        want_m.release()
    assert ours.usage() == ref.usage()
    assert ours.device_errors() == 0


def test_one_k_edit_round_trip_property():
    """1K-edit shapes (60 layers, 24 x 128, bf16, 4608-token prefix, page 64, random page order): the gather equals
    the reference's own index_select on the device, and gather -> append into fresh pages -> gather is the identity."""
    L, H, D, P, T = 60, 24, 128, 64, 4608
    budget = 4 * T * L * 2 * H * D * 2
    pool = PagedKVPool("dit", L, H, D, budget, torch.bfloat16, DEV, page_size=P)
    pool.kv.normal_(generator=torch.Generator(device=DEV).manual_seed(0))
    pages = torch.from_numpy(inputs.permutation(3, pool.capacity // P)[: T // P] + 1)
    host = (pages[:, None] * P + torch.arange(P)).reshape(-1).numpy().copy()
    slots = torch.from_numpy(host).to(DEV)
    slots._qe_host = host
    a = pool.gather(slots)
    assert getattr(slots, "_qe_pages", None) is not None
    assert torch.equal(a, pool.kv.index_select(2, slots))
    fresh = pool.alloc(T)
    pool.write(fresh, a)
    assert torch.equal(pool.gather(fresh), a)
    assert pool.device_errors() == 0


def test_memory_pressure_data_matches_oracle():
    """2K-session turns in a pool that holds two prefixes (LRU eviction every turn), 2 of the 60 layers:
    after every turn each session's cached prefix gathers to exactly what the oracle pool holds."""
    L, H, D, P = 2, 24, 128, 64
    prefix = 16384 + 512
    budget = (2 * prefix + 3 * P) * L * 2 * H * D * 2
    ours = PagedKVPool("dit", L, H, D, budget, torch.bfloat16, DEV, page_size=P)
    ref = RefPagedKVPool("dit", L, H, D, budget, torch.bfloat16, page_size=P)
    ours.kv.zero_()
    ref.kv.zero_()
    rng = np.random.default_rng(5)
    headers = [rng.integers(1, 1 << 62, size=512) for _ in range(4)]
    for step in range(10):
        s = step % 4
        vids = np.concatenate([headers[s], rng.integers(1, 1 << 62, size=16384)])
        for pool in (ours, ref):
            m = pool.match(vids)
            n = len(vids) - m.length
            slots = pool.alloc(n)
            assert slots is not None
            new = _randn(100 + step, (L, 2, n, H, D)).bfloat16()
            pool.write(slots, new.to(DEV) if pool is ours else new)
            idx = torch.cat([m.indices.cpu(), slots.cpu()]) if m.length else slots.cpu()
            pool.insert(vids, idx, owned_from=m.length)
            m.release()
        mo, mr = ours.match(vids), ref.match(vids)
        assert mo.length == mr.length == prefix
        assert torch.equal(ours.gather(mo.indices).cpu(), ref.gather(mr.indices))
        mo.release()
        mr.release()
        assert ours.usage() == ref.usage()
    assert ours.usage()["evicted_tokens"] > 0
    assert ours.device_errors() == 0
