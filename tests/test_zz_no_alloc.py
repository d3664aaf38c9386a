"""The allocation-free append (qe_append_slots_ptrs_noalloc) against the allocating one (qe_append_slots_ptrs).

Some callers cannot allocate device memory (their process hands all of it to another allocator), so they
cannot build the device array of per-plane source pointers qe_append_slots_ptrs needs; the no-alloc entry
point takes the pointers from host memory and keeps its table in the library's own device memory. Both entry
points are called through the C ABI on identical pools, twice in a row with different data, and must leave the
pools bit-identical (the tolerance of every copy test here). This file is collected last on purpose.
"""

import ctypes

import numpy as np
import pytest
import torch

from qwenedit_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
L, H, D = 6, 24, 128
ROWS = 1200


def _planes(t):
    e = t.element_size()
    return _lib.planes(t.data_ptr(), t.stride(0) * e, t.stride(1) * e, 2)


def _sources(seed, n):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [torch.randn(n, H, D, generator=g, device=DEV).bfloat16() for _ in range(2 * L)]


def _call_both(pool_a, pool_b, srcs, slots):
    stream = torch.cuda.current_stream().cuda_stream
    row = H * D * 2
    n = slots.numel()
    err = torch.zeros(2, dtype=torch.int32, device=DEV)
    # existing entry point: a device array of pointers, allocated by the caller
    table = torch.tensor([t.data_ptr() for t in srcs], dtype=torch.int64, device=DEV)
    _lib.call("qe_append_slots_ptrs", _planes(pool_a), ROWS, table.data_ptr(), 2 * L, row, slots.data_ptr(), n,
              err[0:1].data_ptr(), stream)
    # no-alloc entry point: the same pointers from host memory
    host = (ctypes.c_void_p * (2 * L))(*[t.data_ptr() for t in srcs])
    _lib.call("qe_append_slots_ptrs_noalloc", _planes(pool_b), ROWS, ctypes.cast(host, ctypes.c_void_p), 2 * L,
              row, slots.data_ptr(), n, err[1:2].data_ptr(), stream)
    torch.cuda.synchronize()
    assert err.sum().item() == 0
    return table


@pytest.fixture
def copy_mode(request):
    """Run under one of the copy kernels (0 default, 1 warp, 2 TMA bulk, 3 one row per pass, 4 16-byte
    vectors); the default is restored afterwards."""
    _lib.call("qe_set_paged_copy_mode", request.param)
    yield request.param
    _lib.call("qe_set_paged_copy_mode", 0)


@pytest.mark.parametrize("copy_mode", [0, 1, 2, 3, 4], indirect=True)
def test_no_alloc_append_matches_the_allocating_one_twice(copy_mode):
    g = torch.Generator(device=DEV).manual_seed(1)
    pool_a = torch.randn(L, 2, ROWS, H, D, generator=g, device=DEV).bfloat16()
    pool_b = pool_a.clone()
    rng = np.random.default_rng(0)
    for call, n in enumerate((333, 517)):  # two calls in a row, different sizes, slots and data
        slots = torch.from_numpy(rng.permutation(ROWS)[:n].astype(np.int64)).to(DEV)
        srcs = _sources(10 + call, n)
        _call_both(pool_a, pool_b, srcs, slots)
        assert torch.equal(pool_a, pool_b), f"call {call}, copy mode {copy_mode}"
        # and both equal the per-layer index_copy_ the reference runs (hooks.py:136-138)
        ref = pool_a.clone()
        for layer in range(L):
            ref[layer, 0].index_copy_(0, slots, srcs[2 * layer])
            ref[layer, 1].index_copy_(0, slots, srcs[2 * layer + 1])
        assert torch.equal(pool_b, ref)


def test_no_alloc_append_with_16_byte_aligned_sources():
    """Source rows that start 16 bytes past a 32-byte boundary: the copy falls back to 16-byte vectors and the
    pool still equals the per-layer index_copy_."""
    g = torch.Generator(device=DEV).manual_seed(2)
    pool = torch.randn(L, 2, ROWS, H, D, generator=g, device=DEV).bfloat16()
    n = 250
    slots = torch.from_numpy(np.random.default_rng(1).permutation(ROWS)[:n].astype(np.int64)).to(DEV)
    srcs = []
    for t in _sources(20, n):
        buf = torch.empty(t.numel() + 8, dtype=torch.bfloat16, device=DEV)
        view = buf[8:].view(t.shape)
        view.copy_(t)
        assert view.data_ptr() % 32 == 16
        srcs.append(view)
    ref = pool.clone()
    for layer in range(L):
        ref[layer, 0].index_copy_(0, slots, srcs[2 * layer])
        ref[layer, 1].index_copy_(0, slots, srcs[2 * layer + 1])
    host = (ctypes.c_void_p * (2 * L))(*[t.data_ptr() for t in srcs])
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.call("qe_append_slots_ptrs_noalloc", _planes(pool), ROWS, ctypes.cast(host, ctypes.c_void_p), 2 * L,
              H * D * 2, slots.data_ptr(), n, err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.equal(pool, ref)


def test_no_alloc_append_rejects_more_planes_than_its_table():
    pool = torch.zeros(1, 2, 4, 1, 8, dtype=torch.bfloat16, device=DEV)
    host = (ctypes.c_void_p * 1025)()
    slots = torch.zeros(1, dtype=torch.int64, device=DEV)
    with pytest.raises(ValueError, match="exceed the static table"):
        _lib.call("qe_append_slots_ptrs_noalloc", _planes(pool), 4, ctypes.cast(host, ctypes.c_void_p), 1025, 16,
                  slots.data_ptr(), 1, None, torch.cuda.current_stream().cuda_stream)
