"""Paged joint attention (qe_paged_attention) against an fp32 PyTorch attention over the gathered prefix.

The reference path gathers the matched prefix (PagedKVPool.gather, cache/paged.py:106-113) and attends over
[prefix; the step's own K/V] (the DiT's joint attention fed by pipeline/hooks.py:81-83; the encoder tail's SDPA,
cache/encoder.py:173-190, with grouped-query heads and a bottom-right causal mask). The kernel reads the prefix
straight from the pool pages. Every pool row that is not part of the prefix (other pages, and the rows of the
last page past the prefix) holds NaN, so reading one would poison the output.

Tolerance: the kernel takes bf16 inputs, accumulates in fp32 and rounds P to bf16 before P V, and its output is
bf16: |out - ref| <= 1e-2 + 2e-2 |ref| elementwise against fp32 math on the same bf16 inputs, and the mean
absolute error below 2e-3; the log-sum-exp within 1e-3.
"""

import math

import numpy as np
import pytest
import torch

from qwenedit_b200.attention import PagedPrefix, paged_attention
from qwenedit_b200.paged import PagedKVPool

pytestmark = pytest.mark.gpu
DEV = "cuda"
D = 128


@pytest.fixture(autouse=True, params=[1, 2], ids=["one_q_tile", "two_q_tiles"])
def q_tiles(request):
    """Every test with one and with two 128-query tiles per CTA (by default the grid size picks one)."""
    from qwenedit_b200 import _lib

    _lib.call("qe_set_attention_q_tiles", request.param)
    yield request.param
    _lib.call("qe_set_attention_q_tiles", 0)


def _pool(layers, heads, page, n_pages, seed):
    """A page-mode pool of n_pages pages filled with NaN."""
    budget = n_pages * page * layers * 2 * heads * D * 2
    pool = PagedKVPool("attn", layers, heads, D, budget, torch.bfloat16, DEV, page_size=page)
    pool.kv.fill_(float("nan"))
    return pool


def _prefix(pool, n, seed):
    """Scattered pages for an n-token prefix, their rows filled with N(0, 1) values; the rest stays NaN."""
    P = pool.page_size
    rng = np.random.default_rng(seed)
    pages = rng.permutation(np.arange(1, pool.rows // P))[: -(-n // P)]
    t = np.arange(n)
    slots = torch.from_numpy(pages[t // P] * P + t % P).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(seed)
    vals = torch.randn(pool.layers, 2, n, pool.heads, D, generator=g, device=DEV).bfloat16()
    pool.kv[:, :, slots] = vals
    return slots, vals


def _reference(q, k, v, scale, causal, n_local):
    """fp32 attention, q [n_q, Hq, D], k / v [n_k, Hkv, D] (prefix then own); returns out [n_q, Hq, D], lse."""
    n_q, hq = q.shape[:2]
    group = hq // k.shape[1]
    qf = q.float().transpose(0, 1)
    kf = k.float().transpose(0, 1).repeat_interleave(group, 0)
    vf = v.float().transpose(0, 1).repeat_interleave(group, 0)
    s = qf @ kf.transpose(1, 2) * scale
    if causal:
        n_k = k.shape[0]
        n_pre = n_k - n_local
        i = torch.arange(n_q, device=q.device)[:, None]
        j = torch.arange(n_k, device=q.device)[None, :]
        visible = (j < n_pre) | (j - n_pre <= i + n_local - n_q)
        s = s.masked_fill(~visible, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    out = torch.softmax(s, dim=-1) @ vf
    return out.transpose(0, 1), lse


def _check(out, lse, ref_out, ref_lse):
    assert not torch.isnan(out).any(), "NaN in the output: a row outside the prefix was read"
    err = (out.float() - ref_out).abs()
    assert bool((err <= 1e-2 + 2e-2 * ref_out.abs()).all()), f"max abs error {err.max().item()}"
    assert err.mean().item() < 2e-3, err.mean().item()
    if lse is not None:
        assert torch.allclose(lse, ref_lse, atol=1e-3, rtol=1e-4), (lse - ref_lse).abs().max().item()


CASES = [  # (page, heads_q, heads_kv, n_q, n_prefix, n_local, causal, layers, layer)
    (64, 4, 4, 300, 1000, 0, False, 2, 1),      # partial Q tiles, partial last page, prefix only
    (64, 2, 2, 512, 4608, 512, False, 1, 0),    # the DiT's joint attention: whole pages + own tokens
    (16, 28, 4, 77, 777, 77, True, 3, 2),       # the encoder tail: GQA 7, causal own keys
    (128, 3, 3, 130, 300, 45, False, 1, 0),     # one page per tile
    (256, 2, 1, 257, 700, 0, False, 2, 0),      # pages larger than a tile, GQA 2
    (8, 2, 2, 40, 100, 37, True, 1, 0),         # 16 small pages per tile, more queries than own keys
    (32, 2, 2, 1, 33, 1, True, 1, 0),           # one query
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_paged_attention_matches_fp32(case):
    page, hq, hkv, n_q, n_prefix, n_local, causal, layers, layer = case
    n_pages = -(-n_prefix // page) + 3
    pool = _pool(layers, hkv, page, n_pages, seed=page)
    slots, vals = _prefix(pool, n_prefix, seed=n_prefix)
    g = torch.Generator(device=DEV).manual_seed(7)
    q = torch.randn(n_q, hq, D, generator=g, device=DEV).bfloat16()
    k_own = torch.randn(n_local, hkv, D, generator=g, device=DEV).bfloat16() if n_local else None
    v_own = torch.randn(n_local, hkv, D, generator=g, device=DEV).bfloat16() if n_local else None
    scale = 1 / math.sqrt(D)
    out, lse = paged_attention(q, PagedPrefix(pool, slots), layer, k_own, v_own, causal=causal, scale=scale,
                               return_lse=True)
    torch.cuda.synchronize()
    assert pool.device_errors() == 0
    k = vals[layer, 0] if n_local == 0 else torch.cat([vals[layer, 0], k_own])
    v = vals[layer, 1] if n_local == 0 else torch.cat([vals[layer, 1], v_own])
    ref_out, ref_lse = _reference(q, k, v, scale, causal, n_local)
    _check(out, lse, ref_out, ref_lse)


def test_own_keys_only_causal():
    """No prefix (a first turn): causal attention over the step's own keys only."""
    g = torch.Generator(device=DEV).manual_seed(3)
    n, h = 333, 2
    q, k, v = (torch.randn(n, h, D, generator=g, device=DEV).bfloat16() for _ in range(3))
    out, lse = paged_attention(q, None, 0, k, v, causal=True, return_lse=True)
    ref_out, ref_lse = _reference(q, k, v, 1 / math.sqrt(D), True, n)
    _check(out, lse, ref_out, ref_lse)


def test_growing_maximum_rescales_the_output():
    """Scores whose row maximum keeps growing from tile to tile by more than the lazy-rescale threshold, with a
    sharp softmax: the O rescale path has to be exact."""
    page, h, n_prefix = 64, 2, 1024
    pool = _pool(1, h, page, n_prefix // page + 2, seed=1)
    slots, vals = _prefix(pool, n_prefix, seed=2)
    ramp = torch.linspace(0.2, 3.0, n_prefix, device=DEV)[:, None, None]
    vals[0, 0] = (vals[0, 0].float() * ramp).bfloat16()  # later keys: larger scores
    pool.kv[:, :, slots] = vals
    g = torch.Generator(device=DEV).manual_seed(4)
    q = (torch.randn(256, h, D, generator=g, device=DEV) * 3).bfloat16()
    out, lse = paged_attention(q, PagedPrefix(pool, slots), 0, return_lse=True)
    ref_out, ref_lse = _reference(q, vals[0, 0], vals[0, 1], 1 / math.sqrt(D), False, 0)
    _check(out, lse, ref_out, ref_lse)


def test_max_growth_in_each_half_of_a_tile():
    """Scores built so that the row max jumps by about 20 octaves inside the second half of key tile 1 and again
    inside the first half of tile 2, then stays low in tile 3: every row takes the one-pass path with a half-B
    rescale (O, half-A P and row sum scaled by a power of two, half B redone), the two-pass path from a half-A
    jump, and the plain one-pass path."""
    n_q, n_k, h = 128, 512, 2
    scale = 1 / math.sqrt(D)
    step = 20.0 / (scale * math.log2(math.e))  # a score step of 20 octaves after scaling
    g = torch.Generator(device=DEV).manual_seed(61)
    q = torch.zeros(n_q, h, D, device=DEV)
    q[:, :, 0] = 1.0
    q[:, :, 1:] = torch.randn(n_q, h, D - 1, generator=g, device=DEV) * 0.1
    c = torch.zeros(n_k, device=DEV)
    c[128 + 64: 256] = step        # tile 1, half B
    c[256: 256 + 32] = 2 * step    # tile 2, half A
    c[256 + 32: 384] = step
    k = torch.randn(n_k, h, D, generator=g, device=DEV) * 0.1
    k[:, :, 0] = c[:, None] + torch.randn(n_k, h, generator=g, device=DEV)
    v = torch.randn(n_k, h, D, generator=g, device=DEV)
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    out, lse = paged_attention(q, None, 0, k, v, scale=scale, return_lse=True)
    ref_out, ref_lse = _reference(q, k, v, scale, False, n_k)
    _check(out, lse, ref_out, ref_lse)
    # without the last two tiles, the half-B rescale decides the output alone
    out2, lse2 = paged_attention(q, None, 0, k[:256], v[:256], scale=scale, return_lse=True)
    ref2, ref_lse2 = _reference(q, k[:256], v[:256], scale, False, 256)
    _check(out2, lse2, ref2, ref_lse2)
    # growth a half-tile sum does not show: one key 12 octaves up in tile 1 (its p stays below 2^14), then a
    # whole tile there
    k3 = k.clone()
    k3[:, :, 0] = torch.randn(n_k, h, generator=g, device=DEV).bfloat16()
    k3[128 + 5, :, 0] = 0.6 * step
    k3[256:384, :, 0] = 0.6 * step
    out3, lse3 = paged_attention(q, None, 0, k3, v, scale=scale, return_lse=True)
    ref3, ref_lse3 = _reference(q, k3, v, scale, False, n_k)
    _check(out3, lse3, ref3, ref_lse3)


def test_page_outside_the_pool_reads_zeros_and_is_reported():
    page, h, n_prefix = 64, 2, 256
    pool = _pool(1, h, page, 6, seed=5)
    slots, vals = _prefix(pool, n_prefix, seed=6)
    prefix = PagedPrefix(pool, slots)
    prefix.block_table[2] = pool.rows // page + 5  # the third page points past the pool
    g = torch.Generator(device=DEV).manual_seed(8)
    q = torch.randn(128, h, D, generator=g, device=DEV).bfloat16()
    out = paged_attention(q, prefix, 0)
    torch.cuda.synchronize()
    assert pool.device_errors() & 1
    k, v = vals[0, 0].clone(), vals[0, 1].clone()
    k[2 * page: 3 * page] = 0
    v[2 * page: 3 * page] = 0
    ref_out, _ = _reference(q, k, v, 1 / math.sqrt(D), False, 0)
    _check(out, None, ref_out, None)


def test_one_k_edit_layer_joint_attention():
    """One DiT layer of the 1K edit: 4096 latent queries over the 4608-token prefix (page 64, scattered pages)
    and their own 4096 keys, 24 heads; checked on every head."""
    page, h, n_prefix, n = 64, 24, 4608, 4096
    pool = _pool(1, h, page, n_prefix // page + 4, seed=9)
    slots, vals = _prefix(pool, n_prefix, seed=10)
    g = torch.Generator(device=DEV).manual_seed(11)
    q, k_own, v_own = (torch.randn(n, h, D, generator=g, device=DEV).bfloat16() for _ in range(3))
    out, lse = paged_attention(q, PagedPrefix(pool, slots), 0, k_own, v_own, return_lse=True)
    k = torch.cat([vals[0, 0], k_own])
    v = torch.cat([vals[0, 1], v_own])
    for h0 in range(0, h, 6):  # the fp32 reference in slices of heads
        ref_out, ref_lse = _reference(q[:, h0:h0 + 6], k[:, h0:h0 + 6], v[:, h0:h0 + 6], 1 / math.sqrt(D), False, 0)
        _check(out[:, h0:h0 + 6], lse[h0:h0 + 6], ref_out, ref_lse)


def test_strided_views_in_and_out():
    """q, own K/V and out as head slices of wider token rows (as projections produce them)."""
    page, h, n_prefix, n = 32, 2, 200, 150
    pool = _pool(1, h, page, n_prefix // page + 3, seed=12)
    slots, vals = _prefix(pool, n_prefix, seed=13)
    g = torch.Generator(device=DEV).manual_seed(14)
    qkv = torch.randn(n, 3 * h, D, generator=g, device=DEV).bfloat16()
    q, k_own, v_own = qkv[:, :h], qkv[:, h:2 * h], qkv[:, 2 * h:]
    wide = torch.zeros(n, 4 * h, D, dtype=torch.bfloat16, device=DEV)
    out = paged_attention(q, PagedPrefix(pool, slots), 0, k_own, v_own, out=wide[:, h:2 * h])
    assert out.data_ptr() == wide[:, h:2 * h].data_ptr()
    ref_out, _ = _reference(q, torch.cat([vals[0, 0], k_own]), torch.cat([vals[0, 1], v_own]), 1 / math.sqrt(D),
                            False, 0)
    _check(out, None, ref_out, None)
    assert bool((wide[:, :h] == 0).all()) and bool((wide[:, 2 * h:] == 0).all())


# ---- fused append: the own K/V stored into the pool by the attention launch itself ------------------------------
APPEND_CASES = [  # (page, heads_q, heads_kv, n_q, n_prefix, n_local, causal, layers, layer)
    (64, 4, 2, 300, 1000, 300, True, 2, 1),     # GQA, causal, ragged own tokens (4 pages + 44 rows)
    (16, 2, 2, 257, 0, 257, False, 1, 0),      # first turn (no prefix), pages shorter than a key tile
    (256, 2, 1, 512, 512, 700, False, 2, 0),   # pages of two key tiles, more own keys than queries
    (128, 2, 2, 1024, 4096, 1024, False, 1, 0),  # whole pages
    (8, 4, 1, 200, 64, 200, True, 1, 0),       # the smallest page: 16 pages per key tile, 4 query heads per K/V head
]


@pytest.mark.parametrize("case", APPEND_CASES, ids=lambda c: "-".join(map(str, c)))
def test_fused_append_stores_the_own_tokens(case):
    """paged_attention(append=...): the output as without the append, and the pool afterwards equal to the pool
    before with exactly the own tokens' rows of `layer` replaced by k_local / v_local (bit-exact); the rows of
    the last page past the last own token, the other layers and every other page keep their NaN."""
    page, hq, hkv, n_q, n_prefix, n_local, causal, layers, layer = case
    n_app_pages = -(-n_local // page)
    pool = _pool(layers, hkv, page, -(-n_prefix // page) + n_app_pages + 3, seed=page + 1)
    slots, vals = _prefix(pool, n_prefix, seed=n_prefix + 1) if n_prefix else (None, None)
    used = set() if slots is None else set((slots.cpu().numpy() // page).tolist())
    rng = np.random.default_rng(n_local)
    free = [p for p in rng.permutation(np.arange(1, pool.rows // page)).tolist() if p not in used]
    t = np.arange(n_local)
    app_slots = torch.from_numpy(np.array(free[:n_app_pages])[t // page] * page + t % page).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(17)
    q = torch.randn(n_q, hq, D, generator=g, device=DEV).bfloat16()
    kv_own = torch.randn(n_local, 2 * hkv, D, generator=g, device=DEV).bfloat16()
    k_own, v_own = kv_own[:, :hkv], kv_own[:, hkv:]  # strided token rows, as a fused K/V projection gives them
    before = pool.kv.clone()
    prefix = PagedPrefix(pool, slots) if n_prefix else None
    scale = 1 / math.sqrt(D)
    out, lse = paged_attention(q, prefix, layer, k_own, v_own, causal=causal, scale=scale, return_lse=True,
                               append=PagedPrefix(pool, app_slots))
    torch.cuda.synchronize()
    assert pool.device_errors() == 0
    k = k_own if not n_prefix else torch.cat([vals[layer, 0], k_own])
    v = v_own if not n_prefix else torch.cat([vals[layer, 1], v_own])
    ref_out, ref_lse = _reference(q, k, v, scale, causal, n_local)
    _check(out, lse, ref_out, ref_lse)
    want = before
    want[layer, 0, app_slots] = k_own
    want[layer, 1, app_slots] = v_own
    assert torch.equal(pool.kv.view(torch.int16), want.view(torch.int16))


def test_fused_append_skips_a_page_outside_the_pool():
    page, h, n = 32, 2, 100
    pool = _pool(1, h, page, 8, seed=21)
    t = np.arange(n)
    pages = np.array([2, 5, 3, 6])
    app = PagedPrefix(pool, torch.from_numpy(pages[t // page] * page + t % page).to(DEV))
    app.block_table[1] = pool.rows // page + 2  # the second page points past the pool
    g = torch.Generator(device=DEV).manual_seed(22)
    q, k_own, v_own = (torch.randn(n, h, D, generator=g, device=DEV).bfloat16() for _ in range(3))
    before = pool.kv.clone()
    out = paged_attention(q, None, 0, k_own, v_own, causal=True, append=app)
    torch.cuda.synchronize()
    assert pool.device_errors() & 1
    ref_out, _ = _reference(q, k_own, v_own, 1 / math.sqrt(D), True, n)
    _check(out, None, ref_out, None)
    want = before
    keep = torch.from_numpy(np.r_[0:page, 2 * page:n]).to(DEV)
    rows = torch.from_numpy((pages[t // page] * page + t % page)[np.r_[0:page, 2 * page:n]]).to(DEV)
    want[0, 0, rows] = k_own[keep]
    want[0, 1, rows] = v_own[keep]
    assert torch.equal(pool.kv.view(torch.int16), want.view(torch.int16))


def test_fused_append_argument_checks():
    pool = _pool(1, 2, 64, 4, seed=23)
    q = torch.zeros(64, 2, D, dtype=torch.bfloat16, device=DEV)
    app = PagedPrefix(pool, torch.arange(64, 128, device=DEV))
    with pytest.raises(ValueError, match="slots for"):
        paged_attention(q, None, 0, q[:32], q[:32], append=app)
    other = _pool(1, 2, 64, 4, seed=24)
    slots, _ = _prefix(other, 64, seed=25)
    with pytest.raises(ValueError, match="same pool"):
        paged_attention(q, PagedPrefix(other, slots), 0, q, q, append=app)


# ---- the tail computations either side of the pool (f2): encoder partial hit, DiT prefix prefill ----------------
def _sdpa_ref(q, k, v, mask, scale):
    """fp32 attention with a boolean visibility mask [n_q, n_k], GQA by head repetition (the reference's
    F.scaled_dot_product_attention(..., attn_mask=mask, enable_gqa=True))."""
    group = q.shape[1] // k.shape[1]
    qf = q.float().transpose(0, 1)
    kf = k.float().transpose(0, 1).repeat_interleave(group, 0)
    vf = v.float().transpose(0, 1).repeat_interleave(group, 0)
    s = (qf @ kf.transpose(1, 2) * scale).masked_fill(~mask, float("-inf"))
    return (torch.softmax(s, dim=-1) @ vf).transpose(0, 1)


@pytest.mark.parametrize("page", [16, 1])
def test_encoder_tail_attention_matches_the_reference_mask(page):
    """cache/encoder.py:173-190: tail queries over [cached prefix; tail] with ones(n, m + n).tril(diagonal=m),
    grouped-query heads 28 / 4. Page 16: the kernel reads the pool pages; page 1 (token-granular, the reference's
    pool): the head-major gather feeds the kernel, the tail written after the prefix."""
    from qwenedit_b200.attention import encoder_tail_attention

    layers, hq, hkv, m, n = 3, 28, 4, 777, 77
    pool = _pool(layers, hkv, page, -(-m // page) + 4, seed=21)
    slots, vals = _prefix(pool, m, seed=22)
    g = torch.Generator(device=DEV).manual_seed(23)
    scale = 128 ** -0.5
    heads_buf = None if page > 1 else pool.gather_heads(slots, m + n)
    for layer in range(layers):
        q = torch.randn(n, hq, D, generator=g, device=DEV).bfloat16()
        k_t, v_t = (torch.randn(n, hkv, D, generator=g, device=DEV).bfloat16() for _ in range(2))
        out = encoder_tail_attention(q, k_t, v_t, pool, slots, layer, scale, heads_buf=heads_buf)
        mask = torch.ones(n, m + n, dtype=torch.bool, device=DEV).tril(diagonal=m)
        ref = _sdpa_ref(q, torch.cat([vals[layer, 0], k_t]), torch.cat([vals[layer, 1], v_t]), mask, scale)
        _check(out, None, ref, None)
        if heads_buf is not None:
            assert torch.equal(heads_buf[layer, 0, :, m:], k_t.transpose(0, 1))


@pytest.mark.parametrize("start", [0, 100, 700])
def test_prefill_attention_matches_the_segment_loop(start):
    """cache/prefill.py:52-66: each segment (s, e, is_image) of positions [start, total) attends over keys [0, e),
    causally inside text segments; keys before `start` come from the pool."""
    from qwenedit_b200.attention import prefill_attention

    h, total = 4, 900
    segments = [(0, 100, False), (100, 612, True), (612, 900, False)]
    pool = _pool(2, h, 64, 16, seed=31)
    layer = 1
    if start:
        slots, vals = _prefix(pool, start, seed=32)
        pre_k, pre_v = vals[layer, 0], vals[layer, 1]
        prefix = PagedPrefix(pool, slots)
    else:
        pre_k = pre_v = torch.empty(0, h, D, dtype=torch.bfloat16, device=DEV)
        prefix = None
    g = torch.Generator(device=DEV).manual_seed(33)
    q, k, v = (torch.randn(total - start, h, D, generator=g, device=DEV).bfloat16() for _ in range(3))
    scale = 1 / math.sqrt(D)
    out = prefill_attention(q, k, v, prefix, layer, segments, start, scale)
    keys, values = torch.cat([pre_k, k]), torch.cat([pre_v, v])
    for s0, e, is_image in segments:
        if e <= start:
            continue
        s = max(s0, start)
        mask = torch.ones(e - s, e, dtype=torch.bool, device=DEV)
        if not is_image:
            mask = torch.arange(e, device=DEV)[None, :] <= torch.arange(s, e, device=DEV)[:, None]
        ref = _sdpa_ref(q[s - start:e - start], keys[:e], values[:e], mask, scale)
        _check(out[s - start:e - start], None, ref, None)


def _free_slots(pool, used, n, seed):
    """Slots for n tokens on whole pages of `pool` that hold none of the `used` slots (and not page 0)."""
    P = pool.page_size
    taken = set() if used is None else set((used.cpu().numpy() // P).tolist())
    rng = np.random.default_rng(seed)
    pages = np.array([p for p in rng.permutation(np.arange(1, pool.rows // P)).tolist() if p not in taken])
    t = np.arange(n)
    return torch.from_numpy(pages[: -(-n // P)][t // P] * P + t % P).to(DEV)


@pytest.mark.parametrize("start", [0, 128])
def test_prefill_with_fused_append_stores_the_tail_of_every_layer(start):
    """The prefix prefill from a cached head (prefill.py:32-72) with the tail's K/V appended by the attention
    launches themselves: per layer the output equals the plain prefill's, and afterwards the pool holds, at the
    cached slots then the tail slots, every layer's K/V of the whole prefix (what the reference's pool.write of
    kv[:, :, m:] followed by insert leaves). start 0: a miss, the whole prefix computed and stored."""
    from qwenedit_b200.attention import prefill_attention

    h, total, layers = 4, 900, 2
    segments = [(0, 128, False), (128, 640, True), (640, 900, False)]
    pool = _pool(layers, h, 64, 20, seed=41)
    if start:
        slots, vals = _prefix(pool, start, seed=42)
    else:
        slots, vals = None, torch.empty(layers, 2, 0, h, D, dtype=torch.bfloat16, device=DEV)
    tail = _free_slots(pool, slots, total - start, seed=43)
    prefix, app = (PagedPrefix(pool, slots) if start else None), PagedPrefix(pool, tail)
    g = torch.Generator(device=DEV).manual_seed(44)
    kv_tail = torch.empty(layers, 2, total - start, h, D, dtype=torch.bfloat16, device=DEV)
    for layer in range(layers):
        q, k, v = (torch.randn(total - start, h, D, generator=g, device=DEV).bfloat16() for _ in range(3))
        kv_tail[layer, 0], kv_tail[layer, 1] = k, v
        want = prefill_attention(q, k, v, prefix, layer, segments, start)
        got = prefill_attention(q, k, v, prefix, layer, segments, start, append=app)
        assert torch.equal(got, want)
    torch.cuda.synchronize()
    assert pool.device_errors() == 0
    whole = pool.kv[:, :, tail if slots is None else torch.cat([slots, tail])]
    assert torch.equal(whole.view(torch.int16), torch.cat([vals, kv_tail], dim=2).view(torch.int16))
    with pytest.raises(ValueError, match="last segment"):
        prefill_attention(q[:-1], k[:-1], v[:-1], prefix, 0, segments, start, append=app)


def test_encoder_tail_with_fused_append():
    """encoder.py:131-138 after a partial hit: each layer's tail attention also stores the tail K/V into the slots
    allocated for it (page-16 pool, grouped-query heads)."""
    from qwenedit_b200.attention import encoder_tail_attention

    layers, hq, hkv, m, n = 2, 28, 4, 320, 77
    pool = _pool(layers, hkv, 16, -(-m // 16) + -(-n // 16) + 4, seed=51)
    slots, vals = _prefix(pool, m, seed=52)
    app = PagedPrefix(pool, _free_slots(pool, slots, n, seed=53))
    g = torch.Generator(device=DEV).manual_seed(54)
    scale = 128 ** -0.5
    for layer in range(layers):
        q = torch.randn(n, hq, D, generator=g, device=DEV).bfloat16()
        k_t, v_t = (torch.randn(n, hkv, D, generator=g, device=DEV).bfloat16() for _ in range(2))
        out = encoder_tail_attention(q, k_t, v_t, pool, slots, layer, scale, append=app)
        mask = torch.ones(n, m + n, dtype=torch.bool, device=DEV).tril(diagonal=m)
        ref = _sdpa_ref(q, torch.cat([vals[layer, 0], k_t]), torch.cat([vals[layer, 1], v_t]), mask, scale)
        _check(out, None, ref, None)
        assert torch.equal(pool.kv[layer, 0, app.indices], k_t) and torch.equal(pool.kv[layer, 1, app.indices], v_t)
    assert pool.device_errors() == 0
    tok = _pool(1, hkv, 1, 400, seed=55)
    with pytest.raises(ValueError, match="page-mode"):
        encoder_tail_attention(q, k_t, v_t, tok, torch.arange(1, 11, device=DEV), 0, scale, append=app)


def test_prefill_attention_rejects_a_prefix_ending_inside_an_image():
    from qwenedit_b200.attention import prefill_attention

    q = torch.zeros(10, 1, D, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="inside an image block"):
        prefill_attention(q, q, q, None, 0, [(0, 20, True)], 10)
