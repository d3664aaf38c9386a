"""Paged joint attention over a pooled prefix: the consumer side of the DiT prefix cache, without the gather.

The reference materialises the matched prefix every denoising step (``PagedKVPool.gather``, cache/paged.py:106-113,
called from pipeline/hooks.py:101-105) and hands per-layer K/V views to the model's joint attention
(hooks.py:81-83), which attends over [prefix; the step's own tokens]. ``paged_attention`` computes that attention
in one hand-written sm_100a kernel (``qe_paged_attention``) that reads the prefix K/V tiles from the pool pages
through the block table, so the per-step gather copy (6.8 GB per 1K-edit step) never happens.

``PagedPrefix`` is what a hook hands the attention in place of the gathered caches: the pool and the matched
slots, with the device block table cached on first use.

The same kernel takes grouped-query heads and a bottom-right causal mask on the step's own keys, which is the text
encoder's partial-hit attention (cache/encoder.py:173-190: tail queries over [cached prefix; tail], tail position
i sees the prefix and tail [0, i]).
"""

from __future__ import annotations

import math

import torch

from qwenedit_b200 import _lib

HEAD_DIM = 128


class PagedPrefix:
    """The matched prefix of one sample as pool pages: `pool` (a page-mode PagedKVPool) and `indices` (the slots a
    match returned). `block_table` is the device int32 page table, built once and reused by every layer and step."""

    def __init__(self, pool, indices: torch.Tensor):
        self.pool = pool
        self.indices = indices
        self.length = int(indices.numel())
        host = pool._host_slots(indices)
        self.block_table = pool._block_table(indices, host) if self.length else None
        if self.length and self.block_table is None:
            raise ValueError("paged attention needs the prefix as whole-page runs of a page-mode pool "
                             f"(page_size {pool.page_size})")

    def planes(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The pool's K and V planes of `layer`, [rows, H, D]."""
        return self.pool.kv[layer, 0], self.pool.kv[layer, 1]


def _check(name: str, t: torch.Tensor | None, device) -> None:
    if t is None:
        return
    if t.device.type != "cuda" or t.device != device:
        raise ValueError(f"{name} must be a CUDA tensor on {device}")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16")
    if t.dim() != 3 or t.shape[-1] != HEAD_DIM or t.stride(-1) != 1:
        raise ValueError(f"{name} must be [tokens, heads, {HEAD_DIM}] with contiguous head rows")


def paged_attention(q: torch.Tensor, prefix: PagedPrefix | None, layer: int = 0, k_local: torch.Tensor | None = None,
                    v_local: torch.Tensor | None = None, causal: bool = False, scale: float | None = None,
                    out: torch.Tensor | None = None, return_lse: bool = False, append: PagedPrefix | None = None):
    """softmax(q K^T * scale) V with K, V = [prefix K/V of `layer` from the pool; k_local / v_local].

    q [n_q, Hq, 128] bf16; k_local / v_local [n_local, Hkv, 128] bf16 (the step's own keys, may be None);
    Hq a multiple of the pool's Hkv (grouped-query heads); `causal`: query i sees every prefix key and own keys
    j <= i + n_local - n_q (bottom-right alignment). Returns out [n_q, Hq, 128] bf16 (and the log-sum-exp
    [Hq, n_q] fp32 of the scaled scores with `return_lse`). One kernel launch on the current stream.

    `append`: the pool slots of the own tokens (a PagedPrefix over ``pool.alloc(n_local)``, whole pages of a
    page-mode pool); the same launch also writes k_local / v_local into layer `layer` of those slots, from the
    tiles it loads for the attention (the store that cache/prefill.py:69-72 and the encoder's _store,
    cache/encoder.py:131-138, do as separate copies). Rows of the last page past the last own token are not
    written."""
    if q.dim() != 3:
        raise ValueError("q must be [tokens, heads, 128]")
    device = q.device
    _check("q", q, device)
    _check("k_local", k_local, device)
    _check("v_local", v_local, device)
    n_q, heads_q = q.shape[0], q.shape[1]
    n_local = 0 if k_local is None else k_local.shape[0]
    if (k_local is None) != (v_local is None) or (k_local is not None and k_local.shape != v_local.shape):
        raise ValueError("k_local and v_local go together, with equal shapes")
    if k_local is not None and k_local.stride() != v_local.stride():
        raise ValueError("k_local and v_local must have the same strides")
    n_prefix = 0 if prefix is None else prefix.length
    if append is not None:
        if k_local is None or append.length != n_local:
            raise ValueError(f"append holds {append.length} slots for {n_local} own tokens")
        if prefix is not None and append.pool is not prefix.pool:
            raise ValueError("append and prefix must be slots of the same pool")
    pool_of = prefix if prefix is not None else append
    if pool_of is not None:
        pool = pool_of.pool
        heads_kv = pool.heads
        if pool.head_dim != HEAD_DIM or pool.kv.dtype != torch.bfloat16 or pool.device != device:
            raise ValueError(f"the pool must hold bf16 heads of {HEAD_DIM} on {device}")
        if not 0 <= layer < pool.layers:
            raise ValueError(f"layer {layer} outside the pool's {pool.layers}")
    else:
        heads_kv = k_local.shape[1] if k_local is not None else heads_q
    if k_local is not None and k_local.shape[1] != heads_kv:
        raise ValueError(f"local K/V have {k_local.shape[1]} heads, the pool {heads_kv}")
    if heads_q % heads_kv:
        raise ValueError(f"{heads_q} query heads are not a multiple of {heads_kv} K/V heads")
    if n_prefix + n_local == 0:
        raise ValueError("no keys: empty prefix and no local K/V")
    if out is None:
        out = torch.empty(n_q, heads_q, HEAD_DIM, dtype=torch.bfloat16, device=device)
    else:
        _check("out", out, device)
        if tuple(out.shape) != (n_q, heads_q, HEAD_DIM):
            raise ValueError("out must be [n_q, Hq, 128]")
    lse = torch.empty(heads_q, n_q, dtype=torch.float32, device=device) if return_lse else None
    scale = 1.0 / math.sqrt(HEAD_DIM) if scale is None else float(scale)
    e = 2
    if (prefix is not None and n_prefix) or append is not None:
        kp, vp = pool_of.planes(layer)
        err = pool._err
        table = prefix.block_table.data_ptr() if prefix is not None and n_prefix else None
        args_pool = (kp.data_ptr(), vp.data_ptr(), pool.rows, heads_kv, table, pool.page_size, n_prefix)
    else:
        err = None
        args_pool = (None, None, 0, heads_kv, None, 1, 0)
    if k_local is not None:
        args_local = (k_local.data_ptr(), v_local.data_ptr(), k_local.stride(0) * e, k_local.stride(1) * e, n_local)
    else:
        args_local = (None, None, 0, 0, 0)
    tail = (out.data_ptr(), out.stride(0) * e, out.stride(1) * e, None if lse is None else lse.data_ptr())
    with _lib.on_device(device):
        if append is None:
            _lib.call("qe_paged_attention", q.data_ptr(), q.stride(0) * e, q.stride(1) * e, n_q, heads_q, *args_pool,
                      *args_local, 1 if causal else 0, scale, *tail, None if err is None else err.data_ptr(),
                      _lib.stream_of(device))
        else:
            _lib.call("qe_paged_attention_append", q.data_ptr(), q.stride(0) * e, q.stride(1) * e, n_q, heads_q,
                      *args_pool, *args_local, 1 if causal else 0, scale, *tail, append.block_table.data_ptr(),
                      err.data_ptr(), _lib.stream_of(device))
    return (out, lse) if return_lse else out


def encoder_tail_attention(q: torch.Tensor, k_tail: torch.Tensor, v_tail: torch.Tensor, pool, indices: torch.Tensor,
                           layer: int, scale: float, heads_buf: torch.Tensor | None = None,
                           append: PagedPrefix | None = None) -> torch.Tensor:
    """One text-encoder layer's attention on a partial prefix hit (cache/encoder.py:173-190): the n tail queries
    attend over [the m cached prefix tokens; the n tail tokens], tail position i seeing the prefix and tail [0, i]
    (the reference's ``ones(n, m + n).tril(diagonal=m)`` mask), grouped-query heads (enable_gqa).

    q [n, Hq, 128], k_tail / v_tail [n, Hkv, 128] bf16 (token-major: the reference's ``k[0].transpose(0, 1)``).
    A page-mode pool (page size 8 to 128, or a multiple of 128) is read through its block table by the attention
    kernel itself. A token-granular pool (the reference's page size 1) is first gathered head-major with room for
    the tail (``pool.gather_heads``; pass the same `heads_buf` to every layer so it is gathered once), the tail
    K/V written after the prefix, and the kernel attends over that buffer. Returns [n, Hq, 128] bf16.

    `append` (page-mode pools): the slots allocated for the tail (``PagedPrefix(pool, pool.alloc(n))``); the same
    launch stores this layer's tail K/V there (the K/V planes of encoder.py:131-138's _store; the hidden rows stay
    ``pool.write_extra``)."""
    n = q.shape[0]
    m = int(indices.numel())
    if pool.page_size >= 8 and (128 % pool.page_size == 0 or pool.page_size % 128 == 0):
        return paged_attention(q, PagedPrefix(pool, indices) if m else None, layer, k_tail, v_tail, causal=True,
                               scale=scale, append=append)
    if append is not None:
        raise ValueError("a fused append needs a page-mode pool (page size 8 to 128, or a multiple of 128)")
    if heads_buf is None:
        heads_buf = pool.gather_heads(indices, m + n)
    if heads_buf.shape[3] != m + n:
        raise ValueError(f"heads_buf holds {heads_buf.shape[3]} positions, expected {m + n}")
    kh, vh = heads_buf[layer, 0], heads_buf[layer, 1]  # [Hkv, m + n, D]
    kh[:, m:].copy_(k_tail.transpose(0, 1))
    vh[:, m:].copy_(v_tail.transpose(0, 1))
    return paged_attention(q, None, layer, kh.transpose(0, 1), vh.transpose(0, 1), causal=True, scale=scale)


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, prefix: PagedPrefix | None, layer: int,
                      segments, start: int, scale: float | None = None,
                      append: PagedPrefix | None = None) -> torch.Tensor:
    """The attention of the DiT's prefix prefill from position `start` (cache/prefill.py:32-72), one layer: the
    prefix positions [start, total) attend per segment (s, e, is_image) over keys [0, e), causally inside text
    segments (a text query at position p sees keys <= p), fully inside image segments. Keys [0, start) are the
    pooled prefix (read through the block table); keys [start, e) are this call's own k / v.

    q, k, v [total - start, H, 128] bf16 for positions start .. total - 1; `segments` as the reference's layout
    (start and end positions over the whole prefix). Returns [total - start, H, 128]; one kernel launch per
    segment that starts past `start`.

    `append`: the pool slots of positions [start, total) (``PagedPrefix(pool, pool.alloc(total - start))``); the
    last segment's launch, whose own keys are all of k / v, also stores this layer's K/V there (the
    ``kv[l, :, m:]`` write of prefill.py:69-72 that the caller would otherwise append with ``pool.write``)."""
    n = q.shape[0]
    for s0, e, is_image in segments:  # as the reference checks before any layer runs
        if is_image and s0 < start < e:
            raise ValueError("cached prefix ends inside an image block")
    if start and (prefix is None or prefix.length != start):
        raise ValueError(f"the pooled prefix must hold the {start} positions before `start`")
    if append is not None and (not segments or segments[-1][1] - start != n):
        raise ValueError("a fused append needs the last segment to end at the last position given")
    out = torch.empty_like(q)
    for i, (s0, e, is_image) in enumerate(segments):
        if e <= start:
            continue
        s = max(s0, start)
        if is_image and s0 < start:
            raise ValueError("cached prefix ends inside an image block")
        lo, hi = s - start, e - start
        if hi > n:
            raise ValueError(f"segment ends at {e}, past the {start + n} positions given")
        paged_attention(q[lo:hi], prefix if start else None, layer, k[:hi], v[:hi], causal=not is_image,
                        scale=scale, out=out[lo:hi], append=append if i == len(segments) - 1 else None)
    return out
