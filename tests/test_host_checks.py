"""Host-side argument handling of the device entry points, on CPU (no kernel runs): CPU tensors are refused
with RuntimeError (there is no CPU path), bad boxes / dtypes / shapes raise before any launch, and the C ABI
rejects bad sizes with QE_ERR_INVALID (ValueError) without touching the GPU."""

import ctypes

import pytest
import torch

from qwenedit_b200 import _lib, fp4, latents
from qwenedit_b200.paged import pool_geometry


def test_latent_ops_refuse_cpu_tensors():
    x = torch.zeros(1, 16, 4, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        latents.mask_blend(x, x, x, torch.zeros(1, 16, 1), 0.5)
    with pytest.raises(RuntimeError, match="CUDA"):
        latents.crop(x, (4, 4), (0, 0, 2, 2))
    with pytest.raises(RuntimeError, match="CUDA"):
        latents.compose(x, (4, 4), x[:, :4], (0, 0, 2, 2))


def test_latent_box_checks():
    for box in ((0, 0, 5, 1), (2, 2, 2, 3), (-1, 0, 1, 1), (0, 3, 1, 2)):
        with pytest.raises(ValueError):
            latents._box(box, (4, 4))
    assert latents._box((1, 0, 4, 4), (4, 4)) == (1, 0, 4, 4)


def test_nvfp4_wrappers_refuse_cpu_and_bad_dtypes():
    g = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fp4.silu_mul_fp4(g, g, torch.ones(1))
    with pytest.raises(RuntimeError, match="CUDA"):
        fp4.silu_mul_amax(g, g)


def test_global_scale_is_the_reference_expression():
    amax = torch.tensor([3.7])
    assert fp4.global_scale(amax).item() == (448.0 * 6.0 / (amax.clamp(min=1e-8) * 4.0)).item()
    assert fp4.global_scale(torch.tensor([0.0])).item() == (448.0 * 6.0 / (torch.tensor(1e-8) * 4.0)).item()


def test_pool_geometry_matches_the_reference_rule():
    # capacity = budget // bytes per token, whole pages, plus one padding page (paged.py:44-47)
    cap, rows, per_token = pool_geometry(60, 24, 128, 24 << 30, torch.bfloat16, 0, 64)
    assert per_token == 737280 and cap == (24 << 30) // per_token // 64 * 64 and rows == cap + 64
    cap1, rows1, _ = pool_geometry(4, 2, 8, 10, torch.float32, 0, 1)
    assert cap1 == 1 and rows1 == 2


def test_c_abi_rejects_bad_sizes_without_a_gpu():
    planes = _lib.planes(16, 0, 0, 1)
    with pytest.raises(ValueError):
        _lib.call("qe_append_scatter", None, 0, planes, 1, planes, 1, 16, None, 0, None, None)
    with pytest.raises(ValueError):
        _lib.call("qe_mask_blend", None, None, None, None, None, None, 1, 1, 0, 0, 0, 0, 1, 0, 0, 0, None)
    with pytest.raises(ValueError):
        _lib.call("qe_latent_crop", None, None, 4, 4, 8, 0, 0, 5, 1, None)
    with pytest.raises(ValueError):
        _lib.call("qe_gather_slots_heads", planes, 1, planes, 1, 48, 32, 16, 16, None, 1, None, None)
    for fn, bad in (("qe_set_norm_table_mode", 3), ("qe_set_silu_table_mode", 3), ("qe_set_attention_q_tiles", 3),
                    ("qe_set_silu_pipeline", 3), ("qe_set_paged_copy_mode", 5)):
        with pytest.raises(ValueError):
            _lib.call(fn, bad)



def test_no_alloc_append_rejects_a_null_source_pointer():
    host = (ctypes.c_void_p * 2)(4096, None)
    with pytest.raises(ValueError, match="null source pointer 1"):
        _lib.call("qe_append_slots_ptrs_noalloc", _lib.planes(16, 0, 0, 1), 4, ctypes.cast(host, ctypes.c_void_p), 2,
                  16, 16, 1, None, None)


A = 0x10000  # a 64 KiB-aligned stand-in address: every call below fails its checks before touching it


def _rejects(name, match, *args):
    with pytest.raises(ValueError, match=match):
        _lib.call(name, *args)


def test_nvfp4_entry_points_check_sizes_and_alignment_first():
    """The NVFP4 entry points reject bad sizes, missing operands and misaligned pointers with QE_ERR_INVALID
    before any CUDA call (each case below breaks exactly one rule)."""
    base = dict(x=A, w=A, noisy=A, clean=None, mask=None, shift=None, shift_clean=None, gs=A, M=128, S=128,
                K=3072, mod_stride=0, eps=1e-6, q=A, sf=A, stream=None)

    def norm(match, **change):
        a = dict(base, **change)
        _rejects("qe_norm_scale_fp4", match, *a.values())

    norm("null argument", w=None)
    norm("needs `clean`", mask=A)
    norm("needs `shift_clean`", mask=A, clean=A, shift=A)
    norm("bad sizes", S=0)
    norm("multiple of 64", K=100)
    norm("above the supported", K=16448)
    norm("x must be 16-byte aligned", x=A + 8)
    norm("not a multiple of S", M=130)
    norm("negative mod_stride", mod_stride=-1)
    norm("x and w must be 16-byte aligned", w=A + 8)
    norm("q must be 8-byte", q=A + 4)
    norm("sf 4-byte", sf=A + 2)
    _rejects("qe_norm_scale_amax", "null amax", A, A, A, None, None, None, None, 128, 128, 3072, 0, 1e-6, None, None)

    silu = dict(gate=A, value=A, gs=A, M=128, K=12288, q=A, sf=A, table=A, stream=None)

    def silu_call(match, **change):
        a = dict(silu, **change)
        _rejects("qe_silu_mul_fp4", match, *a.values())

    silu_call("null argument", table=None)
    silu_call("bad sizes", M=-1)
    silu_call("multiple of 64", K=100)
    silu_call("16-byte aligned", gate=A + 8)
    silu_call("16-byte aligned", value=A + 8)
    silu_call("q must be 8-byte", q=A + 4)
    _rejects("qe_silu_mul_amax", "null amax", A, A, 128, 12288, A, None, None)
    _rejects("qe_silu_table_init", "16-byte aligned", A + 8, None)


def test_scatter_append_checks_its_geometry_first():
    peers = (ctypes.c_void_p * 2)(A, A)
    pl = _lib.planes(A, 0, 0, 1)
    err = A

    def scatter(match, n_peers=2, slice_bytes=16, pool=pl, src=pl, n_tokens=1):
        _rejects("qe_append_scatter", match, ctypes.cast(peers, ctypes.c_void_p), n_peers, pool, 4, src, 1,
                 slice_bytes, A, n_tokens, err, None)

    scatter("1..8 peer pools", n_peers=9)
    scatter("1..8 peer pools", n_peers=0)
    scatter("multiple of 16", slice_bytes=8)
    scatter("planes_inner", src=_lib.planes(A, 0, 0, 0))
    scatter("multiples of 16 bytes", pool=_lib.planes(A, 24, 0, 1))
    scatter("source must be 16-byte aligned", src=_lib.planes(A + 8, 0, 0, 1))


def test_nvfp4_numerics_setter_checks_its_fields():
    from qwenedit_b200.fp4 import NUMERICS, set_numerics

    for bad in (-1, 0x20, 0x40):
        with pytest.raises(ValueError, match="qe_set_nvfp4_numerics"):
            set_numerics(bad)
    assert NUMERICS == {"ieee": 0, "triton": 21}
    set_numerics("ieee")
    set_numerics("triton")  # the default, restored


def test_paged_attention_checks_arguments_before_any_cuda_call():
    from qwenedit_b200 import _lib
    from qwenedit_b200.attention import paged_attention

    q = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        paged_attention(q, None, 0, q, q)

    def call(**kw):
        args = dict(q=16, qt=512, qh=256, n_q=4, hq=2, kp=16, vp=16, rows=128, hkv=2, bt=16, page=64, n_pre=10,
                    kl=None, vl=None, lt=0, lh=0, n_loc=0, causal=0, scale=0.088, out=16, ot=512, oh=256, lse=None,
                    err=None, stream=None)
        args.update(kw)
        _lib.call("qe_paged_attention", *args.values())

    with pytest.raises(ValueError, match="multiple of heads_kv"):
        call(hq=3)
    with pytest.raises(ValueError, match="page_size"):
        call(page=12)
    with pytest.raises(ValueError, match="page_size"):
        call(page=4)
    with pytest.raises(ValueError, match="pool_rows"):
        call(rows=100)
    with pytest.raises(ValueError, match="null q"):
        call(q=None)
    with pytest.raises(ValueError, match="no keys"):
        call(n_pre=0)
    with pytest.raises(ValueError, match="16-byte"):
        call(qt=200)
    with pytest.raises(ValueError, match="scale"):
        call(scale=float("nan"))
    with pytest.raises(ValueError, match="null pool"):
        call(bt=None)
    with pytest.raises(ValueError, match="local"):
        call(n_loc=5)
    call(n_q=0)  # nothing to do: returns before touching the GPU

    def call_append(**kw):
        args = dict(q=16, qt=512, qh=256, n_q=4, hq=2, kp=16, vp=16, rows=128, hkv=2, bt=None, page=64, n_pre=0,
                    kl=16, vl=16, lt=512, lh=256, n_loc=4, causal=0, scale=0.088, out=16, ot=512, oh=256, lse=None,
                    app=16, err=16, stream=None)
        args.update(kw)
        _lib.call("qe_paged_attention_append", *args.values())

    with pytest.raises(ValueError, match="null append table"):
        call_append(app=None)
    with pytest.raises(ValueError, match="error flag"):
        call_append(err=None)
    with pytest.raises(ValueError, match="nothing to append"):
        call_append(n_loc=0, n_pre=10, bt=16)
    with pytest.raises(ValueError, match="no queries"):
        call_append(n_q=0)
    with pytest.raises(ValueError, match="page_size"):
        call_append(page=4)
    with pytest.raises(ValueError, match="null pool"):
        call_append(kp=None)
