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
    for fn, bad in (("qe_set_norm_table_mode", 3), ("qe_set_silu_table_mode", 3), ("qe_set_silu_pipeline", 3),
                    ("qe_set_paged_copy_mode", 5)):
        with pytest.raises(ValueError):
            _lib.call(fn, bad)



def test_no_alloc_append_rejects_a_null_source_pointer():
    host = (ctypes.c_void_p * 2)(4096, None)
    with pytest.raises(ValueError, match="null source pointer 1"):
        _lib.call("qe_append_slots_ptrs_noalloc", _lib.planes(16, 0, 0, 1), 4, ctypes.cast(host, ctypes.c_void_p), 2,
                  16, 16, 1, None, None)
