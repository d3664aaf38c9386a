"""Fused NVFP4 kernels on the GPU: bit-exact against the reference kernels' golden outputs
(multi_turn/fibo/fp4.py run by tests/golden/gen_golden.py) and against the C oracle over the BASELINE NVFP4
shapes, the reference test's shapes (tests/test_fibo_fp4.py:39-58) and edge cases.

Tolerance (stated by the build's spec for NVFP4): bit-exact codes and scales, or <= 1 code step on <= 1e-4 of
elements with the dequantised max-abs error reported. These tests require bit-exact."""

import json
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import nvfp4_ref
from qwenedit_b200.fp4 import Quantized, norm_scale_fp4, silu_mul_fp4, silu_table
from tests.golden import cases, inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "nvfp4.npz"), json.loads((GOLDEN / "nvfp4.json").read_text())


def _gs(value):
    return torch.tensor([value], dtype=torch.float32, device=DEV)


@pytest.mark.parametrize("case", cases.NORM_CASES, ids=lambda c: c["name"])
def test_norm_scale_matches_reference_golden(golden, case):
    arrays, meta = golden
    x, w, mods_full, mask = cases.norm_inputs(case)
    K, B = case["K"], case["B"]
    mods = mods_full.to(DEV)
    noisy, clean = mods[:B, :K], mods[:B, K:2 * K]  # strided column slices of one [B, 4K] tensor
    norm = SimpleNamespace(weight=w.to(DEV), eps=case["eps"])
    out = norm_scale_fp4(x.to(DEV), norm, noisy, clean, None if mask is None else mask.to(DEV),
                         _gs(meta[case["name"]]["gs"]))
    assert isinstance(out, Quantized) and out.shape == x.shape
    np.testing.assert_array_equal(out.q.cpu().numpy(), arrays[case["name"] + "_q"])
    np.testing.assert_array_equal(out.sf.cpu().numpy(), arrays[case["name"] + "_sf"])


@pytest.mark.parametrize("case", cases.SILU_CASES, ids=lambda c: c["name"])
def test_silu_mul_matches_reference_golden(golden, case):
    arrays, meta = golden
    gate, value = cases.silu_inputs(case)
    out = silu_mul_fp4(gate.to(DEV), value.to(DEV), _gs(meta[case["name"]]["gs"]))
    np.testing.assert_array_equal(out.q.cpu().numpy(), arrays[case["name"] + "_q"])
    np.testing.assert_array_equal(out.sf.cpu().numpy(), arrays[case["name"] + "_sf"])


def _norm_case(B, S, K, eps, masked, shift, seed, x_scale=1.0):
    x = inputs.bf16(seed, (B, S, K), scale=x_scale)
    w = inputs.bf16(seed + 1, (K,), scale=0.02, shift=1.0)
    scale = inputs.bf16(seed + 2, (B, K), scale=0.1)
    clean = inputs.bf16(seed + 3, (B, K), scale=0.1) if masked else None
    mask = None
    if masked:
        mask = torch.from_numpy(inputs.uniforms(seed + 4, S) < 0.5)
    sh = inputs.bf16(seed + 5, (B, K), scale=0.1) if shift else None
    sh_clean = inputs.bf16(seed + 6, (B, K), scale=0.1) if (shift and masked) else None
    y = nvfp4_ref.bf16_values_norm_scale(x, w, eps, scale, clean, mask, sh, sh_clean)
    gs = nvfp4_ref.global_scale(y)
    q_ref, sf_ref = nvfp4_ref.norm_scale_fp4_ref(x, w, eps, scale, clean, mask, gs, sh, sh_clean)
    to = lambda t: None if t is None else t.to(DEV)  # noqa: E731
    out = norm_scale_fp4(to(x), SimpleNamespace(weight=to(w), eps=eps), to(scale), to(clean), to(mask), _gs(gs),
                         shift=to(sh), shift_clean=to(sh_clean))
    return out, q_ref, sf_ref


@pytest.mark.parametrize("T", [4096, 16384])
@pytest.mark.parametrize("shift", [False, True])
def test_norm_scale_baseline_shapes(T, shift):
    """BASELINE NVFP4: x [1, T, 3072] ~N(0,1), eps 1e-6, w ~ 1 + 0.02 N, scale/shift ~ 0.1 N."""
    out, q_ref, sf_ref = _norm_case(1, T, 3072, 1e-6, False, shift, seed=T + shift)
    np.testing.assert_array_equal(out.q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(out.sf.cpu().numpy(), sf_ref)


@pytest.mark.parametrize("K", [64, 128, 192, 1024, 3584, 4096, 4160, 8192, 12288])
def test_norm_scale_widths_masks_batches(K):
    out, q_ref, sf_ref = _norm_case(3, 67, K, 1e-5, True, K % 3 == 0, seed=K, x_scale=3.0)
    np.testing.assert_array_equal(out.q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(out.sf.cpu().numpy(), sf_ref)


@pytest.mark.parametrize("M,K", [(4096, 12288), (300, 9536), (1, 64), (129, 640)])
def test_silu_mul_shapes(M, K):
    gate = inputs.bf16(M + K, (1, M, K))
    value = inputs.bf16(M + K + 1, (1, M, K))
    y = (torch.nn.functional.silu(gate.float()).bfloat16().float() * value.float()).bfloat16()
    gs = nvfp4_ref.global_scale(y)
    q_ref, sf_ref = nvfp4_ref.silu_mul_fp4_ref(gate, value, gs)
    out = silu_mul_fp4(gate.to(DEV), value.to(DEV), _gs(gs))
    np.testing.assert_array_equal(out.q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(out.sf.cpu().numpy(), sf_ref)


def test_extreme_values_saturate_like_the_oracle():
    """Outliers far above the calibrated range (sf saturates at 448), exact zeros, tiny values (subnormal e4m3)."""
    gate = inputs.bf16(5, (1, 256, 256), scale=4.0)
    gate[0, :8] = 0
    gate[0, 8:16] *= 1e-30
    gate[0, 16, :16] = 3e4
    value = inputs.bf16(6, (1, 256, 256))
    for gs in (50.0, 1e4, 1e-3):
        q_ref, sf_ref = nvfp4_ref.silu_mul_fp4_ref(gate, value, gs)
        out = silu_mul_fp4(gate.to(DEV), value.to(DEV), _gs(gs))
        np.testing.assert_array_equal(out.q.cpu().numpy(), q_ref)
        np.testing.assert_array_equal(out.sf.cpu().numpy(), sf_ref)


def test_argument_errors():
    x = torch.zeros(1, 4, 100, dtype=torch.bfloat16, device=DEV)
    norm = SimpleNamespace(weight=torch.ones(100, dtype=torch.bfloat16, device=DEV), eps=1e-6)
    with pytest.raises(ValueError, match="multiple of 64"):
        norm_scale_fp4(x, norm, torch.zeros(1, 100, dtype=torch.bfloat16, device=DEV), None, None, _gs(1.0))
    with pytest.raises(TypeError):
        silu_mul_fp4(torch.zeros(4, 64, device=DEV), torch.zeros(4, 64, device=DEV), _gs(1.0))
    with pytest.raises(RuntimeError, match="CUDA"):
        silu_mul_fp4(torch.zeros(4, 64, dtype=torch.bfloat16), torch.zeros(4, 64, dtype=torch.bfloat16), _gs(1.0))


def test_silu_table_is_exact_for_every_bf16_input():
    """The SiLU table (one entry per bf16 bit pattern) equals the oracle's bf16(g / (1 + exp(-g))) for all 65,536
    inputs; NaN inputs (and -inf, which gives inf/inf) map to a NaN on both sides."""
    table = silu_table(DEV).cpu().numpy().view(np.uint16)
    ref = np.array([nvfp4_ref.lib().ref_silu_bf16(i) for i in range(65536)], np.uint16)
    g = np.arange(65536, dtype=np.uint32)
    nan_in = ((g & 0x7F80) == 0x7F80) & ((g & 0x7F) != 0)
    neg_inf = g == 0xFF80
    def is_nan(bits):
        return ((bits & 0x7F80) == 0x7F80) & ((bits & 0x7F) != 0)
    special = nan_in | neg_inf
    assert is_nan(table[special]).all() and is_nan(ref[special]).all()
    np.testing.assert_array_equal(table[~special], ref[~special])
