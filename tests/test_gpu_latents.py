"""Per-step latent kernels on the GPU, bit-exact against the reference's eager torch ops (oracle/latents_ref.py):
the mask blend in bf16 / fp16 / fp32 with broadcast x0 and mask, fp32 or latent-dtype masks, tensor and Python
float sigmas (including 0 and 1); compose and crop for boxes at the edges and inside the grid."""

import pytest
import torch

from oracle import latents_ref
from qwenedit_b200 import latents

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(B, N, C, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(B, N, C, generator=g).to(dtype)
    x0 = torch.randn(1, N, C, generator=g).to(dtype)
    eps = torch.randn(B, N, C, generator=g).to(dtype)
    m = torch.rand(1, N, 1, generator=g)
    m[:, : N // 4] = 0.0
    m[:, N // 4 : N // 2] = 1.0  # hard zeros and ones next to the feathered edge
    return [t.to(DEV) for t in (lat, x0, eps, m)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("B", [1, 2])
@pytest.mark.parametrize("sigma", [0.0, 0.37, 1.0, "py"])
def test_mask_blend_matches_eager(dtype, B, sigma):
    lat, x0, eps, m = _case(B, 4096, 64, dtype, seed=B * 10)
    s = 0.6180339887 if sigma == "py" else torch.tensor(sigma, dtype=torch.float32, device=DEV)
    want = latents_ref.blend(lat, x0, eps, m, s)
    got = latents.mask_blend(lat, x0, eps, m, s)
    assert got.dtype == want.dtype and got.shape == want.shape
    assert torch.equal(got, want)


def test_mask_blend_latent_dtype_mask_per_channel():
    lat, x0, eps, _ = _case(2, 1024, 16, torch.bfloat16, seed=5)
    g = torch.Generator().manual_seed(6)
    m = torch.rand(2, 1024, 16, generator=g).bfloat16().to(DEV)
    s = torch.tensor(0.25, dtype=torch.bfloat16, device=DEV)
    assert torch.equal(latents.mask_blend(lat, x0, eps, m, s), latents_ref.blend(lat, x0, eps, m, s))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_mask_blend_element_path(dtype):
    """Shapes the 8-channel vector kernel does not take (C not a multiple of 8; latents 2 elements off a 16-byte
    boundary) run the per-element kernel, with the same result as eager."""
    lat, x0, eps, m = _case(2, 999, 12, dtype, seed=7)
    s = torch.tensor(0.41, dtype=torch.float32, device=DEV)
    assert torch.equal(latents.mask_blend(lat, x0, eps, m, s), latents_ref.blend(lat, x0, eps, m, s))
    lat, x0, eps, m = _case(1, 512, 64, dtype, seed=8)
    buf = torch.empty(lat.numel() + 1, dtype=dtype, device=DEV)
    shifted = buf[1:].view(lat.shape)
    shifted.copy_(lat)
    assert torch.equal(latents.mask_blend(shifted, x0, eps, m, s), latents_ref.blend(lat, x0, eps, m, s))


@pytest.mark.parametrize("box", [(0, 0, 64, 64), (3, 5, 17, 40), (60, 0, 64, 1), (0, 63, 64, 64)])
@pytest.mark.parametrize("C,dtype", [(64, torch.bfloat16), (16, torch.float32), (3, torch.float16)])
def test_compose_and_crop_match_eager(box, C, dtype):
    h = w = 64
    g = torch.Generator().manual_seed(C)
    base = torch.randn(1, h * w, C, generator=g).to(dtype).to(DEV)
    x0, y0, x1, y1 = box
    piece = torch.randn(1, (y1 - y0) * (x1 - x0), C, generator=g).to(DEV)  # fp32: converted to the base dtype
    assert torch.equal(latents.compose(base, (h, w), piece, box), latents_ref.compose(base, (h, w), piece, box))
    assert torch.equal(latents.crop(base, (h, w), box), latents_ref.crop(base, (h, w), box))


def test_bad_boxes_raise():
    base = torch.zeros(1, 16, 4, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        latents.crop(base, (4, 4), (0, 0, 5, 1))
    with pytest.raises(ValueError):
        latents.compose(base, (4, 4), torch.zeros(1, 1, 4, device=DEV), (2, 2, 2, 3))


def test_kernels_match_reference_golden():
    """The kernels against the reference's own MaskState.blend / stored_latents outputs (latents.npz, made by
    tests/golden/gen_golden.py from the reference code on CPU)."""
    from pathlib import Path

    import numpy as np

    from tests.golden.gen_golden import CROP_CASES, LATENT_CASES, latent_inputs
    from tests.golden import inputs

    gold = np.load(Path(__file__).resolve().parent / "golden" / "latents.npz")
    for case in LATENT_CASES:
        lat, x0, eps, m = (t.to(DEV) for t in latent_inputs(case))
        sigma = (torch.tensor(case["sigma"], device=DEV) if case["sigma_kind"] == "tensor" else case["sigma"])
        got = latents.mask_blend(lat, x0, eps, m, sigma).cpu()
        bits = torch.int32 if got.dtype == torch.float32 else torch.int16
        np.testing.assert_array_equal(got.view(bits).numpy(), gold[case["name"]], err_msg=case["name"])
    for case in CROP_CASES:
        dt = torch.bfloat16 if "bf16" in case["name"] else torch.float32
        lat = inputs.f32(case["seed"], (1, case["h"] * case["w"], case["C"])).to(dt).to(DEV)
        got = latents.crop(lat, (case["h"], case["w"]), case["box"]).cpu()
        bits = torch.int32 if got.dtype == torch.float32 else torch.int16
        np.testing.assert_array_equal(got.view(bits).numpy(), gold[case["name"]], err_msg=case["name"])


def test_reference_blend_keeps_source_outside_at_sigma_zero():
    """tests/test_core.py:59-63 of the reference, on the kernel."""
    g = torch.Generator().manual_seed(3)
    x0 = torch.randn(1, 4, 3, generator=g).to(DEV)
    eps = torch.randn(1, 4, 3, generator=g).to(DEV)
    out = latents.mask_blend(torch.zeros(1, 4, 3, device=DEV), x0, eps,
                             torch.tensor([1.0, 0, 0, 1], device=DEV).view(1, 4, 1), 0.0)
    assert torch.equal(out[0, 1], x0[0, 1]) and torch.equal(out[0, 0], torch.zeros(3, device=DEV))


def test_compose_hook_stores_the_new_version():
    """hooks.compose against the reference's _compose sequence (oracle restatement): the stored version, its
    grid, and the two refusals (missing base, box not matching the crop grid)."""
    from qwenedit_b200 import hooks, state

    h, w, C = 12, 16, 16
    g = torch.Generator().manual_seed(9)
    base = torch.randn(1, h * w, C, generator=g).bfloat16().to(DEV)
    piece = torch.randn(1, 4 * 5, C, generator=g).to(DEV)
    state.OUTPUT_LATENTS.put("v1", base)
    state.OUTPUT_GRID["v1"] = (h, w)
    assert hooks.compose({"base": "v1", "as": "v2", "box": (3, 2, 8, 6)}, piece, (4, 5))
    want = latents_ref.compose(base, (h, w), piece, (3, 2, 8, 6))
    assert torch.equal(state.OUTPUT_LATENTS.get("v2"), want) and state.OUTPUT_GRID["v2"] == (h, w)
    assert not hooks.compose({"base": "missing", "as": "v3", "box": (0, 0, 1, 1)}, piece, (1, 1))
    assert not hooks.compose({"base": "v1", "as": "v3", "box": (0, 0, 2, 2)}, piece, (4, 5))
    assert state.OUTPUT_LATENTS.get("v3") is None
