"""Pin the CPU oracle before trusting it: NVFP4 restatement vs the reference kernels' golden outputs, its
scalar primitives vs independent definitions, and the reference pool's data movement vs golden digests."""

import hashlib
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nvfp4_ref
from oracle.pool_ref import RefPagedKVPool
from tests.golden import cases, inputs

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def fp4_golden():
    return np.load(GOLDEN / "nvfp4.npz"), json.loads((GOLDEN / "nvfp4.json").read_text())


@pytest.mark.parametrize("case", cases.NORM_CASES, ids=lambda c: c["name"])
def test_oracle_norm_scale_matches_reference_kernel(fp4_golden, case):
    arrays, meta = fp4_golden
    x, w, mods_full, mask = cases.norm_inputs(case)
    K, B = case["K"], case["B"]
    noisy, clean = mods_full[:B, :K], mods_full[:B, K:2 * K]
    q, sf = nvfp4_ref.norm_scale_fp4_ref(x, w, case["eps"], noisy, clean if mask is not None else None, mask,
                                         meta[case["name"]]["gs"])
    np.testing.assert_array_equal(q, arrays[case["name"] + "_q"])
    np.testing.assert_array_equal(sf, arrays[case["name"] + "_sf"])


@pytest.mark.parametrize("case", cases.SILU_CASES, ids=lambda c: c["name"])
def test_oracle_silu_mul_matches_reference_kernel(fp4_golden, case):
    arrays, meta = fp4_golden
    gate, value = cases.silu_inputs(case)
    q, sf = nvfp4_ref.silu_mul_fp4_ref(gate, value, meta[case["name"]]["gs"])
    np.testing.assert_array_equal(q, arrays[case["name"] + "_q"])
    np.testing.assert_array_equal(sf, arrays[case["name"] + "_sf"])


def test_padding_rows_hold_zero_scales(fp4_golden):
    arrays, _ = fp4_golden
    for c in cases.NORM_CASES:
        m = c["B"] * c["S"]
        sf = arrays[c["name"] + "_sf"]
        K = c["K"]
        rows = np.arange(m, sf.shape[0])
        for g in range(K // 16):
            off = (rows // 128) * (K // 64 * 512) + (g // 4) * 512 + (rows % 32) * 16 + (rows % 128 // 32) * 4 + g % 4
            assert (sf.reshape(-1)[off] == 0).all()


def test_e4m3_matches_torch_below_saturation():
    v = torch.from_numpy(inputs.normal(5, (20000,), scale=60.0).astype(np.float32))
    v = torch.cat([v, torch.tensor([0.0, 2 ** -10, 2 ** -9, 1.5 * 2 ** -9, 447.0, 440.0, 0.1, -3.3])])
    v = v[v.abs() < 448]
    ours = np.array([nvfp4_ref.lib().ref_e4m3(float(x)) for x in v], np.uint8)
    theirs = v.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, theirs)
    assert nvfp4_ref.lib().ref_e4m3(1e6) == 0x7E and nvfp4_ref.lib().ref_e4m3(math.inf) == 0x7E


def test_e2m1_thresholds():
    f = nvfp4_ref.lib().ref_e2m1
    grid = {0.0: 0, 0.25: 0, 0.2501: 1, 0.75: 2, 1.25: 2, 1.2501: 3, 1.75: 4, 2.5: 4, 2.51: 5, 3.5: 6, 5.0: 6,
            5.01: 7, 100.0: 7}
    for v, code in grid.items():
        assert f(v) == code and f(-v) == (code | 8 if v != 0 else 0)


def test_exp_within_one_ulp():
    xs = np.linspace(-100, 88, 200001, dtype=np.float32)
    ours = np.array([nvfp4_ref.lib().ref_exp(float(x)) for x in xs[::7]], np.float32)
    exact = np.exp(xs[::7].astype(np.float64))
    ulp = np.spacing(exact.astype(np.float32)).astype(np.float64)
    assert (np.abs(ours - exact) / ulp).max() < 1.0


def test_pairwise_sum_is_numpy_sum():
    from ctypes import POINTER, c_float

    for n in (1, 7, 8, 9, 100, 128, 129, 1000, 3072, 4096, 5000):
        a = (inputs.normal(n, (n,)) ** 2).astype(np.float32)
        got = nvfp4_ref.lib().ref_pairwise_sum(a.ctypes.data_as(POINTER(c_float)), n)
        assert np.float32(got) == np.sum(a)


@pytest.mark.parametrize("name", ["tiny", "c1_slice", "bf16"])
def test_reference_pool_data_movement_matches_golden(name):
    digests = json.loads((GOLDEN / "paged.json").read_text())[name]
    L, H, D, cap, n, dtype = {"tiny": (2, 2, 8, 64, 24, torch.float32), "c1_slice": (4, 24, 128, 1024, 700, torch.float32),
                              "bf16": (3, 4, 16, 256, 100, torch.bfloat16)}[name]
    seed = int(hashlib.sha256(name.encode()).hexdigest()[:8], 16)
    elem = torch.empty((), dtype=dtype).element_size()
    pool = RefPagedKVPool("t", L, H, D, cap * L * 2 * H * D * elem, dtype)
    pool.kv = inputs.f32(seed, (L, 2, cap + 1, H, D)).to(dtype)
    idx = torch.from_numpy(inputs.permutation(seed + 1, cap)[:n] + 1)
    got = pool.gather(idx)
    view = pool.gather(torch.arange(5, 5 + n))
    assert view.data_ptr() == pool.kv[:, :, 5].data_ptr()
    pool.write(idx, inputs.f32(seed + 2, (L, 2, n, H, D)).to(dtype))
    sha = lambda t: hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()  # noqa: E731
    assert sha(got) == digests["gather"]
    assert sha(pool.kv) == digests["write"]
    assert pool.stats.gathers == 1 and pool.stats.contiguous_views == 1


def test_latent_oracle_matches_reference_golden():
    """oracle/latents_ref.py against the reference's own MaskState.blend and stored_latents crop
    (tests/golden/gen_golden.py, latents.npz): bit-exact on CPU."""
    import torch

    from oracle import latents_ref
    from tests.golden.gen_golden import CROP_CASES, LATENT_CASES, latent_inputs

    gold = np.load(Path(__file__).resolve().parent / "golden" / "latents.npz")
    for case in LATENT_CASES:
        lat, x0, eps, m = latent_inputs(case)
        sigma = torch.tensor(case["sigma"]) if case["sigma_kind"] == "tensor" else case["sigma"]
        got = latents_ref.blend(lat, x0, eps, m, sigma)
        bits = torch.int32 if got.dtype == torch.float32 else torch.int16
        np.testing.assert_array_equal(got.contiguous().view(bits).numpy(), gold[case["name"]])
    for case in CROP_CASES:
        dt = torch.bfloat16 if "bf16" in case["name"] else torch.float32
        lat = inputs.f32(case["seed"], (1, case["h"] * case["w"], case["C"])).to(dt)
        got = latents_ref.crop(lat, (case["h"], case["w"]), case["box"])
        bits = torch.int32 if got.dtype == torch.float32 else torch.int16
        np.testing.assert_array_equal(got.contiguous().view(bits).numpy(), gold[case["name"]])
