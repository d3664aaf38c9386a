"""Golden-case definitions shared by gen_golden.py and the tests (inputs are regenerated from seeds)."""

from __future__ import annotations

import torch

from tests.golden import inputs

# RMSNorm + adaLN -> NVFP4. "fibo_mask" mirrors the reference GPU test's shape family (tests/test_fibo_fp4.py:41-49:
# x*3, weight U+0.5, mods [B, 4K]*0.3 with noisy/clean column slices, token mask, partial 128-row tile);
# "c4" the benchmark NVFP4 shape family (eps 1e-6, w = 1 + 0.02 N, scale 0.1 N, B = 1).
NORM_CASES = [
    dict(name="norm_fibo_mask", B=2, S=75, K=3584, eps=1e-5, x_scale=3.0, w_kind="uniform", mod_scale=0.3,
         mask=(20, 60), seed=11),
    dict(name="norm_c4", B=1, S=130, K=3072, eps=1e-6, x_scale=1.0, w_kind="one_plus", mod_scale=0.1,
         mask=None, seed=21),
    dict(name="norm_small_k", B=3, S=40, K=256, eps=1e-6, x_scale=1.0, w_kind="one_plus", mod_scale=0.2,
         mask=(5, 33), seed=31),
]

# SiLU * mul -> NVFP4: Fibo's K=9536 (partial last 1024-column block, tests/test_fibo_fp4.py:53-58) and
# the benchmark's 12288.
SILU_CASES = [
    dict(name="silu_fibo", M=40, K=9536, seed=41),
    dict(name="silu_c4", M=24, K=12288, seed=51),
    dict(name="silu_small", M=130, K=128, seed=61),
]


def norm_inputs(c: dict):
    B, S, K, seed = c["B"], c["S"], c["K"], c["seed"]
    x = inputs.bf16(seed, (B, S, K), scale=c["x_scale"])
    if c["w_kind"] == "uniform":
        w = torch.from_numpy((inputs.uniforms(seed + 1, K) + 0.5).astype("float32")).bfloat16()
    else:
        w = inputs.bf16(seed + 1, (K,), scale=0.02, shift=1.0)
    # one spare zero row after the B real rows: the reference kernel reads row B for its padding rows
    mods_full = torch.zeros(B + 1, 4 * K, dtype=torch.bfloat16)
    mods_full[:B] = inputs.bf16(seed + 2, (B, 4 * K), scale=c["mod_scale"])
    mask = None
    if c["mask"] is not None:
        mask = torch.zeros(S, dtype=torch.bool)
        mask[c["mask"][0]:c["mask"][1]] = True
    return x, w, mods_full, mask


def silu_inputs(c: dict):
    M, K, seed = c["M"], c["K"], c["seed"]
    return inputs.bf16(seed, (1, M, K)), inputs.bf16(seed + 1, (1, M, K))
