"""Generate the golden fixtures under tests/golden/ by running the REFERENCE (QwenEdit) code itself.

    python -m tests.golden.gen_golden --reference <QwenEdit checkout>   (or QWENEDIT_REFERENCE=<checkout>)

Runs only where the reference checkout exists (it is read, never modified); the fixtures it writes are what
the tests use everywhere else. What it runs:

* keys   — multi_turn/cache/keys.py (pure Python/numpy, imported as is) on seeded layouts
           -> keys.npz / keys.json
* nvfp4  — the reference Triton kernels multi_turn/fibo/fp4.py:64-116 under TRITON_INTERPRET=1 on CPU,
           with the interpreter's float conversions replaced by the GPU's (fp32->bf16 round-to-nearest-even,
           fp32->e4m3 round-to-nearest-even with saturation; the stock interpreter truncates to bf16 and
           rounds e4m3 half-up without saturation). sglang-dependent imports of fibo/fp4.py are stubbed:
           ``multi_turn.fibo.dit`` only supplies two eager helpers the kernels never call.
           -> nvfp4.npz (q, sf, gs per case) + nvfp4.json (raw-interpreter agreement, for the record)
* paged  — multi_turn/cache/paged.py's own ``gather`` / ``write`` methods (pure torch: a view or
           index_select, index_copy_) on a seeded pool, with the sglang imports stubbed (the tree is not used)
           -> paged.npz
* latents — multi_turn/pipeline/masking.py's ``MaskState.blend`` and multi_turn/state.py's ``stored_latents``
           crop, imported as is, on seeded latents -> latents.npz
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from tests.golden import cases, inputs  # noqa: E402


def _stub(name: str, **attrs) -> types.ModuleType:
    mod = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(mod, k, v)
    sys.modules[name] = mod
    return mod


def import_reference(ref: Path):
    sys.path.insert(0, str(ref))
    # sglang is not installed: provide the names paged.py imports (never exercised here)
    class _Dummy:
        def __init__(self, *a, **k):
            raise RuntimeError("sglang stub")

    for name in ["sglang", "sglang.srt", "sglang.srt.mem_cache", "sglang.srt.mem_cache.allocator"]:
        _stub(name)
    _stub("sglang.srt.mem_cache.allocator.token", TokenToKVPoolAllocator=_Dummy)
    _stub("sglang.srt.mem_cache.base_prefix_cache", EvictParams=_Dummy, InsertParams=_Dummy,
          MatchPrefixParams=_Dummy)
    _stub("sglang.srt.mem_cache.radix_cache", RadixCache=_Dummy, RadixKey=_Dummy)
    # fibo/fp4.py imports two eager helpers from fibo/dit.py (which needs sglang); the kernels do not use them
    _stub("multi_turn.fibo.dit", _norm_scale=None, silu_mul=None)


# ---- GPU-faithful float conversions for the Triton interpreter ---------------------------------
def _f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    return np.where(nan, ((u >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16), r)


def _f32_to_e4m3_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    v = a.astype(np.float64)
    mag = np.abs(v)
    sign = np.where(np.signbit(a), 0x80, 0).astype(np.uint8)
    out = np.zeros(a.shape, np.uint8)
    with np.errstate(divide="ignore", invalid="ignore"):
        _, e = np.frexp(mag)
        E = np.maximum(e.astype(np.int64) - 1, -6)
        spacing = np.ldexp(1.0, E - 3)
        qv = np.rint(mag / spacing)
    carry = qv >= 16
    qv = np.where(carry, 8, qv)
    E = np.where(carry, E + 1, E)
    normal_bits = (((E + 7) << 3) | (qv.astype(np.int64) - 8)).astype(np.int64)
    sub = (E == -6) & (qv < 8)
    bits = np.where(sub, qv.astype(np.int64), normal_bits)
    bits = np.where(mag == 0, 0, bits)
    bits = np.where(mag >= 448.0, 0x7E, bits)
    out = (bits.astype(np.uint8) | sign)
    return np.where(np.isnan(v), np.uint8(0x7F), out).astype(np.uint8)


def _e4m3_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = b.astype(np.uint32)
    e, m = (b >> 3) & 15, b & 7
    mag = np.where(e == 0, m.astype(np.float64) * 2.0 ** -9, np.ldexp((8 + m).astype(np.float64), e.astype(np.int64) - 10))
    mag = np.where((e == 15) & (m == 7), np.nan, mag)
    return np.where(b & 0x80, -mag, mag).astype(np.float32).view(np.uint32)


def patch_interpreter_conversions():
    import triton.language as tl
    from triton.runtime import interpreter

    original = interpreter._convert_float

    def convert(inp, input_dtype, output_dtype, rounding_mode):
        if input_dtype == tl.float32 and output_dtype == tl.bfloat16:
            return _f32_to_bf16_bits(inp.view(np.float32)).reshape(inp.shape)
        if input_dtype == tl.bfloat16 and output_dtype == tl.float32:
            return (inp.view(np.uint16).astype(np.uint32) << np.uint32(16)).reshape(inp.shape)
        if input_dtype == tl.float32 and output_dtype == tl.float8e4nv:
            return _f32_to_e4m3_bits(inp.view(np.float32)).reshape(inp.shape)
        if input_dtype == tl.float8e4nv and output_dtype == tl.float32:
            return _e4m3_bits_to_f32(inp.view(np.uint8)).reshape(inp.shape)
        return original(inp, input_dtype, output_dtype, rounding_mode)

    interpreter._convert_float = convert
    return lambda: setattr(interpreter, "_convert_float", original)


# ---- cases ------------------------------------------------------------------------------------
def gen_keys(out: Path):
    from PIL import Image

    from multi_turn.cache import keys

    arrays, meta = {}, {}
    root = keys.root_key("dit", "Qwen/Qwen-Image-2.1", None, None, None)
    img_a = Image.frombytes("RGB", (24, 16), bytes((np.arange(24 * 16 * 3) * 7 % 251).astype(np.uint8)))
    img_b = Image.frombytes("RGB", (24, 16), bytes((np.arange(24 * 16 * 3) * 11 % 253).astype(np.uint8)))
    k_a, k_b = keys.image_content_key(img_a), keys.image_content_key(img_b)
    meta["root"] = root.hex()
    meta["image_key_a"] = k_a.hex()
    meta["image_key_b"] = k_b.hex()
    meta["latent_key"] = keys.latent_key("session/v3").hex()
    # DiT layout: text header, image block (32x32 latent tokens), text tail; then a two-image layout
    seg1 = [(0, 40, False), (40, 40 + 32 * 32, True), (1064, 1100, False)]
    text_ids = (np.arange(200) * 37 % 1511 + 3).tolist()
    tidx1 = list(range(40)) + [40] * (32 * 32) + list(range(41, 77))
    arrays["vids_one_image"] = keys.virtual_ids(root, seg1, tidx1, text_ids, [k_a], [(32, 32)])
    seg2 = [(0, 10, False), (10, 10 + 16 * 8, True), (138, 150, False), (150, 150 + 8 * 8, True), (214, 230, False)]
    tidx2 = list(range(10)) + [10] * 128 + list(range(11, 23)) + [23] * 64 + list(range(24, 40))
    arrays["vids_two_images"] = keys.virtual_ids(root, seg2, tidx2, text_ids, [k_a, k_b], [(16, 8), (8, 8)])
    meta["vids_one_image"] = dict(segments=seg1, text_indices=tidx1, image_keys=["a"], image_shapes=[(32, 32)])
    meta["vids_two_images"] = dict(segments=seg2, text_indices=tidx2, image_keys=["a", "b"],
                                   image_shapes=[(16, 8), (8, 8)])
    meta["text_ids"] = text_ids
    enc_root = keys.root_key("encoder", "Qwen2.5-VL", None)
    meta["encoder_root"] = enc_root.hex()
    toks = (np.arange(300) * 13 % 997).tolist()
    runs = [(20, 120, k_a), (200, 240, k_b)]
    arrays["seq_two_runs"] = keys.sequence_ids(enc_root, toks, runs)
    arrays["seq_no_runs"] = keys.sequence_ids(enc_root, toks[:50], [])
    meta["seq_tokens"] = toks
    meta["seq_two_runs"] = [(20, 120, "a"), (200, 240, "b")]
    np.savez_compressed(out / "keys.npz", **arrays)
    (out / "keys.json").write_text(json.dumps(meta, indent=1))


def _run_norm(fp4, c):
    x, w, mods_full, mask = cases.norm_inputs(c)
    K = c["K"]
    noisy, clean = mods_full[: c["B"], :K], mods_full[: c["B"], K:2 * K]
    norm = types.SimpleNamespace(weight=w, eps=c["eps"])
    # calibration as the reference does it: gs from the BF16 values' amax with headroom 4
    from oracle.nvfp4_ref import bf16_values_norm_scale, global_scale

    y = bf16_values_norm_scale(x, w, c["eps"], noisy, clean if mask is not None else None, mask)
    gs = torch.tensor([global_scale(y)], dtype=torch.float32)
    out = fp4.norm_scale_fp4(x, norm, noisy, clean, mask, gs)
    return out.q.numpy().copy(), out.sf.numpy().copy(), float(gs)


def _run_silu(fp4, c):
    gate, value = cases.silu_inputs(c)
    y = (torch.nn.functional.silu(gate.float()).bfloat16().float() * value.float()).bfloat16()
    from oracle.nvfp4_ref import global_scale

    gs = torch.tensor([global_scale(y)], dtype=torch.float32)
    out = fp4.silu_mul_fp4(gate, value, gs)
    return out.q.numpy().copy(), out.sf.numpy().copy(), float(gs)


def gen_nvfp4(out: Path):
    os.environ["TRITON_INTERPRET"] = "1"
    from multi_turn.fibo import fp4

    arrays, meta = {}, {}
    restore = patch_interpreter_conversions()
    try:
        for c in cases.NORM_CASES:
            q, sf, gs = _run_norm(fp4, c)
            arrays[c["name"] + "_q"], arrays[c["name"] + "_sf"] = q, sf
            meta[c["name"]] = dict(gs=gs)
        for c in cases.SILU_CASES:
            q, sf, gs = _run_silu(fp4, c)
            arrays[c["name"] + "_q"], arrays[c["name"] + "_sf"] = q, sf
            meta[c["name"]] = dict(gs=gs)
    finally:
        restore()
    # for the record: how far the stock interpreter (bf16 truncation, unsaturated half-up e4m3) is from it
    for c in cases.NORM_CASES + cases.SILU_CASES:
        runner = _run_norm if c in cases.NORM_CASES else _run_silu
        q, sf, _ = runner(fp4, c)
        meta[c["name"]]["stock_interpreter_q_equal"] = float((q == arrays[c["name"] + "_q"]).mean())
        meta[c["name"]]["stock_interpreter_sf_equal"] = float((sf == arrays[c["name"] + "_sf"]).mean())
    np.savez_compressed(out / "nvfp4.npz", **arrays)
    (out / "nvfp4.json").write_text(json.dumps(meta, indent=1))


def gen_paged(out: Path):
    from multi_turn.cache.paged import PagedKVPool, PoolStats

    arrays = {}
    digests = {}
    for name, (L, H, D, cap, n, dtype) in {
        "tiny": (2, 2, 8, 64, 24, torch.float32),
        "c1_slice": (4, 24, 128, 1024, 700, torch.float32),
        "bf16": (3, 4, 16, 256, 100, torch.bfloat16),
    }.items():
        pool = PagedKVPool.__new__(PagedKVPool)
        pool.kv = inputs.f32(hash_seed(name), (L, 2, cap + 1, H, D)).to(dtype)
        pool.stats = PoolStats()
        perm = inputs.permutation(hash_seed(name) + 1, cap)[:n] + 1
        idx = torch.from_numpy(perm)
        got = pool.gather(idx)
        run = torch.arange(5, 5 + n)
        view = pool.gather(run)
        is_view = view.data_ptr() == pool.kv[:, :, 5].data_ptr()
        new = inputs.f32(hash_seed(name) + 2, (L, 2, n, H, D)).to(dtype)
        pool.write(idx, new)
        after = pool.kv
        digests[name] = dict(
            gather=hashlib.sha256(got.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest(),
            write=hashlib.sha256(after.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest(),
            contiguous_is_view=bool(is_view), stats=pool.stats.__dict__,
        )
        if name == "tiny":
            arrays["tiny_idx"] = perm
            arrays["tiny_gather"] = got.numpy()
            arrays["tiny_after_write"] = after.numpy()
    np.savez_compressed(out / "paged.npz", **arrays)
    (out / "paged.json").write_text(json.dumps(digests, indent=1))


# per-step latent ops: the reference's own MaskState.blend (pipeline/masking.py:82-89) and stored_latents crop
# (state.py:52-62), run on CPU torch (the same op-by-op fp32-then-round arithmetic as on the GPU)
LATENT_CASES = [
    dict(name="blend_bf16", dtype="bfloat16", B=2, N=256, C=16, sigma=0.37, sigma_kind="tensor", seed=501),
    dict(name="blend_fp16_float_sigma", dtype="float16", B=1, N=512, C=8, sigma=0.618, sigma_kind="float", seed=502),
    dict(name="blend_fp32_sigma0", dtype="float32", B=2, N=128, C=4, sigma=0.0, sigma_kind="tensor", seed=503),
    dict(name="blend_bf16_sigma1", dtype="bfloat16", B=1, N=64, C=64, sigma=1.0, sigma_kind="tensor", seed=504),
]
CROP_CASES = [dict(name="crop_bf16", h=16, w=24, C=16, box=(3, 2, 17, 9), seed=601),
              dict(name="crop_fp32_full_width", h=8, w=8, C=4, box=(0, 1, 8, 5), seed=602)]


def latent_inputs(case):
    dt = getattr(torch, case["dtype"])
    B, N, C, seed = case["B"], case["N"], case["C"], case["seed"]
    lat = inputs.f32(seed, (B, N, C)).to(dt)
    x0 = inputs.f32(seed + 1, (1, N, C)).to(dt)
    eps = inputs.f32(seed + 2, (B, N, C)).to(dt)
    m = torch.from_numpy(inputs.uniforms(seed + 3, N).astype(np.float32)).view(1, N, 1)
    m[:, : N // 4] = 0.0
    m[:, N // 4 : N // 2] = 1.0
    return lat, x0, eps, m


def gen_latents(out: Path) -> None:
    from multi_turn import state as ref_state
    from multi_turn.pipeline.masking import MaskState

    arrays = {}
    for case in LATENT_CASES:
        lat, x0, eps, m = latent_inputs(case)
        sigma = torch.tensor(case["sigma"]) if case["sigma_kind"] == "tensor" else case["sigma"]
        got = MaskState(x0=x0, editable=m, eps=eps).blend(lat, sigma)
        bits = torch.int32 if got.dtype == torch.float32 else torch.int16
        arrays[case["name"]] = got.contiguous().view(bits).numpy()
    for case in CROP_CASES:
        h, w, C = case["h"], case["w"], case["C"]
        dt = torch.bfloat16 if "bf16" in case["name"] else torch.float32
        lat = inputs.f32(case["seed"], (1, h * w, C)).to(dt)
        ref_state.OUTPUT_LATENTS.put(case["name"], lat)
        ref_state.OUTPUT_GRID[case["name"]] = (h, w)
        got = ref_state.stored_latents(case["name"], case["box"])
        bits = torch.int32 if got.dtype == torch.float32 else torch.int16
        arrays[case["name"]] = got.contiguous().view(bits).numpy()
    np.savez_compressed(out / "latents.npz", **arrays)


def hash_seed(name: str) -> int:
    return int(hashlib.sha256(name.encode()).hexdigest()[:8], 16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("QWENEDIT_REFERENCE"),
                    required="QWENEDIT_REFERENCE" not in os.environ,
                    help="path of a QwenEdit checkout (default: $QWENEDIT_REFERENCE)")
    ap.add_argument("--only", choices=["keys", "nvfp4", "paged", "latents"], default=None)
    args = ap.parse_args()
    import_reference(Path(args.reference))
    for part, fn in (("keys", gen_keys), ("paged", gen_paged), ("nvfp4", gen_nvfp4), ("latents", gen_latents)):
        if args.only in (None, part):
            fn(HERE)
            print("wrote", part)


if __name__ == "__main__":
    main()
