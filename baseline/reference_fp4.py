"""Load the reference's own Triton NVFP4 kernels (multi_turn/fibo/fp4.py:37-116) from its offline install.

The reference package is installed, unmodified, under ``baseline/_ref`` by

    python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \\
        --target baseline/_ref <QwenEdit checkout copied to a writable path>

(``--no-deps``: its pillow / numpy pins have no wheels offline; the kernels need neither). The install is not
committed; it travels with the working tree to the GPU host. Only tests and ``bench.py`` use it, as the thing the
CUDA kernels are compared with and timed against.

``fibo/fp4.py`` imports ``_norm_scale`` / ``silu_mul`` from ``fibo/dit.py``, which needs SGLang (absent here).
The kernels and their wrappers ``norm_scale_fp4`` / ``silu_mul_fp4`` never call those two helpers, so a stand-in
module supplies the names; they raise if called.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

REF = Path(__file__).resolve().parent / "_ref"


def available() -> bool:
    return (REF / "multi_turn" / "fibo" / "fp4.py").is_file()


def _unavailable(*_a, **_k):
    raise RuntimeError("the reference's SGLang-backed eager helpers are not available in this process")


def load():
    """The reference module ``multi_turn.fibo.fp4`` (Triton kernels compiled by the installed Triton)."""
    if not available():
        raise ImportError(f"reference install not found under {REF.name}/ (see this module's docstring)")
    if "multi_turn.fibo.dit" not in sys.modules:
        stand_in = types.ModuleType("multi_turn.fibo.dit")
        stand_in._norm_scale = _unavailable
        stand_in.silu_mul = _unavailable
        sys.modules["multi_turn.fibo.dit"] = stand_in
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import multi_turn.fibo.fp4 as fp4

    if not str(Path(fp4.__file__).resolve()).startswith(str(REF.resolve())):
        raise ImportError(f"multi_turn.fibo.fp4 resolved to {fp4.__file__}, not the install under {REF.name}/")
    return fp4


# e2m1 magnitude of codes 0..7 (fibo/fp4.py:37-43); bit 3 is the sign
_E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _e4m3_to_f32(sf_bytes):
    import torch

    return sf_bytes.view(torch.float8_e4m3fn).float()


def unswizzle_scales(sf, M: int, K: int):
    """[M, K/16] fp32 block scales from the 128x4-swizzled e4m3 bytes (layout of fibo/fp4.py:59-60)."""
    import torch

    G = K // 16
    m = torch.arange(M, device=sf.device)[:, None]
    g = torch.arange(G, device=sf.device)[None, :]
    off = (m // 128) * (K // 64 * 512) + (g // 4) * 512 + (m % 32) * 16 + (m % 128 // 32) * 4 + g % 4
    return _e4m3_to_f32(sf.reshape(-1)[off])


def compare_nvfp4(q_a, sf_a, q_b, sf_b, gs: float, M: int, K: int) -> dict:
    """Differences between two NVFP4 encodings of the same [M, K] values: codes and scales that differ, the
    largest code step among elements whose block scale agrees (steps counted along the signed e2m1 ladder),
    and the largest absolute difference of the dequantised values code * scale / gs."""
    import torch

    lut = torch.tensor(_E2M1, device=q_a.device)

    def codes(q):
        q = q.reshape(M, K // 2)
        return torch.stack([q & 15, q >> 4], dim=-1).reshape(M, K).to(torch.int64)

    ca, cb = codes(q_a), codes(q_b)
    sa, sb = unswizzle_scales(sf_a, M, K), unswizzle_scales(sf_b, M, K)
    signed = lambda c: torch.where(c >= 8, -(c - 8), c)  # noqa: E731  ladder position, -7..7
    same_scale = (sa == sb).repeat_interleave(16, dim=1)
    step = (signed(ca) - signed(cb)).abs()
    deq = lambda c, s: torch.where(c >= 8, -1.0, 1.0) * lut[c & 7] * s.repeat_interleave(16, dim=1) / gs  # noqa: E731
    da, db = deq(ca, sa), deq(cb, sb)
    diff_el = da != db
    return {
        "elements": M * K,
        "codes_differing": int((ca != cb).sum()),
        "scales_differing": int((sa != sb).sum()),
        "scale_blocks": M * (K // 16),
        "elements_dequant_differing": int(diff_el.sum()),
        "frac_elements_differing": float(diff_el.float().mean()),
        "max_code_step_same_scale": int(step[same_scale].max()) if bool(same_scale.any()) else 0,
        "dequant_max_abs_err": float((da - db).abs().max()),
        "dequant_max_abs": float(da.abs().max()),
        "bit_exact": bool(torch.equal(q_a, q_b) and torch.equal(sf_a, sf_b)),  # sf includes the pad rows
    }
