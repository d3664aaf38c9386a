"""Per-step latent ops next to the prefix cache, one sm_100a launch each (libqeb200):

* ``mask_blend(latents, x0, eps, editable, sigma)`` — ``MaskState.blend`` (multi_turn/pipeline/masking.py:82-89),
  run once per denoising step (pipeline/hooks.py:223); the reference spends about ten eager launches on it
  (three dtype conversions, seven arithmetic ops). Bit-identical to the eager sequence.
* ``compose(base, base_grid, crop_latents, box)`` — the tensor part of ``_compose`` (pipeline/hooks.py:234-247):
  the stored version's latents with the box replaced by the crop's, in one pass (no clone + slice assignment).
* ``crop(latents, grid, box)`` — the cropped copy of ``stored_latents`` (multi_turn/state.py:52-62).

Latents are [1 or B, h*w, C] tensors on a CUDA device; there is no CPU path.
"""

from __future__ import annotations

import torch

from qwenedit_b200 import _lib

_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _code(t: torch.Tensor, name: str) -> int:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the latent kernels have no CPU path)")
    if t.dtype not in _CODES:
        raise TypeError(f"{name}: dtype {t.dtype} not supported (float32, bfloat16, float16)")
    return _CODES[t.dtype]


def _batch_stride(t: torch.Tensor, B: int, name: str) -> int:
    if t.shape[0] == B:
        return t.stride(0) if B > 1 else 0
    if t.shape[0] == 1:
        return 0
    raise ValueError(f"{name} batch {t.shape[0]} does not broadcast to {B}")


def _stream(device) -> int:
    return _lib.stream_of(device)


def mask_blend(latents: torch.Tensor, x0: torch.Tensor, eps: torch.Tensor, editable: torch.Tensor,
               sigma) -> torch.Tensor:
    """``m * latents + (1 - m) * ((1 - s) * x0 + s * eps)`` with ``m = editable.to(dtype)``, ``s = sigma.to(dtype)``
    (a 0-d tensor) or a Python float, computed with the reference's eager roundings in one launch."""
    dtype = _code(latents, "latents")
    if latents.dim() != 3 or not latents.is_contiguous():
        raise ValueError("latents must be a contiguous [B, N, C] tensor")
    B, N, C = latents.shape
    dev = latents.device
    if x0.dtype != latents.dtype or x0.device != dev:
        x0 = x0.to(device=dev, dtype=latents.dtype)  # masking.py:83
    if eps.dtype != latents.dtype or eps.device != dev:
        eps = eps.to(device=dev, dtype=latents.dtype)  # masking.py:84
    for name, t in (("x0", x0), ("eps", eps)):
        if t.dim() != 3 or tuple(t.shape[1:]) != (N, C) or t.stride(2) != 1 or t.stride(1) != C:
            raise ValueError(f"{name} must be [1 or B, {N}, {C}] with contiguous rows")
    if editable.device != dev:
        editable = editable.to(dev)
    mcode = _code(editable, "editable")
    if editable.dim() != 3 or editable.shape[1] != N or editable.shape[2] not in (1, C) or not editable.is_contiguous():
        raise ValueError(f"editable must be a contiguous [1 or B, {N}, 1 or {C}] tensor")
    if isinstance(sigma, torch.Tensor):
        if sigma.numel() != 1:
            raise ValueError("sigma must be a single value")
        sig = sigma.reshape(1).to(dev)
        if sig.dtype not in _CODES:
            sig = sig.float()
        scode = _CODES[sig.dtype]
    else:  # torch keeps a Python scalar in fp32 (s and 1 - s, the latter computed in double by Python)
        s = float(sigma)
        sig = torch.tensor([s, 1.0 - s], dtype=torch.float32).to(dev)
        scode = 3
    out = torch.empty_like(latents)
    with _lib.on_device(dev):
        _lib.call("qe_mask_blend", latents.data_ptr(), x0.data_ptr(), eps.data_ptr(), editable.data_ptr(),
                  sig.data_ptr(), out.data_ptr(), B, N, C, _batch_stride(x0, B, "x0"), _batch_stride(eps, B, "eps"),
                  _batch_stride(editable, B, "editable"), int(editable.shape[2]), dtype, mcode, scode, _stream(dev))
    return out


def _box(box, grid):
    x0, y0, x1, y1 = (int(v) for v in box)
    h, w = grid
    if not (0 <= x0 < x1 <= w and 0 <= y0 < y1 <= h):
        raise ValueError(f"box {box} outside the {h}x{w} latent grid")
    return x0, y0, x1, y1


def compose(base: torch.Tensor, base_grid, crop_latents: torch.Tensor, box) -> torch.Tensor:
    """[1, h*w, C] latents equal to `base` except the box cells, taken from `crop_latents` (converted to the
    base dtype first, as ``.to(full.dtype)`` does)."""
    _code(base, "base")
    h, w = (int(v) for v in base_grid)
    x0, y0, x1, y1 = _box(box, (h, w))
    C = base.numel() // (h * w)
    if base.numel() != h * w * C or not base.is_contiguous():
        raise ValueError("base must be contiguous [1, h*w, C] latents")
    crop = crop_latents.detach()
    if crop.dtype != base.dtype or crop.device != base.device:
        crop = crop.to(device=base.device, dtype=base.dtype)
    crop = crop.contiguous()
    if crop.numel() != (y1 - y0) * (x1 - x0) * C:
        raise ValueError("crop latents do not match the box")
    out = torch.empty(1, h * w, C, dtype=base.dtype, device=base.device)
    with _lib.on_device(base.device):
        _lib.call("qe_latent_compose", base.data_ptr(), crop.data_ptr(), out.data_ptr(), h, w, C * base.element_size(),
                  x0, y0, x1, y1, _stream(base.device))
    return out


def crop(latents: torch.Tensor, grid, box) -> torch.Tensor:
    """The box cells of [1, h*w, C] latents as a new [1, (y1-y0)*(x1-x0), C] tensor."""
    _code(latents, "latents")
    h, w = (int(v) for v in grid)
    x0, y0, x1, y1 = _box(box, (h, w))
    C = latents.numel() // (h * w)
    if latents.numel() != h * w * C or not latents.is_contiguous():
        raise ValueError("latents must be contiguous [1, h*w, C]")
    out = torch.empty(1, (y1 - y0) * (x1 - x0), C, dtype=latents.dtype, device=latents.device)
    with _lib.on_device(latents.device):
        _lib.call("qe_latent_crop", latents.data_ptr(), out.data_ptr(), h, w, C * latents.element_size(), x0, y0, x1,
                  y1, _stream(latents.device))
    return out


__all__ = ["compose", "crop", "mask_blend"]
