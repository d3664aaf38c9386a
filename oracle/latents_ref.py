"""TEST ORACLE (see oracle/__init__.py): the reference's per-step latent ops restated in torch eager, op for op.

* ``blend`` — ``MaskState.blend``, multi_turn/pipeline/masking.py:82-89.
* ``compose`` — the tensor part of ``_compose``, multi_turn/pipeline/hooks.py:244-246.
* ``crop`` — ``stored_latents`` with a crop box, multi_turn/state.py:52-62.
"""

from __future__ import annotations

import torch


def blend(latents, x0, eps, editable, sigma):
    x0 = x0.to(device=latents.device, dtype=latents.dtype)
    eps = eps.to(device=latents.device, dtype=latents.dtype)
    m = editable.to(device=latents.device, dtype=latents.dtype)
    if isinstance(sigma, torch.Tensor):
        sigma = sigma.to(device=latents.device, dtype=latents.dtype)
    keep = (1 - sigma) * x0 + sigma * eps
    return m * latents + (1 - m) * keep


def compose(base, base_grid, crop_latents, box):
    x0, y0, x1, y1 = (int(v) for v in box)
    h, w = base_grid
    full = base.view(1, h, w, -1).clone()
    full[:, y0:y1, x0:x1] = crop_latents.detach().to(full.dtype).view(1, y1 - y0, x1 - x0, -1)
    return full.view(1, h * w, -1)


def crop(latents, grid, box):
    x0, y0, x1, y1 = box
    h, w = grid
    return latents.view(1, h, w, -1)[:, y0:y1, x0:x1].reshape(1, (y1 - y0) * (x1 - x0), -1)
