"""Fused NVFP4 activation quantisers: drop-in for ``multi_turn.fibo.fp4`` (fp4.py:29-116).

``norm_scale_fp4(x, norm, noisy, clean, noise_mask, gs)`` and ``silu_mul_fp4(gate, value, gs, block=1024)``
return the same ``Quantized(q, sf, shape)`` as the reference wrappers (fp4.py:101-116):

* ``q``  [M, K/2] uint8, two e2m1 codes per byte, the even column in the low nibble;
* ``sf`` [pad128(M), K/16] uint8, e4m3 block scales (one per 16 values) in the 128x4-swizzled layout that
  ``flashinfer.mm_fp4`` reads; the padding rows hold zero scales.

Each call is one launch of a hand-written sm_100a kernel from libqeb200 on the current CUDA stream. The
adaLN modulation rows may be strided column slices of one [B, 4K] tensor, as in the reference
(``noisy.stride(0)``, fp4.py:106). ``shift`` / ``shift_clean`` (optional, not in the reference) add an adaLN
shift after the scale: ``bf16(bf16(y * bf16(1 + scale)) + shift)``.

``set_numerics`` picks how the fp32 divisions and the rsqrt the reference leaves to its compiler are evaluated:
"triton" (the default) as the reference's Triton kernels compile for sm_100 (div.full.f32, rsqrt.approx.f32:
bit-identical to them on the B200), "ieee" with correctly rounded operations (the CPU restatement's rounding).
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from qwenedit_b200 import _lib


NUMERICS = {"ieee": 0, "triton": 1 | (1 << 2) | (1 << 4)}


def set_numerics(mode: str | int) -> None:
    """Process-wide evaluation of the quantisers' divisions and rsqrt ("triton" default, "ieee", or the raw bit
    field of qe_set_nvfp4_numerics)."""
    _lib.call("qe_set_nvfp4_numerics", NUMERICS[mode] if isinstance(mode, str) else int(mode))


class Quantized(NamedTuple):
    """An NVFP4 activation: ``q`` [M, K/2] e2m1 pairs, ``sf`` swizzled e4m3 scales, ``shape`` of the BF16 tensor."""

    q: torch.Tensor
    sf: torch.Tensor
    shape: torch.Size


def _buffers(x: torch.Tensor, k: int):
    m = x.numel() // k
    padded = -(-m // 128) * 128
    q = torch.empty(m, k // 2, dtype=torch.uint8, device=x.device)
    sf = torch.empty(padded, k // 16, dtype=torch.uint8, device=x.device)
    return m, padded, q, sf


def _check_cuda_bf16(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the NVFP4 kernels have no CPU path)")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")




def _gs(gs: torch.Tensor, device) -> torch.Tensor:
    if not isinstance(gs, torch.Tensor) or gs.numel() != 1 or gs.dtype != torch.float32:
        raise TypeError("gs must be a one-element float32 tensor")
    if gs.device != device:
        raise ValueError(f"gs on {gs.device}, activations on {device}")
    return gs


def _mod_rows(name: str, t: torch.Tensor | None, k: int) -> torch.Tensor | None:
    if t is None:
        return None
    _check_cuda_bf16(name, t)
    if t.dim() == 1:
        t = t[None]
    if t.dim() != 2 or t.shape[-1] != k or t.stride(-1) != 1:
        raise ValueError(f"{name} must be [B, K] rows with unit column stride")
    return t


class _NormArgs(NamedTuple):
    m: int
    s: int
    k: int
    stride: int
    weight: torch.Tensor
    noisy: torch.Tensor
    clean: torch.Tensor | None
    mask: torch.Tensor | None
    shift: torch.Tensor | None
    shift_clean: torch.Tensor | None

    def pointers(self, x):
        ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        return (x.data_ptr(), self.weight.data_ptr(), self.noisy.data_ptr(), ptr(self.clean), ptr(self.mask),
                ptr(self.shift), ptr(self.shift_clean))


def _norm_args(x, norm, noisy, clean, noise_mask, shift, shift_clean) -> _NormArgs:
    _check_cuda_bf16("x", x)
    k = x.shape[-1]
    if k % 64:
        raise ValueError(f"K={k} must be a multiple of 64")
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    s = x.shape[-2] if x.dim() >= 2 else x.shape[0]
    m = x.numel() // k
    weight = norm.weight
    _check_cuda_bf16("norm.weight", weight)
    if weight.numel() != k or not weight.is_contiguous():
        raise ValueError("norm.weight must be a contiguous [K] tensor")
    noisy = _mod_rows("noisy", noisy, k)
    clean = _mod_rows("clean", clean, k)
    shift = _mod_rows("shift", shift, k)
    shift_clean = _mod_rows("shift_clean", shift_clean, k)
    # one modulation row per batch (row stride shared by all of them), or a single row for every batch
    batches = m // s if s else 0
    rows = {t.shape[0] for t in (noisy, clean, shift, shift_clean) if t is not None}
    if len(rows) != 1:
        raise ValueError("noisy / clean / shift rows must have the same batch count")
    stride = 0
    if noisy.shape[0] > 1:
        stride = noisy.stride(0)
        if noisy.shape[0] < batches:
            raise ValueError(f"{noisy.shape[0]} modulation rows for {batches} batches")
        for name, t in (("clean", clean), ("shift", shift), ("shift_clean", shift_clean)):
            if t is not None and t.stride(0) != stride:
                raise ValueError(f"{name} must share noisy's row stride")
    mask = None
    if noise_mask is not None:
        if noise_mask.numel() != s or noise_mask.device != x.device:
            raise ValueError("noise_mask must be [S] on the activations' device")
        mask = noise_mask.contiguous().view(torch.uint8)
        if clean is None:
            raise ValueError("a noise mask needs clean modulation rows")
    return _NormArgs(m, s, k, stride, weight, noisy, clean, mask, shift, shift_clean)


def norm_scale_fp4(x, norm, noisy, clean, noise_mask, gs, shift=None, shift_clean=None) -> Quantized:
    """RMSNorm (``norm.weight``, ``norm.eps``) then the per-token adaLN scale, quantised to NVFP4 with global scale ``gs``.

    Tokens whose ``noise_mask`` is true take ``noisy`` modulation, the others ``clean`` (fibo/dit.py:37-41).
    """
    a = _norm_args(x, norm, noisy, clean, noise_mask, shift, shift_clean)
    _, _, q, sf = _buffers(x, a.k)
    gs = _gs(gs, x.device)
    with _lib.on_device(x.device):
        _lib.call("qe_norm_scale_fp4", *a.pointers(x), gs.data_ptr(), a.m, a.s, a.k, a.stride, float(norm.eps),
                  q.data_ptr(), sf.data_ptr(), _lib.stream_of(x.device))
    return Quantized(q, sf, x.shape)


FP8_MAX, FP4_MAX = 448.0, 6.0


def global_scale(amax: torch.Tensor, headroom: float = 4.0) -> torch.Tensor:
    """Activation global scale from a calibration amax: ``448 * 6 / (max(amax, 1e-8) * headroom)`` in fp32
    (pipeline/fp4.py:33-35, headroom env ``MULTI_TURN_NVFP4_HEADROOM``, default 4)."""
    return (FP8_MAX * FP4_MAX / (amax.float().clamp(min=1e-8) * headroom)).to(torch.float32)


def norm_scale_amax(x, norm, noisy, clean, noise_mask, shift=None, shift_clean=None) -> torch.Tensor:
    """Calibration pre-pass of ``norm_scale_fp4``: max |y| (one-element fp32 device tensor) over the bf16 values
    the quantiser would encode, in one launch with no bf16 tensor written. Replaces the reference's first-call
    bf16 pass ``_norm_scale(...)`` + ``.float().abs().amax()`` (fibo/fp4.py:128-134, pipeline/fp4.py:33-35)."""
    a = _norm_args(x, norm, noisy, clean, noise_mask, shift, shift_clean)
    amax = torch.empty(1, dtype=torch.float32, device=x.device)
    with _lib.on_device(x.device):
        _lib.call("qe_norm_scale_amax", *a.pointers(x), a.m, a.s, a.k, a.stride, float(norm.eps), amax.data_ptr(),
                  _lib.stream_of(x.device))
    return amax


_silu_tables: dict[int, torch.Tensor] = {}


def silu_table(device) -> torch.Tensor:
    """Per-device table of bf16(silu(g)) for all 65,536 bf16 g (128 KiB), built once by ``qe_silu_table_init``."""
    if isinstance(device, torch.device) and device.index is not None:
        table = _silu_tables.get(device.index)
        if table is not None:
            return table
    device = torch.device(device)
    index = device.index if device.index is not None else torch.cuda.current_device()
    table = _silu_tables.get(index)
    if table is None:
        table = torch.empty(65536, dtype=torch.int16, device=torch.device("cuda", index))
        with torch.cuda.device(index):
            _lib.call("qe_silu_table_init", table.data_ptr(), torch.cuda.current_stream(index).cuda_stream)
        _silu_tables[index] = table
    return table


def _silu_args(gate, value) -> tuple[int, int, torch.Tensor]:
    _check_cuda_bf16("gate", gate)
    _check_cuda_bf16("value", value)
    if gate.shape != value.shape:
        raise ValueError("gate and value must have the same shape")
    if not (gate.is_contiguous() and value.is_contiguous()):
        raise ValueError("gate and value must be contiguous")
    if value.device != gate.device:
        raise ValueError("gate and value on different devices")
    k = gate.shape[-1]
    if k % 64:
        raise ValueError(f"K={k} must be a multiple of 64")
    return gate.numel() // k, k, silu_table(gate.device)


def silu_mul_fp4(gate, value, gs, block=1024) -> Quantized:
    """``silu(gate) * value`` quantised to NVFP4 (``block`` is accepted for signature parity and unused)."""
    m, k, table = _silu_args(gate, value)
    _, _, q, sf = _buffers(gate, k)
    gs = _gs(gs, gate.device)
    with _lib.on_device(gate.device):
        _lib.call("qe_silu_mul_fp4", gate.data_ptr(), value.data_ptr(), gs.data_ptr(), m, k, q.data_ptr(),
                  sf.data_ptr(), table.data_ptr(), _lib.stream_of(gate.device))
    return Quantized(q, sf, gate.shape)


def silu_mul_amax(gate, value) -> torch.Tensor:
    """Calibration pre-pass of ``silu_mul_fp4``: max |bf16(silu(gate) * value)| as a one-element fp32 device
    tensor, in one launch with no bf16 product written (pipeline/fp4.py:33-35)."""
    m, k, table = _silu_args(gate, value)
    amax = torch.empty(1, dtype=torch.float32, device=gate.device)
    with _lib.on_device(gate.device):
        _lib.call("qe_silu_mul_amax", gate.data_ptr(), value.data_ptr(), m, k, table.data_ptr(), amax.data_ptr(),
                  _lib.stream_of(gate.device))
    return amax
