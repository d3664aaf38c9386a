"""ctypes front of oracle/libqe_oracle.so (TEST ORACLE, see oracle/__init__.py).

``norm_scale_fp4_ref`` / ``silu_mul_fp4_ref`` take CPU bf16 tensors and return numpy ``(q, sf)`` in the
exact layout of multi_turn/fibo/fp4.py:94-116 (q [M, K/2], sf [pad128(M), K/16]).
"""

from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_float, c_int, c_int64, c_uint8, c_uint16, c_void_p
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
LIB = HERE / "libqe_oracle.so"
_lib = None


def build() -> Path:
    """Compile the oracle library (gcc via oracle/Makefile)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "nvfp4_ref.c").stat().st_mtime:
            build()
        h = ctypes.CDLL(str(LIB))
        h.ref_norm_scale_fp4.argtypes = [c_void_p] * 7 + [c_float, c_int64, c_int64, c_int64, c_int64, c_float,
                                                          c_void_p, c_void_p, c_void_p]
        h.ref_norm_scale_fp4.restype = c_int
        h.ref_silu_mul_fp4.argtypes = [c_void_p, c_void_p, c_float, c_int64, c_int64, c_void_p, c_void_p, c_void_p]
        h.ref_silu_mul_fp4.restype = c_int
        h.ref_exp.argtypes = [c_float]
        h.ref_exp.restype = c_float
        h.ref_e4m3.argtypes = [c_float]
        h.ref_e4m3.restype = c_uint8
        h.ref_e4m3_value.argtypes = [c_uint8]
        h.ref_e4m3_value.restype = c_float
        h.ref_e2m1.argtypes = [c_float]
        h.ref_e2m1.restype = c_uint8
        h.ref_f_to_bf16.argtypes = [c_float]
        h.ref_f_to_bf16.restype = c_uint16
        h.ref_silu_bf16.argtypes = [c_uint16]
        h.ref_silu_bf16.restype = c_uint16
        h.ref_pairwise_sum.argtypes = [POINTER(c_float), c_int64]
        h.ref_pairwise_sum.restype = c_float
        _lib = h
    return _lib


def _u16(t: torch.Tensor | None) -> np.ndarray | None:
    if t is None:
        return None
    if t.dtype != torch.bfloat16:
        raise TypeError("oracle inputs are bf16")
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(c_void_p)


def norm_scale_fp4_ref(x, weight, eps, noisy, clean=None, noise_mask=None, gs=1.0, shift=None, shift_clean=None):
    """q, sf of RMSNorm + adaLN (+shift) -> NVFP4 for x [..., S, K] (bf16 CPU tensors; modulation rows [B, K])."""
    K = x.shape[-1]
    S = x.shape[-2] if x.dim() >= 2 else x.shape[0]
    M = x.numel() // K
    padded = -(-M // 128) * 128

    def rows(t):
        if t is None:
            return None, 0
        t2 = t if t.dim() == 2 else t[None]
        return _u16(t2.contiguous()), (K if t2.shape[0] > 1 else 0)

    xa, wa = _u16(x.reshape(M, K)), _u16(weight.reshape(K))
    na, stride = rows(noisy)
    ca, _ = rows(clean)
    sa, _ = rows(shift)
    sca, _ = rows(shift_clean)
    mask = None if noise_mask is None else noise_mask.detach().cpu().to(torch.uint8).numpy().copy()
    q = np.zeros((M, K // 2), np.uint8)
    sf = np.zeros((padded, K // 16), np.uint8)
    P = 1
    while P < K:
        P <<= 1
    scratch = np.zeros(2 * P, np.float32)
    rc = lib().ref_norm_scale_fp4(_p(xa), _p(wa), _p(na), _p(ca), _p(mask), _p(sa), _p(sca), float(gs), M, S, K,
                                  stride, float(eps), _p(q), _p(sf), _p(scratch))
    if rc:
        raise ValueError("oracle rejected the sizes")
    return q, sf


def silu_mul_fp4_ref(gate, value, gs):
    K = gate.shape[-1]
    M = gate.numel() // K
    padded = -(-M // 128) * 128
    q = np.zeros((M, K // 2), np.uint8)
    sf = np.zeros((padded, K // 16), np.uint8)
    scratch = np.zeros(K, np.float32)
    rc = lib().ref_silu_mul_fp4(_p(_u16(gate.reshape(M, K))), _p(_u16(value.reshape(M, K))), float(gs), M, K,
                                _p(q), _p(sf), _p(scratch))
    if rc:
        raise ValueError("oracle rejected the sizes")
    return q, sf


def bf16_values_norm_scale(x, weight, eps, noisy, clean=None, noise_mask=None, shift=None, shift_clean=None):
    """The bf16 tensor the norm_scale kernel quantises (for global-scale calibration): eager restatement with the
    reference's per-op roundings (fibo/dit.py:31-49) in float32 torch on CPU, row sums in the oracle's order."""
    K = x.shape[-1]
    xf = x.float().reshape(-1, K)
    P = 1
    while P < K:
        P <<= 1
    sq = torch.zeros(xf.shape[0], P)
    sq[:, :K] = xf * xf
    sums = torch.tensor([lib().ref_pairwise_sum(r.numpy().ctypes.data_as(POINTER(c_float)), P) for r in sq])
    rstd = 1.0 / torch.sqrt(sums / K + torch.tensor(eps, dtype=torch.float32))
    S = x.shape[-2]
    b = torch.arange(xf.shape[0]) // S
    sel = torch.ones(xf.shape[0], dtype=torch.bool) if noise_mask is None else noise_mask.cpu().bool()[
        torch.arange(xf.shape[0]) % S]
    nz = noisy if noisy.dim() == 2 else noisy[None]
    mod = nz.float()[b.clamp(max=nz.shape[0] - 1)]
    if clean is not None:
        cl = clean if clean.dim() == 2 else clean[None]
        mod = torch.where(sel[:, None], mod, cl.float()[b.clamp(max=cl.shape[0] - 1)])
    y = (xf * rstd[:, None]).bfloat16().float()
    y = (y * weight.float()).bfloat16().float()
    y = (y * (1.0 + mod).bfloat16().float()).bfloat16().float()
    if shift is not None:
        sh = shift if shift.dim() == 2 else shift[None]
        shv = sh.float()[b.clamp(max=sh.shape[0] - 1)]
        if shift_clean is not None:
            sc = shift_clean if shift_clean.dim() == 2 else shift_clean[None]
            shv = torch.where(sel[:, None], shv, sc.float()[b.clamp(max=sc.shape[0] - 1)])
        y = (y + shv).bfloat16().float()
    return y.bfloat16().reshape(x.shape)


def global_scale(y: torch.Tensor, headroom: float = 4.0) -> float:
    """448 * 6 / (amax * headroom) in float32, as the reference writes it (tests/test_fibo_fp4.py:18-19;
    pipeline/fp4.py:33-35): a Python scalar over a tensor, which torch evaluates as reciprocal then multiply."""
    amax = y.float().abs().amax().clamp(min=1e-8) * headroom
    return float((448.0 * 6.0 / amax).to(torch.float32))


__all__ = ["build", "lib", "norm_scale_fp4_ref", "silu_mul_fp4_ref", "bf16_values_norm_scale", "global_scale"]
