"""ctypes binding of libqeb200.so (the C ABI declared in include/qeb200.h).

The library is the only implementation of the path: if it is missing this module raises on first use
(there is no CPU or PyTorch fallback). Build it with ``python -m qwenedit_b200.build``.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_uint8, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libqeb200.so")

QE_OK, QE_ERR_INVALID, QE_ERR_CUDA, QE_ERR_NOMEM, QE_ERR_TIMEOUT, QE_ERR_STATE = range(6)


class QEError(RuntimeError):
    """A libqeb200 call failed (CUDA error, bounded wait timeout or object misuse)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Planes(ctypes.Structure):
    """``qe_planes``: plane p starts at base + (p // planes_inner) * outer_stride + (p % planes_inner) * inner_stride."""

    _fields_ = [("base", c_void_p), ("outer_stride", c_int64), ("inner_stride", c_int64),
                ("planes_inner", c_int32), ("_pad", c_int32)]


_P64 = POINTER(c_int64)
_P32 = POINTER(c_int32)
_PU64 = POINTER(c_uint64)

# name -> (argtypes); every entry point returns int status except the two string getters
SIGNATURES: dict[str, list] = {
    "qe_gather_slots": [Planes, c_int64, Planes, c_int32, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    "qe_gather_pages": [Planes, c_int64, Planes, c_int32, c_int64, c_void_p, c_int32, c_int64, c_void_p, c_void_p],
    "qe_append_slots": [Planes, c_int64, Planes, c_int32, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    "qe_append_pages": [Planes, c_int64, Planes, c_int32, c_int64, c_void_p, c_int32, c_int64, c_void_p, c_void_p],
    "qe_append_slots_ptrs": [Planes, c_int64, c_void_p, c_int32, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    "qe_append_slots_ptrs_noalloc": [Planes, c_int64, c_void_p, c_int32, c_int64, c_void_p, c_int64, c_void_p,
                                     c_void_p],
    "qe_norm_scale_fp4": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                          c_int64, c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p],
    "qe_silu_mul_fp4": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    "qe_silu_table_init": [c_void_p, c_void_p],
    "qe_mask_blend": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                      c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p],
    "qe_latent_compose": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                          c_int64, c_void_p],
    "qe_latent_crop": [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p],
    "qe_gather_slots_heads": [Planes, c_int64, Planes, c_int32, c_int64, c_int64, c_int64, c_int64, c_void_p,
                              c_int64, c_void_p, c_void_p],
    "qe_ipc_alloc": [c_int64, POINTER(c_void_p), c_void_p],
    "qe_ipc_free": [c_void_p],
    "qe_ipc_open": [c_void_p, POINTER(c_void_p)],
    "qe_ipc_close": [c_void_p],
    "qe_append_scatter": [c_void_p, c_int32, Planes, c_int64, Planes, c_int32, c_int64, c_void_p, c_int64,
                          c_void_p, c_void_p],
    "qe_set_norm_table_mode": [c_int32],
    "qe_set_attention_q_tiles": [c_int32],
    "qe_set_silu_table_mode": [c_int32],
    "qe_set_silu_pipeline": [c_int32],
    "qe_set_nvfp4_numerics": [c_int32],
    "qe_set_nvfp4_pdl": [c_int32],
    "qe_paged_attention": [c_void_p, c_int64, c_int64, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int32,
                           c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32,
                           c_float, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "qe_paged_attention_append": [c_void_p, c_int64, c_int64, c_int32, c_int32, c_void_p, c_void_p, c_int64,
                                  c_int32, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int64, c_int32,
                                  c_int32, c_float, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                  c_void_p],
    "qe_norm_scale_amax": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_int64, c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p],
    "qe_silu_mul_amax": [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "qe_index_create": [c_int64, c_int32, POINTER(c_void_p)],
    "qe_index_destroy": [c_void_p],
    "qe_index_clear": [c_void_p],
    "qe_index_match": [c_void_p, _P64, c_int64, _P64, _P64, _PU64],
    "qe_index_lock": [c_void_p, c_uint64],
    "qe_index_unlock": [c_void_p, c_uint64],
    "qe_index_insert": [c_void_p, _P64, _P64, c_int64, _P64],
    "qe_index_evict": [c_void_p, c_int64, _P64],
    "qe_index_alloc": [c_void_p, c_int64, _P64, _P32],
    "qe_index_free": [c_void_p, _P64, c_int64],
    "qe_index_usage": [c_void_p, _P64],
    "qe_index_shuffle_free": [c_void_p, c_uint64],
    "qe_set_paged_copy_mode": [c_int32],
    "qe_blake2b16": [c_void_p, c_int64, c_void_p],
    "qe_keys_text_chain": [c_int64, c_void_p, c_int64, c_void_p],
    "qe_keys_block_ids": [c_int64, c_void_p, c_int64, c_int64, c_void_p],
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library (loads it once). Raises ImportError when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(f"{LIB_PATH.name} is not built; run `python -m qwenedit_b200.build`")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = c_int
            handle.qe_last_error.argtypes = []
            handle.qe_last_error.restype = c_char_p
            handle.qe_version.argtypes = []
            handle.qe_version.restype = c_char_p
            _lib = handle
    return _lib


_fns: dict = {}


def call(name: str, *args) -> None:
    """Call entry point `name`; map a non-zero status to ValueError (bad argument) or QEError."""
    fn = _fns.get(name)
    if fn is None:
        fn = _fns[name] = getattr(lib(), name)
    status = fn(*args)
    if status != QE_OK:
        message = f"{name}: {lib().qe_last_error().decode(errors='replace')}"
        if status == QE_ERR_INVALID:
            raise ValueError(message)
        raise QEError(status, message)


class on_device:
    """``torch.cuda.device(d)`` only when `d` is not already the current device (entering it costs a switch)."""

    __slots__ = ("index", "ctx")

    def __init__(self, device):
        self.index = device if isinstance(device, int) else device.index
        self.ctx = None

    def __enter__(self):
        import torch

        if self.index is not None and self.index != torch.cuda.current_device():
            self.ctx = torch.cuda.device(self.index)
            self.ctx.__enter__()
        return self

    def __exit__(self, *exc):
        if self.ctx is not None:
            self.ctx.__exit__(*exc)
        return False


def stream_of(device) -> int:
    """Raw handle of torch's current CUDA stream on `device` (an int: a torch.device or its index)."""
    import torch

    index = device if isinstance(device, int) else device.index
    return torch._C._cuda_getCurrentRawStream(index)


def version() -> str:
    return lib().qe_version().decode()


def planes(base: int, outer_stride: int, inner_stride: int, planes_inner: int) -> Planes:
    return Planes(c_void_p(base), outer_stride, inner_stride, planes_inner, 0)


def ptr64(array) -> "ctypes._Pointer":
    """int64 pointer into a C-contiguous numpy int64 array."""
    return array.ctypes.data_as(_P64)


__all__ = ["LIB_PATH", "QEError", "Planes", "SIGNATURES", "call", "lib", "on_device", "planes", "ptr64",
           "stream_of", "version", "c_uint8"]
