"""The C ABI: the library loads without a GPU and exports every entry point include/qeb200.h declares."""

import ctypes
import re
from pathlib import Path

from qwenedit_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "qeb200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?(?:int|char\s*\*|const\s+char\s*\*)\s*\**\s*(qe_\w+)\s*\(", text,
                                 flags=re.M)))


def test_header_declares_the_path():
    names = declared_functions()
    for required in ("qe_gather_slots", "qe_gather_pages", "qe_append_slots", "qe_append_pages",
                     "qe_append_slots_ptrs", "qe_norm_scale_fp4", "qe_silu_mul_fp4", "qe_index_create",
                     "qe_index_match", "qe_index_insert", "qe_index_evict", "qe_index_alloc", "qe_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    handle = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(handle, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_bindings_cover_the_header():
    names = set(declared_functions()) - {"qe_last_error", "qe_version"}
    assert names <= set(_lib.SIGNATURES), sorted(names - set(_lib.SIGNATURES))
    assert "sm_100a" in _lib.version()


def test_invalid_arguments_raise_not_abort():
    import pytest

    with pytest.raises(ValueError, match="page_size"):
        _lib.call("qe_index_create", 16, 0, ctypes.byref(ctypes.c_void_p()))
    # device entry points validate before touching the GPU
    with pytest.raises(ValueError, match="multiple of 64"):
        _lib.call("qe_silu_mul_fp4", 16, 16, 16, 4, 100, 16, 16, 16, None)
    with pytest.raises(ValueError, match="null"):
        _lib.call("qe_gather_slots", _lib.planes(0, 0, 0, 2), 10, _lib.planes(16, 0, 0, 2), 2, 64, 0, 4, None, None)
