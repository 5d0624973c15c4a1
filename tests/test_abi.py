"""The C-ABI library loads on a CPU-only host and exports every entry point that
include/ragrt_b200.h declares (no compute calls: those need a GPU)."""
import ctypes as C
import os

from ragrt_b200 import _lib


def test_library_exports_every_declared_symbol():
    names = _lib.header_functions()
    assert "ragrt_weft_search" in names and "ragrt_index_create" in names
    L = _lib.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_signatures_cover_the_header():
    assert set(_lib.header_functions()) == set(_lib._SIGS), "ctypes signatures out of sync with the header"


def test_version_and_error_strings():
    L = _lib.lib()
    assert b"sm_100a" in L.ragrt_version()
    assert isinstance(L.ragrt_last_error(), bytes)


def test_argument_errors_need_no_gpu():
    """Argument validation happens before any CUDA call."""
    L = _lib.lib()
    rc = L.ragrt_final_topk(None, None, 1, 1, None, 0, None, 1, None, None, None)
    assert rc == -1 and b"null" in L.ragrt_last_error()
    rc = L.ragrt_index_create(None, None, None)
    assert rc == -1
