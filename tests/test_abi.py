"""The C-ABI library loads on a CPU-only host and exports every entry point that
include/ragrt_b200.h declares (no compute calls: those need a GPU)."""

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


def test_new_entry_points_reject_bad_arguments_without_a_gpu():
    """The encoder, merge and statistics entry points validate their arguments before any
    CUDA call (fake non-null pointers: nothing is dereferenced on these paths)."""
    L = _lib.lib()
    p = 0x1000                                          # 16-byte aligned, never touched
    # N not a multiple of 128
    assert L.ragrt_enc_gemm(p, p, None, None, p, 64, 100, 768, 0, None, 0, None) == -1
    assert b"multiple of 128" in L.ragrt_last_error()
    # the normalising epilogue is for N = 128
    assert L.ragrt_enc_gemm(p, p, None, None, p, 64, 256, 768, 4, None, 0, None) == -1
    # the residual epilogue needs a residual
    assert L.ragrt_enc_gemm(p, p, p, None, p, 64, 256, 768, 3, None, 0, None) == -1
    # attention is built for 32 tokens and 64-wide heads
    assert L.ragrt_enc_attention(p, p, p, 2, 16, 12, 768, None) == -1
    assert L.ragrt_enc_attention(p, p, p, 2, 32, 12, 700, None) == -1
    assert L.ragrt_enc_layernorm(p, p, p, 1e-12, p, 8, 512, None) == -1
    assert L.ragrt_enc_gemm_residual_ln(p, p, p, p, p, p, 1e-12, p, p, 64, 512, 768, None, 0, None) == -1
    # merge: k_top beyond world * k, and null outputs
    assert L.ragrt_merge_topk(p, 2, 4, 10, 21, p, p, None) == -1
    assert L.ragrt_merge_topk(p, 2, 4, 10, 10, None, p, None) == -1
    assert L.ragrt_index_count_distinct(None, 1) == -1
