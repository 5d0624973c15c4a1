"""
ctypes binding of libragrt_b200.so (the C ABI in include/ragrt_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every call raises.
Build it with ``python -m ragrt_b200.build`` (or ``__graft_entry__.build()``).
"""
import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libragrt_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "ragrt_b200.h")

P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
U32 = C.c_uint32

ERR_NAMES = {-1: "RAGRT_ERR_ARG", -2: "RAGRT_ERR_CUDA", -3: "RAGRT_ERR_CAPACITY", -4: "RAGRT_ERR_INDEX",
             -5: "RAGRT_ERR_UNSUPPORTED", -6: "RAGRT_ERR_DEVICE"}

NUM_STATS = 8
STAT_NAMES = ("queries", "postings", "distinct_postings", "touched", "probes", "candidates", "tasks",
              "dense_ranges")


class IndexDesc(C.Structure):
    _fields_ = [
        ("csr_row_ptrs", P), ("csr_col_eids", P), ("eid_bytes", I32), ("csr_block_sums", P),
        ("csr_lengths", P), ("csr_packed_24", P), ("num_lists", I64), ("num_postings", I64),
        ("doc_offsets", P), ("doc_lens", P), ("codes", P), ("residuals", P), ("num_tokens", I64),
        ("centroids", P), ("bucket_weights", P), ("reversed_bit_map", P), ("decomp_table", P),
        ("doc_predicates", P), ("num_passages", I32), ("num_centroids", I32), ("num_eids", I32),
    ]


_SIGS = {
    "ragrt_index_create": (I32, [C.POINTER(IndexDesc), C.POINTER(P), P]),
    "ragrt_index_destroy": (I32, [P]),
    "ragrt_centroid_topk": (I32, [P, P, I32, I32, P, I32, I32, I32, P, P, P, P, P]),
    "ragrt_centroid_topk_noalloc": (I32, [P, P, I32, I32, P, I32, I32, I32, P, P, P, P]),
    "ragrt_centroid_topk_noalloc_error": (I32, [I32]),
    "ragrt_weft_candidates": (I32, [P, P, P, I32, P, I32, I32, I32, I32, P, I32, P, P, P, P]),
    "ragrt_centroid_pass_counts": (I32, [P, C.c_uint32, P, P, P]),
    "ragrt_probe_depth": (I32, [P, I32, I32, P, P, I32, C.c_float, C.c_float, I32, I32, P, P, P]),
    "ragrt_tile_maxsim": (I32, [P, P, I32, I32, P, P, I32, P, P, P, P, P, P, P, I32, P]),
    "ragrt_tile_maxsim_exact": (I32, [P, P, I32, I32, P, P, I32, P, P, P]),
    "ragrt_index_tile_maxsim": (I32, [P, P, P, I32, I32, P, I32, P]),
    "ragrt_final_topk": (I32, [P, P, I32, I32, P, I32, P, I32, P, P, P]),
    "ragrt_weft_search": (I32, [P, P, P, I32, I32, I32, P, I32, I32, I32, P, P, P]),
    "ragrt_weft_search_profiled": (I32, [P, P, P, I32, I32, I32, P, I32, I32, I32, P, P, P, P]),
    "ragrt_index_stats": (I32, [P, C.POINTER(C.c_uint64), I32]),
    "ragrt_index_count_distinct": (I32, [P, I32]),
    "ragrt_index_set_stage3_mode": (I32, [P, I32, I32]),
    "ragrt_last_error": (C.c_char_p, []),
    "ragrt_version": (C.c_char_p, []),
    "ragrt_launch_count": (C.c_uint64, []),
    "ragrt_device_error": (I32, [I32]),
    "ragrt_selftest_wait_timeout": (I32, [C.c_uint32, P]),
    "ragrt_merge_topk": (I32, [P, I32, I32, I32, I32, P, P, P]),
    "ragrt_enc_gemm": (I32, [P, P, P, P, P, I32, I32, I32, I32, P, I64, P]),
    "ragrt_enc_gemm_residual_ln": (I32, [P, P, P, P, P, P, C.c_float, P, P, I32, I32, I32, P, I64, P]),
    "ragrt_enc_layernorm": (I32, [P, P, P, C.c_float, P, I32, I32, P]),
    "ragrt_enc_embed": (I32, [P, P, P, P, P, P, C.c_float, I32, I32, I32, I32, P, P]),
    "ragrt_enc_attention": (I32, [P, P, P, I32, I32, I32, I32, P]),
}

_lib = None


def header_functions():
    """Names of the functions declared in include/ragrt_b200.h."""
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ragrt_[a-z0-9_]+)\s*\(", txt)))


def lib():
    """Load libragrt_b200.so once; raise if it is absent (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build the CUDA library first "
                           f"(python -m ragrt_b200.build); there is no CPU fallback")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


class RagrtError(RuntimeError):
    pass


def check(rc):
    if rc != 0:
        msg = lib().ragrt_last_error().decode(errors="replace")
        raise RagrtError(f"{ERR_NAMES.get(rc, rc)}: {msg}")
    return rc
