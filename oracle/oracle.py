"""
ctypes front end of the CPU oracle (weft_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs as the checker; the product path never imports this module.

Inputs are numpy arrays (fp16 data passed as uint16 views).  `index` is a dict with
the ``CorrIndex3D.bind_index`` names (csr_row_ptrs, csr_col_eids, csr_block_sums,
csr_lengths, csr_packed_24, doc_offsets, doc_lens, codes, residuals, centroids,
bucket_weights, reversed_bit_map, decomp_table, doc_predicates).
"""
import ctypes as C
import os
import subprocess
import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libragrt_ref.so")

_lib = None


def build():
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        L.oracle_rn16_dot.restype = C.c_uint16
        L.oracle_rn16_dot.argtypes = [P, P, C.c_int]
        L.oracle_native_prep.restype = C.c_int
        L.oracle_native_prep.argtypes = [P, C.c_int, P, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P]
        L.oracle_candidates.restype = C.c_int
        L.oracle_candidates.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_uint32, C.c_int, P, P, P]
        L.oracle_tile_maxsim.restype = None
        L.oracle_tile_maxsim.argtypes = [P, P, P, C.c_int, P, C.c_int]
        L.oracle_final_topk.restype = C.c_int
        L.oracle_final_topk.argtypes = [P, P, C.c_int, P, C.c_uint32, C.c_int, P, P]
        L.oracle_weft_search.restype = None
        L.oracle_weft_search.argtypes = [P, P, P, C.c_int, P, P, C.c_int, C.c_int, C.c_int, P,
                                         C.c_int, C.c_int, P, P, P, C.c_int]
        L.oracle_native_prep_batch.restype = None
        L.oracle_native_prep_batch.argtypes = [P, P, C.c_int, P, C.c_int, C.c_int, C.c_int, C.c_int,
                                               P, P, P, C.c_int]
        L.oracle_max_threads.restype = C.c_int
        _lib = L
    return _lib


class _Csr(C.Structure):
    _fields_ = [("row_ptrs", C.c_void_p), ("col_eids", C.c_void_p), ("eid_bytes", C.c_int),
                ("block_sums", C.c_void_p), ("lengths", C.c_void_p), ("packed24", C.c_void_p),
                ("num_lists", C.c_int64), ("num_passages", C.c_int), ("num_centroids", C.c_int),
                ("preds", C.c_void_p)]


class _Docs(C.Structure):
    _fields_ = [("doc_offsets", C.c_void_p), ("doc_lens", C.c_void_p), ("codes", C.c_void_p),
                ("residuals", C.c_void_p), ("centroids", C.c_void_p), ("bucket_weights", C.c_void_p),
                ("rbm", C.c_void_p), ("decomp", C.c_void_p), ("num_passages", C.c_int)]


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _u16(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint16) if a.dtype == np.float16 else a.astype(np.uint16)


class Index:
    """Host copy of a bound index; keeps the arrays alive for the C structs."""

    def __init__(self, d):
        self.row_ptrs = _c(d["csr_row_ptrs"], np.int64)
        eids = np.ascontiguousarray(d["csr_col_eids"])
        if eids.dtype == np.int16:
            eids = eids.view(np.uint16)
        self.col_eids = eids
        self.block_sums = _c(d["csr_block_sums"], np.int64)
        ln = np.ascontiguousarray(d["csr_lengths"])
        self.lengths = ln.view(np.uint16) if ln.dtype == np.int16 else ln.astype(np.uint16)
        self.packed = _c(d["csr_packed_24"], np.uint8)
        self.doc_offsets = _c(d["doc_offsets"], np.int64)
        self.doc_lens = _c(d["doc_lens"], np.int32)
        self.codes = _c(d["codes"], np.int32)
        self.residuals = _c(d["residuals"], np.uint8)
        self.centroids = _u16(d["centroids"])
        self.bw = _u16(d["bucket_weights"])
        self.rbm = _c(d["reversed_bit_map"], np.uint8)
        self.decomp = _c(d["decomp_table"], np.uint8)
        self.N = int(self.doc_lens.shape[0])
        self.NC = int(self.centroids.shape[0])
        pred = d.get("doc_predicates")
        self.preds = _c(pred if pred is not None else np.zeros(self.N, np.uint32), np.uint32)
        self.csr = _Csr(_p(self.row_ptrs), _p(self.col_eids), int(self.col_eids.dtype.itemsize),
                        _p(self.block_sums), _p(self.lengths), _p(self.packed), len(self.lengths),
                        self.N, self.NC, _p(self.preds))
        self.docs = _Docs(_p(self.doc_offsets), _p(self.doc_lens), _p(self.codes), _p(self.residuals),
                          _p(self.centroids), _p(self.bw), _p(self.rbm), _p(self.decomp), self.N)


def rn16_dot(q, c):
    q, c = _u16(q), _u16(c)
    return np.uint16(lib().oracle_rn16_dot(_p(q), _p(c), q.shape[0])).view(np.float16)


def native_prep(Q, C_, nc, impute=True):
    """One query: Q [ntok,128] fp16, C [NC,128] fp16 -> (topc int32 [ntok,ncol],
    scores f32 [ntok,ncol] (compact), m f32 [ntok] or None, vals fp16 [ntok,kk])."""
    Q, C_ = _u16(Q), _u16(C_)
    ntok, dim = Q.shape
    NC = C_.shape[0]
    kk = min(nc + (1 if impute else 0), NC)
    ncol = min(nc, kk)
    topc = np.zeros((ntok, ncol), np.int32)
    sc = np.zeros((ntok, ncol), np.float32)
    m = np.zeros(ntok, np.float32)
    vals = np.zeros((ntok, kk), np.uint16)
    lib().oracle_native_prep(_p(Q), ntok, _p(C_), NC, dim, nc, int(impute), _p(topc), _p(sc), _p(m), _p(vals))
    return topc, sc, (m if (impute and kk > nc) else None), vals.view(np.float16)


def candidates(index, topc, scores, n_eids, mask, K):
    """Stages 1-3 for one query -> (pids int32 [K], sums f32 [K], stats dict)."""
    topc = _c(topc, np.int32)
    scores = _c(scores, np.float32)
    ntok, kc = topc.shape
    pids = np.zeros(K, np.int32)
    sums = np.zeros(K, np.float32)
    st = np.zeros(3, np.int64)
    lib().oracle_candidates(C.byref(index.csr), _p(topc), _p(scores), ntok, kc, n_eids, mask, K,
                            _p(pids), _p(sums), _p(st))
    return pids, sums, {"postings": int(st[0]), "touched": int(st[1]), "tasks": int(st[2])}


def tile_maxsim(index, Q, pids, nthreads=0):
    Q = _u16(Q)
    if Q.shape != (32, 128):
        raise AssertionError("Q must be [32, 128]")
    pids = _c(pids, np.int32)
    out = np.zeros(len(pids), np.float32)
    lib().oracle_tile_maxsim(C.byref(index.docs), _p(Q), _p(pids), len(pids), _p(out), nthreads)
    return out


def final_topk(index, pids, scores, mask, k):
    pids = _c(pids, np.int32)
    scores = _c(scores, np.float32)
    ids = np.full(k, -1, np.int32)
    sc = np.full(k, -np.inf, np.float32)
    lib().oracle_final_topk(_p(pids), _p(scores), len(pids), _p(index.preds), mask, k, _p(ids), _p(sc))
    return ids, sc


def weft_search(index, Q, ntok, nc, n_eids, masks, K, k_top, nthreads=0):
    """Whole path for a batch: Q [B,32,128] fp16 -> (ids [B,k_top], scores, stats [B,3])."""
    Q = _u16(Q)
    B = Q.shape[0]
    ntok = _c(ntok, np.int32)
    masks = _c(masks if masks is not None else np.zeros(B), np.uint32)
    ids = np.full((B, k_top), -1, np.int32)
    sc = np.full((B, k_top), -np.inf, np.float32)
    st = np.zeros((B, 3), np.int64)
    lib().oracle_weft_search(C.byref(index.csr), C.byref(index.docs), _p(index.centroids), 128, _p(Q),
                             _p(ntok), B, nc, n_eids, _p(masks), K, k_top, _p(ids), _p(sc), _p(st), nthreads)
    return ids, sc, st


def topk_agreement(index, Q, ids, sc, oids, osc, masks=None, rel_tol=1e-3):
    """Compare a batch's final top-k (ids int [B, k], scores f32 [B, k]) with the oracle's
    (oids, osc) under the parity rule of this path:

    * every finite oracle score is matched within `rel_tol` relative (denominator
      max(|s|, 1)), and the -inf / padding positions coincide;
    * ids are identical, except at a position where the two differ only because of a
      Stage-4 tie within tolerance: the oracle's own MaxSim of OUR id there is within
      2 * rel_tol of the oracle's score at that position (and, for a filtered query, our
      id passes the filter).

    Returns {"positions", "equal", "ties", "mismatches", "max_rel_score_err"}; a result
    is in parity when "mismatches" is 0 and "max_rel_score_err" < rel_tol."""
    ids, sc = np.asarray(ids), np.asarray(sc)
    oids, osc = np.asarray(oids), np.asarray(osc)
    Q = _u16(Q)
    B, k = oids.shape
    out = {"positions": int(B * k), "equal": 0, "ties": 0, "mismatches": 0, "max_rel_score_err": 0.0}
    for b in range(B):
        fin = np.isfinite(osc[b])
        if not np.array_equal(np.isfinite(sc[b]), fin):
            out["mismatches"] += int((np.isfinite(sc[b]) != fin).sum())
        if fin.any():
            rel = np.abs(sc[b][fin].astype(np.float64) - osc[b][fin]) / np.maximum(np.abs(osc[b][fin]), 1.0)
            out["max_rel_score_err"] = max(out["max_rel_score_err"], float(rel.max()))
        mask = int(masks[b]) if masks is not None else 0
        for i in range(k):
            if ids[b, i] == oids[b, i]:
                out["equal"] += 1
                continue
            p = int(ids[b, i])
            ok = 0 <= p < index.N and np.isfinite(osc[b, i])
            if ok and mask:
                ok = (int(index.preds[p]) & mask) != 0
            if ok:
                s = float(tile_maxsim(index, Q[b], np.array([p], np.int32))[0])
                ok = abs(s - float(osc[b, i])) <= 2 * rel_tol * max(abs(float(osc[b, i])), 1.0)
            if ok:
                out["ties"] += 1
            else:
                out["mismatches"] += 1
    return out


def native_prep_batch(Q, ntok, C_, nc, impute=True, nthreads=0):
    Q, C_ = _u16(Q), _u16(C_)
    B = Q.shape[0]
    ntok = _c(ntok, np.int32)
    topc = np.zeros((B, 32, nc), np.int32)
    sc = np.zeros((B, 32, nc), np.float32)
    m = np.zeros((B, 32), np.float32)
    lib().oracle_native_prep_batch(_p(Q), _p(ntok), B, _p(C_), C_.shape[0], 128, nc, int(impute),
                                   _p(topc), _p(sc), _p(m), nthreads)
    return topc, sc, m


def max_threads():
    return lib().oracle_max_threads()


# ---------------------------------------------------------------- the reference's own kernels

_ref = None


def ref_lib():
    """The reference's CUDA kernels built by oracle/build_ref.sh (None if not built)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB_PATH):
            return None
        L = C.CDLL(REF_LIB_PATH)
        P = C.c_void_p
        L.ref_weft_candidates.restype = C.c_longlong
        L.ref_weft_candidates.argtypes = [P, P, C.c_int, C.c_int, C.c_int, P, P, P, P, P, C.c_int, C.c_int,
                                          C.c_int, P, P, C.c_int, P, P, P, C.c_int, P, C.c_uint32,
                                          C.c_longlong, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                          C.POINTER(C.c_longlong), P]
        L.ref_tile_maxsim.restype = None
        L.ref_tile_maxsim.argtypes = [P, P, P, P, C.c_int, P, P, P, P, P, P, P, C.c_int, P]
        L.ref_copy_d2d.restype = C.c_int
        L.ref_copy_d2d.argtypes = [P, P, C.c_size_t]
        L.ref_mask_failing.restype = None
        L.ref_mask_failing.argtypes = [P, C.c_int, P, C.c_uint32, P, P]
        _ref = L
    return _ref
