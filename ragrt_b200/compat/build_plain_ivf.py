"""
Plain IVF index in RAGRT's CSR format (numpy); drop-in for ``plain_ivf_csr`` of the
reference's ``src/build_plain_ivf.py:28-68``.

One posting list per centroid holding the passages with a token assigned to it,
deduplicated per (centroid, passage) and sorted by pid.  A centroid whose list is
longer than the uint16 length field is split into chunks with eids 0, 1, ... .  All
lists live in "subspace" row 0 of ``row_ptrs``; rows 1-31 are empty.

For corpus-scale builds on the GPU see ``ragrt_b200.index_build`` (same arrays).
"""
import numpy as np

try:                                    # as ragrt_b200.compat.build_plain_ivf
    from . import ragrt_index_lib as L
except ImportError:                     # as a top-level module (compat dir on sys.path)
    import ragrt_index_lib as L


def plain_ivf_csr(codes, pids, num_centroids, max_len=L.MAX_LIST_LENGTH, dedup=True, tokens=False):
    """codes, pids: per token.  Returns dict(row_ptrs int64 [32, NC+1], col_eids, lengths
    (int64), pids_sorted, token_ids (tokens=True only, uint32), E_needed)."""
    codes = np.asarray(codes, dtype=np.int64)
    pids = np.asarray(pids, dtype=np.int64)
    if len(codes) != len(pids):
        raise AssertionError("codes and pids must align")
    if len(pids) and (pids.min() < 0 or pids.max() > L.MAX_PID):
        raise AssertionError("pid out of the 24-bit range")
    tids = None
    if tokens:
        if len(codes) >= (1 << 32):
            raise AssertionError("too many tokens for 32-bit token ids")
        key = np.sort((codes << 32) | np.arange(len(codes), dtype=np.int64))
        c, tids = key >> 32, key & 0xFFFFFFFF
        p = pids[tids]
        tids = tids.astype(np.uint32)
    else:
        key = (codes << 24) | pids
        key = np.unique(key) if dedup else np.sort(key)
        c, p = key >> 24, key & ((1 << 24) - 1)
    per_c = np.bincount(c, minlength=num_centroids).astype(np.int64)
    nchunk = (per_c + max_len - 1) // max_len
    n_lists = int(nchunk.sum())
    list_cid = np.repeat(np.arange(num_centroids, dtype=np.int64), nchunk)
    first = np.cumsum(nchunk) - nchunk
    eids = np.arange(n_lists, dtype=np.int64) - first[list_cid]
    lengths = np.minimum(max_len, per_c[list_cid] - eids * max_len).astype(np.int64)
    row = np.zeros(num_centroids + 1, dtype=np.int64)
    row[1:] = np.cumsum(nchunk)
    row_ptrs = np.empty((L.NUM_SUBSPACES, num_centroids + 1), dtype=np.int64)
    row_ptrs[0] = row
    row_ptrs[1:] = n_lists
    return {"row_ptrs": row_ptrs, "col_eids": eids, "lengths": lengths, "pids_sorted": p,
            "token_ids": tids, "E_needed": int(nchunk.max()) if n_lists else 1}


def to_bind_arrays(csr, E=None):
    """The arrays ``CorrIndex3D.bind_index`` takes, in the on-disk dtypes written by the
    reference's ``build_plain_ivf.main`` (build_plain_ivf.py:98-127)."""
    E = max(4, csr["E_needed"]) if E is None else E
    lengths = csr["lengths"].astype(np.uint16)
    return {
        "csr_row_ptrs": csr["row_ptrs"].astype(np.int64),
        "csr_col_eids": csr["col_eids"].astype(L.eid_dtype(E)),
        "csr_block_sums": L.block_sums(lengths),
        "csr_lengths": lengths,
        "csr_packed_24": L.pack_pids_24(csr["pids_sorted"]),
        "E": E,
    }
