"""
Index-format building blocks of RAGRT's plain-IVF index (numpy only).

Drop-in for the parts of the reference's ``src/ragrt_index_lib.py`` that the `weft`
path uses: the format constants, 24-bit pid packing and the 128-list block sums that
Stage 3 uses to locate a posting list without a per-list offset array.

On-disk / bound layout (ragrt_index_lib.py:9-15, build_plain_ivf.py:115-127):
  csr_row_ptrs        int64  [32, num_centroids + 1]   lists of centroid c in row 0
  csr_col_eids        uint8 (E <= 256) or uint16       chunk id 0..k-1 within a centroid
  csr_lengths         uint16 [num_lists]               postings per list (<= 65535)
  csr_block_sums_128  int64  [ceil(num_lists / 128)]   offset of list 128*b
  csr_packed_24       uint8  [3 * num_postings]        little-endian 24-bit pids
"""
import numpy as np

NUM_SUBSPACES = 32                      # ragrt_index_lib.py:19
SUBSPACE_DIM = 3                        # :20
PROJ_DIM = NUM_SUBSPACES * SUBSPACE_DIM
PID_BITS = 24                           # :23
MAX_PID = (1 << PID_BITS) - 1           # :24
MAX_LIST_LENGTH = np.iinfo(np.uint16).max   # :25
MAX_EIDS_UINT8 = 256                    # :26
MAX_EIDS = 1 << 16                      # :27
BLOCK_SIZE = 128                        # :28 (the Stage 2/3 kernels shift by 7)


def eid_dtype(num_entries):
    """dtype of csr_col_eids for E chunk ids per centroid (ragrt_index_lib.py:105-111)."""
    if num_entries <= MAX_EIDS_UINT8:
        return np.uint8
    if num_entries <= MAX_EIDS:
        return np.uint16
    raise ValueError(f"E={num_entries} > {MAX_EIDS} does not fit 16-bit eids")


def pack_pids_24(pids):
    """int pids -> uint8 [3n] little endian; raises OverflowError outside [0, 2^24)
    (ragrt_index_lib.py:167-180)."""
    pids = np.asarray(pids)
    if not np.issubdtype(pids.dtype, np.integer):
        raise AssertionError(f"pids must be integers, got {pids.dtype}")
    if len(pids):
        lo, hi = int(pids.min()), int(pids.max())
        if lo < 0 or hi > MAX_PID:
            raise OverflowError(f"pid range [{lo}, {hi}] does not fit in {PID_BITS} bits")
    p = pids.astype(np.uint32)
    return np.stack([(p & 0xFF), (p >> 8) & 0xFF, (p >> 16) & 0xFF], axis=1).astype(np.uint8).reshape(-1)


def unpack_pids_24(packed):
    """uint8 [3n] -> int64 pids (ragrt_index_lib.py:183-185)."""
    b = np.asarray(packed, dtype=np.uint8).reshape(-1, 3).astype(np.uint32)
    return (b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)).astype(np.int64)


def block_sums(lengths, block=BLOCK_SIZE):
    """block_sums[b] = sum(lengths[:block * b]) (ragrt_index_lib.py:238-247)."""
    lengths = np.asarray(lengths, dtype=np.int64)
    nb = (len(lengths) + block - 1) // block
    padded = np.zeros(nb * block, dtype=np.int64)
    padded[:len(lengths)] = lengths
    totals = padded.reshape(nb, block).sum(axis=1)
    out = np.zeros(nb, dtype=np.int64)
    if nb > 1:
        out[1:] = np.cumsum(totals[:-1])
    return out


def offsets_from_block_sums(bsums, lengths, list_ids, block=BLOCK_SIZE):
    """Posting offset of each list: its block's sum plus the lengths before it in the block
    (the arithmetic of ragrt_fused_kernel.cu:208-213; ragrt_index_lib.py:250-257)."""
    lengths = np.asarray(lengths, dtype=np.int64)
    list_ids = np.asarray(list_ids, dtype=np.int64)
    csum = np.concatenate([[0], np.cumsum(lengths)])
    b = list_ids // block
    return np.asarray(bsums, dtype=np.int64)[b] + (csum[list_ids] - csum[b * block])
