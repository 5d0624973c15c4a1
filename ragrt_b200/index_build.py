"""
Corpus-scale plain-IVF index build in torch, on the GPU (or the CPU for small tests): from the
per-token centroid codes of a corpus to the arrays ``CorrIndex3D.bind_index`` takes, in the
layout the reference's ``build_plain_ivf.py`` writes (the layout is the interface; the build
here is this package's own):

  csr_row_ptrs    int64  [32, NC + 1]  row 0: the lists of centroid c are [row[c], row[c+1]);
                                        rows 1-31 all equal the number of lists (plain IVF)
  csr_col_eids    uint8 (E <= 256) or int16  chunk number of each list within its centroid
  csr_lengths     uint16 [n_lists]     postings per list, at most max_len (65,535)
  csr_block_sums  int64  [ceil(n_lists / 128)]  first posting of list 128 b
  csr_packed_24   uint8  [3 P]         pids, 24-bit little endian, sorted by (centroid, pid)

A posting is a distinct (centroid, passage) pair.  A centroid's postings are cut into chunks
of max_len in pid order; chunk k of centroid c is list row[c] + k.  A 240 M-token corpus builds
in seconds on a B200.
"""
import torch

PID_BITS = 24
MAX_LIST_LENGTH = 65535
NUM_SUBSPACES = 32
BLOCK = 128


def _exclusive_cumsum(x):
    out = torch.zeros_like(x)
    if x.numel() > 1:
        out[1:] = torch.cumsum(x[:-1], 0)
    return out


def pack_pids_24(pids):
    """Passage ids (integer tensor) -> uint8 [3 n], each pid as 3 little-endian bytes; raises
    OverflowError for a pid outside [0, 2^24)."""
    b = pids.to(torch.int64).reshape(-1)
    if b.numel() and (int(b.min()) < 0 or int(b.max()) >= (1 << PID_BITS)):
        raise OverflowError(f"pids must lie in [0, 2^{PID_BITS})")
    return torch.stack([b & 0xFF, (b >> 8) & 0xFF, (b >> 16) & 0xFF], 1).to(torch.uint8).reshape(-1)


def unpack_pids_24(packed):
    """uint8 [3 n] -> int64 pids [n]."""
    b = packed.reshape(-1, 3).to(torch.int64)
    return b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)


def plain_ivf_index(codes, doclens, num_centroids, max_len=MAX_LIST_LENGTH, E=None):
    """codes int32 [T] (the tokens of passage p follow those of passage p - 1), doclens int32
    [N] -> dict of bind arrays (torch, on the inputs' device), plus "E" (chunk ids per centroid,
    at least 4) and "num_postings"."""
    dev = codes.device
    N = int(doclens.shape[0])
    if N > (1 << PID_BITS):
        raise OverflowError(f"{N} passages do not fit 24-bit pids")
    span = max(N, 1)
    # every token as (centroid, passage); one posting per distinct pair, in (centroid, pid) order
    owner = torch.repeat_interleave(torch.arange(N, device=dev, dtype=torch.int64), doclens.long())
    pair = torch.unique(codes.long() * span + owner)
    del owner
    cent = pair // span
    pid = (pair - cent * span).to(torch.int32)
    del pair
    P = int(pid.shape[0])
    # chunking: a posting's rank inside its centroid decides its chunk
    per_centroid = torch.bincount(cent, minlength=num_centroids)
    first_posting = _exclusive_cumsum(per_centroid)
    chunks = (per_centroid + max_len - 1) // max_len
    first_list = _exclusive_cumsum(chunks)
    n_lists = int(chunks.sum())
    rank = torch.arange(P, device=dev, dtype=torch.int64) - first_posting[cent]
    list_of_posting = first_list[cent] + rank // max_len
    del rank
    lengths = torch.bincount(list_of_posting, minlength=n_lists)
    del list_of_posting, cent
    # chunk number of each list: list index minus its centroid's first list
    list_centroid = torch.repeat_interleave(torch.arange(num_centroids, device=dev), chunks)
    chunk_no = torch.arange(n_lists, device=dev) - first_list[list_centroid]
    row = torch.empty(num_centroids + 1, dtype=torch.int64, device=dev)
    row[0] = 0
    row[1:] = torch.cumsum(chunks, 0)
    row_ptrs = row.new_full((NUM_SUBSPACES, num_centroids + 1), n_lists)
    row_ptrs[0] = row
    # first posting of every 128th list
    list_start = _exclusive_cumsum(lengths)
    block_sums = list_start[::BLOCK].contiguous() if n_lists else torch.zeros(0, dtype=torch.int64, device=dev)
    e_max = int(chunks.max()) if n_lists else 1
    E = max(4, e_max) if E is None else E
    return {
        "csr_row_ptrs": row_ptrs,
        "csr_col_eids": chunk_no.to(torch.uint8 if E <= 256 else torch.int16),
        "csr_block_sums": block_sums,
        "csr_lengths": lengths.to(torch.int32).to(torch.uint16) if hasattr(torch, "uint16") else lengths.to(torch.int16),
        "csr_packed_24": pack_pids_24(pid),
        "E": E,
        "num_postings": P,
    }
