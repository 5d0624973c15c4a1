"""
Corpus-scale plain-IVF build in torch (CPU or GPU): the same arrays as
``compat.build_plain_ivf.plain_ivf_csr`` + ``to_bind_arrays`` (the reference's
build_plain_ivf.py:28-68, :98-127), computed with sort/unique so a 240 M-token corpus
builds in seconds on a B200 instead of minutes in numpy.
"""
import torch

PID_BITS = 24
MAX_LIST_LENGTH = 65535
NUM_SUBSPACES = 32
BLOCK = 128


def plain_ivf_index(codes, doclens, num_centroids, max_len=MAX_LIST_LENGTH, E=None):
    """codes int32 [T], doclens int32 [N] -> dict of bind arrays (torch, same device)."""
    dev = codes.device
    N = doclens.shape[0]
    if N > (1 << PID_BITS):
        raise OverflowError(f"{N} passages do not fit 24-bit pids")
    pid = torch.repeat_interleave(torch.arange(N, device=dev, dtype=torch.int64), doclens.long())
    key = (codes.long() << PID_BITS) | pid
    del pid
    key = torch.unique(key)                     # sorted, deduplicated per (centroid, pid)
    c = key >> PID_BITS
    p = (key & ((1 << PID_BITS) - 1)).to(torch.int32)
    del key
    per_c = torch.bincount(c, minlength=num_centroids)
    del c
    nchunk = (per_c + max_len - 1) // max_len
    n_lists = int(nchunk.sum())
    list_cid = torch.repeat_interleave(torch.arange(num_centroids, device=dev), nchunk)
    first = torch.cumsum(nchunk, 0) - nchunk
    eids = torch.arange(n_lists, device=dev) - first[list_cid]
    lengths = torch.minimum(torch.full_like(eids, max_len), per_c[list_cid] - eids * max_len)
    row = torch.zeros(num_centroids + 1, dtype=torch.int64, device=dev)
    row[1:] = torch.cumsum(nchunk, 0)
    row_ptrs = torch.empty(NUM_SUBSPACES, num_centroids + 1, dtype=torch.int64, device=dev)
    row_ptrs[0] = row
    row_ptrs[1:] = n_lists
    e_needed = int(nchunk.max()) if n_lists else 1
    E = max(4, e_needed) if E is None else E
    nb = (n_lists + BLOCK - 1) // BLOCK
    padded = torch.zeros(nb * BLOCK, dtype=torch.int64, device=dev)
    padded[:n_lists] = lengths
    tot = padded.view(nb, BLOCK).sum(1)
    bsums = torch.zeros(nb, dtype=torch.int64, device=dev)
    if nb > 1:
        bsums[1:] = torch.cumsum(tot[:-1], 0)
    packed = torch.stack([p & 0xFF, (p >> 8) & 0xFF, (p >> 16) & 0xFF], dim=1).to(torch.uint8).reshape(-1)
    return {
        "csr_row_ptrs": row_ptrs,
        "csr_col_eids": eids.to(torch.uint8 if E <= 256 else torch.int16),
        "csr_block_sums": bsums,
        "csr_lengths": lengths.to(torch.int32).to(torch.uint16) if hasattr(torch, "uint16") else lengths.to(torch.int16),
        "csr_packed_24": packed,
        "E": E,
        "num_postings": int(p.shape[0]),
    }
