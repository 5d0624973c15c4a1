"""Shared fixtures: small seeded corpora in the plain-IVF layout (CPU tensors) and oracle views."""
import functools

import numpy as np
import torch

from ragrt_b200 import synth, index_build

BIND_KEYS = ("csr_row_ptrs", "csr_col_eids", "csr_block_sums", "csr_lengths", "csr_packed_24", "doc_offsets",
             "doc_lens", "codes", "residuals", "centroids", "bucket_weights", "reversed_bit_map", "decomp_table",
             "doc_predicates")


@functools.lru_cache(maxsize=8)
def small_corpus(num_docs=3000, num_centres=64, subs=8, len_range=(8, 60), seed=0, max_len=65535, nq=6):
    """A small plain-IVF corpus + queries, CPU tensors (deterministic)."""
    centres, cents = synth.make_centroids(num_centres=num_centres, subs=subs, seed=seed)
    corp = synth.make_corpus(num_docs, centres, cents, seed=seed, len_range=len_range)
    ix = index_build.plain_ivf_index(corp["codes"], corp["doclens"], cents.shape[0], max_len=max_len)
    preds = synth.make_predicates(num_docs, seed=1)
    Q = synth.make_queries(centres, nq, seed=seed + 100)
    d = {
        "csr_row_ptrs": ix["csr_row_ptrs"], "csr_col_eids": ix["csr_col_eids"],
        "csr_block_sums": ix["csr_block_sums"], "csr_lengths": ix["csr_lengths"],
        "csr_packed_24": ix["csr_packed_24"], "doc_offsets": corp["doc_offsets"], "doc_lens": corp["doclens"],
        "codes": corp["codes"], "residuals": corp["residuals"], "centroids": cents,
        "bucket_weights": corp["bucket_weights"], "reversed_bit_map": corp["reversed_bit_map"],
        "decomp_table": corp["decomp_table"], "doc_predicates": preds,
    }
    return d, Q, ix["E"], centres


def to_numpy(d):
    out = {}
    for k, v in d.items():
        if torch.is_tensor(v):
            if v.dtype == torch.float16:
                out[k] = v.cpu().numpy()
            elif v.dtype == torch.uint16:
                out[k] = v.cpu().view(torch.int16).numpy().view(np.uint16)
            elif v.dtype == torch.uint32:
                out[k] = v.cpu().to(torch.int64).numpy().astype(np.uint32)
            else:
                out[k] = v.cpu().numpy()
        else:
            out[k] = v
    return out


def oracle_index(d):
    from oracle import oracle as O
    return O.Index(to_numpy(d))


def to_cuda(d):
    out = {}
    for k, v in d.items():
        if torch.is_tensor(v):
            out[k] = v.view(torch.int16).cuda().view(torch.uint16) if v.dtype == torch.uint16 else (
                v.to(torch.int64).to(torch.int32).cuda() if v.dtype == torch.uint32 else v.cuda())
        else:
            out[k] = v
    return out


def weft_index(d, E):
    from ragrt_b200.weft import WeftIndex
    g = to_cuda(d)
    return WeftIndex(*[g[k] for k in BIND_KEYS], num_passages=g["doc_lens"].shape[0],
                     num_centroids=g["centroids"].shape[0], E=E)


MAX_PASSAGES = 1 << 24                    # 24-bit packed pids (ragrt_index_lib.py:23-24)


@functools.lru_cache(maxsize=1)
def max_pid_corpus(num_docs=2000, nq=4):
    """The largest corpus the 24-bit posting format holds: 2^24 passages, of which only the
    first and the last num_docs/2 have tokens (the documents of small_corpus), so pids reach
    2^24 - 1 while the arrays stay small.  Returns (d, Q, E, pid_map): pid_map[i] is the pid of
    small_corpus document i in this corpus."""
    d0, Q, _, _ = small_corpus(num_docs=num_docs, nq=nq)
    N, half = MAX_PASSAGES, num_docs // 2
    pid_map = torch.cat([torch.arange(half), torch.arange(N - (num_docs - half), N)])
    doclens = torch.zeros(N, dtype=torch.int32)
    doclens[pid_map] = d0["doc_lens"]
    offsets = torch.zeros(N + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(doclens.long(), 0)
    preds = torch.zeros(N, dtype=torch.int64)
    preds[pid_map] = d0["doc_predicates"].to(torch.int64)
    ix = index_build.plain_ivf_index(d0["codes"], doclens, d0["centroids"].shape[0])
    d = dict(d0)
    d.update({"csr_row_ptrs": ix["csr_row_ptrs"], "csr_col_eids": ix["csr_col_eids"],
              "csr_block_sums": ix["csr_block_sums"], "csr_lengths": ix["csr_lengths"],
              "csr_packed_24": ix["csr_packed_24"], "doc_offsets": offsets, "doc_lens": doclens,
              "doc_predicates": preds.to(torch.uint32)})
    return d, Q, ix["E"], pid_map
