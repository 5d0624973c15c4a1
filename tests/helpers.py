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
