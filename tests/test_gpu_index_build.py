"""
The GPU index build (ragrt_b200.index_build on CUDA tensors) against the reference builder's
arrays: the golden fixture that tests/golden/make_golden.py made by running the reference's own
plain_ivf_csr / block_sums / pack_pids_24 (src/build_plain_ivf.py:28-68,
src/ragrt_index_lib.py:167-247), for the default list cap and a tiny one that splits lists into
chunks; then a corpus large enough to split lists (70,000 passages on 8,192 centroids, cap 100)
built on the GPU and on the CPU, array for array, and bound for a search.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "plain_ivf.npz")


def _arrays(ix):
    lens = ix["csr_lengths"].view(torch.int16).cpu().numpy().view(np.uint16).astype(np.int64)
    return {"row_ptrs": ix["csr_row_ptrs"].cpu().numpy(),
            "col_eids": ix["csr_col_eids"].cpu().numpy().astype(np.int64),
            "lengths": lens, "block_sums": ix["csr_block_sums"].cpu().numpy(),
            "packed": ix["csr_packed_24"].cpu().numpy()}


def test_gpu_build_matches_reference_golden():
    from ragrt_b200 import index_build
    g = np.load(GOLDEN)
    codes = torch.from_numpy(np.asarray(g["codes"], np.int32)).cuda()
    dl = torch.from_numpy(np.asarray(g["doclens"], np.int32)).cuda()
    for ml in (65535, 5):
        ix = index_build.plain_ivf_index(codes, dl, int(g["num_centroids"]), max_len=ml)
        assert ix["csr_row_ptrs"].is_cuda and ix["csr_packed_24"].is_cuda
        a = _arrays(ix)
        assert np.array_equal(a["row_ptrs"], g[f"row_ptrs_{ml}"]), ml
        assert np.array_equal(a["col_eids"], g[f"col_eids_{ml}"].astype(np.int64)), ml
        assert np.array_equal(a["lengths"], g[f"lengths_{ml}"].astype(np.int64)), ml
        assert np.array_equal(a["block_sums"], g[f"block_sums_{ml}"]), ml
        assert np.array_equal(a["packed"], g[f"packed_{ml}"]), ml
        assert ix["num_postings"] == len(g[f"pids_sorted_{ml}"])
        assert ix["E"] == max(4, int(g[f"E_needed_{ml}"]))


def test_gpu_build_equals_cpu_build_and_binds():
    from ragrt_b200 import index_build, synth
    from ragrt_b200.weft import WeftIndex
    centres, C = synth.make_centroids(num_centres=128, subs=64, seed=4, device="cuda")
    corp = synth.make_corpus(70_000, centres, C, len_range=(20, 120), seed=4, device="cuda")
    gpu = index_build.plain_ivf_index(corp["codes"], corp["doclens"], C.shape[0], max_len=100)
    cpu = index_build.plain_ivf_index(corp["codes"].cpu(), corp["doclens"].cpu(), C.shape[0], max_len=100)
    ag, ac = _arrays(gpu), _arrays(cpu)
    for k in ag:
        assert np.array_equal(ag[k], ac[k]), k
    assert gpu["E"] == cpu["E"] > 4                      # lists were split into several chunks
    wix = WeftIndex(gpu["csr_row_ptrs"], gpu["csr_col_eids"], gpu["csr_block_sums"], gpu["csr_lengths"],
                    gpu["csr_packed_24"], corp["doc_offsets"], corp["doclens"], corp["codes"], corp["residuals"], C,
                    corp["bucket_weights"], corp["reversed_bit_map"], corp["decomp_table"], E=gpu["E"])
    Q = synth.make_queries(centres, 4, seed=5)
    ids, sc = wix.search(Q, nc=16, K=512, k_top=10)
    assert bool((ids >= 0).all()) and bool(torch.isfinite(sc).all())
