"""
Parity at the benchmarked configuration's shape: 65,536 fp16 centroids (1,024 centres x 64
sub-centroids), nprobe 32 with imputation, K = 4,096 candidates, top-10, passages of U[60,180]
tokens.  The corpus is 250,000 passages (cfg3 has 2 M; the oracle must finish in seconds) and
8 queries of one 256-query batch are checked, unfiltered and with each of the cfg4 predicate
masks (bits with selectivity 1 %, 10 %, 50 %).

Bit-exact: Stage-2 probes and scores, Stage-3 candidate lists (pids, order, fp32 sums).
Tolerance: final top-10 scores within 1e-3 relative of the oracle's fp64 MaxSim; ids equal
except where Stage-4 scores tie within that tolerance (oracle.topk_agreement).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import oracle_index

pytestmark = pytest.mark.gpu

NUM_DOCS = 250_000
NQ = 8
NC, K, K_TOP = 32, 4096, 10
REL_TOL = 1e-3


@pytest.fixture(scope="module")
def cfg3():
    from ragrt_b200 import synth, index_build
    from ragrt_b200.weft import WeftIndex
    dev = "cuda"
    centres, cents = synth.make_centroids(num_centres=1024, subs=64, seed=0, device=dev)
    corp = synth.make_corpus(NUM_DOCS, centres, cents, len_range=(60, 180), seed=0, device=dev)
    preds = synth.make_predicates(NUM_DOCS, seed=1, device=dev)
    ix = index_build.plain_ivf_index(corp["codes"], corp["doclens"], cents.shape[0])
    d = {"csr_row_ptrs": ix["csr_row_ptrs"], "csr_col_eids": ix["csr_col_eids"],
         "csr_block_sums": ix["csr_block_sums"], "csr_lengths": ix["csr_lengths"],
         "csr_packed_24": ix["csr_packed_24"], "doc_offsets": corp["doc_offsets"], "doc_lens": corp["doclens"],
         "codes": corp["codes"], "residuals": corp["residuals"], "centroids": cents,
         "bucket_weights": corp["bucket_weights"], "reversed_bit_map": corp["reversed_bit_map"],
         "decomp_table": corp["decomp_table"], "doc_predicates": preds}
    wix = WeftIndex(d["csr_row_ptrs"], d["csr_col_eids"], d["csr_block_sums"], d["csr_lengths"],
                    d["csr_packed_24"], d["doc_offsets"], d["doc_lens"], d["codes"], d["residuals"], cents,
                    d["bucket_weights"], d["reversed_bit_map"], d["decomp_table"],
                    doc_predicates=preds.to(torch.int64).to(torch.int32), num_passages=NUM_DOCS,
                    num_centroids=cents.shape[0], E=ix["E"])
    oix = oracle_index(d)
    # a 256-query batch (Stage 2's tensor-core tiling at the benchmarked batch); 8 are checked
    Q = synth.make_queries(centres, 256, seed=1000)
    otopc, os2, om = O.native_prep_batch(Q[:NQ].cpu().numpy(), np.full(NQ, 32, np.int32), cents.cpu().numpy(), NC)
    return wix, oix, Q, ix["E"], otopc, os2, om


def test_cfg3_stage2_bit_exact(cfg3):
    wix, oix, Q, E, otopc, os2, om = cfg3
    topc, sc, m, _ = wix.centroid_topk(Q, NC)
    topc, sc, m = topc[:NQ].cpu().numpy(), sc[:NQ].cpu().numpy(), m[:NQ].cpu().numpy()
    assert np.array_equal(topc, otopc), "probed centroids differ from the oracle at 65,536 centroids"
    assert np.array_equal(sc.view(np.uint32), os2.view(np.uint32)), "probe scores differ"
    assert np.array_equal(m, om)


@pytest.mark.parametrize("mask", [0, 1, 2, 4])
def test_cfg3_candidates_and_top10(cfg3, mask):
    wix, oix, Q, E, otopc, os2, om = cfg3
    masks = torch.full((Q.shape[0],), mask, dtype=torch.int32, device="cuda")
    topc, sc, _, _ = wix.centroid_topk(Q, NC)
    cp, cs, touched = wix.candidates(topc, sc, K, masks=masks)
    ids, fsc = wix.search(Q, nc=NC, K=K, k_top=K_TOP, masks=masks)
    cp, cs, touched = cp[:NQ].cpu().numpy(), cs[:NQ].cpu().numpy(), touched[:NQ].cpu().numpy()
    for b in range(NQ):
        op, osum, st = O.candidates(oix, otopc[b], os2[b], E, mask, K)
        assert touched[b] == st["touched"], (b, touched[b], st["touched"])
        assert np.array_equal(cp[b], op), f"query {b} mask {mask}: Stage-3 candidates differ"
        assert np.array_equal(cs[b].view(np.uint32), osum.view(np.uint32)), f"query {b}: Stage-3 sums differ"
    q = Q[:NQ].cpu().numpy()
    mk = np.full(NQ, mask, np.uint32)
    oids, osc, _ = O.weft_search(oix, q, np.full(NQ, 32, np.int32), NC, E, mk, K, K_TOP)
    a = O.topk_agreement(oix, q, ids[:NQ].cpu().numpy(), fsc[:NQ].cpu().numpy(), oids, osc, masks=mk,
                         rel_tol=REL_TOL)
    assert a["max_rel_score_err"] < REL_TOL, a
    assert a["mismatches"] == 0, a
