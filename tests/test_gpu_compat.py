"""The drop-in modules as the reference's `weft` engine drives them (engines.py:403-426, :573-609):
`weft_prep.native_prep` for Stage 2, then `rtrag_corr_3d.CorrIndex3D` -- build, all-codewords
Stage 1, bind_index -- and its per-query, pipelined and batched searches, plus the module-level
MaxSim and the error conventions.  Results are checked against the oracle and against the
package's own batched search."""
import os
import sys

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import small_corpus, oracle_index, to_cuda, weft_index, BIND_KEYS

pytestmark = pytest.mark.gpu

COMPAT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "ragrt_b200", "compat")
if COMPAT not in sys.path:
    sys.path.insert(0, COMPAT)

import rtrag_corr_3d as R  # noqa: E402
from weft_prep import native_prep  # noqa: E402

REL_TOL = 1e-3
NC, K, K_TOP = 16, 300, 10


@pytest.fixture(scope="module")
def setup():
    d, Q, E, _ = small_corpus()
    g = to_cuda(d)
    R.set_codeword_weight(0.0)
    R.set_compact_scores(True)
    R.set_stage3_mode(0)
    R.set_rerank_mode("wmma")
    idx = R.CorrIndex3D("unused.ptx")
    idx.build(torch.zeros(32, E, 3, device="cuda"))
    idx.set_stage1_mode(2)
    idx.set_stage3_sparse(True)
    idx.bind_index(*[g[k] for k in BIND_KEYS], g["doc_lens"].shape[0], g["centroids"].shape[0])
    return d, g, Q.reshape(-1, 32, 128), E, idx


def _query_args(g, q):
    """The per-query arguments the engine passes: fp32 and fp16 query, an all-zero Q_sub3d
    (codeword weight 0) and native_prep's compact, imputed scores."""
    q16 = q.cuda().half().contiguous()
    topc, scores, _ = native_prep(q16, g["centroids"], NC, impute=True, compact=True)
    q_sub = torch.zeros(32, 32, 3, device="cuda")
    return q16.float(), q16, q_sub, topc, scores


def test_info_and_knobs(setup):
    d, g, Q, E, idx = setup
    info = idx.info()
    assert info["stage1"] == "all_codewords" and info["num_entries"] == E
    assert R.get_codeword_weight() == 0.0 and R.get_compact_scores() and R.get_stage3_mode() == 0


def test_single_query_native_matches_batched_search_and_oracle(setup):
    d, g, Q, E, idx = setup
    wix = weft_index(d, E)
    oix = oracle_index(d)
    ids_b, _ = wix.search(Q.cuda(), nc=NC, K=K, k_top=K_TOP)
    oids, osc, _ = O.weft_search(oix, Q.numpy(), np.full(Q.shape[0], 32, np.int32), NC, E, None, K, K_TOP)
    for b in range(Q.shape[0]):
        ids = idx.search_single_query_native(*_query_args(g, Q[b]), NC, K, K_TOP, 0, E)
        assert torch.equal(ids.cpu(), ids_b[b].cpu())
        got = ids.cpu().numpy()
        for i in np.flatnonzero(got != oids[b]):          # ties within the Stage-4 tolerance only
            s = O.tile_maxsim(oix, Q[b].numpy(), np.array([got[i]], np.int32))[0]
            assert abs(s - osc[b][i]) <= 2 * REL_TOL * max(abs(osc[b][i]), 1.0)


def test_profiled_and_pipelined_agree(setup):
    d, g, Q, E, idx = setup
    per_query = []
    for b in range(Q.shape[0]):
        ids, times = idx.search_single_query_profiled(*_query_args(g, Q[b]), NC, K, K_TOP, 0, E)
        assert len(times) == 4 and all(t >= 0 for t in times)
        per_query.append(ids.cpu())
    args = [_query_args(g, Q[b]) for b in range(Q.shape[0])]
    out = idx.search_batch_pipelined([a[0] for a in args], [a[1] for a in args], [a[2] for a in args],
                                     [a[3] for a in args], [a[4] for a in args], NC, K, K_TOP, 0, E)
    assert out.shape == (Q.shape[0], K_TOP)
    for b in range(Q.shape[0]):
        assert torch.equal(out[b].cpu(), per_query[b])


@pytest.mark.parametrize("mask", [0, 2])
def test_candidates_and_filter(setup, mask):
    d, g, Q, E, idx = setup
    wix = weft_index(d, E)
    a = _query_args(g, Q[0])
    pids, approx = idx.candidates(a[2], a[3], a[4], NC, K, mask, E)
    ref, ref_s, _ = wix.candidates(a[3][None], a[4][None], K, masks=torch.tensor([mask], dtype=torch.int32,
                                                                                   device="cuda") if mask else None)
    assert torch.equal(pids, ref[0]) and torch.equal(approx, ref_s[0])
    if mask:                                              # every kept candidate passes the filter
        kept = pids[pids >= 0].long()
        assert bool(((g["doc_predicates"][kept] & mask) != 0).all())


def test_drop_stats_count_postings_and_tasks(setup):
    """get_drop_stats() reports the reference's counters for the weft path: launches, rays,
    tasks (posting lists of the kept (token, probe) pairs) and postings (their postings),
    equal to the oracle's counts for the same queries; all zero while the stats are off."""
    d, g, Q, E, idx = setup
    oix = oracle_index(d)
    R.set_drop_stats(False)
    R.reset_drop_stats()
    a = _query_args(g, Q[0])
    idx.candidates(a[2], a[3], a[4], NC, K, 0, E)
    assert all(v == 0 for v in R.get_drop_stats().values())
    R.set_drop_stats(True)
    try:
        exp_post = exp_tasks = 0
        for b in range(2):
            a = _query_args(g, Q[b])
            idx.candidates(a[2], a[3], a[4], NC, K, 0, E)
            _, _, st = O.candidates(oix, a[3].cpu().numpy(), a[4].cpu().numpy(), E, 0, K)
            exp_post += st["postings"]
            exp_tasks += st["tasks"]
        got = R.get_drop_stats()
        assert got["launches"] == 2 and got["rays"] == 2 * 32 * 32
        assert got["postings"] == exp_post and got["tasks"] == exp_tasks, (got, exp_post, exp_tasks)
        assert exp_post > 0
    finally:
        R.set_drop_stats(False)
        R.reset_drop_stats()


def test_search_batch_entry(setup):
    d, g, Q, E, idx = setup
    wix = weft_index(d, E)
    ids, sc = idx.search_batch(Q.cuda().half(), NC, K, K_TOP)
    rids, rsc = wix.search(Q.cuda(), nc=NC, K=K, k_top=K_TOP)
    assert torch.equal(ids, rids) and torch.equal(sc, rsc)


def test_module_tile_maxsim(setup):
    d, g, Q, E, idx = setup
    oix = oracle_index(d)
    pids = torch.arange(0, 200, 3, dtype=torch.int32, device="cuda")
    q16 = Q[0].cuda().half().contiguous()
    got = R.native_tile_maxsim_fused_decomp(q16, pids, g["doc_offsets"], g["doc_lens"], g["codes"], g["residuals"],
                                            g["centroids"], g["bucket_weights"], g["reversed_bit_map"],
                                            g["decomp_table"]).cpu().numpy()
    ref = O.tile_maxsim(oix, Q[0].numpy(), pids.cpu().numpy())
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)) < REL_TOL


def test_error_conventions(setup):
    d, g, Q, E, idx = setup
    a = _query_args(g, Q[0])
    fresh = R.CorrIndex3D()
    with pytest.raises(RuntimeError):                     # search before bind_index
        fresh.search_single_query_native(*a, NC, K, K_TOP, 0, E)
    with pytest.raises(RuntimeError):                     # k_candidates out of range
        idx.search_single_query_native(*a, NC, 0, K_TOP, 0, E)
    with pytest.raises(RuntimeError):                     # wrong query shape for the fused MaxSim
        R.native_tile_maxsim_fused_decomp(a[1][:16], torch.zeros(4, dtype=torch.int32, device="cuda"),
                                          g["doc_offsets"], g["doc_lens"], g["codes"], g["residuals"],
                                          g["centroids"], g["bucket_weights"], g["reversed_bit_map"],
                                          g["decomp_table"])
    idx.set_stage1_mode(0)                                # the RT Stage 1 is another engine
    try:
        with pytest.raises(NotImplementedError):
            idx.search_single_query_native(*a, NC, K, K_TOP, 0, E)
    finally:
        idx.set_stage1_mode(2)
