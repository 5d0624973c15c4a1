"""Edge cases of the `weft` search through the C ABI against the CPU oracle:
  * null queries: all-zero query tokens make every centroid score tie at 0, so after the
    imputation shift no probe passes the base > 0 rule (ragrt_fused_kernel.cu:206) and the
    query gets no candidates: its top-k is all -1 with -inf scores; a query whose tokens are
    partly zero keeps the contribution of the others;
  * the smallest and largest probe counts (nc = 1: Stage 2 keeps the top 2 and shifts by the
    second; nc = 128, the interface's maximum, on the SIMT Stage-2 kernel);
  * batches below one 128-row Stage-2 tile (1 and 3 queries);
  * the largest final cut (k_top = K: the whole candidate list, ranked)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import small_corpus, oracle_index, weft_index

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


@pytest.fixture(scope="module")
def corpus():
    d, Q, E, centres = small_corpus()
    return d, Q, E, oracle_index(d), weft_index(d, E)


def _check(ids, sc, oids, osc, oix, Q):
    for b in range(Q.shape[0]):
        assert np.array_equal(ids[b] < 0, oids[b] < 0)
        assert np.array_equal(np.isinf(sc[b]), np.isinf(osc[b]))
        fin = np.isfinite(osc[b])
        rel = np.abs(sc[b][fin] - osc[b][fin]) / np.maximum(np.abs(osc[b][fin]), 1.0)
        assert rel.max(initial=0) < REL_TOL
        for i in np.flatnonzero((ids[b] != oids[b]) & fin):          # Stage-4 ties within tolerance
            s_ours = O.tile_maxsim(oix, Q[b].numpy(), np.array([ids[b][i]], np.int32))[0]
            assert abs(s_ours - osc[b][i]) <= 2 * REL_TOL * max(abs(osc[b][i]), 1.0), (b, i)


def _run(corpus, Q, nc, K, k_top):
    d, _, E, oix, wix = corpus
    ids, sc = wix.search(Q.cuda(), nc=nc, K=K, k_top=k_top)
    oids, osc, _ = O.weft_search(oix, Q.numpy(), np.full(Q.shape[0], 32, np.int32), nc, E, None, K, k_top)
    _check(ids.cpu().numpy(), sc.cpu().numpy(), oids, osc, oix, Q)
    return ids.cpu().numpy(), sc.cpu().numpy()


def test_null_queries(corpus):
    Q = corpus[1].clone()
    Q[1] = 0
    Q[3, 5:] = 0
    ids, sc = _run(corpus, Q, 16, 300, 10)
    assert (ids[1] == -1).all() and np.isneginf(sc[1]).all()
    assert (ids[3] >= 0).all()


@pytest.mark.parametrize("nc", [1, 128])
def test_probe_count_limits(corpus, nc):
    _run(corpus, corpus[1], nc, 300, 10)


@pytest.mark.parametrize("B", [1, 3])
def test_small_batches(corpus, B):
    _run(corpus, corpus[1][:B].contiguous(), 16, 300, 10)


def test_whole_candidate_list_ranked(corpus):
    ids, sc = _run(corpus, corpus[1], 16, 500, 500)
    for b in range(ids.shape[0]):
        fin = np.isfinite(sc[b])
        assert np.all(np.diff(sc[b][fin]) <= 0)
