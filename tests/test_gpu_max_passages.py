"""The CUDA path at the maximum corpus size of the posting format: 2^24 passages, pids up to
2^24 - 1, through the C ABI against the CPU oracle.  Stage-3 candidates are bit-exact; the
search's ids are identical except where Stage-4 scores tie within the 1e-3 tolerance."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_PASSAGES, max_pid_corpus, oracle_index, weft_index

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
NC, K, K_TOP = 16, 300, 10


@pytest.fixture(scope="module")
def corpus():
    d, Q, E, _ = max_pid_corpus()
    return d, Q, E, oracle_index(d), weft_index(d, E)


def test_index_binds_the_full_pid_space(corpus):
    d, Q, E, oix, wix = corpus
    assert wix.N == MAX_PASSAGES


def test_candidates_bit_exact(corpus):
    d, Q, E, oix, wix = corpus
    topc, sc, _, _ = wix.centroid_topk(Q.cuda(), NC)
    pids, sums, _ = wix.candidates(topc, sc, K)
    pids, sums = pids.cpu().numpy(), sums.cpu().numpy()
    topc, sc = topc.cpu().numpy(), sc.cpu().numpy()
    for b in range(Q.shape[0]):
        op, os_, _ = O.candidates(oix, topc[b], sc[b], E, 0, K)
        assert np.array_equal(pids[b], op) and np.array_equal(sums[b], os_)
    assert pids.max() >= MAX_PASSAGES - 1000


def test_search_matches_oracle(corpus):
    d, Q, E, oix, wix = corpus
    ntok = torch.tensor([32, 29, 32, 23], dtype=torch.int32)
    masks = torch.tensor([0, 1, 0, 2], dtype=torch.int32)
    ids, sc = wix.search(Q.cuda(), nc=NC, K=K, k_top=K_TOP, ntok=ntok.cuda(), masks=masks.cuda())
    ids, sc = ids.cpu().numpy(), sc.cpu().numpy()
    oids, osc, _ = O.weft_search(oix, Q.numpy(), ntok.numpy(), NC, E, masks.numpy().astype(np.uint32), K, K_TOP)
    for b in range(Q.shape[0]):
        fin = np.isfinite(osc[b])
        rel = np.abs(sc[b][fin] - osc[b][fin]) / np.maximum(np.abs(osc[b][fin]), 1.0)
        assert rel.max(initial=0) < REL_TOL
        for i in np.flatnonzero(ids[b] != oids[b]):
            s_ours = O.tile_maxsim(oix, Q[b].numpy(), np.array([ids[b][i]], np.int32))[0]
            assert abs(s_ours - osc[b][i]) <= 2 * REL_TOL * max(abs(osc[b][i]), 1.0), (b, i, ids[b], oids[b])
