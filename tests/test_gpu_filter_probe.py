"""Filter-aware probing (the `weft_oracle` / `weft_adapt` callers, src/weft_prep.py:75-170) on
the sm_100a kernels: per-centroid passing / total posting counts against a numpy count over the
index arrays, and the probe selections against the same rules applied to the CPU oracle's exact
Stage-2 scores (bit-exact: both rank by the exact fp16 score, ties to the lower centroid)."""
import numpy as np
import pytest

from oracle import oracle as O
from ragrt_b200.compat import weft_prep as wp
from tests.helpers import small_corpus, to_numpy, weft_index

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def corpus():
    d, Q, E, _ = small_corpus()
    return d, Q, E, weft_index(d, E)


def _numpy_counts(d, mask):
    n = to_numpy(d)
    rp = n["csr_row_ptrs"][0]
    lens = n["csr_lengths"].astype(np.int64)
    off = np.concatenate([[0], np.cumsum(lens)])
    packed = n["csr_packed_24"].reshape(-1, 3).astype(np.int64)
    pids = packed[:, 0] | (packed[:, 1] << 8) | (packed[:, 2] << 16)
    preds = n["doc_predicates"].astype(np.int64)
    NC = rp.shape[0] - 1
    tot = np.zeros(NC, np.int64)
    pas = np.zeros(NC, np.int64)
    for c in range(NC):
        a, b = off[rp[c]], off[rp[c + 1]]
        tot[c] = b - a
        pas[c] = (b - a) if mask == 0 else int(((preds[pids[a:b]] & mask) != 0).sum())
    return pas, tot


@pytest.mark.parametrize("mask", [0, 1, 2, 4])
def test_pass_counts(corpus, mask):
    d, Q, E, wix = corpus
    pc, tc = wix.pass_counts(mask)
    pas, tot = _numpy_counts(d, mask)
    assert np.array_equal(tc.cpu().numpy(), tot)
    assert np.array_equal(pc.cpu().numpy(), pas)


def test_oracle_fast_prep_on_compacted_centroids(corpus):
    d, Q, E, wix = corpus
    pass_c, tot_c, empty, n_ok = wp.centroid_filter_counts(wix, 1)        # 1 % selectivity: empties exist
    assert bool(empty.any()) and n_ok > 16
    C = d["centroids"].cuda()
    C_ok, ids = wp.compact_centroids(C, empty)
    q = Q[0].cuda()
    topc, sc, last = wp.oracle_fast_prep(q, C_ok, ids, 16)
    t, s, _, _ = O.native_prep(Q[0].numpy(), C_ok.cpu().numpy(), 16, impute=True)
    assert np.array_equal(topc.cpu().numpy(), ids.cpu().numpy()[t])
    assert np.array_equal(sc.cpu().numpy(), s)
    assert not bool(empty[topc.long()].any())


@pytest.mark.parametrize("sel_mask,q_", [(1, 1.0), (4, 0.5)])
def test_adaptive_probe_rule(corpus, sel_mask, q_):
    d, Q, E, wix = corpus
    pass_c, tot_c, _, _ = wp.centroid_filter_counts(wix, sel_mask)
    sel = float(pass_c.sum()) / float(tot_c.sum())
    C = d["centroids"].cuda()
    nc, ncap = 8, 40
    topc, sc, nc2 = wp.adaptive_probe(Q[1].cuda(), C, nc, ncap, pass_c, tot_c, sel, q=q_, slack=1.0)
    # the same rule on the oracle's exact top-(ncap+1)
    t, v, _, _ = O.native_prep(Q[1].numpy(), C.cpu().numpy(), ncap + 1, impute=False)
    pc, tc = pass_c.cpu().numpy(), tot_c.cpu().numpy()
    target = sel * tc[t[:, :nc]].sum(1)
    short = float(np.mean(pc[t[:, :nc]].sum(1) < target))
    if short <= 1.0 - q_ + 1e-9:
        want = nc
    else:
        cum = np.cumsum(pc[t[:, :ncap]], 1)
        need = np.clip((cum < target[:, None]).sum(1) + 1, nc, ncap).astype(np.float32)
        want = int(np.ceil(np.quantile(need, q_))) if q_ < 1.0 else int(need.max())
        want = max(nc, min(ncap, want))
    assert nc2 == want
    assert np.array_equal(topc.cpu().numpy(), t[:, :nc2])
    assert np.allclose(sc.cpu().numpy(), v[:, :nc2] - v[:, nc2:nc2 + 1], rtol=0, atol=0)
