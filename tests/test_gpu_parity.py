"""
Parity of the sm_100a CUDA path with the CPU oracle on seeded inputs, through the C ABI.

Bit-exact: Stage-2 probed centroids and scores, Stage-3 candidate sets, sums and order,
final top-k ids (where the Stage-4 scores do not tie within tolerance).
Tolerance: Stage-4 MaxSim scores within 1e-3 relative of the oracle (fp64 reference).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import small_corpus, oracle_index, weft_index

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3          # Stage-4 scores vs the fp64 oracle


@pytest.fixture(scope="module")
def corpus():
    d, Q, E, centres = small_corpus()
    return d, Q, E, oracle_index(d), weft_index(d, E)


def _ntok(B):
    return torch.tensor([32 - 3 * (b % 5) for b in range(B)], dtype=torch.int32)


@pytest.mark.parametrize("nc,impute", [(32, True), (32, False), (8, True), (128, True)])
def test_stage2_bit_exact(corpus, nc, impute):
    d, Q, E, oix, wix = corpus
    C = d["centroids"]
    ntok = _ntok(Q.shape[0])
    from ragrt_b200.weft import centroid_topk
    topc, sc, m, _ = centroid_topk(Q.cuda(), C.cuda(), nc, impute=impute, ntok=ntok.cuda())
    topc, sc, m = topc.cpu().numpy(), sc.cpu().numpy(), m.cpu().numpy()
    for b in range(Q.shape[0]):
        nt = int(ntok[b])
        ot, osc, om, _ = O.native_prep(Q[b, :nt].numpy(), C.numpy(), nc, impute=impute)
        assert np.array_equal(topc[b, :nt], ot), f"query {b}: probed centroids differ"
        assert np.array_equal(sc[b, :nt].view(np.uint32), osc.view(np.uint32)), f"query {b}: scores differ"
        if om is not None:
            assert np.array_equal(m[b, :nt], om)
        assert (topc[b, nt:] == -1).all()


def test_stage2_full_matrix_exact(corpus):
    d, Q, E, oix, wix = corpus
    from ragrt_b200.weft import centroid_topk
    C = d["centroids"]
    _, _, _, full = centroid_topk(Q[:1].cuda(), C.cuda(), 32, impute=True, full=True)
    full = full[0].cpu().numpy()
    ex = np.array([[O.rn16_dot(Q[0, t].numpy(), C[c].numpy()) for c in range(C.shape[0])] for t in range(32)])
    assert np.array_equal(full.view(np.uint16), ex.view(np.uint16))


def _stage2_oracle(Q, C, ntok, nc):
    B = Q.shape[0]
    topc = np.full((B, 32, nc), -1, np.int32)
    sc = np.zeros((B, 32, nc), np.float32)
    for b in range(B):
        nt = int(ntok[b])
        t, s, _, _ = O.native_prep(Q[b, :nt].numpy(), C.numpy(), nc, impute=True)
        topc[b, :nt], sc[b, :nt] = t, s
    return topc, sc


@pytest.mark.parametrize("K,mask", [(4096, 0), (300, 0), (50, 0), (300, 1), (300, 2), (2000, 4)])
def test_stage3_bit_exact(corpus, K, mask):
    d, Q, E, oix, wix = corpus
    ntok = _ntok(Q.shape[0])
    nc = 16
    topc, sc = _stage2_oracle(Q, d["centroids"], ntok, nc)
    masks = torch.full((Q.shape[0],), mask, dtype=torch.int32)
    K = min(K, wix.N)
    pids, sums, touched = wix.candidates(torch.from_numpy(topc).cuda(), torch.from_numpy(sc).cuda(), K,
                                         ntok=ntok.cuda(), masks=masks.cuda())
    pids, sums, touched = pids.cpu().numpy(), sums.cpu().numpy(), touched.cpu().numpy()
    for b in range(Q.shape[0]):
        nt = int(ntok[b])
        op, os_, st = O.candidates(oix, topc[b, :nt], sc[b, :nt], E, mask, K)
        assert touched[b] == st["touched"], (b, touched[b], st["touched"])
        assert np.array_equal(pids[b], op), f"query {b}: candidates differ"
        assert np.array_equal(sums[b].view(np.uint32), os_.view(np.uint32)), f"query {b}: sums differ"


@pytest.mark.parametrize("mask,range_passages", [(0, 0), (2, 0), (0, 8192)])
def test_stage3_modes_bit_identical(corpus, mask, range_passages):
    """Stage 3's walk-once kernel (mode 0, with the per-token kernel on ranges too dense for it)
    and the per-token kernel alone (mode 1) give the same candidates, sums and counts."""
    d, Q, E, oix, wix = corpus
    ntok = _ntok(Q.shape[0]).cuda()
    from ragrt_b200.weft import centroid_topk
    topc, sc, _, _ = centroid_topk(Q.cuda(), d["centroids"].cuda(), 32, impute=True, ntok=ntok)
    masks = torch.full((Q.shape[0],), mask, dtype=torch.int32, device="cuda")
    out = []
    for mode in (0, 1):
        wix.set_stage3_mode(mode, range_passages)
        wix.stats(reset=True)
        out.append(wix.candidates(topc, sc, 700, ntok=ntok, masks=masks) + (wix.stats(),))
    wix.set_stage3_mode(0)
    (p0, s0, t0, st0), (p1, s1, t1, st1) = out
    assert torch.equal(p0, p1) and torch.equal(s0, s1) and torch.equal(t0, t1)
    for k in ("postings", "distinct_postings", "touched", "probes", "tasks"):
        assert st0[k] == st1[k], k


def test_stage3_full_scores_and_eid_limit(corpus):
    d, Q, E, oix, wix = corpus
    ntok = _ntok(Q.shape[0])
    nc = 16
    from ragrt_b200.weft import centroid_topk
    topc, sc, m, full = centroid_topk(Q.cuda(), d["centroids"].cuda(), nc, impute=True, ntok=ntok.cuda(), full=True)
    fullsc = full.float() - m[:, :, None]
    p1, s1, _ = wix.candidates(topc, sc, 500, ntok=ntok.cuda())
    p2, s2, _ = wix.candidates(topc, fullsc, 500, ntok=ntok.cuda(), full_scores=True)
    assert torch.equal(p1, p2) and torch.equal(s1, s2)


@pytest.mark.parametrize("mode", [1, 0])
def test_stage4_matches_oracle(corpus, mode):
    d, Q, E, oix, wix = corpus
    g = torch.Generator().manual_seed(3)
    B, n = 3, 700
    pids = torch.randint(0, wix.N, (B, n), generator=g).to(torch.int32)
    pids[:, ::37] = -1
    pids[0, 5] = wix.N + 7                       # out of range -> -inf
    out = wix.tile_maxsim(Q[:B].cuda(), pids.cuda(), mode=mode).cpu().numpy()
    for b in range(B):
        ref = O.tile_maxsim(oix, Q[b].numpy(), pids[b].numpy())
        ref[pids[b].numpy() >= wix.N] = -np.inf
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(out[b]), fin)
        rel = np.abs(out[b][fin] - ref[fin]) / np.maximum(np.abs(ref[fin]), 1.0)
        assert rel.max() < REL_TOL, (mode, b, rel.max())


def test_stage4_golden_fp32_reference():
    """The reference test's fp32 TileMaxSim (tests/test_gpu_kernels.py:294-305), golden file."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "stage4.npz"))
    from ragrt_b200.weft import tile_maxsim
    t = lambda k, dt=None: torch.from_numpy(g[k]).cuda() if dt is None else torch.from_numpy(g[k]).to(dt).cuda()
    for mode in (1, 0):
        out = tile_maxsim(t("Q"), t("pids"), t("doc_offsets"), t("doc_lens"), t("codes"), t("residuals"),
                          t("centroids"), t("bucket_weights"), t("reversed_bit_map"), t("decomp_table"),
                          mode=mode).cpu().numpy()
        ref = g["ref"]
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(out), fin)
        assert np.abs(out[fin] - ref[fin]).max() < 0.02          # the reference test's own bound
        assert (np.abs(out[fin] - ref[fin]) / np.abs(ref[fin])).max() < REL_TOL


def test_stage4_empty_document():
    d, Q, E, _ = small_corpus()
    from ragrt_b200.weft import tile_maxsim
    lens = d["doc_lens"].clone()
    lens[3] = 0
    out = tile_maxsim(Q[0].cuda(), torch.tensor([3, 4], dtype=torch.int32).cuda(), d["doc_offsets"].cuda(),
                      lens.cuda(), d["codes"].cuda(), d["residuals"].cuda(), d["centroids"].cuda(),
                      d["bucket_weights"].cuda(), d["reversed_bit_map"].cuda(), d["decomp_table"].cuda())
    assert float(out[0]) == -3.2e10 and np.isfinite(float(out[1]))


def test_final_topk_rules(corpus):
    d, Q, E, oix, wix = corpus
    pids = torch.tensor([[5, -1, 7, 9, 3, 11], [2, 2, 4, -1, -1, 8]], dtype=torch.int32)
    sc = torch.tensor([[1.0, 9.0, 2.0, 2.0, 0.5, 2.0], [3.0, 3.0, 1.0, 0.0, 0.0, -1.0]])
    ids, s = wix.final_topk(pids.cuda(), sc.cuda(), 4)
    assert ids.cpu().tolist() == [[7, 9, 11, 5], [2, 2, 4, 8]]
    masks = torch.tensor([1, 0], dtype=torch.int32)
    ids, s = wix.final_topk(pids.cuda(), sc.cuda(), 6, masks=masks.cuda())
    for i in range(6):
        p = int(ids[0, i])
        if p >= 0 and not (int(d["doc_predicates"][p]) & 1):
            assert float(s[0, i]) == -np.inf


@pytest.mark.parametrize("rerank", ["tc", "simt"])
def test_weft_search_end_to_end(corpus, rerank):
    d, Q, E, oix, wix = corpus
    ntok = _ntok(Q.shape[0])
    masks = torch.tensor([0, 0, 1, 2, 4, 0], dtype=torch.int32)[:Q.shape[0]]
    nc, K, k_top = 16, 400, 10
    ids, sc = wix.search(Q.cuda(), nc=nc, K=K, k_top=k_top, ntok=ntok.cuda(), masks=masks.cuda(), rerank=rerank)
    ids, sc = ids.cpu().numpy(), sc.cpu().numpy()
    oids, osc, _ = O.weft_search(oix, Q.numpy(), ntok.numpy(), nc, E, masks.numpy(), K, k_top)
    for b in range(Q.shape[0]):
        fin = np.isfinite(osc[b])
        rel = np.abs(sc[b][fin] - osc[b][fin]) / np.maximum(np.abs(osc[b][fin]), 1.0)
        assert rel.max(initial=0) < REL_TOL
        # ids are identical except where Stage-4 scores tie within tolerance: the id at each
        # differing position must have an oracle score within tolerance of the oracle's there
        for i in np.flatnonzero(ids[b] != oids[b]):
            s_ours = O.tile_maxsim(oix, Q[b].numpy(), np.array([ids[b][i]], np.int32))[0]
            assert abs(s_ours - osc[b][i]) <= 2 * REL_TOL * max(abs(osc[b][i]), 1.0), (b, i, ids[b], oids[b])


def test_weft_search_matches_stagewise(corpus):
    d, Q, E, oix, wix = corpus
    ntok = _ntok(Q.shape[0]).cuda()
    nc, K = 16, 300
    ids, sc = wix.search(Q.cuda(), nc=nc, K=K, k_top=10, ntok=ntok)
    topc, s2, _, _ = wix.centroid_topk(Q.cuda(), nc, ntok=ntok)
    pids, _, _ = wix.candidates(topc, s2, K, ntok=ntok)
    f = wix.tile_maxsim(Q.cuda(), pids)
    ids2, sc2 = wix.final_topk(pids, f, 10)
    assert torch.equal(ids, ids2) and torch.equal(sc, sc2)


def test_invalid_index_is_rejected():
    d, Q, E, _ = small_corpus()
    from ragrt_b200._lib import RagrtError
    bad = dict(d)
    rp = d["csr_row_ptrs"].clone()
    rp[1, 5] = 0                                  # a non-empty "subspace" row: not plain IVF
    bad["csr_row_ptrs"] = rp
    from tests.helpers import weft_index as mk
    with pytest.raises(RagrtError, match="not a valid plain-IVF index"):
        mk(bad, E)


def test_documents_outside_the_codes_are_rejected():
    """A passage whose tokens reach past the bound codes / residuals fails at bind time (the
    search, which would read them on the device, never runs)."""
    d, Q, E, _ = small_corpus()
    from ragrt_b200._lib import RagrtError
    from tests.helpers import weft_index as mk
    bad = dict(d)
    lens = d["doc_lens"].clone()
    lens[-1] += 5                                 # the last passage ends 5 tokens past the codes
    bad["doc_lens"] = lens
    with pytest.raises(RagrtError, match="outside the num_tokens codes"):
        mk(bad, E)


@pytest.mark.parametrize("bad_code", [-1, "NC"])
def test_codes_outside_the_centroids_are_rejected(bad_code):
    """A doc token whose centroid code is not a row of the bound centroids fails at bind time,
    so neither rerank mode ever gathers outside the centroid table."""
    d, Q, E, _ = small_corpus()
    from ragrt_b200._lib import RagrtError
    from tests.helpers import weft_index as mk
    bad = dict(d)
    codes = d["codes"].clone()
    codes[len(codes) // 2] = -1 if bad_code == -1 else d["centroids"].shape[0]
    bad["codes"] = codes
    with pytest.raises(RagrtError, match="code is outside"):
        mk(bad, E)


@pytest.mark.parametrize("nq,ntok_drop", [(8, 0), (5, 7)])
def test_stage2_tensor_core_many_tiles(nq, ntok_drop):
    """Stage 2 with several 128-row tiles and centroid slices (the tcgen05 path) is bit-exact."""
    from ragrt_b200 import synth
    from ragrt_b200.weft import centroid_topk
    centres, C = synth.make_centroids(num_centres=256, subs=32, seed=9)        # 8,192 centroids
    Q = synth.make_queries(centres, nq, seed=9)
    ntok = torch.tensor([32 - (ntok_drop if b % 2 else 0) for b in range(nq)], dtype=torch.int32)
    topc, sc, m, _ = centroid_topk(Q.cuda(), C.cuda(), 32, impute=True, ntok=ntok.cuda())
    topc, sc, m = topc.cpu().numpy(), sc.cpu().numpy(), m.cpu().numpy()
    for b in range(nq):
        nt = int(ntok[b])
        ot, osc, om, _ = O.native_prep(Q[b, :nt].numpy(), C.numpy(), 32, impute=True)
        assert np.array_equal(topc[b, :nt], ot), f"query {b}: probed centroids differ"
        assert np.array_equal(sc[b, :nt].view(np.uint32), osc.view(np.uint32)), f"query {b}: scores differ"
        assert np.array_equal(m[b, :nt], om)
    from ragrt_b200 import _lib
    assert _lib.lib().ragrt_device_error(1) == 0
