"""Exact TileMaxSim over uncompressed fp16 passages (the exact-rerank workload: 64 queries x 32
tokens, 1,000 candidates per query with 20-180 tokens each, clustered unit-norm tokens).

Reference: score = sum over query rows of max over the passage's tokens of q . d, computed here
in fp64 from the same fp16 inputs.  Tolerance: 1e-3 relative (the tensor cores accumulate the
fp16 products in fp32).  The final top-10 must agree wherever the 10th and 11th reference
scores are separated by more than that tolerance.
"""
import numpy as np
import pytest
import torch

from ragrt_b200 import synth
from ragrt_b200.weft import final_topk, tile_maxsim_exact

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _reference(Q, pids, offsets, lens, emb):
    Qd = Q.double().cpu()
    offs, ln, E = offsets.cpu(), lens.cpu(), emb.double().cpu()
    out = np.empty(pids.shape, np.float64)
    for b in range(pids.shape[0]):
        for j, pid in enumerate(pids[b].tolist()):
            if pid < 0 or pid >= ln.shape[0]:
                out[b, j] = -np.inf
                continue
            L = int(ln[pid])
            if L <= 0:
                out[b, j] = -3.2e10
                continue
            d = E[int(offs[pid]):int(offs[pid]) + L]
            out[b, j] = float((Qd[b] @ d.T).max(dim=1).values.sum())
    return out


@pytest.fixture(scope="module")
def workload():
    centres, _ = synth.make_centroids(num_centres=1024, subs=1, seed=0, device="cuda")
    nq, per_q = 8, 1000
    docs = synth.make_exact_docs(nq * per_q, centres, len_range=(20, 180), seed=0, device="cuda")
    Q = synth.make_queries(centres, nq, seed=7).reshape(nq, 32, 128).contiguous()
    pids = torch.arange(nq * per_q, dtype=torch.int32, device="cuda").view(nq, per_q).contiguous()
    return Q, pids, docs


def test_exact_maxsim_matches_fp64(workload):
    Q, pids, docs = workload
    got = tile_maxsim_exact(Q, pids, docs["doc_offsets"], docs["doclens"], docs["emb"]).cpu().numpy()
    ref = _reference(Q, pids.cpu(), docs["doc_offsets"], docs["doclens"], docs["emb"])
    assert np.isfinite(got).all()
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)
    assert rel.max() < REL_TOL, rel.max()


def test_exact_maxsim_top10(workload):
    Q, pids, docs = workload
    got = tile_maxsim_exact(Q, pids, docs["doc_offsets"], docs["doclens"], docs["emb"])
    ids, _ = final_topk(pids, got, 10)
    ref = _reference(Q, pids.cpu(), docs["doc_offsets"], docs["doclens"], docs["emb"])
    for b in range(pids.shape[0]):
        order = sorted(range(ref.shape[1]), key=lambda j: (-ref[b, j], int(pids[b, j])))
        sep = ref[b, order[9]] - ref[b, order[10]]
        if sep > 2 * REL_TOL * abs(ref[b, order[9]]):
            assert ids[b].tolist() == [int(pids[b, j]) for j in order[:10]]


def test_exact_maxsim_edge_cases(workload):
    Q, pids, docs = workload
    lens = docs["doclens"].clone()
    lens[3] = 0                                  # empty passage
    p = torch.tensor([[3, -1, lens.shape[0] + 5, 7]], dtype=torch.int32, device="cuda")
    got = tile_maxsim_exact(Q[:1], p, docs["doc_offsets"], lens, docs["emb"]).cpu().numpy()[0]
    ref = _reference(Q[:1], p.cpu(), docs["doc_offsets"], lens, docs["emb"])[0]
    assert got[0] == np.float32(-3.2e10) and np.isneginf(got[1]) and np.isneginf(got[2])
    assert abs(got[3] - ref[3]) <= REL_TOL * max(abs(ref[3]), 1.0)
