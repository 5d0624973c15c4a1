"""Zero-sync batches: the whole batched search (Stages 2-4 + final top-k) is captured in one CUDA
graph and replayed on new queries written into the captured input buffer.  The replay equals the
eager calls bit for bit, unfiltered and with per-query filters (the reference defines its graph
path as equal to eager with or without a filter, graph_search.py:113-126), and matches the CPU
oracle under the parity rule (ids equal except at Stage-4 score ties within 1e-3).  Workspace
growth happens on the eager warm-up call, outside the capture."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import small_corpus, oracle_index, weft_index

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


@pytest.mark.parametrize("filtered", [False, True])
def test_search_captured_in_cuda_graph_matches_eager_and_oracle(filtered):
    d, Q, E, _ = small_corpus()
    wix = weft_index(d, E)
    oix = oracle_index(d)
    Qa = Q[:4].cuda().contiguous()
    Qb = Q[2:6].cuda().contiguous()
    nc, K, k_top = 16, 300, 10
    masks = torch.tensor([1, 2, 4, 0], dtype=torch.int32, device="cuda") if filtered else None
    ids_a, sc_a = wix.search(Qa, nc=nc, K=K, k_top=k_top, masks=masks)      # eager (also sizes the workspace)
    ids_b, sc_b = wix.search(Qb, nc=nc, K=K, k_top=k_top, masks=masks)
    torch.cuda.synchronize()

    q_in = Qa.clone()
    ids = torch.empty(4, k_top, dtype=torch.int32, device="cuda")
    sc = torch.empty(4, k_top, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        wix.search(q_in, nc=nc, K=K, k_top=k_top, masks=masks, out=(ids, sc))   # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        wix.search(q_in, nc=nc, K=K, k_top=k_top, masks=masks, out=(ids, sc))
    mk = masks.cpu().numpy().astype(np.uint32) if filtered else None
    for Qx, ref_ids, ref_sc in ((Qa, ids_a, sc_a), (Qb, ids_b, sc_b)):
        q_in.copy_(Qx)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids) and torch.equal(sc, ref_sc)
        q = Qx.cpu().numpy()
        oids, osc, _ = O.weft_search(oix, q, np.full(4, 32, np.int32), nc, E, mk, K, k_top)
        a = O.topk_agreement(oix, q, ids.cpu().numpy(), sc.cpu().numpy(), oids, osc, masks=mk, rel_tol=REL_TOL)
        assert a["mismatches"] == 0 and a["max_rel_score_err"] < REL_TOL, a
    del g
