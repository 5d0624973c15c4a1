"""Zero-sync batches: the whole batched search (Stages 2-4 + final top-k) is captured in one CUDA
graph and replayed on new queries written into the captured input buffer; results equal the
eager calls.  (Workspace growth happens on the eager warm-up call, outside the capture.)"""
import pytest
import torch

from tests.helpers import small_corpus, weft_index

pytestmark = pytest.mark.gpu


def test_search_captured_in_cuda_graph_matches_eager():
    d, Q, E, _ = small_corpus()
    wix = weft_index(d, E)
    Qa = Q[:4].cuda().contiguous()
    Qb = Q[2:6].cuda().contiguous()
    nc, K, k_top = 16, 300, 10
    ids_a, sc_a = wix.search(Qa, nc=nc, K=K, k_top=k_top)      # eager (also sizes the workspace)
    ids_b, sc_b = wix.search(Qb, nc=nc, K=K, k_top=k_top)
    torch.cuda.synchronize()

    q_in = Qa.clone()
    ids = torch.empty(4, k_top, dtype=torch.int32, device="cuda")
    sc = torch.empty(4, k_top, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        wix.search(q_in, nc=nc, K=K, k_top=k_top, out=(ids, sc))   # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        wix.search(q_in, nc=nc, K=K, k_top=k_top, out=(ids, sc))
    for Qx, ref_ids, ref_sc in ((Qa, ids_a, sc_a), (Qb, ids_b, sc_b)):
        q_in.copy_(Qx)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids) and torch.equal(sc, ref_sc)
    del g
