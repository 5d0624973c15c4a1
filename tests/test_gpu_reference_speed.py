"""
Speed against the reference's own GPU path on the same B200 and the same inputs (cfg3 shape:
2 M synthetic passages, 65,536 centroids, nprobe 32 with imputation, 4,096 candidates).

  * Stage 2: the reference's native_prep semantics (src/weft_prep.py:32-47) run as torch ops on
    the GPU -- an fp16 cuBLAS GEMM and torch.topk -- one query at a time as Engines.ragrt_prep
    calls it (src/engines.py:421), against our batched tensor-core kernel.
  * Stages 1-3: the reference's kernels (all-codewords Stage 1, ragrt_stage2, CUB-sorted
    ragrt_stage3_sparse; oracle/_ref, built unmodified from its sources) per query, against
    our batched Stage 3.
  * Stage 4: the reference's wmma kernel (tile_maxsim_fused_decomp.cu) per query, against
    our tcgen05 kernel on the same candidates.
The test fails if a stage of ours is slower than the reference's; it prints one JSON line with
the per-query times (run with -s to see it).
"""
import ctypes as C
import json

import pytest
import torch

from oracle import oracle as O
from ragrt_b200 import index_build, synth
from ragrt_b200.weft import WeftIndex, centroid_topk

pytestmark = pytest.mark.gpu

REF = O.ref_lib()
NQ = 16           # queries timed on the reference's per-query path


def _p(t):
    return C.c_void_p(t.data_ptr())


def _ms(fn, reps=3, rounds=3):
    """Mean time of `reps` calls after a warm-up, the best of `rounds` rounds (the same for the
    reference and for ours), so that one disturbance on a shared GPU does not decide the test."""
    fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(rounds):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) / reps)
    return best


def _ref_native_prep(q, C16, nc):
    # restatement of weft_prep.native_prep(Q, C, nc, impute=True, compact=True) in torch
    s = q @ C16.t()
    vals, idx = s.topk(nc + 1, dim=1)
    m = vals[:, nc].float()
    return idx[:, :nc].to(torch.int32), vals[:, :nc].float() - m[:, None]


@pytest.mark.skipif(REF is None, reason="oracle/_ref/libragrt_ref.so not built (oracle/build_ref.sh)")
def test_stages_not_slower_than_reference_kernels():
    dev = "cuda"
    centres, Cm = synth.make_centroids(num_centres=1024, subs=64, seed=0, device=dev)
    corp = synth.make_corpus(2_000_000, centres, Cm, seed=0, device=dev)
    ix = index_build.plain_ivf_index(corp["codes"], corp["doclens"], Cm.shape[0])
    wix = WeftIndex(ix["csr_row_ptrs"], ix["csr_col_eids"], ix["csr_block_sums"], ix["csr_lengths"],
                    ix["csr_packed_24"], corp["doc_offsets"], corp["doclens"], corp["codes"], corp["residuals"], Cm,
                    corp["bucket_weights"], corp["reversed_bit_map"], corp["decomp_table"], E=ix["E"])
    B, nc, K, E = 256, 32, 4096, ix["E"]
    Q = synth.make_queries(centres, B, seed=1000).reshape(B, 32, 128).contiguous()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    # ---- Stage 2
    ref_s2 = _ms(lambda: [_ref_native_prep(Q[i], Cm, nc) for i in range(NQ)]) / NQ
    our_s2 = _ms(lambda: centroid_topk(Q, Cm, nc)) / B

    # ---- Stages 1-3 (reference buffers are reused between its calls)
    topc, sc, _, _ = centroid_topk(Q, Cm, nc)
    max_hits = 256
    qp = torch.zeros(32 * 32 * 3, device=dev)
    cw = torch.zeros(32 * E * 3, device=dev)
    oc = torch.full((32 * 32 * max_hits,), -1, dtype=torch.int32, device=dev)
    ov = torch.zeros(32 * 32 * max_hits, device=dev)
    on = torch.zeros(32 * 32, dtype=torch.int32, device=dev)
    preds = torch.zeros(wix.N, dtype=torch.int32, device=dev)
    pp, ps, U = C.c_void_p(), C.c_void_p(), C.c_longlong()
    tq = [topc[i].contiguous() for i in range(NQ)]
    sq = [sc[i].contiguous() for i in range(NQ)]

    def ref_s3():
        for i in range(NQ):
            REF.ref_weft_candidates(_p(qp), _p(cw), 32, E, max_hits, _p(oc), _p(ov), _p(on), _p(tq[i]), _p(sq[i]),
                                    nc, E, wix.NC, _p(wix.row_ptrs), _p(wix.col_eids), wix.eid_bytes,
                                    _p(wix.block_sums), _p(wix.lengths), _p(wix.packed), wix.N, _p(preds), 0, K,
                                    C.byref(pp), C.byref(ps), C.byref(U), stream)
    ref_s3_ms = _ms(ref_s3) / NQ
    our_s3_ms = _ms(lambda: wix.candidates(topc, sc, K)) / B

    # ---- Stage 4 on our candidates
    cand, _, _ = wix.candidates(topc, sc, K)
    out = torch.empty(K, device=dev)
    cq = [cand[i].contiguous() for i in range(NQ)]

    def ref_s4():
        for i in range(NQ):
            REF.ref_tile_maxsim(_p(Q[i]), _p(cq[i]), _p(wix.doc_offsets), _p(wix.doc_lens), K, _p(wix.codes),
                                _p(wix.residuals), _p(wix.centroids), _p(wix.bucket_weights), _p(wix.rbm),
                                _p(wix.decomp), _p(out), 1, stream)
    ref_s4_ms = _ms(ref_s4) / NQ
    our_s4_ms = _ms(lambda: wix.tile_maxsim(Q, cand, mode=1)) / B

    line = {"per_query_ms": {"s2": {"reference": ref_s2, "ours": our_s2},
                             "s1_s3": {"reference": ref_s3_ms, "ours": our_s3_ms},
                             "s4": {"reference": ref_s4_ms, "ours": our_s4_ms}},
            "speedup": {"s2": ref_s2 / our_s2, "s1_s3": ref_s3_ms / our_s3_ms, "s4": ref_s4_ms / our_s4_ms},
            "config": "cfg3 shape: 2M passages, 65,536 centroids, nprobe 32, K 4,096; reference per query "
                      f"({NQ} queries), ours batched (256 queries)"}
    print(json.dumps(line))
    assert our_s2 < ref_s2 and our_s3_ms < ref_s3_ms and our_s4_ms < ref_s4_ms, line
