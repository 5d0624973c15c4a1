"""
The CUDA path against the REFERENCE's own CUDA kernels (ragrt_fused_kernel.cu and
tile_maxsim_fused_decomp.cu built unmodified by oracle/build_ref.sh into oracle/_ref),
driven in `weft` configuration on the same device buffers.  Also pins the CPU oracle to
the reference implementation.

Expected agreement:
  * touched passage sets: identical;
  * per-passage sums: the reference adds fp32 maxima in CUB's order, the oracle exactly ->
    equal within 32 fp32 ulps;
  * candidates (U > K): identical up to ties at the K-th sum (torch.topk has no tie rule);
  * Stage 4: the reference's wmma kernel vs ours within 1e-3 relative.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import small_corpus, oracle_index, weft_index

pytestmark = pytest.mark.gpu

REF = O.ref_lib()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref/libragrt_ref.so not built (oracle/build_ref.sh)")


@pytest.fixture(scope="module")
def corpus():
    d, Q, E, _ = small_corpus()
    return d, Q, E, oracle_index(d), weft_index(d, E)


def _p(t):
    return C.c_void_p(t.data_ptr())


def _ref_candidates(wix, E, topc, sc, mask, K):
    ntok, kc = topc.shape
    max_hits = 256
    dev = "cuda"
    qp = torch.zeros(ntok * 32 * 3, device=dev)
    cw = torch.zeros(32 * E * 3, device=dev)
    oc = torch.full((ntok * 32 * max_hits,), -1, dtype=torch.int32, device=dev)
    ov = torch.zeros(ntok * 32 * max_hits, device=dev)
    on = torch.zeros(ntok * 32, dtype=torch.int32, device=dev)
    topc, sc = topc.cuda().contiguous(), sc.cuda().contiguous()
    pp, ps, U = C.c_void_p(), C.c_void_p(), C.c_longlong()
    preds = wix.preds if wix.preds is not None else torch.zeros(wix.N, dtype=torch.int32, device=dev)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = REF.ref_weft_candidates(_p(qp), _p(cw), ntok, E, max_hits, _p(oc), _p(ov), _p(on), _p(topc), _p(sc), kc, E,
                                wix.NC, _p(wix.row_ptrs), _p(wix.col_eids), wix.eid_bytes, _p(wix.block_sums),
                                _p(wix.lengths), _p(wix.packed), wix.N, _p(preds), mask, K, C.byref(pp), C.byref(ps),
                                C.byref(U), stream)
    torch.cuda.synchronize()
    pids = torch.empty(L, dtype=torch.int32, device=dev)
    sums = torch.empty(L, dtype=torch.float32, device=dev)
    assert REF.ref_copy_d2d(_p(pids), pp, 4 * L) == 0
    assert REF.ref_copy_d2d(_p(sums), ps, 4 * L) == 0
    return pids.cpu().numpy(), sums.cpu().numpy(), int(U.value), L


@needs_ref
@pytest.mark.parametrize("K,mask", [(3000, 0), (200, 0), (200, 2)])
def test_candidates_vs_reference_kernels(corpus, K, mask):
    d, Q, E, oix, wix = corpus
    nc = 16
    for b in range(3):
        ntok = 32 - 4 * b
        t, s, _, _ = O.native_prep(Q[b, :ntok].numpy(), d["centroids"].numpy(), nc, impute=True)
        rp, rs, U, L = _ref_candidates(wix, E, torch.from_numpy(t), torch.from_numpy(s), mask, K)
        real = rp >= 0
        op, os_, st = O.candidates(oix, t, s, E, mask, wix.N)          # every touched passage
        oreal = op >= 0
        our = dict(zip(op[oreal].tolist(), os_[oreal].tolist()))
        assert st["touched"] == U - (1 if (rp[:U] < 0).any() else 0) or st["touched"] == U
        ref_all = dict(zip(rp[real].tolist(), rs[real].tolist()))
        if L == K and U <= K:
            assert set(ref_all) == set(our), "touched sets differ from the reference"
        for pid, v in ref_all.items():
            assert pid in our
            assert abs(v - our[pid]) <= 32 * np.spacing(np.float32(max(abs(v), 1e-30))), (pid, v, our[pid])
        # candidate selection: ours vs torch.topk on the reference's sums (ties at the cut excepted)
        cp, cs, _ = wix.candidates(torch.from_numpy(t[None]).cuda(), torch.from_numpy(s[None]).cuda(), K,
                                   masks=torch.tensor([mask], dtype=torch.int32).cuda())
        cp = cp[0].cpu().numpy()
        if L > K:
            top = torch.topk(torch.from_numpy(rs), K)
            ref_sel = set(rp[top.indices.numpy()].tolist()) - {-1}
            cut = float(top.values[-1])
            ours_sel = set(cp[cp >= 0].tolist())
            for pid in ours_sel ^ ref_sel:
                assert abs(our[pid] - cut) <= 32 * np.spacing(np.float32(cut)), "selection differs beyond ties"
        else:
            assert np.array_equal(cp[cp >= 0], np.sort(rp[real]))


@needs_ref
def test_tile_maxsim_vs_reference_wmma(corpus):
    d, Q, E, oix, wix = corpus
    g = torch.Generator().manual_seed(5)
    pids = torch.randint(0, wix.N, (600,), generator=g).to(torch.int32).cuda()
    pids[::41] = -1
    Qc = Q[0].cuda().contiguous()
    ref = torch.empty(600, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    REF.ref_tile_maxsim(_p(Qc), _p(pids), _p(wix.doc_offsets), _p(wix.doc_lens), 600, _p(wix.codes),
                        _p(wix.residuals), _p(wix.centroids), _p(wix.bucket_weights), _p(wix.rbm), _p(wix.decomp),
                        _p(ref), 1, stream)
    ours = wix.tile_maxsim(Qc, pids, mode=1)
    torch.cuda.synchronize()
    ref, ours = ref.cpu().numpy(), ours.cpu().numpy()
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(ours), fin)
    assert (np.abs(ours[fin] - ref[fin]) / np.maximum(np.abs(ref[fin]), 1.0)).max() < 1e-3
