"""The allocation-free Stage-2 entry point (ragrt_centroid_topk_noalloc) against the
allocating one (ragrt_centroid_topk), both called through the C ABI.

Stage 2 is exact (fp16 scores are the exact dot products rounded once; ties go to the
lower centroid id), so the tolerance here is the one every Stage-2 test uses: bit-identical
ids, scores and imputation values.  Two calls in a row with different inputs show that the
shared static scratch carries nothing from one call into the next.  Collected last so it
also runs after every other test in the same process.
"""
import ctypes as C

import pytest
import torch

from ragrt_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def _call(fn_name, Q, ntok, C_, nc, impute):
    B, rows, _ = Q.shape
    NC = C_.shape[0]
    kk = min(nc + (1 if impute else 0), NC)
    ncol = min(nc, kk)
    topc = torch.full((B, rows, ncol), -7, dtype=torch.int32, device=Q.device)
    scores = torch.full((B, rows, ncol), 7.0, dtype=torch.float32, device=Q.device)
    m = torch.full((B, rows), 7.0, dtype=torch.float32, device=Q.device)
    L = _lib.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [_p(Q), _p(ntok), B, rows, _p(C_), NC, nc, int(impute), _p(topc), _p(scores), _p(m)]
    if fn_name == "ragrt_centroid_topk":
        args.append(C.c_void_p(0))            # no full score matrix
    rc = getattr(L, fn_name)(*args, stream)
    torch.cuda.synchronize()
    return rc, topc, scores, m


def _inputs(B, NC, seed, ragged):
    centres, Cm = synth.make_centroids(num_centres=max(1, NC // 64), subs=64, seed=seed, device="cuda")
    Q = synth.make_queries(centres, B, seed=seed + 1).reshape(B, 32, 128).contiguous()
    g = torch.Generator().manual_seed(seed)
    ntok = torch.randint(1, 33, (B,), generator=g, dtype=torch.int32).cuda() if ragged else None
    return Q, ntok, Cm[:NC].contiguous()


def _same(a, b):
    rc_a, ta, sa, ma = a
    rc_b, tb, sb, mb = b
    assert rc_a == 0 and rc_b == 0, _lib.lib().ragrt_last_error()
    assert torch.equal(ta, tb)
    assert torch.equal(sa, sb)
    assert torch.equal(ma, mb)


def test_noalloc_matches_allocating_entry_point_twice():
    L = _lib.lib()
    cases = [
        # (B, NC, nc, impute, ragged, seed): two tensor-core calls in a row, then the SIMT path
        (16, 8192, 32, True, False, 11),
        (8, 4096, 16, True, True, 23),
        (4, 2048, 64, True, True, 37),     # kk = 65 > 64: SIMT kernel
    ]
    for B, NC, nc, impute, ragged, seed in cases:
        Q, ntok, Cm = _inputs(B, NC, seed, ragged)
        ref = _call("ragrt_centroid_topk", Q, ntok, Cm, nc, impute)
        got = _call("ragrt_centroid_topk_noalloc", Q, ntok, Cm, nc, impute)
        _same(ref, got)
        if ragged:
            # rows past ntok carry the documented padding
            t = torch.arange(32, device="cuda")[None, :] >= ntok[:, None]
            assert bool((got[1][t] == -1).all()) and bool((got[2][t] == 0).all())
    assert L.ragrt_centroid_topk_noalloc_error(1) == 0


def test_noalloc_slice_layouts_in_a_row():
    """The tensor-core path lays its per-row lists out by slice count, which follows the batch
    size: 4 queries (one 128-row block) split 8,192 centroids into 32 slices, 320 queries (80
    row blocks on 148 SMs) use a single slice.  Calls with the two layouts back to back, each
    against the allocating entry point bit for bit, show that no region of the shared array
    carries a previous layout's contents into the next call."""
    cases = [(4, 8192, 32, True, True, 41), (320, 8192, 32, True, True, 43), (4, 8192, 32, True, False, 47)]
    for B, NC, nc, impute, ragged, seed in cases:
        Q, ntok, Cm = _inputs(B, NC, seed, ragged)
        ref = _call("ragrt_centroid_topk", Q, ntok, Cm, nc, impute)
        got = _call("ragrt_centroid_topk_noalloc", Q, ntok, Cm, nc, impute)
        _same(ref, got)
    assert _lib.lib().ragrt_centroid_topk_noalloc_error(1) == 0


def test_noalloc_rejects_oversized_scratch():
    L = _lib.lib()
    Q, _, Cm = _inputs(4, 2048, 5, False)
    topc = torch.empty(1, dtype=torch.int32, device="cuda")
    sc = torch.empty(1, dtype=torch.float32, device="cuda")
    # 100,000 queries x 32 rows needs far more than 32 MiB of per-row lists: rejected
    # before anything is launched (the small buffers are never touched)
    rc = L.ragrt_centroid_topk_noalloc(_p(Q), C.c_void_p(0), 100_000, 32, _p(Cm), Cm.shape[0], 32, 1,
                                       _p(topc), _p(sc), C.c_void_p(0),
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert _lib.ERR_NAMES.get(rc) == "RAGRT_ERR_ARG"
    assert b"static maximum" in L.ragrt_last_error()
    torch.cuda.synchronize()
