"""
Drop-in for ``native_prep`` of the reference's ``src/weft_prep.py:32-47`` (Stage 0b of the
`weft` engine), computed by the sm_100a Stage-2 kernel of libragrt_b200.so.

  native_prep(Q, C, nc, impute=False, compact=False) -> (topc, scores, m)

Same signature and return triple: topc int32 [ntok, nc]; scores float32 [ntok, nc]
(compact) or [ntok, num_centroids]; m float32 [ntok] (the (nc+1)-th best score, when
imputing) or None.  Scores are fp16 dot products rounded once from the exact value and
ties are broken by the lower centroid id (the reference's torch.topk leaves both open).
Inputs must be fp16 CUDA tensors: the weft path scores in fp16 on the GPU and there is no
CPU path.

``imputed_passage_scores`` (the reference's test helper, weft_prep.py:70-72) is kept for
callers that use it.

Filter-aware probing (the `weft_oracle` / `weft_adapt` engines, weft_prep.py:75-170): the same
functions with the same arguments and results, their top-k on the Stage-2 kernel.  The per-
centroid inputs they need (postings passing a filter, all postings; a centroid with no passing
posting is "empty") come from ``WeftIndex.pass_counts(mask)`` / ``centroid_filter_counts``.
"""
import torch

from ragrt_b200 import weft as _W


def native_prep(Q, C, nc, impute=False, compact=False):
    if not (Q.is_cuda and C.is_cuda):
        raise RuntimeError("native_prep: the B200 path runs on CUDA tensors only")
    if Q.dtype != torch.float16 or C.dtype != torch.float16:
        raise RuntimeError("native_prep: the weft path scores in fp16; pass fp16 Q and C")
    if Q.dim() != 2 or C.dim() != 2 or Q.shape[1] != 128 or C.shape[1] != 128:
        raise RuntimeError("native_prep: Q [ntok, 128] and C [num_centroids, 128] expected")
    ntok, NC = Q.shape[0], C.shape[0]
    k = min(nc + (1 if impute else 0), NC)
    imputed = impute and k > nc
    tops, scs, ms, fulls = [], [], [], []
    for a in range(0, ntok, 32):                      # the kernel takes up to 32 rows per query
        t, s, m, f = _W.centroid_topk(Q[a:a + 32][None], C, nc, impute=impute, full=not compact)
        tops.append(t[0])
        scs.append(s[0])
        ms.append(m[0])
        if f is not None:
            fulls.append(f[0])
    topc = torch.cat(tops) if tops else torch.empty(0, min(nc, k), dtype=torch.int32, device=Q.device)
    m = torch.cat(ms) if ms else torch.empty(0, device=Q.device)
    if compact:
        scores = torch.cat(scs) if scs else torch.empty(0, min(nc, k), device=Q.device)
        return topc, scores.contiguous(), (m if imputed else None)
    full = torch.cat(fulls).float() if fulls else torch.empty(0, NC, device=Q.device)
    if imputed:
        return topc, (full - m[:, None]).contiguous(), m
    return topc, full.contiguous(), None


def imputed_passage_scores(best, found, m):
    """best/found [P, T] per passage and token, m [T] -> imputed sums (weft_prep.py:70-72)."""
    return torch.where(found, best, m[None, :]).sum(1)


# ---------------------------------------------------------------- filter-aware probing
def centroid_filter_counts(index, mask):
    """(pass_c int64 [NC], tot_c int64 [NC], empty bool [NC], n_ok) for a WeftIndex and a filter."""
    pass_c, tot_c = index.pass_counts(mask)
    empty = pass_c == 0
    return pass_c, tot_c, empty, int((~empty).sum())


def _topk_values(Q, C, k):
    """(vals float32 [ntok, k], idx int64 [ntok, k]): the k best fp16 scores (exact, ties to
    the lower id), unshifted."""
    topc, vals, _ = native_prep(Q, C, k, impute=False, compact=True)
    return vals, topc.long()


def compact_centroids(C, empty):
    """(C_ok [n_ok, d], ids int64 [n_ok]) -- the non-empty centroids (weft_prep.py:128-133);
    C itself and None when no centroid is empty."""
    if not bool(empty.any()):
        return C, None
    ids = (~empty).nonzero().squeeze(1)
    return C[ids].contiguous(), ids


def oracle_fast_prep(Q, C_ok, ids, nc):
    """Probe the nc nearest non-empty centroids, impute from the (nc+1)-th (weft_prep.py:136-144).
    Returns (topc int32 [ntok, nc'], compact shifted scores, raw score of the last probed)."""
    nc = min(nc, C_ok.shape[0] - 1)
    topc, scores, m = native_prep(Q, C_ok, nc, impute=True, compact=True)
    if ids is not None:
        topc = ids[topc.long()].to(torch.int32).contiguous()
    return topc, scores, scores[:, -1] + m


def oracle_prep(Q, C, nc, empty, n_ok):
    """Reference form of oracle_fast_prep (weft_prep.py:112-125); also returns depth = mean over
    tokens of how many centroids (empty or not) score >= the last probed one."""
    C_ok, ids = compact_centroids(C, empty)
    topc, scores, last = oracle_fast_prep(Q, C_ok, ids, min(nc, n_ok - 1))
    return topc, scores, unfiltered_depth(Q, C, last)


def unfiltered_depth(Q, C, last):
    """Mean over tokens of the number of centroids scoring >= `last` (weft_prep.py:147-149)."""
    _, full, _ = native_prep(Q, C, 1, impute=False, compact=False)
    return (full >= last.float()[:, None]).sum(1).float().mean()


def adaptive_probe(Q, C, nc, ncap, pass_c, tot_c, sel, q=1.0, slack=1.0, stats=None):
    """weft_adapt's probe depth under a filter (weft_prep.py:75-105), same arguments and result
    (topc int32 [ntok, nc'], compact shifted scores, nc')."""
    NC = C.shape[0]
    nc = min(nc, NC - 1)
    ncap = min(ncap, NC - 1)
    vals, idx = _topk_values(Q, C, nc + 1)
    target = sel * tot_c[idx[:, :nc]].sum(1)
    short = (pass_c[idx[:, :nc]].sum(1) < slack * target).float().mean()
    if float(short) <= 1.0 - q + 1e-9:
        nc2 = nc
    else:
        vals, idx = _topk_values(Q, C, ncap + 1)
        cum = pass_c[idx[:, :ncap]].cumsum(1)
        need = ((cum < target[:, None]).sum(1) + 1).clamp(nc, ncap).float()
        nc2 = int(torch.quantile(need, q).ceil()) if q < 1.0 else int(need.max())
        nc2 = max(nc, min(ncap, nc2))
    m = vals[:, nc2]
    if stats is not None:
        stats["last"] = vals[:, nc2 - 1]
    return idx[:, :nc2].to(torch.int32).contiguous(), (vals[:, :nc2] - m[:, None]).contiguous(), nc2
