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


def _ranked(Q, C, k):
    """Each token's k best centroids, best first (ties to the lower id), and their fp16 scores
    as fp32, unshifted: (ids int32 [ntok, k], scores f32 [ntok, k])."""
    ids, sc, _ = native_prep(Q, C, k, impute=False, compact=True)
    return ids, sc


def compact_centroids(C, empty):
    """The centroids a filter leaves non-empty, once per filter (weft_prep.py:128-133):
    (C_ok [n_ok, d], their ids int64 [n_ok]); when none is empty, C itself and None."""
    keep = torch.nonzero(~empty).flatten()
    if keep.numel() == C.shape[0]:
        return C, None
    return C.index_select(0, keep).contiguous(), keep


def oracle_fast_prep(Q, C_ok, ids, nc):
    """weft_oracle's probes (weft_prep.py:136-144): each token's nc nearest non-empty centroids,
    scores shifted by the (nc+1)-th.  Returns (topc int32 [ntok, nc'] as ids of the full centroid
    set, shifted scores f32 [ntok, nc'], raw score of each token's last probed centroid)."""
    depth = min(nc, C_ok.shape[0] - 1)
    probes, raw = _ranked(Q, C_ok, depth + 1)
    shifted = raw[:, :depth] - raw[:, depth:depth + 1]
    if ids is not None:
        probes = ids.index_select(0, probes.reshape(-1).long()).view(probes.shape).to(torch.int32)
    return probes[:, :depth].contiguous(), shifted.contiguous(), raw[:, depth - 1]


def oracle_prep(Q, C, nc, empty, n_ok):
    """weft_oracle's probes with its diagnostic depth (weft_prep.py:112-125): also returns the
    mean over tokens of how many centroids, empty or not, score at least the last probed one."""
    C_ok, ids = compact_centroids(C, empty)
    topc, scores, last = oracle_fast_prep(Q, C_ok, ids, min(nc, n_ok - 1))
    return topc, scores, unfiltered_depth(Q, C, last)


def unfiltered_depth(Q, C, last):
    """Mean over tokens of the number of centroids scoring >= `last` (weft_prep.py:147-149),
    from the fp16 score matrix of the Stage-2 kernel."""
    _, full, _ = native_prep(Q, C, 1, impute=False, compact=False)
    return (full >= last.float()[:, None]).sum(1).float().mean()


def _depths(probes, pass_c, tot_c, sel, nc, ncap, slack):
    """ragrt_probe_depth on a token x probe list: (short int32 [ntok], need int32 [ntok])."""
    from ragrt_b200._lib import lib, check
    from ragrt_b200.weft import _ptr, _stream
    probes = probes.to(torch.int32).contiguous()
    ntok, width = probes.shape
    pc = pass_c.to(device=probes.device, dtype=torch.int64).contiguous()
    tc = tot_c.to(device=probes.device, dtype=torch.int64).contiguous()
    short = torch.empty(ntok, dtype=torch.int32, device=probes.device)
    need = torch.empty(ntok, dtype=torch.int32, device=probes.device)
    check(lib().ragrt_probe_depth(_ptr(probes), ntok, width, _ptr(pc), _ptr(tc), pc.shape[0], float(sel),
                                  float(slack), nc, ncap, _ptr(short), _ptr(need), _stream()))
    return short, need


def adaptive_probe(Q, C, nc, ncap, pass_c, tot_c, sel, q=1.0, slack=1.0, stats=None):
    """weft_adapt's probe depth under a filter (weft_prep.py:75-105); same arguments and result:
    (topc int32 [ntok, d], compact scores shifted by the (d+1)-th f32 [ntok, d], d).

    The depth d is nc unless more than a (1 - q) share of the tokens is short (their first nc
    probes hold fewer than slack x the target passing postings, ragrt_probe_depth); then every
    token's need is measured on its first ncap probes and d is their q-quantile (q = 1: the
    largest), within [nc, ncap]."""
    NC = C.shape[0]
    nc, ncap = min(nc, NC - 1), min(ncap, NC - 1)
    probes, raw = _ranked(Q, C, nc + 1)
    short, _ = _depths(probes, pass_c, tot_c, sel, nc, nc, slack)
    depth = nc
    if float(short.float().mean()) > 1.0 - q + 1e-9:
        probes, raw = _ranked(Q, C, ncap + 1)
        _, need = _depths(probes, pass_c, tot_c, sel, nc, ncap, slack)
        need = need.float()
        d = int(need.max()) if q >= 1.0 else int(torch.quantile(need, q).ceil())
        depth = max(nc, min(ncap, d))
    if stats is not None:
        stats["last"] = raw[:, depth - 1]
    shifted = raw[:, :depth] - raw[:, depth:depth + 1]
    return probes[:, :depth].contiguous(), shifted.contiguous(), depth
