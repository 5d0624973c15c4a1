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
