"""
Doc-range sharding of the `weft` path over several GPUs (one process per GPU).

Each rank holds the passages [lo, hi) of the corpus (contiguous pid range) with its own
plain-IVF index over local pids, runs Stages 2-4 locally and produces its top-k as
(score, local pid).  `merge_topk` moves every rank's list with one all-gather (`gather_topk`)
and merges them on the GPU by (score desc, global pid asc), the tie rule this build uses for
every final selection (the reference's torch::topk at src/optix_corr_torch_3d.cpp:603-606
leaves ties unspecified).  The result equals running each shard alone and merging; because
the candidate budget applies per shard it is not the 1-GPU result over the union of shards.

Stage 2 (query tokens x centroids) does not depend on the shard, so `sharded_search` does not
repeat it on every rank: rank r scores its slice of the query batch and `gather_probes` gives
every rank the whole batch's probe lists with one all-gather.  Stage 2 is exact and each query's
result is independent of the rest of the batch, so this equals every rank running Stage 2 on
the whole batch.
"""
import torch


def shard_range(num_docs, rank, world):
    """[lo, hi) pids of `rank` when `num_docs` passages are split into `world` ranges."""
    return (num_docs * rank) // world, (num_docs * (rank + 1)) // world


def slice_docs(doc_offsets, doclens, codes, residuals, preds, lo, hi):
    """The passages [lo, hi) as a self-contained shard (local pids 0..hi-lo-1)."""
    t_lo, t_hi = int(doc_offsets[lo]), int(doc_offsets[hi])
    return {
        "doclens": doclens[lo:hi].contiguous(),
        "doc_offsets": (doc_offsets[lo:hi + 1] - t_lo).contiguous(),
        "codes": codes[t_lo:t_hi].contiguous(),
        "residuals": residuals[t_lo:t_hi].contiguous(),
        "preds": preds[lo:hi].contiguous() if preds is not None else None,
        "pid_base": lo,
    }


def gather_topk(ids, scores, world, pid_base, group=None):
    """ids int32 [B, k] (local pids, -1 padding), scores f32 [B, k] (-inf padding) on this rank
    -> every rank's list, rank-major, as int32 words [world * 2, B, k]: the scores' f32 bit
    patterns, then the global pids (-1 padding), with one all_gather_into_tensor.  The pids
    travel as integers, so every pid below 2^31 arrives exactly."""
    import torch.distributed as dist
    gpid = torch.where(ids >= 0, ids.to(torch.int64) + pid_base, torch.full_like(ids, -1, dtype=torch.int64))
    if pid_base + (1 << 24) >= 2 ** 31:
        raise RuntimeError("global pids must stay below 2^31")
    pack = torch.stack([scores.to(torch.float32).contiguous().view(torch.int32), gpid.to(torch.int32)], 0)
    out = torch.empty(world * 2, *pack.shape[1:], dtype=torch.int32, device=pack.device)
    dist.all_gather_into_tensor(out, pack.contiguous(), group=group)
    return out


def merge_topk(ids, scores, world, k_top, pid_base, group=None):
    """ids int32 [B, k] (local pids, -1 padding), scores f32 [B, k] (-inf padding) on this
    rank's GPU -> (global pids int64 [B, k_top], scores f32 [B, k_top]) merged over all ranks
    by (score desc, pid asc): gather_topk, then one ragrt_merge_topk kernel."""
    if not (ids.is_cuda and scores.is_cuda):
        raise RuntimeError("ragrt_b200 runs on CUDA tensors only (there is no CPU path)")
    from . import _lib
    from .weft import _ptr, _stream
    out = gather_topk(ids, scores, world, pid_base, group=group)
    B, k = ids.shape
    o_ids = torch.empty(B, k_top, dtype=torch.int64, device=out.device)
    o_sc = torch.empty(B, k_top, dtype=torch.float32, device=out.device)
    _lib.check(_lib.lib().ragrt_merge_topk(_ptr(out), world, B, k, k_top, _ptr(o_ids), _ptr(o_sc), _stream()))
    return o_ids, o_sc


def query_slice(B, world, rank):
    """Rank `rank`'s slice [lo, hi) of a B-query batch for Stage 2, and the padded slice size."""
    per = -(-B // world)
    return min(B, rank * per), min(B, (rank + 1) * per), per


def gather_probes(topc, scores, world, B, group=None):
    """This rank's Stage-2 output for its query slice (topc int32 [per, rows, kc], scores f32
    [per, rows, kc], rows past the batch padded) -> the whole batch's (topc [B, rows, kc],
    scores [B, rows, kc]) on every rank, with one all_gather_into_tensor."""
    import torch.distributed as dist
    pack = torch.stack([topc.to(torch.int32), scores.to(torch.float32).view(torch.int32)], 0)
    out = torch.empty(world * 2, *topc.shape, dtype=torch.int32, device=topc.device)
    dist.all_gather_into_tensor(out, pack.contiguous(), group=group)     # rank-major concatenation
    out = out.view(world, 2, *topc.shape)
    t = out[:, 0].reshape(-1, *topc.shape[1:])[:B].contiguous()
    s = out[:, 1].reshape(-1, *topc.shape[1:])[:B].contiguous().view(torch.float32)
    return t, s


def sharded_search(wix, Q, world, rank, pid_base, nc=32, K=4096, k_top=10, ntok=None, masks=None, events=None,
                   group=None):
    """The `weft` search of a query batch Q [B, 32, 128] fp16 over a corpus split by doc range:
    Stage 2 on this rank's query slice, probe lists all-gathered, Stages 1-4 and the top-k on
    this rank's shard `wix` (local pids + pid_base), then the merge over ranks.  `ntok` (int32
    [B], optional) limits the query tokens of Stages 2-3 as in WeftIndex.search; Stage 4 scores
    all 32 rows of Q, as the single-GPU search does.  Returns (global pids int64 [B, k_top],
    scores f32 [B, k_top]), the same on every rank.  `events`: optional 7 torch.cuda.Event
    recorded before Stage 2, after Stage 2, after the probe all-gather, after Stages 1-3, after
    Stage 4, after the local top-k and after the top-k all-gather and merge."""
    def mark(i):
        if events is not None:
            events[i].record()
    B = Q.shape[0]
    lo, hi, per = query_slice(B, world, rank)
    nts = None
    if hi - lo == per:
        Qs = Q[lo:hi]
        if ntok is not None:
            nts = ntok[lo:hi]
    else:                                        # the last slice of a batch that world does not divide
        Qs = Q.new_zeros(per, *Q.shape[1:])
        Qs[:hi - lo] = Q[lo:hi]
        if ntok is not None:                     # padding queries: full length, results dropped
            nts = torch.full((per,), 32, dtype=ntok.dtype, device=ntok.device)
            nts[:hi - lo] = ntok[lo:hi]
    mark(0)
    topc, sc, _, _ = wix.centroid_topk(Qs, nc, ntok=nts)
    mark(1)
    topc, sc = gather_probes(topc, sc, world, B, group=group)
    mark(2)
    pids, _, _ = wix.candidates(topc, sc, K, ntok=ntok, masks=masks)
    mark(3)
    f = wix.tile_maxsim(Q, pids)
    mark(4)
    ids, s = wix.final_topk(pids, f, k_top, masks=masks)
    mark(5)
    out = merge_topk(ids, s, world, k_top, pid_base, group=group)
    mark(6)
    return out
