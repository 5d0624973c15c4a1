"""
Doc-range sharding of the `weft` path over several GPUs (one process per GPU).

Each rank holds the passages [lo, hi) of the corpus (contiguous pid range) with its own
plain-IVF index over local pids, runs Stages 2-4 locally and produces its top-k as
(score, local pid).  `merge_topk` moves every rank's list with one all-gather and merges by
(score desc, global pid asc), the tie rule this build uses for every final selection (the
reference's torch::topk at src/optix_corr_torch_3d.cpp:603-606 leaves ties unspecified).  The
result equals running each shard alone and merging; because the
candidate budget applies per shard it is not the 1-GPU result over the union of shards.
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


def merge_topk(ids, scores, world, k_top, pid_base, group=None):
    """ids int32 [B, k] (local pids, -1 padding), scores f32 [B, k] (-inf padding) on this
    rank -> (global pids int64 [B, k_top], scores f32 [B, k_top]) merged over all ranks.
    Uses one all_gather_into_tensor (NCCL on GPUs, gloo on CPU)."""
    import torch.distributed as dist
    gpid = torch.where(ids >= 0, ids.to(torch.int64) + pid_base, torch.full_like(ids, -1, dtype=torch.int64))
    pack = torch.stack([scores.to(torch.float32), gpid.to(torch.float32)], 0)   # pids < 2^24: exact in fp32
    out = torch.empty(world * 2, *pack.shape[1:], dtype=pack.dtype, device=pack.device)
    dist.all_gather_into_tensor(out, pack, group=group)          # rank-major concatenation
    out = out.view(world, *pack.shape)
    B = ids.shape[0]
    sc = out[:, 0].permute(1, 0, 2).reshape(B, -1)
    pid = out[:, 1].permute(1, 0, 2).reshape(B, -1).to(torch.int64)
    key = torch.where(pid >= 0, pid, torch.full_like(pid, 1 << 40))
    order = torch.argsort(key, dim=1, stable=True)                       # pid asc ...
    sc, pid = torch.gather(sc, 1, order), torch.gather(pid, 1, order)
    order = torch.argsort(sc, dim=1, descending=True, stable=True)       # ... then score desc
    return torch.gather(pid, 1, order)[:, :k_top], torch.gather(sc, 1, order)[:, :k_top]
