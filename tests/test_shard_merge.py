"""Doc-range sharding on CPU with world_size-2 `gloo` ranks: every rank slices its shard of a
small corpus, runs the CPU restatement of the whole path (oracle) on it, and exchanges the
per-shard top-k with ragrt_b200.shard.gather_topk (the all-gather that merge_topk runs over
NCCL before its merge kernel).  Merged by the rule (score desc, global pid asc), the exchanged
lists must equal the single-process merge of both shards' results, on every rank.  The merge
kernel itself is checked against the same rule on the GPU (test_gpu_sharded.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ragrt_b200 import index_build, shard
from tests.helpers import small_corpus, oracle_index

WORLD = 2
K_TOP = 10


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard_search(rank, world):
    d, Q, E, _ = small_corpus()
    N = d["doc_lens"].shape[0]
    lo, hi = shard.shard_range(N, rank, world)
    sh = shard.slice_docs(d["doc_offsets"], d["doc_lens"], d["codes"], d["residuals"], d["doc_predicates"], lo, hi)
    ix = index_build.plain_ivf_index(sh["codes"], sh["doclens"], d["centroids"].shape[0])
    ds = dict(d)
    ds.update({"csr_row_ptrs": ix["csr_row_ptrs"], "csr_col_eids": ix["csr_col_eids"],
               "csr_block_sums": ix["csr_block_sums"], "csr_lengths": ix["csr_lengths"],
               "csr_packed_24": ix["csr_packed_24"], "doc_offsets": sh["doc_offsets"], "doc_lens": sh["doclens"],
               "codes": sh["codes"], "residuals": sh["residuals"], "doc_predicates": sh["preds"]})
    from oracle import oracle as O
    B = Q.shape[0]
    ntok = np.full(B, 32, np.int32)
    ids, sc, _ = O.weft_search(oracle_index(ds), Q.reshape(B, 32, 128).numpy(), ntok, 8, ix["E"], None,
                               200, K_TOP, nthreads=1)
    return ids, sc, lo


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids, sc, lo = _shard_search(rank, world)
        out = shard.gather_topk(torch.from_numpy(ids), torch.from_numpy(sc), world, lo)
        g_ids, g_sc = _merge_rule(out, world, ids.shape[0], K_TOP)
        q.put((rank, g_ids.numpy(), g_sc.numpy()))
    finally:
        dist.destroy_process_group()


def _merge_rule(gathered, world, B, k_top):
    """The merge rule applied to gather_topk's output int32 words [world * 2, B, k] (score bits,
    global pids) with torch sorts: score desc, then pid asc, padding (-1) after every real pid
    of equal score."""
    out = gathered.view(world, 2, B, -1)
    sc = out[:, 0].permute(1, 0, 2).reshape(B, -1).contiguous().view(torch.float32)
    pid = out[:, 1].permute(1, 0, 2).reshape(B, -1).to(torch.int64)
    key = torch.where(pid >= 0, pid, torch.full_like(pid, 1 << 40))
    order = torch.argsort(key, dim=1, stable=True)                       # pid asc ...
    sc, pid = torch.gather(sc, 1, order), torch.gather(pid, 1, order)
    order = torch.argsort(sc, dim=1, descending=True, stable=True)       # ... then score desc
    return torch.gather(pid, 1, order)[:, :k_top], torch.gather(sc, 1, order)[:, :k_top]


def _expected(world):
    per = [_shard_search(r, world) for r in range(world)]
    B = per[0][0].shape[0]
    out_ids = np.full((B, K_TOP), -1, np.int64)
    out_sc = np.full((B, K_TOP), -np.inf, np.float32)
    for b in range(B):
        items = []
        for ids, sc, lo in per:
            for j in range(ids.shape[1]):
                pid = int(ids[b, j])
                items.append((float(sc[b, j]), pid + lo if pid >= 0 else -1))
        items.sort(key=lambda t: (-t[0], t[1] if t[1] >= 0 else 1 << 40))
        for j, (s, p) in enumerate(items[:K_TOP]):
            out_sc[b, j], out_ids[b, j] = s, p
    return out_ids, out_sc


def test_merge_refuses_host_tensors():
    """No CPU path: merge_topk raises before it enters the collective."""
    ids = torch.zeros(2, K_TOP, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        shard.merge_topk(ids, torch.zeros(2, K_TOP), WORLD, K_TOP, 0)


def test_slice_docs_covers_corpus():
    d, _, _, _ = small_corpus()
    N = d["doc_lens"].shape[0]
    toks = 0
    for r in range(3):
        lo, hi = shard.shard_range(N, r, 3)
        sh = shard.slice_docs(d["doc_offsets"], d["doc_lens"], d["codes"], d["residuals"], d["doc_predicates"], lo, hi)
        assert int(sh["doc_offsets"][0]) == 0 and int(sh["doc_offsets"][-1]) == sh["codes"].shape[0]
        assert torch.equal(sh["codes"], d["codes"][int(d["doc_offsets"][lo]):int(d["doc_offsets"][hi])])
        toks += sh["codes"].shape[0]
    assert toks == d["codes"].shape[0]


def test_two_rank_gloo_merge_matches_single_process():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(WORLD):
        r, ids, sc = q.get(timeout=180)
        got[r] = (ids, sc)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    exp_ids, exp_sc = _expected(WORLD)
    for r in range(WORLD):
        np.testing.assert_array_equal(got[r][0], exp_ids)
        np.testing.assert_array_equal(got[r][1], exp_sc)
    # the merge really mixes both shards
    assert (exp_ids >= shard.shard_range(small_corpus()[0]["doc_lens"].shape[0], 1, WORLD)[0]).any()


def _probes(Q, C, nc):
    """Stage 2 of each query (the oracle): topc int32 [n, 32, nc], scores f32 [n, 32, nc]."""
    from oracle import oracle as O
    ts, ss = [], []
    for q in Q:
        t, s, _, _ = O.native_prep(q.numpy(), C, nc, impute=True)
        ts.append(torch.from_numpy(np.ascontiguousarray(t, dtype=np.int32)))
        ss.append(torch.from_numpy(np.ascontiguousarray(s, dtype=np.float32)))
    return torch.stack(ts), torch.stack(ss)


def _probe_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        d, Q, _, _ = small_corpus()
        Q = Q.reshape(-1, 32, 128)[:5]                   # 5 queries over 2 ranks: the last slice is padded
        C = d["centroids"].numpy()
        B = Q.shape[0]
        lo, hi, per = shard.query_slice(B, world, rank)
        t, s = _probes(Q[lo:hi], C, 8)
        pad = per - (hi - lo)
        if pad:
            t = torch.cat([t, torch.zeros(pad, *t.shape[1:], dtype=t.dtype)])
            s = torch.cat([s, torch.zeros(pad, *s.shape[1:], dtype=s.dtype)])
        gt, gs = shard.gather_probes(t, s, world, B)
        q.put((rank, gt.numpy(), gs.numpy()))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_probe_exchange_equals_whole_batch():
    """The Stage-2 split of sharded_search: each rank scores its query slice and gather_probes
    rebuilds the whole batch's probe lists on every rank, equal to scoring the whole batch."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_probe_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(WORLD):
        r, t, s = q.get(timeout=180)
        got[r] = (t, s)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    d, Q, _, _ = small_corpus()
    et, es = _probes(Q.reshape(-1, 32, 128)[:5], d["centroids"].numpy(), 8)
    for r in range(WORLD):
        np.testing.assert_array_equal(got[r][0], et.numpy())
        np.testing.assert_array_equal(got[r][1], es.numpy())


def test_query_slices_cover_batch():
    for B in (1, 5, 256, 257):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                lo, hi, per = shard.query_slice(B, world, r)
                assert 0 <= hi - lo <= per and per * world >= B
                seen.extend(range(lo, hi))
            assert seen == list(range(B))
