"""The sharded configuration's data shape on one GPU: a corpus whose topic popularity is
Zipf(1.1) (a few centroids' posting lists hold a large share of the postings, split into many
65,535-capped chunks; here the chunk cap is lowered so lists span dozens of chunks), searched
whole and as three doc-range shards merged by (score desc, pid asc) -- what bench.py does over
NCCL.  Both are checked against the CPU restatement (oracle/), the sharded one per shard and
merged the same way.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from ragrt_b200 import index_build, shard, synth
from tests.helpers import oracle_index, to_cuda, BIND_KEYS

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _bind(d, ix, sh, cents, corp):
    out = dict(d)
    out.update({"csr_row_ptrs": ix["csr_row_ptrs"], "csr_col_eids": ix["csr_col_eids"],
                "csr_block_sums": ix["csr_block_sums"], "csr_lengths": ix["csr_lengths"],
                "csr_packed_24": ix["csr_packed_24"], "doc_offsets": sh["doc_offsets"], "doc_lens": sh["doclens"],
                "codes": sh["codes"], "residuals": sh["residuals"], "doc_predicates": sh["preds"]})
    return out


@pytest.fixture(scope="module")
def zipf_corpus():
    centres, cents = synth.make_centroids(num_centres=256, subs=64, seed=3)
    corp = synth.make_corpus(30_000, centres, cents, seed=3, len_range=(20, 120), topic_zipf=1.1)
    preds = synth.make_predicates(30_000, seed=1)
    Q = synth.make_queries(centres, 6, seed=77, topic_zipf=1.1)
    base = {"centroids": cents, "bucket_weights": corp["bucket_weights"],
            "reversed_bit_map": corp["reversed_bit_map"], "decomp_table": corp["decomp_table"]}
    return centres, cents, corp, preds, Q, base


def _index(corp, preds, cents, base, lo, hi, max_len):
    sh = shard.slice_docs(corp["doc_offsets"], corp["doclens"], corp["codes"], corp["residuals"], preds, lo, hi)
    ix = index_build.plain_ivf_index(sh["codes"], sh["doclens"], cents.shape[0], max_len=max_len)
    d = _bind(base, ix, sh, cents, corp)
    return d, ix["E"], sh["pid_base"]


def _weft(d, E):
    from ragrt_b200.weft import WeftIndex
    g = to_cuda(d)
    return WeftIndex(*[g[k] for k in BIND_KEYS], num_passages=g["doc_lens"].shape[0],
                     num_centroids=g["centroids"].shape[0], E=E)


def _merge(parts, k_top):
    """parts: list of (ids [B, k], scores [B, k], pid_base) -> merged (ids, scores) by (score desc, pid asc)."""
    B = parts[0][0].shape[0]
    ids = np.full((B, k_top), -1, np.int64)
    sc = np.full((B, k_top), -np.inf, np.float32)
    for b in range(B):
        items = [(float(s[b, j]), int(i[b, j]) + base) for i, s, base in parts for j in range(i.shape[1])
                 if i[b, j] >= 0]
        items.sort(key=lambda t: (-t[0], t[1]))
        for j, (s_, p_) in enumerate(items[:k_top]):
            ids[b, j], sc[b, j] = p_, s_
    return ids, sc


def _check(ids, sc, oids, osc, score_of):
    for b in range(ids.shape[0]):
        fin = np.isfinite(osc[b])
        rel = np.abs(sc[b][fin] - osc[b][fin]) / np.maximum(np.abs(osc[b][fin]), 1.0)
        assert rel.max(initial=0) < REL_TOL
        for i in np.flatnonzero(ids[b] != oids[b]):          # ties within tolerance only
            assert abs(score_of(b, int(ids[b][i])) - osc[b][i]) <= 2 * REL_TOL * max(abs(osc[b][i]), 1.0)


def test_zipf_corpus_many_chunks_matches_oracle(zipf_corpus):
    centres, cents, corp, preds, Q, base = zipf_corpus
    N = corp["doclens"].shape[0]
    d, E, _ = _index(corp, preds, cents, base, 0, N, max_len=128)
    assert E > 16                                   # lists really are split into many chunks
    wix, oix = _weft(d, E), oracle_index(d)
    B = Q.shape[0]
    ntok = torch.full((B,), 32, dtype=torch.int32)
    masks = torch.tensor([0, 1, 2, 4, 0, 0], dtype=torch.int32)
    nc, K, k_top = 32, 1000, 10
    ids, sc = wix.search(Q.cuda(), nc=nc, K=K, k_top=k_top, ntok=ntok.cuda(), masks=masks.cuda())
    oids, osc, _ = O.weft_search(oix, Q.numpy(), ntok.numpy(), nc, E, masks.numpy(), K, k_top)
    _check(ids.cpu().numpy(), sc.cpu().numpy(), oids, osc,
           lambda b, pid: O.tile_maxsim(oix, Q[b].numpy(), np.array([pid], np.int32))[0])


def test_three_shards_merged_match_oracle_shards(zipf_corpus):
    centres, cents, corp, preds, Q, base = zipf_corpus
    N = corp["doclens"].shape[0]
    B = Q.shape[0]
    ntok = np.full(B, 32, np.int32)
    nc, K, k_top = 32, 400, 10
    ours, ref, oixs = [], [], []
    for r in range(3):
        lo, hi = shard.shard_range(N, r, 3)
        d, E, pb = _index(corp, preds, cents, base, lo, hi, max_len=65535)
        wix, oix = _weft(d, E), oracle_index(d)
        i, s = wix.search(Q.cuda(), nc=nc, K=K, k_top=k_top)
        ours.append((i.cpu().numpy(), s.cpu().numpy(), pb))
        oi, os_, _ = O.weft_search(oix, Q.numpy(), ntok, nc, E, None, K, k_top)
        ref.append((oi, os_, pb))
        oixs.append((oix, lo, hi))
    ids, sc = _merge(ours, k_top)
    oids, osc = _merge(ref, k_top)

    def score_of(b, pid):
        for oix, lo, hi in oixs:
            if lo <= pid < hi:
                return O.tile_maxsim(oix, Q[b].numpy(), np.array([pid - lo], np.int32))[0]
        raise AssertionError(pid)
    _check(ids, sc, oids, osc, score_of)


@pytest.mark.parametrize("world", [2, 8, 32])
def test_stage2_on_query_slices_equals_whole_batch(zipf_corpus, world):
    """sharded_search scores each rank's query slice and all-gathers the probe lists: the
    concatenated slices must equal Stage 2 over the whole batch bit for bit (32 queries over
    2 ranks use the tensor-core kernel, over 32 ranks the CUDA-core one)."""
    from ragrt_b200.weft import centroid_topk
    centres, cents, corp, preds, Q, base = zipf_corpus
    Qb = synth.make_queries(centres, 32, seed=5, topic_zipf=1.1).reshape(32, 32, 128).cuda()
    C = cents.cuda()
    t_all, s_all, _, _ = centroid_topk(Qb, C, 16)
    parts_t, parts_s = [], []
    for r in range(world):
        lo, hi, per = shard.query_slice(32, world, r)
        t, s, _, _ = centroid_topk(Qb[lo:hi], C, 16)
        parts_t.append(t)
        parts_s.append(s)
    assert torch.equal(torch.cat(parts_t), t_all)
    assert torch.equal(torch.cat(parts_s), s_all)


def test_sharded_search_single_rank_equals_search(zipf_corpus):
    import socket
    import torch.distributed as dist
    centres, cents, corp, preds, Q, base = zipf_corpus
    N = corp["doclens"].shape[0]
    d, E, pb = _index(corp, preds, cents, base, 0, N, max_len=65535)
    wix = _weft(d, E)
    Qc = Q.reshape(-1, 32, 128).cuda()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    # ragged query lengths go through the sharded path as through WeftIndex.search
    ntok = torch.tensor([32 - 5 * (b % 4) for b in range(Qc.shape[0])], dtype=torch.int32, device="cuda")
    try:
        ids, sc = shard.sharded_search(wix, Qc, 1, 0, pb, nc=32, K=400, k_top=10)
        rids_nt, rsc_nt = shard.sharded_search(wix, Qc, 1, 0, pb, nc=32, K=400, k_top=10, ntok=ntok)
    finally:
        dist.destroy_process_group()
    rids, rsc = wix.search(Qc, nc=32, K=400, k_top=10)
    assert torch.equal(ids, rids.to(torch.int64)) and torch.equal(sc, rsc)
    nids, nsc = wix.search(Qc, nc=32, K=400, k_top=10, ntok=ntok)
    assert torch.equal(rids_nt, nids.to(torch.int64)) and torch.equal(rsc_nt, nsc)


@pytest.mark.parametrize("world,k,k_top,pid_hi", [(8, 10, 10, 5000), (3, 7, 12, 5000), (1, 10, 5, 5000),
                                                  (8, 10, 10, 1 << 27)])
def test_merge_kernel_orders_like_the_rule(world, k, k_top, pid_hi):
    """ragrt_merge_topk: (score desc, pid asc), padding (-1) after real pids of equal score --
    ties, -inf scores and padding included; global pids past 2^24 (8 shards of up to 2^24
    passages each) come back exactly."""
    from ragrt_b200 import _lib
    from ragrt_b200.weft import _ptr, _stream
    g = np.random.default_rng(world * 100 + k)
    B = 16
    sc = g.choice(np.array([0.5, 0.25, 1.0, -np.inf, 2.0], np.float32), size=(world, B, k))
    pid = g.integers(0, pid_hi, size=(world, B, k)).astype(np.int32)
    if pid_hi > (1 << 24):
        pid[:, :, 0] = (1 << 24) + 1 + 2 * np.arange(B)[None, :]      # odd: not representable in fp32
    pad = g.random((world, B, k)) < 0.2
    pid[pad], sc[pad] = -1, -np.inf
    gathered = torch.from_numpy(np.stack([sc.view(np.int32), pid], 1)).cuda()        # [world, 2, B, k] words
    ids = torch.empty(B, k_top, dtype=torch.int64, device="cuda")
    out = torch.empty(B, k_top, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().ragrt_merge_topk(_ptr(gathered), world, B, k, k_top, _ptr(ids), _ptr(out), _stream()))
    ids, out = ids.cpu().numpy(), out.cpu().numpy()
    for b in range(B):
        items = [(float(sc[r, b, j]), int(pid[r, b, j])) for r in range(world) for j in range(k)]
        items.sort(key=lambda t: (-t[0], t[1] if t[1] >= 0 else 1 << 40))
        assert ids[b].tolist() == [p for _, p in items[:k_top]]
        assert np.array_equal(out[b], np.array([s for s, _ in items[:k_top]], np.float32))
