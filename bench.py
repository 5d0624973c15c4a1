#!/usr/bin/env python
"""
bench.py -- throughput of the B200 `weft` search path (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg3]

One step = one batch of queries through the whole path (Stage 2 centroid scoring +
top-nprobe, Stages 1-3 posting aggregation + candidate selection, Stage 4 fused
decompress + TileMaxSim, final top-k).  The default workload is BASELINE config 3:
2,000,000 synthetic passages (lengths U[60,180], mean 120), 65,536 fp16 centroids,
2-bit residuals, batch 256 x 32 query tokens, nprobe 32, 4,096 candidates, top-10.
Inputs are seeded synthetic data (ragrt_b200.synth) standing in for LoTTE / MS MARCO.

Prints ONE JSON line on rank 0.  `value` is queries/s with inputs resident in HBM; `e2e`
is the same through the public API with the query batch copied from pinned host memory
and the results copied back inside every timed step.  `stages` and `roofline` come from a
second timed pass that records CUDA events at the stage boundaries on the launching stream.

Multi-GPU (--gpus N under torchrun): the corpus is sharded by contiguous pid ranges.  Each
rank runs Stage 2 for its slice of the query batch and one NCCL all-gather gives every rank
the whole batch's probe lists; every rank then runs Stages 1-4 for the whole batch against its
shard (per-shard K = ceil(K / N)), and the per-shard top-k lists are merged with a second
all-gather (ragrt_b200.shard.sharded_search).  Whole-job work is fixed ("scaling": "strong").

--impl reference times the CPU restatement of the reference path (oracle/, all host
threads) on a bounded sample of the same workload, rank 0 only.
"""
import argparse
import datetime
import json
import math
import os
import shutil
import subprocess
import sys
import threading
import time
import warnings

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "queries/s at 1/2/4/8 B200 (weft, batch 256, top-10); Stage-4 doc-tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

CONFIGS = {
    "cfg3": dict(num_docs=2_000_000, len_range=(60, 180), centres=1024, subs=64, batch=256, nc=32, K=4096,
                 k_top=10, masks=None,
                 desc="full weft, 2M docs (len U[60,180], mean 120), 65,536 fp16 centroids, 2-bit residuals, "
                      "batch 256 x 32 tokens, nprobe 32, 4,096 candidates, top-10"),
    "cfg4": dict(num_docs=2_000_000, len_range=(60, 180), centres=1024, subs=64, batch=256, nc=32, K=4096,
                 k_top=10, masks=(1, 2, 4),
                 desc="cfg3 + predicate filters inside Stage 3 (bits with selectivity 1%, 10%, 50%; "
                      "queries cycle through the three masks)"),
    "cfg5": dict(num_docs=8_800_000, len_range=(20, 120), centres=4096, subs=64, batch=1024, nc=32, K=4096,
                 k_top=10, masks=None, zipf=1.1, k_per_shard=True,
                 desc="sharded weft: 8.8M docs (len U[20,120], mean 70), 262,144 fp16 centroids with Zipf(1.1) "
                      "topic popularity, batch 1,024 x 32 tokens, nprobe 32, 4,096 candidates per shard, top-10"),
    "small": dict(num_docs=200_000, len_range=(60, 180), centres=1024, subs=64, batch=256, nc=32, K=4096,
                  k_top=10, masks=None, desc="cfg3 at 1/10 of the corpus (quick runs)"),
}


# ----------------------------------------------------------------------------- helpers
def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_traffic():
    """Per-unit DRAM traffic of the dominant kernels from the committed ncu summaries."""
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "traffic.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {k: float(d[k]) for k in FALLBACK_PEAKS if k in d}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms, started before the warm-up so
    that it is running when the timed region begins; `summary` keeps the samples whose own
    nvidia-smi timestamp lies inside the window set by `mark_start` / `mark_end`."""
    Q = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = []
        self.t0 = self.t1 = None

    def mark_start(self):
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        self.t1 = datetime.datetime.now()

    def __enter__(self):
        try:
            # line-buffered (stdbuf) so that each sample reaches the reader when it is taken
            pre = ["stdbuf", "-oL"] if shutil.which("stdbuf") else []
            self.proc = subprocess.Popen(pre + ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes up to a second to start: wait for its first sample, so that the
            # (sub-second) timed region is sampled
            deadline = time.time() + 10.0
            while not self.out and self.proc.poll() is None and time.time() < deadline:
                time.sleep(0.01)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.out.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.2)                      # the samples of the region's last interval
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f")
                if self.t0 is not None and not (self.t0 <= ts <= (self.t1 or ts)):
                    continue
                sm.append(float(f[1]))
                smax = max(smax, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        window = (self.t1 - self.t0).total_seconds() if self.t0 and self.t1 else None
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax or None,
                "reasons": sorted(reasons), "samples": len(sm), "window_s": window,
                "interval_ms": 20}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    if world != n_gpus:
        log(f"note: --gpus {n_gpus} but WORLD_SIZE={world}; using {world}")
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- data
def build_workload(cfg, rank, world, seed=0):
    """Synthetic corpus (generated on the GPU) and this rank's shard of it."""
    from ragrt_b200 import synth, index_build
    t0 = time.time()
    dev = "cuda"
    centres, cents = synth.make_centroids(num_centres=cfg["centres"], subs=cfg["subs"], seed=seed, device=dev)
    corp = synth.make_corpus(cfg["num_docs"], centres, cents, len_range=cfg["len_range"], seed=seed, device=dev,
                             topic_zipf=cfg.get("zipf"))
    preds = synth.make_predicates(cfg["num_docs"], seed=1, device=dev)
    N = cfg["num_docs"]
    from ragrt_b200.shard import shard_range, slice_docs
    lo, hi = shard_range(N, rank, world)
    shard = slice_docs(corp["doc_offsets"], corp["doclens"], corp["codes"], corp["residuals"], preds, lo, hi)
    t_lo, t_hi = int(corp["doc_offsets"][lo]), int(corp["doc_offsets"][hi])
    del corp["codes"], corp["residuals"]
    torch.cuda.empty_cache()
    ix = index_build.plain_ivf_index(shard["codes"], shard["doclens"], cents.shape[0])
    log(f"[rank {rank}] corpus: {hi - lo:,} docs, {t_hi - t_lo:,} tokens, {ix['num_postings']:,} postings, "
        f"E={ix['E']} ({time.time() - t0:.1f} s)")
    return centres, cents, corp, shard, ix


def make_index(cents, corp, shard, ix):
    from ragrt_b200.weft import WeftIndex
    return WeftIndex(ix["csr_row_ptrs"], ix["csr_col_eids"], ix["csr_block_sums"], ix["csr_lengths"],
                     ix["csr_packed_24"], shard["doc_offsets"], shard["doclens"], shard["codes"], shard["residuals"],
                     cents, corp["bucket_weights"], corp["reversed_bit_map"], corp["decomp_table"],
                     doc_predicates=shard["preds"], num_passages=shard["doclens"].shape[0],
                     num_centroids=cents.shape[0], E=ix["E"])


# ----------------------------------------------------------------------------- reference arm (CPU)
def host_arrays(cents, corp, shard, ix):
    """Host (numpy) copies of the bound index arrays, with the bind_index names."""
    return {
        "csr_row_ptrs": ix["csr_row_ptrs"].cpu().numpy(), "csr_col_eids": ix["csr_col_eids"].cpu().numpy(),
        "csr_block_sums": ix["csr_block_sums"].cpu().numpy(),
        "csr_lengths": ix["csr_lengths"].cpu().view(torch.int16).numpy().view(np.uint16),
        "csr_packed_24": ix["csr_packed_24"].cpu().numpy(), "doc_offsets": shard["doc_offsets"].cpu().numpy(),
        "doc_lens": shard["doclens"].cpu().numpy(), "codes": shard["codes"].cpu().numpy(),
        "residuals": shard["residuals"].cpu().numpy(), "centroids": cents.cpu().numpy(),
        "bucket_weights": corp["bucket_weights"].cpu().numpy(),
        "reversed_bit_map": corp["reversed_bit_map"].cpu().numpy(), "decomp_table": corp["decomp_table"].cpu().numpy(),
        "doc_predicates": shard["preds"].cpu().to(torch.int64).numpy().astype(np.uint32),
    }


def torch_reference_step(host, cfg, Q, masks, sample, K, nthreads):
    """The reference's torch path for `sample` queries of a batch on the host cores; returns
    seconds.  Stage 2 is the reference's weft_prep.native_prep computation itself (fp16 Q @ C^T,
    topk(nc + 1), the (nc+1)-th score subtracted: src/weft_prep.py:32-47).  Stages 1-3 follow
    the reference test's centroid-interaction rule (tests/test_gpu_kernels.py:259-263: per token
    the max over its probed lists holding the passage, summed over tokens) with the kernels'
    fp16 base scores and base > 0 rule, scattered per token over the posting lists instead of a
    dense passage x centroid matrix, which a corpus of this size does not allow; top-K by a stable
    sort.  Stage 4 is the test's fp32 rerank (tests/test_gpu_kernels.py:294-305: fp16 decode,
    fp32 normalise, Q @ D^T, max over tokens, sum), over a query's candidates at once."""
    torch.set_num_threads(nthreads)
    nc, k_top = cfg["nc"], cfg["k_top"]
    C = torch.from_numpy(host["centroids"])
    lens = torch.from_numpy(host["csr_lengths"].astype(np.int64))
    list_off = torch.zeros(lens.numel() + 1, dtype=torch.int64)
    list_off[1:] = torch.cumsum(lens, 0)
    row0 = torch.from_numpy(host["csr_row_ptrs"][0])
    pk = host["csr_packed_24"].reshape(-1, 3).astype(np.int64)
    pids = torch.from_numpy(pk[:, 0] | (pk[:, 1] << 8) | (pk[:, 2] << 16))
    offs = torch.from_numpy(host["doc_offsets"])
    dl = torch.from_numpy(host["doc_lens"].astype(np.int64))
    codes = torch.from_numpy(host["codes"].astype(np.int64))
    res = torch.from_numpy(host["residuals"])
    bw = torch.from_numpy(host["bucket_weights"])
    buck = torch.from_numpy(host["decomp_table"].astype(np.int64))[torch.from_numpy(host["reversed_bit_map"].astype(np.int64))]
    preds = torch.from_numpy(host["doc_predicates"].astype(np.int64))
    N = dl.numel()
    Qc = Q[:sample].cpu()
    mk = masks[:sample].cpu().tolist() if masks is not None else [0] * sample
    t0 = time.time()
    for b in range(sample):
        q = Qc[b]
        s = q @ C.T                                              # native_prep, fp16
        vals, idx = s.topk(nc + 1, dim=-1)
        topc = idx[:, :nc]
        scores = vals[:, :nc].float() - vals[:, nc].float()[:, None]
        total = torch.zeros(N)
        touched = torch.zeros(N, dtype=torch.bool)
        for t in range(32):
            best = torch.zeros(N)
            for j in range(nc):
                base = float(scores[t, j])
                if not base > 0.0:                               # MIN_BASE_SCORE
                    continue
                c = int(topc[t, j])
                p = pids[list_off[row0[c]]:list_off[row0[c + 1]]]
                if mk[b]:
                    p = p[(preds[p] & mk[b]) != 0]
                v = float(torch.tensor(base).half())             # fp16 base score
                best[p] = torch.maximum(best[p], torch.tensor(v))
                touched[p] = True
            total += best
        cand = torch.nonzero(touched).flatten()
        if cand.numel() > K:
            order = torch.sort(-total[cand], stable=True).indices[:K]   # score desc, pid asc
            cand = cand[order]
        # Stage 4: fp16 decode, fp32 normalise, max over tokens, sum over rows
        cl = dl[cand]
        tok = torch.repeat_interleave(offs[cand], cl) + (torch.arange(int(cl.sum())) -
                                                        torch.repeat_interleave(torch.cumsum(cl, 0) - cl, cl))
        D = (C[codes[tok]] + bw[buck[res[tok].long()].view(-1, 128)]).float()
        D = D / D.norm(dim=1, keepdim=True)
        S = (q.float() @ D.T).T                                  # [tokens, 32]
        seg = torch.repeat_interleave(torch.arange(cand.numel()), cl)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")                      # index_reduce_ is marked beta
            mx = torch.full((cand.numel(), 32), -float("inf")).index_reduce_(0, seg, S, "amax")
        f = mx.sum(1)
        if mk[b]:
            f[(preds[cand] & mk[b]) == 0] = -float("inf")
        order = torch.sort(-f, stable=True).indices[:k_top]
        _ = cand[order]
    return time.time() - t0


def host_oracle_index(cents, corp, shard, ix):
    """Host copy of the bound index for the CPU restatement (oracle/)."""
    from oracle import oracle as O
    return O.Index(host_arrays(cents, corp, shard, ix))


def oracle_step(oix, cfg, E, Q, masks, sample, nthreads, K=None):
    """The CPU restatement on `sample` queries of a batch; returns (seconds, ids, scores)."""
    from oracle import oracle as O
    q = Q[:sample].cpu().numpy()
    mk = masks[:sample].cpu().numpy().astype(np.uint32) if masks is not None else None
    t0 = time.time()
    ids, sc, _ = O.weft_search(oix, q, np.full(sample, 32, np.int32), cfg["nc"], int(E), mk,
                               min(K or cfg["K"], oix.N), cfg["k_top"], nthreads=nthreads)
    return time.time() - t0, ids, sc


def parity_check(wix, oix, cfg, E, Q, masks, K, sample, oids, osc, nthreads):
    """Our results for the first `sample` queries of batch Q against the oracle's, stage by
    stage: Stage-2 probes and scores bit-exact, Stage-3 candidate lists (pids, order and fp32
    sums) bit-exact, final top-k ids equal except at Stage-4 score ties within 1e-3 (the
    oracle's own top-k, oids / osc, comes from the timed CPU leg on the same queries)."""
    from oracle import oracle as O
    nc, k_top = cfg["nc"], cfg["k_top"]
    topc, s2, _, _ = wix.centroid_topk(Q, nc)
    cp, cs, _ = wix.candidates(topc, s2, K, masks=masks)
    ids, sc = wix.search(Q, nc=nc, K=K, k_top=k_top, masks=masks)
    topc, s2 = topc[:sample].cpu().numpy(), s2[:sample].cpu().numpy()
    cp, cs = cp[:sample].cpu().numpy(), cs[:sample].cpu().numpy()
    ids, sc = ids[:sample].cpu().numpy(), sc[:sample].cpu().numpy()
    q = Q[:sample].cpu().numpy()
    mk = masks[:sample].cpu().numpy().astype(np.uint32) if masks is not None else np.zeros(sample, np.uint32)
    otopc, os2, _ = O.native_prep_batch(q, np.full(sample, 32, np.int32), wix.centroids.cpu().numpy(), nc,
                                        nthreads=nthreads)
    s2_ok = bool(np.array_equal(topc, otopc) and np.array_equal(s2.view(np.uint32), os2.view(np.uint32)))
    s3_ok = True
    for b in range(sample):
        op, osum, _ = O.candidates(oix, otopc[b], os2[b], int(E), int(mk[b]), K)
        s3_ok &= bool(np.array_equal(cp[b], op) and np.array_equal(cs[b].view(np.uint32), osum.view(np.uint32)))
    a = O.topk_agreement(oix, q, ids, sc, oids, osc, masks=mk, rel_tol=1e-3)
    return {"queries": sample, "s2_exact": s2_ok, "s3_exact": s3_ok,
            "top10_ids_equal": a["mismatches"] == 0, "top10_positions_equal": a["equal"],
            "top10_score_ties": a["ties"], "top10_mismatches": a["mismatches"],
            "max_rel_score_err": a["max_rel_score_err"],
            "rule": "Stage 2/3 bit-exact; top-k ids equal except at Stage-4 score ties within 1e-3 relative"}


def run_reference(args, cfg, rank, world):
    if rank != 0:
        return 0
    nthreads = os.cpu_count() or 1
    centres, cents, corp, shard, ix = build_workload(cfg, 0, 1)
    Qall = make_queries(centres, cfg, args.warmup + args.steps, 0)
    sample = max(1, min(cfg["batch"], args.cpu_sample or nthreads))
    masks = make_masks(cfg, sample)
    oix = host_oracle_index(cents, corp, shard, ix)
    for i in range(args.warmup):
        oracle_step(oix, cfg, ix["E"], Qall[i], masks, sample, nthreads)
    times = [oracle_step(oix, cfg, ix["E"], Qall[i], masks, sample, nthreads)[0]
             for i in range(args.warmup, args.warmup + args.steps)]
    tot = sum(times)
    v = sample * len(times) / tot
    line = {"metric": METRIC, "value": v, "unit": "queries/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * tot / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16 in, exact/f64 (CPU)",
            "data": "synthetic", "config": {"workload": f"{args.config}: {cfg['desc']}",
                                           "sample_per_step": f"{sample} queries of a 256-query batch"},
            "cpu_baseline": {"value": v, "unit": "queries/s", "cores": nthreads, "kind": "port",
                             "sample": f"{sample} queries per step through all stages (oracle/weft_oracle.c, "
                                       f"OpenMP over queries)"},
            "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def make_queries(centres, cfg, nbatches, seed):
    from ragrt_b200 import synth
    Q = synth.make_queries(centres, nbatches * cfg["batch"], seed=1000 + seed, topic_zipf=cfg.get("zipf"))
    return Q.view(nbatches, cfg["batch"], 32, 128)


def make_masks(cfg, B):
    if not cfg["masks"]:
        return None
    m = torch.tensor([cfg["masks"][i % len(cfg["masks"])] for i in range(B)], dtype=torch.int32, device="cuda")
    return m


# ----------------------------------------------------------------------------- ours
def sharded_search(*a, **kw):
    """Stage 2 by query slice + probe all-gather, Stages 1-4 on the doc shard, merged top-k."""
    from ragrt_b200.shard import sharded_search as ss
    return ss(*a, **kw)


def run_ours(args, cfg, rank, world, local):
    from ragrt_b200 import _lib
    centres, cents, corp, shard, ix = build_workload(cfg, rank, world)
    wix = make_index(cents, corp, shard, ix)
    nb = args.warmup + args.steps
    Q = make_queries(centres, cfg, nb, 0)
    B, nc, k_top = cfg["batch"], cfg["nc"], cfg["k_top"]
    K = min(cfg["K"] if cfg.get("k_per_shard") else int(math.ceil(cfg["K"] / world)), wix.N)
    masks = make_masks(cfg, B)
    ids = torch.empty(nb, B, k_top, dtype=torch.int32, device="cuda")
    sc = torch.empty(nb, B, k_top, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()

    # events at the stage boundaries of every timed step, on the launching stream
    nev = 5 if world == 1 else 7
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(nb)]

    def step(i):
        if world == 1:
            wix.search_profiled(Q[i], ev[i], nc=nc, K=K, k_top=k_top, masks=masks, out=(ids[i], sc[i]))
        else:                # Stage 2 split over the ranks by query, the rest on this rank's doc shard
            sharded_search(wix, Q[i], world, rank, shard["pid_base"], nc=nc, K=K, k_top=k_top, masks=masks,
                           events=ev[i])

    # ---- warm-up, then the timed region (inputs resident in HBM, a new query batch per step)
    with ClockSampler(local) as clocks:
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        barrier(world)
        wix.stats(reset=True)
        l0 = _lib.lib().ragrt_launch_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        barrier(world)
        clocks.mark_start()
        e0.record(stream)
        for i in range(args.warmup, nb):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
        clocks.mark_end()
        barrier(world)
    launches = _lib.lib().ragrt_launch_count() - l0
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    value = B * args.steps / (ms / 1000.0)

    # ---- end to end through the public API: pinned host queries in, results out, every step
    Qh = Q.cpu().pin_memory()
    Qd = torch.empty_like(Q[0])
    ids_h = torch.empty(nb, B, k_top, dtype=torch.int32).pin_memory()
    sc_h = torch.empty(nb, B, k_top, dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    barrier(world)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for i in range(args.warmup, nb):
        Qd.copy_(Qh[i], non_blocking=True)
        if world == 1:
            o_ids, o_sc = wix.search(Qd, nc=nc, K=K, k_top=k_top, masks=masks)
        else:
            o_ids, o_sc = sharded_search(wix, Qd, world, rank, shard["pid_base"], nc=nc, K=K, k_top=k_top,
                                         masks=masks)
        ids_h[i].copy_(o_ids.to(torch.int32), non_blocking=True)
        sc_h[i].copy_(o_sc, non_blocking=True)
    e3.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(e2.elapsed_time(e3), world)
    e2e = B * args.steps / (ms_e2e / 1000.0)

    # ---- stage breakdown of the timed steps (events recorded inside the timed region)
    # per rank, mean over the timed steps; then the max over ranks of every interval
    stage_ms = np.array([[ev[i][s].elapsed_time(ev[i][s + 1]) for s in range(nev - 1)]
                         for i in range(args.warmup, nb)]).mean(0)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor(stage_ms, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        stage_ms = t.cpu().numpy()
        # 0 Stage 2 (this rank's query slice), 1 probe all-gather, 2 Stages 1-3, 3 Stage 4,
        # 4 local top-k, 5 top-k all-gather + merge
        idx = {"s2": 0, "s3": 2, "s4": 3, "topk": 4}
    else:
        idx = {"s2": 0, "s3": 1, "s4": 2, "topk": 3}
    # Stage-4 algorithmic work per launch: candidates and their doc tokens, averaged over the
    # timed batches (recomputed after the timed region)
    # (the distinct-postings statistic needs an extra kernel, so it is counted here, outside the
    # timed region, over the same batches)
    cand_tokens = n_cand = 0
    wix.count_distinct(True)
    wix.stats(reset=True)
    for i in range(args.warmup, nb):
        topc, s2sc, _, _ = wix.centroid_topk(Q[i], nc)
        cp, _, _ = wix.candidates(topc, s2sc, K, masks=masks)
        valid = cp >= 0
        cand_tokens += int(wix.doc_lens[cp[valid].long()].sum())
        n_cand += int(valid.sum())
    cand_tokens //= args.steps
    n_cand //= args.steps
    st2 = stats = wix.stats()
    wix.count_distinct(False)
    peaks, peak_kind = load_peaks()
    s2_flops = 2.0 * -(-B // world) * 32 * wix.NC * 128       # this rank's query slice
    s3_bytes = (3.0 * st2["distinct_postings"] + 8.0 * st2["touched"]) / args.steps
    s4_bytes = 36.0 * cand_tokens + 16.0 * n_cand
    stages = {
        "s2_centroid_topk": {"ms": stage_ms[idx["s2"]], "achieved": s2_flops / (stage_ms[idx["s2"]] / 1e3) / 1e12,
                             "unit": "TFLOP/s", "peak": peaks["bf16_tflops"], "bound": "tensor",
                             "work": f"{s2_flops / 1e9:.1f} GFLOP/step"},
        "s3_aggregate": {"ms": stage_ms[idx["s3"]], "achieved": s3_bytes / (stage_ms[idx["s3"]] / 1e3) / 1e9,
                         "unit": "GB/s",
                         "peak": peaks["hbm_gbs"], "bound": "hbm",
                         "work": f"{s3_bytes / 1e6:.1f} MB/step (3 B x distinct postings + 8 B x touched)",
                         "algorithmic": s3_bytes / 1e9},
        "s4_maxsim": {"ms": stage_ms[idx["s4"]], "achieved": s4_bytes / (stage_ms[idx["s4"]] / 1e3) / 1e9,
                      "unit": "GB/s",
                      "peak": peaks["hbm_gbs"], "bound": "hbm",
                      "work": f"{s4_bytes / 1e6:.1f} MB/step (36 B x {cand_tokens:,} doc tokens + 16 B x cand)",
                      "doc_tokens_per_s": cand_tokens / (stage_ms[idx["s4"]] / 1e3), "algorithmic": s4_bytes / 1e9},
        "final_topk": {"ms": stage_ms[idx["topk"]]},
    }
    if world > 1:
        pb = 8.0 * B * 32 * nc                     # (centroid id, score) words of the whole batch
        stages["probe_allgather"] = {"ms": stage_ms[1], "bytes_gathered": pb,
                                     "gbs_per_rank": pb * (world - 1) / world / (stage_ms[1] / 1e3) / 1e9}
        stages["topk_allgather_merge"] = {"ms": stage_ms[5], "bytes_gathered": 8.0 * world * B * k_top}
    limiter = max(stages, key=lambda k: stages[k]["ms"])
    for s in stages.values():
        if "achieved" in s:
            s["frac"] = s["achieved"] / s["peak"]
    dom = max(("s2_centroid_topk", "s3_aggregate", "s4_maxsim"), key=lambda k: stages[k]["ms"])
    d = stages[dom]
    traffic = None
    tr = load_traffic().get(dom) or {}
    if "dram_bytes_per_doc_token" in tr:                                   # Stage 4: one launch per step
        traffic = tr["dram_bytes_per_doc_token"] * cand_tokens / 1e9
    elif "dram_bytes_per_algorithmic_byte" in tr and d.get("algorithmic"):
        traffic = tr["dram_bytes_per_algorithmic_byte"] * d["algorithmic"]
    roofline = {"bound": d["bound"], "achieved": d["achieved"], "peak": d["peak"], "unit": d["unit"],
                "frac": d["frac"], "traffic": traffic, "traffic_unit": "GB per step (ncu DRAM bytes per unit of work, scaled)" if traffic else None,
                "algorithmic": d.get("algorithmic"), "kernel": dom, "peak_source": peak_kind,
                "timing": "CUDA events at stage boundaries inside the timed region, mean over steps"}

    cpu = parity = cpu_torch = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        nthreads = os.cpu_count() or 1
        sample = max(1, min(B, args.cpu_sample or nthreads))
        oix = host_oracle_index(cents, corp, shard, ix)
        dt, oids, osc = oracle_step(oix, cfg, ix["E"], Q[args.warmup], masks, sample, nthreads, K=K)
        cpu = {"value": sample / dt, "unit": "queries/s", "cores": nthreads, "kind": "port",
               "sample": f"{sample} queries of one batch through all stages ({dt:.1f} s; oracle/weft_oracle.c, "
                         f"OpenMP over queries)"}
        # parity of the benchmarked configuration: the same queries through our path
        parity = parity_check(wix, oix, cfg, ix["E"], Q[args.warmup], masks, K, sample, oids, osc, nthreads)
        ts = max(1, args.torch_sample)
        dtt = torch_reference_step(host_arrays(cents, corp, shard, ix), cfg, Q[args.warmup], masks, ts, K, nthreads)
        cpu_torch = {"value": ts / dtt, "unit": "queries/s", "cores": nthreads, "kind": "reference-torch",
                     "sample": f"{ts} queries of one batch ({dtt:.1f} s): the reference's native_prep (fp16 "
                               f"matmul + topk) and its tests' Stage-3 / Stage-4 formulas in torch on the host"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"{args.config}: {cfg['desc']}", "batch": B, "nprobe": nc,
                       "candidates_per_shard": K, "top_k": k_top, "docs": cfg["num_docs"],
                       "parallelism": f"doc-sharded x{world}, Stage 2 split by query" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (index ~9 GB) and a distinct query batch per step"},
            "e2e": {"value": e2e, "unit": "queries/s", "h2d_bytes_per_step": int(Q[0].numel() * 2),
                    "d2h_bytes_per_step": int(B * k_top * 8)},
            "roofline": roofline,
            "stages": {k: {kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                       for k, v in stages.items()},
            "stage4_doc_tokens_per_s": stages["s4_maxsim"]["doc_tokens_per_s"],
            "limiter": {"stage": limiter, "ms": stages[limiter]["ms"],
                        "note": "per-rank stage times, mean over the timed steps, max over ranks"},
            "cpu_baseline": cpu,
            "cpu_baseline_torch": cpu_torch,
            "parity": parity,
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
            "counters": {k: int(v) for k, v in stats.items()},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg3")
    ap.add_argument("--cpu-sample", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--torch-sample", type=int, default=4, help="queries of the torch CPU reference leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    cfg = CONFIGS[args.config]
    rank, world, local = dist_setup(args.gpus)
    if args.impl == "reference":
        return run_reference(args, cfg, rank, world)
    return run_ours(args, cfg, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
