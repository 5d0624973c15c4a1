"""
Per-stage benchmark of the `weft` kernels on seeded synthetic data (one GPU).

    python -m ragrt_b200.stagebench --stage s2|s3|s4|all [--docs N] [--batch B] [--steps K]

  s2   Stage 2 alone: B x 32 query tokens against 65,536 fp16 centroids, top-(nc+1).
  s3   Stages 1-3 alone on Stage-2 output (posting aggregation + candidate selection).
  s4   Stage 4 alone: 4,096 candidates per query drawn uniformly
       without replacement from the corpus (seeded per query), fused 2-bit decompression
       + TileMaxSim, batch B.
  exact  exact TileMaxSim on uncompressed fp16 passages: 64 queries x
       1,000 candidates each, 20-180 tokens per candidate.
Prints one JSON line per stage with the mean time per step (CUDA events on the launching
stream, after warm-up) and the stage's algorithmic work.  Also the program that the ncu
captures in profiles/ run.
"""
import argparse
import json
import sys
import time

import torch

from . import synth, index_build
from .weft import WeftIndex, centroid_topk, tile_maxsim_exact


def timed(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def random_bert_weights(seed=0, layers=12, D=768, F_=3072, heads=12, vocab=30522, dim=128):
    """BERT-base shaped fp16 weights in the layout of encoder.flat_weights (random: there is no
    checkpoint offline; the speed does not depend on the values)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *sh: (torch.randn(*sh, generator=g, device="cuda") * 0.02).half()
    ln = lambda: (torch.ones(D, device="cuda").half(), torch.zeros(D, device="cuda").half())
    W = {"emb_word": r(vocab, D), "emb_pos": r(512, D), "emb_type": r(D), "emb_ln": ln(), "heads": heads,
         "eps": 1e-12, "act": "gelu", "linear": r(dim, D), "layers": []}
    for _ in range(layers):
        W["layers"].append({"qkv_w": r(3 * D, D), "qkv_b": r(3 * D), "o_w": r(D, D), "o_b": r(D), "ln1": ln(),
                            "i_w": r(F_, D), "i_b": r(F_), "f_w": r(D, F_), "f_b": r(D), "ln2": ln()})
    return W


def torch_forward(W, ids, mask):
    """The same network with torch operations (cuBLAS fp16 GEMMs, PyTorch's fused attention,
    LayerNorm, GELU): the computation of the reference's torch encoder, timed beside ours."""
    import torch.nn.functional as F
    B, L = ids.shape
    H = W["heads"]
    x = W["emb_word"][ids] + W["emb_pos"][:L][None] + W["emb_type"]
    D = x.shape[-1]
    x = F.layer_norm(x, (D,), *W["emb_ln"], eps=W["eps"])
    bias = (1.0 - mask[:, None, None, :].to(x.dtype)) * torch.finfo(x.dtype).min
    for lw in W["layers"]:
        qkv = F.linear(x, lw["qkv_w"], lw["qkv_b"]).view(B, L, 3, H, D // H).permute(2, 0, 3, 1, 4)
        c = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], attn_mask=bias).transpose(1, 2).reshape(B, L, D)
        x = F.layer_norm(x + F.linear(c, lw["o_w"], lw["o_b"]), (D,), *lw["ln1"], eps=W["eps"])
        h = F.gelu(F.linear(x, lw["i_w"], lw["i_b"]))
        x = F.layer_norm(x + F.linear(h, lw["f_w"], lw["f_b"]), (D,), *lw["ln2"], eps=W["eps"])
    return F.normalize(F.linear(x, W["linear"]).float(), p=2, dim=-1).half()


def _graphed(fn, *args):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.no_grad():
        for _ in range(2):
            fn(*args)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g), torch.no_grad():
        fn(*args)
    return g


def encode_stage(B, steps, warmup):
    """Stage 0a: B queries x 32 tokens through BERT-base + ColBERT's linear, as one CUDA graph
    of this build's kernels, and the same network in torch (cuBLAS + SDPA) as one graph."""
    from .encoder import flat_forward
    W = random_bert_weights()
    g = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.randint(1000, 30000, (B, 32), generator=g, device="cuda")
    mask = torch.ones(B, 32, dtype=torch.int64, device="cuda")
    mask[:, 24:] = 0
    ours = _graphed(flat_forward, W, ids, mask)
    ref = _graphed(torch_forward, W, ids, mask)
    ms = timed(ours.replay, steps, warmup)
    ms_ref = timed(ref.replay, steps, warmup)
    D, F_, layers = 768, 3072, 12
    per_tok = layers * (2 * D * (3 * D + D + F_) + 2 * F_ * D + 4 * 32 * D) + 2 * D * 128
    flops = per_tok * B * 32.0
    return {"stage": "encode", "batch": B, "ms": ms, "queries_per_s": B / ms * 1e3, "tflops": flops / ms / 1e9,
            "torch_ms": ms_ref, "torch_queries_per_s": B / ms_ref * 1e3, "work_gflop": flops / 1e9}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--stage", default="all", choices=("s2", "s3", "s4", "exact", "encode", "all"))
    ap.add_argument("--docs", type=int, default=2_000_000)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--nc", type=int, default=32)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--rerank", default="tc", choices=("tc", "simt"))
    ap.add_argument("--s3-mode", type=int, default=0, choices=(0, 1),
                    help="Stage 3: 0 walk-once (per-token for dense ranges), 1 per-token only")
    ap.add_argument("--s3-range", type=int, default=0, help="Stage 3 walk range width in passages (0: auto)")
    a = ap.parse_args()
    dev = "cuda"
    t0 = time.time()
    centres, C = synth.make_centroids(num_centres=1024, subs=64, seed=0, device=dev)
    Q = synth.make_queries(centres, a.batch, seed=1000).view(a.batch, 32, 128)
    stages = ("s2", "s3", "s4") if a.stage == "all" else (a.stage,)
    out = []
    if "s2" in stages:
        ms = timed(lambda: centroid_topk(Q, C, a.nc), a.steps, a.warmup)
        flops = 2.0 * a.batch * 32 * C.shape[0] * 128
        out.append({"stage": "s2", "ms": ms, "tflops": flops / ms / 1e9, "work_gflop": flops / 1e9})
    if "s3" in stages or "s4" in stages:
        corp = synth.make_corpus(a.docs, centres, C, seed=0, device=dev)
        ix = index_build.plain_ivf_index(corp["codes"], corp["doclens"], C.shape[0])
        wix = WeftIndex(ix["csr_row_ptrs"], ix["csr_col_eids"], ix["csr_block_sums"], ix["csr_lengths"],
                        ix["csr_packed_24"], corp["doc_offsets"], corp["doclens"], corp["codes"], corp["residuals"],
                        C, corp["bucket_weights"], corp["reversed_bit_map"], corp["decomp_table"], E=ix["E"])
        print(f"corpus ready in {time.time() - t0:.1f} s", file=sys.stderr)
        if "s3" in stages:
            wix.set_stage3_mode(a.s3_mode, a.s3_range)
            topc, sc, _, _ = centroid_topk(Q, C, a.nc)
            ms = timed(lambda: wix.candidates(topc, sc, a.K), a.steps, a.warmup)
            wix.stats(reset=True)             # work counts from one more, untimed pass
            wix.candidates(topc, sc, a.K)
            st = wix.stats()
            b = 3.0 * st["distinct_postings"] + 8.0 * st["touched"]
            out.append({"stage": "s3", "s3_mode": a.s3_mode, "s3_range": a.s3_range, "ms": ms, "gbs": b / ms / 1e6,
                        "postings_per_query": st["postings"] / a.batch,
                        "distinct_postings_per_query": st["distinct_postings"] / a.batch,
                        "touched_per_query": st["touched"] / a.batch, "dense_ranges": st["dense_ranges"]})
        if "s4" in stages:
            cand = synth.random_candidates(a.docs, a.batch, a.K, seed=0, device=dev)
            mode = 1 if a.rerank == "tc" else 0
            ms = timed(lambda: wix.tile_maxsim(Q, cand, mode=mode), a.steps, a.warmup)
            toks = int(wix.doc_lens[cand.long()].sum())
            b = 36.0 * toks + 16.0 * cand.numel()
            out.append({"stage": "s4", "ms": ms, "gbs": b / ms / 1e6, "doc_tokens_per_s": toks / ms * 1e3,
                        "tflops": 2.0 * 32 * 128 * toks / ms / 1e9, "doc_tokens": toks, "rerank": a.rerank})
    if a.stage == "exact":
        nq, per_q = 64, 1000
        docs = synth.make_exact_docs(nq * per_q, centres, len_range=(20, 180), seed=0, device=dev)
        Qx = synth.make_queries(centres, nq, seed=7).reshape(nq, 32, 128).contiguous()
        pids = torch.arange(nq * per_q, dtype=torch.int32, device=dev).view(nq, per_q).contiguous()
        ms = timed(lambda: tile_maxsim_exact(Qx, pids, docs["doc_offsets"], docs["doclens"], docs["emb"]),
                   a.steps, a.warmup)
        toks = int(docs["doclens"].long().sum())
        b = 256.0 * toks + 16.0 * pids.numel()
        out.append({"stage": "exact", "ms": ms, "gbs": b / ms / 1e6, "doc_tokens_per_s": toks / ms * 1e3,
                    "tflops": 2.0 * 32 * 128 * toks / ms / 1e9, "doc_tokens": toks})
    if a.stage == "encode":
        out.append(encode_stage(a.batch, a.steps, a.warmup))
    for o in out:
        print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in o.items()}), flush=True)


if __name__ == "__main__":
    main()
