"""
Seeded synthetic corpora and queries with the shapes of the `weft` benchmark configs.

The reference measures on LoTTE / MS MARCO ColBERT indexes, which are not available
here; these generators stand in for them with the value distributions the benchmark
configs name.  Fixed choices (the configs leave them open):

* 1,024 unit-sphere centres; each centre owns ``subs`` sub-centroids
  normalize(centre + SUB_SIGMA * g) (``subs`` = 64 -> 65,536 centroids).  Centroid id =
  centre * subs + k.  Centroids are stored fp16.
* A document has DOC_TOPICS (4) topic centres drawn uniformly; each token picks one of
  them uniformly, its embedding is normalize(centre + TOKEN_SIGMA * g) (sigma 0.15 per
  dim) and its code is the EXACT nearest sub-centroid of that centre.
* Residual r = x - centroid[code] per dim, quantised to 2 bits with cut points at the
  25/50/75 % quantiles of a seeded sample of residual values; the 4 bucket weights are
  the per-bucket means (the reference supports 4 weights shared by all dims).  Bytes use
  ColBERT's 2-bit packing: decomp_table[reversed_bit_map[byte]] gives the bucket of dims
  4j..4j+3 (first dim in the high bits).
* A query has QUERY_TOPICS (4) topic centres; its 32 tokens are drawn like doc tokens,
  L2-normalised, fp16.
* Predicates: bit b of a passage is Bernoulli(p_b) with p = (1%, 10%, 50%) on bits 0-2,
  seed 1; stored uint32 (the reference's predicate dtype).
* Skewed occupancy (the sharded config): with ``topic_zipf = s`` a topic centre is drawn
  with probability proportional to rank^-s over a seeded random ranking of the centres, for
  documents and queries alike, so a few centres' posting lists hold a large share of the
  corpus.

Everything runs in torch on the CPU (tests) or on the GPU (benchmark scale); each
centre uses its own generator seeded from (seed, centre), so the output does not depend
on chunking.
"""
import itertools
import numpy as np
import torch

NUM_CENTRES = 1024
TOKEN_SIGMA = 0.15
SUB_SIGMA = 0.06
DOC_TOPICS = 4
QUERY_TOPICS = 4
DIM = 128


def colbert_reversed_bit_map(nbits=2):
    """byte -> byte with the bit order reversed inside every nbits group (ColBERT's
    ResidualCodec.reversed_bit_map for nbits = 2)."""
    out = np.zeros(256, dtype=np.uint8)
    for i in range(256):
        z = 0
        for g in range(8 // nbits):
            x = (i >> (g * nbits)) & ((1 << nbits) - 1)
            y = 0
            for b in range(nbits):
                y |= ((x >> b) & 1) << (nbits - 1 - b)
            z |= y << (g * nbits)
        out[i] = z
    return out


def colbert_decomp_table(nbits=2):
    """[256, 4] bucket indices of the 4 dims of a byte (itertools.product order)."""
    return np.array(list(itertools.product(range(1 << nbits), repeat=8 // nbits)), dtype=np.uint8)


def _gen(seed, salt, device):
    g = torch.Generator(device=device)
    g.manual_seed((int(seed) * 1_000_003 + int(salt)) % (2 ** 63 - 1))
    return g


def topic_sampler(num_centres, seed, zipf, device):
    """Draw n topic centres: uniform, or Zipf(zipf) over a seeded ranking of the centres."""
    if not zipf:
        return lambda n, g: torch.randint(0, num_centres, (n,), generator=g, device=device)
    gp = _gen(seed, 23, device)
    rank_to_centre = torch.randperm(num_centres, generator=gp, device=device)
    w = torch.arange(1, num_centres + 1, device=device, dtype=torch.float64).pow(-float(zipf))
    w = (w / w.sum()).float()
    return lambda n, g: rank_to_centre[torch.multinomial(w, n, replacement=True, generator=g)]


def _normalize(x):
    return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12)


def make_centroids(num_centres=NUM_CENTRES, subs=64, seed=0, device="cpu"):
    """(centres fp32 [C, 128], centroids fp16 [C*subs, 128])."""
    g = _gen(seed, 7, device)
    centres = _normalize(torch.randn(num_centres, DIM, generator=g, device=device))
    noise = torch.randn(num_centres, subs, DIM, generator=g, device=device)
    cents = _normalize(centres[:, None, :] + SUB_SIGMA * noise).reshape(-1, DIM)
    return centres, cents.half().contiguous()


def make_queries(centres, nq, seed=0, ntok=32, topics=QUERY_TOPICS, device=None, topic_zipf=None):
    """Q fp16 [nq, ntok, 128], L2-normalised rows."""
    device = device or centres.device
    g = _gen(seed, 11, device)
    C = centres.shape[0]
    qt = topic_sampler(C, 0, topic_zipf, device)(nq * topics, g).view(nq, topics)
    pick = torch.randint(0, topics, (nq, ntok), generator=g, device=device)
    cen = torch.gather(qt, 1, pick)
    x = centres[cen] + TOKEN_SIGMA * torch.randn(nq, ntok, DIM, generator=g, device=device)
    return _normalize(x).half().contiguous()


def make_corpus(num_docs, centres, centroids, len_range=(60, 180), seed=0, topics=DOC_TOPICS,
                device=None, sample_tokens=1 << 16, topic_zipf=None):
    """Documents drawn from the centres; codes are the exact nearest sub-centroid.

    Returns dict(doclens int32 [N], doc_offsets int64 [N+1], codes int32 [T],
    residuals uint8 [T, 32], bucket_weights fp16 [4], bucket_cutoffs fp32 [3],
    reversed_bit_map uint8 [256], decomp_table uint8 [256, 4]) as torch tensors on `device`.
    """
    device = device or centres.device
    C = centres.shape[0]
    subs = centroids.shape[0] // C
    cent32 = centroids.float().view(C, subs, DIM)
    g = _gen(seed, 13, device)
    lo, hi = len_range
    doclens = torch.randint(lo, hi + 1, (num_docs,), generator=g, device=device, dtype=torch.int64)
    offsets = torch.zeros(num_docs + 1, dtype=torch.int64, device=device)
    offsets[1:] = torch.cumsum(doclens, 0)
    T = int(offsets[-1])
    dtopics = topic_sampler(C, 0, topic_zipf, device)(num_docs * topics, g).view(num_docs, topics)
    pid = torch.repeat_interleave(torch.arange(num_docs, device=device), doclens)
    tpick = torch.randint(0, topics, (T,), generator=g, device=device)
    tok_centre = dtopics[pid, tpick]
    del pid, tpick
    order = torch.argsort(tok_centre)
    counts = torch.bincount(tok_centre, minlength=C).tolist()
    starts = np.concatenate([[0], np.cumsum(counts)])
    del tok_centre

    rbm = colbert_reversed_bit_map()
    dt = colbert_decomp_table()
    inv_rbm = np.argsort(rbm).astype(np.int64)          # rbm[inv_rbm[v]] == v
    inv_rbm_t = torch.from_numpy(inv_rbm).to(device)

    CHUNK = 1 << 22                     # tokens generated at once (popular centres are split)

    def tokens_of_centre(c, i=0):
        # chunk i of centre c's tokens; chunk 0 uses the centre's own generator, so centres
        # with at most CHUNK tokens come out as one draw
        n = min(CHUNK, counts[c] - i * CHUNK)
        gc = _gen(seed, 1_000 + c, device) if i == 0 else _gen(seed, 10_000_000 + c * 65_536 + i, device)
        x = _normalize(centres[c][None, :] + TOKEN_SIGMA * torch.randn(n, DIM, generator=gc, device=device))
        s = x @ cent32[c].T
        k = s.argmax(dim=1)
        r = x - cent32[c][k]
        return k, r

    # bucket cut points / weights from a seeded sample of residual values
    samp = []
    got = 0
    for c in range(C):
        if counts[c] == 0:
            continue
        _, r = tokens_of_centre(c)
        samp.append(r.reshape(-1))
        got += r.shape[0]
        if got >= sample_tokens:
            break
    samp = torch.cat(samp).float().cpu()
    cut = torch.quantile(samp[: 1 << 24], torch.tensor([0.25, 0.5, 0.75]))
    bidx = torch.bucketize(samp, cut)
    bw = torch.stack([samp[bidx == b].mean() for b in range(4)])

    codes = torch.empty(T, dtype=torch.int32, device=device)
    residuals = torch.empty(T, 32, dtype=torch.uint8, device=device)
    cut_d = cut.to(device)
    shifts = torch.tensor([6, 4, 2, 0], device=device)
    for c in range(C):
        for i in range((counts[c] + CHUNK - 1) // CHUNK):
            k, r = tokens_of_centre(c, i)
            idx = order[starts[c] + i * CHUNK:starts[c] + i * CHUNK + k.shape[0]]
            codes[idx] = (c * subs + k).to(torch.int32)
            b = torch.bucketize(r, cut_d).view(-1, 32, 4)             # bucket per dim
            v = (b << shifts).sum(-1)                                  # decomp_table row index
            residuals[idx] = inv_rbm_t[v].to(torch.uint8)
            del k, r, b, v
    return {
        "doclens": doclens.to(torch.int32), "doc_offsets": offsets, "codes": codes,
        "residuals": residuals, "bucket_weights": bw.half().to(device), "bucket_cutoffs": cut.to(device),
        "reversed_bit_map": torch.from_numpy(rbm).to(device),
        "decomp_table": torch.from_numpy(dt).to(device),
    }


def make_exact_docs(num_docs, centres, len_range=(20, 180), seed=0, topics=DOC_TOPICS, device=None):
    """Uncompressed passages for the exact-rerank workload: token = normalize(centre +
    TOKEN_SIGMA * g) of one of the passage's topic centres, fp16.  Returns dict(doclens int32
    [N], doc_offsets int64 [N+1], emb fp16 [T, 128])."""
    device = device or centres.device
    C = centres.shape[0]
    g = _gen(seed, 29, device)
    lo, hi = len_range
    doclens = torch.randint(lo, hi + 1, (num_docs,), generator=g, device=device, dtype=torch.int64)
    offsets = torch.zeros(num_docs + 1, dtype=torch.int64, device=device)
    offsets[1:] = torch.cumsum(doclens, 0)
    T = int(offsets[-1])
    dtopics = torch.randint(0, C, (num_docs, topics), generator=g, device=device)
    pid = torch.repeat_interleave(torch.arange(num_docs, device=device), doclens)
    tc = dtopics[pid, torch.randint(0, topics, (T,), generator=g, device=device)]
    emb = _normalize(centres[tc] + TOKEN_SIGMA * torch.randn(T, DIM, generator=g, device=device)).half()
    return {"doclens": doclens.to(torch.int32), "doc_offsets": offsets, "emb": emb.contiguous()}


def make_predicates(num_docs, selectivities=(0.01, 0.10, 0.50), seed=1, device="cpu"):
    """uint32 [N]: bit b set with probability selectivities[b]."""
    g = _gen(seed, 17, device)
    pred = torch.zeros(num_docs, dtype=torch.int64, device=device)
    for b, p in enumerate(selectivities):
        pred |= (torch.rand(num_docs, generator=g, device=device) < p).long() << b
    return pred.to(torch.uint32)


def random_candidates(num_docs, nq, K, seed=0, device="cpu"):
    """[nq, K] int32 pids drawn uniformly without replacement per query (Stage-4 config)."""
    out = torch.empty(nq, K, dtype=torch.int32, device=device)
    for q in range(nq):
        g = _gen(seed, 100_000 + q, device)
        out[q] = torch.randperm(num_docs, generator=g, device=device)[:K].to(torch.int32)
    return out
