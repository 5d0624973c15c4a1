"""
Generates the golden fixtures in tests/golden/ by running the REFERENCE's own Python
code (imported from the reference source tree, which exists only in the build
container) on small seeded inputs.  The fixtures are committed; the tests never read
the reference tree.

  python tests/golden/make_golden.py [--reference /path/to/RAGRT]

Fixtures
  native_prep.npz   weft_prep.native_prep (src/weft_prep.py:32-47) on CPU fp16 tensors,
                    compact and full forms, impute on/off.
  plain_ivf.npz     build_plain_ivf.plain_ivf_csr (src/build_plain_ivf.py:28-68) for
                    max_len 65535 and 5, plus ragrt_index_lib.block_sums / pack_pids_24.
  stage3.npz        the centroid-interaction reference of tests/test_gpu_kernels.py:259-263
                    (per token, max over its probed centroids that hold the passage of the
                    centroid score; summed over tokens) on native_prep's compact outputs.
  stage4.npz        the fp32 TileMaxSim reference of tests/test_gpu_kernels.py:294-305
                    (fp16 add of centroid and bucket weight, fp32 normalise, Q.float() @ D^T,
                    max over tokens, sum), including pid -1 padding.
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from ragrt_b200 import synth  # noqa: E402


def small_corpus(num_docs=300, num_centres=64, subs=8, seed=0, len_range=(8, 60)):
    centres, cents = synth.make_centroids(num_centres=num_centres, subs=subs, seed=seed)
    corp = synth.make_corpus(num_docs, centres, cents, seed=seed, len_range=len_range)
    return centres, cents, corp


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get(
        "RAGRT_REFERENCE_DIR", os.path.join(os.path.dirname(REPO), "reference")),
        help="the reference source tree (default: RAGRT_REFERENCE_DIR, else `reference` beside this repository)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "src"))
    import weft_prep as RW                   # the reference's own modules
    import build_plain_ivf as RB
    import ragrt_index_lib as RL

    torch.manual_seed(0)
    # ---------------------------------------------------------------- native_prep
    centres, cents = synth.make_centroids(num_centres=256, subs=8, seed=3)          # 2,048 centroids
    Q = synth.make_queries(centres, 4, seed=3)                                       # [4, 32, 128] fp16
    out = {"C": cents.numpy(), "Q": Q.numpy(), "nc": np.int32(32)}
    for b in range(Q.shape[0]):
        ntok = 32 - 5 * b                                                            # ragged token counts
        out[f"ntok_{b}"] = np.int32(ntok)
        for impute in (True, False):
            t, s, m = RW.native_prep(Q[b, :ntok], cents, 32, impute=impute, compact=True)
            tag = f"{b}_{int(impute)}"
            out[f"topc_{tag}"] = t.numpy()
            out[f"scores_{tag}"] = s.numpy()
            if b == 0:                                                           # the full form once
                tf, sf, mf = RW.native_prep(Q[b, :ntok], cents, 32, impute=impute, compact=False)
                out[f"full_topc_{tag}"] = tf.numpy()
                out[f"full_scores_{tag}"] = sf.numpy()
            if m is not None:
                out[f"m_{tag}"] = m.numpy()
        if b < 2:
            out[f"s16_{b}"] = (Q[b, :ntok] @ cents.T).numpy()                        # the fp16 score matrix
    np.savez_compressed(os.path.join(HERE, "native_prep.npz"), **out)

    # ---------------------------------------------------------------- plain IVF
    _, c2, corp = small_corpus(num_docs=400, num_centres=16, subs=4, seed=1, len_range=(1, 40))
    codes = corp["codes"].numpy().astype(np.int64)
    dl = corp["doclens"].numpy()
    pids = np.repeat(np.arange(len(dl)), dl)
    out = {"codes": codes.astype(np.int32), "doclens": dl, "num_centroids": np.int32(c2.shape[0])}
    for ml in (65535, 5):
        r = RB.plain_ivf_csr(codes, pids, c2.shape[0], max_len=ml)
        lens16 = r["lengths"].astype(np.uint16)
        out[f"row_ptrs_{ml}"] = r["row_ptrs"]
        out[f"col_eids_{ml}"] = r["col_eids"]
        out[f"lengths_{ml}"] = r["lengths"]
        out[f"pids_sorted_{ml}"] = r["pids_sorted"]
        out[f"E_needed_{ml}"] = np.int32(r["E_needed"])
        out[f"block_sums_{ml}"] = RL.block_sums(lens16)
        out[f"packed_{ml}"] = RL.pack_pids_24(r["pids_sorted"])
    edge = np.array([0, 1, 255, 256, 65535, 65536, 4194303, 4194304, 8388608, RL.MAX_PID], dtype=np.int64)
    out["edge_pids"] = edge
    out["edge_packed"] = RL.pack_pids_24(edge)
    np.savez_compressed(os.path.join(HERE, "plain_ivf.npz"), **out)

    # ---------------------------------------------------------------- Stage 3 (centroid interaction)
    centres, cents, corp = small_corpus(num_docs=300, num_centres=64, subs=8, seed=5)
    codes = corp["codes"].numpy().astype(np.int64)
    dl = corp["doclens"].numpy()
    N, NC = len(dl), cents.shape[0]
    pids = np.repeat(np.arange(N), dl)
    csr = RB.plain_ivf_csr(codes, pids, NC)
    lens16 = csr["lengths"].astype(np.uint16)
    Qs = synth.make_queries(centres, 3, seed=5)
    has = np.zeros((N, NC), dtype=bool)
    has[pids, codes] = True
    out = {"C": cents.numpy(), "Q": Qs.numpy(), "codes": codes.astype(np.int32), "doclens": dl,
           "row_ptrs": csr["row_ptrs"], "col_eids": csr["col_eids"].astype(np.uint8), "lengths": lens16,
           "block_sums": RL.block_sums(lens16), "packed": RL.pack_pids_24(csr["pids_sorted"]),
           "E": np.int32(max(4, csr["E_needed"])), "nc": np.int32(8)}
    for b in range(Qs.shape[0]):
        topc, sc, m = RW.native_prep(Qs[b], cents, 8, impute=True, compact=True)
        tc, s = topc.numpy(), sc.numpy()
        ref = np.zeros(N)
        for t in range(tc.shape[0]):                                   # test_gpu_kernels.py:259-263
            v = np.where(has[:, tc[t]], s[t][None, :], -np.inf).max(1)
            v = np.where(v > 0, v, -np.inf)                            # Stage 2 keeps base > 0 only
            ref += np.where(np.isfinite(v), v, 0)
        touched = np.zeros(N, dtype=bool)
        for t in range(tc.shape[0]):
            keep = s[t] > 0
            touched |= has[:, tc[t][keep]].any(1)
        out[f"topc_{b}"] = tc
        out[f"scores_{b}"] = s
        out[f"ref_sums_{b}"] = ref
        out[f"touched_{b}"] = touched
    np.savez_compressed(os.path.join(HERE, "stage3.npz"), **out)

    # ---------------------------------------------------------------- Stage 4 (fp32 TileMaxSim)
    centres, cents, corp = small_corpus(num_docs=200, num_centres=64, subs=8, seed=7, len_range=(1, 40))
    g = torch.Generator().manual_seed(1)
    Qr = torch.nn.functional.normalize(torch.randn(32, 128, generator=g), dim=-1).half()
    N = corp["doclens"].shape[0]
    pids_t = torch.randint(0, N, (96,), generator=g).to(torch.int32)
    pids_t[::10] = -1
    doc_off = corp["doc_offsets"]
    rbm = corp["reversed_bit_map"].long()
    dt = corp["decomp_table"].long()
    bw = corp["bucket_weights"]
    ref = torch.empty(len(pids_t))
    for i, p in enumerate(pids_t.tolist()):                            # test_gpu_kernels.py:294-305
        if p < 0:
            ref[i] = float("-inf")
            continue
        a, b_ = int(doc_off[p]), int(doc_off[p + 1])
        cen = cents[corp["codes"][a:b_].long()]
        buckets = dt[rbm[corp["residuals"][a:b_].long()]].view(b_ - a, 128)
        D = (cen + bw[buckets]).float()
        D = D / D.norm(dim=1, keepdim=True)
        ref[i] = (Qr.float() @ D.T).max(dim=1).values.sum()
    out = {"Q": Qr.numpy(), "pids": pids_t.numpy(), "ref": ref.numpy(), "centroids": cents.numpy(),
           "doc_offsets": doc_off.numpy(), "doc_lens": corp["doclens"].numpy(), "codes": corp["codes"].numpy(),
           "residuals": corp["residuals"].numpy(), "bucket_weights": bw.numpy(),
           "reversed_bit_map": corp["reversed_bit_map"].numpy(), "decomp_table": corp["decomp_table"].numpy()}
    np.savez_compressed(os.path.join(HERE, "stage4.npz"), **out)
    for f in ("native_prep", "plain_ivf", "stage3", "stage4"):
        print(f, os.path.getsize(os.path.join(HERE, f + ".npz")), "bytes")


if __name__ == "__main__":
    main()
