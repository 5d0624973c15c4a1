"""
Drop-in replacement of the reference's ``rtrag_corr_3d`` extension for the plain-IVF
`weft` path, backed by libragrt_b200.so (sm_100a).  Put ``ragrt_b200/compat`` on
``sys.path`` ahead of the reference's ``src`` and ``import rtrag_corr_3d`` as before.

Mirrors the pybind surface of the reference (src/optix_corr_torch_3d.cpp:902-971): class
``CorrIndex3D`` and the module-level knobs, with the same argument meaning and the same
error type (``RuntimeError``) for invalid input.  What is built is the `weft`
configuration: all-codewords Stage 1 (set_stage1_mode(2)), codeword weight 0 (or all-zero
sub-queries), sparse Stage 3 (any stage-3 mode gives the same results), the tensor-core
rerank ("wmma" -> tcgen05 kernel) or the CUDA-core rerank ("simt").  The OptiX RT-core
Stage 1, the CUDA-core codebook Stage 1, residual (LUT) scoring and the static CUDA-graph
path belong to other engines and raise ``NotImplementedError``.

Ordering notes (the reference leaves ties unspecified): candidates come back in ascending
pid order when every touched passage fits in k_candidates, else by (approximate score
desc, pid asc); final results by (score desc, pid asc).
"""
import torch

from ragrt_b200 import weft as _W
from ragrt_b200._lib import RagrtError

_NUM_SUBSPACES = 32
_MAX_HITS_CAP = 256          # polar scenes: E <= 256 in all-codewords mode (optix_corr_torch_3d.cpp:540)
_DROP_STAT_NAMES = ("launches", "rays", "rays_overflow", "hits_lost_to_cap", "combos", "combos_found",
                    "min_score_drops", "tasks", "tasks_dropped", "hits", "rays_short", "postings")

_knobs = {"rerank": "wmma", "codeword_weight": 1.0, "compact_scores": False, "stage3_mode": 0, "stats": False}
_stats = {k: 0 for k in _DROP_STAT_NAMES}


# ------------------------------------------------------------------ module knobs (reference :941-970)
def set_rerank_mode(mode):
    if mode not in ("wmma", "simt"):
        raise RuntimeError("rerank mode must be 'wmma' or 'simt'")
    _knobs["rerank"] = mode


def get_rerank_mode():
    return _knobs["rerank"]


def set_codeword_weight(w):
    _knobs["codeword_weight"] = float(w)


def get_codeword_weight():
    return _knobs["codeword_weight"]


def set_compact_scores(on):
    _knobs["compact_scores"] = bool(on)


def get_compact_scores():
    return _knobs["compact_scores"]


def set_stage3_mode(mode):
    _knobs["stage3_mode"] = int(mode) if 0 <= int(mode) <= 2 else 0


def get_stage3_mode():
    return _knobs["stage3_mode"]


def set_stage3_hash(on):
    _knobs["stage3_mode"] = 1 if on else 0


def get_stage3_hash():
    return _knobs["stage3_mode"] == 1


def set_drop_stats(enabled):
    _knobs["stats"] = bool(enabled)


def reset_drop_stats():
    for k in _stats:
        _stats[k] = 0


def get_drop_stats():
    """Counters since the last reset (all zero unless set_drop_stats(True)), with the
    reference's meaning (ragrt_fused_kernel.cu:33-47): launches (queries), rays (tokens x 32
    subspaces), tasks (posting lists of the kept (token, probe) pairs, ST_TASKS) and postings
    (their postings, ST_POSTINGS), the last two read from the index's device counters after
    each search while the stats are on (one device synchronisation per call, as the reference
    asks to leave stats off for timing).  The RT / codebook counters stay 0 in the weft
    configuration."""
    return dict(_stats)


def native_tile_maxsim_fused_decomp(Q, pids, doc_offsets, doc_lens, codes, residuals, centroids, bucket_weights,
                                    reversed_bit_map, decomp_table):
    """Stage 4 for one query (optix_corr_torch_3d.cpp:865-883): Q [32, 128] fp16 -> f32 [n]."""
    if Q.dim() != 2 or Q.shape[0] != 32 or Q.shape[1] != 128:
        raise RuntimeError(f"fused MaxSim kernel reads Q as [32, 128]; got [{', '.join(map(str, Q.shape))}]")
    if Q.dtype != torch.float16 or not Q.is_contiguous():
        raise RuntimeError("Q must be contiguous fp16")
    if bucket_weights.numel() != 4:
        raise RuntimeError("2-bit residuals expected")
    return _W.tile_maxsim(Q, pids.reshape(-1), doc_offsets, doc_lens, codes, residuals, centroids, bucket_weights,
                          reversed_bit_map, decomp_table, mode=_W.RERANK_MODES[_knobs["rerank"]])


def bruteforce_stage1(q_points, codewords, k, max_hits):
    raise NotImplementedError("the CUDA-core codebook Stage 1 belongs to the codebook engines (not the weft path)")


def _record(**kw):
    if _knobs["stats"]:
        for k, v in kw.items():
            _stats[k] += int(v)


# ------------------------------------------------------------------ CorrIndex3D
class CorrIndex3D:
    def __init__(self, ptx_path=None):
        self.ptx_path = ptx_path            # accepted and ignored: no OptiX pipeline
        self.E = 0
        self.geometry = 0
        self.stage1_mode = 0
        self.stage3_sparse = 1
        self.levels = []
        self._ix = None
        self._token_ids = None

    # -------------------------------------------------------------- scene (Stage 1 is all-codewords)
    def build(self, codebooks, base_radius=0.95, num_tris=4):
        """Only E (codewords per subspace) matters for the all-codewords Stage 1."""
        if codebooks.dim() != 3 or codebooks.shape[0] != _NUM_SUBSPACES or codebooks.shape[2] != 3:
            raise RuntimeError("codebooks must be [32, E, 3]")
        self.E = int(codebooks.shape[1])

    def set_polar_levels(self, taus, ks):
        """Recorded for info(); the RT scenes are not built (Stage 1 enumerates every codeword)."""
        self.levels = [{"k": int(k), "tau": [float(x) for x in t]} for t, k in zip(taus.tolist(), ks)]

    def level_for(self, k_eids):
        if not self.levels:
            return 0
        for i, lv in enumerate(self.levels):
            if lv["k"] >= k_eids:
                return i
        return len(self.levels) - 1

    def set_geometry(self, geometry):
        if geometry not in (0, 1, 2):
            raise RuntimeError("geometry must be 0 (fan), 1 (polar) or 2 (polar_iter)")
        self.geometry = geometry

    def set_stage1_mode(self, mode):
        if mode not in (0, 1, 2):
            raise RuntimeError("stage1 mode must be 0 (RT), 1 (CUDA cores) or 2 (all codewords)")
        self.stage1_mode = mode

    def set_stage3_sparse(self, sparse):
        self.stage3_sparse = 1 if sparse else 0

    def info(self):
        return {"num_entries": self.E, "geometry": ("fan", "polar", "polar_iter")[self.geometry],
                "stage1": ("rt", "cuda_cores", "all_codewords")[self.stage1_mode],
                "stage3": "sparse" if self.stage3_sparse else "dense", "rerank": _knobs["rerank"],
                "eid_bytes": self._ix.eid_bytes if self._ix else 1, "codeword_weight": _knobs["codeword_weight"],
                "compact_scores": int(_knobs["compact_scores"]), "stage3_hash": int(get_stage3_hash()),
                "stage3_mode": _knobs["stage3_mode"], "residual_scoring": 0,
                "token_level_index": self._token_ids is not None, "levels": self.levels,
                "backend": "ragrt_b200 (sm_100a)"}

    # -------------------------------------------------------------- binding (reference :453-488)
    def bind_index(self, csr_row_ptrs, csr_col_eids, csr_block_sums, csr_lengths, map_packed, doc_offsets, doc_lens,
                   codes, residuals, centroids_128, bucket_weights, reversed_bit_map, decomp_table, doc_predicates,
                   num_passages, num_centroids):
        if csr_col_eids.element_size() not in (1, 2):
            raise RuntimeError("csr_col_eids must be 8- or 16-bit")
        if csr_lengths.element_size() != 2:
            raise RuntimeError("csr_lengths must be 16-bit")
        if bucket_weights.numel() != 4:
            raise RuntimeError("rerank kernels assume 2-bit residuals (4 bucket weights)")
        if not (self.E == 0 or csr_col_eids.element_size() == 2 or self.E <= 256):
            raise RuntimeError("E > 256 needs 16-bit csr_col_eids")
        if csr_row_ptrs.numel() != _NUM_SUBSPACES * (num_centroids + 1):
            raise RuntimeError("csr_row_ptrs must be [32, num_centroids + 1]")
        n = int(doc_predicates.shape[0])         # the reference takes N from the predicates
        E = self.E if self.E > 0 else (256 if csr_col_eids.element_size() == 1 else 65536)
        try:
            self._ix = _W.WeftIndex(csr_row_ptrs, csr_col_eids, csr_block_sums, csr_lengths, map_packed,
                                    doc_offsets, doc_lens, codes, residuals, centroids_128, bucket_weights,
                                    reversed_bit_map, decomp_table, doc_predicates=doc_predicates, num_passages=n,
                                    num_centroids=num_centroids, E=E)
        except RagrtError as e:
            raise RuntimeError(str(e)) from None

    def bind_token_ids(self, token_ids):
        if self._ix is None:
            raise RuntimeError("bind_index first")
        if token_ids.numel() * 3 != self._ix.packed.numel():
            raise RuntimeError("one token id per posting")
        self._token_ids = token_ids

    def set_residual_lut(self, lut):
        if lut.numel() != 0:
            raise NotImplementedError("residual (LUT) scoring belongs to weft_resid, not the weft path")

    # -------------------------------------------------------------- searches
    def _check_query(self, Q_sub3d, k_candidates, k_eids):
        if self._ix is None:
            raise RuntimeError("Index must be bound before search!")
        if self.E <= 0:
            raise RuntimeError("build() first")
        if Q_sub3d.dim() != 3 or Q_sub3d.shape[1] != _NUM_SUBSPACES or Q_sub3d.shape[2] != 3:
            raise RuntimeError("Q_sub3d must be [ntok, 32, 3]")
        if not 1 <= Q_sub3d.shape[0] <= 32:
            raise RuntimeError("1..32 query tokens")
        if not 1 <= k_candidates <= self._ix.N:
            raise RuntimeError("bad k_candidates")
        if not 1 <= k_eids <= 256:
            raise RuntimeError("k_eids must be in [1, 256]")

    def _check_mode(self, Q_sub3d):
        if self.stage1_mode != 2:
            raise NotImplementedError("only the all-codewords Stage 1 (set_stage1_mode(2), the weft engine) is built")
        if self.E > _MAX_HITS_CAP:
            raise RuntimeError(f"all-codewords mode needs E <= {_MAX_HITS_CAP}")
        if _knobs["codeword_weight"] != 0.0 and bool((Q_sub3d != 0).any()):
            raise NotImplementedError("codeword-weighted Stage 2 scores belong to the codebook engines; "
                                      "weft uses set_codeword_weight(0)")

    def _n_eids(self, k_eids):
        return min(int(k_eids), self.E)

    def _stats_begin(self):
        if _knobs["stats"]:
            self._ix.stats(reset=True)             # drop what calls made with the stats off counted

    def _stats_end(self):
        if _knobs["stats"]:
            st = self._ix.stats(reset=True)
            _record(tasks=st["tasks"], postings=st["postings"])

    def _candidates(self, topc, scores, k_cent, k_candidates, query_mask, k_eids, ntok=None):
        full = not _knobs["compact_scores"]
        if topc.dim() == 2:
            topc, scores = topc[None], scores[None]
        topc = topc[:, :, :k_cent]
        masks = torch.full((topc.shape[0],), int(query_mask) & 0xFFFFFFFF, dtype=torch.int64,
                           device=topc.device).to(torch.int32) if query_mask else None
        try:
            self._stats_begin()
            out = self._ix.candidates(topc, scores, k_candidates, ntok=ntok, masks=masks,
                                      n_eids=self._n_eids(k_eids), full_scores=full)
            self._stats_end()
            return out
        except RagrtError as e:
            raise RuntimeError(str(e)) from None

    def _rerank(self, Q_fp16, cand, k_top, query_mask):
        mode = _W.RERANK_MODES[_knobs["rerank"]]
        Q = Q_fp16 if Q_fp16.dim() == 3 else Q_fp16[None]
        if Q.shape[1:] != (32, 128):
            raise RuntimeError(f"fused MaxSim kernel reads Q as [32, 128]; got {tuple(Q.shape[1:])}")
        f = self._ix.tile_maxsim(Q, cand, mode=mode)
        masks = torch.full((cand.shape[0],), int(query_mask) & 0xFFFFFFFF, dtype=torch.int64,
                           device=cand.device).to(torch.int32) if query_mask else None
        return self._ix.final_topk(cand, f, min(k_top, cand.shape[1]), masks=masks)

    def candidates(self, Q_sub3d, topc, scores, k_cent, k_candidates, query_mask=0, k_eids=16):
        """Stages 1-3 only: (pids int32 [k_candidates] with -1 padding, approximate scores)."""
        self._check_query(Q_sub3d, k_candidates, k_eids)
        self._check_mode(Q_sub3d)
        p, s, _ = self._candidates(topc, scores, k_cent, k_candidates, query_mask, k_eids)
        _record(launches=1, rays=Q_sub3d.shape[0] * _NUM_SUBSPACES)
        return [p[0].clone(), s[0].clone()]

    def search_single_query_native(self, Q_full_128_fp32, Q_full_fp16, Q_sub3d, topc, scores, k_cent, k_candidates,
                                   k_top, query_mask=0, k_eids=16):
        self._check_query(Q_sub3d, k_candidates, k_eids)
        self._check_mode(Q_sub3d)
        cand, _, _ = self._candidates(topc, scores, k_cent, k_candidates, query_mask, k_eids)
        ids, _ = self._rerank(Q_full_fp16, cand, k_top, query_mask)
        _record(launches=1, rays=Q_sub3d.shape[0] * _NUM_SUBSPACES)
        return ids[0]

    def search_single_query_profiled(self, Q_full_128_fp32, Q_full_fp16, Q_sub3d, topc, scores, k_cent,
                                     k_candidates, k_top, query_mask=0, k_eids=16):
        """(ids, [s1, s2, s3, s4] ms) as the reference: s1 (Stage 1) and s2 (task collection)
        are fused into s3 here and report 0."""
        self._check_query(Q_sub3d, k_candidates, k_eids)
        self._check_mode(Q_sub3d)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        cand, _, _ = self._candidates(topc, scores, k_cent, k_candidates, query_mask, k_eids)
        ev[1].record()
        ids, _ = self._rerank(Q_full_fp16, cand, k_top, query_mask)
        ev[2].record()
        ev[2].synchronize()
        return ids[0], [0.0, 0.0, ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])]

    def search_batch_pipelined(self, Q_full_128_list, Q_full_fp16_list, Q_sub3d_list, topc_list, scores_list,
                               k_cent, k_candidates, k_top, query_mask=0, k_eids=16):
        """All queries in one batched launch sequence (no per-query loop): [B, k_top], -1 padded."""
        B = len(Q_full_fp16_list)
        if B < 1:
            raise RuntimeError("empty batch")
        for q in Q_sub3d_list:
            self._check_query(q, k_candidates, k_eids)
            self._check_mode(q)
        dev = Q_full_fp16_list[0].device
        ntok = torch.tensor([q.shape[0] for q in Q_sub3d_list], dtype=torch.int32, device=dev)
        full = not _knobs["compact_scores"]
        width = self._ix.NC if full else k_cent
        topc = torch.full((B, 32, k_cent), -1, dtype=torch.int32, device=dev)
        sc = torch.zeros(B, 32, width, dtype=torch.float32, device=dev)
        for b, (t, s) in enumerate(zip(topc_list, scores_list)):
            topc[b, :t.shape[0]] = t[:, :k_cent]
            sc[b, :s.shape[0]] = s[:, :width]
        cand, _, _ = self._candidates(topc, sc, k_cent, k_candidates, query_mask, k_eids, ntok=ntok)
        Q = torch.stack([q.to(torch.float16) for q in Q_full_fp16_list])
        ids, _ = self._rerank(Q, cand, k_top, query_mask)
        out = torch.full((B, k_top), -1, dtype=torch.int32, device=dev)
        out[:, :ids.shape[1]] = ids
        _record(launches=B, rays=int(ntok.sum()) * _NUM_SUBSPACES)
        return out

    def search_batch(self, Q_fp16, k_cent, k_candidates, k_top, query_mask=0, ntok=None):
        """New batched entry: Stage 2 included.  Q_fp16 [B, 32, 128] -> (ids [B, k_top], scores).
        query_mask: one uint32 for the batch or a per-query tensor [B]; ntok: per-query token
        counts [B] (list or tensor).  Host-side masks / ntok are moved to Q's device."""
        if self._ix is None:
            raise RuntimeError("Index must be bound before search!")
        B = Q_fp16.shape[0]
        if ntok is not None:
            ntok = torch.as_tensor(ntok, dtype=torch.int32).to(Q_fp16.device)
        masks = None
        if torch.is_tensor(query_mask):
            masks = query_mask.to(torch.int64).bitwise_and(0xFFFFFFFF).to(torch.int32).to(Q_fp16.device)
        elif query_mask:
            masks = torch.full((B,), int(query_mask) & 0xFFFFFFFF, dtype=torch.int64,
                               device=Q_fp16.device).to(torch.int32)
        try:
            self._stats_begin()
            out = self._ix.search(Q_fp16, nc=k_cent, K=k_candidates, k_top=k_top, ntok=ntok, masks=masks,
                                  rerank="tc" if _knobs["rerank"] == "wmma" else "simt")
            self._stats_end()
            n = int(ntok.sum()) if ntok is not None else 32 * B
            _record(launches=B, rays=n * _NUM_SUBSPACES)
            return out
        except RagrtError as e:
            raise RuntimeError(str(e)) from None

    # -------------------------------------------------------------- other engines
    def stage1_hits(self, Q_sub3d, k_eids=16):
        raise NotImplementedError("Stage-1 hits come from the RT / codebook engines, not the weft path")

    def reserve_static(self, cap, k_candidates):
        raise NotImplementedError("the static CUDA-graph path (weft_graph) is not built; the batched search "
                                  "needs no host synchronisation")

    def sparse_capacity(self):
        raise NotImplementedError("the static CUDA-graph path (weft_graph) is not built")

    def total_postings_tensor(self):
        raise NotImplementedError("the static CUDA-graph path (weft_graph) is not built")

    def static_phase_a(self, *a, **k):
        raise NotImplementedError("the static CUDA-graph path (weft_graph) is not built")

    def static_phase_b(self, *a, **k):
        raise NotImplementedError("the static CUDA-graph path (weft_graph) is not built")
