"""
Host side of the B200 `weft` path: torch tensors in, torch tensors out, every compute
step in libragrt_b200.so (sm_100a CUDA).  torch is used for device memory and streams
only; nothing here computes scores.

  WeftIndex        a bound plain-IVF index (CorrIndex3D.bind_index's arrays) and the
                   batched search: centroid_topk (Stage 2) -> candidates (Stages 1-3)
                   -> tile_maxsim (Stage 4) -> final_topk, or all of it in search().
  centroid_topk    Stage 2 for arbitrary Q / C (weft_prep.native_prep's computation).
  tile_maxsim      Stage 4 for arbitrary arrays (native_tile_maxsim_fused_decomp).
"""
import ctypes as C

import torch

from . import _lib

RERANK_MODES = {"tc": 1, "wmma": 1, "simt": 0}


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def _need_cuda(*ts):
    """Every tensor argument of a call (None for an absent optional one) must live on the
    current CUDA device: the kernels dereference each pointer on that device, on torch's
    current stream."""
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("ragrt_b200 runs on CUDA tensors only (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors of one call are on {dev} and {t.device}: all must be on one device")
    if dev is not None and dev.index != torch.cuda.current_device():
        raise RuntimeError(f"tensors are on {dev} but the current device is cuda:{torch.cuda.current_device()}")


def _c(t, dtype):
    return t.to(dtype).contiguous()


def centroid_topk(Q, C_, nc, impute=True, ntok=None, full=False):
    """Stage 2 for a batch.  Q [B, rows, 128] (rows <= 32) fp16 CUDA, C [NC, 128] fp16.
    Returns (topc int32 [B, rows, ncol], scores f32 [B, rows, ncol], m f32 [B, rows],
    full16 fp16 [B, rows, NC] or None); ncol = min(nc, min(nc + impute, NC))."""
    _need_cuda(Q, C_, ntok)
    Q = _c(Q, torch.float16)
    C_ = _c(C_, torch.float16)
    if Q.dim() == 2:
        Q = Q[None]
    B, rows, dim = Q.shape
    NC = C_.shape[0]
    kk = min(nc + (1 if impute else 0), NC)
    ncol = min(nc, kk)
    dev = Q.device
    topc = torch.empty(B, rows, ncol, dtype=torch.int32, device=dev)
    scores = torch.empty(B, rows, ncol, dtype=torch.float32, device=dev)
    m = torch.empty(B, rows, dtype=torch.float32, device=dev)
    full16 = torch.empty(B, rows, NC, dtype=torch.float16, device=dev) if full else None
    nt = _c(ntok, torch.int32) if ntok is not None else None
    _lib.check(_lib.lib().ragrt_centroid_topk(_ptr(Q), _ptr(nt), B, rows, _ptr(C_), NC, nc, int(bool(impute)),
                                             _ptr(topc), _ptr(scores), _ptr(m), _ptr(full16), _stream()))
    return topc, scores, m, full16


def tile_maxsim_exact(Q, pids, doc_offsets, doc_lens, doc_emb):
    """Exact TileMaxSim over raw fp16 doc-token embeddings.  Q [B, 32, 128] (or [32, 128])
    fp16, pids [B, n] (or [n]) int32, doc_emb [T, 128] fp16 -> f32 scores [B, n] (or [n])."""
    _need_cuda(Q, pids, doc_offsets, doc_lens, doc_emb)
    squeeze = Q.dim() == 2
    Q = _c(Q, torch.float16)
    if squeeze:
        Q = Q[None]
        pids = pids.reshape(1, -1)
    if Q.shape[1:] != (32, 128):
        raise RuntimeError(f"MaxSim kernel reads Q as [32, 128]; got {tuple(Q.shape[1:])}")
    pids = _c(pids, torch.int32)
    emb = _c(doc_emb, torch.float16)
    B, n = pids.shape
    out = torch.empty(B, n, dtype=torch.float32, device=Q.device)
    if n:
        _lib.check(_lib.lib().ragrt_tile_maxsim_exact(_ptr(Q), _ptr(pids), B, n, _ptr(_c(doc_offsets, torch.int64)),
                                                      _ptr(_c(doc_lens, torch.int32)), doc_lens.shape[0], _ptr(emb),
                                                      _ptr(out), _stream()))
    return out[0] if squeeze else out


def tile_maxsim(Q, pids, doc_offsets, doc_lens, codes, residuals, centroids, bucket_weights,
                reversed_bit_map, decomp_table, mode=1):
    """Stage 4.  Q [B, 32, 128] (or [32, 128]) fp16, pids [B, n] (or [n]) int32 -> f32 scores."""
    _need_cuda(Q, pids, doc_offsets, doc_lens, codes, residuals, centroids, bucket_weights, reversed_bit_map,
               decomp_table)
    squeeze = Q.dim() == 2
    Q = _c(Q, torch.float16)
    if squeeze:
        Q = Q[None]
        pids = pids.reshape(1, -1)
    if Q.shape[1:] != (32, 128):
        raise RuntimeError(f"fused MaxSim kernel reads Q as [32, 128]; got {tuple(Q.shape[1:])}")
    if bucket_weights.numel() != 4:
        raise RuntimeError("2-bit residuals expected (4 bucket weights)")
    pids = _c(pids, torch.int32)
    B, n = pids.shape
    out = torch.empty(B, n, dtype=torch.float32, device=Q.device)
    if n == 0:
        return out[0] if squeeze else out
    args = [_c(doc_offsets, torch.int64), _c(doc_lens, torch.int32), _c(codes, torch.int32),
            residuals.contiguous(), _c(centroids, torch.float16), _c(bucket_weights, torch.float16),
            _c(reversed_bit_map, torch.uint8), _c(decomp_table, torch.uint8)]
    N = args[1].shape[0]
    _lib.check(_lib.lib().ragrt_tile_maxsim(_ptr(Q), _ptr(pids), B, n, _ptr(args[0]), _ptr(args[1]), N,
                                           _ptr(args[2]), _ptr(args[3]), _ptr(args[4]), _ptr(args[5]),
                                           _ptr(args[6]), _ptr(args[7]), _ptr(out), int(mode), _stream()))
    return out[0] if squeeze else out


def final_topk(pids, scores, k, preds=None, masks=None, num_preds=None):
    """Failing / padding candidates -> -inf, then top-k by (score desc, pid asc)."""
    _need_cuda(pids, scores, preds, masks)
    pids = _c(pids, torch.int32)
    scores = _c(scores, torch.float32)
    if pids.dim() == 1:
        pids, scores = pids[None], scores[None]
    B, n = pids.shape
    k = min(k, n)
    ids = torch.empty(B, k, dtype=torch.int32, device=pids.device)
    sc = torch.empty(B, k, dtype=torch.float32, device=pids.device)
    pr = _c(preds, torch.int32) if preds is not None else None
    mk = _c(masks, torch.int32) if masks is not None else None
    npred = int(num_preds) if num_preds is not None else (pr.shape[0] if pr is not None else 0)
    _lib.check(_lib.lib().ragrt_final_topk(_ptr(pids), _ptr(scores), B, n, _ptr(pr), npred, _ptr(mk), k,
                                          _ptr(ids), _ptr(sc), _stream()))
    return ids, sc


class WeftIndex:
    """A bound plain-IVF index (the arrays of CorrIndex3D.bind_index,
    optix_corr_torch_3d.cpp:453-488).  Keeps references to the tensors it binds (converted
    to the kernel dtypes where needed), like the reference."""

    def __init__(self, csr_row_ptrs, csr_col_eids, csr_block_sums, csr_lengths, csr_packed_24,
                 doc_offsets, doc_lens, codes, residuals, centroids, bucket_weights, reversed_bit_map,
                 decomp_table, doc_predicates=None, num_passages=None, num_centroids=None, E=None):
        _need_cuda(csr_row_ptrs, csr_col_eids, csr_block_sums, csr_lengths, csr_packed_24, doc_offsets,
                   doc_lens, codes, residuals, centroids, bucket_weights, reversed_bit_map, decomp_table,
                   doc_predicates)
        if csr_col_eids.element_size() not in (1, 2):
            raise RuntimeError("csr_col_eids must be 8- or 16-bit")
        if csr_lengths.element_size() != 2:
            raise RuntimeError("csr_lengths must be 16-bit")
        if bucket_weights.numel() != 4:
            raise RuntimeError("rerank kernels assume 2-bit residuals (4 bucket weights)")
        self.device = csr_row_ptrs.device
        self.row_ptrs = _c(csr_row_ptrs, torch.int64)
        self.col_eids = csr_col_eids.contiguous()
        self.eid_bytes = self.col_eids.element_size()
        self.block_sums = _c(csr_block_sums, torch.int64)
        self.lengths = csr_lengths.contiguous()
        self.packed = _c(csr_packed_24, torch.uint8)
        self.doc_offsets = _c(doc_offsets, torch.int64)
        self.doc_lens = _c(doc_lens, torch.int32)
        self.codes = _c(codes, torch.int32)
        self.residuals = _c(residuals, torch.uint8)
        self.centroids = _c(centroids, torch.float16)
        self.bucket_weights = _c(bucket_weights, torch.float16)
        self.rbm = _c(reversed_bit_map, torch.uint8)
        self.decomp = _c(decomp_table, torch.uint8)
        N = int(num_passages) if num_passages is not None else self.doc_lens.shape[0]
        if doc_predicates is not None:
            self.preds = _c(doc_predicates.to(torch.int64) & 0xFFFFFFFF, torch.int64).to(torch.int32) \
                if doc_predicates.dtype != torch.int32 else doc_predicates.contiguous()
            N = self.preds.shape[0] if num_passages is None else N
        else:
            self.preds = None
        self.N = N
        self.NC = int(num_centroids) if num_centroids is not None else self.centroids.shape[0]
        self.E = int(E) if E is not None else (256 if self.eid_bytes == 1 else 65536)
        if self.row_ptrs.numel() != 32 * (self.NC + 1):
            raise RuntimeError("csr_row_ptrs must be [32, num_centroids + 1]")
        d = _lib.IndexDesc()
        d.csr_row_ptrs = self.row_ptrs.data_ptr()
        d.csr_col_eids = self.col_eids.data_ptr()
        d.eid_bytes = self.eid_bytes
        d.csr_block_sums = self.block_sums.data_ptr()
        d.csr_lengths = self.lengths.data_ptr()
        d.csr_packed_24 = self.packed.data_ptr()
        d.num_lists = self.lengths.numel()
        d.num_postings = self.packed.numel() // 3
        d.doc_offsets = self.doc_offsets.data_ptr()
        d.doc_lens = self.doc_lens.data_ptr()
        d.codes = self.codes.data_ptr()
        d.residuals = self.residuals.data_ptr()
        d.num_tokens = self.codes.numel()
        d.centroids = self.centroids.data_ptr()
        d.bucket_weights = self.bucket_weights.data_ptr()
        d.reversed_bit_map = self.rbm.data_ptr()
        d.decomp_table = self.decomp.data_ptr()
        d.doc_predicates = self.preds.data_ptr() if self.preds is not None else None
        d.num_passages = self.N
        d.num_centroids = self.NC
        d.num_eids = self.E
        self._desc = d
        h = C.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().ragrt_index_create(C.byref(d), C.byref(h), _stream()))
        self._h = h

    @property
    def handle(self):
        if not self._h:
            raise RuntimeError("index closed")
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().ragrt_index_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ stages
    def centroid_topk(self, Q, nc, ntok=None, impute=True):
        return centroid_topk(Q, self.centroids, nc, impute=impute, ntok=ntok)

    def candidates(self, topc, scores, K, ntok=None, masks=None, n_eids=None, full_scores=False):
        """Stages 1-3: topc [B, rows, kc], scores (compact [B, rows, kc] or full [B, rows, NC]).
        Returns (pids int32 [B, K] -1-padded, sums f32 [B, K] -inf-padded, touched int64 [B])."""
        _need_cuda(topc, scores, ntok, masks)
        topc = _c(topc, torch.int32)
        scores = _c(scores, torch.float32)
        if topc.dim() == 2:
            topc, scores = topc[None], scores[None]
        B, rows, kc = topc.shape
        pids = torch.empty(B, K, dtype=torch.int32, device=topc.device)
        sums = torch.empty(B, K, dtype=torch.float32, device=topc.device)
        touched = torch.empty(B, dtype=torch.int64, device=topc.device)
        nt = _c(ntok, torch.int32) if ntok is not None else None
        mk = _c(masks, torch.int32) if masks is not None else None
        ne = self.E if n_eids is None else min(int(n_eids), self.E)
        _lib.check(_lib.lib().ragrt_weft_candidates(self.handle, _ptr(topc), _ptr(scores), int(bool(full_scores)),
                                                   _ptr(nt), B, rows, kc, ne, _ptr(mk), K, _ptr(pids),
                                                   _ptr(sums), _ptr(touched), _stream()))
        return pids, sums, touched

    def tile_maxsim(self, Q, pids, mode=1):
        """Stage 4 on the bound index (the kernel the batched search runs): Q [B, 32, 128] (or
        [32, 128]) fp16, pids [B, n] (or [n]) int32 -> f32 scores."""
        _need_cuda(Q, pids)
        squeeze = Q.dim() == 2
        Q = _c(Q, torch.float16)
        if squeeze:
            Q = Q[None]
            pids = pids.reshape(1, -1)
        if Q.shape[1:] != (32, 128):
            raise RuntimeError(f"fused MaxSim kernel reads Q as [32, 128]; got {tuple(Q.shape[1:])}")
        pids = _c(pids, torch.int32)
        B, n = pids.shape
        out = torch.empty(B, n, dtype=torch.float32, device=Q.device)
        if n:
            _lib.check(_lib.lib().ragrt_index_tile_maxsim(self.handle, _ptr(Q), _ptr(pids), B, n, _ptr(out), int(mode),
                                                          _stream()))
        return out[0] if squeeze else out

    def final_topk(self, pids, scores, k, masks=None):
        return final_topk(pids, scores, k, preds=self.preds, masks=masks, num_preds=self.N)

    def search(self, Q, nc=32, K=4096, k_top=10, ntok=None, masks=None, rerank="tc", n_eids=None, out=None):
        """The fused batched search.  Q [B, 32, 128] fp16 -> (ids int32 [B, k_top], scores f32)."""
        _need_cuda(Q, ntok, masks, *(out or ()))
        Q = _c(Q, torch.float16)
        if Q.dim() == 2:
            Q = Q[None]
        B = Q.shape[0]
        if out is None:
            ids = torch.empty(B, k_top, dtype=torch.int32, device=Q.device)
            sc = torch.empty(B, k_top, dtype=torch.float32, device=Q.device)
        else:
            ids, sc = out
        nt = _c(ntok, torch.int32) if ntok is not None else None
        mk = _c(masks, torch.int32) if masks is not None else None
        ne = self.E if n_eids is None else min(int(n_eids), self.E)
        _lib.check(_lib.lib().ragrt_weft_search(self.handle, _ptr(Q), _ptr(nt), B, nc, ne, _ptr(mk), K, k_top,
                                               RERANK_MODES[rerank], _ptr(ids), _ptr(sc), _stream()))
        return ids, sc

    def search_profiled(self, Q, events, nc=32, K=4096, k_top=10, ntok=None, masks=None, rerank="tc",
                        n_eids=None, out=None):
        """search() recording 5 torch.cuda.Event objects at the stage boundaries (no sync)."""
        _need_cuda(Q, ntok, masks, *(out or ()))
        Q = _c(Q, torch.float16)
        B = Q.shape[0]
        ids, sc = out if out is not None else (torch.empty(B, k_top, dtype=torch.int32, device=Q.device),
                                               torch.empty(B, k_top, dtype=torch.float32, device=Q.device))
        for e in events:
            if not e.cuda_event:
                e.record()                       # torch creates the event lazily
        arr = (C.c_void_p * 5)(*[C.c_void_p(e.cuda_event) for e in events])
        nt = _c(ntok, torch.int32) if ntok is not None else None
        mk = _c(masks, torch.int32) if masks is not None else None
        ne = self.E if n_eids is None else min(int(n_eids), self.E)
        _lib.check(_lib.lib().ragrt_weft_search_profiled(self.handle, _ptr(Q), _ptr(nt), B, nc, ne, _ptr(mk), K,
                                                        k_top, RERANK_MODES[rerank], _ptr(ids), _ptr(sc), arr,
                                                        _stream()))
        return ids, sc

    def pass_counts(self, mask=0):
        """(pass int64 [NC], total int64 [NC]): postings per centroid whose passage passes
        (pred & mask) != 0, and all postings per centroid (mask 0: every posting passes)."""
        dev = self.centroids.device
        pc = torch.empty(self.NC, dtype=torch.int64, device=dev)
        tc = torch.empty(self.NC, dtype=torch.int64, device=dev)
        _lib.check(_lib.lib().ragrt_centroid_pass_counts(self.handle, int(mask) & 0xFFFFFFFF, _ptr(pc), _ptr(tc),
                                                         _stream()))
        return pc, tc

    def count_distinct(self, enable=True):
        """Kept for compatibility: distinct postings are always counted (Stage 3 finds each
        query's distinct lists anyway)."""
        _lib.check(_lib.lib().ragrt_index_count_distinct(self.handle, int(bool(enable))))

    def set_stage3_mode(self, mode, range_passages=0):
        """0 (default): walk each distinct probed list once per pid range (ranges too dense for
        the walk go to the per-token kernel); 1: the per-token kernel on every range.  Results
        are bit-identical.  range_passages: the walk's pid-range width (0: automatic)."""
        _lib.check(_lib.lib().ragrt_index_set_stage3_mode(self.handle, int(mode), int(range_passages)))

    def stats(self, reset=False):
        """Counters since the last reset: queries, postings (scanned per kept (token, probe),
        the reference's ST_POSTINGS), distinct_postings (each probed list once per query),
        touched, probes (kept), candidates, tasks (the reference's ST_TASKS), dense_ranges (pid-range
        blocks Stage 3 handed from its walk-once kernel to the per-token one)."""
        buf = (C.c_uint64 * _lib.NUM_STATS)()
        _lib.check(_lib.lib().ragrt_index_stats(self.handle, buf, int(bool(reset))))
        return dict(zip(_lib.STAT_NAMES, list(buf)))
