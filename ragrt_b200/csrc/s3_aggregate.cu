// s3_aggregate.cu -- Stages 1-3 of the reference in `weft` mode (all-codewords Stage 1,
// codeword weight 0): for every query token t and probed centroid c_tj whose base score
// (the imputation-shifted centroid score) is > 0, every posting of c_tj contributes
// fp16(base) to (pid, t); a passage's score is the sum over tokens of its per-token max.
// Reference: ragrt_fused_kernel.cu:64-263 (task collection, MIN_BASE_SCORE :206),
// :343-392 (expand, filter :387, fp16 key :366), :403-431 + :1120-1156 (max per
// (pid, token), sum per pid), optix_corr_torch_3d.cpp:569-585 (top-k candidates).
//
// B200 design (no sort, no host synchronisation):
//   * The pid space is cut into ranges of W = 2^w_shift passages.  A work item is one query
//     and 8 consecutive ranges (so the query's probe table is built once per item); for each
//     range the CTA keeps, per passage, a 64-bit accumulator in shared memory: (sum of fp16
//     maxima in units of 2^-24) << 6 | (number of tokens).
//   * A warp processes one query token at a time.  Its probes are sorted by score
//     (native_prep returns them best first), so the FIRST probe of token t that holds a
//     passage carries that token's max: a per-warp "seen" bitmap over the range marks
//     (passage, t); duplicates inside one 32-posting chunk are resolved with
//     __match_any_sync in favour of the lowest lane (= the better probe).
//   * The posting sub-list of centroid c that falls in range r is read directly through
//     the index's range-offset table (boff), coalesced, once per (token, probe).
//   * Touched passages (non-zero accumulators, found by a scan at the end of each range) are
//     emitted as 64-bit ranking keys into a per-query pool; a per-query CTA then selects the
//     K candidates exactly (radix select + bitonic sort).
// Sums are exact (fixed point) and rounded once to fp32; ties in candidate selection go to
// the lower pid.
#include <algorithm>

#include "common.cuh"
#include "index.cuh"
#include "s3_common.cuh"

namespace ragrt {

constexpr int kS3Warps = 8;
constexpr int kS3Threads = kS3Warps * 32;
constexpr int kS3RangesPerJob = 8;   // consecutive pid ranges of one query per work item (one probe table),
                                     // fewer when the items would not give each CTA several
constexpr int kS3Batch = 8;       // 32-posting chunks whose pid loads a warp keeps in flight together

struct S3Params {
    // index
    const uint8_t* packed;
    const uint32_t* preds;
    const int64_t* rp;
    const int64_t* list_off;
    const int64_t* cstart;
    const int32_t* clists;
    const uint32_t* boff;
    int N, NC, R, w_shift, n_eids;
    // queries
    const int32_t* topc;
    const float* scores;
    int full_scores, rows, kc;
    const int32_t* ntok;
    const uint32_t* masks;
    int q0, nq;                  // queries [q0, q0 + nq) of the batch
    int rpj;                     // pid ranges per work item
    // output
    uint64_t* pool;              // [nq][pool_cap]
    int64_t pool_cap;
    unsigned long long* pool_count;   // [nq]
    unsigned int* work;          // work counter
    unsigned long long* stats;
    // queue mode: the work items are the pid-range blocks the walk deferred, (qi << 32 | block),
    // block b covering index ranges [b * m, b * m + m); their number is read on the device
    const unsigned long long* dense;
    const unsigned int* dense_count;
    int m;
};

__device__ __forceinline__ uint16_t f2h_pos15(float base) {
    return (uint16_t)(__half_as_ushort(__float2half_rn(base)) & 0x7FFF);   // ragrt_fused_kernel.cu:366
}

__global__ void __launch_bounds__(kS3Threads, 4)
s3_accumulate(S3Params p) {
    extern __shared__ __align__(16) unsigned char s3_smem[];
    const int W = 1 << p.w_shift;
    unsigned long long* sums = reinterpret_cast<unsigned long long*>(s3_smem);          // [W]
    uint32_t* seen = reinterpret_cast<uint32_t*>(sums + W);                              // [warps][W/32]
    int64_t* pcs = reinterpret_cast<int64_t*>(seen + kS3Warps * (W >> 5));               // [32][kc] cstart
    int32_t* pc = reinterpret_cast<int32_t*>(pcs + kRows * p.kc);                        // [32][kc] centroid
    int32_t* pcnt = pc + kRows * p.kc;                                                   // [32][kc] postings
    uint16_t* pv = reinterpret_cast<uint16_t*>(pcnt + kRows * p.kc);                     // [32][kc] fp16 bits
    __shared__ int s_np[kRows];
    __shared__ unsigned s_wcnt[kS3Warps];
    __shared__ unsigned s_unit;
    __shared__ unsigned long long s_base;

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    uint32_t* my_seen = seen + w * (W >> 5);
    for (int i = tid; i < W; i += kS3Threads) sums[i] = 0ull;
    for (int i = tid; i < kS3Warps * (W >> 5); i += kS3Threads) seen[i] = 0u;
    unsigned long long st_post = 0, st_probes = 0;
    int cached_q = -1;
    const unsigned nrb = ((unsigned)p.R + p.rpj - 1) / p.rpj;
    const unsigned total_jobs = p.dense ? *p.dense_count : (unsigned)p.nq * nrb;
    __syncthreads();

    for (;;) {
        if (tid == 0) s_unit = atomicAdd(p.work, 1u);
        __syncthreads();
        const unsigned job = s_unit;
        if (job >= total_jobs) break;
        int qi, r0, r1;
        if (p.dense) {
            const unsigned long long d = p.dense[job];
            qi = (int)(d >> 32);
            r0 = (int)(d & 0xFFFFFFFFu) * p.m;
            r1 = min(p.R, r0 + p.m);
        } else {
            qi = (int)(job / nrb);
            r0 = (int)(job % nrb) * p.rpj;
            r1 = min(p.R, r0 + p.rpj);
        }
      for (int r = r0; r < r1; ++r) {
        const int q = p.q0 + qi;
        const uint32_t mask = p.masks ? p.masks[q] : 0u;
        const int nt = p.ntok ? min(p.ntok[q], p.rows) : p.rows;

        // ---- kept probes of query q (warp t handles token t)
        if (q != cached_q) {
            for (int t = w; t < kRows; t += kS3Warps) {
                int n = 0;
                if (t < nt) {
                    for (int j0 = 0; j0 < p.kc; j0 += 32) {
                        int j = j0 + lane;
                        int c = -1;
                        float base = 0.f;
                        if (j < p.kc) {
                            c = p.topc[((int64_t)q * p.rows + t) * p.kc + j];
                            if (c >= 0 && c < p.NC)
                                base = p.full_scores ? p.scores[((int64_t)q * p.rows + t) * p.NC + c]
                                                     : p.scores[((int64_t)q * p.rows + t) * p.kc + j];
                        }
                        bool keep = c >= 0 && c < p.NC && base > 0.0f;     // MIN_BASE_SCORE
                        unsigned bal = __ballot_sync(0xFFFFFFFFu, keep);
                        if (keep) {
                            int slot = n + __popc(bal & ((1u << lane) - 1));
                            const int nl = min(p.clists[c], p.n_eids);
                            const int64_t cs = p.cstart[c];
                            pc[t * p.kc + slot] = c;
                            pv[t * p.kc + slot] = f2h_pos15(base);
                            pcs[t * p.kc + slot] = cs;
                            pcnt[t * p.kc + slot] = nl > 0 ? (int32_t)(p.list_off[p.rp[c] + nl] - cs) : 0;
                        }
                        n += __popc(bal);
                    }
                }
                if (lane == 0) s_np[t] = n;
            }
            cached_q = q;
            __syncthreads();
        }

        // ---- accumulate: warp w takes tokens w, w + warps, ...
        const int64_t range_lo = (int64_t)r << p.w_shift;
        for (int t = w; t < nt; t += kS3Warps) {
            const int np = s_np[t];
            if (np == 0) continue;
            if (lane == 0) st_probes += (unsigned long long)(r == 0 ? np : 0);
            // probes are handled in groups of 32 (one per lane); np <= kc <= 128
            for (int g0 = 0; g0 < np; g0 += 32) {
                const int j = g0 + lane;
                int64_t start = 0;
                int len = 0;
                uint16_t v = 0;
                if (j < np) {
                    const int c = pc[t * p.kc + j];
                    v = pv[t * p.kc + j];
                    const int64_t cnt = pcnt[t * p.kc + j];
                    const uint32_t* bo = p.boff + (int64_t)c * (p.R + 1) + r;
                    const int64_t hi = (int64_t)bo[1] < cnt ? (int64_t)bo[1] : cnt;
                    const int64_t lo = (int64_t)bo[0] < hi ? (int64_t)bo[0] : hi;
                    start = pcs[t * p.kc + j] + lo;
                    len = (int)(hi - lo);
                }
                // inclusive scan of len over the group
                int incl = len;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                    if (lane >= o) incl += y;
                }
                const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
                const int excl = incl - len;
                st_post += (unsigned long long)len;
                // posting e of the group lives at (start - excl) + e in the probe's list: that base
                // (signed, 48 bits) and the probe's fp16 value travel in one 64-bit shuffle
                const unsigned long long bv = ((unsigned long long)v << 48) |
                                              ((unsigned long long)(start - excl) & 0xFFFFFFFFFFFFull);
                // kS3Batch chunks of 32 postings at a time: all their pid (and predicate) loads
                // are issued before the first chunk is merged, in posting order
                for (int e0 = 0; e0 < total; e0 += 32 * kS3Batch) {
                    int32_t pid[kS3Batch];
                    uint16_t vb[kS3Batch];
#pragma unroll
                    for (int u = 0; u < kS3Batch; ++u) {
                        const int e = e0 + 32 * u + lane;
                        // source probe: the last lane whose exclusive prefix is <= e
                        int src = 0;
#pragma unroll
                        for (int step = 16; step; step >>= 1) {
                            int cand = src + step;
                            int ex = __shfl_sync(0xFFFFFFFFu, excl, cand & 31);
                            if (cand < 32 && ex <= e) src = cand;
                        }
                        const unsigned long long bv_src = __shfl_sync(0xFFFFFFFFu, bv, src);
                        vb[u] = (uint16_t)(bv_src >> 48);
                        const int64_t base = (int64_t)(bv_src << 16) >> 16;
                        pid[u] = e < total ? load_pid24(p.packed, base + e) : -1;
                    }
                    uint32_t pr[kS3Batch];
#pragma unroll
                    for (int u = 0; u < kS3Batch; ++u)
                        pr[u] = (mask && pid[u] >= 0 && pid[u] < p.N) ? p.preds[pid[u]] : 0xFFFFFFFFu;
#pragma unroll
                    for (int u = 0; u < kS3Batch; ++u) {
                        if (e0 + 32 * u >= total) break;                    // warp-uniform
                        const int local = pid[u] - (int)range_lo;
                        bool ok = pid[u] >= 0 && pid[u] < p.N && local >= 0 && local < W;
                        if (ok && mask) ok = (pr[u] & mask) != 0u;         // ragrt_fused_kernel.cu:387
                        const int key = ok ? local : (0x40000000 | lane);
                        const unsigned peers = __match_any_sync(0xFFFFFFFFu, key);
                        if (ok && lane == __ffs(peers) - 1) {
                            const uint32_t bit = 1u << (local & 31);
                            const uint32_t old = atomicOr(&my_seen[local >> 5], bit);
                            if (!(old & bit)) {
                                const unsigned long long add = (h_fixed24(vb[u]) << 6) | 1ull;
                                const unsigned long long prev = atomicAdd(&sums[local], add);
                                (void)prev;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            for (int i = lane; i < (W >> 5); i += 32) my_seen[i] = 0u;
            __syncwarp();
        }
        __syncthreads();

        // ---- emit the tile's touched passages into the query's pool: warp w scans accumulators
        // [w W/8, (w+1) W/8), counts the non-zero ones, one pool reservation per tile, then
        // writes their ranking keys and clears them
        const int seg = W / kS3Warps;
        const unsigned long long* sw = sums + w * seg;
        unsigned cnt = 0;
        for (int i = lane; i < seg; i += 32) cnt += __popc(__ballot_sync(0xFFFFFFFFu, sw[i] != 0ull));
        if (lane == 0) s_wcnt[w] = cnt;
        __syncthreads();
        if (tid == 0) {
            unsigned tot = 0;
            for (int i = 0; i < kS3Warps; ++i) { const unsigned c = s_wcnt[i]; s_wcnt[i] = tot; tot += c; }
            s_base = tot ? atomicAdd(&p.pool_count[qi], (unsigned long long)tot) : 0ull;
        }
        __syncthreads();
        uint64_t* pool = p.pool + (int64_t)qi * p.pool_cap;
        unsigned long long pos = s_base + s_wcnt[w];
        for (int i = lane; i < seg; i += 32) {
            const unsigned long long acc = sums[w * seg + i];
            const unsigned m = __ballot_sync(0xFFFFFFFFu, acc != 0ull);
            if (acc) {
                sums[w * seg + i] = 0ull;
                const float sc = __ull2float_rn(acc >> 6) * 0x1p-24f;
                pool[pos + __popc(m & ((1u << lane) - 1u))] = rank_key(sc, (int32_t)(range_lo + w * seg + i));
            }
            pos += __popc(m);
        }
        __syncthreads();
      }
    }
    // stats: postings scanned (per kept probe, whole list), kept probes
    for (int o = 16; o; o >>= 1) {
        st_post += __shfl_xor_sync(0xFFFFFFFFu, st_post, o);
        st_probes += __shfl_xor_sync(0xFFFFFFFFu, st_probes, o);
    }
    if (lane == 0 && p.stats) {
        atomicAdd(&p.stats[1], st_post);
        atomicAdd(&p.stats[4], st_probes);
    }
}

}  // namespace ragrt

using namespace ragrt;

namespace ragrt {

size_t s3_workspace_bytes(const ragrt_index* ix, int nq_sub) {
    return sizeof(uint64_t) * (size_t)nq_sub * ix->d.num_passages        // pool
           + sizeof(unsigned long long) * (size_t)nq_sub                // pool counts
           + 256                                                          // work counters, queue count
           + s3_walk_lists_bytes(nq_sub, kRows * RAGRT_MAX_PROBE)        // distinct lists per query
           + s3_walk_dense_bytes(ix, nq_sub) + 1024;                     // deferred range blocks
}

int s3_max_sub_batch(const ragrt_index* ix, int B) {
    // The candidate pool holds 8 B per passage per query.  Up to 8 GiB of it lets a whole
    // batch run as one pass (256 queries over 2 M passages: 4 GB), which avoids a second
    // pass's tail and gives the selection one CTA per query of the whole batch; larger
    // batches or corpora run in sub-batches.
    int64_t per_q = (int64_t)ix->d.num_passages * 8;
    int64_t sub = std::max<int64_t>(1, ((int64_t)8 << 30) / per_q);
    return (int)std::min<int64_t>(sub, B);
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int s3_run(ragrt_index* ix, const int32_t* topc, const float* scores, int full_scores, const int32_t* ntok, int B,
           int rows, int kc, int n_eids, const uint32_t* masks, int K, int32_t* cand_pids, float* cand_sums,
           int64_t* num_touched, void* ws, size_t ws_bytes, cudaStream_t stream) {
    const int sub = s3_max_sub_batch(ix, B);
    const size_t need = s3_workspace_bytes(ix, sub);
    if (ws_bytes < need) return fail(RAGRT_ERR_CAPACITY, "internal: stage-3 workspace %zu < %zu", ws_bytes, need);
    const int W = 1 << ix->w_shift;
    char* wsp = (char*)ws;
    uint64_t* pool = (uint64_t*)wsp;
    wsp += align256(sizeof(uint64_t) * (size_t)sub * ix->d.num_passages);
    unsigned long long* counts = (unsigned long long*)wsp;        // [sub] pool counts
    wsp += align256(sizeof(unsigned long long) * (size_t)sub);
    unsigned int* ctr = (unsigned int*)wsp;                       // [0] walk work, [1] queue work, [2] queue count
    wsp += 256;
    void* lists = wsp;
    wsp += align256(s3_walk_lists_bytes(sub, rows * kc));
    unsigned long long* dense = (unsigned long long*)wsp;

    const size_t smem = sizeof(unsigned long long) * W + sizeof(uint32_t) * kS3Warps * (W >> 5) +
                        (sizeof(int64_t) + 2 * sizeof(int32_t) + sizeof(uint16_t)) * kRows * kc + 16;
    if (smem > 220 * 1024) return fail(RAGRT_ERR_CAPACITY, "stage-3 tile needs %zu bytes of shared memory", smem);
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s3_accumulate, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    RAGRT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, s3_accumulate, kS3Threads, smem));
    per_sm = std::max(1, per_sm);
    for (int q0 = 0; q0 < B; q0 += sub) {
        const int nq = std::min(sub, B - q0);
        RAGRT_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(unsigned long long) * sub, stream));
        RAGRT_CUDA_TRY(cudaMemsetAsync(ctr, 0, 16, stream));
        const uint32_t* mk = ix->d.doc_predicates ? masks : nullptr;   // no predicates bound: no filter
        // 1. every distinct probed list walked once per pid range; dense ranges are queued
        int rc = s3_walk_run(ix, topc, scores, full_scores, ntok, q0, nq, rows, kc, n_eids, mk, pool, counts,
                             ctr + 0, dense, ctr + 2, lists, stream);
        if (rc) return rc;
        // 2. the queued ranges by the per-token kernel (no per-passage rows; exits at once when
        //    the queue is empty)
        S3Params p;
        p.packed = ix->d.csr_packed_24;
        p.preds = ix->d.doc_predicates;
        p.rp = ix->d.csr_row_ptrs;
        p.list_off = ix->list_off;
        p.cstart = ix->cstart;
        p.clists = ix->clists;
        p.boff = ix->boff;
        p.N = ix->d.num_passages;
        p.NC = ix->d.num_centroids;
        p.R = ix->num_ranges;
        p.w_shift = ix->w_shift;
        p.n_eids = n_eids;
        p.topc = topc;
        p.scores = scores;
        p.full_scores = full_scores;
        p.rows = rows;
        p.kc = kc;
        p.ntok = ntok;
        p.masks = mk;
        p.q0 = q0;
        p.nq = nq;
        p.rpj = 1;
        p.pool = pool;
        p.pool_cap = ix->d.num_passages;
        p.pool_count = counts;
        p.work = ctr + 1;
        p.stats = nullptr;                    // the statistics are counted once, by the walk's prep
        p.dense = dense;
        p.dense_count = ctr + 2;
        p.m = s3_walk_ranges(ix);
        const int grid = (int)std::min<int64_t>((int64_t)per_sm * num_sms(),
                                                (int64_t)nq * ceil_div(ix->num_ranges, p.m));
        s3_accumulate<<<grid, kS3Threads, smem, stream>>>(p);
        RAGRT_LAUNCH_CHECK();
        rc = s3_select_launch(pool, ix->d.num_passages, counts, q0, nq, K, cand_pids, cand_sums, num_touched,
                              ix->stats, stream);
        if (rc) return rc;
    }
    return RAGRT_OK;
}

}  // namespace ragrt

extern "C" int ragrt_weft_candidates(ragrt_index* ix, const int32_t* d_topc, const float* d_scores,
                                     int32_t full_scores, const int32_t* d_ntok, int32_t B, int32_t rows,
                                     int32_t kc, int32_t n_eids, const uint32_t* d_masks, int32_t K,
                                     int32_t* d_cand_pids, float* d_cand_sums, int64_t* d_num_touched,
                                     void* stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    RAGRT_REQUIRE(ix && d_topc && d_scores && d_cand_pids && d_cand_sums, "null argument");
    int rc = check_device(ix);
    if (rc) return rc;
    RAGRT_REQUIRE(B >= 1 && rows >= 1 && rows <= kRows, "B >= 1 and 1 <= rows <= 32 required");
    RAGRT_REQUIRE(kc >= 1 && kc <= RAGRT_MAX_PROBE, "kc must be in [1, %d]", RAGRT_MAX_PROBE);
    RAGRT_REQUIRE(K >= 1 && K <= RAGRT_MAX_CANDIDATES && K <= ix->d.num_passages,
                  "K=%d must be in [1, min(N, %d)]", K, RAGRT_MAX_CANDIDATES);
    RAGRT_REQUIRE(n_eids >= 1, "n_eids must be >= 1");
    const int sub = s3_max_sub_batch(ix, B);
    rc = ensure_workspace(ix, s3_workspace_bytes(ix, sub), stream);
    if (rc) return rc;
    return s3_run(ix, d_topc, d_scores, full_scores, d_ntok, B, rows, kc, n_eids, d_masks, K, d_cand_pids,
                  d_cand_sums, d_num_touched, ix->ws.base, ix->ws.bytes, stream);
}

namespace ragrt {

// warp per centroid: postings of all its lists, and those whose passage passes `mask`
__global__ void k_centroid_pass_counts(const uint8_t* __restrict__ packed, const uint32_t* __restrict__ preds,
                                       const int64_t* __restrict__ cstart, const int32_t* __restrict__ clists,
                                       const int64_t* __restrict__ rp, const int64_t* __restrict__ off, int NC,
                                       uint32_t mask, int64_t* __restrict__ pass, int64_t* __restrict__ total) {
    const int c = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (c >= NC) return;
    const int64_t a = cstart[c];
    const int64_t b = clists[c] ? off[rp[c] + clists[c]] : a;
    long long n = 0;
    if (!mask || !preds) {
        n = (long long)(b - a) * (lane == 0);
    } else {
        for (int64_t i = a + lane; i < b; i += 32) n += (preds[load_pid24(packed, i)] & mask) != 0u;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) n += __shfl_xor_sync(0xFFFFFFFFu, n, o);
    if (lane == 0) {
        pass[c] = n;
        if (total) total[c] = b - a;
    }
}

}  // namespace ragrt

extern "C" int ragrt_centroid_pass_counts(ragrt_index* ix, uint32_t mask, int64_t* d_pass, int64_t* d_total,
                                          void* stream) {
    RAGRT_REQUIRE(ix && d_pass, "null argument");
    int rc = check_device(ix);
    if (rc) return rc;
    const int NC = ix->d.num_centroids;
    k_centroid_pass_counts<<<(unsigned)ceil_div((int64_t)NC * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        ix->d.csr_packed_24, ix->d.doc_predicates, ix->cstart, ix->clists, ix->d.csr_row_ptrs, ix->list_off, NC,
        mask, d_pass, d_total);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}
