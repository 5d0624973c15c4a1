// s3_walk.cu -- Stages 1-3 with every distinct probed posting list walked once per query.
//
// Semantics (the reference's `weft` mode: all-codewords Stage 1, codeword weight 0): for query
// token t and probed centroid c with base score b_tc > 0 (MIN_BASE_SCORE), every posting pid of
// c's first n_eids chunk lists contributes v_tc = fp16(b_tc) to (pid, t); a passage's score is
// the sum over tokens of the per-token maximum.  Reference: ragrt_fused_kernel.cu:187-213
// (task collection, base > 0), :343-392 (expand, filter :387, fp16 key :366), :403-431 +
// :1120-1156 (max per (pid, token), sum per pid).
//
// A query's 32 tokens x nprobe probes name far fewer distinct lists (the tokens of one query
// share topics: about 1,000 kept probes but 250 distinct lists on the benchmark corpus), so
// walking per (token, probe) reads every list about four times.  Here:
//
//   s3_prep    (a CTA per query) sorts the kept (centroid, token, v) triples by centroid and
//              writes the query's distinct lists, each with its row of 32 per-token values
//              (fp16 bits, 0 for a token that did not probe the list); it also counts the
//              diagnostic statistics (postings of every kept probe, distinct postings, kept
//              probes, tasks).
//   s3_bucket  (persistent CTAs, five per SM; a work item is one query and a block of pid
//              ranges) takes one pid range at a time and
//                A. finds each distinct list's sub-list inside the range (the index's
//                   range-offset table) and their prefix: the range's entries;
//                B. walks the entries once, coalesced (units of three 32-entry chunks per
//                   warp); an entry (passage, list) takes the next
//                   slot of its passage (a 16-bit counter per passage, two per shared word), and
//                   the entry that takes slot 0 records the passage as touched;
//                C. scans the touched passages' counts into their offsets;
//                D. files every entry's list under its passage (a counting sort);
//                E. gives each touched passage four lanes, 8 tokens each, which max-reduce the
//                   value rows of the passage's lists with 16-byte loads (from global memory,
//                   through L1 / L2), then sum the 32 maxima exactly (fp64), round once to fp32
//                   and emit the ranking key into the query's pool, as the per-token kernel does.
//              The two CTA scans of a range alternate scratch buffers, and the counter reset
//              needs no barrier of its own: eight barriers per range.
//              A range whose entries or touched passages exceed the staging area is pushed to a
//              queue and handled by the per-token kernel (s3_accumulate in queue mode), which has
//              no such limit.
//
// Both kernels produce bit-identical sums (the per-(passage, token) maximum is order-free and the
// sum is exact), so the split between them never changes a result.
#include <algorithm>

#include "common.cuh"
#include "index.cuh"
#include "s3_common.cuh"

namespace ragrt {

constexpr int kPrepThreads = 512;
constexpr int kBkWarps = 8;
constexpr int kBkThreads = kBkWarps * 32;
constexpr int kBkMaxW = 4096;             // passages per pid range (12-bit local pids)
constexpr int kBkMaxLists = 1024;         // distinct lists per query (10-bit list ids)
constexpr int kBkStage = 3072;            // entries per range held in shared memory
constexpr int kBkTouched = 1024;          // touched passages per range held in shared memory
constexpr int kBatch = 3;                 // 32-entry chunks whose pid loads a warp issues together
constexpr int kUnit = 32 * kBatch;        // entries of one list group per work unit of a warp
constexpr uint32_t kNoEntry = 0xFFFFFFFFu;

__device__ __forceinline__ uint16_t s3_v15(float base) {
    return (uint16_t)(__half_as_ushort(__float2half_rn(base)) & 0x7FFF);   // ragrt_fused_kernel.cu:366
}

// Exclusive scan of one int per thread over the CTA; returns the thread's exclusive prefix and
// writes the total to *total.  `s` holds 33 ints.
__device__ __forceinline__ int cta_excl_scan(int v, int* s, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s[w] = incl;
    __syncthreads();
    if (w == 0) {
        int x = lane < nw ? s[lane] : 0;
        int xi = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, xi, o);
            if (lane >= o) xi += y;
        }
        s[lane] = xi - x;
        if (lane == 31) s[32] = xi;
    }
    __syncthreads();
    const int r = s[w] + incl - v;
    *total = s[32];
    __syncthreads();
    return r;
}

// The same scan without its trailing barrier: `s` must not be written by another scan until every
// thread has passed a later barrier (the walk alternates two scratch buffers).
__device__ __forceinline__ int cta_excl_scan_open(int v, int* s, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s[w] = incl;
    __syncthreads();
    if (w == 0) {
        int x = lane < nw ? s[lane] : 0;
        int xi = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, xi, o);
            if (lane >= o) xi += y;
        }
        s[lane] = xi - x;
        if (lane == 31) s[32] = xi;
    }
    __syncthreads();
    *total = s[32];
    return s[w] + incl - v;
}

// ------------------------------------------------------------------ per-query distinct lists
struct S3PrepParams {
    const int32_t* topc;
    const float* scores;
    int full_scores, rows, kc, NC;
    const int32_t* ntok;
    int q0;
    const int32_t* clists;
    const int64_t* cstart;
    const int64_t* rp;
    const int64_t* list_off;
    int n_eids;
    int LM;                          // list capacity per query (rows * kc)
    int32_t* nl;                     // [nq]
    int32_t* lc;                     // [nq][LM] centroid of list j
    int32_t* lpc;                    // [nq][LM] postings of list j (its first n_eids chunk lists)
    uint16_t* val;                   // [nq][LM][32] value of token t for list j (fp16 bits; 0: not probed)
    unsigned long long* stats;
};

__global__ void __launch_bounds__(kPrepThreads)
s3_prep(S3PrepParams p) {
    extern __shared__ uint64_t pk[];             // [next_pow2(rows * kc)]
    __shared__ int s_scan[33];
    const int qi = blockIdx.x, q = p.q0 + qi;
    const int nt = p.ntok ? min(p.ntok[q], p.rows) : p.rows;
    const int n = p.rows * p.kc, P = next_pow2(n);
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        uint64_t key = ~0ull;
        if (i < n) {
            const int t = i / p.kc, j = i % p.kc;
            if (t < nt) {
                const int c = p.topc[((int64_t)q * p.rows + t) * p.kc + j];
                if (c >= 0 && c < p.NC) {
                    const float base = p.full_scores ? p.scores[((int64_t)q * p.rows + t) * p.NC + c]
                                                     : p.scores[((int64_t)q * p.rows + t) * p.kc + j];
                    if (base > 0.0f)                                     // MIN_BASE_SCORE
                        key = ((uint64_t)(uint32_t)c << 32) | ((uint64_t)t << 16) | s3_v15(base);
                }
            }
        }
        pk[i] = key;
    }
    __syncthreads();
    cta_bitonic_sort<false>(pk, P);
    // each thread owns a contiguous run of the sorted keys; lists start where the centroid changes
    const int per = (P + blockDim.x - 1) / blockDim.x;
    const int i0 = threadIdx.x * per, i1 = min(P, i0 + per);
    int starts = 0;
    for (int i = i0; i < i1; ++i)
        if (pk[i] != ~0ull && (i == 0 || (pk[i] >> 32) != (pk[i - 1] >> 32))) ++starts;
    int nlists = 0;
    const int j0 = cta_excl_scan(starts, s_scan, &nlists);
    int32_t* lc = p.lc + (int64_t)qi * p.LM;
    int32_t* lpc = p.lpc + (int64_t)qi * p.LM;
    uint16_t* val = p.val + (int64_t)qi * p.LM * 32;
    for (int i = threadIdx.x; i < nlists * 16; i += blockDim.x) reinterpret_cast<uint32_t*>(val)[i] = 0u;
    __syncthreads();
    unsigned long long st_post = 0, st_dist = 0, st_tasks = 0, st_probes = 0;
    int j = j0 - 1;                       // list of the previous key (this run may start inside one)
    for (int i = i0; i < i1; ++i) {
        const uint64_t k = pk[i];
        if (k == ~0ull) break;
        const int c = (int)(k >> 32);
        const int nle = min(p.clists[c], p.n_eids);
        const int64_t cnt = nle > 0 ? p.list_off[p.rp[c] + nle] - p.cstart[c] : 0;
        if (i == 0 || (pk[i - 1] >> 32) != (uint64_t)(uint32_t)c) {
            ++j;
            lc[j] = c;
            lpc[j] = (int32_t)cnt;
            st_dist += (unsigned long long)cnt;
        }
        val[(int64_t)j * 32 + ((k >> 16) & 31)] = (uint16_t)(k & 0xFFFFu);
        ++st_probes;
        st_tasks += (unsigned long long)max(nle, 0);
        st_post += (unsigned long long)cnt;
    }
    if (threadIdx.x == 0) p.nl[qi] = nlists;
    if (p.stats) {
        for (int o = 16; o; o >>= 1) {
            st_post += __shfl_xor_sync(0xFFFFFFFFu, st_post, o);
            st_dist += __shfl_xor_sync(0xFFFFFFFFu, st_dist, o);
            st_tasks += __shfl_xor_sync(0xFFFFFFFFu, st_tasks, o);
            st_probes += __shfl_xor_sync(0xFFFFFFFFu, st_probes, o);
        }
        if ((threadIdx.x & 31) == 0 && st_probes) {
            atomicAdd(&p.stats[1], st_post);
            atomicAdd(&p.stats[2], st_dist);
            atomicAdd(&p.stats[4], st_probes);
            atomicAdd(&p.stats[6], st_tasks);
        }
    }
}

// ------------------------------------------------------------------ the bucketed walk
struct S3BucketParams {
    const uint8_t* packed;
    const uint32_t* preds;
    const uint32_t* boff;
    const int64_t* cstart;
    int N, R, w_shift;
    const int32_t* nl;
    const int32_t* lc;
    const int32_t* lpc;
    const uint16_t* val;
    int LM;
    const uint32_t* masks;
    int q0, nq;
    int rpj;                         // pid ranges per work item
    uint64_t* pool;
    int64_t pool_cap;
    unsigned long long* pool_count;  // [nq]
    unsigned int* work;
    unsigned long long* dense;       // deferred (qi << 32 | range)
    unsigned int* dense_count;
    unsigned long long* stats;       // [7] += deferred ranges
};

__host__ __device__ inline size_t align128(size_t x) { return (x + 127) & ~(size_t)127; }
// shared memory: counters [W/2] u32 | staging [kBkStage] u32 | filed lists [kBkStage] u16 |
// touched passages [kBkTouched] u16 | their first slot [kBkTouched] u16 | per list: first
// posting in the range [LM] i64, entry prefix [LM + 1] i32: 43 KB at LM = 1,024, five CTAs per
// SM.  The value rows and the lists' centroids and lengths stay in global memory, read through
// L1 / L2: holding them in shared memory costs CTAs per SM, and the walk is bound by how many
// warps are resident, not by those reads.
__host__ __device__ inline size_t bucket_smem_bytes(int LM) {
    return align128(4 * (kBkMaxW / 2)) + align128(4 * kBkStage) + align128(2 * kBkStage) + 2 * align128(2 * kBkTouched) +
           align128(8 * (size_t)LM) + align128(4 * (size_t)(LM + 1));
}

constexpr int kBkCtasPerSm = 5;           // at most 51 registers per thread (48 used)
__global__ void __launch_bounds__(kBkThreads, kBkCtasPerSm)
s3_bucket(S3BucketParams p) {
    extern __shared__ __align__(128) unsigned char bk_smem[];
    const int LM = p.LM;
    unsigned char* sp = bk_smem;
    uint32_t* cnt = reinterpret_cast<uint32_t*>(sp);    sp += align128(4 * (kBkMaxW / 2));
    uint32_t* stg = reinterpret_cast<uint32_t*>(sp);    sp += align128(4 * kBkStage);
    uint16_t* srt = reinterpret_cast<uint16_t*>(sp);    sp += align128(2 * kBkStage);
    uint16_t* tpp = reinterpret_cast<uint16_t*>(sp);    sp += align128(2 * kBkTouched);
    uint16_t* tpo = reinterpret_cast<uint16_t*>(sp);    sp += align128(2 * kBkTouched);
    int64_t* segs = reinterpret_cast<int64_t*>(sp);     sp += align128(8 * (size_t)LM);
    int32_t* segpre = reinterpret_cast<int32_t*>(sp);
    __shared__ int s_scan2[2][33];          // A's and C's scans alternate buffers
    __shared__ unsigned s_job;
    __shared__ int s_nl, s_valid;
    __shared__ unsigned s_touched;
    __shared__ unsigned long long s_base;

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int W = 1 << p.w_shift;
    uint16_t* cnt16 = reinterpret_cast<uint16_t*>(cnt);
    for (int i = tid; i < (W >> 1); i += kBkThreads) cnt[i] = 0u;
    if (tid == 0) s_touched = 0;
    const unsigned nrb = ((unsigned)p.R + p.rpj - 1) / p.rpj;
    const unsigned total_jobs = (unsigned)p.nq * nrb;
    int cached_q = -1;
    __syncthreads();

    for (;;) {
        if (tid == 0) s_job = atomicAdd(p.work, 1u);
        __syncthreads();
        const unsigned job = s_job;
        if (job >= total_jobs) break;
        const int qi = (int)(job / nrb);
        const int r0 = (int)(job % nrb) * p.rpj, r1 = min(p.R, r0 + p.rpj);
        if (qi != cached_q) {
            if (tid == 0) s_nl = p.nl[qi];
            cached_q = qi;
            __syncthreads();
        }
        // the query's lists: centroid and postings, read through L1 by phase A of each range
        const int32_t* lcx = p.lc + (int64_t)qi * LM;
        const int32_t* lpcx = p.lpc + (int64_t)qi * LM;
        const int nl = s_nl;
        const int ngroups = (nl + 31) >> 5;
        const uint32_t mask = p.masks ? p.masks[p.q0 + qi] : 0u;
        const uint4* qval = reinterpret_cast<const uint4*>(p.val + (int64_t)qi * LM * 32);

        for (int r = r0; r < r1; ++r) {
            const int64_t range_lo = (int64_t)r << p.w_shift;

            // ---- A. each list's sub-list inside the range; entry prefix over the lists
            const int per = (nl + kBkThreads - 1) / kBkThreads;
            const int ja = tid * per, jb = min(nl, ja + per);
            int mylen = 0;
            for (int j = ja; j < jb; ++j) {
                const uint32_t* bo = p.boff + (int64_t)lcx[j] * (p.R + 1);
                const int64_t hi = min((int64_t)bo[r + 1], (int64_t)lpcx[j]);
                const int64_t lo = min((int64_t)bo[r], hi);
                segs[j] = p.cstart[lcx[j]] + lo;
                segpre[j] = (int)(hi - lo);                  // length for now
                mylen += (int)(hi - lo);
            }
            int total = 0;
            int run = cta_excl_scan_open(mylen, s_scan2[0], &total);
            if (tid == 0) s_touched = 0;                     // every thread is past the last range's F
            for (int j = ja; j < jb; ++j) {
                const int len = segpre[j];
                segpre[j] = run;
                run += len;
            }
            if (tid == 0) segpre[nl] = total;
            __syncthreads();
            if (total > kBkStage) {                          // too many entries: the per-token kernel
                if (tid == 0) {
                    const unsigned pos = atomicAdd(p.dense_count, 1u);
                    p.dense[pos] = ((unsigned long long)qi << 32) | (unsigned)r;
                    if (p.stats) atomicAdd(&p.stats[7], 1ull);
                }
                __syncthreads();
                continue;
            }
            if (total == 0) continue;                        // CTA-uniform

            // ---- B. walk: units of kUnit entries of one group of 32 lists, warps round robin
            {
                int ubase = 0;
                for (int g = 0; g < ngroups; ++g) {
                    const int gb = segpre[32 * g];
                    const int tg = segpre[min(nl, 32 * g + 32)] - gb;
                    const int ug = (tg + kUnit - 1) / kUnit;
                    const int k0 = ((w - ubase) % kBkWarps + kBkWarps) % kBkWarps;
                    ubase += ug;
                    if (k0 >= ug) continue;                  // warp-uniform
                    const int jl = 32 * g + lane;
                    const int excl = (jl < nl ? segpre[jl] : segpre[nl]) - gb;
                    const int64_t sbase = (jl < nl ? segs[jl] : 0) - excl;    // posting of entry e: sbase + e
                    for (int k = k0; k < ug; k += kBkWarps) {
                        const int e_beg = k * kUnit, e_end = min(tg, e_beg + kUnit);
                        int32_t pid[kBatch];
                        int src[kBatch];
#pragma unroll
                        for (int b = 0; b < kBatch; ++b) {
                            const int e = e_beg + 32 * b + lane;
                            int s = 0;
#pragma unroll
                            for (int step = 16; step; step >>= 1) {
                                const int cand = s + step;
                                const int ex = __shfl_sync(0xFFFFFFFFu, excl, cand & 31);
                                if (cand < 32 && ex <= e) s = cand;
                            }
                            const int64_t sb = __shfl_sync(0xFFFFFFFFu, sbase, s);
                            src[b] = 32 * g + s;
                            pid[b] = e < e_end ? load_pid24(p.packed, sb + e) : -1;
                        }
                        if (mask) {
#pragma unroll
                            for (int b = 0; b < kBatch; ++b)
                                if (pid[b] >= 0 && pid[b] < p.N && !(p.preds[pid[b]] & mask)) pid[b] = -2;  // :387
                        }
#pragma unroll
                        for (int b = 0; b < kBatch; ++b) {
                            const int e = e_beg + 32 * b + lane;
                            const int64_t pl = (int64_t)pid[b] - range_lo;
                            uint32_t word = kNoEntry;
                            bool first = false;
                            if (e < e_end && pid[b] >= 0 && pl >= 0 && pl < W) {
                                const int sh = 16 * ((int)pl & 1);
                                const uint32_t old = atomicAdd(&cnt[pl >> 1], 1u << sh);
                                const uint32_t slot = (old >> sh) & 0xFFFFu;
                                word = (uint32_t)pl | ((uint32_t)src[b] << 12) | (slot << 22);
                                first = slot == 0;
                            }
                            // the passages this chunk touches first: one reservation per warp
                            const unsigned fm = __ballot_sync(0xFFFFFFFFu, first);
                            unsigned tb = 0;
                            if (fm && lane == 0) tb = atomicAdd(&s_touched, (unsigned)__popc(fm));
                            tb = __shfl_sync(0xFFFFFFFFu, tb, 0);
                            const unsigned ti = tb + __popc(fm & ((1u << lane) - 1u));
                            if (first && ti < (unsigned)kBkTouched) tpp[ti] = (uint16_t)pl;
                            if (e < e_end) stg[gb + e] = word;
                        }
                    }
                }
            }
            __syncthreads();

            if (s_touched > (unsigned)kBkTouched) {          // too many passages: the per-token kernel
                for (int i = tid; i < (W >> 1); i += kBkThreads) cnt[i] = 0u;
                if (tid == 0) {
                    const unsigned pos = atomicAdd(p.dense_count, 1u);
                    p.dense[pos] = ((unsigned long long)qi << 32) | (unsigned)r;
                    if (p.stats) atomicAdd(&p.stats[7], 1ull);
                }
                __syncthreads();
                if (tid == 0) s_touched = 0;
                continue;
            }
            // ---- C. offsets of the touched passages' entries (written over their counters)
            {
                const int T = (int)s_touched;
                const int per_t = (T + kBkThreads - 1) / kBkThreads;
                const int ta = tid * per_t, tb = min(T, ta + per_t);
                int mine = 0;
                for (int i = ta; i < tb; ++i) mine += cnt16[tpp[i]];
                int valid = 0;
                int run = cta_excl_scan_open(mine, s_scan2[1], &valid);
                for (int i = ta; i < tb; ++i) {
                    const int pl = tpp[i];
                    const int c = cnt16[pl];
                    tpo[i] = (uint16_t)run;
                    cnt16[pl] = (uint16_t)run;
                    run += c;
                }
                if (tid == 0) {
                    s_valid = valid;
                    s_base = T ? atomicAdd(&p.pool_count[qi], (unsigned long long)T) : 0ull;
                }
            }
            __syncthreads();

            // ---- D. file every entry's list under its passage
            for (int e = tid; e < total; e += kBkThreads) {
                const uint32_t word = stg[e];
                if (word == kNoEntry) continue;
                const int pl = (int)(word & 0xFFFu);
                const uint32_t off = (cnt[pl >> 1] >> (16 * (pl & 1))) & 0xFFFFu;
                srt[off + (word >> 22)] = (uint16_t)((word >> 12) & 0x3FFu);
            }
            __syncthreads();

            // ---- E. per touched passage: max over its lists' value rows, exact sum, ranking key
            {
                const int T = (int)s_touched, V = s_valid;
                uint64_t* pool = p.pool + (int64_t)qi * p.pool_cap + s_base;
                const int qd = lane & 3;
                for (int t0 = w * 8; t0 < T; t0 += kBkWarps * 8) {
                    const int ti = t0 + (lane >> 2);
                    double sum = 0.0;                               // exact: 32 fp16 values need <= 45 bits
                    if (ti < T) {
                        const int a = tpo[ti], b = ti + 1 < T ? tpo[ti + 1] : V;
                        uint4 acc = make_uint4(0u, 0u, 0u, 0u);      // fp16 bits >= 0: unsigned max
                        auto vmax = [&](const uint4 v) {
                            acc.x = __vmaxu2(acc.x, v.x);
                            acc.y = __vmaxu2(acc.y, v.y);
                            acc.z = __vmaxu2(acc.z, v.z);
                            acc.w = __vmaxu2(acc.w, v.w);
                        };
                        for (int k = a; k < b; ++k) vmax(qval[(int)srt[k] * 4 + qd]);   // 8 tokens of row j at [4 j + qd]
                        const uint32_t w4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
                            sum += (double)f.x;
                            sum += (double)f.y;
                        }
                    }
                    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
                    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
                    if (ti < T && qd == 0) {
                        // the exact sum rounded once: equal to the fixed-point sum (2^-24 units) of the
                        // per-token kernel rounded to fp32
                        const float sc = __double2float_rn(sum);
                        pool[ti] = rank_key(sc, (int32_t)(range_lo + tpp[ti]));
                    }
                }
            }
            // ---- F. the touched passages' counters back to zero for the next range (ordered before
            // its walk by the barriers of its scan)
            {
                const int T = (int)s_touched;
                for (int i = tid; i < T; i += kBkThreads) cnt16[tpp[i]] = 0;
            }
        }
    }
}

// every (query, range) into the per-token kernel's queue (Stage-3 mode 1, or no room for the walk)
__global__ void s3_queue_all(int nq, int R, unsigned long long* dense, unsigned int* dense_count) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (int64_t)nq * R) dense[i] = ((unsigned long long)(i / R) << 32) | (unsigned)(i % R);
    if (i == 0) *dense_count = (unsigned)((int64_t)nq * R);
}

// ------------------------------------------------------------------ host side
size_t s3_walk_lists_bytes(int nq, int LM) {
    return sizeof(int32_t) * (size_t)nq * (1 + 2 * (size_t)LM) + sizeof(uint16_t) * (size_t)nq * LM * 32 + 1024;
}

int s3_walk_ranges(const ragrt_index*) { return 1; }

size_t s3_walk_dense_bytes(const ragrt_index* ix, int nq) {
    return sizeof(unsigned long long) * (size_t)nq * ix->num_ranges + 256;
}

int s3_walk_run(ragrt_index* ix, const int32_t* topc, const float* scores, int full_scores, const int32_t* ntok,
                int q0, int nq, int rows, int kc, int n_eids, const uint32_t* masks, uint64_t* pool,
                unsigned long long* pool_count, unsigned int* work, unsigned long long* dense,
                unsigned int* dense_count, void* lists_ws, cudaStream_t stream) {
    const int LM = rows * kc;
    char* w = (char*)lists_ws;
    int32_t* nl = (int32_t*)w;
    int32_t* lc = nl + nq;
    int32_t* lpc = lc + (size_t)nq * LM;
    uint16_t* val = (uint16_t*)(((uintptr_t)(lpc + (size_t)nq * LM) + 15) & ~(uintptr_t)15);

    S3PrepParams pp;
    pp.topc = topc;
    pp.scores = scores;
    pp.full_scores = full_scores;
    pp.rows = rows;
    pp.kc = kc;
    pp.NC = ix->d.num_centroids;
    pp.ntok = ntok;
    pp.q0 = q0;
    pp.clists = ix->clists;
    pp.cstart = ix->cstart;
    pp.rp = ix->d.csr_row_ptrs;
    pp.list_off = ix->list_off;
    pp.n_eids = n_eids;
    pp.LM = LM;
    pp.nl = nl;
    pp.lc = lc;
    pp.lpc = lpc;
    pp.val = val;
    pp.stats = ix->stats;
    const size_t psmem = sizeof(uint64_t) * next_pow2(LM);
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s3_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem));
    s3_prep<<<nq, kPrepThreads, psmem, stream>>>(pp);
    RAGRT_LAUNCH_CHECK();

    const int R = ix->num_ranges;
    const size_t smem = bucket_smem_bytes(LM);
    const bool fits = ix->w_shift <= 12 && LM <= kBkMaxLists && smem <= 227 * 1024;
    if (ix->s3_mode == 1 || !fits) {     // per-token only: queue every range for s3_accumulate
        s3_queue_all<<<(unsigned)ceil_div((int64_t)nq * R, 256), 256, 0, stream>>>(nq, R, dense, dense_count);
        RAGRT_LAUNCH_CHECK();
        return RAGRT_OK;
    }

    S3BucketParams p;
    p.packed = ix->d.csr_packed_24;
    p.preds = ix->d.doc_predicates;
    p.boff = ix->boff;
    p.cstart = ix->cstart;
    p.N = ix->d.num_passages;
    p.R = R;
    p.w_shift = ix->w_shift;
    p.nl = nl;
    p.lc = lc;
    p.lpc = lpc;
    p.val = val;
    p.LM = LM;
    p.masks = ix->d.doc_predicates ? masks : nullptr;
    p.q0 = q0;
    p.nq = nq;
    p.pool = pool;
    p.pool_cap = ix->d.num_passages;
    p.pool_count = pool_count;
    p.work = work;
    p.dense = dense;
    p.dense_count = dense_count;
    p.stats = ix->stats;
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s3_bucket, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    RAGRT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, s3_bucket, kBkThreads, smem));
    per_sm = std::max(1, per_sm);
    const int64_t ctas = (int64_t)per_sm * num_sms();
    int rpj = 8;
    while (rpj > 1 && (int64_t)nq * ((R + rpj - 1) / rpj) < 8 * ctas) rpj >>= 1;
    p.rpj = rpj;
    const int64_t jobs = (int64_t)nq * ((R + rpj - 1) / rpj);
    const int grid = (int)std::min<int64_t>(jobs, ctas);
    s3_bucket<<<grid, kBkThreads, smem, stream>>>(p);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
