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
//   s3_prep   (a CTA per query) sorts the kept (centroid, token, v) triples by centroid and
//             writes the query's distinct lists, each with its (token, v) pairs; it also counts
//             the diagnostic statistics (postings of every kept probe, distinct postings, kept
//             probes, tasks).
//   s3_walk   (persistent CTAs; a work item is one query and a block of pid ranges) splits each
//             CTA into independent teams of warps.  A team walks one pid range at a time: each
//             distinct list's sub-list in the range once, coalesced.  A touched passage gets a
//             row of 32 per-token maxima (fp16 bits, 16-bit compare-and-swap maximum: positive
//             fp16 values order like their bits) in the team's shared-memory hash table, keyed
//             by pid; every posting applies its list's (token, v) pairs to that row.  At the
//             end of the range each row's 32 maxima are summed exactly (fixed point, 2^-24
//             units), rounded once to fp32 and emitted as a ranking key into the query's pool,
//             as the per-token kernel does.  A range that touches more passages than the table
//             holds is pushed to a queue and handled by the per-token kernel (s3_accumulate in
//             queue mode), which needs no per-passage rows.  Teams synchronise on their own
//             named barrier only, so a range's short phases do not hold up the whole CTA.
//
// Both kernels produce bit-identical sums (the per-(passage, token) maximum is order-free and the
// sum is exact), so the split between them never changes a result.
#include <algorithm>

#include "common.cuh"
#include "index.cuh"
#include "s3_common.cuh"

namespace ragrt {

constexpr int kPrepThreads = 512;
constexpr int kTeamWarps = 4;            // warps of a team: one walk range at a time, own hash table
constexpr int kWalkTeams = 2;
constexpr int kWalkWarps = kWalkTeams * kTeamWarps;
constexpr int kWalkThreads = kWalkWarps * 32;
constexpr int kBatch = 2;                // 32-entry chunks whose pid loads a warp issues together
constexpr int kUnit = 32 * kBatch;       // entries of one list group per work unit of a warp
constexpr uint32_t kEmpty = 0xFFFFFFFFu;

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
    int LM;                          // list / pair capacity per query (rows * kc)
    int32_t* nl;                     // [nq]
    int32_t* lc;                     // [nq][LM] centroid of list j
    int32_t* lpc;                    // [nq][LM] postings of list j (its first n_eids chunk lists)
    int32_t* lpo;                    // [nq][LM + 1] first pair of list j
    uint32_t* pairs;                 // [nq][LM] (token << 16) | fp16 bits of v, grouped by list
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
    // each thread owns a contiguous run of the sorted keys; list starts are where c changes
    const int per = (P + blockDim.x - 1) / blockDim.x;
    const int i0 = threadIdx.x * per, i1 = min(P, i0 + per);
    int starts = 0;
    for (int i = i0; i < i1; ++i)
        if (pk[i] != ~0ull && (i == 0 || (pk[i] >> 32) != (pk[i - 1] >> 32))) ++starts;
    int nlists = 0;
    int j = cta_excl_scan(starts, s_scan, &nlists);
    unsigned long long st_post = 0, st_dist = 0, st_tasks = 0, st_probes = 0;
    int32_t* lc = p.lc + (int64_t)qi * p.LM;
    int32_t* lpc = p.lpc + (int64_t)qi * p.LM;
    int32_t* lpo = p.lpo + (int64_t)qi * (p.LM + 1);
    uint32_t* pairs = p.pairs + (int64_t)qi * p.LM;
    int last = -1;
    for (int i = i0; i < i1; ++i) {
        const uint64_t k = pk[i];
        if (k == ~0ull) {
            if (i == 0 || pk[i - 1] != ~0ull) lpo[nlists] = i;          // end of the last list
            break;
        }
        const int c = (int)(k >> 32);
        pairs[i] = (uint32_t)(k & 0xFFFFFFFFu);
        const int nle = min(p.clists[c], p.n_eids);
        const int64_t cnt = nle > 0 ? p.list_off[p.rp[c] + nle] - p.cstart[c] : 0;
        ++st_probes;
        st_tasks += (unsigned long long)max(nle, 0);
        st_post += (unsigned long long)cnt;
        if (i == 0 || (pk[i - 1] >> 32) != (uint64_t)(uint32_t)c) {
            lc[j] = c;
            lpc[j] = (int32_t)cnt;
            lpo[j] = i;
            ++j;
            st_dist += (unsigned long long)cnt;
        }
        last = i;
    }
    // a run of kept keys that fills P exactly has no sentinel after it
    if (last == P - 1) lpo[nlists] = P;
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

// ------------------------------------------------------------------ the walk
struct S3WalkParams {
    const uint8_t* packed;
    const uint32_t* preds;
    const uint32_t* boff;
    const int64_t* cstart;
    int N, R, w_shift;
    int m;                           // index ranges per walk range
    int RP;                          // walk ranges: ceil(R / m)
    const int32_t* nl;
    const int32_t* lc;
    const int32_t* lpc;
    const int32_t* lpo;
    const uint32_t* pairs;
    int LM;
    const uint32_t* masks;
    int q0, nq;
    int rpj;                         // walk ranges per work item
    int rcap_log2;                   // hash rows per team: 1 << rcap_log2
    uint64_t* pool;
    int64_t pool_cap;
    unsigned long long* pool_count;  // [nq]
    unsigned int* work;
    unsigned long long* dense;       // deferred (qi << 32 | walk range)
    unsigned int* dense_count;
    unsigned long long* stats;       // [7] += deferred range blocks
};

// Shared memory: the work item's query (its distinct lists, read by both teams), then one
// block per team: its hash rows (32 per-token maxima as fp16 bits; token t of row h at column
// t ^ (h & 31)), the rows' keys (pid - range_lo, or kEmpty) and its list groups' entry counts.
__host__ __device__ inline size_t align128(size_t x) { return (x + 127) & ~(size_t)127; }
__host__ __device__ inline size_t walk_query_bytes(int LM) {
    return align128(sizeof(int64_t) * LM + 3 * sizeof(int32_t) * LM + sizeof(int32_t) * (LM + 1));
}
__host__ __device__ inline size_t walk_team_bytes(int LM, int rcap) {
    return align128(sizeof(uint16_t) * (size_t)rcap * 32 + sizeof(uint32_t) * rcap + sizeof(int32_t) * (LM / 32 + 2));
}
__host__ __device__ inline size_t walk_smem_bytes(int LM, int rcap) {
    return walk_query_bytes(LM) + kWalkTeams * walk_team_bytes(LM, rcap);
}

__device__ __forceinline__ void team_sync(int team) {
    asm volatile("bar.sync %0, %1;" ::"r"(team + 1), "r"(kTeamWarps * 32) : "memory");
}

// per-token maximum of positive fp16 bits in a 16-bit slot (fp16 order = bit order for v >= 0)
__device__ __forceinline__ void max16(uint16_t* a, uint16_t v) {
    unsigned short old = *(volatile unsigned short*)a;
    while (v > old) {
        const unsigned short prev = atomicCAS(reinterpret_cast<unsigned short*>(a), old, (unsigned short)v);
        if (prev == old) break;
        old = prev;
    }
}

__global__ void __launch_bounds__(kWalkThreads, 2)
s3_walk(S3WalkParams p) {
    extern __shared__ __align__(16) unsigned char walk_smem[];
    const int rcap = 1 << p.rcap_log2;
    const int LM = p.LM;
    int64_t* lcs = reinterpret_cast<int64_t*>(walk_smem);                 // [LM] cstart of list j
    int32_t* lcx = reinterpret_cast<int32_t*>(lcs + LM);                  // [LM] centroid
    int32_t* lpcx = lcx + LM;                                              // [LM] postings
    uint32_t* pairsx = reinterpret_cast<uint32_t*>(lpcx + LM);            // [LM]
    int32_t* lpox = reinterpret_cast<int32_t*>(pairsx + LM);              // [LM + 1]
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int team = w / kTeamWarps, tw = w % kTeamWarps, tt = tid % (kTeamWarps * 32);
    unsigned char* tbase = walk_smem + walk_query_bytes(LM) + (size_t)team * walk_team_bytes(LM, rcap);
    uint16_t* rows = reinterpret_cast<uint16_t*>(tbase);                  // [rcap][32]
    uint32_t* keys = reinterpret_cast<uint32_t*>(rows + (size_t)rcap * 32);
    int32_t* gtot = reinterpret_cast<int32_t*>(keys + rcap);              // [LM / 32 + 1]

    __shared__ unsigned s_job, s_rctr;
    __shared__ int s_nl;
    __shared__ int s_trange[kWalkTeams];
    __shared__ unsigned s_nkeys[kWalkTeams];
    __shared__ int s_overflow[kWalkTeams];
    __shared__ unsigned s_wcnt[kWalkTeams][kTeamWarps];
    __shared__ unsigned long long s_base[kWalkTeams];
    __shared__ uint32_t s_slots[kWalkWarps][32];      // emission: the warp's occupied slots in order

    for (int i = tt; i < rcap * 16; i += kTeamWarps * 32) reinterpret_cast<uint32_t*>(rows)[i] = 0u;
    for (int i = tt; i < rcap; i += kTeamWarps * 32) keys[i] = kEmpty;
    if (tt == 0) { s_nkeys[team] = 0; s_overflow[team] = 0; }
    const unsigned nrb = ((unsigned)p.RP + p.rpj - 1) / p.rpj;
    const unsigned total_jobs = (unsigned)p.nq * nrb;
    const unsigned max_keys = (unsigned)(rcap - (rcap >> 2) - (rcap >> 3));   // 5/8 load
    int cached_q = -1;
    __syncthreads();

    for (;;) {
        if (tid == 0) {
            s_job = atomicAdd(p.work, 1u);
            s_rctr = 0;
        }
        __syncthreads();
        const unsigned job = s_job;
        if (job >= total_jobs) break;
        const int qi = (int)(job / nrb);
        const int rp0 = (int)(job % nrb) * p.rpj, rp1 = min(p.RP, rp0 + p.rpj);
        if (qi != cached_q) {
            const int nl = p.nl[qi];
            const int32_t* lc = p.lc + (int64_t)qi * LM;
            const int32_t* lpc = p.lpc + (int64_t)qi * LM;
            const int32_t* lpo = p.lpo + (int64_t)qi * (LM + 1);
            for (int j = tid; j < nl; j += kWalkThreads) {
                const int c = lc[j];
                lcx[j] = c;
                lpcx[j] = lpc[j];
                lcs[j] = p.cstart[c];
            }
            for (int j = tid; j <= nl; j += kWalkThreads) lpox[j] = lpo[j];
            const int np = nl ? lpo[nl] : 0;
            const uint32_t* pr = p.pairs + (int64_t)qi * LM;
            for (int k = tid; k < np; k += kWalkThreads) pairsx[k] = pr[k];
            if (tid == 0) s_nl = nl;
            cached_q = qi;
            __syncthreads();
        }
        const int nl = s_nl;
        const int ngroups = (nl + 31) >> 5;
        const uint32_t mask = p.masks ? p.masks[p.q0 + qi] : 0u;

        // the teams take the work item's walk ranges one at a time
        for (;;) {
            if (tt == 0) s_trange[team] = rp0 + (int)atomicAdd(&s_rctr, 1u);
            team_sync(team);
            const int rpi = s_trange[team];
            if (rpi >= rp1) break;                                            // team-uniform
            const int r = rpi * p.m, rend = min(p.R, r + p.m);
            const int64_t range_lo = (int64_t)r << p.w_shift;
            const int64_t range_w = ((int64_t)(rend - r)) << p.w_shift;

            // ---- 1. entries per group of 32 lists: the lists' sub-lists inside the range
            for (int g = tw; g < ngroups; g += kTeamWarps) {
                const int j = 32 * g + lane;
                int len = 0;
                if (j < nl) {
                    const uint32_t* bo = p.boff + (int64_t)lcx[j] * (p.R + 1);
                    const int64_t hi = min((int64_t)bo[rend], (int64_t)lpcx[j]);
                    len = (int)(hi - min((int64_t)bo[r], hi));
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) len += __shfl_xor_sync(0xFFFFFFFFu, len, o);
                if (lane == 0) gtot[g] = len;
            }
            team_sync(team);

            // ---- 2. walk: the team's warps take units of kUnit consecutive entries of a group
            int ubase = 0;
            for (int g = 0; g < ngroups; ++g) {
                const int tg = gtot[g];
                const int ug = (tg + kUnit - 1) / kUnit;
                const int k0 = ((tw - ubase) % kTeamWarps + kTeamWarps) % kTeamWarps;
                ubase += ug;
                if (k0 >= ug) continue;                                       // warp-uniform
                // this warp's view of the group: lane = list, its sub-list and exclusive prefix
                const int j = 32 * g + lane;
                int len = 0;
                int64_t start = 0;
                if (j < nl) {
                    const uint32_t* bo = p.boff + (int64_t)lcx[j] * (p.R + 1);
                    const int64_t hi = min((int64_t)bo[rend], (int64_t)lpcx[j]);
                    const int64_t lo = min((int64_t)bo[r], hi);
                    len = (int)(hi - lo);
                    start = lcs[j] + lo;
                }
                int incl = len;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                    if (lane >= o) incl += y;
                }
                const int excl = j < nl ? incl - len : tg;                    // past the lists: never chosen
                const int64_t sbase = start - excl;                           // posting of entry e: sbase + e
                for (int k = k0; k < ug; k += kTeamWarps) {
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
                            if (pid[b] >= 0 && pid[b] < p.N && !(p.preds[pid[b]] & mask)) pid[b] = -1;  // :387
                    }
#pragma unroll
                    for (int b = 0; b < kBatch; ++b) {
                        if (e_beg + 32 * b >= e_end) break;                   // warp-uniform
                        const int64_t pl64 = (int64_t)pid[b] - range_lo;
                        const bool ok = pid[b] >= 0 && pl64 >= 0 && pl64 < range_w &&
                                        !*(volatile int*)&s_overflow[team];
                        int row = -1;
                        bool fresh = false;
                        if (ok) {
                            const uint32_t pl = (uint32_t)pl64;
                            uint32_t h = (pl * 0x9E3779B1u) >> (32 - p.rcap_log2);
                            for (int probe = 0; probe < rcap; ++probe) {
                                const uint32_t old = atomicCAS(&keys[h], kEmpty, pl);
                                if (old == kEmpty || old == pl) {
                                    row = (int)h;
                                    fresh = old == kEmpty;
                                    break;
                                }
                                h = (h + 1) & (uint32_t)(rcap - 1);
                            }
                            if (row < 0) s_overflow[team] = 1;
                        }
                        const unsigned nf = __ballot_sync(0xFFFFFFFFu, fresh);
                        if (nf && lane == 0) {
                            const unsigned before = atomicAdd(&s_nkeys[team], (unsigned)__popc(nf));
                            if (before + __popc(nf) > max_keys) s_overflow[team] = 1;
                        }
                        if (row >= 0) {
                            const int js = src[b];
                            const int a0 = lpox[js], a1 = lpox[js + 1];
                            uint16_t* rw = rows + (size_t)row * 32;
                            const int sw = row & 31;
                            for (int a = a0; a < a1; ++a) {
                                const uint32_t tv = pairsx[a];
                                max16(rw + ((tv >> 16) ^ sw), (uint16_t)(tv & 0xFFFFu));
                            }
                        }
                    }
                }
            }
            team_sync(team);

            // ---- 3. emit every touched passage's exact sum, or defer the range
            const int per_w = rcap / kTeamWarps;
            if (s_overflow[team]) {
                for (int i = tt; i < rcap; i += kTeamWarps * 32) {
                    if (keys[i] != kEmpty) {
                        uint4* rr = reinterpret_cast<uint4*>(rows + (size_t)i * 32);
#pragma unroll
                        for (int x = 0; x < 4; ++x) rr[x] = make_uint4(0u, 0u, 0u, 0u);
                        keys[i] = kEmpty;
                    }
                }
                if (tt == 0) {
                    const unsigned pos = atomicAdd(p.dense_count, 1u);
                    p.dense[pos] = ((unsigned long long)qi << 32) | (unsigned)rpi;
                    if (p.stats) atomicAdd(&p.stats[7], 1ull);
                }
            } else {
                unsigned cnt = 0;
                for (int i0 = 0; i0 < per_w; i0 += 32)
                    cnt += __popc(__ballot_sync(0xFFFFFFFFu,
                                                i0 + lane < per_w && keys[tw * per_w + i0 + lane] != kEmpty));
                if (lane == 0) s_wcnt[team][tw] = cnt;
                team_sync(team);
                if (tt == 0) {
                    unsigned t = 0;
                    for (int i = 0; i < kTeamWarps; ++i) { const unsigned c = s_wcnt[team][i]; s_wcnt[team][i] = t; t += c; }
                    s_base[team] = t ? atomicAdd(&p.pool_count[qi], (unsigned long long)t) : 0ull;
                }
                team_sync(team);
                uint64_t* pool = p.pool + (int64_t)qi * p.pool_cap + s_base[team] + s_wcnt[team][tw];
                unsigned done = 0;
                for (int i0 = 0; i0 < per_w; i0 += 32) {
                    const int slot = tw * per_w + i0 + lane;
                    const bool occ = i0 + lane < per_w && keys[slot] != kEmpty;
                    const unsigned mk = __ballot_sync(0xFFFFFFFFu, occ);
                    if (occ) s_slots[w][__popc(mk & ((1u << lane) - 1u))] = (uint32_t)slot;
                    __syncwarp();
                    const int n = __popc(mk);
                    for (int r0 = 0; r0 < n; r0 += 8) {                     // 4 lanes per row
                        const int ri = r0 + (lane >> 2), qd = lane & 3;
                        unsigned long long sum = 0;
                        int sl = 0;
                        if (ri < n) {
                            sl = (int)s_slots[w][ri];
                            uint4* rr = reinterpret_cast<uint4*>(rows + (size_t)sl * 32 + qd * 8);
                            const uint4 a = rr[0];
                            sum = h_fixed24((uint16_t)a.x) + h_fixed24((uint16_t)(a.x >> 16)) +
                                  h_fixed24((uint16_t)a.y) + h_fixed24((uint16_t)(a.y >> 16)) +
                                  h_fixed24((uint16_t)a.z) + h_fixed24((uint16_t)(a.z >> 16)) +
                                  h_fixed24((uint16_t)a.w) + h_fixed24((uint16_t)(a.w >> 16));
                            rr[0] = make_uint4(0u, 0u, 0u, 0u);
                        }
                        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
                        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
                        if (ri < n && qd == 0) {
                            const float sc = __ull2float_rn(sum) * 0x1p-24f;
                            pool[done + ri] = rank_key(sc, (int32_t)(range_lo + keys[sl]));
                            keys[sl] = kEmpty;
                        }
                    }
                    done += n;
                    __syncwarp();
                }
            }
            if (tt == 0) { s_nkeys[team] = 0; s_overflow[team] = 0; }
            team_sync(team);
        }
        __syncthreads();                                                      // the item is done
    }
}

// every (query, range block) into the per-token kernel's queue (Stage-3 mode 1)
__global__ void s3_queue_all(int nq, int RP, unsigned long long* dense, unsigned int* dense_count) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (int64_t)nq * RP) dense[i] = ((unsigned long long)(i / RP) << 32) | (unsigned)(i % RP);
    if (i == 0) *dense_count = (unsigned)((int64_t)nq * RP);
}

// ------------------------------------------------------------------ host side
size_t s3_walk_lists_bytes(int nq, int LM) {
    return sizeof(int32_t) * (size_t)nq * (1 + LM + LM + (LM + 1)) + sizeof(uint32_t) * (size_t)nq * LM + 1024;
}

int s3_walk_ranges(const ragrt_index* ix) {
    // index ranges per walk range: one by default (4,096 passages on the benchmark corpus, about
    // 130 touched passages per range against the table's 320-passage limit)
    if (ix->s3_range > 0) return std::max(1, ix->s3_range >> ix->w_shift);
    return 1;
}

size_t s3_walk_dense_bytes(const ragrt_index* ix, int nq) {
    return sizeof(unsigned long long) * (size_t)nq * ceil_div(ix->num_ranges, 1) + 256;
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
    int32_t* lpo = lpc + (size_t)nq * LM;
    uint32_t* pairs = (uint32_t*)(lpo + (size_t)nq * (LM + 1));

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
    pp.lpo = lpo;
    pp.pairs = pairs;
    pp.stats = ix->stats;
    const size_t psmem = sizeof(uint64_t) * next_pow2(LM);
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s3_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem));
    s3_prep<<<nq, kPrepThreads, psmem, stream>>>(pp);
    RAGRT_LAUNCH_CHECK();

    const int m = s3_walk_ranges(ix);
    const int RP = (int)ceil_div(ix->num_ranges, m);
    int rcap_log2 = 9;
    while (rcap_log2 > 8 && walk_smem_bytes(LM, 1 << rcap_log2) > 227 * 1024) --rcap_log2;
    const bool fits = walk_smem_bytes(LM, 1 << rcap_log2) <= 227 * 1024;
    if (ix->s3_mode == 1 || !fits) {     // per-token only: queue every range block for s3_accumulate
        s3_queue_all<<<(unsigned)ceil_div((int64_t)nq * RP, 256), 256, 0, stream>>>(nq, RP, dense, dense_count);
        RAGRT_LAUNCH_CHECK();
        return RAGRT_OK;
    }

    S3WalkParams p;
    p.packed = ix->d.csr_packed_24;
    p.preds = ix->d.doc_predicates;
    p.boff = ix->boff;
    p.cstart = ix->cstart;
    p.N = ix->d.num_passages;
    p.R = ix->num_ranges;
    p.w_shift = ix->w_shift;
    p.m = m;
    p.RP = RP;
    p.nl = nl;
    p.lc = lc;
    p.lpc = lpc;
    p.lpo = lpo;
    p.pairs = pairs;
    p.LM = LM;
    p.masks = ix->d.doc_predicates ? masks : nullptr;
    p.q0 = q0;
    p.nq = nq;
    p.rcap_log2 = rcap_log2;
    p.pool = pool;
    p.pool_cap = ix->d.num_passages;
    p.pool_count = pool_count;
    p.work = work;
    p.dense = dense;
    p.dense_count = dense_count;
    p.stats = ix->stats;
    const size_t smem = walk_smem_bytes(LM, 1 << p.rcap_log2);
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s3_walk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    RAGRT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, s3_walk, kWalkThreads, smem));
    per_sm = std::max(1, per_sm);
    const int64_t ctas = (int64_t)per_sm * num_sms();
    int rpj = 16;
    while (rpj > 2 && (int64_t)nq * ((p.RP + rpj - 1) / rpj) < 8 * ctas) rpj >>= 1;
    p.rpj = rpj;
    const int64_t jobs = (int64_t)nq * ((p.RP + rpj - 1) / rpj);
    const int grid = (int)std::min<int64_t>(jobs, ctas);
    s3_walk<<<grid, kWalkThreads, smem, stream>>>(p);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
