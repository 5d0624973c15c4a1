/*
 * weft_oracle.c -- CPU restatement of RAGRT's plain-IVF `weft` search path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path in
 * ragrt_b200/csrc is compared against; it is never linked into the product
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs load it.
 *
 * Every stage follows the reference's algorithm; tie and rounding rules that the
 * reference leaves unspecified are fixed here (and the CUDA path implements the
 * same rules bit for bit):
 *
 *   Stage 2  centroid scores     src/weft_prep.py:32-47 (native_prep)
 *            s = Q @ C^T rounded to fp16.  The dot product is computed EXACTLY
 *            (integer arithmetic on the fp16 significands) and rounded once,
 *            round-to-nearest-even.  top-(nc+1) by (value desc, centroid asc).
 *            scores = float(v_j) - float(v_nc)  (fp32 subtraction), m = float(v_nc).
 *   Stage 3  posting aggregation src/ragrt_fused_kernel.cu:64-263 (task collection,
 *            all-codewords Stage 1 :721-742, codeword weight 0, compact scores),
 *            :343-392 (expand: 24-bit pid, filter, fp16(base) & 0x7FFF),
 *            :403-431 + :1120-1156 (per (pid, token) max, per pid sum, padding),
 *            src/optix_corr_torch_3d.cpp:569-585 (candidate top-k).
 *            Per-pid sums are exact (fixed point, units of 2^-24) rounded once to
 *            fp32.  Candidates: U <= K -> all touched pids in ascending pid order;
 *            else top-K by (sum desc, pid asc).
 *   Stage 4  TileMaxSim          src/tile_maxsim_fused_decomp.cu:125-229 and the fp32
 *            reference of tests/test_gpu_kernels.py:294-305: d = fp16 add of centroid
 *            and bucket weight, score = sum_r max_t (q_r . d_t) / |d_t|, computed in
 *            double.  pid < 0 -> -inf; an empty document -> 32 * -1e9.
 *   Final    src/optix_corr_torch_3d.cpp:596-607, ragrt_fused_kernel.cu:621-640:
 *            failing candidates -> -inf, top-k by (score desc, pid asc).
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp).  No dependency beyond libc/libm.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define NUM_SUBSPACES 32
#define BLOCK_SHIFT 7          /* ragrt_index_lib.py:28 BLOCK_SIZE = 128 */

/* ------------------------------------------------------------------ fp16 helpers */

static double h2d(uint16_t h) {
    int s = h >> 15, e = (h >> 10) & 0x1F, m = h & 0x3FF;
    double v;
    if (e == 0) v = ldexp((double)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexp((double)(m | 0x400), e - 25);
    return s ? -v : v;
}

float oracle_h2f(uint16_t h) { return (float)h2d(h); }

/* Round an exact value  a * 2^-48  (a >= 0, 128-bit) to fp16 bits, RNE. */
static uint16_t rn16_from_u128(unsigned __int128 a, int neg) {
    if (a == 0) return neg ? 0x8000 : 0;
    int msb = 127;
    while (!((a >> msb) & 1)) --msb;            /* value in [2^(msb-48), 2^(msb-47)) */
    int E = msb - 48;                           /* unbiased exponent */
    int qexp = (E - 10 > -24) ? E - 10 : -24;   /* quantum 2^qexp (subnormal floor 2^-24) */
    int s = qexp + 48;                          /* >= 24 */
    unsigned __int128 half = (unsigned __int128)1 << (s - 1);
    unsigned __int128 rem = a & (((unsigned __int128)1 << s) - 1);
    unsigned __int128 q = a >> s;
    if (rem > half || (rem == half && (q & 1))) q += 1;
    uint32_t bits;
    if (qexp == -24) {
        bits = (uint32_t)q;                     /* fp16 bits are linear up to 2^-13 */
    } else {
        int e = qexp;
        if (q >= 0x800) { q >>= 1; e += 1; }    /* rounding carry (q was 0x800, exact shift) */
        int be = e + 10 + 15;                   /* q in [2^10, 2^11): value = 1.f * 2^(e+10) */
        bits = (be >= 31) ? 0x7C00u : (((uint32_t)be << 10) | ((uint32_t)q & 0x3FF));
    }
    return (uint16_t)(bits | (neg ? 0x8000u : 0u));
}

/* Exact fp16 dot product rounded once to fp16 (RNE).  Returns fp16 bits; -0 -> +0. */
uint16_t oracle_rn16_dot(const uint16_t* q, const uint16_t* c, int d) {
    __int128 acc = 0;
    for (int k = 0; k < d; ++k) {
        uint16_t a = q[k], b = c[k];
        int ea = (a >> 10) & 0x1F, eb = (b >> 10) & 0x1F;
        int64_t ma = a & 0x3FF, mb = b & 0x3FF;
        if (ea) ma |= 0x400; else ea = 1;       /* value = ma * 2^(ea-25) */
        if (eb) mb |= 0x400; else eb = 1;
        int64_t p = ma * mb;                    /* value = p * 2^(ea+eb-50) */
        int sh = ea + eb - 50 + 48;             /* units of 2^-48: >= 0 */
        __int128 t = (__int128)p << sh;
        if ((a ^ b) & 0x8000) acc -= t; else acc += t;
    }
    int neg = acc < 0;
    unsigned __int128 mag = neg ? (unsigned __int128)(-acc) : (unsigned __int128)acc;
    uint16_t r = rn16_from_u128(mag, neg);
    if (r == 0x8000) r = 0;
    return r;
}

/* Order-preserving map fp16 bits -> uint16 (larger value -> larger code). */
static inline uint32_t ord16(uint16_t h) {
    return (h & 0x8000) ? (uint32_t)(~h & 0xFFFF) : (uint32_t)(h | 0x8000);
}

/* ------------------------------------------------------------------ Stage 2 */

/*
 * native_prep for one query (weft_prep.py:32-47), compact=True form.
 *   Q [ntok,128] fp16, C [NC,128] fp16.
 *   kk = min(nc + impute, NC) values are selected; topc/scores get min(nc, kk) columns.
 *   topc [ntok, ncol] int32, scores [ntok, ncol] f32, m [ntok] f32 (only if imputed),
 *   vals16 [ntok, kk] (optional) the selected fp16 values, best first.
 * Returns ncol.
 */
int oracle_native_prep(const uint16_t* Q, int ntok, const uint16_t* C, int NC, int dim,
                       int nc, int impute, int32_t* topc, float* scores, float* m,
                       uint16_t* vals16) {
    int kk = nc + (impute ? 1 : 0);
    if (kk > NC) kk = NC;
    int ncol = nc < kk ? nc : kk;
    int imputed = impute && kk > nc;
    uint64_t* best = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(kk + 1));
    for (int t = 0; t < ntok; ++t) {
        int nb = 0;
        for (int c = 0; c < NC; ++c) {
            uint16_t v = oracle_rn16_dot(Q + (size_t)t * dim, C + (size_t)c * dim, dim);
            uint64_t key = ((uint64_t)ord16(v) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)c);
            if (nb < kk) {
                int i = nb++;
                while (i > 0 && best[i - 1] < key) { best[i] = best[i - 1]; --i; }
                best[i] = key;
            } else if (key > best[kk - 1]) {
                int i = kk - 1;
                while (i > 0 && best[i - 1] < key) { best[i] = best[i - 1]; --i; }
                best[i] = key;
            }
        }
        float mt = 0.0f;
        if (imputed) {
            uint32_t o = (uint32_t)(best[nc] >> 32);
            uint16_t h = (uint16_t)((o & 0x8000) ? (o & 0x7FFF) : (~o & 0xFFFF));
            mt = oracle_h2f(h);
            m[t] = mt;
        }
        for (int j = 0; j < kk; ++j) {
            uint32_t o = (uint32_t)(best[j] >> 32);
            uint16_t h = (uint16_t)((o & 0x8000) ? (o & 0x7FFF) : (~o & 0xFFFF));
            int cid = (int)(0xFFFFFFFFu - (uint32_t)(best[j] & 0xFFFFFFFFu));
            if (vals16) vals16[(size_t)t * kk + j] = h;
            if (j < ncol) {
                topc[(size_t)t * ncol + j] = cid;
                float v = oracle_h2f(h);
                scores[(size_t)t * ncol + j] = imputed ? (v - mt) : v;
            }
        }
    }
    free(best);
    return ncol;
}

/* ------------------------------------------------------------------ Stage 3 */

typedef struct {
    const int64_t* row_ptrs;     /* [32, NC+1] */
    const void* col_eids;        /* [n_lists] uint8 or uint16 */
    int eid_bytes;
    const int64_t* block_sums;   /* [ceil(n_lists/128)] */
    const uint16_t* lengths;     /* [n_lists] */
    const uint8_t* packed24;     /* [3 * postings] */
    int64_t num_lists;
    int num_passages;            /* N */
    int num_centroids;           /* NC */
    const uint32_t* preds;       /* [N] */
} oracle_csr;

static inline int eid_at(const oracle_csr* x, int64_t i) {
    return x->eid_bytes == 1 ? ((const uint8_t*)x->col_eids)[i] : ((const uint16_t*)x->col_eids)[i];
}

/* RN fp32 -> fp16 bits (__float2half_rn) for a positive finite float; base scores are > 0. */
static uint16_t f2h_rn(float f) {
    if (!(f > 0.0f)) return 0;
    if (f < 0x1p-24f) return (f > 0x1p-25f) ? 1 : 0;       /* below the smallest subnormal */
    int e; double fr = frexp((double)f, &e);               /* f = fr * 2^e, fr in [0.5, 1) */
    uint64_t mant = (uint64_t)ldexp(fr, 24);               /* exact 24-bit significand */
    int sh = e - 24 + 48;                                  /* f = mant * 2^sh * 2^-48, sh >= 1 */
    return rn16_from_u128((unsigned __int128)mant << sh, 0);
}

/* Posting offset of list li: block sum + lengths before it in its block (ragrt_fused_kernel.cu:208-213). */
static int64_t list_offset(const oracle_csr* x, int64_t li) {
    int64_t b = li >> BLOCK_SHIFT;
    int64_t off = x->block_sums[b];
    for (int64_t k = b << BLOCK_SHIFT; k < li; ++k) off += x->lengths[k];
    return off;
}

typedef struct { int32_t pid; float sum; } oracle_cand;

static int cmp_desc(const void* a, const void* b) {
    const oracle_cand* x = (const oracle_cand*)a; const oracle_cand* y = (const oracle_cand*)b;
    if (x->sum > y->sum) return -1;
    if (x->sum < y->sum) return 1;
    return (x->pid < y->pid) ? -1 : (x->pid > y->pid);
}

/*
 * Candidate generation for one query (Stages 1-3 of the reference in weft mode).
 *   topc/scores [ntok, kc] (compact scores aligned with topc), n_eids = number of
 *   codeword ids enumerated per probed centroid (all-codewords Stage 1: 0..n_eids-1).
 *   Outputs cand_pids [K] (-1 padding), cand_sums [K] (-inf padding).
 *   stats[0] = postings scanned (sum over kept (token, probe) tasks of list lengths),
 *   stats[1] = touched passages U, stats[2] = tasks kept.
 * Returns the number of real candidates written.
 */
int oracle_candidates(const oracle_csr* x, const int32_t* topc, const float* scores,
                      int ntok, int kc, int n_eids, uint32_t mask, int K,
                      int32_t* cand_pids, float* cand_sums, int64_t* stats) {
    int N = x->num_passages, NC = x->num_centroids;
    /* per (pid, token) max of fp16 bits, and a touched flag */
    uint16_t* best = (uint16_t*)calloc((size_t)N * 32, sizeof(uint16_t));
    uint8_t* touched = (uint8_t*)calloc((size_t)N, 1);
    int64_t postings = 0, tasks = 0;
    for (int t = 0; t < ntok && t < 32; ++t) {
        for (int j = 0; j < kc; ++j) {
            int cid = topc[(size_t)t * kc + j];
            if (cid < 0 || cid >= NC) continue;
            float base = scores[(size_t)t * kc + j];          /* cw_weight = 0: base = centroid score */
            for (int s = 0; s < NUM_SUBSPACES; ++s) {
                const int64_t* rp = x->row_ptrs + (int64_t)s * (NC + 1);
                for (int e = 0; e < n_eids; ++e) {
                    int64_t lo = rp[cid], hi = rp[cid + 1], found = -1;
                    while (lo < hi) {                          /* ragrt_fused_kernel.cu:191-197 */
                        int64_t mid = lo + ((hi - lo) >> 1);
                        int ee = eid_at(x, mid);
                        if (ee == e) { found = mid; break; }
                        else if (ee < e) lo = mid + 1;
                        else hi = mid;
                    }
                    if (found < 0) continue;
                    int len = x->lengths[found];
                    if (len <= 0) continue;
                    if (!(base > 0.0f)) continue;              /* MIN_BASE_SCORE, :206 */
                    ++tasks;
                    postings += len;
                    int64_t off = list_offset(x, found);
                    uint16_t sb = (uint16_t)(f2h_rn(base) & 0x7FFF);
                    for (int i = 0; i < len; ++i) {
                        const uint8_t* p = x->packed24 + (off + i) * 3;
                        int pid = p[0] | (p[1] << 8) | (p[2] << 16);
                        if (pid >= N) continue;
                        if (mask && !(x->preds[pid] & mask)) continue;
                        touched[pid] = 1;
                        uint16_t* b = best + (size_t)pid * 32 + t;
                        if (sb > *b) *b = sb;
                    }
                }
            }
        }
    }
    /* per pid exact sum of token maxima (units of 2^-24), rounded once to fp32 */
    int64_t U = 0;
    for (int p = 0; p < N; ++p) U += touched[p];
    oracle_cand* all = (oracle_cand*)malloc(sizeof(oracle_cand) * (size_t)(U > 0 ? U : 1));
    int64_t n = 0;
    for (int p = 0; p < N; ++p) {
        if (!touched[p]) continue;
        uint64_t acc = 0;
        for (int t = 0; t < 32; ++t) {
            uint16_t h = best[(size_t)p * 32 + t];
            if (!h) continue;
            int e = (h >> 10) & 0x1F; uint64_t mm = h & 0x3FF;
            if (e) { mm |= 0x400; acc += mm << (e - 1); } else acc += mm;   /* units of 2^-24 */
        }
        all[n].pid = p;
        all[n].sum = ldexpf((float)acc, -24);   /* (float)u64 is RN; the power-of-2 scale is exact */
        ++n;
    }
    int nreal;
    if (U <= K) {
        for (int64_t i = 0; i < n; ++i) { cand_pids[i] = all[i].pid; cand_sums[i] = all[i].sum; }
        nreal = (int)n;
    } else {
        qsort(all, (size_t)n, sizeof(oracle_cand), cmp_desc);
        for (int i = 0; i < K; ++i) { cand_pids[i] = all[i].pid; cand_sums[i] = all[i].sum; }
        nreal = K;
    }
    for (int i = nreal; i < K; ++i) { cand_pids[i] = -1; cand_sums[i] = -INFINITY; }
    if (stats) { stats[0] = postings; stats[1] = U; stats[2] = tasks; }
    free(all); free(best); free(touched);
    return nreal;
}

/* ------------------------------------------------------------------ Stage 4 */

typedef struct {
    const int64_t* doc_offsets;  /* [N+1] */
    const int32_t* doc_lens;     /* [N] */
    const int32_t* codes;        /* [T] */
    const uint8_t* residuals;    /* [T, 32] */
    const uint16_t* centroids;   /* [NC, 128] fp16 */
    const uint16_t* bucket_weights; /* [4] fp16 */
    const uint8_t* rbm;          /* [256] */
    const uint8_t* decomp;       /* [256, 4] */
    int num_passages;            /* N: pids outside [0, N) score -inf */
} oracle_docs;

/* RN fp16 addition of two fp16 values (the kernels' __hadd). */
static uint16_t hadd_rn(uint16_t a, uint16_t b) {
    /* exact sum in units of 2^-24 fits easily in int64 */
    int ea = (a >> 10) & 0x1F, eb = (b >> 10) & 0x1F;
    int64_t ma = a & 0x3FF, mb = b & 0x3FF;
    if (ea) ma |= 0x400; else ea = 1;
    if (eb) mb |= 0x400; else eb = 1;
    int64_t va = ma << (ea - 1), vb = mb << (eb - 1);     /* units of 2^-24 */
    if (a & 0x8000) va = -va;
    if (b & 0x8000) vb = -vb;
    int64_t s = va + vb;
    int neg = s < 0;
    unsigned __int128 mag = (unsigned __int128)(neg ? -s : s) << 24;  /* to units of 2^-48 */
    uint16_t r = rn16_from_u128(mag, neg);
    if (s == 0) r = ((a & b) & 0x8000) ? 0x8000 : 0;      /* IEEE: (-0)+(-0) = -0, else +0 */
    return r;
}

/* score of one candidate; Q [32,128] fp16 */
static float tile_maxsim_one(const oracle_docs* D, const uint16_t* Q, int pid) {
    if (pid < 0 || pid >= D->num_passages) return -INFINITY;
    int64_t start = D->doc_offsets[pid];
    int L = D->doc_lens[pid];
    double runmax[32];
    for (int r = 0; r < 32; ++r) runmax[r] = -1e9;
    double qd[32][128];
    for (int r = 0; r < 32; ++r) for (int k = 0; k < 128; ++k) qd[r][k] = h2d(Q[r * 128 + k]);
    for (int t = 0; t < L; ++t) {
        int64_t tok = start + t;
        int cid = D->codes[tok];
        double d[128]; double ss = 0.0;
        for (int j = 0; j < 32; ++j) {
            uint8_t byte = D->residuals[tok * 32 + j];
            uint8_t rev = D->rbm[byte];
            for (int u = 0; u < 4; ++u) {
                int k = 4 * j + u;
                uint16_t w = D->bucket_weights[D->decomp[rev * 4 + u]];
                uint16_t h = hadd_rn(D->centroids[(int64_t)cid * 128 + k], w);
                d[k] = h2d(h);
                ss += d[k] * d[k];
            }
        }
        double inv = 1.0 / sqrt(ss + 1e-12);
        for (int r = 0; r < 32; ++r) {
            double s = 0.0;
            for (int k = 0; k < 128; ++k) s += qd[r][k] * d[k];
            s *= inv;
            if (s > runmax[r]) runmax[r] = s;
        }
    }
    double tot = 0.0;
    for (int r = 0; r < 32; ++r) tot += runmax[r];
    return (float)tot;
}

void oracle_tile_maxsim(const oracle_docs* D, const uint16_t* Q, const int32_t* pids, int n,
                        float* out, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 16)
#endif
    for (int i = 0; i < n; ++i) out[i] = tile_maxsim_one(D, Q, pids[i]);
}

/* ------------------------------------------------------------------ final top-k */

/* failing / padding candidates -> -inf (when mask != 0), then top-k by (score desc, pid asc). */
int oracle_final_topk(const int32_t* pids, const float* scores, int n, const uint32_t* preds,
                      uint32_t mask, int k, int32_t* out_ids, float* out_scores) {
    oracle_cand* a = (oracle_cand*)malloc(sizeof(oracle_cand) * (size_t)(n > 0 ? n : 1));
    for (int i = 0; i < n; ++i) {
        float s = scores[i];
        if (pids[i] < 0) s = -INFINITY;
        else if (mask && !(preds[pids[i]] & mask)) s = -INFINITY;
        a[i].pid = pids[i]; a[i].sum = s;
    }
    qsort(a, (size_t)n, sizeof(oracle_cand), cmp_desc);
    int kk = k < n ? k : n;
    for (int i = 0; i < kk; ++i) { out_ids[i] = a[i].pid; if (out_scores) out_scores[i] = a[i].sum; }
    free(a);
    return kk;
}

/* ------------------------------------------------------------------ whole path */

/*
 * The full weft search for a batch of queries (the CPU baseline): for each query
 * Stage 2 -> Stage 3 -> Stage 4 -> final top-k.  Queries run in parallel (OpenMP);
 * Stage 4 of one query runs serially inside its thread.
 *   Q [B,32,128] fp16, ntok [B], masks [B] (or NULL = 0).
 *   out_ids [B, k_top] (-1 padded), out_scores [B, k_top].
 */
void oracle_weft_search(const oracle_csr* x, const oracle_docs* D, const uint16_t* Cent, int dim,
                        const uint16_t* Q, const int32_t* ntok, int B, int nc, int n_eids,
                        const uint32_t* masks, int K, int k_top, int32_t* out_ids,
                        float* out_scores, int64_t* stats, int nthreads) {
    int NC = x->num_centroids;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int b = 0; b < B; ++b) {
        int nt = ntok[b] < 32 ? ntok[b] : 32;
        int32_t* topc = (int32_t*)malloc(sizeof(int32_t) * 32 * (size_t)nc);
        float* sc = (float*)malloc(sizeof(float) * 32 * (size_t)nc);
        float m[32];
        int ncol = oracle_native_prep(Q + (size_t)b * 32 * dim, nt, Cent, NC, dim, nc, 1, topc, sc, m, NULL);
        int32_t* cp = (int32_t*)malloc(sizeof(int32_t) * (size_t)K);
        float* cs = (float*)malloc(sizeof(float) * (size_t)K);
        uint32_t mk = masks ? masks[b] : 0;
        int64_t st[3];
        oracle_candidates(x, topc, sc, nt, ncol, n_eids, mk, K, cp, cs, st);
        float* fs = (float*)malloc(sizeof(float) * (size_t)K);
        for (int i = 0; i < K; ++i) fs[i] = tile_maxsim_one(D, Q + (size_t)b * 32 * dim, cp[i]);
        int32_t* ids = out_ids + (size_t)b * k_top;
        float* osc = out_scores ? out_scores + (size_t)b * k_top : NULL;
        for (int i = 0; i < k_top; ++i) { ids[i] = -1; if (osc) osc[i] = -INFINITY; }
        oracle_final_topk(cp, fs, K, x->preds, mk, k_top, ids, osc);
        if (stats) { stats[3 * b] = st[0]; stats[3 * b + 1] = st[1]; stats[3 * b + 2] = st[2]; }
        free(topc); free(sc); free(cp); free(cs); free(fs);
    }
}

/* Batched Stage 2 (for the CPU timing of that stage alone). */
void oracle_native_prep_batch(const uint16_t* Q, const int32_t* ntok, int B, const uint16_t* C,
                              int NC, int dim, int nc, int impute, int32_t* topc, float* scores,
                              float* m, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int b = 0; b < B; ++b) {
        int nt = ntok[b] < 32 ? ntok[b] : 32;
        oracle_native_prep(Q + (size_t)b * 32 * dim, nt, C, NC, dim, nc, impute,
                           topc + (size_t)b * 32 * nc, scores + (size_t)b * 32 * nc,
                           m + (size_t)b * 32, NULL);
    }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
