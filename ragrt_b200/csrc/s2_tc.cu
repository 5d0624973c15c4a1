// s2_tc.cu -- Stage 2 on the tensor cores: fp16 query-token x centroid scores with tcgen05
// (accumulators in tensor memory, operands staged by TMA) and a fused, exact top-(nc+1)
// epilogue.  The reference computes Q @ C^T with a cuBLAS fp16 GEMM and torch.topk per
// query (src/weft_prep.py:32-47); the full [32, NC] score matrix is never materialised here.
//
// CTA = 128 query rows (4 queries of 32 tokens; the pre-pass below: two such row blocks) x one
// slice of the centroids.
//   warp 0 : TMA producer -- the 128 x 128 query tile once, then 128-centroid x 128-dim
//            tiles of C through a ring of shared-memory stages (128-byte swizzle, K-major)
//   warp 1 : MMA issuer -- per tile 8 x tcgen05.mma (M=128, N=128, K=16) per row block into
//            tensor-memory accumulators (4 x 128 columns = all 512)
//   warps 2-9 (epilogue, two sets of four, one warp per tensor-memory lane quadrant): drain
//            the accumulator with tcgen05.ld and release it.  Each fp32 accumulation brackets
//            the exact fp16 score: lo = RN16(acc - eps) <= RN16(exact) <= hi = RN16(acc + eps)
//            (s2_common.cuh).
//            Lane l filters its row's 128 scores against the row's admission key Te (a
//            lower bound on the row's final kk-th key); rows with survivors in a 32-column
//            chunk are then taken one at a time by the whole warp, lane = centroid, which
//            appends raw entries (fp32 accumulation, centroid) to the row's 64-slot list.  A
//            full list is settled -- raw entries become superset keys (lo, centroid asc, bit 0 =
//            "lo != hi"), those whose upper bound cannot beat Te are dropped -- and compacted
//            warp-wide: bitonic sort, T = kk-th lower-bound key, keep the first kk and the
//            entries whose upper bound still beats T (if none can be dropped, the ambiguous ones
//            are resolved with an exact fp64 dot product first).  T is published per row with
//            atomicMax, so the slices of a row share one admission key.  The path taken on
//            tiles with survivors is kept small (rolled loops) so that it stays in the
//            instruction cache.
// Each CTA writes its rows' sorted supersets to partial[query][slice][token][64];
// s2_merge_tc takes the global superset across slices, resolves only its ambiguous
// members with an exact fp64 dot product and selects the exact top-kk.  All waits are
// bounded; a timeout raises an error flag and every role exits.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "s2_common.cuh"
#include "tc.cuh"

namespace ragrt {

constexpr int kQM = 128;                       // query rows per CTA
constexpr int kCN = 128;                       // centroids per tile
constexpr int kAccBufs = 4;                    // tensor-memory accumulators (128 columns each)
constexpr int kS2TcThreads = 320;             // producer, MMA, 2 x 4 epilogue warps (both passes)
constexpr uint32_t kTileBytes = kCN * 256;     // 32 KB: two 16 KB K-atoms
constexpr uint32_t kQTileBytes = kQM * 256;    // 32 KB
constexpr uint32_t kS2WaitLimit = 1u << 24;

struct S2TcParams {
    const __half* Q;
    const __half* C;
    const float* cnorm;
    const float* cnmax;          // device scalar: max centroid norm
    const int32_t* ntok;
    uint64_t* partial;
    unsigned long long* gthr;    // [rows_total] best k-th lower-bound key of the row over all slices
    uint16_t* tilemax;           // [rows_total][tiles_total] pre-pass: fp16 lower bound of each tile's best score
    int* err;
    int rows_total, rows, NC, kk, tiles_total, tiles_per_slice, nslices, stages;
};

constexpr int kListCap = 64;                   // per-row list slots (kk <= 63)

// superset key: (ord16(lo) << 32) | ((0x7FFFFFFF - id) << 1) | ambiguous;  orders by (lo desc, id asc)
__device__ __forceinline__ uint64_t sk_make(uint16_t lo, uint32_t id, uint32_t amb) {
    if (lo == 0x8000u) lo = 0;
    return ((uint64_t)ord16(lo) << 32) | ((uint64_t)(0x7FFFFFFFu - id) << 1) | (uint64_t)amb;
}
__device__ __forceinline__ uint32_t sk_id(uint64_t k) { return 0x7FFFFFFFu - ((uint32_t)k >> 1); }
__device__ __forceinline__ uint16_t f16_next(uint16_t h) {
    if (h == 0x8000u || h == 0) return 1;
    return (h & 0x8000u) ? (uint16_t)(h - 1) : (uint16_t)(h + 1);
}
// key of the upper bound (flag cleared): hi = next(lo) for an ambiguous entry
__device__ __forceinline__ uint64_t sk_hi(uint64_t k) {
    if (!(k & 1)) return k;
    const uint16_t lo = unord16((uint32_t)(k >> 32));
    return sk_make(f16_next(lo), sk_id(k), 0);
}

// Score filter for admission key `te` (a lower-bound key, flag clear): a score whose fp32
// accumulation is below the returned value rounds (with its error bound eps <= eps_max added)
// to an fp16 value strictly below te's value, so its upper-bound key is below te whatever its
// id.  The bound is the midpoint between te's value and the next SMALLER fp16 value.
__device__ __forceinline__ float s2_filter_threshold(uint64_t te, float eps_max) {
    const uint16_t h = unord16((uint32_t)(te >> 32));
    uint16_t pv;
    if (h == 0x8000u || h == 0) pv = 0x8001u;
    else if (h & 0x8000u) pv = (uint16_t)(h + 1);
    else pv = (uint16_t)(h - 1);
    const float a = __half2float(__ushort_as_half(h)), b = __half2float(__ushort_as_half(pv));
    const float mid = 0.5f * (a + b);
    return mid - (eps_max + fabsf(mid) * 2.4e-7f + 1e-30f);
}

// fp16 value of the exact dot product of q and c, warp-wide (4 dims per lane; the fp64
// partial sums of fp16 products are exact while |q||c| < 32), on every lane.
__device__ __forceinline__ uint16_t s2_warp_exact(const __half* q, const __half* c, int lane) {
    const uint2 qv = *reinterpret_cast<const uint2*>(q + 4 * lane);
    const uint2 cv = __ldg(reinterpret_cast<const uint2*>(c + 4 * lane));
    const __half* qh = reinterpret_cast<const __half*>(&qv);
    const __half* ch = reinterpret_cast<const __half*>(&cv);
    double d = 0.0;
#pragma unroll
    for (int u = 0; u < 4; ++u) d = fma((double)__half2float(qh[u]), (double)__half2float(ch[u]), d);
#pragma unroll
    for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
    const uint16_t h = d2h_rn(d);
    return h == 0x8000u ? 0 : h;
}

// Bitonic sort of 64 keys held two per lane (element i = lane + 32 h), descending.
__device__ __forceinline__ void s2_sort64_desc(uint64_t& a0, uint64_t& a1, int lane) {
#pragma unroll
    for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j == 32) {               // partner is the lane's other element (k == 64: descending)
                const uint64_t mx = a0 > a1 ? a0 : a1, mn = a0 > a1 ? a1 : a0;
                a0 = mx;
                a1 = mn;
                continue;
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint64_t& a = h ? a1 : a0;
                const int i = lane + 32 * h;
                const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, a, j);
                const bool lower = (i & j) == 0, desc = (i & k) == 0;
                const uint64_t mx = a > o ? a : o, mn = a > o ? o : a;
                a = (lower == desc) ? mx : mn;
            }
        }
    }
}

// Raw list entry, appended by the row's lane without any per-entry work: bit 63 set, the fp32
// accumulation in bits 31..62, the centroid id in bits 0..30.  Keys (sk_make) have bits 48..63
// clear, so the two kinds share a list.
__device__ __forceinline__ uint64_t raw_make(float acc, int c) {
    return (1ull << 63) | ((uint64_t)__float_as_uint(acc) << 31) | (uint64_t)(uint32_t)c;
}

// Settle one row's list (warp-wide): turn every raw entry into its superset key -- the fp16
// bracket lo <= RN16(exact) <= hi of its accumulation, bit 0 = "lo != hi", resolved exactly where
// the bracket spans more than one fp16 step -- and drop the entries whose upper bound does not
// beat the row's admission key te.
__device__ __noinline__ void s2_settle(uint64_t* lst, int n, uint64_t te, float qn, const float* __restrict__ cnorm,
                                       const __half* qrow, const __half* C, int lane) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e = lane + 32 * h;
        uint64_t a = e < n ? lst[e] : 0ull;
        bool exact = false;
        if (a >> 63) {
            const float acc = __uint_as_float((uint32_t)(a >> 31));
            const uint32_t c = (uint32_t)a & 0x7FFFFFFFu;
            const float eps = fmaf(fabsf(acc), 1.2e-7f, qn * __ldg(cnorm + c) * kEpsTc);
            uint16_t hi = __half_as_ushort(__float2half_rn(acc + eps));
            if (hi == 0x8000u) hi = 0;
            if (sk_make(hi, c, 0) <= te) {
                a = 0ull;
            } else {
                uint16_t lo = __half_as_ushort(__float2half_rn(acc - eps));
                if (lo == 0x8000u) lo = 0;
                const uint32_t amb = lo != hi;
                exact = amb && f16_next(lo) != hi;       // tiny scores: the bracket spans several steps
                a = sk_make(lo, c, exact ? 0 : amb);
            }
        }
        unsigned need = __ballot_sync(0xFFFFFFFFu, exact);
        while (need) {
            const int s = __ffs(need) - 1;
            need &= need - 1;
            const uint32_t id = sk_id(__shfl_sync(0xFFFFFFFFu, a, s));
            const uint16_t hx = s2_warp_exact(qrow, C + (int64_t)id * kDim, lane);
            if (lane == s) a = sk_make(hx, id, 0) <= te ? 0ull : sk_make(hx, id, 0);
        }
        if (e < n) lst[e] = a;
    }
    __syncwarp();
}

// Compact one row's list (warp-wide): optionally resolve every ambiguous entry exactly, sort
// by key, take T = the kk-th lower-bound key (0 while fewer than kk entries), and keep the
// first kk entries plus those whose upper bound beats T.  Returns T; updates n.
__device__ __noinline__ uint64_t s2_compact(uint64_t* lst, int& n, int kk, bool resolve, const __half* qrow,
                                            const __half* C, int lane) {
    uint64_t a0 = lane < n ? lst[lane] : 0ull;
    uint64_t a1 = lane + 32 < n ? lst[lane + 32] : 0ull;
    if (resolve) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint64_t& a = h ? a1 : a0;
            unsigned need = __ballot_sync(0xFFFFFFFFu, (a & 1ull) != 0);
            while (need) {
                const int s = __ffs(need) - 1;
                need &= need - 1;
                const uint32_t id = sk_id(__shfl_sync(0xFFFFFFFFu, a, s));
                const uint16_t hx = s2_warp_exact(qrow, C + (int64_t)id * kDim, lane);
                if (lane == s) a = sk_make(hx, id, 0);
            }
        }
    }
    s2_sort64_desc(a0, a1, lane);
    uint64_t T = 0;
    if (n >= kk) T = __shfl_sync(0xFFFFFFFFu, ((kk - 1) >> 5) ? a1 : a0, (kk - 1) & 31) & ~1ull;
    const bool k0 = a0 != 0 && (lane < kk || sk_hi(a0) > T);
    const bool k1 = a1 != 0 && (lane + 32 < kk || sk_hi(a1) > T);
    const unsigned b0 = __ballot_sync(0xFFFFFFFFu, k0), b1 = __ballot_sync(0xFFFFFFFFu, k1);
    const unsigned lt = (1u << lane) - 1u;
    __syncwarp();
    if (k0) lst[__popc(b0 & lt)] = a0;
    if (k1) lst[__popc(b0) + __popc(b1 & lt)] = a1;
    __syncwarp();
    n = __popc(b0) + __popc(b1);
    return T;
}

// kTileMax: the pre-pass.  Same GEMM; the epilogue only records, per row and 128-centroid
// tile, RN16(max acc - eps), a lower bound of the tile's best fp16 score.  A pre-pass CTA covers
// two 128-row blocks, so that every centroid tile it streams serves 256 rows (the pass is bound
// by that stream out of L2): per tile two accumulators, one per row block, in two tile buffers.
// Both passes run two epilogue warp sets of four (one warp per lane quadrant), and both sets
// take every tile: in the pre-pass set s drains row block s; in the selecting pass the sets
// split each quadrant's 32 rows, set s admitting candidates for rows 16 s .. 16 s + 15 only, so
// that each row list has one owner.
template <bool kTileMax>
__global__ void __launch_bounds__(kS2TcThreads, 1)
s2_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmC, S2TcParams p) {
    constexpr int kRB = kTileMax ? 2 : 1;            // 128-row blocks per CTA
    constexpr int kTB = kAccBufs / kRB;              // tile buffers in tensor memory
    extern __shared__ uint8_t s2_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)s2_raw + 1023) & ~(uintptr_t)1023);
    const int S = p.stages, kk = p.kk;
    uint8_t* sA = sm;
    uint8_t* sB = sm + kRB * kQTileBytes;
    uint64_t* lists = reinterpret_cast<uint64_t*>(sB + (size_t)S * kTileBytes);    // [128 rows][kListCap]
    float* scratch = reinterpret_cast<float*>(lists + (kTileMax ? 0 : (size_t)kListCap * kQM));  // [128][33]
    uint64_t* bars = reinterpret_cast<uint64_t*>(scratch + (kTileMax ? 0 : kQM * 33));   // 8-byte aligned
    uint64_t* fullA = bars;
    uint64_t* full = bars + 1;
    uint64_t* empty = full + S;
    uint64_t* accf = empty + S;
    uint64_t* acce = accf + kAccBufs;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(acce + kAccBufs);
    volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slice = blockIdx.x, rb = blockIdx.y;
    const int t0 = slice * p.tiles_per_slice;
    const int ntiles = min(p.tiles_total, t0 + p.tiles_per_slice) - t0;

    if constexpr (!kTileMax)
        for (int i = threadIdx.x; i < kListCap * kQM; i += blockDim.x) lists[i] = 0ull;
    if (threadIdx.x == 0) {
        tc::mbar_init(fullA, 1);
        for (int s = 0; s < S; ++s) { tc::mbar_init(full + s, 1); tc::mbar_init(empty + s, 1); }
        // a tile buffer is drained by both warp sets
        for (int b = 0; b < kTB; ++b) {
            tc::mbar_init(accf + b, 1);
            tc::mbar_init(acce + b, 8);
        }
        *abort = 0;
        tc::mbar_fence_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tslot, kAccBufs * kCN);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0 && ntiles > 0) {
            tc::mbar_arrive_expect_tx(fullA, kRB * kQTileBytes);
#pragma unroll
            for (int j = 0; j < kRB; ++j) {           // rows past the end are zero-filled
                tc::tma_load_2d(sA + j * kQTileBytes, &tmQ, 0, (rb * kRB + j) * kQM, fullA);
                tc::tma_load_2d(sA + j * kQTileBytes + kQTileBytes / 2, &tmQ, 64, (rb * kRB + j) * kQM, fullA);
            }
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % S;
                if (i >= S && !tc::mbar_wait_or_abort(empty + s, ((i / S) - 1) & 1, abort, kS2WaitLimit)) break;
                uint8_t* dst = sB + (size_t)s * kTileBytes;
                tc::mbar_arrive_expect_tx(full + s, kTileBytes);
                tc::tma_load_2d(dst, &tmC, 0, (t0 + i) * kCN, full + s);
                tc::tma_load_2d(dst + kTileBytes / 2, &tmC, 64, (t0 + i) * kCN, full + s);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0 && ntiles > 0) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(kQM, kCN);
            const uint32_t aBase = tc::smem_u32(sA);
            bool ok = tc::mbar_wait_or_abort(fullA, 0, abort, kS2WaitLimit);
            for (int i = 0; ok && i < ntiles; ++i) {
                const int s = i % S, b = i % kTB;
                if (!tc::mbar_wait_or_abort(full + s, (i / S) & 1, abort, kS2WaitLimit)) break;
                if (i >= kTB && !tc::mbar_wait_or_abort(acce + b, ((i / kTB) - 1) & 1, abort, kS2WaitLimit))
                    break;
                tc::fence_after();
                const uint32_t bBase = tc::smem_u32(sB + (size_t)s * kTileBytes);
#pragma unroll
                for (int j = 0; j < kRB; ++j) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint32_t koffA = (uint32_t)(j * kQTileBytes + (k >> 2) * (kQTileBytes / 2) + (k & 3) * 32);
                        const uint32_t koffB = (uint32_t)((k >> 2) * (kTileBytes / 2) + (k & 3) * 32);
                        tc::mma_ss(tbase + (uint32_t)((b * kRB + j) * kCN), tc::sw128_kmajor_desc(aBase + koffA),
                                   tc::sw128_kmajor_desc(bBase + koffB), idesc, k > 0);
                    }
                }
                tc::mma_commit(empty + s);
                tc::mma_commit(accf + b);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (warp-cooperative)
        // Lane l of warp (quad) owns TMEM lane 32*quad + l = one query row: it filters that
        // row's scores with a per-row threshold.  Rows with survivors in a 32-column chunk are
        // then handled one at a time by the whole warp (lane = centroid column), which appends
        // raw entries (accumulation, centroid) to the row's list; a full list is settled into
        // superset keys and compacted (bitonic sort + trim) warp-wide.
        const int quad = warp & 3;
        const int wset = (warp - 2) >> 2;               // warp set 0 or 1
        const int blk = kTileMax ? wset : 0;            // this warp's row block in the CTA
        const bool own = kTileMax || (lane >> 4) == wset;  // selecting pass: this lane's row is this warp's
        const int r = quad * 32 + lane;
        const int grow = (rb * kRB + blk) * kQM + r;
        const int qb = grow / p.rows, tok = grow % p.rows;
        const bool valid = grow < p.rows_total && tok < (p.ntok ? min(p.ntok[qb], p.rows) : p.rows);
        const __half* qrow = p.Q + (int64_t)(valid ? grow : 0) * kDim;
        float qn = 0.f;
        if (valid) {
            for (int k = 0; k < kDim; k += 8) {
                uint4 u = *reinterpret_cast<const uint4*>(qrow + k);
                const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = __half22float2(h[j]);
                    qn = fmaf(f.x, f.x, fmaf(f.y, f.y, qn));
                }
            }
            qn = __fsqrt_ru(qn) * (1.0f + 1e-6f);
        }
        const float eps_max = qn * (*p.cnmax) * kEpsTc;
        // this lane's row: list length, admission key, and the score filter derived from it
        int n = 0;
        uint64_t Te = 0;
        float thr = -INFINITY;
        unsigned long long* gT = p.gthr + (valid ? grow : 0);
        uint64_t* wl = lists + (size_t)quad * 32 * kListCap;        // the warp's 32 row lists
        float* sc = scratch + (quad * 32 + lane) * 33;              // this lane's staged chunk scores
        for (int i = 0; i < ntiles; ++i) {
            const int b = i % kTB;
            // other slices' progress on this row (issued before the wait to hide its latency)
            const unsigned long long g =
                (!kTileMax && valid) ? *reinterpret_cast<volatile unsigned long long*>(gT) : 0ull;
            const bool ok = tc::mbar_wait_or_abort(accf + b, (i / kTB) & 1, abort, kS2WaitLimit);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;          // warp-uniform: tcgen05.ld is warp-collective
            tc::fence_after();
            const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + (uint32_t)((b * kRB + blk) * kCN);
            const int c0 = (t0 + i) * kCN;
            if constexpr (kTileMax) {
                uint32_t v[4][32];
                tc::ld32x32(taddr, v[0]);
                tc::ld32x32(taddr + 32, v[1]);
                tc::ld32x32(taddr + 64, v[2]);
                tc::ld32x32(taddr + 96, v[3]);
                tc::wait_ld();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(acce + b);
                if (valid) {
                    const int ncv = min(kCN, p.NC - c0);            // columns past NC hold zero-filled rows
                    float m4[4];
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch) {
                        float m16[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float a = (ch * 32 + j < ncv) ? __uint_as_float(v[ch][j]) : -INFINITY;
                            const float b2 = (ch * 32 + j + 16 < ncv) ? __uint_as_float(v[ch][j + 16]) : -INFINITY;
                            m16[j] = fmaxf(a, b2);
                        }
#pragma unroll
                        for (int w2 = 8; w2 >= 1; w2 >>= 1)
#pragma unroll
                            for (int j = 0; j < w2; ++j) m16[j] = fmaxf(m16[j], m16[j + w2]);
                        m4[ch] = m16[0];
                    }
                    const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
                    uint16_t lo = __half_as_ushort(__float2half_rn(mx - (eps_max + fabsf(mx) * 1.2e-7f + 1e-30f)));
                    if (lo == 0x8000u) lo = 0;
                    p.tilemax[(int64_t)grow * p.tiles_total + t0 + i] = lo;
                }
            } else {
                if (g > Te) {
                    Te = g;
                    thr = s2_filter_threshold(Te, eps_max);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t v[2][32];
                    tc::ld32x32(taddr + 64 * h, v[0]);
                    tc::ld32x32(taddr + 64 * h + 32, v[1]);
                    tc::wait_ld();
                    if (h == 1) {                               // both halves read: release the accumulator
                        tc::fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(acce + b);
                    }
                    // the tile in two halves of 64 columns (32 score registers each): per half the two
                    // 32-column chunk maxima (independent trees), then one vote
                    float mx[2];
#pragma unroll
                    for (int ch = 0; ch < 2; ++ch) {
                        float m16[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) m16[j] = fmaxf(__uint_as_float(v[ch][j]), __uint_as_float(v[ch][j + 16]));
#pragma unroll
                        for (int w2 = 8; w2 >= 1; w2 >>= 1)
#pragma unroll
                            for (int j = 0; j < w2; ++j) m16[j] = fmaxf(m16[j], m16[j + w2]);
                        mx[ch] = m16[0];
                    }
                    const bool hit = valid && own && fmaxf(mx[0], mx[1]) >= thr;
                    if (!__any_sync(0xFFFFFFFFu, hit)) continue;
                    // The candidate path runs on a minority of tiles: it is kept small (a rolled loop over
                    // the chunks, the chunk's scores staged in this lane's scratch row) so that it stays
                    // in the instruction cache.
#pragma unroll 1
                    for (int ch = 0; ch < 2; ++ch) {
                        const float mxc = ch == 0 ? mx[0] : mx[1];
                        const bool cb_hit = hit && mxc >= thr;
                        if (!__any_sync(0xFFFFFFFFu, cb_hit)) continue;
                        const int cb = c0 + 64 * h + ch * 32;
                        // columns of this chunk that hold real centroids (the rest are zero-filled)
                        const uint32_t colmask = cb + 32 <= p.NC ? 0xFFFFFFFFu : (cb < p.NC ? (1u << (p.NC - cb)) - 1u : 0u);
                        if (cb_hit) {
                            switch (ch) {
#define RAGRT_S2_STAGE(K)                                                                  \
        case K:                                                                                \
            _Pragma("unroll") for (int j = 0; j < 32; ++j) sc[j] = __uint_as_float(v[K][j]);   \
            break;
                                RAGRT_S2_STAGE(0)
                                RAGRT_S2_STAGE(1)
#undef RAGRT_S2_STAGE
                            }
                        }
                        uint32_t cand = 0;
                        if (cb_hit) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) cand |= sc[j] >= thr ? (1u << j) : 0u;
                            cand &= colmask;
                        }
                        __syncwarp();                                // the staged rows, visible warp-wide
                        // ---- each row with survivors in turn, lane = column: raw entries, no per-entry work
                        unsigned act = __ballot_sync(0xFFFFFFFFu, cand != 0);
                        while (act) {
                            const int src = __ffs(act) - 1;
                            uint32_t cm = __shfl_sync(0xFFFFFFFFu, cand, src);
                            int n_s = __shfl_sync(0xFFFFFFFFu, n, src);
                            uint64_t* lst = wl + src * kListCap;
                            const int pos = n_s + __popc(cm & ((1u << lane) - 1u));
                            const bool put = ((cm >> lane) & 1u) && pos < kListCap;
                            if (put) lst[pos] = raw_make(scratch[(quad * 32 + src) * 33 + lane], cb + lane);
                            const unsigned put_m = __ballot_sync(0xFFFFFFFFu, put);
                            n_s += __popc(put_m);
                            cm &= ~put_m;
                            if (cm) {
                                // the row's list is full: settle + compact it warp-wide, then place the rest
                                __syncwarp();
                                const uint64_t Te_s = __shfl_sync(0xFFFFFFFFu, Te, src);
                                const float qn_s = __shfl_sync(0xFFFFFFFFu, qn, src);
                                const __half* qrow_s = p.Q + (int64_t)(rb * kQM + quad * 32 + src) * kDim;
                                s2_settle(lst, n_s, Te_s, qn_s, p.cnorm, qrow_s, p.C, lane);
                                uint64_t T = s2_compact(lst, n_s, kk, false, qrow_s, p.C, lane);
                                if (n_s == kListCap) T = s2_compact(lst, n_s, kk, true, qrow_s, p.C, lane);
                                if (lane == src && T > Te) {
                                    Te = T;
                                    thr = s2_filter_threshold(Te, eps_max);
                                    atomicMax(gT, (unsigned long long)Te);
                                }
                            } else {
                                act &= act - 1;
                            }
                            if (lane == src) {
                                n = n_s;
                                cand = cm;
                            }
                        }
                        __syncwarp();                                // scratch rows are restaged by the next chunk
                    }
                }
            }
        }
        // ---- every valid row: final compaction (sorted, trimmed) and write-out
        for (int src = 16 * wset; src < 16 * wset + 16 && !kTileMax; ++src) {
            if (!__shfl_sync(0xFFFFFFFFu, valid, src)) continue;
            int n_s = __shfl_sync(0xFFFFFFFFu, n, src);
            const int grow_s = rb * kQM + quad * 32 + src;
            uint64_t* lst = wl + src * kListCap;
            const __half* qrow_s = p.Q + (int64_t)grow_s * kDim;
            s2_settle(lst, n_s, __shfl_sync(0xFFFFFFFFu, Te, src), __shfl_sync(0xFFFFFFFFu, qn, src), p.cnorm, qrow_s,
                      p.C, lane);
            s2_compact(lst, n_s, kk, false, qrow_s, p.C, lane);
            const int qb_s = grow_s / p.rows, tok_s = grow_s % p.rows;
            uint64_t* out = p.partial + (((int64_t)qb_s * p.nslices + slice) * p.rows + tok_s) * kListCap;
            out[lane] = lane < n_s ? lst[lane] : 0ull;
            out[lane + 32] = lane + 32 < n_s ? lst[lane + 32] : 0ull;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && *abort) atomicExch(p.err, 1);
    if (warp == 1) {
        tc::fence_after();
        tc::tmem_dealloc(tbase, kAccBufs * kCN);
    }
}

// ------------------------------------------------------------------ merge of the slice supersets
// Warp per (query, row).  T = kk-th best lower-bound key over all slices (a tournament over
// the slices' sorted lists, lane = slice); members of the global superset are the entries
// whose upper bound beats T; the ambiguous ones get an exact fp64 dot product (warp-wide, 4
// dims per lane; every partial sum is a multiple of 2^-48 below 2^5, hence exact); the exact
// top-kk is then taken by (value desc, centroid asc).
__global__ void s2_merge_tc(const uint64_t* __restrict__ partial, int nslices, int KX, const int32_t* __restrict__ ntok,
                            int B, int rows, int kk, int nc, int impute, const __half* __restrict__ Q,
                            const __half* __restrict__ C, int32_t* __restrict__ topc, float* __restrict__ scores,
                            float* __restrict__ m) {
    extern __shared__ uint64_t s_ent[];
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = nslices * KX;
    uint64_t* ent = s_ent + (size_t)wib * (E + kk);
    uint64_t* outk = ent + E;
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + wib;
    if (gw >= (int64_t)B * rows) return;
    const int b = (int)(gw / rows), t = (int)(gw % rows);
    const int ncol = min(nc, kk);
    const bool imputed = impute && kk > nc;
    const int nt = ntok ? min(ntok[b], rows) : rows;
    int32_t* tc_ = topc + ((int64_t)b * rows + t) * ncol;
    float* sc = scores + ((int64_t)b * rows + t) * ncol;
    if (t >= nt) {
        for (int j = lane; j < ncol; j += 32) { tc_[j] = -1; sc[j] = 0.f; }
        if (m && lane == 0) m[(int64_t)b * rows + t] = 0.f;
        return;
    }
    for (int i = lane; i < E; i += 32) {
        const int s = i / KX, j = i % KX;
        ent[i] = partial[(((int64_t)b * nslices + s) * rows + t) * KX + j];
    }
    __syncwarp();
    // 1. T: the kk-th lower-bound key over all slices
    uint64_t T = 0;
    {
        int pos = 0;
        for (int j = 0; j < kk; ++j) {
            const uint64_t h = (lane < nslices && pos < KX) ? ent[lane * KX + pos] : 0ull;
            uint64_t mx = h;
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const uint64_t x = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
                mx = x > mx ? x : mx;
            }
            const unsigned win = __ballot_sync(0xFFFFFFFFu, h == mx && mx != 0);
            if (win && lane == __ffs(win) - 1) ++pos;
            T = mx & ~1ull;
        }
    }
    // 2. keep the global superset; resolve its ambiguous members exactly
    const __half* qrow = Q + ((int64_t)b * rows + t) * kDim;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        uint64_t k = e < E ? ent[e] : 0ull;
        bool member = k != 0 && ((k & ~1ull) >= T || sk_hi(k) > T);
        if (!member && e < E) ent[e] = 0ull;
        unsigned need = __ballot_sync(0xFFFFFFFFu, member && (k & 1));
        while (need) {
            const int src = __ffs(need) - 1;
            need &= need - 1;
            const uint64_t ks = __shfl_sync(0xFFFFFFFFu, k, src);
            const uint32_t id = sk_id(ks);
            const uint2 qv = *reinterpret_cast<const uint2*>(qrow + 4 * lane);
            const uint2 cv = *reinterpret_cast<const uint2*>(C + (int64_t)id * kDim + 4 * lane);
            const __half* qh = reinterpret_cast<const __half*>(&qv);
            const __half* ch = reinterpret_cast<const __half*>(&cv);
            double d = 0.0;
#pragma unroll
            for (int u = 0; u < 4; ++u) d = fma((double)__half2float(qh[u]), (double)__half2float(ch[u]), d);
#pragma unroll
            for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
            if (lane == src) {
                uint16_t h = d2h_rn(d);
                k = sk_make(h == 0x8000u ? 0 : h, id, 0);
                ent[e] = k;
            }
        }
    }
    __syncwarp();
    // 3. exact top-kk by (value desc, centroid asc)
    for (int j = 0; j < kk; ++j) {
        uint64_t best = 0;
        int bi = -1;
        for (int e = lane; e < E; e += 32) {
            const uint64_t k = ent[e];
            if (k > best) { best = k; bi = e; }
        }
        uint64_t mx = best;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const uint64_t x = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
            mx = x > mx ? x : mx;
        }
        const unsigned win = __ballot_sync(0xFFFFFFFFu, best == mx && mx != 0);
        if (win && lane == __ffs(win) - 1) ent[bi] = 0ull;
        if (lane == 0) outk[j] = mx;
        __syncwarp();
    }
    __syncwarp();
    float mt = 0.f;
    if (imputed) mt = __half2float(__ushort_as_half(unord16((uint32_t)(outk[nc] >> 32))));
    for (int j = lane; j < ncol; j += 32) {
        const uint64_t k = outk[j];
        tc_[j] = k ? (int32_t)sk_id(k) : -1;
        const float v = __half2float(__ushort_as_half(unord16((uint32_t)(k >> 32))));
        sc[j] = imputed ? __fsub_rn(v, mt) : v;
    }
    if (m && lane == 0) m[(int64_t)b * rows + t] = imputed ? mt : 0.f;
}

// Warp per row: the kk-th largest of the row's tile lower bounds (radix select on the
// order-preserving 16-bit code).  kk distinct tiles hold a centroid scoring at least that, so
// it lower-bounds the row's kk-th fp16 score; it seeds the row's admission key (id part 0:
// every centroid with an upper bound of that value or more is admitted).
__global__ void s2_seed_threshold(const uint16_t* __restrict__ tilemax, int tiles, int rows_total, int kk,
                                  unsigned long long* __restrict__ gthr) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows_total) return;
    const uint16_t* t = tilemax + row * tiles;
    uint32_t prefix = 0;
    if (tiles >= kk) {
        for (int bit = 15; bit >= 0; --bit) {
            const uint32_t cand = prefix | (1u << bit);
            int cnt = 0;
            for (int i = lane; i < tiles; i += 32) cnt += ord16(t[i]) >= cand ? 1 : 0;
#pragma unroll
            for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
            if (cnt >= kk) prefix = cand;
        }
    }
    if (lane == 0) gthr[row] = tiles >= kk ? (unsigned long long)prefix << 32 : 0ull;
}

// max centroid norm (for the chunk filter's error bound) and, optionally, all norms
__global__ void s2_centroid_norms(const __half* __restrict__ C, int NC, float* __restrict__ cn,
                                  float* __restrict__ cnmax) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= NC) return;
    float s = 0.f;
    for (int k = lane; k < kDim; k += 32) {
        const float v = __half2float(C[(int64_t)warp * kDim + k]);
        s = fmaf(v, v, s);
    }
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) {
        const float n = __fsqrt_ru(s) * (1.0f + 1e-6f);
        cn[warp] = n;
        atomicMax(reinterpret_cast<unsigned int*>(cnmax), __float_as_uint(n));   // non-negative floats
    }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)f;
    }
    return fn;
}

// 2-D fp16 tensor [rows, 128] with a [128 rows x 64 cols] box, 128-byte swizzle
static int make_map(CUtensorMap* m, const void* base, int64_t rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(RAGRT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)kDim, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kDim * 2};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RAGRT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return RAGRT_OK;
}

static size_t s2_tc_smem(bool tilemax, int stages) {
    const size_t lists = tilemax ? 0 : (size_t)kListCap * kQM * 8 + (size_t)kQM * 33 * 4;
    return 1024 + (tilemax ? 2 : 1) * (size_t)kQTileBytes + (size_t)stages * kTileBytes + lists +
           8 * (1 + 2 * stages + 2 * kAccBufs) + 16;
}

bool s2_tc_supported(int kk, int64_t rows_total) {
    return rows_total >= kQM && kk < kListCap && s2_tc_smem(false, 2) <= 227 * 1024;
}

// Centroid slices for CTAs of `cta_rows` query rows (the selecting pass: 128; the pre-pass: 256).
static void s2_tc_plan_rows(int B, int rows, int NC, int cta_rows, int& nslices, int& tiles_per_slice) {
    const int rbs = (int)ceil_div((int64_t)B * rows, cta_rows);
    const int tiles = (int)ceil_div(NC, kCN);
    const int sms = num_sms();
    // one wave of CTAs: every extra slice re-pays the top-k warm-up of each row
    const int best = (int)std::max<int64_t>(1, std::min<int64_t>({32, (int64_t)tiles, sms / std::max(1, rbs)}));
    tiles_per_slice = (int)ceil_div(tiles, best);
    nslices = (int)ceil_div(tiles, tiles_per_slice);
}

void s2_tc_plan(int B, int rows, int NC, int& nslices, int& tiles_per_slice) {
    s2_tc_plan_rows(B, rows, NC, kQM, nslices, tiles_per_slice);
}

size_t s2_tc_partial_bytes(int B, int rows, int NC, int kk) {
    int ns, tps;
    s2_tc_plan(B, rows, NC, ns, tps);
    return sizeof(uint64_t) * (size_t)B * ns * rows * kListCap + sizeof(uint64_t) * (size_t)B * rows +
           sizeof(uint16_t) * (size_t)B * rows * ceil_div(NC, kCN) + 512;
}

int s2_tc_run(const __half* Q, const int32_t* ntok, int B, int rows, const __half* C, int NC, const float* cnorm,
              const float* cnmax, int nc, int impute, int32_t* topc, float* scores, float* m, uint64_t* partial,
              int* err, cudaStream_t stream) {
    const int kk = std::min(nc + (impute ? 1 : 0), NC);
    int nslices, tps;
    s2_tc_plan(B, rows, NC, nslices, tps);
    CUtensorMap tmQ, tmC;
    int rc = make_map(&tmQ, Q, (int64_t)B * rows);
    if (rc) return rc;
    if ((rc = make_map(&tmC, C, NC))) return rc;
    int stages = 4;
    while (stages > 2 && s2_tc_smem(false, stages) > 227 * 1024) --stages;
    const size_t smem = s2_tc_smem(false, stages);
    int pre_stages = 6;                           // the pre-pass keeps no lists: a deeper ring fits
    while (pre_stages > 2 && s2_tc_smem(true, pre_stages) > 227 * 1024) --pre_stages;
    const size_t pre_smem = s2_tc_smem(true, pre_stages);
    int pre_ns, pre_tps;
    s2_tc_plan_rows(B, rows, NC, 2 * kQM, pre_ns, pre_tps);
    unsigned long long* gthr = reinterpret_cast<unsigned long long*>(
        partial + (size_t)B * nslices * rows * kListCap);
    const int tiles_total = (int)ceil_div(NC, kCN);
    uint16_t* tilemax = reinterpret_cast<uint16_t*>(gthr + (size_t)B * rows);
    S2TcParams p{Q, C, cnorm, cnmax, ntok, partial, gthr, tilemax, err, B * rows, rows, NC, kk, tiles_total, tps,
                 nslices, stages};
    S2TcParams pp = p;
    pp.stages = pre_stages;
    pp.tiles_per_slice = pre_tps;
    pp.nslices = pre_ns;
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s2_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pre_smem));
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s2_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid(nslices, (unsigned)ceil_div((int64_t)B * rows, kQM));
    dim3 pre_grid(pre_ns, (unsigned)ceil_div((int64_t)B * rows, 2 * kQM));
    // pre-pass: per-row tile bounds -> seeded admission keys; then the selecting pass
    s2_tc<true><<<pre_grid, kS2TcThreads, pre_smem, stream>>>(tmQ, tmC, pp);
    RAGRT_LAUNCH_CHECK();
    s2_seed_threshold<<<(unsigned)ceil_div((int64_t)B * rows * 32, 256), 256, 0, stream>>>(tilemax, tiles_total,
                                                                                          B * rows, kk, gthr);
    RAGRT_LAUNCH_CHECK();
    s2_tc<false><<<grid, kS2TcThreads, smem, stream>>>(tmQ, tmC, p);
    RAGRT_LAUNCH_CHECK();
    const int KX = kListCap;
    const int warps = 4;
    const size_t msmem = sizeof(uint64_t) * warps * ((size_t)nslices * KX + kk);
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s2_merge_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
    s2_merge_tc<<<(unsigned)ceil_div((int64_t)B * rows, warps), warps * 32, msmem, stream>>>(
        partial, nslices, KX, ntok, B, rows, kk, nc, impute, Q, C, topc, scores, m);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

int s2_norms_launch(const __half* C, int NC, float* cn, float* cnmax, cudaStream_t stream) {
    RAGRT_CUDA_TRY(cudaMemsetAsync(cnmax, 0, sizeof(float), stream));
    s2_centroid_norms<<<(unsigned)ceil_div((int64_t)NC * 32, 256), 256, 0, stream>>>(C, NC, cn, cnmax);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
