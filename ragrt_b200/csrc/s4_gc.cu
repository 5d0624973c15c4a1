// s4_gc.cu -- Stage 4 of a bound index on the 5th-generation tensor cores: fused 2-bit
// residual decompression + TileMaxSim with the centroid and the residual parts of every doc
// token taken by two MMAs.  Replaces the reference's wmma kernel (tile_maxsim_fused_decomp.cu:
// 125-229); the score of a passage is
//   score(pid) = sum_r max_t (q_r . c_t + q_r . w_t) * dinv_t
// where c_t = centroid[code_t] (fp16), w_t = the bucket weights of its 2-bit residuals (fp16,
// exact), dinv_t = 1 / sqrt(|fp16(c_t + w_t)|^2 + 1e-12) computed at index bind with the
// reference's fp16 addition.  The reference dots q with fp16(c_t + w_t); here the sum is kept in
// fp32, which moves a score by about 1e-5 relative (under 1e-4 on the benchmark corpus) and no
// further than 2^-11 |q| |d| per dot.
//
// Warp-specialised pipeline, one CTA per SM, cpc = 256 (or 128) candidates per CTA in 4 streams
// (stream q = candidates q, q+4, ...; chunks of 32 tokens, one candidate per chunk).  Tile k of
// the CTA holds chunk k of every stream (128 tokens), stream q in rows / tensor-memory lanes
// 32q..32q+31:
//   * 8 decoder warps (warp w: lane quadrant w % 4, tiles of parity w / 4).  Two tiles ahead, a
//     decoder copies its chunk's centroid rows (16-byte cp.async per piece, codes loaded a tile
//     earlier) straight into its quadrant's rows of a 128-byte-swizzled K-major shared-memory
//     tile: the MMA's A operand, in a ring of 4 tiles.  For the current tile it loads the
//     chunk's residual bytes into registers (32 B per token, lane = token), expands them through
//     a replicated byte LUT to the 128 bucket weights and writes them to tensor memory.
//   * 2 MMA threads (one warp each, so the two issue streams run in parallel: the tensor-core
//     instruction stream, not its arithmetic, bounds a tile of N = 32): per tile D1 = C.Q^T (A
//     from shared memory) and D2 = W.Q^T (A from tensor memory), into one of 4 accumulator slot
//     pairs.
//   * 4 epilogue warps (quadrant w % 4): tcgen05.ld of the chunk's 32 tokens x 32 rows of D1
//     and D2, their sum scaled by dinv, max over tokens per row (redux.sync.max.f32), running max per candidate, sum
//     over rows after the candidate's last chunk.
// mbarriers: afull / aempty per decoder parity (the tile's gathered rows and its weights; both
// MMA threads release it), dfull / dempty per accumulator slot pair.  All waits are bounded; a timeout raises the device error flag, every
// role leaves its loop, copies and MMAs in flight are awaited (bounded) and tensor memory is
// freed.
#include "common.cuh"
#include "s4_common.cuh"
#include "tc.cuh"

namespace ragrt {

constexpr int kGcDecWarps = 8;                               // warps 0..7
constexpr int kGcMmaWarp = kGcDecWarps;                      // warps 8 (C . Q^T) and 9 (W . Q^T)
constexpr int kGcEpiWarp0 = kGcMmaWarp + 2;                  // warps 10..13
constexpr int kGcThreads = (kGcEpiWarp0 + 4) * 32;           // 448
constexpr int kGcCand = 256;
constexpr int kGcStreams = 4;
constexpr int kGcStages = 4;
constexpr int kGcASlots = 2, kGcDSlots = 4;
constexpr uint32_t kGcColA = 0;                              // residual slot a: columns 64 a
constexpr uint32_t kGcColD = 128;                            // accumulator slot d: D1 at 128 + 64 d, D2 32 further
constexpr uint32_t kGcTmemCols = 512;
constexpr uint32_t kGcWaitLimit = 1u << 24;                  // polls before a wait is declared failed
constexpr int kGcLutCopies = 16;

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kGcCBytes = 128 * 256;                         // one gathered tile: 128 rows x 128 fp16, SW128
constexpr int kGcSmC = 0;
constexpr int kGcSmQ = kGcSmC + kGcStages * kGcCBytes;       // 32 rows x 256 B, SW128 K-major
constexpr int kGcSmLut = kGcSmQ + 8192;                      // [256][16] uint2
constexpr int kGcSmMetaT = kGcSmLut + 256 * kGcLutCopies * 8;
constexpr int kGcSmMetaL = kGcSmMetaT + kGcCand * 8;
constexpr int kGcSmTab = kGcSmMetaL + kGcCand * 4;           // rbm [256], decomp [1024], bw [4] fp16
constexpr int kGcSmChunks = kGcSmTab + 256 + 1024 + 16;
constexpr int kGcSmBar = kGcSmChunks + 16;
constexpr int kGcNumBars = 2 * kGcASlots + 2 * kGcDSlots;
constexpr int kGcSmTmem = kGcSmBar + 8 * kGcNumBars;
constexpr int kGcSmAbort = kGcSmTmem + 4;
constexpr int kGcSmBytes = kGcSmAbort + 4;
constexpr int kGcSmDynamic = kGcSmBytes + 1024;

namespace {
struct GcCursor {
    int ci;        // candidate slot (kGcCand once the stream is exhausted)
    int pos;       // first token of the chunk
    int L;
    int64_t tstart;
};
}  // namespace

__global__ void __launch_bounds__(kGcThreads, 1)
s4_gc(const __half* __restrict__ Q, const int32_t* __restrict__ pids, int n, int cpc, S4Docs D,
      float* __restrict__ out, int* __restrict__ err) {
    extern __shared__ uint8_t gc_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)gc_raw + 1023) & ~(uintptr_t)1023);
    uint2* lut = reinterpret_cast<uint2*>(sm + kGcSmLut);
    int64_t* meta_t = reinterpret_cast<int64_t*>(sm + kGcSmMetaT);
    int32_t* meta_l = reinterpret_cast<int32_t*>(sm + kGcSmMetaL);
    uint8_t* tab_rbm = sm + kGcSmTab;
    uint8_t* tab_dec = tab_rbm + 256;
    __half* tab_bw = reinterpret_cast<__half*>(tab_dec + 1024);
    int* s_chunks = reinterpret_cast<int*>(sm + kGcSmChunks);
    uint64_t* afull = reinterpret_cast<uint64_t*>(sm + kGcSmBar);
    uint64_t* aempty = afull + kGcASlots;
    uint64_t* dfull = aempty + kGcASlots;
    uint64_t* dempty = dfull + kGcDSlots;
    uint32_t* tbase_s = reinterpret_cast<uint32_t*>(sm + kGcSmTmem);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + kGcSmAbort);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y;
    const int64_t cbase = (int64_t)blockIdx.x * cpc;

    // ---- codec tables, the candidates' metadata and trivial outputs, Q, barriers, tensor memory
    for (int i = tid; i < 256; i += kGcThreads) tab_rbm[i] = D.rbm[i];
    for (int i = tid; i < 1024; i += kGcThreads) tab_dec[i] = D.decomp[i];
    if (tid < 4) tab_bw[tid] = D.bw[tid];
    for (int ci = tid; ci < kGcCand; ci += kGcThreads) {
        int L = -1;
        int64_t ts = 0;
        if (ci < cpc && cbase + ci < n) {
            const int64_t slot = (int64_t)b * n + cbase + ci;
            const int32_t pid = pids[slot];
            if (pid < 0 || pid >= D.N) {
                out[slot] = -INFINITY;
            } else {
                L = D.doc_lens[pid];
                ts = D.doc_offsets[pid];
                if (L <= 0) out[slot] = -3.2e10f;    // 32 rows x the -1e9 running-max start
            }
        }
        meta_t[ci] = ts;
        meta_l[ci] = L;
    }
    const __half* Qb = Q + (int64_t)b * kRows * kDim;
    for (int i = tid; i < kRows * 16; i += kGcThreads) {
        const int row = i >> 4, c16 = i & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(Qb + row * kDim + c16 * 8);
        *reinterpret_cast<uint4*>(sm + kGcSmQ + tc::sw128_offset(row, c16, kRows)) = v;
    }
    if (tid == 0) {
        for (int i = 0; i < kGcASlots; ++i) {
            tc::mbar_init(afull + i, 4);
            tc::mbar_init(aempty + i, 2);
        }
        for (int i = 0; i < kGcDSlots; ++i) {
            tc::mbar_init(dfull + i, 2);
            tc::mbar_init(dempty + i, 4);
        }
        *abort = 0;
        tc::mbar_fence_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tbase_s, kGcTmemCols);
        tc::tmem_relinquish();
    }
    __syncthreads();
    for (int i = tid; i < 256 * kGcLutCopies; i += kGcThreads) {
        const int byte = i / kGcLutCopies;
        const int rev = tab_rbm[byte];
        __half wv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) wv[u] = tab_bw[tab_dec[rev * 4 + u] & 3];
        lut[i] = *reinterpret_cast<uint2*>(wv);
    }
    if (warp < kGcStreams) {                 // chunks per stream (warp q sums stream q)
        int c = 0;
        for (int ci = warp + kGcStreams * lane; ci < kGcCand; ci += kGcStreams * 32) {
            const int L = meta_l[ci];
            c += L > 0 ? (L + 31) >> 5 : 0;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
        if (lane == 0) s_chunks[warp] = c;
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tbase_s;
    const int n_tiles = max(max(s_chunks[0], s_chunks[1]), max(s_chunks[2], s_chunks[3]));
    bool bad_code = false, failed = false;

    // stream q, chunk by chunk
    auto advance = [&](GcCursor& c, int q) {
        c.pos += 32;
        if (c.ci >= 0 && c.ci < kGcCand && c.pos < c.L) return;
        for (;;) {
            c.ci = c.ci < 0 ? q : c.ci + kGcStreams;
            c.pos = 0;
            if (c.ci >= kGcCand) {
                c.ci = kGcCand;
                c.L = 0;
                return;
            }
            const int L = meta_l[c.ci];
            if (L <= 0) continue;
            c.L = L;
            c.tstart = meta_t[c.ci];
            return;
        }
    };

    if (warp < kGcDecWarps) {
        // ================================================================ decoders
        const int q = warp & 3, par = warp >> 2;
        const uint32_t tq = tbase + ((uint32_t)(32 * q) << 16) + kGcColA + (uint32_t)(par * 64);
        const int lc = lane & (kGcLutCopies - 1);
        const int l16 = lane & 15, hh = lane >> 4;
        // the load is only issued here; its value is checked where it is used
        auto load_code = [&](const GcCursor& x) {
            return (x.ci < kGcCand && x.pos + lane < x.L) ? D.codes[x.tstart + x.pos + lane] : 0;
        };
        // the chunk's centroid rows into this quadrant's rows of gather stage st (one commit group)
        auto issue = [&](const GcCursor& x, int code, int st) {
            if (x.ci < kGcCand) {
                const int ntv = min(32, x.L - x.pos);
                if ((unsigned)code >= (unsigned)D.NC) { bad_code = true; code = 0; }   // never gather outside C
                uint8_t* dst = sm + kGcSmC + st * kGcCBytes;
#pragma unroll 4
                for (int i = 0; i < 16; ++i) {
                    const int t = 2 * i + hh;
                    const int ct = __shfl_sync(0xFFFFFFFFu, code, t);
                    if (t < ntv)
                        tc::cp_async16(dst + tc::sw128_offset(32 * q + t, l16, 128),
                                       D.centroids + (int64_t)ct * kDim + l16 * 8);
                }
            }
            tc::cp_async_commit();
        };
        auto load_res = [&](const GcCursor& x, uint4& r0, uint4& r1) {
            if (x.ci < kGcCand && x.pos + lane < x.L) {
                const uint4* src = reinterpret_cast<const uint4*>(D.residuals + (x.tstart + x.pos + lane) * 32);
                r0 = src[0];
                r1 = src[1];
            } else {
                r0 = make_uint4(0u, 0u, 0u, 0u);
                r1 = r0;
            }
        };
        GcCursor c{-1, -32, 0, 0};
        advance(c, q);
        if (par) advance(c, q);
        GcCursor cn = c;
        advance(cn, q);
        advance(cn, q);
        issue(c, load_code(c), par);                      // tile par into stage par
        int code_n = load_code(cn);
        uint4 r0, r1;
        load_res(c, r0, r1);
        for (int k = par; k < n_tiles; k += 2) {
            // the MMAs of tile k - 2 are done with this parity's weight slot and with gather
            // stage (k + 2) % 4, which the copies for tile k + 2 now fill
            if (k >= 2 && !tc::mbar_wait_or_abort(aempty + par, ((k - 2) >> 1) & 1, abort, kGcWaitLimit)) {
                failed = true;
                break;
            }
            tc::fence_after();
            issue(cn, code_n, (k + 2) % kGcStages);
            GcCursor cnn = cn;
            advance(cnn, q);
            advance(cnn, q);
            const int code_nn = load_code(cnn);
            uint4 n0, n1;
            load_res(cn, n0, n1);                         // the next tile's residuals, in flight meanwhile
            if (c.ci < kGcCand) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint4 rr = half ? r1 : r0;
                    const uint32_t rw[4] = {rr.x, rr.y, rr.z, rr.w};
                    uint32_t a[32];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {        // byte j: dims 4j..4j+3 of this half
                        const uint32_t by = (rw[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                        const uint2 wv = lut[by * kGcLutCopies + lc];
                        a[2 * j] = wv.x;
                        a[2 * j + 1] = wv.y;
                    }
                    tc::st32x32(tq + half * 32, a);
                }
                tc::wait_st();
            }
            tc::cp_async_wait<1>();                       // tile k's rows (issued an iteration ago) have landed
            tc::fence_proxy_async();
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(afull + par);
            c = cn;
            cn = cnn;
            code_n = code_nn;
            r0 = n0;
            r1 = n1;
        }
        tc::cp_async_wait<0>();                           // no copy may land after the CTA exits
    } else if (warp < kGcEpiWarp0) {
        // ================================================================ MMA issuers
        // warp 8: D1 = C . Q^T (A: the gathered rows in shared memory); warp 9: D2 = W . Q^T
        // (A: the weights in tensor memory).  Each commits to aempty and dfull (count 2 each).
        const bool wpart = warp == kGcMmaWarp + 1;
        if (lane == 0) {
            const uint32_t sQ = tc::smem_u32(sm + kGcSmQ), sC = tc::smem_u32(sm + kGcSmC);
            constexpr uint32_t idesc = tc::idesc_f16_f32(128, 32);
            int issued = 0;
            for (int k = 0; k < n_tiles; ++k) {
                const int s = k % kGcStages, a = k & 1, d = k & 3;
                if (!tc::mbar_wait_or_abort(afull + a, (k >> 1) & 1, abort, kGcWaitLimit) ||
                    (k >= kGcDSlots && !tc::mbar_wait_or_abort(dempty + d, ((k >> 2) - 1) & 1, abort, kGcWaitLimit))) {
                    failed = true;
                    break;
                }
                tc::fence_after();
                const uint32_t td = tbase + kGcColD + (uint32_t)(d * 64) + (wpart ? 32u : 0u);
                if (!wpart) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t koffC = (uint32_t)((kk >> 2) * (128 * 128) + (kk & 3) * 32);
                        const uint32_t koffQ = (uint32_t)((kk >> 2) * (kRows * 128) + (kk & 3) * 32);
                        tc::mma_ss(td, tc::sw128_kmajor_desc(sC + s * kGcCBytes + koffC),
                                   tc::sw128_kmajor_desc(sQ + koffQ), idesc, kk > 0);
                    }
                } else {
                    const uint32_t ta = tbase + kGcColA + (uint32_t)(a * 64);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t koffQ = (uint32_t)((kk >> 2) * (kRows * 128) + (kk & 3) * 32);
                        tc::mma_ts(td, ta + 8 * kk, tc::sw128_kmajor_desc(sQ + koffQ), idesc, kk > 0);
                    }
                }
                tc::mma_commit(aempty + a);
                tc::mma_commit(dfull + d);
                issued = k + 1;
            }
            if (failed && issued > 0)                    // let the last MMAs finish before memory is freed
                (void)tc::mbar_wait_bounded(dfull + ((issued - 1) & 3), ((issued - 1) >> 2) & 1, kGcWaitLimit);
        }
        __syncwarp();
    } else {
        // ================================================================ epilogue
        const int q = warp & 3;
        GcCursor e{-1, -32, 0, 0};
        advance(e, q);
        auto load_inv = [&](const GcCursor& x) {
            return (x.ci < kGcCand && x.pos + lane < x.L) ? D.dinv[x.tstart + x.pos + lane] : 0.f;
        };
        float inv = load_inv(e);
        float run_max = -1e9f;
        for (int k = 0; k < n_tiles; ++k) {
            const int d = k & 3;
            GcCursor en = e;
            advance(en, q);
            const float inv_n = load_inv(en);
            if (!tc::mbar_wait_or_abort(dfull + d, (k >> 2) & 1, abort, kGcWaitLimit)) { failed = true; break; }
            tc::fence_after();
            uint32_t acc[32], acc2[32];
            const uint32_t tdq = tbase + kGcColD + (uint32_t)(d * 64) + ((uint32_t)(32 * q) << 16);
            tc::ld32x32(tdq, acc);
            tc::ld32x32(tdq + 32, acc2);
            tc::wait_ld();
#pragma unroll
            for (int r = 0; r < 32; ++r) acc[r] = __float_as_uint(__uint_as_float(acc[r]) + __uint_as_float(acc2[r]));
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(dempty + d);
            if (e.ci < kGcCand) {
                const bool valid = e.pos + lane < e.L;
                float mine = -INFINITY;
                if (e.pos + 32 <= e.L) {                         // full chunk: no token to mask
#pragma unroll
                    for (int r = 0; r < 32; ++r) {
                        const float mx = tc::warp_max_f32(__uint_as_float(acc[r]) * inv);
                        mine = (lane == r) ? mx : mine;
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < 32; ++r) {
                        const float v = valid ? __uint_as_float(acc[r]) * inv : -INFINITY;
                        const float mx = tc::warp_max_f32(v);
                        mine = (lane == r) ? mx : mine;
                    }
                }
                run_max = fmaxf(run_max, mine);
                if (e.pos + 32 >= e.L) {
                    float s_ = run_max;
#pragma unroll
                    for (int o = 16; o; o >>= 1) s_ += __shfl_xor_sync(0xFFFFFFFFu, s_, o);
                    if (lane == 0) out[(int64_t)b * n + cbase + e.ci] = s_;
                    run_max = -1e9f;
                }
            }
            e = en;
            inv = inv_n;
        }
    }
    if (failed && lane == 0) atomicExch(err, 1);
    if (__any_sync(0xFFFFFFFFu, bad_code) && lane == 0) atomicExch(err, 2);
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(*tbase_s, kGcTmemCols);
    }
}

int s4_gc_launch(const __half* Q, const int32_t* pids, int B, int n, const S4Docs& D, float* out,
                 cudaStream_t stream) {
    if (B <= 0 || n <= 0) return RAGRT_OK;
    if (!D.dinv) return fail(RAGRT_ERR_ARG, "internal: stage-4 gather kernel needs the index's token norms");
    int* d_err = device_error_flag();
    if (!d_err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
    static_assert(kGcSmBytes + 1024 <= kGcSmDynamic, "shared memory map exceeds the allocation");
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s4_gc, cudaFuncAttributeMaxDynamicSharedMemorySize, kGcSmDynamic));
    // candidates per CTA: 256, or 128 when that fills the last wave of CTAs (one per SM) clearly better
    const int sms = num_sms();
    auto waste = [&](int cpc) {
        const int64_t ctas = ceil_div((int64_t)n, (int64_t)cpc) * B;
        return (double)(ceil_div(ctas, (int64_t)sms) * sms) / (double)ctas - 1.0;
    };
    const int cpc = waste(kGcCand / 2) < waste(kGcCand) - 0.03 ? kGcCand / 2 : kGcCand;
    dim3 grid((unsigned)ceil_div(n, cpc), (unsigned)B);
    s4_gc<<<grid, kGcThreads, kGcSmDynamic, stream>>>(Q, pids, n, cpc, D, out, d_err);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
