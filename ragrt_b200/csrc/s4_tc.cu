// s4_tc.cu -- Stage 4 on the 5th-generation tensor cores (tcgen05 + tensor memory): fused
// 2-bit residual decompression + TileMaxSim.  Replaces the reference's wmma kernel
// (tile_maxsim_fused_decomp.cu:125-229), same result definition:
//   score(pid) = sum_r max_t (q_r . d_t) * rsqrt(|d_t|^2 + 1e-12)
// with d_t = fp16(centroid[code_t] + bucket_weight[bucket of dim]) per dim.
//
// Warp-specialised pipeline, one CTA per SM, cpc = 256 (or 128) candidates per CTA in 4 streams
// (stream q = candidates q, q+4, ...; chunks of 32 tokens, one candidate per chunk).  Tile k of the
// CTA holds chunk k of every stream, stream q in tensor-memory lane quadrant q:
//   * 8 decoder warps (warp w: quadrant w % 4, tiles k = w / 4 mod 2).  For its next chunk a
//     decoder issues coalesced 16-byte cp.async copies (a half-warp per 256-byte centroid
//     row) into a padded shared-memory staging buffer, then decodes its current chunk with
//     lane = token: d = hadd(centroid, LUT[residual byte]) (16-way replicated byte LUT),
//     written to tensor memory with tcgen05.st (the decoder's A slot), and d*d (A2).
//   * 2 MMA threads (one warp each, so both issue streams run in parallel): per tile, with A
//     from tensor memory, D = A.Q^T (N = 32) and D2 = A2.1 (N = 16; column 0 = |d|^2, fp16
//     squares summed in fp32) into one of 4 accumulator slots.
//   * 4 epilogue warps (quadrant q): tcgen05.ld of the chunk's 32 tokens x 32 query rows,
//     scale by rsqrt(|d|^2 + 1e-12), max over tokens per row (redux.sync.max.f32), running
//     max per candidate, sum over rows after the candidate's last chunk.
// mbarriers: afull[2] (decoders -> MMA), aempty[2] (both MMA streams done reading A), dfull[4]
// (MMA -> epilogue), dempty[4] (epilogue done reading D; awaited by the MMA threads).  All waits are bounded; a timeout raises
// the device error flag, every role leaves its loop, copies and MMAs in flight are awaited
// (bounded) and tensor memory is freed.
#include "common.cuh"
#include "s4_common.cuh"
#include "tc.cuh"

namespace ragrt {

constexpr int kDecWarps = 8;
constexpr int kMmaWarp = kDecWarps;                   // warps 8 (dots) and 9 (norms)
constexpr int kTcThreads = (kDecWarps + 2 + 4) * 32;  // 448
constexpr int kTcCandPerCta = 256;
constexpr int kStreamsTc = 4;
constexpr int kASlots = 2, kDSlots = 4;
constexpr uint32_t kColA = 0;                         // A slot a: columns 128 a: A (64), A2 (64)
constexpr uint32_t kColA2 = 64;                       // inside an A slot
constexpr uint32_t kColD = 256;                       // D slot d: columns 256 + 64 d: 32 dots, D2 (16)
constexpr uint32_t kColNorm = 32;                     // inside a D slot
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kWaitLimit = 1u << 24;             // polls (or 2 s) before a wait is declared failed
constexpr int kLutCopies = 16;
constexpr int kRowStride = 272;                       // staging row: 256 B + 16 B padding (conflict free)
constexpr int kStageBytes = 32 * kRowStride + 32 * 32;

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kSmQ = 0;                                       // 32 rows x 256 B, SW128 K-major
constexpr int kSmOnes = 8192;                                 // 16 rows x 256 B of fp16 1.0
constexpr int kSmStage = 12288;                               // [8 decoders][2] staging buffers
constexpr int kSmLut = kSmStage + kDecWarps * 2 * kStageBytes;       // [256][16] uint2
constexpr int kSmMetaT = kSmLut + 256 * kLutCopies * 8;       // [256] int64 first token
constexpr int kSmMetaL = kSmMetaT + kTcCandPerCta * 8;        // [256] int32 length (<= 0: no work)
constexpr int kSmTab = kSmMetaL + kTcCandPerCta * 4;          // rbm [256], decomp [1024], bw [4] fp16
constexpr int kSmChunks = kSmTab + 256 + 1024 + 16;           // [4] chunks per stream
constexpr int kSmBar = kSmChunks + 16;                        // afull[2] aempty[2] dfull[4] dempty[4]
constexpr int kNumBars = 2 * kASlots + 2 * kDSlots;
constexpr int kSmTmem = kSmBar + 8 * kNumBars;
constexpr int kSmAbort = kSmTmem + 4;
constexpr int kSmBytes = kSmAbort + 4;
constexpr int kSmDynamic = kSmBytes + 1024;

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hadd2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a) {
    __half2 x = *reinterpret_cast<__half2*>(&a);
    __half2 r = __hmul2(x, x);
    return *reinterpret_cast<uint32_t*>(&r);
}

// A stream's position: candidate `ci` (kTcCandPerCta once exhausted), token offset `pos`.
struct Cursor {
    int ci;
    int pos;
    int L;
    int64_t tstart;
};

// kRaw: exact MaxSim over raw fp16 embeddings (D.emb): the decoders copy the doc's own rows
// (no codes, residuals or LUT) and the epilogue does not normalise.
template <bool kRaw>
__global__ void __launch_bounds__(kTcThreads, 1)
s4_tc(const __half* __restrict__ Q, const int32_t* __restrict__ pids, int n, int cpc, S4Docs D,
      float* __restrict__ out, int* __restrict__ err) {
    extern __shared__ uint8_t s4_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)s4_raw + 1023) & ~(uintptr_t)1023);
    uint2* lut = reinterpret_cast<uint2*>(sm + kSmLut);
    int64_t* meta_t = reinterpret_cast<int64_t*>(sm + kSmMetaT);
    int32_t* meta_l = reinterpret_cast<int32_t*>(sm + kSmMetaL);
    uint8_t* tab_rbm = sm + kSmTab;
    uint8_t* tab_dec = tab_rbm + 256;
    __half* tab_bw = reinterpret_cast<__half*>(tab_dec + 1024);
    int* s_chunks = reinterpret_cast<int*>(sm + kSmChunks);
    uint64_t* afull = reinterpret_cast<uint64_t*>(sm + kSmBar);
    uint64_t* aempty = afull + kASlots;
    uint64_t* dfull = aempty + kASlots;
    uint64_t* dempty = dfull + kDSlots;
    uint32_t* tbase_s = reinterpret_cast<uint32_t*>(sm + kSmTmem);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + kSmAbort);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y;
    const int64_t cbase = (int64_t)blockIdx.x * cpc;     // this CTA: candidates cbase .. cbase + cpc - 1

    // ---- stage the codec tables and the candidates' metadata; trivial outputs
    if constexpr (!kRaw) {
        for (int i = tid; i < 256; i += kTcThreads) tab_rbm[i] = D.rbm[i];
        for (int i = tid; i < 1024; i += kTcThreads) tab_dec[i] = D.decomp[i];
        if (tid < 4) tab_bw[tid] = D.bw[tid];
    }
    for (int ci = tid; ci < kTcCandPerCta; ci += kTcThreads) {
        int L = -1;                                       // slots past cpc stay empty
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
    for (int i = tid; i < 256; i += kTcThreads)
        reinterpret_cast<uint4*>(sm + kSmOnes)[i] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    const __half* Qb = Q + (int64_t)b * kRows * kDim;
    for (int i = tid; i < kRows * 16; i += kTcThreads) {
        const int row = i >> 4, c16 = i & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(Qb + row * kDim + c16 * 8);
        *reinterpret_cast<uint4*>(sm + kSmQ + tc::sw128_offset(row, c16, kRows)) = v;
    }
    if (tid == 0) {
        for (int i = 0; i < kASlots; ++i) {
            tc::mbar_init(afull + i, 4);
            tc::mbar_init(aempty + i, 2);
        }
        for (int i = 0; i < kDSlots; ++i) {
            tc::mbar_init(dfull + i, 2);
            tc::mbar_init(dempty + i, 4);
        }
        *abort = 0;
        tc::mbar_fence_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tbase_s, kTmemCols);
        tc::tmem_relinquish();
    }
    __syncthreads();
    for (int i = tid; i < (kRaw ? 0 : 256 * kLutCopies); i += kTcThreads) {
        const int byte = i / kLutCopies;
        const int rev = tab_rbm[byte];
        __half wv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) wv[u] = tab_bw[tab_dec[rev * 4 + u] & 3];
        lut[i] = *reinterpret_cast<uint2*>(wv);
    }
    if (warp < kStreamsTc) {                 // chunks per stream (warp q sums stream q)
        int c = 0;
        for (int ci = warp + kStreamsTc * lane; ci < kTcCandPerCta; ci += kStreamsTc * 32) {
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

    // stream q, chunk by chunk (step = chunks to skip per call)
    auto advance = [&](Cursor& c, int q) {
        c.pos += 32;
        if (c.ci >= 0 && c.ci < kTcCandPerCta && c.pos < c.L) return;
        for (;;) {
            c.ci = c.ci < 0 ? q : c.ci + kStreamsTc;
            c.pos = 0;
            if (c.ci >= kTcCandPerCta) {
                c.ci = kTcCandPerCta;
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

    if (warp < kDecWarps) {
        // ================================================================ decoders
        const int q = warp & 3, par = warp >> 2;
        const uint32_t tq = tbase + ((uint32_t)(32 * q) << 16) + kColA + (uint32_t)(par * 128);   // A slot = par
        uint8_t* stg = sm + kSmStage + warp * 2 * kStageBytes;
        // the load is only issued here; its value is checked where it is used
        auto load_code = [&](const Cursor& c) {
            if constexpr (kRaw) return 0;
            return (c.ci < kTcCandPerCta && c.pos + lane < c.L) ? D.codes[c.tstart + c.pos + lane] : 0;
        };
        // coalesced cp.async of chunk c into staging buffer bf (one commit group, maybe empty)
        auto issue = [&](const Cursor& c, int code_c, int bf) {
            if (c.ci < kTcCandPerCta) {
                const int ntv = min(32, c.L - c.pos);
                if constexpr (!kRaw) {
                    if ((unsigned)code_c >= (unsigned)D.NC) { bad_code = true; code_c = 0; }   // never gather outside C
                }
                uint8_t* dst = stg + bf * kStageBytes;
                const int hh = lane >> 4, l16 = lane & 15;
#pragma unroll 4
                for (int i = 0; i < 16; ++i) {
                    const int t = 2 * i + hh;
                    if constexpr (kRaw) {
                        if (t < ntv)
                            tc::cp_async16(dst + t * kRowStride + l16 * 16, D.emb + (c.tstart + c.pos + t) * kDim + l16 * 8);
                    } else {
                        const int code = __shfl_sync(0xFFFFFFFFu, code_c, t);
                        if (t < ntv)
                            tc::cp_async16(dst + t * kRowStride + l16 * 16,
                                           D.centroids + (int64_t)code * kDim + l16 * 8);
                    }
                }
                if constexpr (kRaw) {
                    tc::cp_async_commit();
                    return;
                }
                const uint8_t* res = D.residuals + (c.tstart + c.pos) * 32;
                uint8_t* rdst = dst + 32 * kRowStride;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int off = (j * 32 + lane) * 16;             // 64 pieces of 16 B = 32 tokens
                    if ((off >> 5) < ntv) tc::cp_async16(rdst + off, res + off);
                }
            }
            tc::cp_async_commit();
        };
        Cursor c{-1, -32, 0, 0};
        advance(c, q);
        if (par) advance(c, q);
        int code_c = load_code(c);
        issue(c, code_c, 0);
        Cursor cn = c;
        advance(cn, q);
        advance(cn, q);
        int code_n = load_code(cn);
        int bf = 0;
        for (int k = par; k < n_tiles; k += 2) {
            issue(cn, code_n, bf ^ 1);
            Cursor cnn = cn;
            advance(cnn, q);
            advance(cnn, q);
            const int code_nn = load_code(cnn);
            tc::cp_async_wait<1>();
            __syncwarp();
            // the MMAs of this slot's previous tile (k - 2) have finished reading A
            if (k >= 2 && !tc::mbar_wait_or_abort(aempty + par, ((k - 2) >> 1) & 1, abort, kWaitLimit)) {
                failed = true;
                break;
            }
            tc::fence_after();
            if (c.ci < kTcCandPerCta) {
                const bool valid = c.pos + lane < c.L;
                const uint8_t* row = stg + bf * kStageBytes + lane * kRowStride;
                const uint8_t* rsd = stg + bf * kStageBytes + 32 * kRowStride + lane * 32;
                const int lc = lane & (kLutCopies - 1);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t a[32];
                    const uint4 rr = *reinterpret_cast<const uint4*>(rsd + half * 16);
                    const uint32_t rw[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {        // 8 dims = 2 residual bytes per step
                        const uint4 cv = *reinterpret_cast<const uint4*>(row + (half * 8 + cc) * 16);
                        if constexpr (kRaw) {
                            a[4 * cc + 0] = cv.x;
                            a[4 * cc + 1] = cv.y;
                            a[4 * cc + 2] = cv.z;
                            a[4 * cc + 3] = cv.w;
                            continue;
                        }
                        const uint32_t word = rw[cc >> 1];
                        const uint32_t by0 = __byte_perm(word, 0u, 0x4440u + (cc & 1) * 2);
                        const uint32_t by1 = __byte_perm(word, 0u, 0x4441u + (cc & 1) * 2);
                        const uint2 w0 = lut[by0 * kLutCopies + lc], w1 = lut[by1 * kLutCopies + lc];
                        a[4 * cc + 0] = hadd2_u32(cv.x, w0.x);
                        a[4 * cc + 1] = hadd2_u32(cv.y, w0.y);
                        a[4 * cc + 2] = hadd2_u32(cv.z, w1.x);
                        a[4 * cc + 3] = hadd2_u32(cv.w, w1.y);
                    }
                    if (c.pos + 32 > c.L && !valid) {              // only the last chunk of a candidate
#pragma unroll
                        for (int j = 0; j < 32; ++j) a[j] = 0u;
                    }
                    tc::st32x32(tq + half * 32, a);
                    if constexpr (!kRaw) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) a[j] = hmul2_u32(a[j]);
                        tc::st32x32(tq + kColA2 + half * 32, a);
                    }
                }
                tc::wait_st();
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(afull + par);
            c = cn;
            cn = cnn;
            code_n = code_nn;
            bf ^= 1;
        }
        tc::cp_async_wait<0>();                 // no copy may land after the CTA exits
    } else if (warp < kMmaWarp + 2) {
        // ================================================================ MMA issuers
        // warp 8: D = A.Q^T; warp 9: D2 = A2.1 (|d|^2).  Each commits to aempty and dfull
        // (count 2 each).  In exact mode (no normalisation) warp 9 only keeps the protocol.
        const bool norms = warp == kMmaWarp + 1;
        if (lane == 0) {
            const uint32_t sQ = tc::smem_u32(sm + kSmQ), sOnes = tc::smem_u32(sm + kSmOnes);
            constexpr uint32_t idD = tc::idesc_f16_f32(128, 32);
            constexpr uint32_t idD2 = tc::idesc_f16_f32(128, 16);
            int issued = 0;
            for (int k = 0; k < n_tiles; ++k) {
                const int a = k & 1, d = k & 3;
                if (!tc::mbar_wait_or_abort(afull + a, (k >> 1) & 1, abort, kWaitLimit)) { failed = true; break; }
                if (k >= kDSlots && !tc::mbar_wait_or_abort(dempty + d, ((k >> 2) - 1) & 1, abort, kWaitLimit)) {
                    failed = true;
                    break;
                }
                tc::fence_after();
                const uint32_t ta = tbase + kColA + (uint32_t)(a * 128), td = tbase + kColD + (uint32_t)(d * 64);
                if (!norms) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t koff = (uint32_t)((kk >> 2) * (kRows * 128) + (kk & 3) * 32);
                        tc::mma_ts(td, ta + 8 * kk, tc::sw128_kmajor_desc(sQ + koff), idD, kk > 0);
                    }
                } else if (!kRaw) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t koff = (uint32_t)((kk >> 2) * (16 * 128) + (kk & 3) * 32);
                        tc::mma_ts(td + kColNorm, ta + kColA2 + 8 * kk, tc::sw128_kmajor_desc(sOnes + koff), idD2,
                                   kk > 0);
                    }
                }
                tc::mma_commit(aempty + a);
                tc::mma_commit(dfull + d);
                issued = k + 1;
            }
            if (failed && issued > 0)                // let the last MMAs finish before memory is freed
                (void)tc::mbar_wait_bounded(dfull + ((issued - 1) & 3), ((issued - 1) >> 2) & 1, kWaitLimit);
        }
        __syncwarp();
    } else {
        // ================================================================ epilogue
        const int q = warp & 3;                  // warps 10..13 -> quadrants 2, 3, 0, 1
        Cursor e{-1, -32, 0, 0};
        advance(e, q);
        float run_max = -1e9f;
        for (int k = 0; k < n_tiles; ++k) {
            const int d = k & 3;
            if (!tc::mbar_wait_or_abort(dfull + d, (k >> 2) & 1, abort, kWaitLimit)) { failed = true; break; }
            tc::fence_after();
            const uint32_t td = tbase + kColD + (uint32_t)(d * 64) + ((uint32_t)(32 * q) << 16);
            uint32_t acc[32];
            tc::ld32x32(td, acc);
            const float ssv = __uint_as_float(tc::ld32x1(td + kColNorm));
            tc::wait_ld();
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(dempty + d);
            if (e.ci < kTcCandPerCta) {
                const bool valid = e.pos + lane < e.L;
                const float inv = kRaw ? 1.0f : rsqrtf(ssv + 1e-12f);
                float mine = -INFINITY;
                const float sc = valid ? inv : 0.f;
                if (e.pos + 32 <= e.L) {                         // full chunk: no token to mask
#pragma unroll
                    for (int r = 0; r < 32; ++r) {
                        const float mx = tc::warp_max_f32(__uint_as_float(acc[r]) * sc);
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
            advance(e, q);
        }
    }
    if (failed && lane == 0) atomicExch(err, 1);
    if (__any_sync(0xFFFFFFFFu, bad_code) && lane == 0) atomicExch(err, 2);
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(*tbase_s, kTmemCols);
    }
}

int s4_tc_launch(const __half* Q, const int32_t* pids, int B, int n, const S4Docs& D, float* out,
                 cudaStream_t stream) {
    if (B <= 0 || n <= 0) return RAGRT_OK;
    int* d_err = device_error_flag();
    if (!d_err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
    static_assert(kSmBytes + 1024 <= kSmDynamic, "shared memory map exceeds the allocation");
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s4_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmDynamic));
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s4_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmDynamic));
    // candidates per CTA: 256, or 128 when that fills the last wave of CTAs (one per SM)
    // clearly better (small per-shard candidate counts)
    const int sms = num_sms();
    auto waste = [&](int cpc) {
        const int64_t ctas = ceil_div((int64_t)n, (int64_t)cpc) * B;
        return (double)(ceil_div(ctas, (int64_t)sms) * sms) / (double)ctas - 1.0;
    };
    const int cpc = waste(kTcCandPerCta / 2) < waste(kTcCandPerCta) - 0.03 ? kTcCandPerCta / 2 : kTcCandPerCta;
    dim3 grid((unsigned)ceil_div(n, cpc), (unsigned)B);
    if (D.emb)
        s4_tc<true><<<grid, kTcThreads, kSmDynamic, stream>>>(Q, pids, n, cpc, D, out, d_err);
    else
        s4_tc<false><<<grid, kTcThreads, kSmDynamic, stream>>>(Q, pids, n, cpc, D, out, d_err);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
