// s4_tc.cu -- Stage 4 on the 5th-generation tensor cores (tcgen05 + tensor memory): fused
// 2-bit residual decompression + TileMaxSim.  Replaces the reference's wmma kernel
// (tile_maxsim_fused_decomp.cu:125-229), same result definition:
//   score(pid) = sum_r max_t (q_r . d_t) * rsqrt(|d_t|^2 + 1e-12)
//
// One MMA tile = M 128 doc tokens x N 32 query rows x K 128 dims:
//   * A = decoded doc tokens, written from registers straight into TENSOR MEMORY
//     (tcgen05.st): the thread that decodes a token owns its TMEM lane, so decoded tokens
//     never touch shared memory.  Lanes 32q..32q+31 (quadrant q) hold 32 consecutive tokens
//     of ONE candidate of the warp that owns quadrant q.
//   * B = the query's 32 x 128 fp16 rows in shared memory (128-byte swizzle, K-major).
//   * D = 128 x 32 fp32 in tensor memory; each warp reads back its own quadrant.
//   * |d_t|^2 also runs on the tensor core: A2 = d*d (fp16) times a ones matrix (N = 16);
//     column 0 of that accumulator is the squared norm of the lane's token.
// A CTA runs two independent tile groups (4 warps each, 176 TMEM columns each) so one
// group's decode overlaps the other's MMA and epilogue, and every warp software-pipelines
// its gathers: the code of chunk i+2 and the centroid rows / residual bytes of chunk i+1
// are in flight while chunk i is stored, multiplied and reduced.
// Epilogue per warp: scale the 32 dot products of its lane's token by the inverse norm,
// max over the chunk's 32 tokens (= lanes) with redux.sync.max.f32 per query row, a
// running max per candidate in the lane of that row, and the sum over rows when the
// candidate's last chunk is done.  All waits are bounded; a timeout raises the device
// error flag and the CTA exits.
#include "common.cuh"
#include "s4_common.cuh"
#include "tc.cuh"

namespace ragrt {

constexpr int kGroups = 2;
constexpr int kGroupWarps = 4;
constexpr int kTcThreads = kGroups * kGroupWarps * 32;
constexpr int kStreams = kGroups * kGroupWarps;     // candidate streams per CTA (one per warp)
constexpr int kTcCandPerCta = 256;
constexpr uint32_t kColA = 0;      // 64 columns: 128 fp16 dims per token lane
constexpr uint32_t kColA2 = 64;    // 64 columns: squared dims
constexpr uint32_t kColD = 128;    // 32 columns: dot products with the 32 query rows
constexpr uint32_t kColD2 = 160;   // 16 columns: squared norm (column 0)
constexpr uint32_t kGroupCols = 256;
constexpr uint32_t kTmemCols = kGroups * kGroupCols;
constexpr uint32_t kWaitLimit = 1u << 22;           // polls before a wait is declared failed

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kSmQ = 0;            // 32 rows x 256 B, SW128 K-major (two 4 KB atoms)
constexpr int kSmOnes = 8192;      // 16 rows x 256 B of fp16 1.0
constexpr int kSmLut = 12288;      // [256 bytes][32 lanes] uint2: byte -> 4 fp16 bucket weights
constexpr int kSmBar = kSmLut + 256 * 32 * 8;   // kGroups mbarriers
constexpr int kSmTmem = kSmBar + 8 * kGroups;
constexpr int kSmAbort = kSmTmem + 4;
constexpr int kSmBytes = kSmAbort + 4;
constexpr int kSmDynamic = 1024 + 150 * 1024;       // > half an SM: one CTA per SM (it holds all 512 TMEM columns)

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hadd2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a) {
    __half2 x = *reinterpret_cast<__half2*>(&a);
    __half2 r = __hmul2(x, x);
    return *reinterpret_cast<uint32_t*>(&r);
}

// A stream's position: candidate `ci` (index within the CTA's range), token offset `pos`.
struct Cursor {
    int ci;
    int pos;
    int L;
    int64_t slot;
    int64_t tstart;
};

__global__ void __launch_bounds__(kTcThreads, 1)
s4_tc(const __half* __restrict__ Q, const int32_t* __restrict__ pids, int n, S4Docs D, float* __restrict__ out,
      int* __restrict__ err) {
    extern __shared__ uint8_t s4_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)s4_raw + 1023) & ~(uintptr_t)1023);
    uint2* lut = reinterpret_cast<uint2*>(sm + kSmLut);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kSmBar);
    uint32_t* tbase_s = reinterpret_cast<uint32_t*>(sm + kSmTmem);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + kSmAbort);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = warp / kGroupWarps, quad = warp % kGroupWarps;   // warp % 4 == its TMEM lane quadrant
    const int stream = warp;
    const int b = blockIdx.y;
    const int64_t cbase = (int64_t)blockIdx.x * kTcCandPerCta;

    // ---- query tile (SW128 K-major), ones tile, replicated byte LUT, barriers, tensor memory
    const __half* Qb = Q + (int64_t)b * kRows * kDim;
    for (int i = tid; i < kRows * 16; i += kTcThreads) {
        const int row = i >> 4, c16 = i & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(Qb + row * kDim + c16 * 8);
        *reinterpret_cast<uint4*>(sm + kSmQ + tc::sw128_offset(row, c16, kRows)) = v;
    }
    for (int i = tid; i < 256; i += kTcThreads)
        reinterpret_cast<uint4*>(sm + kSmOnes)[i] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    for (int i = tid; i < 256 * 32; i += kTcThreads) {
        const int byte = i >> 5;                     // one copy per lane: no bank conflicts
        const int rev = D.rbm[byte];
        __half wv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) wv[u] = D.bw[D.decomp[rev * 4 + u] & 3];
        lut[i] = *reinterpret_cast<uint2*>(wv);
    }
    if (tid == 0) {
        for (int i = 0; i < kGroups; ++i) tc::mbar_init(mbar + i, 1);
        *abort = 0;
        tc::mbar_fence_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tbase_s, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tbase_s + (uint32_t)(g * kGroupCols);
    const uint32_t tq = tbase + ((uint32_t)(32 * quad) << 16);      // this warp's lane quadrant
    const uint32_t sQ = tc::smem_u32(sm + kSmQ), sOnes = tc::smem_u32(sm + kSmOnes);
    constexpr uint32_t idD = tc::idesc_f16_f32(128, 32);
    constexpr uint32_t idD2 = tc::idesc_f16_f32(128, 16);
    const int bar_id = 1 + g, bar_n = kGroupWarps * 32;

    // outputs of candidates that need no MMA (padding / out of range / no tokens)
    if (lane == 0) {
        for (int ci = stream; ci < kTcCandPerCta && cbase + ci < n; ci += kStreams) {
            const int64_t slot = (int64_t)b * n + cbase + ci;
            const int32_t pid = pids[slot];
            if (pid < 0 || pid >= D.N) out[slot] = -INFINITY;
            else if (D.doc_lens[pid] <= 0) out[slot] = -3.2e10f;    // 32 rows x the -1e9 running-max start
        }
    }
    // ---- cursors over this warp's candidates (cbase + stream + k * kStreams), 32 tokens a step
    auto advance = [&](Cursor& c) {
        c.pos += 32;
        if (c.slot >= 0 && c.pos < c.L) return;
        for (;;) {
            c.ci = (c.slot < 0 && c.ci < 0) ? stream : c.ci + kStreams;
            c.pos = 0;
            if (c.ci >= kTcCandPerCta || cbase + c.ci >= n) {
                c.ci = kTcCandPerCta;
                c.slot = -2;                          // exhausted
                c.L = 0;
                return;
            }
            c.slot = (int64_t)b * n + cbase + c.ci;
            const int32_t pid = pids[c.slot];
            if (pid < 0 || pid >= D.N) continue;
            const int L = D.doc_lens[pid];
            if (L <= 0) continue;
            c.L = L;
            c.tstart = D.doc_offsets[pid];
            return;
        }
    };
    auto tok_valid = [&](const Cursor& c) { return c.slot >= 0 && c.pos + lane < c.L; };

    Cursor cc{-1, -32, 0, -1, 0};
    advance(cc);                 // chunk computed in this iteration
    Cursor fc = cc;              // chunk whose centroid rows / residuals are in flight
    Cursor kc = cc;              // chunk whose code is in flight
    advance(kc);

    uint4 cv[16], r0 = make_uint4(0, 0, 0, 0), r1 = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 16; ++j) cv[j] = make_uint4(0, 0, 0, 0);
    auto fetch_rows = [&](const Cursor& c, int code) {
        if (tok_valid(c)) {
            const int64_t tok = c.tstart + c.pos + lane;
            const uint4* cr = reinterpret_cast<const uint4*>(D.centroids + (int64_t)code * kDim);
#pragma unroll
            for (int j = 0; j < 16; ++j) cv[j] = __ldg(cr + j);
            r0 = *reinterpret_cast<const uint4*>(D.residuals + tok * 32);
            r1 = *reinterpret_cast<const uint4*>(D.residuals + tok * 32 + 16);
        }
    };
    {
        const int code_f = tok_valid(fc) ? D.codes[fc.tstart + fc.pos + lane] : 0;
        fetch_rows(fc, code_f);
    }
    int code_k = tok_valid(kc) ? D.codes[kc.tstart + kc.pos + lane] : 0;

    float run_max = -1e9f;
    uint32_t phase = 0;
    bool failed = false;
    for (;;) {
        const bool have = cc.slot >= 0;
        // ---- decode chunk cc from the registers fetched one iteration ago
        if (have) {
            const bool valid = tok_valid(cc);
            uint32_t a[64];
            if (valid) {
                const uint32_t rw[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
                for (int c = 0; c < 16; ++c) {             // 8 dims = 2 residual bytes per step
                    const uint32_t word = rw[c >> 1];
                    const uint32_t by0 = (word >> ((c & 1) * 16)) & 0xFFu;
                    const uint32_t by1 = (word >> ((c & 1) * 16 + 8)) & 0xFFu;
                    const uint2 w0 = lut[by0 * 32 + lane], w1 = lut[by1 * 32 + lane];
                    a[4 * c + 0] = hadd2_u32(cv[c].x, w0.x);
                    a[4 * c + 1] = hadd2_u32(cv[c].y, w0.y);
                    a[4 * c + 2] = hadd2_u32(cv[c].z, w1.x);
                    a[4 * c + 3] = hadd2_u32(cv[c].w, w1.y);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) a[c] = 0u;
            }
            // ---- issue the next chunk's gathers (their latency overlaps this chunk's MMA/epilogue)
            fc = kc;
            fetch_rows(fc, code_k);
            advance(kc);
            code_k = tok_valid(kc) ? D.codes[kc.tstart + kc.pos + lane] : 0;
            tc::st32x32(tq + kColA, *reinterpret_cast<uint32_t(*)[32]>(&a[0]));
            tc::st32x32(tq + kColA + 32, *reinterpret_cast<uint32_t(*)[32]>(&a[32]));
            uint32_t a2[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) a2[c] = hmul2_u32(a[c]);
            tc::st32x32(tq + kColA2, a2);
#pragma unroll
            for (int c = 0; c < 32; ++c) a2[c] = hmul2_u32(a[32 + c]);
            tc::st32x32(tq + kColA2 + 32, a2);
            tc::wait_st();
        }
        tc::fence_before();
        // ---- group barrier: every quadrant written (or the whole group is done)
        if (!tc::bar_red_or(bar_id, bar_n, have)) break;
        if (quad == 0 && lane == 0) {
            tc::fence_after();
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t koff = (uint32_t)((k >> 2) * (kRows * 128) + (k & 3) * 32);
                tc::mma_ts(tbase + kColD, tbase + kColA + 8 * k, tc::sw128_kmajor_desc(sQ + koff), idD, k > 0);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t koff = (uint32_t)((k >> 2) * (16 * 128) + (k & 3) * 32);
                tc::mma_ts(tbase + kColD2, tbase + kColA2 + 8 * k, tc::sw128_kmajor_desc(sOnes + koff), idD2, k > 0);
            }
            tc::mma_commit(mbar + g);
        }
        const bool ok = tc::mbar_wait_or_abort(mbar + g, phase, abort, kWaitLimit);
        if (!tc::bar_red_and(bar_id, bar_n, ok)) { failed = true; break; }
        phase ^= 1u;
        tc::fence_after();
        if (have) {
            // ---- epilogue: this warp's quadrant = its 32 tokens x 32 query rows
            uint32_t acc[32];
            tc::ld32x32(tq + kColD, acc);
            const uint32_t ssb = tc::ld32x1(tq + kColD2);
            tc::wait_ld();
            const bool valid = tok_valid(cc);
            const float inv = rsqrtf(__uint_as_float(ssb) + 1e-12f);
            float mine = -INFINITY;
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                const float v = valid ? __uint_as_float(acc[r]) * inv : -INFINITY;
                const float mx = tc::warp_max_f32(v);
                mine = (lane == r) ? mx : mine;
            }
            run_max = fmaxf(run_max, mine);
            if (cc.pos + 32 >= cc.L) {
                float s = run_max;
#pragma unroll
                for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
                if (lane == 0) out[cc.slot] = s;
                run_max = -1e9f;
            }
            advance(cc);
        }
        tc::fence_before();
    }
    if (failed && quad == 0 && lane == 0) atomicExch(err, 1);   // either group may have failed
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
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s4_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmDynamic));
    dim3 grid((unsigned)ceil_div(n, kTcCandPerCta), (unsigned)B);
    s4_tc<<<grid, kTcThreads, kSmDynamic, stream>>>(Q, pids, n, D, out, d_err);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
