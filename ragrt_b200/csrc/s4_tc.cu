// s4_tc.cu -- Stage 4 on the 5th-generation tensor cores (tcgen05 + tensor memory): fused
// 2-bit residual decompression + TileMaxSim.  Replaces the reference's wmma kernel
// (tile_maxsim_fused_decomp.cu:125-229), same result definition:
//   score(pid) = sum_r max_t (q_r . d_t) * rsqrt(|d_t|^2 + 1e-12)
//
// Layout of one MMA tile (M = 128 doc tokens, N = 32 query rows, K = 128 dims):
//   * A = decoded doc tokens, K-major, written straight from registers into TENSOR MEMORY
//     (tcgen05.st): the thread that decodes a token owns its TMEM lane, so decoded tokens
//     never touch shared memory.  Lanes 32w..32w+31 (warp w's quadrant) hold 32
//     consecutive tokens of ONE candidate of warp w's candidate stream.
//   * B = the query's 32 x 128 fp16 rows in shared memory (128-byte swizzle, K-major).
//   * D = 128 x 32 fp32 accumulator in tensor memory; warp w reads back its own quadrant.
//   * |d_t|^2 also runs on the tensor core: A2 = d*d (fp16) times a ones matrix (N = 16);
//     column 0 of that accumulator is the squared norm of the lane's token.
// Epilogue per warp: scale the 32 dot products of its lane's token by the inverse norm,
// take the max over the 32 tokens (= lanes) of the chunk with redux.sync.max.f32 for
// each query row, keep a per-candidate running max in the lane of that row, and sum the
// 32 rows when the candidate's last chunk is done.
#include "common.cuh"
#include "s4_common.cuh"
#include "tc.cuh"

namespace ragrt {

constexpr int kTcWarps = 4;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcCandPerCta = 64;
constexpr uint32_t kColA = 0;      // 64 columns: 128 fp16 dims per token lane
constexpr uint32_t kColA2 = 64;    // 64 columns: squared dims
constexpr uint32_t kColD = 128;    // 32 columns: dot products with the 32 query rows
constexpr uint32_t kColD2 = 160;   // 16 columns: squared norm (column 0)
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kWaitLimit = 1u << 22;   // polls before a wait is declared failed

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kSmQ = 0;            // 32 rows x 256 B, SW128 K-major (two 4 KB atoms)
constexpr int kSmOnes = 8192;      // 16 rows x 256 B of fp16 1.0
constexpr int kSmLut = 12288;      // 256 x uint2: byte -> 4 fp16 bucket weights
constexpr int kSmBar = 14336;      // mbarrier
constexpr int kSmTmem = 14344;     // tensor-memory base address
constexpr int kSmBytes = 14352;
constexpr int kSmDynamic = kSmBytes + 1024 + 96 * 1024;   // padding caps residency at 2 CTAs/SM (TMEM)

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hadd2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a) {
    __half2 x = *reinterpret_cast<__half2*>(&a);
    __half2 r = __hmul2(x, x);
    return *reinterpret_cast<uint32_t*>(&r);
}

__global__ void __launch_bounds__(kTcThreads)
s4_tc(const __half* __restrict__ Q, const int32_t* __restrict__ pids, int n, S4Docs D, float* __restrict__ out,
      int* __restrict__ err) {
    extern __shared__ uint8_t s4_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)s4_raw + 1023) & ~(uintptr_t)1023);
    uint2* lut = reinterpret_cast<uint2*>(sm + kSmLut);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kSmBar);
    uint32_t* tbase_s = reinterpret_cast<uint32_t*>(sm + kSmTmem);

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y;
    const int64_t cbase = (int64_t)blockIdx.x * kTcCandPerCta;

    // query rows -> SW128 K-major tile; ones tile; byte LUT
    const __half* Qb = Q + (int64_t)b * kRows * kDim;
    for (int i = tid; i < kRows * 16; i += kTcThreads) {
        const int row = i >> 4, c16 = i & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(Qb + row * kDim + c16 * 8);
        *reinterpret_cast<uint4*>(sm + kSmQ + tc::sw128_offset(row, c16, kRows)) = v;
    }
    for (int i = tid; i < 256; i += kTcThreads)
        reinterpret_cast<uint4*>(sm + kSmOnes)[i] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    for (int i = tid; i < 256; i += kTcThreads) {
        const int rev = D.rbm[i];
        __half wv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) wv[u] = D.bw[D.decomp[rev * 4 + u] & 3];
        lut[i] = *reinterpret_cast<uint2*>(wv);
    }
    if (tid == 0) {
        tc::mbar_init(mbar, 1);
        tc::mbar_fence_init();
    }
    if (w == 0) {
        tc::tmem_alloc(tbase_s, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tbase_s;
    const uint32_t tq = tbase + ((uint32_t)(32 * w) << 16);     // this warp's lane quadrant
    const uint32_t sQ = tc::smem_u32(sm + kSmQ), sOnes = tc::smem_u32(sm + kSmOnes);
    constexpr uint32_t idD = tc::idesc_f16_f32(128, 32);
    constexpr uint32_t idD2 = tc::idesc_f16_f32(128, 16);

    // this warp's candidate stream: cbase + w, + kTcWarps, ...
    int ci = w - kTcWarps;
    int64_t slot = -1;
    int64_t tstart = 0;
    int L = 0, pos = 0;
    float run_max = -1e9f;
    auto next_candidate = [&]() {
        for (;;) {
            ci += kTcWarps;
            if (ci >= kTcCandPerCta || cbase + ci >= n) { slot = -1; return; }
            slot = (int64_t)b * n + cbase + ci;
            const int32_t pid = pids[slot];
            if (pid < 0 || pid >= D.N) {
                if (lane == 0) out[slot] = -INFINITY;
                continue;
            }
            L = D.doc_lens[pid];
            if (L <= 0) {
                if (lane == 0) out[slot] = -3.2e10f;     // 32 rows x the -1e9 running-max start
                continue;
            }
            tstart = D.doc_offsets[pid];
            pos = 0;
            run_max = -1e9f;
            return;
        }
    };
    next_candidate();

    uint32_t phase = 0;
    bool timed_out = false;
    for (;;) {
        const bool have = slot >= 0;
        if (!__syncthreads_or(have)) break;
        if (have) {
            // ---- decode 32 tokens of the current candidate, one per lane
            const bool valid = pos + lane < L;
            uint32_t a[64], a2[64];
            if (valid) {
                const int64_t tok = tstart + pos + lane;
                const int code = D.codes[tok];
                const uint4* cr = reinterpret_cast<const uint4*>(D.centroids + (int64_t)code * kDim);
                const uint4 r0 = *reinterpret_cast<const uint4*>(D.residuals + tok * 32);
                const uint4 r1 = *reinterpret_cast<const uint4*>(D.residuals + tok * 32 + 16);
                const uint8_t* rb0 = reinterpret_cast<const uint8_t*>(&r0);
                const uint8_t* rb1 = reinterpret_cast<const uint8_t*>(&r1);
#pragma unroll
                for (int c = 0; c < 16; ++c) {             // 8 dims = 2 residual bytes per step
                    const uint4 cv = __ldg(cr + c);
                    const uint8_t by0 = c < 8 ? rb0[2 * c] : rb1[2 * c - 16];
                    const uint8_t by1 = c < 8 ? rb0[2 * c + 1] : rb1[2 * c - 15];
                    const uint2 w0 = lut[by0], w1 = lut[by1];
                    a[4 * c + 0] = hadd2_u32(cv.x, w0.x);
                    a[4 * c + 1] = hadd2_u32(cv.y, w0.y);
                    a[4 * c + 2] = hadd2_u32(cv.z, w1.x);
                    a[4 * c + 3] = hadd2_u32(cv.w, w1.y);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) a[c] = 0u;
            }
#pragma unroll
            for (int c = 0; c < 64; ++c) a2[c] = hmul2_u32(a[c]);
            tc::st32x32(tq + kColA, *reinterpret_cast<uint32_t(*)[32]>(&a[0]));
            tc::st32x32(tq + kColA + 32, *reinterpret_cast<uint32_t(*)[32]>(&a[32]));
            tc::st32x32(tq + kColA2, *reinterpret_cast<uint32_t(*)[32]>(&a2[0]));
            tc::st32x32(tq + kColA2 + 32, *reinterpret_cast<uint32_t(*)[32]>(&a2[32]));
            tc::wait_st();
        }
        tc::fence_before();
        __syncthreads();
        // ---- one thread issues the MMAs of the tile
        if (tid == 0) {
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
            tc::mma_commit(mbar);
        }
        const bool ok = tc::mbar_wait_bounded(mbar, phase, kWaitLimit);
        if (__syncthreads_or(!ok)) {            // uniform decision: every thread leaves together
            timed_out = true;
            if (tid == 0) atomicExch(err, 1);
            break;
        }
        phase ^= 1u;
        tc::fence_after();
        if (have) {
            // ---- epilogue: this warp's quadrant = its 32 tokens x 32 query rows
            uint32_t acc[32];
            tc::ld32x32(tq + kColD, acc);
            const uint32_t ssb = tc::ld32x1(tq + kColD2);
            tc::wait_ld();
            const bool valid = pos + lane < L;
            const float inv = rsqrtf(__uint_as_float(ssb) + 1e-12f);
            float mine = -INFINITY;
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                const float v = valid ? __uint_as_float(acc[r]) * inv : -INFINITY;
                const float m = tc::warp_max_f32(v);
                mine = (lane == r) ? m : mine;
            }
            run_max = fmaxf(run_max, mine);
            pos += 32;
            if (pos >= L) {
                float s = run_max;
#pragma unroll
                for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
                if (lane == 0) out[slot] = s;
                next_candidate();
            }
        }
        tc::fence_before();
    }
    __syncthreads();
    if (timed_out && tid == 0) tc::mbar_wait_bounded(mbar, phase, kWaitLimit);   // give in-flight MMAs a last chance
    __syncthreads();
    if (w == 0) {
        tc::fence_after();
        tc::tmem_dealloc(tbase, kTmemCols);
    }
}

int s4_tc_launch(const __half* Q, const int32_t* pids, int B, int n, const S4Docs& D, float* out,
                 cudaStream_t stream) {
    if (B <= 0 || n <= 0) return RAGRT_OK;
    static int* d_err = nullptr;
    if (!d_err) {
        RAGRT_CUDA_TRY(cudaMalloc(&d_err, sizeof(int)));
        RAGRT_CUDA_TRY(cudaMemset(d_err, 0, sizeof(int)));
    }
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s4_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmDynamic));
    dim3 grid((unsigned)ceil_div(n, kTcCandPerCta), (unsigned)B);
    s4_tc<<<grid, kTcThreads, kSmDynamic, stream>>>(Q, pids, n, D, out, d_err);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
