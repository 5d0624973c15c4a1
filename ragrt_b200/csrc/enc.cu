// enc.cu -- Stage 0a, the ColBERT query encoder (BERT-base over [B, 32] query tokens, ColBERT's
// linear 768 -> 128, L2 normalisation), as sm_100a kernels.  Same network and operation order
// as the reference's flat forward (fast_encoder.py:57-77):
//   x = LN(word[ids] + pos[0..L) + type[0])
//   per layer: qkv = x Wqkv^T + b; ctx = softmax(q k^T / sqrt(d) + maskbias) v (per head);
//              x = LN(x + ctx Wo^T + bo); x = LN(x + gelu(x Wi^T + bi) Wf^T + bf)
//   out = normalize(fp16(x Wl^T)) per token
//
//   enc_gemm       D[M, N] = A[M, K] . W[N, K]^T on the tensor cores (tcgen05.mma kind::f16,
//                  fp32 accumulators in tensor memory), A and W tiles brought in by TMA
//                  (128-byte swizzle, K-major, each CTA loads its own tiles).  Fused epilogues: + bias,
//                  gelu (erf or tanh form), + residual, or the final fp16 rounding + L2
//                  normalisation of a 128-wide row.  Warp 0 issues the TMA loads, warp 1 the
//                  MMAs, warps 2-9 drain the accumulator (two per 32-row quadrant, each
//                  taking half of the tile's columns).
//   enc_embed_ln   embedding sum + LayerNorm, a warp per token row.
//   enc_layernorm  LayerNorm of a [rows, dim] fp16 matrix, a warp per row (fp32 statistics).
//   enc_attention  two warps per (query, head): 32 tokens x head_dim 64; scores, masked
//                  softmax and the weighted sum in fp32 (the 32 x 32 products are too small
//                  for the tensor cores to pay).
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <utility>

#include "common.cuh"
#include "tc.cuh"

namespace ragrt {

namespace {

constexpr int kEM = 128;                 // rows per tile (MMA M)
constexpr int kEK = 64;                  // K per stage: one 128-byte swizzle atom of fp16
constexpr int kETileA = kEM * kEK * 2;   // 16 KB
constexpr int kEThreads = 320;           // 10 warps: TMA, MMA, 8 epilogue
constexpr uint32_t kEWaitLimit = 1u << 26;
constexpr int kEStageBudget = 192 * 1024;

template <int BN>
struct EncCfg {
    static constexpr int kTileB = BN * kEK * 2;
    static constexpr int kStages = kEStageBudget / (kETileA + kTileB);
    static constexpr int kSmem = 1024 + kStages * (kETileA + kTileB) + 256;
    static constexpr uint32_t kTmemCols = 2 * BN;       // two accumulator buffers
};

// Programmatic dependent launch: every encoder kernel is launched so that it may start while
// its predecessor in the stream drains; it does its own set-up, then waits for the
// predecessor's results (griddepcontrol.wait returns at once for a normal launch) and lets
// its own successor start early.
__device__ __forceinline__ void pdl_wait_then_release() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

enum EncEpilogue : int { kEpiBias = 0, kEpiBiasGelu = 1, kEpiBiasGeluTanh = 2, kEpiBiasResidual = 3, kEpiNorm = 4 };

struct EncGemmParams {
    int M, N, K, epi;
    const __half* bias;       // [N] or null
    const __half* residual;   // [M, N] or null
    __half* out;              // [M, N]
    int* err;
    int ksplit;               // > 1: each unit sums a slice of K into partial[slice][M][N] (fp32)
    float* partial;
};

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float gelu_tanh(float x) {
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(u));
}

// Persistent: CTA c takes tiles c, c + grid, ... (N-tile index fastest, so neighbouring CTAs
// share the A row block).  The TMA ring runs across tile boundaries; the MMA warp alternates
// between two accumulator buffers in tensor memory so that the epilogue of one tile overlaps
// the main loop of the next.
template <int BN>
__global__ void __launch_bounds__(kEThreads, 1)
enc_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, EncGemmParams p) {
    using Cfg = EncCfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t enc_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)enc_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = sm;
    uint8_t* sB = sm + S * kETileA;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kTileB);
    uint64_t* empty = full + S;
    uint64_t* accf = empty + S;          // [2] accumulator ready (MMA -> epilogue)
    uint64_t* acce = accf + 2;           // [2] accumulator drained (epilogue -> MMA)
    uint32_t* tslot = reinterpret_cast<uint32_t*>(acce + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = p.K / kEK;
    const int tiles_n = p.N / BN;
    const int tiles = tiles_n * (int)((p.M + kEM - 1) / kEM);
    const int units = tiles * p.ksplit;             // unit u: tile u / ksplit, K slice u % ksplit

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(full + s, 1);
            tc::mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(accf + b, 1);
            tc::mbar_init(acce + b, 8);
        }
        *abort = 0;
        tc::mbar_fence_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tslot, Cfg::kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tslot;
    bool failed = false;
    pdl_wait_then_release();

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int g = 0;                                   // k-chunk counter over all of this CTA's tiles
            for (int u = blockIdx.x; u < units && !failed; u += gridDim.x) {
                const int t = u / p.ksplit, ks = u % p.ksplit;
                const int m0 = (t / tiles_n) * kEM, n0 = (t % tiles_n) * BN;
                const int k0 = nk * ks / p.ksplit, k1 = nk * (ks + 1) / p.ksplit;
                for (int i = k0; i < k1; ++i, ++g) {
                    const int s = g % S;
                    if (g >= S && !tc::mbar_wait_or_abort(empty + s, ((g / S) - 1) & 1, abort, kEWaitLimit)) {
                        failed = true;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(full + s, kETileA + Cfg::kTileB);
                    tc::tma_load_2d(sA + s * kETileA, &tmA, i * kEK, m0, full + s);
                    tc::tma_load_2d(sB + s * Cfg::kTileB, &tmW, i * kEK, n0, full + s);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(kEM, BN);
            int g = 0, j = 0, issued_g = -1;
            for (int u = blockIdx.x; u < units && !failed; u += gridDim.x, ++j) {
                const int ks = u % p.ksplit;
                const int k0 = nk * ks / p.ksplit, k1 = nk * (ks + 1) / p.ksplit;
                const int b = j & 1;
                if (j >= 2 && !tc::mbar_wait_or_abort(acce + b, ((j >> 1) - 1) & 1, abort, kEWaitLimit)) {
                    failed = true;
                    break;
                }
                tc::fence_after();
                const uint32_t d = tbase + (uint32_t)(b * BN);
                for (int i = k0; i < k1; ++i, ++g) {
                    const int s = g % S;
                    if (!tc::mbar_wait_or_abort(full + s, (g / S) & 1, abort, kEWaitLimit)) {
                        failed = true;
                        break;
                    }
                    tc::fence_after();
                    const uint32_t a = tc::smem_u32(sA + s * kETileA), bb = tc::smem_u32(sB + s * Cfg::kTileB);
#pragma unroll
                    for (int k = 0; k < kEK / 16; ++k)
                        tc::mma_ss(d, tc::sw128_kmajor_desc(a + 32 * k), tc::sw128_kmajor_desc(bb + 32 * k), idesc,
                                   (i != k0 || k != 0) ? 1u : 0u);
                    tc::mma_commit(empty + s);
                    issued_g = g;
                }
                if (!failed) tc::mma_commit(accf + b);
            }
            if (failed && issued_g >= 0)   // the last MMAs read shared memory: let them finish
                (void)tc::mbar_wait_bounded(empty + issued_g % S, (issued_g / S) & 1, kEWaitLimit);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3;                  // tensor-memory lane quadrant of this warp
        const int half = (warp - 2) >> 2;          // which half of the tile's columns
        const int c0 = half * (BN / 64), c1 = c0 + BN / 64;
        int j = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
            const int t = u / p.ksplit, ks = u % p.ksplit;
            const int b = j & 1;
            const int m0 = (t / tiles_n) * kEM, n0 = (t % tiles_n) * BN;
            const int row = m0 + quad * 32 + lane;
            const bool ok = tc::mbar_wait_or_abort(accf + b, (j >> 1) & 1, abort, kEWaitLimit);
            if (!__all_sync(0xFFFFFFFFu, ok)) {
                failed = true;
                break;
            }
            tc::fence_after();
            const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * BN);
            if (p.ksplit > 1) {
                // this K slice's fp32 partial sums; enc_splitk_reduce applies the epilogue
#pragma unroll 1
                for (int c = c0; c < c1; ++c) {
                    uint32_t r[32];
                    tc::ld32x32(taddr + 32 * c, r);
                    tc::wait_ld();
                    if (row < p.M) {
                        float* o = p.partial + ((int64_t)ks * p.M + row) * p.N + n0 + 32 * c;
#pragma unroll
                        for (int q = 0; q < 32; q += 4)
                            *reinterpret_cast<uint4*>(o + q) = make_uint4(r[q], r[q + 1], r[q + 2], r[q + 3]);
                    }
                }
            } else if (p.epi == kEpiNorm) {
                // the whole 128-wide row is in one thread (of the first half's warps): fp16
                // rounding, then L2 norm in fp32
                if (half == 0) {
                float v[128];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t r[32];
                    tc::ld32x32(taddr + 32 * c, r);
                    tc::wait_ld();
#pragma unroll
                    for (int q = 0; q < 32; ++q) v[32 * c + q] = __half2float(__float2half_rn(__uint_as_float(r[q])));
                }
                float ss = 0.f;
#pragma unroll
                for (int q = 0; q < 128; ++q) ss = fmaf(v[q], v[q], ss);
                const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
                if (row < p.M) {
                    __half* o = p.out + (int64_t)row * p.N + n0;
#pragma unroll
                    for (int q = 0; q < 128; q += 8) {
                        uint4 u;
                        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
                        for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[q + 2 * e] * inv, v[q + 2 * e + 1] * inv);
                        *reinterpret_cast<uint4*>(o + q) = u;
                    }
                }
                }
            } else {
#pragma unroll 1
                for (int c = c0; c < c1; ++c) {
                    uint32_t r[32];
                    tc::ld32x32(taddr + 32 * c, r);
                    tc::wait_ld();
                    if (row < p.M) {
                        const int col = n0 + 32 * c;
                        const __half* bp = p.bias ? p.bias + col : nullptr;
                        const __half* rp = p.epi == kEpiBiasResidual ? p.residual + (int64_t)row * p.N + col : nullptr;
                        __half* o = p.out + (int64_t)row * p.N + col;
#pragma unroll
                        for (int q = 0; q < 32; q += 8) {
                            float f[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[q + e]);
                            if (bp) {
                                const uint4 bu = __ldg(reinterpret_cast<const uint4*>(bp + q));
                                const __half2* bh = reinterpret_cast<const __half2*>(&bu);
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float2 b2 = __half22float2(bh[e]);
                                    f[2 * e] += b2.x;
                                    f[2 * e + 1] += b2.y;
                                }
                            }
                            if (p.epi == kEpiBiasGelu) {
#pragma unroll
                                for (int e = 0; e < 8; ++e) f[e] = gelu_erf(f[e]);
                            } else if (p.epi == kEpiBiasGeluTanh) {
#pragma unroll
                                for (int e = 0; e < 8; ++e) f[e] = gelu_tanh(f[e]);
                            } else if (rp) {
                                const uint4 ru = *reinterpret_cast<const uint4*>(rp + q);
                                const __half2* rh = reinterpret_cast<const __half2*>(&ru);
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float2 r2 = __half22float2(rh[e]);
                                    f[2 * e] += r2.x;
                                    f[2 * e + 1] += r2.y;
                                }
                            }
                            uint4 u;
                            __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
                            for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
                            *reinterpret_cast<uint4*>(o + q) = u;
                        }
                    }
                }
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(acce + b);
        }
    }
    if (failed && lane == 0) atomicExch(p.err, 1);
    tc::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        tc::tmem_dealloc(tbase, Cfg::kTmemCols);
    }
}

// Sum of the K-slice partials of a split GEMM + the epilogue.  Elementwise epilogues: a thread
// per 8 columns; the normalising one: a warp per 128-wide row.
__global__ void enc_splitk_reduce(const float* __restrict__ partial, int ksplit, int M, int N, int epi,
                                  const __half* __restrict__ bias, const __half* __restrict__ residual,
                                  __half* __restrict__ out) {
    pdl_wait_then_release();
    if (epi == kEpiNorm) {
        const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
        if (row >= M) return;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < ksplit; ++s) {
            const float4 f = *reinterpret_cast<const float4*>(partial + ((int64_t)s * M + row) * N + 4 * lane);
            v[0] += f.x; v[1] += f.y; v[2] += f.z; v[3] += f.w;
        }
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[e] = __half2float(__float2half_rn(v[e]));
            ss = fmaf(v[e], v[e], ss);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
        __half2* o2 = reinterpret_cast<__half2*>(out + (int64_t)row * N + 4 * lane);
        o2[0] = __floats2half2_rn(v[0] * inv, v[1] * inv);
        o2[1] = __floats2half2_rn(v[2] * inv, v[3] * inv);
        return;
    }
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;     // group of 8 columns
    if (g >= (int64_t)M * (N / 8)) return;
    const int row = (int)(g / (N / 8)), col = (int)(g % (N / 8)) * 8;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < ksplit; ++s) {
        const float* src = partial + ((int64_t)s * M + row) * N + col;
        const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 4);
        f[0] += a.x; f[1] += a.y; f[2] += a.z; f[3] += a.w;
        f[4] += b.x; f[5] += b.y; f[6] += b.z; f[7] += b.w;
    }
    if (bias) {
        const uint4 bu = __ldg(reinterpret_cast<const uint4*>(bias + col));
        const __half2* bh = reinterpret_cast<const __half2*>(&bu);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 b2 = __half22float2(bh[e]);
            f[2 * e] += b2.x;
            f[2 * e + 1] += b2.y;
        }
    }
    if (epi == kEpiBiasGelu) {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = gelu_erf(f[e]);
    } else if (epi == kEpiBiasGeluTanh) {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = gelu_tanh(f[e]);
    } else if (epi == kEpiBiasResidual) {
        const uint4 ru = *reinterpret_cast<const uint4*>(residual + (int64_t)row * N + col);
        const __half2* rh = reinterpret_cast<const __half2*>(&ru);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 r2 = __half22float2(rh[e]);
            f[2 * e] += r2.x;
            f[2 * e + 1] += r2.y;
        }
    }
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
    *reinterpret_cast<uint4*>(out + (int64_t)row * N + col) = u;
}

// LayerNorm of one row held by a warp: 8 fp16 per lane per 256 columns.
template <int kDimT>
__device__ __forceinline__ void warp_layernorm_store(float (&v)[kDimT / 32], const __half* gamma, const __half* beta,
                                                     float eps, __half* out, int lane) {
    constexpr int kPer = kDimT / 32;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) s += v[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    const float mean = s * (1.0f / kDimT);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const float d = v[i] - mean;
        q = fmaf(d, d, q);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
    const float rstd = rsqrtf(q * (1.0f / kDimT) + eps);
#pragma unroll
    for (int g = 0; g < kPer / 8; ++g) {
        const int col = (g * 32 + lane) * 8;
        const uint4 gu = __ldg(reinterpret_cast<const uint4*>(gamma + col));
        const uint4 bu = __ldg(reinterpret_cast<const uint4*>(beta + col));
        const __half2* gh = reinterpret_cast<const __half2*>(&gu);
        const __half2* bh = reinterpret_cast<const __half2*>(&bu);
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 g2 = __half22float2(gh[t]), b2 = __half22float2(bh[t]);
            h[t] = __floats2half2_rn((v[g * 8 + 2 * t] - mean) * rstd * g2.x + b2.x,
                                     (v[g * 8 + 2 * t + 1] - mean) * rstd * g2.y + b2.y);
        }
        *reinterpret_cast<uint4*>(out + col) = u;
    }
}

template <int kDimT>
__device__ __forceinline__ void load_row(const __half* src, float (&v)[kDimT / 32], int lane) {
#pragma unroll
    for (int g = 0; g < kDimT / 256; ++g) {
        const uint4 u = *reinterpret_cast<const uint4*>(src + (g * 32 + lane) * 8);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 f = __half22float2(h[t]);
            v[g * 8 + 2 * t] = f.x;
            v[g * 8 + 2 * t + 1] = f.y;
        }
    }
}

template <int kDimT>
__global__ void enc_layernorm(const __half* __restrict__ x, const __half* __restrict__ gamma,
                              const __half* __restrict__ beta, float eps, __half* __restrict__ out, int rows) {
    pdl_wait_then_release();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    float v[kDimT / 32];
    load_row<kDimT>(x + (int64_t)warp * kDimT, v, lane);
    warp_layernorm_store<kDimT>(v, gamma, beta, eps, out + (int64_t)warp * kDimT, lane);
}

// out = LN(sum of the K-slice partials + bias + residual), a CTA of kDimT / 3 threads per row
// (3 columns per thread, coalesced partial reads; mean and variance by block reduction).  A
// CTA reads its residual row before writing its output row, so out may be the residual.
template <int kDimT>
__global__ void __launch_bounds__(kDimT / 3)
enc_splitk_reduce_ln(const float* __restrict__ partial, int ksplit, int M, const __half* __restrict__ bias,
                     const __half* residual, const __half* __restrict__ gamma, const __half* __restrict__ beta,
                     float eps, __half* out) {
    constexpr int kT = kDimT / 3, kW = kT / 32;
    __shared__ float red[2][kW];
    pdl_wait_then_release();
    const int row = blockIdx.x, t = threadIdx.x, lane = t & 31, w = t >> 5;
    float v[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int col = t + c * kT;
        v[c] = __half2float(bias[col]) + __half2float(residual[(int64_t)row * kDimT + col]);
    }
    for (int s_ = 0; s_ < ksplit; ++s_) {
        const float* src = partial + ((int64_t)s_ * M + row) * kDimT;
#pragma unroll
        for (int c = 0; c < 3; ++c) v[c] += src[t + c * kT];
    }
    // the unfused path rounds the residual sum to fp16 before its LayerNorm: so does this one
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        v[c] = __half2float(__float2half_rn(v[c]));
        sum += v[c];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) red[0][w] = sum;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kW; ++i) tot += red[0][i];
    const float mean = tot * (1.0f / kDimT);
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float d = v[c] - mean;
        q = fmaf(d, d, q);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
    if (lane == 0) red[1][w] = q;
    __syncthreads();
    float qt = 0.f;
#pragma unroll
    for (int i = 0; i < kW; ++i) qt += red[1][i];
    const float rstd = rsqrtf(qt * (1.0f / kDimT) + eps);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int col = t + c * kT;
        out[(int64_t)row * kDimT + col] =
            __float2half_rn((v[c] - mean) * rstd * __half2float(gamma[col]) + __half2float(beta[col]));
    }
}

// x[row] = LN(word[ids[row]] + pos[row % L] + type), summed in fp32 (token ids outside the
// vocabulary are clamped to 0 and raise the error word)
template <int kDimT>
__global__ void enc_embed_ln(const int64_t* __restrict__ ids, const __half* __restrict__ word,
                             const __half* __restrict__ pos, const __half* __restrict__ type,
                             const __half* __restrict__ gamma, const __half* __restrict__ beta, float eps, int vocab,
                             int L, int rows, __half* __restrict__ out, int* err) {
    pdl_wait_then_release();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    int64_t id = ids[warp];
    if (id < 0 || id >= vocab) {
        if (lane == 0) atomicExch(err, 4);
        id = 0;
    }
    float v[kDimT / 32], a[kDimT / 32], b[kDimT / 32];
    load_row<kDimT>(word + id * kDimT, v, lane);
    load_row<kDimT>(pos + (int64_t)(warp % L) * kDimT, a, lane);
    load_row<kDimT>(type, b, lane);
#pragma unroll
    for (int i = 0; i < kDimT / 32; ++i) v[i] += a[i] + b[i];
    warp_layernorm_store<kDimT>(v, gamma, beta, eps, out + (int64_t)warp * kDimT, lane);
}

// Attention of one (query, head): L = 32 tokens, head_dim 64, two warps.  Lanes 2i and 2i+1
// own query token i (of the CTA's 16 in warp w: i = 16 w + lane / 2) and half of the head's
// dimensions each: partial q.k dots are combined with one shuffle, the softmax runs in fp32 on
// both lanes, and each lane accumulates its half of p.V.  K and V are staged in shared memory
// as fp32 rows of 68 floats, the second half of a row 4 floats further on (so that the two
// halves read in one instruction fall in different banks), read as broadcast float4.  qkv [B*L, 3*D] with Q, K, V in column blocks of D; mask [B, L] (1 = attended key);
// ctx [B*L, D].
constexpr int kHd = 64;
constexpr int kKvStride = 68;
__global__ void __launch_bounds__(64)
enc_attention(const __half* __restrict__ qkv, const int64_t* __restrict__ mask, __half* __restrict__ ctx, int B,
              int H, int D, float scale) {
    __shared__ __align__(16) float sK[32][kKvStride];
    __shared__ __align__(16) float sV[32][kKvStride];
    pdl_wait_then_release();
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int b = blockIdx.x / H, h = blockIdx.x % H;
    // stage K and V: thread t loads token t / 2, half t % 2 (32 dims = 4 x 16 B) of each
    {
        const int tok = tid >> 1, half = tid & 1;
        const __half* src = qkv + ((int64_t)b * 32 + tok) * (3 * D) + h * kHd + half * 32;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint4 uk = *reinterpret_cast<const uint4*>(src + D + g * 8);
            const uint4 uv = *reinterpret_cast<const uint4*>(src + 2 * D + g * 8);
            const __half2* hk = reinterpret_cast<const __half2*>(&uk);
            const __half2* hv = reinterpret_cast<const __half2*>(&uv);
            float4 k0, k1, v0, v1;
            float2 t;
            t = __half22float2(hk[0]); k0.x = t.x; k0.y = t.y;
            t = __half22float2(hk[1]); k0.z = t.x; k0.w = t.y;
            t = __half22float2(hk[2]); k1.x = t.x; k1.y = t.y;
            t = __half22float2(hk[3]); k1.z = t.x; k1.w = t.y;
            t = __half22float2(hv[0]); v0.x = t.x; v0.y = t.y;
            t = __half22float2(hv[1]); v0.z = t.x; v0.w = t.y;
            t = __half22float2(hv[2]); v1.x = t.x; v1.y = t.y;
            t = __half22float2(hv[3]); v1.z = t.x; v1.w = t.y;
            float* kd = &sK[tok][half * 36 + g * 8];
            float* vd = &sV[tok][half * 36 + g * 8];
            *reinterpret_cast<float4*>(kd) = k0;
            *reinterpret_cast<float4*>(kd + 4) = k1;
            *reinterpret_cast<float4*>(vd) = v0;
            *reinterpret_cast<float4*>(vd + 4) = v1;
        }
    }
    const int i = w * 16 + (lane >> 1), half = lane & 1;
    const int64_t row = (int64_t)b * 32 + i;
    float q[32];
    {
        const __half* qs = qkv + row * (3 * D) + h * kHd + half * 32;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint4 u = *reinterpret_cast<const uint4*>(qs + g * 8);
            const __half2* hq = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 f = __half22float2(hq[t]);
                q[g * 8 + 2 * t] = f.x * scale;
                q[g * 8 + 2 * t + 1] = f.y * scale;
            }
        }
    }
    const unsigned kept = __ballot_sync(0xFFFFFFFFu, mask[(int64_t)b * 32 + lane] != 0);
    __syncthreads();
    float s[32];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float4* kr = reinterpret_cast<const float4*>(&sK[j][half * 36]);
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float4 k4 = kr[c];
            d = fmaf(q[4 * c], k4.x, d);
            d = fmaf(q[4 * c + 1], k4.y, d);
            d = fmaf(q[4 * c + 2], k4.z, d);
            d = fmaf(q[4 * c + 3], k4.w, d);
        }
        d += __shfl_xor_sync(0xFFFFFFFFu, d, 1);
        s[j] = ((kept >> j) & 1u) ? d : -INFINITY;
        mx = fmaxf(mx, s[j]);
    }
    float o[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) o[k] = 0.f;
    float den = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float e = __expf(s[j] - mx);
            den += e;
            const float4* vr = reinterpret_cast<const float4*>(&sV[j][half * 36]);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 v4 = vr[c];
                o[4 * c] = fmaf(e, v4.x, o[4 * c]);
                o[4 * c + 1] = fmaf(e, v4.y, o[4 * c + 1]);
                o[4 * c + 2] = fmaf(e, v4.z, o[4 * c + 2]);
                o[4 * c + 3] = fmaf(e, v4.w, o[4 * c + 3]);
            }
        }
    }
    const float inv = den > 0.f ? 1.0f / den : 0.f;
    __half* out = ctx + row * D + h * kHd + half * 32;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        uint4 u;
        __half2* hh = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int t = 0; t < 4; ++t) hh[t] = __floats2half2_rn(o[g * 8 + 2 * t] * inv, o[g * 8 + 2 * t + 1] * inv);
        *reinterpret_cast<uint4*>(out + g * 8) = u;
    }
}

// Launch with programmatic stream serialisation (see pdl_wait_then_release).
template <typename... KArgs, typename... Args>
int enc_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(RAGRT_ERR_CUDA, "encoder kernel launch: %s", cudaGetErrorString(e));
    }
    count_launch();
    return RAGRT_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn enc_encode_fn() {
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

// fp16 [rows, cols] row-major, box [box_rows x 64 cols], 128-byte swizzle (out-of-range rows read 0)
int enc_make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
    EncodeTiledFn fn = enc_encode_fn();
    if (!fn) return fail(RAGRT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kEK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RAGRT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return RAGRT_OK;
}

}  // namespace
}  // namespace ragrt

using namespace ragrt;

template <int BN>
static int enc_gemm_launch(const void* d_A, const void* d_W, int32_t M, int32_t N, int32_t K, const EncGemmParams& p,
                           cudaStream_t stream) {
    CUtensorMap tA, tW;
    int rc = enc_make_map(&tA, d_A, M, K, kEM);
    if (rc || (rc = enc_make_map(&tW, d_W, N, K, BN))) return rc;
    // the shared-memory attribute is per device: set it once for each device used
    static std::atomic<uint64_t> attr_set{0};
    int dev = 0;
    RAGRT_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        RAGRT_CUDA_TRY(cudaFuncSetAttribute(enc_gemm<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            EncCfg<BN>::kSmem));
        attr_set.fetch_or(bit);
    }
    const int units = (N / BN) * (int)ceil_div(M, kEM) * p.ksplit;
    return enc_launch(enc_gemm<BN>, dim3((unsigned)std::min(units, num_sms())), dim3(kEThreads), EncCfg<BN>::kSmem,
                      stream, tA, tW, p);
}

extern "C" int ragrt_enc_gemm(const void* d_A, const void* d_W, const void* d_bias, const void* d_residual, void* d_out,
                              int32_t M, int32_t N, int32_t K, int32_t epilogue, void* d_ws, int64_t ws_bytes,
                              void* stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    RAGRT_REQUIRE(d_A && d_W && d_out, "null argument");
    RAGRT_REQUIRE(M >= 1 && N >= 128 && N % 128 == 0 && K >= kEK && K % kEK == 0,
                  "enc_gemm needs M >= 1, N a multiple of 128 and K a multiple of %d (M=%d N=%d K=%d)", kEK,
                  (int)M, (int)N, (int)K);
    RAGRT_REQUIRE(epilogue >= kEpiBias && epilogue <= kEpiNorm, "unknown epilogue %d", (int)epilogue);
    RAGRT_REQUIRE(epilogue != kEpiNorm || N == 128, "the normalising epilogue needs N == 128");
    RAGRT_REQUIRE(epilogue != kEpiBiasResidual || d_residual, "the residual epilogue needs a residual");
    RAGRT_REQUIRE(((uintptr_t)d_A & 15) == 0 && ((uintptr_t)d_W & 15) == 0 && ((uintptr_t)d_out & 15) == 0 &&
                      ((uintptr_t)d_bias & 15) == 0 && ((uintptr_t)d_residual & 15) == 0 &&
                      ((uintptr_t)d_ws & 15) == 0,
                  "enc_gemm operands must be 16-byte aligned");
    int* err = device_error_flag();
    if (!err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
    EncGemmParams p{M, N, K, epilogue, (const __half*)d_bias, (const __half*)d_residual, (__half*)d_out, err, 1,
                    nullptr};
    const int sms = num_sms();
    const int64_t mt = ceil_div(M, kEM);
    // tiles of 128 x 256 (half the W re-reads per flop) when they fill the GPU and their last
    // round of persistent CTAs is about as full as with 128 x 128 tiles; else 128 x 128
    auto fill = [&](int bn) {
        const int64_t t = (int64_t)(N / bn) * mt;
        return (double)t / (double)(ceil_div(t, (int64_t)sms) * sms);
    };
    const bool wide = epilogue != kEpiNorm && N % 256 == 0 && (N / 256) * mt >= sms && fill(256) >= fill(128) - 0.05;
    const int bn = wide ? 256 : 128;
    const int64_t tiles = (N / bn) * mt;
    // too few tiles to occupy the SMs (small batches): split K across CTAs, fp32 partials in
    // the caller's workspace, then one reduction that applies the epilogue
    if (tiles * 2 <= sms) {
        int64_t ks = std::min<int64_t>(K / kEK, sms / tiles);
        const int64_t per = (int64_t)M * N * 4;
        ks = std::min<int64_t>(ks, d_ws ? ws_bytes / per : 0);
        if (ks > 1) {
            p.ksplit = (int)ks;
            p.partial = (float*)d_ws;
        }
    }
    int rc = wide ? enc_gemm_launch<256>(d_A, d_W, M, N, K, p, stream) : enc_gemm_launch<128>(d_A, d_W, M, N, K, p, stream);
    if (rc || p.ksplit == 1) return rc;
    const int threads = 256;
    const int64_t work = epilogue == kEpiNorm ? (int64_t)M * 32 : (int64_t)M * (N / 8);
    return enc_launch(enc_splitk_reduce, dim3((unsigned)ceil_div(work, (int64_t)threads)), dim3(threads), 0, stream,
                      (const float*)p.partial, p.ksplit, (int)M, (int)N, (int)epilogue, (const __half*)d_bias,
                      (const __half*)d_residual, (__half*)d_out);
}

extern "C" int ragrt_enc_layernorm(const void* d_x, const void* d_gamma, const void* d_beta, float eps, void* d_out,
                                   int32_t rows, int32_t dim, void* stream_);

extern "C" int ragrt_enc_gemm_residual_ln(const void* d_A, const void* d_W, const void* d_bias, const void* d_residual,
                                          const void* d_gamma, const void* d_beta, float eps, void* d_tmp,
                                          void* d_out, int32_t M, int32_t N, int32_t K, void* d_ws,
                                          int64_t ws_bytes, void* stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    RAGRT_REQUIRE(d_bias && d_residual && d_gamma && d_beta && d_tmp && d_out, "null argument");
    RAGRT_REQUIRE(N == 768, "enc_gemm_residual_ln is built for N = 768 (BERT-base); got %d", (int)N);
    // the split decision of ragrt_enc_gemm, with its partials reduced straight into the LayerNorm
    const int sms = num_sms();
    const int64_t tiles = (int64_t)(N / 128) * ceil_div(M, kEM);
    int64_t ks = 1;
    if (tiles * 2 <= sms && K % kEK == 0) {
        ks = std::min<int64_t>(K / kEK, sms / tiles);
        ks = std::min<int64_t>(ks, d_ws ? ws_bytes / ((int64_t)M * N * 4) : 0);
    }
    if (ks <= 1) {
        int rc = ragrt_enc_gemm(d_A, d_W, d_bias, d_residual, d_tmp, M, N, K, kEpiBiasResidual, nullptr, 0, stream_);
        if (rc) return rc;
        return ragrt_enc_layernorm(d_tmp, d_gamma, d_beta, eps, d_out, M, N, stream_);
    }
    RAGRT_REQUIRE(M >= 1 && K >= kEK && K % kEK == 0, "enc_gemm needs K a multiple of %d", kEK);
    RAGRT_REQUIRE(((uintptr_t)d_A & 15) == 0 && ((uintptr_t)d_W & 15) == 0 && ((uintptr_t)d_ws & 15) == 0 &&
                      ((uintptr_t)d_residual & 15) == 0 && ((uintptr_t)d_out & 15) == 0,
                  "enc_gemm operands must be 16-byte aligned");
    int* err = device_error_flag();
    if (!err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
    EncGemmParams p{M, N, K, kEpiBiasResidual, (const __half*)d_bias, (const __half*)d_residual, (__half*)d_tmp, err,
                    (int)ks, (float*)d_ws};
    int rc = enc_gemm_launch<128>(d_A, d_W, M, N, K, p, stream);
    if (rc) return rc;
    return enc_launch(enc_splitk_reduce_ln<768>, dim3((unsigned)M), dim3(768 / 3), 0, stream, (const float*)d_ws,
                      (int)ks, (int)M, (const __half*)d_bias,
                      (const __half*)d_residual, (const __half*)d_gamma, (const __half*)d_beta, eps, (__half*)d_out);
}

extern "C" int ragrt_enc_layernorm(const void* d_x, const void* d_gamma, const void* d_beta, float eps, void* d_out,
                                   int32_t rows, int32_t dim, void* stream_) {
    RAGRT_REQUIRE(d_x && d_gamma && d_beta && d_out, "null argument");
    RAGRT_REQUIRE(dim == 768, "enc_layernorm is built for dim 768 (BERT-base); got %d", (int)dim);
    RAGRT_REQUIRE(rows >= 0, "rows must be >= 0");
    if (rows == 0) return RAGRT_OK;
    const int threads = 256;
    return enc_launch(enc_layernorm<768>, dim3((unsigned)ceil_div((int64_t)rows * 32, threads)), dim3(threads), 0,
                      (cudaStream_t)stream_, (const __half*)d_x, (const __half*)d_gamma, (const __half*)d_beta, eps,
                      (__half*)d_out, (int)rows);
}

extern "C" int ragrt_enc_embed(const int64_t* d_ids, const void* d_word, const void* d_pos, const void* d_type,
                               const void* d_gamma, const void* d_beta, float eps, int32_t vocab, int32_t B, int32_t L,
                               int32_t dim, void* d_out, void* stream_) {
    RAGRT_REQUIRE(d_ids && d_word && d_pos && d_type && d_gamma && d_beta && d_out, "null argument");
    RAGRT_REQUIRE(dim == 768, "enc_embed is built for dim 768 (BERT-base); got %d", (int)dim);
    RAGRT_REQUIRE(B >= 1 && L >= 1 && vocab >= 1, "B, L and vocab must be >= 1");
    int* err = device_error_flag();
    if (!err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
    const int rows = B * L, threads = 256;
    return enc_launch(enc_embed_ln<768>, dim3((unsigned)ceil_div((int64_t)rows * 32, threads)), dim3(threads), 0,
                      (cudaStream_t)stream_, d_ids, (const __half*)d_word, (const __half*)d_pos, (const __half*)d_type,
                      (const __half*)d_gamma, (const __half*)d_beta, eps, (int)vocab, (int)L, (int)rows,
                      (__half*)d_out, err);
}

extern "C" int ragrt_enc_attention(const void* d_qkv, const int64_t* d_mask, void* d_ctx, int32_t B, int32_t L,
                                   int32_t heads, int32_t dim, void* stream_) {
    RAGRT_REQUIRE(d_qkv && d_mask && d_ctx, "null argument");
    RAGRT_REQUIRE(L == 32, "enc_attention is built for 32 query tokens; got %d", (int)L);
    RAGRT_REQUIRE(heads >= 1 && dim == heads * kHd, "enc_attention needs head_dim %d (dim %d, heads %d)", kHd,
                  (int)dim, (int)heads);
    RAGRT_REQUIRE(B >= 1, "B must be >= 1");
    return enc_launch(enc_attention, dim3((unsigned)(B * heads)), dim3(64), 0, (cudaStream_t)stream_,
                      (const __half*)d_qkv, d_mask, (__half*)d_ctx, (int)B, (int)heads, (int)dim,
                      1.0f / sqrtf((float)kHd));
}
