// s4_maxsim.cu -- Stage 4 CUDA-core kernel (the reference's "simt" rerank mode,
// tile_maxsim_fused_decomp.cu:24-116) and the final filter + top-k
// (ragrt_fused_kernel.cu:621-640, optix_corr_torch_3d.cpp:603-606).
//
// score(pid) = sum over the 32 query rows r of max over the passage's tokens t of
//              (q_r . d_t) * rsqrt(|d_t|^2 + 1e-12),
// d_t[k] = fp16 add of centroid[code_t][k] and bucket_weights[decomp[rbm[byte]][k % 4]]
// (byte = residual byte k / 4 of token t), exactly the reference's decode
// (tile_maxsim_fused_decomp.cu:168-201).  A passage with no tokens scores 32 * -1e9 (the
// reference's running-max start); pid < 0 scores -inf; pid >= N (out of range) -inf.
#include "common.cuh"
#include "s3_common.cuh"
#include "s4_common.cuh"

namespace ragrt {

constexpr int kS4Warps = 8;

// byte -> the 4 fp16 bucket weights of its dims, built once per CTA
__device__ __forceinline__ void build_byte_lut(uint2* lut, const __half* bw, const uint8_t* rbm, const uint8_t* dt) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        const int rev = rbm[i];
        __half w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) w[u] = bw[dt[rev * 4 + u] & 3];
        lut[i] = *reinterpret_cast<uint2*>(w);
    }
}

__global__ void __launch_bounds__(kS4Warps * 32)
s4_simt(const __half* __restrict__ Q, const int32_t* __restrict__ pids, int n, int64_t total,
        S4Docs D, float* __restrict__ out) {
    __shared__ uint2 lut[256];
    __shared__ __align__(16) __half s_d[kS4Warps][kDim];
    build_byte_lut(lut, D.bw, D.rbm, D.decomp);
    __syncthreads();
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t i = (int64_t)blockIdx.x * kS4Warps + w; i < total; i += (int64_t)gridDim.x * kS4Warps) {
        const int64_t b = i / n;
        const int32_t pid = pids[i];
        if (pid < 0 || pid >= D.N) {
            if (lane == 0) out[i] = -INFINITY;
            continue;
        }
        float q[kDim];
        const __half* qr = Q + (b * kRows + lane) * kDim;
#pragma unroll
        for (int k = 0; k < kDim; k += 8) {
            uint4 u = *reinterpret_cast<const uint4*>(qr + k);
            const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f = __half22float2(h[j]);
                q[k + 2 * j] = f.x;
                q[k + 2 * j + 1] = f.y;
            }
        }
        const int64_t start = D.doc_offsets[pid];
        const int L = D.doc_lens[pid];
        float run_max = -1e9f;
        for (int t = 0; t < L; ++t) {
            const int64_t tok = start + t;
            const int code = D.codes[tok];
            const uint2 c4 = *reinterpret_cast<const uint2*>(D.centroids + (int64_t)code * kDim + 4 * lane);
            const uint2 w4 = lut[D.residuals[tok * 32 + lane]];
            __half2 d01 = __hadd2(*reinterpret_cast<const __half2*>(&c4.x), *reinterpret_cast<const __half2*>(&w4.x));
            __half2 d23 = __hadd2(*reinterpret_cast<const __half2*>(&c4.y), *reinterpret_cast<const __half2*>(&w4.y));
            float2 f01 = __half22float2(d01), f23 = __half22float2(d23);
            float ss = f01.x * f01.x + f01.y * f01.y + f23.x * f23.x + f23.y * f23.y;
#pragma unroll
            for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
            const float inv = rsqrtf(ss + 1e-12f);
            uint2 st;
            st.x = *reinterpret_cast<uint32_t*>(&d01);
            st.y = *reinterpret_cast<uint32_t*>(&d23);
            *reinterpret_cast<uint2*>(&s_d[w][4 * lane]) = st;
            __syncwarp();
            float dot = 0.f;
#pragma unroll
            for (int k = 0; k < kDim; k += 8) {
                uint4 u = *reinterpret_cast<const uint4*>(&s_d[w][k]);
                const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = __half22float2(h[j]);
                    dot = fmaf(q[k + 2 * j], f.x, dot);
                    dot = fmaf(q[k + 2 * j + 1], f.y, dot);
                }
            }
            run_max = fmaxf(run_max, dot * inv);
            __syncwarp();
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) run_max += __shfl_xor_sync(0xFFFFFFFFu, run_max, o);
        if (lane == 0) out[i] = run_max;
    }
}

int s4_simt_launch(const __half* Q, const int32_t* pids, int B, int n, const S4Docs& D, float* out,
                   cudaStream_t stream) {
    const int64_t total = (int64_t)B * n;
    if (total == 0) return RAGRT_OK;
    const int grid = (int)std::min<int64_t>(ceil_div(total, kS4Warps), (int64_t)num_sms() * 8);
    s4_simt<<<grid, kS4Warps * 32, 0, stream>>>(Q, pids, n, total, D, out);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

// ------------------------------------------------------------------ final top-k
__global__ void __launch_bounds__(1024)
final_topk(const int32_t* __restrict__ pids, const float* __restrict__ scores, int n,
           const uint32_t* __restrict__ preds, int num_preds, const uint32_t* __restrict__ masks, int k,
           int32_t* __restrict__ out_ids, float* __restrict__ out_scores) {
    extern __shared__ uint64_t keys[];
    const int b = blockIdx.x;
    const int NP = next_pow2(n);
    const uint32_t mask = (masks && preds) ? masks[b] : 0u;
    for (int i = threadIdx.x; i < NP; i += blockDim.x) {
        uint64_t key = 0;
        if (i < n) {
            const int32_t pid = pids[(int64_t)b * n + i];
            float s = scores[(int64_t)b * n + i];
            if (pid < 0 || (preds && pid >= num_preds)) s = -INFINITY;
            else if (mask && !(preds[pid] & mask)) s = -INFINITY;
            key = rank_key(s, pid);
        }
        keys[i] = key;
    }
    __syncthreads();
    cta_bitonic_sort<true>(keys, NP);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        out_ids[(int64_t)b * k + i] = rank_pid(keys[i]);
        if (out_scores) out_scores[(int64_t)b * k + i] = unordf((uint32_t)(keys[i] >> 32));
    }
}

int final_topk_launch(const int32_t* pids, const float* scores, int B, int n, const uint32_t* preds, int num_preds,
                      const uint32_t* masks, int k, int32_t* out_ids, float* out_scores, cudaStream_t stream) {
    const size_t smem = sizeof(uint64_t) * next_pow2(n);
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(final_topk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    final_topk<<<B, 1024, smem, stream>>>(pids, scores, n, preds, num_preds, masks, k, out_ids, out_scores);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

// ------------------------------------------------------------------ merge over doc shards
// gathered [world][2][B][k] 32-bit words (rank-major all-gather of every rank's (score as f32
// bits, global pid as int32; -1 = padding)) -> per query the top k_top by (score desc, pid
// asc), padding (pid -1) after every real pid of equal score.  A CTA per query, bitonic sort
// in shared memory.
__global__ void __launch_bounds__(256)
merge_shards_topk(const uint32_t* __restrict__ gathered, int world, int B, int k, int k_top,
                  int64_t* __restrict__ out_ids, float* __restrict__ out_scores) {
    extern __shared__ uint64_t mkeys[];
    const int b = blockIdx.x;
    const int n = world * k, NP = next_pow2(n);
    for (int i = threadIdx.x; i < NP; i += blockDim.x) {
        uint64_t key = 0;                                   // sorts after every real entry
        if (i < n) {
            const int r = i / k, j = i % k;
            const float s = __uint_as_float(gathered[(((int64_t)r * 2 + 0) * B + b) * k + j]);
            const int32_t pw = (int32_t)gathered[(((int64_t)r * 2 + 1) * B + b) * k + j];
            const int32_t pid = pw < 0 ? INT32_MAX : pw;
            key = rank_key(s, pid);
        }
        mkeys[i] = key;
    }
    __syncthreads();
    cta_bitonic_sort<true>(mkeys, NP);
    for (int i = threadIdx.x; i < k_top; i += blockDim.x) {
        const int32_t pid = rank_pid(mkeys[i]);
        out_ids[(int64_t)b * k_top + i] = pid == INT32_MAX ? -1 : pid;
        out_scores[(int64_t)b * k_top + i] = unordf((uint32_t)(mkeys[i] >> 32));
    }
}

}  // namespace ragrt

using namespace ragrt;

extern "C" int ragrt_merge_topk(const void* d_gathered, int32_t world, int32_t B, int32_t k, int32_t k_top,
                                int64_t* d_out_ids, float* d_out_scores, void* stream) {
    RAGRT_REQUIRE(d_gathered && d_out_ids && d_out_scores, "null argument");
    RAGRT_REQUIRE(world >= 1 && B >= 1 && k >= 1 && k_top >= 1 && k_top <= world * k,
                  "need world, B, k >= 1 and 1 <= k_top <= world * k");
    RAGRT_REQUIRE((int64_t)world * k <= 8192, "at most 8,192 entries per query");
    const size_t smem = sizeof(uint64_t) * next_pow2(world * k);
    merge_shards_topk<<<B, 256, smem, (cudaStream_t)stream>>>((const uint32_t*)d_gathered, world, B, k, k_top, d_out_ids, d_out_scores);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

extern "C" int ragrt_final_topk(const int32_t* d_pids, const float* d_scores, int32_t B, int32_t n,
                                const uint32_t* d_preds, int32_t num_preds, const uint32_t* d_masks, int32_t k,
                                int32_t* d_out_ids, float* d_out_scores, void* stream) {
    RAGRT_REQUIRE(d_pids && d_scores && d_out_ids, "null argument");
    RAGRT_REQUIRE(B >= 1 && n >= 1 && n <= RAGRT_MAX_CANDIDATES, "n must be in [1, %d]", RAGRT_MAX_CANDIDATES);
    RAGRT_REQUIRE(k >= 1 && k <= n, "k must be in [1, n]");
    RAGRT_REQUIRE(!d_preds || num_preds >= 1, "num_preds must be >= 1 with predicates");
    return final_topk_launch(d_pids, d_scores, B, n, d_preds, num_preds, d_masks, k, d_out_ids, d_out_scores,
                             (cudaStream_t)stream);
}

extern "C" int ragrt_tile_maxsim(const void* d_Q, const int32_t* d_pids, int32_t B, int32_t n,
                                 const int64_t* d_doc_offsets, const int32_t* d_doc_lens, int32_t num_passages,
                                 const int32_t* d_codes, const uint8_t* d_residuals, const void* d_centroids,
                                 const void* d_bucket_weights, const uint8_t* d_reversed_bit_map,
                                 const uint8_t* d_decomp_table, float* d_out, int32_t mode, void* stream) {
    RAGRT_REQUIRE(d_Q && d_doc_offsets && d_doc_lens && d_codes && d_residuals && d_centroids &&
                  d_bucket_weights && d_reversed_bit_map && d_decomp_table, "null argument");
    RAGRT_REQUIRE(B >= 1 && n >= 0, "B >= 1, n >= 0 required");
    if (n == 0) return RAGRT_OK;
    RAGRT_REQUIRE(d_pids && d_out, "null argument");
    RAGRT_REQUIRE(((uintptr_t)d_Q & 15) == 0 && ((uintptr_t)d_residuals & 15) == 0 &&
                  ((uintptr_t)d_centroids & 15) == 0, "Q, residuals and centroids must be 16-byte aligned");
    S4Docs D{d_doc_offsets, d_doc_lens, d_codes, d_residuals, (const __half*)d_centroids,
             (const __half*)d_bucket_weights, d_reversed_bit_map, d_decomp_table, num_passages, INT32_MAX};
    if (mode == 1) return s4_tc_launch((const __half*)d_Q, d_pids, B, n, D, d_out, (cudaStream_t)stream);
    return s4_simt_launch((const __half*)d_Q, d_pids, B, n, D, d_out, (cudaStream_t)stream);
}

extern "C" int ragrt_tile_maxsim_exact(const void* d_Q, const int32_t* d_pids, int32_t B, int32_t n,
                                       const int64_t* d_doc_offsets, const int32_t* d_doc_lens,
                                       int32_t num_passages, const void* d_doc_emb, float* d_out, void* stream) {
    RAGRT_REQUIRE(d_Q && d_doc_offsets && d_doc_lens && d_doc_emb, "null argument");
    RAGRT_REQUIRE(B >= 1 && n >= 0 && num_passages >= 0, "B >= 1, n >= 0, num_passages >= 0 required");
    if (n == 0) return RAGRT_OK;
    RAGRT_REQUIRE(d_pids && d_out, "null argument");
    RAGRT_REQUIRE(((uintptr_t)d_Q & 15) == 0 && ((uintptr_t)d_doc_emb & 15) == 0,
                  "Q and the doc embeddings must be 16-byte aligned");
    S4Docs D{d_doc_offsets, d_doc_lens, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, num_passages, 0,
             (const __half*)d_doc_emb};
    return s4_tc_launch((const __half*)d_Q, d_pids, B, n, D, d_out, (cudaStream_t)stream);
}
