// s3_select.cu -- exact candidate selection per query (the reference's
// `if (L == k) copy else torch::topk(sums, k)`, optix_corr_torch_3d.cpp:578-585):
//   U <= K : every touched passage, in ascending pid order, then (-1, -inf) padding;
//   U  > K : the K best by (sum desc, pid asc) -- an MSB-first radix select over the pool's
//            64-bit ranking keys (8-bit digits; it stops at the first digit whose boundary bucket
//            holds exactly the keys still needed), then a
//            bitonic sort of the K winners.
#include "s3_common.cuh"

namespace ragrt {

__global__ void __launch_bounds__(1024)
s3_select(const uint64_t* __restrict__ pool, int64_t cap, const unsigned long long* __restrict__ counts, int q0, int K,
          int32_t* __restrict__ cand_pids, float* __restrict__ cand_sums, int64_t* __restrict__ num_touched,
          unsigned long long* __restrict__ stats) {
    extern __shared__ uint64_t buf[];               // [next_pow2(K)]
    __shared__ unsigned hist[256];
    __shared__ uint64_t s_prefix, s_pmask;
    __shared__ unsigned s_need, s_nsel, s_done;
    const int qi = blockIdx.x, q = q0 + qi;
    const int64_t U = (int64_t)counts[qi];
    const uint64_t* keys = pool + (int64_t)qi * cap;
    int32_t* op = cand_pids + (int64_t)q * K;
    float* os = cand_sums + (int64_t)q * K;
    const int KP = next_pow2(K);
    if (U <= K) {
        for (int i = threadIdx.x; i < KP; i += blockDim.x) {
            uint64_t k = ~0ull;
            if (i < U) {
                const uint64_t key = keys[i];
                k = ((uint64_t)(uint32_t)rank_pid(key) << 32) | (key >> 32);
            }
            buf[i] = k;
        }
        __syncthreads();
        cta_bitonic_sort<false>(buf, KP);
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            if (i < U) {
                op[i] = (int32_t)(buf[i] >> 32);
                os[i] = unordf((uint32_t)(buf[i] & 0xFFFFFFFFu));
            } else {
                op[i] = -1;
                os[i] = -INFINITY;
            }
        }
    } else {
        if (threadIdx.x == 0) { s_prefix = 0; s_pmask = 0; s_need = (unsigned)K; s_nsel = 0; s_done = 0; }
        __syncthreads();
        for (int shift = 56; shift >= 0 && !s_done; shift -= 8) {
            for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
            __syncthreads();
            const uint64_t pre = s_prefix, pm = s_pmask;
            for (int64_t i = threadIdx.x; i < U; i += blockDim.x) {
                const uint64_t k = keys[i];
                if ((k & pm) == pre) atomicAdd(&hist[(k >> shift) & 255], 1u);
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                unsigned cum = 0, need = s_need;
                int d = 255;
                for (; d > 0; --d) {
                    if (cum + hist[d] >= need) break;
                    cum += hist[d];
                }
                s_need = need - cum;
                s_prefix = pre | ((uint64_t)d << shift);
                s_pmask = pm | ((uint64_t)255 << shift);
                // the boundary bucket holds exactly the keys still needed: the K winners are the keys
                // whose masked prefix is at least the new prefix
                if (hist[d] == need - cum) s_done = 1;
            }
            __syncthreads();
        }
        const uint64_t kth = s_prefix, kmask = s_pmask;
        for (int64_t i = threadIdx.x; i < U; i += blockDim.x) {
            const uint64_t k = keys[i];
            if ((k & kmask) >= kth) {
                const unsigned pos = atomicAdd(&s_nsel, 1u);
                if (pos < (unsigned)K) buf[pos] = k;
            }
        }
        for (int i = K + threadIdx.x; i < KP; i += blockDim.x) buf[i] = 0ull;
        __syncthreads();
        cta_bitonic_sort<true>(buf, KP);
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            op[i] = rank_pid(buf[i]);
            os[i] = unordf((uint32_t)(buf[i] >> 32));
        }
    }
    if (threadIdx.x == 0) {
        if (num_touched) num_touched[q] = U;
        if (stats) {
            atomicAdd(&stats[0], 1ull);
            atomicAdd(&stats[3], (unsigned long long)U);
            atomicAdd(&stats[5], (unsigned long long)(U < K ? U : K));
        }
    }
}

int s3_select_launch(const uint64_t* pool, int64_t pool_cap, const unsigned long long* counts, int q0, int nq, int K,
                     int32_t* cand_pids, float* cand_sums, int64_t* num_touched, unsigned long long* stats,
                     cudaStream_t stream) {
    const size_t smem = sizeof(uint64_t) * next_pow2(K);
    RAGRT_CUDA_TRY(cudaFuncSetAttribute(s3_select, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    s3_select<<<nq, 1024, smem, stream>>>(pool, pool_cap, counts, q0, K, cand_pids, cand_sums, num_touched, stats);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
