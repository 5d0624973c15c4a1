// s3_common.cuh -- declarations shared by the Stage-3 sources and the C ABI.
#pragma once
#include "common.cuh"
#include "index.cuh"

namespace ragrt {

size_t s3_workspace_bytes(const ragrt_index* ix, int nq_sub);
int s3_max_sub_batch(const ragrt_index* ix, int B);
int s3_run(ragrt_index* ix, const int32_t* topc, const float* scores, int full_scores, const int32_t* ntok, int B,
           int rows, int kc, int n_eids, const uint32_t* masks, int K, int32_t* cand_pids, float* cand_sums,
           int64_t* num_touched, void* ws, size_t ws_bytes, cudaStream_t stream);

// The walk-once path (s3_walk.cu): per-query distinct lists, then one walk of each per pid range;
// ranges too dense for its hash rows are queued for the per-token kernel.
size_t s3_walk_lists_bytes(int nq, int LM);
size_t s3_walk_dense_bytes(const ragrt_index* ix, int nq);
int s3_walk_ranges(const ragrt_index* ix);
int s3_walk_run(ragrt_index* ix, const int32_t* topc, const float* scores, int full_scores, const int32_t* ntok,
                int q0, int nq, int rows, int kc, int n_eids, const uint32_t* masks, uint64_t* pool,
                unsigned long long* pool_count, unsigned int* work, unsigned long long* dense,
                unsigned int* dense_count, void* lists_ws, cudaStream_t stream);

// Exact per-query candidate selection from the ranking-key pool.
int s3_select_launch(const uint64_t* pool, int64_t pool_cap, const unsigned long long* counts, int q0, int nq, int K,
                     int32_t* cand_pids, float* cand_sums, int64_t* num_touched, unsigned long long* stats,
                     cudaStream_t stream);

// In-place bitonic sort of n (power of two) 64-bit keys in shared memory by the whole CTA.
template <bool kDescending>
__device__ __forceinline__ void cta_bitonic_sort(uint64_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const bool up = ((i & k) == 0) != kDescending;
                    const uint64_t x = a[i], y = a[ixj];
                    if ((x > y) == up) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__host__ __device__ __forceinline__ int next_pow2(int n) {
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

}  // namespace ragrt
