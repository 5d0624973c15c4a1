// s2_common.cuh -- exact fp16 score resolution, per-row top-k lists and the slice merge
// shared by the CUDA-core and tensor-core Stage-2 kernels.
#pragma once
#include "common.cuh"

namespace ragrt {

struct S2Candidate {
    uint64_t key;
    uint16_t h;
    bool enter;
};

// Exact dot product of two fp16 rows in fp64 (exact when |q| |c| < 32: every partial
// sum is a multiple of 2^-48 below 2^5), rounded once to fp16.
__device__ __forceinline__ uint16_t s2_exact(const __half* __restrict__ q, const __half* __restrict__ c) {
    double s = 0.0;
#pragma unroll 4
    for (int k = 0; k < kDim; k += 8) {
        uint4 uq = *reinterpret_cast<const uint4*>(q + k);
        uint4 uc = __ldg(reinterpret_cast<const uint4*>(c + k));
        const __half* hq = reinterpret_cast<const __half*>(&uq);
        const __half* hc = reinterpret_cast<const __half*>(&uc);
#pragma unroll
        for (int j = 0; j < 8; ++j) s = fma((double)__half2float(hq[j]), (double)__half2float(hc[j]), s);
    }
    uint16_t h = d2h_rn(s);
    return h == 0x8000u ? 0 : h;
}

// Accumulation error bounds, as a multiple of |q| |c| (>= sum |q_k c_k|):
//   CUDA cores, one fp32 FMA chain of 128 exact products: 129 * 2^-24 (7.69e-6);
//   tensor cores, 8 MMA steps of 16 exact products each, allowing the accumulator to be
//   aligned and truncated at every step: (8 * 17 + 1) * 2^-23 (1.63e-5); used with a 2x
//   margin as 512 * 2^-24.
constexpr float kEpsSimt = 7.8e-6f;
constexpr float kEpsTc = 3.06e-5f;

// Resolve the fp16 score of (row, centroid c) from its fp32 accumulation `acc`.
// qncn >= |q| |c|.  thr: the row's current k-th best key, meaningful when `full`.
// need_value: the caller needs the exact fp16 value even if it cannot enter.
__device__ __forceinline__ S2Candidate s2_resolve(float acc, float qncn, int c, uint64_t thr, bool full,
                                                  bool need_value, const __half* q, const __half* cr,
                                                  float eps_factor = kEpsSimt) {
    S2Candidate r;
    r.enter = false;
    r.h = 0;
    r.key = 0;
    float eps = fmaf(fabsf(acc), 1.2e-7f, qncn * eps_factor);   // accumulation bound + fp32 slack
    uint16_t hi = __half_as_ushort(__float2half_rn(acc + eps));
    if (!need_value && full && score_key(hi, (uint32_t)c) <= thr) return r;
    uint16_t lo = __half_as_ushort(__float2half_rn(acc - eps));
    uint16_t h = (hi == lo) ? hi : s2_exact(q, cr);
    if (h == 0x8000u) h = 0;
    r.h = h;
    r.key = score_key(h, (uint32_t)c);
    r.enter = !full || r.key > thr;
    return r;
}

// Insert into a descending list L[kk][32] (this lane's column) of length cnt.
__device__ __forceinline__ void s2_insert(uint64_t* L, int kk, int& cnt, uint64_t& thr, uint64_t key, int lane) {
    int i = cnt < kk ? cnt : kk - 1;
    while (i > 0 && L[(i - 1) * 32 + lane] < key) {
        L[i * 32 + lane] = L[(i - 1) * 32 + lane];
        --i;
    }
    L[i * 32 + lane] = key;
    if (cnt < kk) ++cnt;
    if (cnt == kk) thr = L[(kk - 1) * 32 + lane];
}

size_t s2_partial_bytes(int B, int rows, int NC, int nc, int impute);
int s2_check(const void* d_Q, const void* d_C, int B, int rows, int NC, int nc, const void* d_topc,
             const void* d_scores);
int s2_run(const __half* Q, const int32_t* ntok, int B, int rows, const __half* C, int NC, int nc, int impute,
           int32_t* topc, float* scores, float* m, __half* full16, uint64_t* partial, cudaStream_t stream);

// tensor-core Stage 2 (s2_tc.cu)
// the tensor-core path takes batches of at least one 128-row tile and kk <= 64
bool s2_tc_supported(int kk, int64_t rows_total);
size_t s2_tc_partial_bytes(int B, int rows, int NC, int kk);
int s2_tc_run(const __half* Q, const int32_t* ntok, int B, int rows, const __half* C, int NC, const float* cnorm,
              const float* cnmax, int nc, int impute, int32_t* topc, float* scores, float* m, uint64_t* partial,
              int* err, cudaStream_t stream);
int s2_norms_launch(const __half* C, int NC, float* cn, float* cnmax, cudaStream_t stream);

// Merge nslices sorted partial lists per (query, row) -> topc / scores / m.
// partial: [B][nslices][rows][kk] descending keys (0 = empty).
int s2_merge_launch(const uint64_t* partial, int nslices, const int32_t* ntok, int B, int rows, int kk,
                    int nc, int impute, int32_t* topc, float* scores, float* m, cudaStream_t stream);

}  // namespace ragrt
