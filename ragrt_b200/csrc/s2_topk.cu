// s2_topk.cu -- Stage 2: fp16 centroid scores + per-token top-(nc+1) with missing-score
// imputation (the reference's weft_prep.native_prep, src/weft_prep.py:32-47).
//
// Exactness.  The reference rounds a tensor-core fp32 accumulation to fp16 and takes
// torch.topk; both the accumulation order and the tie order are unspecified.  Here every
// selected score is the exact dot product rounded once (RNE), ties broken by the lower
// centroid id, so the result is a deterministic function of the inputs:
//   acc    fp32 accumulation (fixed order on CUDA cores, tensor cores in s2_tc.cu), with
//          |acc - exact| <= eps = 129 * 2^-24 * |q| * |c|  (products of fp16 are exact in
//          fp32; Cauchy-Schwarz bounds sum |q_k c_k| by |q| |c|).
//   If RN16(acc - eps) == RN16(acc + eps) that is RN16(exact); otherwise (a rounding-
//   boundary value) the dot product is recomputed in fp64, which is exact when
//   |q| |c| < 32, and rounded once.  Values whose upper bound cannot enter the running
//   top-k are skipped without rounding.
#include <algorithm>

#include "common.cuh"
#include "s2_common.cuh"

namespace ragrt {

// One CTA: one query (up to 32 rows = lanes) x a slice of centroids; warp w takes
// centroids slice_start + w, + NW, ...  Each (warp, row) keeps a sorted top-kk list in
// shared memory; the CTA merges its warps' lists into partial[b][slice][row][kk].
constexpr int kS2Warps = 4;

template <bool kFull>
__global__ void __launch_bounds__(kS2Warps * 32)
s2_simt_partial(const __half* __restrict__ Q, const int32_t* __restrict__ ntok, int rows,
                const __half* __restrict__ C, int NC, int kk, int slice_len,
                uint64_t* __restrict__ partial, __half* __restrict__ full16) {
    extern __shared__ uint64_t s_lists[];            // [kS2Warps][kk][32]
    const int b = blockIdx.y, slice = blockIdx.x, nslices = gridDim.x;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nt = ntok ? min(ntok[b], rows) : rows;
    const bool active = lane < nt;
    const __half* q = Q + ((int64_t)b * rows + (active ? lane : 0)) * kDim;

    float qf[kDim];
#pragma unroll
    for (int k = 0; k < kDim; k += 8) {
        uint4 u = *reinterpret_cast<const uint4*>(q + k);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float2 f = __half22float2(h[j]);
            qf[k + 2 * j] = f.x;
            qf[k + 2 * j + 1] = f.y;
        }
    }
    float qn = 0.f;
#pragma unroll
    for (int k = 0; k < kDim; ++k) qn = fmaf(qf[k], qf[k], qn);
    qn = __fsqrt_ru(qn) * (1.0f + 1e-6f);

    // empty lists (key 0): a warp may see fewer than kk centroids of its slice
    for (int i = threadIdx.x; i < kS2Warps * kk * 32; i += blockDim.x) s_lists[i] = 0ull;
    __syncthreads();
    uint64_t* L = s_lists + (size_t)w * kk * 32;
    int cnt = 0;
    uint64_t thr = 0;
    const int c0 = slice * slice_len, c1 = min(NC, c0 + slice_len);
    for (int c = c0 + w; c < c1; c += kS2Warps) {
        const __half* cr = C + (int64_t)c * kDim;
        float acc = 0.f, cn = 0.f;
#pragma unroll
        for (int k = 0; k < kDim; k += 8) {
            uint4 u = __ldg(reinterpret_cast<const uint4*>(cr + k));
            const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f = __half22float2(h[j]);
                acc = fmaf(qf[k + 2 * j], f.x, acc);
                acc = fmaf(qf[k + 2 * j + 1], f.y, acc);
                cn = fmaf(f.x, f.x, cn);
                cn = fmaf(f.y, f.y, cn);
            }
        }
        if (!active) continue;
        cn = __fsqrt_ru(cn) * (1.0f + 1e-6f);
        S2Candidate cand = s2_resolve(acc, qn * cn, c, thr, cnt >= kk, kFull, q, cr);
        if (kFull) full16[((int64_t)b * rows + lane) * NC + c] = __ushort_as_half(cand.h);
        if (!cand.enter) continue;
        s2_insert(L, kk, cnt, thr, cand.key, lane);
    }
    __syncthreads();
    // merge the kS2Warps lists of each row (lane) into this slice's partial list
    if (w == 0) {
        int pos[kS2Warps];
        int n[kS2Warps];
        (void)n;
        for (int i = 0; i < kS2Warps; ++i) pos[i] = 0;
        uint64_t* out = partial + (((int64_t)b * nslices + slice) * rows + lane) * kk;
        if (lane < rows) {
            for (int j = 0; j < kk; ++j) {
                uint64_t best = 0;
                int bi = -1;
                for (int i = 0; i < kS2Warps; ++i) {
                    if (pos[i] < kk) {
                        uint64_t v = s_lists[((size_t)i * kk + pos[i]) * 32 + lane];
                        if (v > best) { best = v; bi = i; }
                    }
                }
                if (bi >= 0) pos[bi]++;
                out[j] = best;                        // 0 = empty slot
            }
        }
    }
}

}  // namespace ragrt

using namespace ragrt;

namespace ragrt {

void s2_plan(int B, int NC, int& nslices, int& slice_len) {
    // slices so that the grid covers the GPU at least twice (at most 32 slices for the merge)
    const int sms = num_sms();
    nslices = (int)std::min<int64_t>(32, std::max<int64_t>(1, ceil_div(2 * sms, B)));
    nslices = (int)std::min<int64_t>(nslices, ceil_div(NC, kS2Warps));
    slice_len = (int)ceil_div(NC, nslices);
    nslices = (int)ceil_div(NC, slice_len);
}

size_t s2_partial_bytes(int B, int rows, int NC, int nc, int impute) {
    int ns, sl;
    s2_plan(B, NC, ns, sl);
    const int kk = std::min(nc + (impute ? 1 : 0), NC);
    return sizeof(uint64_t) * (size_t)B * ns * rows * kk;
}

int s2_check(const void* d_Q, const void* d_C, int B, int rows, int NC, int nc, const void* d_topc,
             const void* d_scores) {
    RAGRT_REQUIRE(d_Q && d_C && d_topc && d_scores, "null argument");
    RAGRT_REQUIRE(B >= 1 && rows >= 1 && rows <= kRows, "B >= 1 and 1 <= rows <= 32 required");
    RAGRT_REQUIRE(NC >= 1 && nc >= 1 && nc <= RAGRT_MAX_PROBE, "nc must be in [1, %d]", RAGRT_MAX_PROBE);
    RAGRT_REQUIRE(((uintptr_t)d_Q & 15) == 0 && ((uintptr_t)d_C & 15) == 0, "Q and C must be 16-byte aligned");
    return RAGRT_OK;
}

int s2_run(const __half* Q, const int32_t* ntok, int B, int rows, const __half* C, int NC, int nc, int impute,
           int32_t* topc, float* scores, float* m, __half* full16, uint64_t* partial, cudaStream_t stream) {
    const int kk = std::min(nc + (impute ? 1 : 0), NC);
    int nslices, slice_len;
    s2_plan(B, NC, nslices, slice_len);
    const size_t smem = sizeof(uint64_t) * kS2Warps * kk * 32;
    dim3 grid(nslices, B);
    if (full16) {
        RAGRT_CUDA_TRY(cudaFuncSetAttribute(s2_simt_partial<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        s2_simt_partial<true><<<grid, kS2Warps * 32, smem, stream>>>(Q, ntok, rows, C, NC, kk, slice_len, partial, full16);
    } else {
        RAGRT_CUDA_TRY(cudaFuncSetAttribute(s2_simt_partial<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        s2_simt_partial<false><<<grid, kS2Warps * 32, smem, stream>>>(Q, ntok, rows, C, NC, kk, slice_len, partial, nullptr);
    }
    RAGRT_LAUNCH_CHECK();
    return s2_merge_launch(partial, nslices, ntok, B, rows, kk, nc, impute, topc, scores, m, stream);
}

}  // namespace ragrt

extern "C" int ragrt_centroid_topk(const void* d_Q, const int32_t* d_ntok, int32_t B, int32_t rows,
                                   const void* d_C, int32_t NC, int32_t nc, int32_t impute,
                                   int32_t* d_topc, float* d_scores, float* d_m, void* d_full16,
                                   void* stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    int rc = s2_check(d_Q, d_C, B, rows, NC, nc, d_topc, d_scores);
    if (rc) return rc;
    const int kk = std::min(nc + (impute ? 1 : 0), NC);
    uint64_t* partial = nullptr;
    if (!d_full16 && s2_tc_supported(kk, (int64_t)B * rows)) {
        // tensor-core path: centroid norms for the exactness bound, then the fused GEMM + top-k
        int* err = device_error_flag();
        if (!err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
        float* norms = nullptr;
        RAGRT_CUDA_TRY(cudaMallocAsync((void**)&norms, sizeof(float) * (NC + 1), stream));
        RAGRT_CUDA_TRY(cudaMallocAsync((void**)&partial, s2_tc_partial_bytes(B, rows, NC, kk), stream));
        rc = s2_norms_launch((const __half*)d_C, NC, norms, norms + NC, stream);
        if (!rc)
            rc = s2_tc_run((const __half*)d_Q, d_ntok, B, rows, (const __half*)d_C, NC, norms, norms + NC, nc, impute,
                           d_topc, d_scores, d_m, partial, err, stream);
        cudaFreeAsync(partial, stream);
        cudaFreeAsync(norms, stream);
        return rc;
    }
    RAGRT_CUDA_TRY(cudaMallocAsync((void**)&partial, s2_partial_bytes(B, rows, NC, nc, impute), stream));
    rc = s2_run((const __half*)d_Q, d_ntok, B, rows, (const __half*)d_C, NC, nc, impute, d_topc, d_scores, d_m,
                (__half*)d_full16, partial, stream);
    cudaFreeAsync(partial, stream);
    return rc;
}

namespace ragrt {

// warp per (query, row); lane s walks slice s's sorted list (nslices <= 32)
__global__ void s2_merge(const uint64_t* __restrict__ partial, int nslices, const int32_t* __restrict__ ntok,
                         int B, int rows, int kk, int nc, int impute, int32_t* __restrict__ topc,
                         float* __restrict__ scores, float* __restrict__ m) {
    extern __shared__ uint64_t s_keys[];                 // [warps][kk]
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + wib;
    if (gw >= (int64_t)B * rows) return;
    const int b = (int)(gw / rows), t = (int)(gw % rows);
    const int ncol = min(nc, kk);
    const bool imputed = impute && kk > nc;
    const int nt = ntok ? min(ntok[b], rows) : rows;
    int32_t* tc = topc + ((int64_t)b * rows + t) * ncol;
    float* sc = scores + ((int64_t)b * rows + t) * ncol;
    if (t >= nt) {
        for (int j = lane; j < ncol; j += 32) { tc[j] = -1; sc[j] = 0.f; }
        if (m && lane == 0) m[(int64_t)b * rows + t] = 0.f;
        return;
    }
    uint64_t* keys = s_keys + (size_t)wib * kk;
    const uint64_t* P = partial + (((int64_t)b * nslices + lane) * rows + t) * kk;
    int pos = 0;
    for (int j = 0; j < kk; ++j) {
        uint64_t h = (lane < nslices && pos < kk) ? P[pos] : 0ull;
        uint64_t mx = h;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            uint64_t other = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
            mx = other > mx ? other : mx;
        }
        unsigned win = __ballot_sync(0xFFFFFFFFu, h == mx && mx != 0);
        if (win && lane == __ffs(win) - 1) ++pos;
        if (lane == 0) keys[j] = mx;
    }
    __syncwarp();
    float mt = 0.f;
    if (imputed) mt = __half2float(__ushort_as_half(key_h(keys[nc])));
    for (int j = lane; j < ncol; j += 32) {
        uint64_t k = keys[j];
        tc[j] = k ? (int32_t)key_id(k) : -1;
        float v = __half2float(__ushort_as_half(key_h(k)));
        sc[j] = imputed ? __fsub_rn(v, mt) : v;
    }
    if (m && lane == 0) m[(int64_t)b * rows + t] = imputed ? mt : 0.f;
}

int s2_merge_launch(const uint64_t* partial, int nslices, const int32_t* ntok, int B, int rows, int kk, int nc,
                    int impute, int32_t* topc, float* scores, float* m, cudaStream_t stream) {
    if (nslices > 32) return fail(RAGRT_ERR_ARG, "internal: %d slices > 32", nslices);
    const int warps = 4;
    int64_t nw = (int64_t)B * rows;
    size_t smem = sizeof(uint64_t) * warps * kk;
    s2_merge<<<(unsigned)ceil_div(nw, warps), warps * 32, smem, stream>>>(partial, nslices, ntok, B, rows, kk, nc,
                                                                          impute, topc, scores, m);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}

}  // namespace ragrt
