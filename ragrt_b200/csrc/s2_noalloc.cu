// s2_noalloc.cu -- Stage 2 (centroid scores + per-token top-k) with no memory allocation.
//
// ragrt_centroid_topk_noalloc computes exactly what ragrt_centroid_topk computes without a
// full score matrix (d_full16 = NULL): the same kernels on the same inputs, so the outputs
// are bit-identical.  The only difference is where the kernels' scratch lives: instead of
// cudaMallocAsync / cudaFreeAsync per call, it uses one file-scope device array of
// kNoAllocScratchBytes (32 MiB) per device, and its own device-side error word.
//
//   * Set-up: the first call on a device (with that device current) looks up the array's
//     address with cudaGetSymbolAddress and caches it; that lookup may load this module
//     on the device.  Make that first call before any stream capture.
//   * Limit: a call whose scratch would exceed 32 MiB is rejected with RAGRT_ERR_ARG and
//     launches nothing.  The tensor-core path needs 4 (NC + 1) bytes of centroid norms plus,
//     per query row, 8 B x (64 nslices + 1) of candidate lists and 2 B per 128-centroid tile
//     of pre-pass bounds: about 17 MB for B = 256 queries x 32 rows x 65,536 centroids.
//   * Sharing: every call on a device uses the same array, which keeps the previous call's
//     contents; each call clears the centroid-norm maximum and rewrites the per-row
//     admission keys and tile bounds on its stream before they are read.  Calls whose kernels
//     overlap on the GPU (different streams, or different host threads) race on the array.
//   * Errors: a bounded wait that gives up inside the tensor-core kernel sets this entry
//     point's own error word, read by ragrt_centroid_topk_noalloc_error.
#include <mutex>

#include "common.cuh"
#include "s2_common.cuh"

namespace ragrt {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr size_t kAlign = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_s2_scratch[kNoAllocScratchBytes];
static __device__ int g_s2_err;

struct DeviceScratch {
    unsigned char* base = nullptr;
    int* err = nullptr;
};

std::mutex g_mu;
DeviceScratch g_dev[kMaxDevices];

size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

// Once per device, with that device current: addresses of the file-scope array and error word.
int scratch_for_current_device(DeviceScratch* out) {
    int dev = -1;
    RAGRT_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(RAGRT_ERR_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceScratch& s = g_dev[dev];
    if (!s.base) {
        void* p = nullptr;
        void* e = nullptr;
        cudaError_t rc = cudaGetSymbolAddress(&p, g_s2_scratch);
        if (rc != cudaSuccess) {
            cudaGetLastError();
            return fail(RAGRT_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                        cudaGetErrorString(rc));
        }
        rc = cudaGetSymbolAddress(&e, g_s2_err);
        if (rc != cudaSuccess) {
            cudaGetLastError();
            return fail(RAGRT_ERR_CUDA, "cudaGetSymbolAddress(error word) failed on device %d: %s", dev,
                        cudaGetErrorString(rc));
        }
        s.base = static_cast<unsigned char*>(p);
        s.err = static_cast<int*>(e);
    }
    *out = s;
    return RAGRT_OK;
}

}  // namespace
}  // namespace ragrt

using namespace ragrt;

extern "C" int ragrt_centroid_topk_noalloc(const void* d_Q, const int32_t* d_ntok, int32_t B, int32_t rows,
                                           const void* d_C, int32_t NC, int32_t nc, int32_t impute,
                                           int32_t* d_topc, float* d_scores, float* d_m, void* stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    int rc = s2_check(d_Q, d_C, B, rows, NC, nc, d_topc, d_scores);
    if (rc) return rc;
    const int kk = std::min(nc + (impute ? 1 : 0), NC);
    const bool tc = s2_tc_supported(kk, (int64_t)B * rows);
    const size_t norm_bytes = tc ? align_up(sizeof(float) * ((size_t)NC + 1)) : 0;
    const size_t list_bytes = tc ? s2_tc_partial_bytes(B, rows, NC, kk) : s2_partial_bytes(B, rows, NC, nc, impute);
    const size_t need = norm_bytes + align_up(list_bytes);
    if (need > kNoAllocScratchBytes)
        return fail(RAGRT_ERR_ARG,
                    "ragrt_centroid_topk_noalloc needs %zu bytes of scratch for B=%d rows=%d NC=%d nc=%d; "
                    "its static maximum is %zu bytes (use ragrt_centroid_topk or a smaller batch)",
                    need, (int)B, (int)rows, (int)NC, (int)nc, kNoAllocScratchBytes);
    DeviceScratch s;
    if ((rc = scratch_for_current_device(&s))) return rc;
    uint64_t* partial = reinterpret_cast<uint64_t*>(s.base + norm_bytes);
    if (tc) {
        float* norms = reinterpret_cast<float*>(s.base);
        rc = s2_norms_launch((const __half*)d_C, NC, norms, norms + NC, stream);   // clears norms[NC] first
        if (rc) return rc;
        return s2_tc_run((const __half*)d_Q, d_ntok, B, rows, (const __half*)d_C, NC, norms, norms + NC, nc, impute,
                         d_topc, d_scores, d_m, partial, s.err, stream);
    }
    return s2_run((const __half*)d_Q, d_ntok, B, rows, (const __half*)d_C, NC, nc, impute, d_topc, d_scores, d_m,
                  nullptr, partial, stream);
}

extern "C" int ragrt_centroid_topk_noalloc_error(int32_t reset) {
    DeviceScratch s;
    int rc = scratch_for_current_device(&s);
    if (rc) return rc;
    int h = 0;
    RAGRT_CUDA_TRY(cudaMemcpy(&h, s.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (reset && h) RAGRT_CUDA_TRY(cudaMemset(s.err, 0, sizeof(int)));
    return h;
}
