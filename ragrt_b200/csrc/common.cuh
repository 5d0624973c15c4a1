// common.cuh -- shared helpers of the ragrt_b200 CUDA sources (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "../../include/ragrt_b200.h"

namespace ragrt {

// ------------------------------------------------------------------ errors
void set_error(const char* fmt, ...);
void count_launch();
int fail(int code, const char* fmt, ...);          // set_error + return code

#define RAGRT_CUDA_TRY(call)                                                              \
    do {                                                                                  \
        cudaError_t e_ = (call);                                                          \
        if (e_ != cudaSuccess)                                                            \
            return ::ragrt::fail(RAGRT_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__, #call,   \
                                 cudaGetErrorString(e_));                                 \
    } while (0)

// every kernel launch of the library is followed by this check, which also counts it
#define RAGRT_LAUNCH_CHECK()                                                              \
    do {                                                                                  \
        ::ragrt::count_launch();                                                          \
        cudaError_t e_ = cudaGetLastError();                                              \
        if (e_ != cudaSuccess)                                                            \
            return ::ragrt::fail(RAGRT_ERR_CUDA, "%s:%d kernel launch: %s", __FILE__,       \
                                 __LINE__, cudaGetErrorString(e_));                       \
    } while (0)

#define RAGRT_REQUIRE(cond, ...)                                                          \
    do {                                                                                  \
        if (!(cond)) return ::ragrt::fail(RAGRT_ERR_ARG, __VA_ARGS__);                    \
    } while (0)

// ------------------------------------------------------------------ constants
constexpr int kDim = RAGRT_DIM;
constexpr int kRows = RAGRT_QUERY_ROWS;
constexpr int kBlockShift = 7;           // block sums over 128 lists (ragrt_fused_kernel.cu:208)
constexpr int kPidBits = 24;

// ------------------------------------------------------------------ fp16 ordering keys
// ord16: order-preserving map of fp16 bits to uint16 (larger value -> larger code).
__host__ __device__ __forceinline__ uint32_t ord16(uint16_t h) {
    return (h & 0x8000u) ? (uint32_t)(~h & 0xFFFFu) : (uint32_t)(h | 0x8000u);
}
__host__ __device__ __forceinline__ uint16_t unord16(uint32_t o) {
    return (uint16_t)((o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu));
}
// Selection key of a centroid score: (value desc, id asc) == larger key first.
__host__ __device__ __forceinline__ uint64_t score_key(uint16_t h, uint32_t id) {
    if (h == 0x8000u) h = 0;                                   // -0 == +0
    return ((uint64_t)ord16(h) << 32) | (uint64_t)(0xFFFFFFFFu - id);
}
__host__ __device__ __forceinline__ uint32_t key_id(uint64_t k) {
    return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu);
}
__host__ __device__ __forceinline__ uint16_t key_h(uint64_t k) { return unord16((uint32_t)(k >> 32)); }

// Order-preserving map of fp32 bits to uint32.
__device__ __forceinline__ uint32_t ordf(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unordf(uint32_t o) {
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}
// Ranking key of (score, pid): score desc, then pid asc (signed: -1 before 0).
__device__ __forceinline__ uint64_t rank_key(float s, int32_t pid) {
    return ((uint64_t)ordf(s) << 32) | (uint64_t)(uint32_t)(0x7FFFFFFF - pid);
}
__host__ __device__ __forceinline__ int32_t rank_pid(uint64_t k) {
    return (int32_t)(0x7FFFFFFF - (int64_t)(uint32_t)(k & 0xFFFFFFFFu));
}

// fp16 value in units of 2^-24 (non-negative fp16 only).
__device__ __forceinline__ uint64_t h_fixed24(uint16_t h) {
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    return e ? ((uint64_t)(m | 0x400) << (e - 1)) : (uint64_t)m;
}

// Correctly rounded double -> fp16 (round-to-odd to fp32, then RNE to fp16).
__device__ __forceinline__ uint16_t d2h_rn(double d) {
    float f = __double2float_rz(d);
    if ((double)f != d) f = __uint_as_float(__float_as_uint(f) | 1u);
    return __half_as_ushort(__float2half_rn(f));
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// 24-bit little-endian pid at posting i.
__device__ __forceinline__ int32_t load_pid24(const uint8_t* __restrict__ p, int64_t i) {
    const uint8_t* q = p + i * 3;
    return (int32_t)q[0] | ((int32_t)q[1] << 8) | ((int32_t)q[2] << 16);
}

int num_sms();
// Per-device error flag that kernels raise (bounded waits that gave up); read and cleared
// by ragrt_device_error().  Returns nullptr if it cannot be allocated.
int* device_error_flag();

}  // namespace ragrt
