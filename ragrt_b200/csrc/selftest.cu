// selftest.cu -- exercises the bounded-wait error path that every pipelined kernel uses: one
// warp waits on an mbarrier that nothing arrives on with tc::mbar_wait_or_abort (suspend-time
// hinted polls, a poll limit, a global-time deadline and the shared abort flag), gives up after
// `polls` polls, raises the device error flag (value 3) and returns, leaving the context usable.
#include "common.cuh"
#include "tc.cuh"

namespace ragrt {

__global__ void k_wait_timeout(uint32_t polls, int* err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        abort_flag = 0;
        tc::mbar_fence_init();
    }
    __syncwarp();
    // phase 0 never completes: the first lane to reach the limit raises the abort flag, the others
    // see it within four polls
    const bool ok = tc::mbar_wait_or_abort(&bar, 0, &abort_flag, polls);
    __syncwarp();
    if (!__all_sync(0xFFFFFFFFu, ok) && threadIdx.x == 0) atomicExch(err, abort_flag == 1 ? 3 : 4);
}

}  // namespace ragrt

using namespace ragrt;

extern "C" int ragrt_selftest_wait_timeout(uint32_t polls, void* stream) {
    RAGRT_REQUIRE(polls >= 1 && polls <= (1u << 24), "polls must be in [1, 2^24]");
    int* err = device_error_flag();
    if (!err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
    k_wait_timeout<<<1, 32, 0, (cudaStream_t)stream>>>(polls, err);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}
