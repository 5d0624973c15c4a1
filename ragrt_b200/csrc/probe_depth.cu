// probe_depth.cu -- per-token probe depth under a filter (the `weft_adapt` engine's rule,
// src/weft_prep.py:75-106).
//
// A token's probes are its centroids best first.  With pass_c / tot_c the postings per
// centroid that pass the filter / all postings and sel the filter's global pass rate, the
// token's target is sel x (all postings of its first nc probes): the passing postings an
// uncorrelated filter would leave.  The token is "short" when its first nc probes hold fewer
// than slack x target passing postings, and it needs the smallest depth d in [nc, ncap] whose
// first d probes hold the target: 1 + the number of prefixes (of the first ncap probes) whose
// passing count is still below the target, clamped to [nc, ncap].  Counts are compared in fp32
// as torch compares an int64 count with an fp32 target.
//
// One warp per token: the prefix sums run as warp scans over 32 probes at a time.
#include "common.cuh"

namespace ragrt {

__global__ void k_probe_depth(const int32_t* __restrict__ topc, int ntok, int width, const int64_t* __restrict__ pass_c,
                              const int64_t* __restrict__ tot_c, int NC, float sel, float slack, int nc, int ncap,
                              int32_t* __restrict__ short_out, int32_t* __restrict__ need_out) {
    const int t = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= ntok) return;
    const int32_t* row = topc + (int64_t)t * width;
    // totals over the first nc probes
    long long tot = 0, pass = 0;
    for (int j = lane; j < nc; j += 32) {
        const int c = row[j];
        if (c >= 0 && c < NC) {
            tot += tot_c[c];
            pass += pass_c[c];
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
        pass += __shfl_xor_sync(0xFFFFFFFFu, pass, o);
    }
    const float target = (float)tot * sel;
    // prefixes of the first ncap probes whose passing count is below the target
    long long run = 0;
    int below = 0;
    for (int j0 = 0; j0 < ncap; j0 += 32) {
        const int j = j0 + lane;
        long long v = 0;
        if (j < ncap) {
            const int c = row[j];
            if (c >= 0 && c < NC) v = pass_c[c];
        }
        long long incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += y;
        }
        const bool lt = j < ncap && (float)(run + incl) < target;
        below += __popc(__ballot_sync(0xFFFFFFFFu, lt));
        run += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) {
        short_out[t] = (float)pass < slack * target ? 1 : 0;
        need_out[t] = min(max(below + 1, nc), ncap);
    }
}

}  // namespace ragrt

using namespace ragrt;

extern "C" int ragrt_probe_depth(const int32_t* d_topc, int32_t ntok, int32_t width, const int64_t* d_pass_c,
                                 const int64_t* d_tot_c, int32_t NC, float sel, float slack, int32_t nc, int32_t ncap,
                                 int32_t* d_short, int32_t* d_need, void* stream) {
    RAGRT_REQUIRE(d_topc && d_pass_c && d_tot_c && d_short && d_need, "null argument");
    RAGRT_REQUIRE(ntok >= 0 && NC >= 1, "ntok >= 0 and NC >= 1 required");
    RAGRT_REQUIRE(nc >= 1 && nc <= ncap && ncap <= width, "need 1 <= nc <= ncap <= width");
    if (ntok == 0) return RAGRT_OK;
    k_probe_depth<<<(unsigned)ceil_div((int64_t)ntok * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        d_topc, ntok, width, d_pass_c, d_tot_c, NC, sel, slack, nc, ncap, d_short, d_need);
    RAGRT_LAUNCH_CHECK();
    return RAGRT_OK;
}
