// index.cuh -- the bound index handle and its derived device structures.
#pragma once
#include "common.cuh"

// Workspace owned by a handle; grown on demand (never inside a stream capture).
struct ragrt_workspace {
    void* base = nullptr;
    size_t bytes = 0;
};

struct ragrt_index {
    ragrt_index_desc d;
    int device = 0;

    // pid ranges ("tiles") used by Stage 3: range r holds pids [r << w_shift, (r+1) << w_shift)
    int w_shift = 12;
    int num_ranges = 0;            // R = ceil(N / W)

    int64_t* list_off = nullptr;   // [num_lists + 1] posting offset of every list
    int64_t* cstart = nullptr;     // [NC] first posting of centroid c (row 0)
    int32_t* clists = nullptr;     // [NC] number of lists (chunks) of centroid c
    uint32_t* boff = nullptr;      // [NC, R + 1] first posting (relative to cstart) with pid >= r*W
    float* cnorm = nullptr;        // [NC] |c|_2 of each centroid, rounded up
    float* cnmax = nullptr;        // [1] max over cnorm

    ragrt_workspace ws;
    unsigned long long* stats = nullptr;   // [RAGRT_NUM_STATS]
    int count_distinct = 0;                // kept for the ABI; out[2] is always counted
    int s3_mode = 0;                       // 0 walk-once (+ per-token for dense ranges), 1 per-token only
    int s3_range = 0;                      // passages per walk-once range (0: automatic)
};

namespace ragrt {
// Make sure the handle's workspace holds at least `bytes` (synchronous growth).
int ensure_workspace(ragrt_index* ix, size_t bytes, cudaStream_t stream);
int check_device(const ragrt_index* ix);
}  // namespace ragrt
