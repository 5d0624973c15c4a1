// index.cu -- ragrt_index_create / destroy: validation of the bound plain-IVF arrays
// (layout of the reference's build_plain_ivf.py:28-68) and the derived structures the
// search kernels use instead of the reference's per-query binary searches
// (ragrt_fused_kernel.cu:187-213):
//   list_off  posting offset of every list, from the 128-list block sums
//   cstart    first posting of each centroid (its lists are consecutive in row 0)
//   boff      per centroid and pid range, the first posting with pid >= range start
//             (postings of a centroid are sorted by pid), so a Stage-3 tile reads only
//             the sub-list that falls in its pid range.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "index.cuh"
#include "s2_common.cuh"

namespace ragrt {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

static std::atomic<unsigned long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int* device_error_flag() {
    static int* flags[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!flags[dev]) {
        int* f = nullptr;
        if (cudaMalloc(&f, sizeof(int)) != cudaSuccess) { cudaGetLastError(); return nullptr; }
        cudaMemset(f, 0, sizeof(int));
        flags[dev] = f;
    }
    return flags[dev];
}

int num_sms() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

int check_device(const ragrt_index* ix) {
    int dev = -1;
    RAGRT_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != ix->device)
        return fail(RAGRT_ERR_DEVICE, "index lives on device %d, current device is %d", ix->device, dev);
    return RAGRT_OK;
}

int ensure_workspace(ragrt_index* ix, size_t bytes, cudaStream_t stream) {
    if (ix->ws.bytes >= bytes) return RAGRT_OK;
    RAGRT_CUDA_TRY(cudaStreamSynchronize(stream));
    if (ix->ws.base) RAGRT_CUDA_TRY(cudaFree(ix->ws.base));
    ix->ws.base = nullptr;
    ix->ws.bytes = 0;
    size_t grow = bytes + bytes / 4;
    cudaError_t e = cudaMalloc(&ix->ws.base, grow);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(RAGRT_ERR_CAPACITY, "workspace of %zu bytes could not be allocated: %s", grow,
                    cudaGetErrorString(e));
    }
    ix->ws.bytes = grow;
    return RAGRT_OK;
}

// ------------------------------------------------------------------ validation kernels
enum : int {
    kBadRow0 = 1 << 0,       // row 0 not non-decreasing / out of range
    kBadRows = 1 << 1,       // a subspace row 1-31 is not empty
    kBadEids = 1 << 2,       // a centroid's chunk ids are not 0..k-1
    kBadOffsets = 1 << 3,    // block sums disagree with the lengths
    kBadPids = 1 << 4,       // a pid >= N or pids of a centroid not sorted
    kBadDocs = 1 << 5,       // a passage's tokens are not inside [0, num_tokens)
    kBadCodes = 1 << 6,      // a doc token's centroid code is outside [0, NC)
};

// thread per passage: its tokens [doc_offsets[i], doc_offsets[i] + doc_lens[i]) lie inside
// the bound codes / residuals, so Stage 4 never reads past them
__global__ void k_check_docs(const int64_t* __restrict__ off, const int32_t* __restrict__ lens, int N,
                             int64_t num_tokens, int* __restrict__ flags) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    const int64_t o = off[i];
    const int32_t L = lens[i];
    if (o < 0 || L < 0 || o > num_tokens - L) atomicOr(flags, kBadDocs);
}

// every doc token's code must index a centroid row: Stage 4 gathers centroids[code]
__global__ void k_check_codes(const int32_t* __restrict__ codes, int64_t num_tokens, int NC,
                              int* __restrict__ flags) {
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < num_tokens;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t c = codes[i];
        bad |= (c < 0) | (c >= NC);
    }
    if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicOr(flags, kBadCodes);
}

__global__ void k_list_offsets(const int64_t* __restrict__ bsums, const uint16_t* __restrict__ lengths,
                               int64_t num_lists, int64_t* __restrict__ off) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i > num_lists) return;
    int64_t b = i >> kBlockShift;
    if (i == num_lists) {
        // total postings: the last list's offset + its length (computed by thread num_lists-1 too)
        if (num_lists == 0) { off[0] = 0; return; }
        int64_t j = num_lists - 1, bj = j >> kBlockShift;
        int64_t o = bsums[bj];
        for (int64_t k = bj << kBlockShift; k < j; ++k) o += lengths[k];
        off[i] = o + lengths[j];
        return;
    }
    int64_t o = bsums[b];
    for (int64_t k = b << kBlockShift; k < i; ++k) o += lengths[k];   // ragrt_fused_kernel.cu:208-213
    off[i] = o;
}

__global__ void k_check_lists(const int64_t* __restrict__ off, const uint16_t* __restrict__ lengths,
                              int64_t num_lists, int64_t num_postings, int* __restrict__ flags) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= num_lists) return;
    if (off[i + 1] - off[i] != (int64_t)lengths[i]) atomicOr(flags, kBadOffsets);
    if (i == num_lists - 1 && off[num_lists] != num_postings) atomicOr(flags, kBadOffsets);
}

template <typename EidT>
__global__ void k_centroids(const int64_t* __restrict__ rp, const EidT* __restrict__ eids, int NC,
                            int64_t num_lists, const int64_t* __restrict__ off, int64_t* __restrict__ cstart,
                            int32_t* __restrict__ clists, int* __restrict__ flags) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= NC) return;
    int64_t lo = rp[c], hi = rp[c + 1];
    if (lo < 0 || hi < lo || hi > num_lists) { atomicOr(flags, kBadRow0); clists[c] = 0; cstart[c] = 0; return; }
    for (int64_t i = lo; i < hi; ++i)
        if ((int64_t)eids[i] != i - lo) { atomicOr(flags, kBadEids); break; }
    clists[c] = (int32_t)(hi - lo);
    cstart[c] = (hi > lo) ? off[lo] : 0;
}

__global__ void k_check_rows(const int64_t* __restrict__ rp, int NC, int* __restrict__ flags) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // over rows 1..31
    int64_t total = (int64_t)31 * (NC + 1);
    if (i >= total) return;
    int64_t s = 1 + i / (NC + 1), c = i % (NC + 1);
    const int64_t* row = rp + s * (NC + 1);
    if (row[c] != row[0]) atomicOr(flags, kBadRows);
    if (i == 0 && rp[0] != 0) atomicOr(flags, kBadRow0);
}

// warp per centroid: pids of the centroid's postings are < N and non-decreasing
__global__ void k_check_pids(const uint8_t* __restrict__ packed, const int64_t* __restrict__ cstart,
                             const int32_t* __restrict__ clists, const int64_t* __restrict__ rp,
                             const int64_t* __restrict__ off, int NC, int N, int* __restrict__ flags) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= NC) return;
    int64_t a = cstart[warp];
    int64_t b = clists[warp] ? off[rp[warp] + clists[warp]] : a;
    bool bad = false;
    for (int64_t i = a + lane; i < b; i += 32) {
        int32_t p = load_pid24(packed, i);
        if (p >= N) bad = true;
        if (i > a && load_pid24(packed, i - 1) > p) bad = true;
    }
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(flags, kBadPids);
}

// thread per (centroid, range boundary): first posting with pid >= r * W (binary search)
__global__ void k_range_offsets(const uint8_t* __restrict__ packed, const int64_t* __restrict__ cstart,
                                const int32_t* __restrict__ clists, const int64_t* __restrict__ rp,
                                const int64_t* __restrict__ off, int NC, int R, int w_shift,
                                uint32_t* __restrict__ boff) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)NC * (R + 1)) return;
    int c = (int)(i / (R + 1)), r = (int)(i % (R + 1));
    int64_t a = cstart[c];
    int64_t n = clists[c] ? off[rp[c] + clists[c]] - a : 0;
    int64_t target = (int64_t)r << w_shift;
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        int64_t mid = (lo + hi) >> 1;
        if ((int64_t)load_pid24(packed, a + mid) < target) lo = mid + 1; else hi = mid;
    }
    boff[i] = (uint32_t)lo;
}

}  // namespace ragrt

using namespace ragrt;

extern "C" int ragrt_index_create(const ragrt_index_desc* desc, ragrt_index** out, void* stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    RAGRT_REQUIRE(desc && out, "null argument");
    *out = nullptr;
    const ragrt_index_desc& d = *desc;
    RAGRT_REQUIRE(d.csr_row_ptrs && d.csr_col_eids && d.csr_block_sums && d.csr_lengths && d.csr_packed_24,
                  "CSR arrays must be non-null");
    RAGRT_REQUIRE(d.doc_offsets && d.doc_lens && d.codes && d.residuals && d.centroids && d.bucket_weights &&
                  d.reversed_bit_map && d.decomp_table, "document arrays must be non-null");
    RAGRT_REQUIRE(d.eid_bytes == 1 || d.eid_bytes == 2, "csr_col_eids must be 8- or 16-bit");
    RAGRT_REQUIRE(d.num_passages >= 1 && d.num_passages <= (1 << kPidBits), "num_passages must be in [1, 2^24]");
    RAGRT_REQUIRE(d.num_centroids >= 1, "num_centroids must be >= 1");
    RAGRT_REQUIRE(d.num_eids >= 1 && d.num_eids <= (d.eid_bytes == 1 ? 256 : 65536),
                  "E=%d does not fit %d-bit eids", d.num_eids, 8 * d.eid_bytes);
    RAGRT_REQUIRE(d.num_lists >= 0 && d.num_postings >= 0 && d.num_tokens >= 0, "negative sizes");
    RAGRT_REQUIRE(((uintptr_t)d.residuals & 15) == 0 && ((uintptr_t)d.centroids & 15) == 0,
                  "residuals and centroids must be 16-byte aligned");

    ragrt_index* ix = new ragrt_index();
    ix->d = d;
    cudaGetDevice(&ix->device);
    const int NC = d.num_centroids;
    // pid range width: 4096 passages (3 Stage-3 CTAs per SM) unless the range-offset table
    // would exceed 1 GiB
    int ws = 12;
    while ((double)NC * (ceil_div(d.num_passages, (int64_t)1 << ws) + 1) * 4.0 > (double)(1ull << 30) && ws < 16)
        ++ws;
    ix->w_shift = ws;
    ix->num_ranges = (int)ceil_div(d.num_passages, (int64_t)1 << ws);
    const int R = ix->num_ranges;

    auto cleanup = [&](int code) {
        ragrt_index_destroy(ix);
        return code;
    };
    int* flags = nullptr;
#define TRY_ALLOC(p, n)                                                                      \
    do {                                                                                     \
        cudaError_t e_ = cudaMalloc(&(p), (n));                                              \
        if (e_ != cudaSuccess) {                                                             \
            cudaGetLastError();                                                              \
            if (flags) cudaFree(flags);                                                      \
            return cleanup(fail(RAGRT_ERR_CUDA, "cudaMalloc(%zu): %s", (size_t)(n), cudaGetErrorString(e_))); \
        }                                                                                    \
    } while (0)
    TRY_ALLOC(flags, sizeof(int));
    TRY_ALLOC(ix->list_off, sizeof(int64_t) * (d.num_lists + 1));
    TRY_ALLOC(ix->cstart, sizeof(int64_t) * NC);
    TRY_ALLOC(ix->clists, sizeof(int32_t) * NC);
    TRY_ALLOC(ix->boff, sizeof(uint32_t) * (size_t)NC * (R + 1));
    TRY_ALLOC(ix->cnorm, sizeof(float) * NC);
    TRY_ALLOC(ix->cnmax, sizeof(float));
    TRY_ALLOC(ix->stats, sizeof(unsigned long long) * RAGRT_NUM_STATS);
#undef TRY_ALLOC
    cudaMemsetAsync(flags, 0, sizeof(int), stream);
    cudaMemsetAsync(ix->stats, 0, sizeof(unsigned long long) * RAGRT_NUM_STATS, stream);

    const int T = 256;
    k_list_offsets<<<(unsigned)ceil_div(d.num_lists + 1, T), T, 0, stream>>>(d.csr_block_sums, d.csr_lengths,
                                                                          d.num_lists, ix->list_off);
    if (d.num_lists > 0)
        k_check_lists<<<(unsigned)ceil_div(d.num_lists, T), T, 0, stream>>>(ix->list_off, d.csr_lengths, d.num_lists,
                                                                           d.num_postings, flags);
    k_check_rows<<<(unsigned)ceil_div((int64_t)31 * (NC + 1), T), T, 0, stream>>>(d.csr_row_ptrs, NC, flags);
    k_check_docs<<<(unsigned)ceil_div((int64_t)d.num_passages, T), T, 0, stream>>>(d.doc_offsets, d.doc_lens,
                                                                                 d.num_passages, d.num_tokens, flags);
    if (d.num_tokens > 0)
        k_check_codes<<<(unsigned)std::min<int64_t>(ceil_div(d.num_tokens, T), (int64_t)num_sms() * 8), T, 0,
                        stream>>>(d.codes, d.num_tokens, NC, flags);
    if (d.eid_bytes == 1)
        k_centroids<uint8_t><<<(unsigned)ceil_div(NC, T), T, 0, stream>>>(
            d.csr_row_ptrs, (const uint8_t*)d.csr_col_eids, NC, d.num_lists, ix->list_off, ix->cstart, ix->clists, flags);
    else
        k_centroids<uint16_t><<<(unsigned)ceil_div(NC, T), T, 0, stream>>>(
            d.csr_row_ptrs, (const uint16_t*)d.csr_col_eids, NC, d.num_lists, ix->list_off, ix->cstart, ix->clists, flags);
    int h_flags = 0;
    cudaError_t e = cudaMemcpyAsync(&h_flags, flags, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) { cudaFree(flags); return cleanup(fail(RAGRT_ERR_CUDA, "index validation: %s", cudaGetErrorString(e))); }
    if (h_flags) {
        cudaFree(flags);
        return cleanup(fail(RAGRT_ERR_INDEX,
                            "not a valid plain-IVF index (flags 0x%x:%s%s%s%s%s%s)", h_flags,
                            (h_flags & kBadRow0) ? " row_ptrs row 0 malformed;" : "",
                            (h_flags & kBadRows) ? " subspace rows 1-31 not empty (weft needs a plain-IVF index);" : "",
                            (h_flags & kBadEids) ? " chunk ids of a centroid are not 0..k-1;" : "",
                            (h_flags & kBadOffsets) ? " block sums disagree with lengths / num_postings;" : "",
                            (h_flags & kBadDocs) ? " doc_offsets / doc_lens reach outside the num_tokens codes;" : "",
                            (h_flags & kBadCodes) ? " a doc token's code is outside [0, num_centroids);" : ""));
    }
    k_check_pids<<<(unsigned)ceil_div((int64_t)NC * 32, T), T, 0, stream>>>(d.csr_packed_24, ix->cstart, ix->clists,
                                                                          d.csr_row_ptrs, ix->list_off, NC,
                                                                          d.num_passages, flags);
    k_range_offsets<<<(unsigned)ceil_div((int64_t)NC * (R + 1), T), T, 0, stream>>>(
        d.csr_packed_24, ix->cstart, ix->clists, d.csr_row_ptrs, ix->list_off, NC, R, ws, ix->boff);
    if (s2_norms_launch((const __half*)d.centroids, NC, ix->cnorm, ix->cnmax, stream) != RAGRT_OK) {
        cudaFree(flags);
        return cleanup(RAGRT_ERR_CUDA);
    }
    e = cudaMemcpyAsync(&h_flags, flags, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    cudaFree(flags);
    if (e != cudaSuccess) return cleanup(fail(RAGRT_ERR_CUDA, "index build: %s", cudaGetErrorString(e)));
    if (h_flags & kBadPids)
        return cleanup(fail(RAGRT_ERR_INDEX, "not a valid plain-IVF index: a pid >= num_passages or the "
                                             "postings of a centroid are not sorted by pid"));
    *out = ix;
    return RAGRT_OK;
}

extern "C" int ragrt_index_destroy(ragrt_index* ix) {
    if (!ix) return RAGRT_OK;
    cudaFree(ix->list_off);
    cudaFree(ix->cstart);
    cudaFree(ix->clists);
    cudaFree(ix->boff);
    cudaFree(ix->cnorm);
    cudaFree(ix->cnmax);
    cudaFree(ix->stats);
    cudaFree(ix->ws.base);
    delete ix;
    return RAGRT_OK;
}

extern "C" int ragrt_index_count_distinct(ragrt_index* ix, int32_t enable) {
    RAGRT_REQUIRE(ix, "null index");
    ix->count_distinct = enable ? 1 : 0;
    return RAGRT_OK;
}

extern "C" int ragrt_index_set_stage3_mode(ragrt_index* ix, int32_t mode, int32_t range_passages) {
    RAGRT_REQUIRE(ix, "null index");
    RAGRT_REQUIRE(mode == 0 || mode == 1, "stage-3 mode must be 0 (walk-once) or 1 (per-token)");
    RAGRT_REQUIRE(range_passages >= 0 && range_passages <= (1 << 20), "range_passages must be in [0, 2^20]");
    ix->s3_mode = mode;
    ix->s3_range = range_passages;
    return RAGRT_OK;
}

extern "C" int ragrt_index_stats(ragrt_index* ix, uint64_t* out, int32_t reset) {
    RAGRT_REQUIRE(ix, "null index");
    if (out) {
        RAGRT_CUDA_TRY(cudaDeviceSynchronize());
        RAGRT_CUDA_TRY(cudaMemcpy(out, ix->stats, sizeof(uint64_t) * RAGRT_NUM_STATS, cudaMemcpyDeviceToHost));
    }
    if (reset) {
        RAGRT_CUDA_TRY(cudaMemset(ix->stats, 0, sizeof(uint64_t) * RAGRT_NUM_STATS));
        RAGRT_CUDA_TRY(cudaDeviceSynchronize());
    }
    return RAGRT_OK;
}

extern "C" const char* ragrt_last_error(void) { return ragrt::g_err; }
extern "C" int ragrt_device_error(int32_t reset) {
    int* f = ragrt::device_error_flag();
    if (!f) return ragrt::fail(RAGRT_ERR_CUDA, "device error flag unavailable");
    int h = 0;
    RAGRT_CUDA_TRY(cudaMemcpy(&h, f, sizeof(int), cudaMemcpyDeviceToHost));
    if (reset && h) RAGRT_CUDA_TRY(cudaMemset(f, 0, sizeof(int)));
    return h;
}

extern "C" uint64_t ragrt_launch_count(void) { return ragrt::g_launches.load(); }
extern "C" const char* ragrt_version(void) { return "ragrt_b200 0.1.0 (sm_100a)"; }
