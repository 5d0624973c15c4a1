// capi.cu -- ragrt_weft_search: the whole `weft` search for a batch of queries in one
// stream-ordered sequence (Stage 2 -> Stages 1-3 -> Stage 4 -> final top-k) with no host
// synchronisation, using the index handle's workspace.  The reference runs these steps
// per query from Python and synchronises twice inside Stage 3
// (engines.py:573-609, optix_corr_torch_3d.cpp:558-723, ragrt_fused_kernel.cu:1044-1045,
// :1141-1143).
#include <algorithm>

#include "common.cuh"
#include "index.cuh"
#include "s2_common.cuh"
#include "s3_common.cuh"
#include "s4_common.cuh"

namespace ragrt {

namespace {
struct Carve {
    char* p;
    size_t used = 0;
    template <typename T>
    T* take(size_t count) {
        used = (used + 255) & ~(size_t)255;
        T* r = reinterpret_cast<T*>(p + used);
        used += sizeof(T) * count;
        return r;
    }
};
}  // namespace

static size_t s2_ws_bytes(int B, int NC, int nc) {
    const int kk = std::min(nc + 1, NC);
    return std::max(s2_partial_bytes(B, kRows, NC, nc, 1),
                    s2_tc_supported(kk, (int64_t)B * kRows) ? s2_tc_partial_bytes(B, kRows, NC, kk) : 0);
}

size_t weft_search_bytes(const ragrt_index* ix, int B, int nc, int K) {
    const int NC = ix->d.num_centroids;
    Carve c{nullptr};
    c.take<int32_t>((size_t)B * kRows * nc);       // topc
    c.take<float>((size_t)B * kRows * nc);         // scores
    c.take<uint64_t>(s2_ws_bytes(B, NC, nc) / sizeof(uint64_t) + 1);
    c.take<int32_t>((size_t)B * K);                // candidate pids
    c.take<float>((size_t)B * K);                  // candidate sums
    c.take<float>((size_t)B * K);                  // stage-4 scores
    c.take<char>(s3_workspace_bytes(ix, s3_max_sub_batch(ix, B)));
    return c.used + 256;
}

}  // namespace ragrt

using namespace ragrt;

static int weft_search_impl(ragrt_index* ix, const void* d_Q, const int32_t* d_ntok, int32_t B, int32_t nc,
                            int32_t n_eids, const uint32_t* d_masks, int32_t K, int32_t k_top, int32_t rerank_mode,
                            int32_t* d_out_ids, float* d_out_scores, void* const* events, cudaStream_t stream) {
    auto mark = [&](int i) -> int {
        if (events && events[i]) RAGRT_CUDA_TRY(cudaEventRecord((cudaEvent_t)events[i], stream));
        return RAGRT_OK;
    };
    RAGRT_REQUIRE(ix && d_Q && d_out_ids, "null argument");
    int rc = check_device(ix);
    if (rc) return rc;
    const int NC = ix->d.num_centroids;
    RAGRT_REQUIRE(B >= 1, "B must be >= 1");
    RAGRT_REQUIRE(nc >= 1 && nc <= RAGRT_MAX_PROBE && nc <= NC, "nc must be in [1, min(NC, %d)]", RAGRT_MAX_PROBE);
    RAGRT_REQUIRE(K >= 1 && K <= RAGRT_MAX_CANDIDATES && K <= ix->d.num_passages,
                  "K=%d must be in [1, min(N, %d)]", K, RAGRT_MAX_CANDIDATES);
    RAGRT_REQUIRE(k_top >= 1 && k_top <= K, "k_top must be in [1, K]");
    RAGRT_REQUIRE(n_eids >= 1, "n_eids must be >= 1");
    RAGRT_REQUIRE(((uintptr_t)d_Q & 15) == 0, "Q must be 16-byte aligned");
    rc = ensure_workspace(ix, weft_search_bytes(ix, B, nc, K), stream);
    if (rc) return rc;

    Carve c{(char*)ix->ws.base};
    int32_t* topc = c.take<int32_t>((size_t)B * kRows * nc);
    float* scores = c.take<float>((size_t)B * kRows * nc);
    uint64_t* partial = c.take<uint64_t>(s2_ws_bytes(B, NC, nc) / sizeof(uint64_t) + 1);
    int32_t* cand = c.take<int32_t>((size_t)B * K);
    float* csum = c.take<float>((size_t)B * K);
    float* fsc = c.take<float>((size_t)B * K);
    const int sub = s3_max_sub_batch(ix, B);
    const size_t s3b = s3_workspace_bytes(ix, sub);
    char* s3ws = c.take<char>(s3b);

    if ((rc = mark(0))) return rc;
    const int kk = std::min(nc + 1, NC);
    if (s2_tc_supported(kk, (int64_t)B * kRows)) {
        int* err = device_error_flag();
        if (!err) return fail(RAGRT_ERR_CUDA, "device error flag unavailable");
        rc = s2_tc_run((const __half*)d_Q, d_ntok, B, kRows, (const __half*)ix->d.centroids, NC, ix->cnorm, ix->cnmax,
                       nc, 1, topc, scores, nullptr, partial, err, stream);
    } else {
        rc = s2_run((const __half*)d_Q, d_ntok, B, kRows, (const __half*)ix->d.centroids, NC, nc, 1, topc, scores,
                    nullptr, nullptr, partial, stream);
    }
    if (rc || (rc = mark(1))) return rc;
    rc = s3_run(ix, topc, scores, 0, d_ntok, B, kRows, nc, std::min(n_eids, ix->d.num_eids), d_masks, K, cand, csum,
                nullptr, s3ws, s3b, stream);
    if (rc || (rc = mark(2))) return rc;
    S4Docs D{ix->d.doc_offsets, ix->d.doc_lens, ix->d.codes, ix->d.residuals, (const __half*)ix->d.centroids,
             (const __half*)ix->d.bucket_weights, ix->d.reversed_bit_map, ix->d.decomp_table, ix->d.num_passages,
             ix->d.num_centroids};
    rc = rerank_mode == 1 ? s4_tc_launch((const __half*)d_Q, cand, B, K, D, fsc, stream)
                          : s4_simt_launch((const __half*)d_Q, cand, B, K, D, fsc, stream);
    if (rc || (rc = mark(3))) return rc;
    rc = final_topk_launch(cand, fsc, B, K, ix->d.doc_predicates, ix->d.num_passages, d_masks, k_top, d_out_ids,
                           d_out_scores, stream);
    if (rc) return rc;
    return mark(4);
}

extern "C" int ragrt_index_tile_maxsim(ragrt_index* ix, const void* d_Q, const int32_t* d_pids, int32_t B, int32_t n,
                                       float* d_out, int32_t mode, void* stream) {
    RAGRT_REQUIRE(ix && d_Q, "null argument");
    int rc = check_device(ix);
    if (rc) return rc;
    RAGRT_REQUIRE(B >= 1 && n >= 0, "B >= 1, n >= 0 required");
    if (n == 0) return RAGRT_OK;
    RAGRT_REQUIRE(d_pids && d_out, "null argument");
    RAGRT_REQUIRE(((uintptr_t)d_Q & 15) == 0, "Q must be 16-byte aligned");
    S4Docs D{ix->d.doc_offsets, ix->d.doc_lens, ix->d.codes, ix->d.residuals, (const __half*)ix->d.centroids,
             (const __half*)ix->d.bucket_weights, ix->d.reversed_bit_map, ix->d.decomp_table, ix->d.num_passages,
             ix->d.num_centroids};
    if (mode == 1) return s4_tc_launch((const __half*)d_Q, d_pids, B, n, D, d_out, (cudaStream_t)stream);
    return s4_simt_launch((const __half*)d_Q, d_pids, B, n, D, d_out, (cudaStream_t)stream);
}

extern "C" int ragrt_weft_search(ragrt_index* ix, const void* d_Q, const int32_t* d_ntok, int32_t B, int32_t nc,
                                 int32_t n_eids, const uint32_t* d_masks, int32_t K, int32_t k_top,
                                 int32_t rerank_mode, int32_t* d_out_ids, float* d_out_scores, void* stream) {
    return weft_search_impl(ix, d_Q, d_ntok, B, nc, n_eids, d_masks, K, k_top, rerank_mode, d_out_ids, d_out_scores,
                            nullptr, (cudaStream_t)stream);
}

extern "C" int ragrt_weft_search_profiled(ragrt_index* ix, const void* d_Q, const int32_t* d_ntok, int32_t B,
                                          int32_t nc, int32_t n_eids, const uint32_t* d_masks, int32_t K,
                                          int32_t k_top, int32_t rerank_mode, int32_t* d_out_ids,
                                          float* d_out_scores, void* const* events, void* stream) {
    return weft_search_impl(ix, d_Q, d_ntok, B, nc, n_eids, d_masks, K, k_top, rerank_mode, d_out_ids, d_out_scores,
                            events, (cudaStream_t)stream);
}
