// ref_shim.cu -- TEST INFRASTRUCTURE ONLY.  Drives the reference's own CUDA kernels
// (compiled unmodified from the reference source tree by oracle/build_ref.sh) in the
// `weft` configuration, so tests can compare the product path against the reference
// implementation itself on the same device buffers.
//
// The call sequence restates CorrIndex3D::stages23 / rerank of the reference
// (src/optix_corr_torch_3d.cpp:558-607) without OptiX or torch:
//   all-codewords Stage 1 (launch_all_codewords_stage1, ragrt_fused_kernel.cu:737-742)
//   -> ragrt_stage2 (:979-1014) -> ragrt_stage3_sparse (:1038-1157)
// with codeword weight 0, compact scores and the 64-bit radix-sort Stage 3, as
// engines.py:536-549 sets them for `weft`.  The top-k steps are left to the caller
// (torch.topk in the tests, as the reference uses torch::topk).
#include <cuda_runtime.h>
#include <stdint.h>

extern "C" void launch_all_codewords_stage1(const float*, const float*, int, int, int, int*, float*, int*, cudaStream_t);
extern "C" void ragrt_stage2(const int*, const float*, const int*, const int*, const float*, int, int, int, int, int, int,
                             const int64_t*, const void*, int, const int64_t*, const uint16_t*, const int*, int, int, cudaStream_t);
extern "C" long long ragrt_stage3_sparse(const uint8_t*, int, const uint32_t*, uint32_t, long long, int, cudaStream_t,
                                         int**, float**, long long*);
extern "C" void launch_tile_maxsim_fused_decomp(const void*, const int*, const int64_t*, const int*, int, const int*,
                                                const uint8_t*, const void*, const void*, const uint8_t*, const uint8_t*,
                                                float*, cudaStream_t);
extern "C" void launch_mask_failing_candidates(const int*, int, const uint32_t*, uint32_t, float*, cudaStream_t);
extern "C" void ragrt_set_codeword_weight(float);
extern "C" void ragrt_set_compact_scores(int);
extern "C" void ragrt_set_stage3_mode(int);
extern "C" void ragrt_set_rerank_mode(int);
extern "C" void ragrt_set_drop_stats(int);
extern "C" void ragrt_reset_drop_stats();
extern "C" void ragrt_drop_stats(unsigned long long*);

// Stages 1-3 for one query.  d_out_c / d_out_v: [ntok*32, max_hits], d_out_n: [ntok*32];
// d_qpoints: [ntok*32, 3] (zeros for weft), d_codewords: [32*E, 3].
// On return *out_pids / *out_sums point at L = max(U, K) device entries (reference-owned
// buffers, valid until the next call): touched pids in ascending order then (-1, -inf).
extern "C" long long ref_weft_candidates(
    const float* d_qpoints, const float* d_codewords, int ntok, int E, int max_hits,
    int* d_out_c, float* d_out_v, int* d_out_n,
    const int* d_topc, const float* d_scores, int k_cent, int k_eids, int num_centroids,
    const int64_t* d_row_ptrs, const void* d_col_eids, int eid_bytes,
    const int64_t* d_block_sums, const uint16_t* d_lengths, const uint8_t* d_packed,
    int num_passages, const uint32_t* d_preds, uint32_t mask, long long K,
    int** out_pids, float** out_sums, long long* out_U, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    ragrt_set_codeword_weight(0.0f);
    ragrt_set_compact_scores(1);
    ragrt_set_stage3_mode(0);
    int total_rays = ntok * 32;
    launch_all_codewords_stage1(d_qpoints, d_codewords, total_rays, E, max_hits, d_out_c, d_out_v, d_out_n, s);
    ragrt_stage2(d_out_c, d_out_v, d_out_n, d_topc, d_scores, total_rays, max_hits, k_eids, k_cent, ntok,
                 num_centroids, d_row_ptrs, d_col_eids, eid_bytes, d_block_sums, d_lengths, nullptr, E, 0, s);
    return ragrt_stage3_sparse(d_packed, num_passages, d_preds, mask, K, 0, s, out_pids, out_sums, out_U);
}

// Stage 4 (tensor-core wmma kernel, the reference default) for one query.
extern "C" void ref_tile_maxsim(const void* d_Q, const int* d_pids, const int64_t* d_doc_offsets,
                                const int* d_doc_lens, int n, const int* d_codes, const uint8_t* d_residuals,
                                const void* d_centroids, const void* d_bw, const uint8_t* d_rbm,
                                const uint8_t* d_decomp, float* d_out, int wmma, void* stream) {
    ragrt_set_rerank_mode(wmma ? 1 : 0);
    launch_tile_maxsim_fused_decomp(d_Q, d_pids, d_doc_offsets, d_doc_lens, n, d_codes, d_residuals,
                                    d_centroids, d_bw, d_rbm, d_decomp, d_out, (cudaStream_t)stream);
}

extern "C" void ref_mask_failing(const int* d_pids, int n, const uint32_t* d_preds, uint32_t mask,
                                 float* d_scores, void* stream) {
    launch_mask_failing_candidates(d_pids, n, d_preds, mask, d_scores, (cudaStream_t)stream);
}

// postings counter of the last Stage 2 (the reference's diagnostic "postings" stat)
extern "C" void ref_stats(int enable, int reset, unsigned long long* out12) {
    ragrt_set_drop_stats(enable);
    if (reset) ragrt_reset_drop_stats();
    if (out12) ragrt_drop_stats(out12);
}

// device-to-device copy out of the reference-owned Stage-3 buffers (test convenience)
extern "C" int ref_copy_d2d(void* dst, const void* src, size_t bytes) {
    return (int)cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToDevice);
}
