// s4_common.cuh -- Stage-4 declarations shared by the kernels and the C ABI.
#pragma once
#include "common.cuh"

namespace ragrt {

struct S4Docs {
    const int64_t* doc_offsets;
    const int32_t* doc_lens;
    const int32_t* codes;
    const uint8_t* residuals;
    const __half* centroids;
    const __half* bw;
    const uint8_t* rbm;
    const uint8_t* decomp;
    int N;
    int NC;           // centroid rows (codes outside [0, NC) are rejected in-kernel); INT32_MAX = unchecked
    const __half* emb = nullptr;   // raw fp16 doc-token embeddings [T, 128]: exact MaxSim, no decode
};

int s4_simt_launch(const __half* Q, const int32_t* pids, int B, int n, const S4Docs& D, float* out,
                   cudaStream_t stream);
// D.emb != nullptr: exact MaxSim over raw fp16 doc-token embeddings (sum_r max_t q_r . d_t,
// no decompression, no normalisation)
int s4_tc_launch(const __half* Q, const int32_t* pids, int B, int n, const S4Docs& D, float* out,
                 cudaStream_t stream);
int final_topk_launch(const int32_t* pids, const float* scores, int B, int n, const uint32_t* preds, int num_preds,
                      const uint32_t* masks, int k, int32_t* out_ids, float* out_scores, cudaStream_t stream);

}  // namespace ragrt
