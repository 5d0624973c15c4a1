/*
 * ragrt_b200.h -- C ABI of the B200-native (sm_100a) `weft` search path.
 *
 * Plain pointers, sizes and an opaque index handle; no C++ or torch types.  Every
 * pointer argument named d_* is a device pointer on the calling thread's current CUDA
 * device; `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Every entry point returns 0 on success or a negative RAGRT_ERR_* code, with a
 * readable message available from ragrt_last_error() (thread-local).  Nothing is
 * silently truncated: a capacity or argument problem is an error.
 *
 * Work is enqueued on `stream`; entry points do not synchronise the host except
 * ragrt_index_create (one synchronisation at the end of its validation) and
 * ragrt_index_stats.
 */
#ifndef RAGRT_B200_H
#define RAGRT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RAGRT_OK                0
#define RAGRT_ERR_ARG          -1   /* bad argument (shape, range, alignment, null pointer)  */
#define RAGRT_ERR_CUDA         -2   /* a CUDA runtime call failed                             */
#define RAGRT_ERR_CAPACITY     -3   /* a size exceeds a documented limit                      */
#define RAGRT_ERR_INDEX        -4   /* the bound arrays are not a valid plain-IVF index       */
#define RAGRT_ERR_UNSUPPORTED  -5   /* a configuration outside the weft path                  */
#define RAGRT_ERR_DEVICE       -6   /* called on a different device than the index's          */

/* Limits of this build. */
#define RAGRT_DIM              128  /* embedding dimension (fixed by the 2-bit codec)         */
#define RAGRT_QUERY_ROWS        32  /* query rows per query (Stage 4 reads all 32)            */
#define RAGRT_MAX_PROBE        128  /* nprobe (nc) per query token                            */
#define RAGRT_MAX_CANDIDATES 16384  /* ndocs (k_candidates) per query and shard               */

typedef struct ragrt_index ragrt_index;

/*
 * The arrays CorrIndex3D::bind_index takes (reference src/optix_corr_torch_3d.cpp:453-488),
 * in the plain-IVF layout of src/build_plain_ivf.py:28-68, :98-127.  The caller keeps
 * ownership; the arrays must stay alive and unchanged while the index is used.
 */
typedef struct {
    const int64_t*  csr_row_ptrs;     /* [32, num_centroids + 1]; rows 1-31 must be empty    */
    const void*     csr_col_eids;     /* [num_lists] uint8 (eid_bytes 1) or uint16 (2)        */
    int32_t         eid_bytes;
    const int64_t*  csr_block_sums;   /* [ceil(num_lists / 128)]                              */
    const uint16_t* csr_lengths;      /* [num_lists]                                          */
    const uint8_t*  csr_packed_24;    /* [3 * num_postings] little-endian 24-bit pids         */
    int64_t         num_lists;
    int64_t         num_postings;
    const int64_t*  doc_offsets;      /* [num_passages + 1]                                   */
    const int32_t*  doc_lens;         /* [num_passages]                                       */
    const int32_t*  codes;            /* [num_tokens]                                         */
    const uint8_t*  residuals;        /* [num_tokens, 32], 16-byte aligned                    */
    int64_t         num_tokens;       /* every passage's tokens lie in [0, num_tokens)        */
    const void*     centroids;        /* fp16 [num_centroids, 128], 16-byte aligned           */
    const void*     bucket_weights;   /* fp16 [4]                                             */
    const uint8_t*  reversed_bit_map; /* [256]                                                */
    const uint8_t*  decomp_table;     /* [256, 4]                                             */
    const uint32_t* doc_predicates;   /* [num_passages]; may be NULL (no filters)             */
    int32_t         num_passages;     /* N <= 2^24 (24-bit pids)                              */
    int32_t         num_centroids;    /* NC                                                   */
    int32_t         num_eids;         /* E: chunk ids enumerated per probed centroid          */
} ragrt_index_desc;

/*
 * Validates the bound arrays and builds the index's derived device structures (per
 * centroid posting ranges, per pid-range sub-list offsets, centroid norms).  Replaces
 * CorrIndex3D::bind_index (optix_corr_torch_3d.cpp:453-488).  Synchronises `stream`.
 */
int ragrt_index_create(const ragrt_index_desc* desc, ragrt_index** out, void* stream);
int ragrt_index_destroy(ragrt_index* index);

/*
 * Stage 2: centroid scores and per-token top-nprobe with missing-score imputation, for
 * B queries at once.  Replaces weft_prep.native_prep (src/weft_prep.py:32-47), which the
 * reference runs per query as a torch fp16 GEMM + topk.
 *   d_Q [B, rows, 128] fp16; d_ntok [B] int32 tokens per query (NULL = rows for all);
 *   d_C [NC, 128] fp16.
 * Selects kk = min(nc + impute, NC) centroids per token by (fp16 score desc, centroid
 * id asc); fp16 scores are the exact dot products rounded once (RNE).
 *   d_topc [B, rows, ncol] int32 and d_scores [B, rows, ncol] f32 with ncol = min(nc, kk);
 *   scores = float(v_j) - m_t when imputed (kk > nc) else float(v_j);
 *   d_m [B, rows] f32 = float(v_nc) (may be NULL);
 *   d_full16 [B, rows, NC] fp16 (may be NULL): every score (the compact=False form).
 * Rows t >= ntok get topc = -1, scores = 0, m = 0.
 */
int ragrt_centroid_topk(const void* d_Q, const int32_t* d_ntok, int32_t B, int32_t rows,
                        const void* d_C, int32_t NC, int32_t nc, int32_t impute,
                        int32_t* d_topc, float* d_scores, float* d_m, void* d_full16, void* stream);

/*
 * Stage 2 without any memory allocation.  No counterpart in the reference: it exists for
 * callers that must not allocate device memory per call.  Same arguments and bit-identical
 * outputs as ragrt_centroid_topk with d_full16 = NULL, but the scratch lives in one static
 * 32 MiB device array per device instead of cudaMallocAsync/cudaFreeAsync.
 *   - The first call on a device (with it current) looks up the array's address
 *     (cudaGetSymbolAddress; may load the module): make it before any stream capture.
 *   - A call that needs more than 32 MiB of scratch returns RAGRT_ERR_ARG.  On the
 *     tensor-core path (kk = nc + impute <= 64) the need is 4 (NC + 1) bytes of centroid
 *     norms plus, per query row, 8 x (64 S + 1) + 2 ceil(NC / 128) bytes.  S, the number of
 *     centroid slices (1 to 32), depends on the batch and the SM count: with
 *     T = ceil(NC / 128) and G = ceil(B x rows / 128),
 *     S = ceil(T / ceil(T / min(32, T, max(1, SMs / G)))).  Small batches use many slices
 *     (on 148 SMs, S = 32 up to 4 x 128 rows), batches of more than SMs / 2 x 128 rows use one.
 *     At 65,536 centroids: 8 queries x 32 rows (S = 32) 4.5 MB, 256 x 32 (S = 2) 17 MB,
 *     320 x 32 (S = 1) 16 MB; the largest one-slice batch is about 21,500 rows (670 queries
 *     of 32 rows).
 *   - All calls on a device share the array: calls that overlap on the GPU race.
 * ragrt_centroid_topk_noalloc_error reads (and with reset != 0 clears) the error word that
 * the tensor-core kernel sets when one of its bounded waits gives up (synchronous).
 */
int ragrt_centroid_topk_noalloc(const void* d_Q, const int32_t* d_ntok, int32_t B, int32_t rows,
                                const void* d_C, int32_t NC, int32_t nc, int32_t impute,
                                int32_t* d_topc, float* d_scores, float* d_m, void* stream);
int ragrt_centroid_topk_noalloc_error(int32_t reset);

/*
 * Stages 1-3 in `weft` mode for B queries: every chunk (eid < n_eids) of every probed
 * centroid whose base score is > 0, per (passage, token) the max fp16 base score, per
 * passage the sum over tokens, then candidate selection.  Replaces the all-codewords
 * Stage 1 + ragrt_stage2 + ragrt_stage3_sparse + torch::topk of CorrIndex3D::stages23
 * (optix_corr_torch_3d.cpp:558-594; ragrt_fused_kernel.cu:64-263, :343-431, :1038-1157).
 *   d_topc [B, rows, kc] int32, d_scores f32: [B, rows, kc] (full_scores = 0, compact)
 *   or [B, rows, NC] (full_scores = 1); d_ntok [B] (NULL = rows); d_masks [B] uint32
 *   filter per query (NULL = none; a passage passes if (pred & mask) != 0).
 *   K <= RAGRT_MAX_CANDIDATES candidates per query:
 *   d_cand_pids [B, K] int32 (-1 padding), d_cand_sums [B, K] f32 (-inf padding),
 *   d_num_touched [B] int64 (may be NULL): passages touched (U).
 * Order: U <= K -> ascending pid; otherwise (sum desc, pid asc).  Sums are exact sums
 * of the fp16 maxima rounded once to fp32.
 */
int ragrt_weft_candidates(ragrt_index* index, const int32_t* d_topc, const float* d_scores,
                          int32_t full_scores, const int32_t* d_ntok, int32_t B, int32_t rows,
                          int32_t kc, int32_t n_eids, const uint32_t* d_masks, int32_t K,
                          int32_t* d_cand_pids, float* d_cand_sums, int64_t* d_num_touched,
                          void* stream);

/*
 * Per centroid: postings of all its lists (d_total [NC] int64, may be NULL) and those whose
 * passage passes the filter (pred & mask) != 0 (d_pass [NC] int64; mask 0 = no filter: all).
 * The inputs of the reference's filter-aware probing: the empty-centroid set of weft_oracle and
 * pass_c / tot_c of weft_adapt (src/weft_prep.py:75-170, src/engines.py:434-526), which the
 * reference derives from its filtered index in Python.
 */
int ragrt_centroid_pass_counts(ragrt_index* index, uint32_t mask, int64_t* d_pass, int64_t* d_total, void* stream);

/*
 * Per-token probe depth under a filter: the rule of the reference's adaptive probing
 * (src/weft_prep.py:75-106, engine weft_adapt).  d_topc [ntok, width] int32 holds each token's
 * probed centroids best first; d_pass_c / d_tot_c [NC] int64 the passing / all postings per
 * centroid (ragrt_centroid_pass_counts); sel the filter's global pass rate.  For each token,
 * with target = sel x (all postings of its first nc probes), computed in fp32:
 *   d_short[t] = 1 if its first nc probes hold fewer than slack x target passing postings;
 *   d_need[t]  = 1 + the number of prefixes of its first ncap probes whose passing postings
 *                are below the target, clamped to [nc, ncap].
 * Needs 1 <= nc <= ncap <= width.
 */
int ragrt_probe_depth(const int32_t* d_topc, int32_t ntok, int32_t width, const int64_t* d_pass_c,
                      const int64_t* d_tot_c, int32_t NC, float sel, float slack, int32_t nc, int32_t ncap,
                      int32_t* d_short, int32_t* d_need, void* stream);

/*
 * Stage 4: fused 2-bit residual decompression + TileMaxSim for B queries with n
 * candidates each.  Replaces launch_tile_maxsim_fused_decomp / native_tile_maxsim_fused_decomp
 * (tile_maxsim_fused_decomp.cu:125-251, optix_corr_torch_3d.cpp:865-883).
 *   d_Q [B, 32, 128] fp16, d_pids [B, n] int32 -> d_out [B, n] f32;
 *   score = sum over the 32 query rows of the max over the passage's tokens of
 *   q . d / |d|, d = fp16 add of centroid and bucket weight.  pid < 0 or >= N -> -inf;
 *   a passage with no tokens -> 32 * -1e9.
 *   mode 1: tensor-core kernel (tcgen05; the reference's "wmma" mode);
 *   mode 0: CUDA-core kernel (the reference's "simt" mode).
 */
int ragrt_tile_maxsim(const void* d_Q, const int32_t* d_pids, int32_t B, int32_t n,
                      const int64_t* d_doc_offsets, const int32_t* d_doc_lens, int32_t num_passages,
                      const int32_t* d_codes, const uint8_t* d_residuals, const void* d_centroids,
                      const void* d_bucket_weights, const uint8_t* d_reversed_bit_map,
                      const uint8_t* d_decomp_table, float* d_out, int32_t mode, void* stream);

/*
 * Exact TileMaxSim over uncompressed fp16 doc-token embeddings (the exact-rerank workload):
 * score(pid) = sum over the 32 query rows of max over the passage's tokens of q_r . d_t, fp32
 * accumulation, no normalisation; pid < 0 or >= num_passages -> -inf, an empty passage ->
 * -3.2e10.  The reference scores 2-bit compressed tokens only
 * (tile_maxsim_fused_decomp.cu:125-229); this is the same pipeline without the decode.
 *   d_Q [B, 32, 128] fp16; d_pids [B, n]; d_doc_emb [T, 128] fp16 (16-byte aligned);
 *   d_out [B, n] f32.
 */
int ragrt_tile_maxsim_exact(const void* d_Q, const int32_t* d_pids, int32_t B, int32_t n,
                            const int64_t* d_doc_offsets, const int32_t* d_doc_lens, int32_t num_passages,
                            const void* d_doc_emb, float* d_out, void* stream);

/*
 * Final filter + top-k per query: a candidate whose pid is < 0 or fails the query's mask
 * scores -inf (ragrt_fused_kernel.cu:621-640), then the k best by (score desc, pid asc)
 * (optix_corr_torch_3d.cpp:603-606).  d_preds [num_preds] may be NULL (no filters); a
 * pid >= num_preds scores -inf when predicates are given.
 *   d_pids/d_scores [B, n]; k <= n -> d_out_ids [B, k] int32, d_out_scores [B, k] f32
 *   (may be NULL).
 */
/*
 * Stage 4 over a bound index: the fused decompress + TileMaxSim of ragrt_tile_maxsim for
 * d_pids [B, n] into d_out [B, n] f32, with the index's arrays (tile_maxsim_fused_decomp.cu:
 * 125-229).  mode 1: the tensor-core kernel the batched search runs; mode 0: the CUDA-core
 * kernel.
 */
int ragrt_index_tile_maxsim(ragrt_index* index, const void* d_Q, const int32_t* d_pids, int32_t B, int32_t n,
                            float* d_out, int32_t mode, void* stream);

int ragrt_final_topk(const int32_t* d_pids, const float* d_scores, int32_t B, int32_t n,
                     const uint32_t* d_preds, int32_t num_preds, const uint32_t* d_masks, int32_t k,
                     int32_t* d_out_ids, float* d_out_scores, void* stream);

/*
 * The whole `weft` search for a batch: Stage 2 -> Stages 1-3 -> Stage 4 -> final top-k,
 * with no host synchronisation.  The batched entry the reference lacks (it loops over
 * queries in CorrIndex3D::search_batch_pipelined, optix_corr_torch_3d.cpp:667-723).
 *   d_Q [B, 32, 128] fp16, d_ntok [B] (NULL = 32), d_masks [B] (NULL = none),
 *   nc probes per token, K candidates, k_top results, rerank_mode as ragrt_tile_maxsim.
 *   d_out_ids [B, k_top] int32 (-1 padding), d_out_scores [B, k_top] f32 (may be NULL).
 */
int ragrt_weft_search(ragrt_index* index, const void* d_Q, const int32_t* d_ntok, int32_t B,
                      int32_t nc, int32_t n_eids, const uint32_t* d_masks, int32_t K, int32_t k_top,
                      int32_t rerank_mode, int32_t* d_out_ids, float* d_out_scores, void* stream);

/*
 * ragrt_weft_search with stage timing: records events[0..4] (cudaEvent_t, created by the
 * caller; NULL entries skipped) on `stream` before Stage 2, after Stage 2, after Stages 1-3,
 * after Stage 4 and after the final top-k.  The counterpart of the reference's
 * CorrIndex3D::search_single_query_profiled (optix_corr_torch_3d.cpp:638-665), without
 * its host synchronisation.
 */
int ragrt_weft_search_profiled(ragrt_index* index, const void* d_Q, const int32_t* d_ntok, int32_t B,
                               int32_t nc, int32_t n_eids, const uint32_t* d_masks, int32_t K, int32_t k_top,
                               int32_t rerank_mode, int32_t* d_out_ids, float* d_out_scores,
                               void* const* events, void* stream);

/*
 * Counters accumulated over calls since the last reset (the reference's drop stats,
 * ragrt_fused_kernel.cu:33-47, :884-899): out[0] queries, out[1] postings scanned
 * (sum over kept (token, probe) pairs of list length: the reference's ST_POSTINGS),
 * out[2] distinct postings read (each probed list once per query: what Stage 3 walks),
 * out[3] passages touched, out[4] kept probes, out[5] candidates reranked, out[6] tasks
 * (sum over kept probes of their chunk lists below n_eids: the reference's ST_TASKS),
 * out[7] pid-range blocks that Stage 3 found too dense for its walk-once table and handed
 * to the per-token kernel (no reference counterpart).  Synchronises the device.
 * ragrt_index_count_distinct is kept for compatibility: every counter is always counted (the
 * distinct lists are a by-product of Stage 3).
 */
int ragrt_index_count_distinct(ragrt_index* index, int32_t enable);

/*
 * Stage-3 algorithm of an index (the reference's set_stage3_mode, optix_corr_torch_3d.cpp:941-943,
 * selects among its sort- and hash-based Stage 3 the same way): 0 (default) walks every distinct
 * probed list of a query once per pid range and hands ranges too dense for its per-passage
 * table to the per-token kernel; 1 runs the per-token kernel on every range.  Both give
 * bit-identical candidates.  range_passages sets the walk's pid-range width (rounded down to a
 * multiple of the index's range-offset granularity, at least one granule); 0 chooses it.
 */
int ragrt_index_set_stage3_mode(ragrt_index* index, int32_t mode, int32_t range_passages);
#define RAGRT_NUM_STATS 8
int ragrt_index_stats(ragrt_index* index, uint64_t* out, int32_t reset);

/* Message of the last failing call on this thread ("" if none). */
const char* ragrt_last_error(void);

/*
 * Device-side failure status of the current device since the last reset: 0 none, 1 a kernel
 * gave up a bounded wait (a tensor-core pipeline stage that never completed), 2 a code
 * outside [0, num_centroids) was met (the centroid row was not read), 3 the self-test below,
 * 4 a token id outside the vocabulary (ragrt_enc_embed);
 * <0 on error.  Synchronises with the device's error flag.  reset != 0 clears it.
 */
int ragrt_device_error(int32_t reset);

/* Number of kernels this library has launched in the process (all entry points). */
uint64_t ragrt_launch_count(void);

/*
 * Test hook, no counterpart in the reference: launches one warp that waits on an mbarrier
 * nothing arrives on, with the same bounded wait the pipelined kernels use (polls with a
 * suspend-time hint, a poll limit, a 2 s global-time deadline and an abort flag shared by the
 * waiting threads), so that the wait gives up after `polls` polls and sets the device error flag
 * to 3 (read it with ragrt_device_error).  The CUDA context stays usable.
 */
int ragrt_selftest_wait_timeout(uint32_t polls, void* stream);

/*
 * Merge of the per-shard top-k lists of a doc-sharded search (one process per GPU, corpus split
 * by pid range): d_gathered [world][2][B][k] 32-bit words holds, rank-major as an all-gather
 * leaves them, every rank's scores (f32 bit patterns) and global pids (int32; -1 = padding).  Writes
 * per query the top k_top by (score desc, pid asc), padding after every real pid of equal score:
 * d_out_ids [B, k_top] int64 (-1 padding), d_out_scores [B, k_top] f32.  No reference
 * counterpart (the reference searches one GPU).
 */
int ragrt_merge_topk(const void* d_gathered, int32_t world, int32_t B, int32_t k, int32_t k_top,
                     int64_t* d_out_ids, float* d_out_scores, void* stream);

/* ------------------------------------------------------------------------------------ *
 * Stage 0a: the ColBERT query encoder (BERT-base over [B, 32] query tokens, then ColBERT's
 * linear 768 -> 128 and L2 normalisation).  Replaces the reference's flat forward
 * (src/fast_encoder.py:57-77: embeddings + LayerNorm, 12 x [self-attention, LayerNorm, GELU
 * MLP, LayerNorm], linear, normalize), one kernel per operation; ragrt_b200/encoder.py
 * strings them together and captures them in a CUDA graph.  All matrices fp16 row-major.
 * ------------------------------------------------------------------------------------ */

/*
 * d_out[M, N] = epilogue(d_A[M, K] . d_W[N, K]^T) on the tensor cores, fp32 accumulation.
 * The nn.Linear products of the reference (F.linear(x, w, b), fast_encoder.py:70-76).
 *   epilogue 0: + d_bias[N]                 (Q, K, V projection)
 *   epilogue 1: gelu(+ d_bias), erf form    (intermediate dense, hidden_act "gelu")
 *   epilogue 2: gelu(+ d_bias), tanh form   (hidden_act "gelu_new")
 *   epilogue 3: + d_bias + d_residual[M, N] (attention output / output dense + residual)
 *   epilogue 4: fp16 rounding, then each row divided by its L2 norm (ColBERT linear + F.normalize,
 *               no bias; N must be 128)
 * N a multiple of 128, K a multiple of 64, all pointers 16-byte aligned; d_bias may be NULL.
 * d_ws (ws_bytes, may be NULL / 0): scratch for small M, where the product is split along K
 * over more CTAs and summed in fp32 by a second kernel (up to 148 x M x N x 4 bytes are used;
 * fewer splits when the workspace is smaller).
 */
int ragrt_enc_gemm(const void* d_A, const void* d_W, const void* d_bias, const void* d_residual, void* d_out,
                   int32_t M, int32_t N, int32_t K, int32_t epilogue, void* d_ws, int64_t ws_bytes, void* stream);

/*
 * d_out = LayerNorm(d_A . d_W^T + d_bias + d_residual) with d_gamma / d_beta, N = 768: the
 * attention-output and output-dense blocks (fast_encoder.py:73, :76).  When the product is
 * split along K (small M, workspace d_ws as for ragrt_enc_gemm) the partial sums are reduced
 * straight into the LayerNorm; otherwise the product goes through d_tmp [M, N] and the
 * LayerNorm kernel.  d_out may be d_residual.
 */
int ragrt_enc_gemm_residual_ln(const void* d_A, const void* d_W, const void* d_bias, const void* d_residual,
                               const void* d_gamma, const void* d_beta, float eps, void* d_tmp, void* d_out,
                               int32_t M, int32_t N, int32_t K, void* d_ws, int64_t ws_bytes, void* stream);

/* LayerNorm of d_x[rows, dim] (fp32 statistics) with d_gamma / d_beta [dim]; dim 768. */
int ragrt_enc_layernorm(const void* d_x, const void* d_gamma, const void* d_beta, float eps, void* d_out,
                        int32_t rows, int32_t dim, void* stream);

/*
 * d_out[B*L, dim] = LayerNorm(word[d_ids] + pos[0..L) + type) (fast_encoder.py:60-63); ids
 * outside [0, vocab) read row 0 and set the device error flag to 4.  dim 768.
 */
int ragrt_enc_embed(const int64_t* d_ids, const void* d_word, const void* d_pos, const void* d_type,
                    const void* d_gamma, const void* d_beta, float eps, int32_t vocab, int32_t B, int32_t L,
                    int32_t dim, void* d_out, void* stream);

/*
 * Multi-head self-attention of each query's L = 32 tokens: d_qkv[B*L, 3*dim] holds Q, K, V in
 * column blocks of dim, heads of 64 columns; keys with d_mask[b, j] == 0 are not attended
 * (the reference's additive finfo.min bias); softmax(q k^T / 8) v -> d_ctx[B*L, dim]
 * (F.scaled_dot_product_attention, fast_encoder.py:71-72).
 */
int ragrt_enc_attention(const void* d_qkv, const int64_t* d_mask, void* d_ctx, int32_t B, int32_t L, int32_t heads,
                        int32_t dim, void* stream);

/* Library version string. */
const char* ragrt_version(void);

#ifdef __cplusplus
}
#endif
#endif /* RAGRT_B200_H */
