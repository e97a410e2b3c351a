// cq_prefill.cuh -- host entry points of the tensor-core query-chunk path (cq_prefill.cu).
#pragma once

#include "cq_common.cuh"

namespace cq {

// head_dim 128, at least 16 query tokens, GQA group a power of two <= 16
bool prefill_supported(const cq_paged_cache &c, int n_q_heads, int q_len);
// workspace bytes (0 when unsupported): K and V^T tile images of every key, query tile images
size_t prefill_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len);
int run_prefill(const cq_paged_cache &cache, const CacheView &cv, int64_t T, const void *q, int q_dtype, int Hq,
                int q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, void *out, int out_dtype,
                float *lse_out, void *ws, size_t ws_bytes, bool causal, cudaStream_t st);
// the two halves of run_prefill: tile images of the history and the queries, then the attention
int prefill_prepare(const cq_paged_cache &cache, const CacheView &cv, int64_t T, const void *q, int q_dtype, int Hq,
                    int q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, void *ws, size_t ws_bytes,
                    cudaStream_t st);
int prefill_attend(const cq_paged_cache &cache, int64_t T, int Hq, int q_len, bool causal, void *out, int out_dtype,
                   float *lse_out, void *ws, size_t ws_bytes, cudaStream_t st);
int read_prefill_error(int clear);
// merge of split-KV partials (m natural-log, l, unnormalised o; [row][split]) into out and lse (cq_attention.cu)
int launch_split_combine(const float *ws_m, const float *ws_l, const float *ws_o, int64_t rows, int splits, int D,
                         void *out, int out_dtype, float *lse_out, cudaStream_t st);

}  // namespace cq
