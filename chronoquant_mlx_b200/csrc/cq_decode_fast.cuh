// cq_decode_fast.cuh -- the sm_100a split-KV decode kernel's host interface.
#pragma once
#include "cq_common.cuh"

namespace cq {

// True when the fast decode kernel handles this shape (q_len == 1,
// head_dim 128, GQA group <= 8, pages of <= 256 tokens laid out for it).
bool fast_decode_supported(const cq_paged_cache &c, int n_q_heads, int q_len);
// Chunk tokens of the fast kernel for these strides (0: the kernel does not
// take them); a cache stored in chunk blocks of this size decodes on it.
namespace fast {
int fast_chunk_tokens(int stride_k, int stride_v, int page_tokens);
}
size_t fast_decode_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req);
// Offset and size in bytes of the fast kernel's per-unit completion words in
// its workspace for this shape (size 0 when the kernel does not take it).
size_t fast_decode_done_words(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req,
                              size_t *offset);
// A decode step's new token per (sequence, kv-head): K and V inputs at
// b*sb + h*sh (unit dim stride), dtype f16/bf16, and the device length
// {tokens cached, arrival counter} the step reads and advances.
struct StepInputs {
  const void *x[2];
  int64_t sb[2], sh[2];
  int dtype;
  int64_t *len;
};

// T_dev != nullptr: the length is read from device memory at launch and T is
// the largest length the launch (grid, workspace) is sized for.  in != nullptr:
// the kernel also encodes token *in->len of every unit, attends over one more
// token and advances *in->len (T_dev is then in->len).
int run_fast_decode(const cq_paged_cache &c, const CacheView &cv, int64_t T, const void *q, int q_dtype,
                    int n_q_heads, int64_t q_sb, int64_t q_sh, float scale, void *out, int out_dtype,
                    float *lse_out, void *ws, size_t ws_bytes, int splits_req, cudaStream_t st,
                    const int64_t *T_dev = nullptr, const StepInputs *in = nullptr);

}  // namespace cq
