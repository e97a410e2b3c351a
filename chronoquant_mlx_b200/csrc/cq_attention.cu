// cq_attention.cu -- attention over the compressed cache: dispatch, the
// general split-KV kernel, the split combine and the sequence-shard merge.
//
// Semantics follow attention.py:23-74: scores = (q*scale rounded to the query
// dtype) . k, softmax over the keys (causal, end-aligned when q_len > 1,
// attention.py:8-20), output = softmax . v.  K and V are decoded as the fused
// Metal kernel does (kernels.py:152-155, 173-176): fp32 anchor + code*scale.
//
// The general kernel handles every supported shape (head_dim <= 256, any
// GQA ratio, any q_len, the reference layout); the sm_100a fast decode kernel
// (cq_decode_fast.cu) takes the common shapes.
#include <algorithm>
#include <cmath>

#include "cq_common.cuh"
#include "cq_decode_fast.cuh"
#include "cq_prefill.cuh"

namespace cq {

constexpr int kGenWarps = 4;
constexpr int kMaxSlots = 8;  // head_dim <= 256 -> 8 dims per lane

struct AttnArgs {
  CacheView cv;
  const void *q;
  int q_dtype;
  int Hq, q_len, splits;
  int64_t q_sb, q_sh, q_sq;
  float scale;
  int64_t T;
  int64_t chunk;  // tokens per split
  float *ws_m, *ws_l, *ws_o;
  // optional explicit mask [B?][H?][q_len][T] (element strides; 0 broadcasts)
  const void *mask;
  int mask_kind;  // 0 none, 1 boolean (uint8, nonzero = keep), 2 additive
  int mask_dtype; // additive mask element type (CQ_F16/CQ_BF16/CQ_F32)
  int64_t m_sb, m_sh, m_sq, m_st;
  float masked_score;  // finfo(score dtype).min, as attention.py:19
  int causal;          // end-aligned causal rule when q_len > 1 and no explicit mask
};

__device__ __forceinline__ float decode_val(const TokLoc &L, int d, int D, int order) {
  float a = __half2float(L.anchor[d]);
  if (!L.codes) return a;
  int nib = nibble_at(L.codes, d, D, order);
  return fmaf((float)(nib - 8), L.scale, a);
}

__global__ void __launch_bounds__(kGenWarps * 32) attn_generic_kernel(AttnArgs A) {
  __shared__ float s_m[kGenWarps], s_l[kGenWarps];
  __shared__ float s_o[kGenWarps][256];
  const CacheView &cv = A.cv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t blk = blockIdx.x;
  const int sp = (int)(blk % A.splits);
  const int64_t row = blk / A.splits;  // (b, hq, qi)
  const int qi = (int)(row % A.q_len);
  const int hq = (int)((row / A.q_len) % A.Hq);
  const int b = (int)(row / ((int64_t)A.q_len * A.Hq));
  const int D = cv.D;
  const int kvh = hq / (A.Hq / cv.H);

  const int64_t t_lim = (A.q_len > 1 && A.causal && A.mask_kind == 0) ? (A.T - A.q_len + qi + 1) : A.T;
  const int64_t start = (int64_t)sp * A.chunk;
  const int64_t end = min(t_lim, start + A.chunk);

  // q*scale in the query dtype (attention.py:46, 65), then fp32
  float qv[kMaxSlots];
  const float sc = (A.q_dtype == CQ_F32) ? A.scale : round_dt(A.scale, A.q_dtype);
  const int64_t qbase = b * A.q_sb + hq * A.q_sh + qi * A.q_sq;
#pragma unroll
  for (int i = 0; i < kMaxSlots; ++i) {
    int d = lane + 32 * i;
    float v = 0.f;
    if (d < D) {
      v = load_as_float(A.q, qbase + d, A.q_dtype) * sc;
      if (A.q_dtype != CQ_F32) v = round_dt(v, A.q_dtype);
    }
    qv[i] = v;
  }

  float m = -INFINITY, l = 0.f, acc[kMaxSlots];
#pragma unroll
  for (int i = 0; i < kMaxSlots; ++i) acc[i] = 0.f;

  for (int64_t t = start + warp; t < end; t += kGenWarps) {
    TokLoc Lk = locate(cv, 0, b, kvh, t);
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxSlots; ++i) {
      int d = lane + 32 * i;
      if (d < D) part = fmaf(qv[i], decode_val(Lk, d, D, cv.c[0].order), part);
    }
    float s = warp_sum(part);
    if (A.mask_kind) {
      const int64_t mi = b * A.m_sb + hq * A.m_sh + qi * A.m_sq + t * A.m_st;
      if (A.mask_kind == 1)
        s = ((const uint8_t *)A.mask)[mi] ? s : A.masked_score;
      else
        s += load_as_float(A.mask, mi, A.mask_dtype);
    }
    float mn = fmaxf(m, s);
    float f = expf(m - mn);
    float p = expf(s - mn);
    m = mn;
    l = l * f + p;
    TokLoc Lv = locate(cv, 1, b, kvh, t);
#pragma unroll
    for (int i = 0; i < kMaxSlots; ++i) {
      int d = lane + 32 * i;
      if (d < D) acc[i] = fmaf(p, decode_val(Lv, d, D, cv.c[1].order), acc[i] * f);
    }
  }

  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < kMaxSlots; ++i) {
    int d = lane + 32 * i;
    if (d < D) s_o[warp][d] = acc[i];
  }
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY;
    for (int w = 0; w < kGenWarps; ++w) M = fmaxf(M, s_m[w]);
    float L = 0.f, fw[kGenWarps];
    for (int w = 0; w < kGenWarps; ++w) {
      fw[w] = (s_m[w] == -INFINITY) ? 0.f : expf(s_m[w] - M);
      L += s_l[w] * fw[w];
    }
    const int64_t o = row * A.splits + sp;
    if (lane == 0) {
      A.ws_m[o] = M;
      A.ws_l[o] = L;
    }
    for (int d = lane; d < D; d += 32) {
      float v = 0.f;
      for (int w = 0; w < kGenWarps; ++w) v += s_o[w][d] * fw[w];
      A.ws_o[o * D + d] = v;
    }
  }
}

// Combine the split partials of each row: one warp per row.
__global__ void combine_kernel(const float *ws_m, const float *ws_l, const float *ws_o, int64_t rows, int splits,
                               int D, void *out, int out_dtype, float *lse_out) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *m = ws_m + row * splits;
  const float *l = ws_l + row * splits;
  if (D == 128 && splits <= 8 && ((uintptr_t)ws_o & 15) == 0) {
    // one float4 of head dims per lane: weights exp(m_s - M) once per row, 16-byte loads
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, m[s]);
    float w[8], L = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      w[s] = (s < splits && m[s] != -INFINITY) ? expf(m[s] - M) : 0.f;
      if (s < splits) L += l[s] * w[s];
    }
    const float inv = (L > 0.f) ? 1.f / L : 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      if (s < splits && w[s] != 0.f) {
        const float4 o = reinterpret_cast<const float4 *>(ws_o + (row * splits + s) * 128)[lane];
        acc.x += o.x * w[s];
        acc.y += o.y * w[s];
        acc.z += o.z * w[s];
        acc.w += o.w * w[s];
      }
    }
    const int64_t base = row * 128 + lane * 4;
    store_from_float(out, base, acc.x * inv, out_dtype);
    store_from_float(out, base + 1, acc.y * inv, out_dtype);
    store_from_float(out, base + 2, acc.z * inv, out_dtype);
    store_from_float(out, base + 3, acc.w * inv, out_dtype);
    if (lse_out && lane == 0) lse_out[row] = (L > 0.f) ? M + logf(L) : -INFINITY;
    return;
  }
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, m[s]);
  float L = 0.f;
  for (int s = 0; s < splits; ++s)
    if (m[s] != -INFINITY) L += l[s] * expf(m[s] - M);
  const float inv = (L > 0.f) ? 1.f / L : 0.f;
  for (int d = lane; d < D; d += 32) {
    float v = 0.f;
    for (int s = 0; s < splits; ++s)
      if (m[s] != -INFINITY) v += ws_o[(row * splits + s) * D + d] * expf(m[s] - M);
    store_from_float(out, row * D + d, v * inv, out_dtype);
  }
  if (lse_out && lane == 0) lse_out[row] = (L > 0.f) ? M + logf(L) : -INFINITY;
}

// out[r] = sum_i exp(lse_i - L) o_i over sequence shards (one warp per row).
// Part i's log-sum-exp of row r at lse[i * lse_ps + r], its output at
// o[i * o_ps + r * D + d] (separate arrays, or one packed buffer per part).
__global__ void lse_merge_kernel(const float *lse, const float *o, int n_parts, int64_t rows, int D, int64_t lse_ps,
                                 int64_t o_ps, void *out, int out_dtype) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int i = 0; i < n_parts; ++i) M = fmaxf(M, lse[(int64_t)i * lse_ps + row]);
  float W = 0.f;
  for (int i = 0; i < n_parts; ++i) {
    float x = lse[(int64_t)i * lse_ps + row];
    if (x != -INFINITY) W += expf(x - M);
  }
  const float inv = (W > 0.f) ? 1.f / W : 0.f;
  for (int d = lane; d < D; d += 32) {
    float v = 0.f;
    for (int i = 0; i < n_parts; ++i) {
      float x = lse[(int64_t)i * lse_ps + row];
      if (x != -INFINITY) v += expf(x - M) * o[(int64_t)i * o_ps + row * D + d];
    }
    store_from_float(out, row * D + d, v * inv, out_dtype);
  }
}

static int pick_splits(int64_t rows, int64_t T, int requested) {
  if (requested > 0) return (int)std::min<int64_t>(requested, std::max<int64_t>(T, 1));
  int64_t want = (2 * 148 * 4 + rows - 1) / rows;
  int64_t max_by_len = std::max<int64_t>(1, T / 64);
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, std::min<int64_t>(max_by_len, 256)));
}

size_t generic_workspace(int64_t rows, int splits, int D) {
  return (size_t)rows * splits * (2 + D) * sizeof(float);
}

struct MaskSpec {
  const void *ptr = nullptr;
  int kind = 0, dtype = CQ_F32;
  int64_t sb = 0, sh = 0, sq = 0, st = 0;
};

int run_generic(const CacheView &cv, int64_t T, const void *q, int q_dtype, int Hq, int q_len, int64_t q_sb,
                int64_t q_sh, int64_t q_sq, float scale, void *out, int out_dtype, float *lse_out, void *ws,
                size_t ws_bytes, int splits_req, cudaStream_t st, const MaskSpec &mk = MaskSpec(),
                bool causal = true) {
  const int64_t rows = (int64_t)cv.B * Hq * q_len;
  const int splits = pick_splits(rows, T, splits_req);
  const size_t need = generic_workspace(rows, splits, cv.D);
  CQ_REQUIRE(ws && ws_bytes >= need, CQ_ERR_WORKSPACE, "cq_attention: workspace too small");
  AttnArgs A;
  A.cv = cv;
  A.q = q;
  A.q_dtype = q_dtype;
  A.Hq = Hq;
  A.q_len = q_len;
  A.splits = splits;
  A.q_sb = q_sb;
  A.q_sh = q_sh;
  A.q_sq = q_sq;
  A.scale = scale;
  A.T = T;
  A.chunk = (T + splits - 1) / splits;
  A.ws_m = (float *)ws;
  A.ws_l = A.ws_m + rows * splits;
  A.ws_o = A.ws_l + rows * splits;
  A.mask = mk.ptr;
  A.mask_kind = mk.kind;
  A.causal = causal ? 1 : 0;
  A.mask_dtype = mk.dtype;
  A.m_sb = mk.sb;
  A.m_sh = mk.sh;
  A.m_sq = mk.sq;
  A.m_st = mk.st;
  // scores are fp16 for fp16 queries (fp16 @ fp16), fp32 for bf16 (bf16 @ fp16 promotes)
  A.masked_score = (q_dtype == CQ_F16) ? -65504.0f : -3.4028234663852886e38f;
  int64_t blocks = rows * splits;
  CQ_REQUIRE(blocks < (1LL << 31), CQ_ERR_INVALID, "cq_attention: grid too large");
  attn_generic_kernel<<<(unsigned)blocks, kGenWarps * 32, 0, st>>>(A);
  int r = check_launch("attn_generic_kernel");
  if (r) return r;
  int64_t cblocks = (rows * 32 + 255) / 256;
  combine_kernel<<<(unsigned)cblocks, 256, 0, st>>>(A.ws_m, A.ws_l, A.ws_o, rows, splits, cv.D, out, out_dtype,
                                                     lse_out);
  return check_launch("combine_kernel");
}

int launch_split_combine(const float *ws_m, const float *ws_l, const float *ws_o, int64_t rows, int splits, int D,
                         void *out, int out_dtype, float *lse_out, cudaStream_t st) {
  const int64_t cblocks = (rows * 32 + 255) / 256;
  combine_kernel<<<(unsigned)cblocks, 256, 0, st>>>(ws_m, ws_l, ws_o, rows, splits, D, out, out_dtype, lse_out);
  return check_launch("combine_kernel");
}

int read_bounds_error_attention(int clear) { return read_bounds_error_here(clear); }

}  // namespace cq

using namespace cq;

static int attention_common_checks(const cq_paged_cache *cache, int64_t T, int32_t n_q_heads, int32_t q_len) {
  int r = validate_cache(cache);
  if (r) return r;
  CQ_REQUIRE(T >= 1, CQ_ERR_INVALID, "cq_attention: T must be >= 1 (empty cache)");
  CQ_REQUIRE(n_q_heads >= 1 && n_q_heads % cache->kv_heads == 0, CQ_ERR_INVALID,
             "cq_attention: n_q_heads must be a positive multiple of kv_heads");
  CQ_REQUIRE(q_len >= 1 && q_len <= T, CQ_ERR_INVALID, "cq_attention: need 1 <= q_len <= T");
  CQ_REQUIRE((T + cache->page_tokens - 1) / cache->page_tokens <= cache->max_pages, CQ_ERR_INVALID,
             "cq_attention: T beyond mapped pages");
  return CQ_OK;
}

extern "C" int cq_attention_workspace(const cq_paged_cache *cache, int64_t T, int32_t n_q_heads, int32_t q_len,
                                      int32_t num_splits, size_t *bytes) {
  int r = attention_common_checks(cache, T, n_q_heads, q_len);
  if (r) return r;
  CQ_REQUIRE(bytes, CQ_ERR_INVALID, "cq_attention_workspace: bytes is null");
  const int64_t rows = (int64_t)cache->batch * n_q_heads * q_len;
  size_t need = generic_workspace(rows, pick_splits(rows, T, num_splits), cache->head_dim);
  size_t fast = fast_decode_workspace(*cache, T, n_q_heads, q_len, num_splits);
  size_t chunk = prefill_workspace(*cache, T, n_q_heads, q_len);
  *bytes = std::max(need, std::max(fast, chunk));
  return CQ_OK;
}

extern "C" int cq_prefill_prepare(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype,
                                  int32_t n_q_heads, int32_t q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq,
                                  float scale, void *workspace, size_t workspace_bytes, void *stream) {
  int r = attention_common_checks(cache, T, n_q_heads, q_len);
  if (r) return r;
  CQ_REQUIRE(q, CQ_ERR_INVALID, "cq_prefill_prepare: q null");
  CQ_REQUIRE(q_dtype == CQ_F16 || q_dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_prefill_prepare: q dtype must be f16/bf16");
  return prefill_prepare(*cache, make_view(*cache), T, q, q_dtype, n_q_heads, q_len, q_sb, q_sh, q_sq, scale,
                         workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int cq_prefill_attend(const cq_paged_cache *cache, int64_t T, int32_t n_q_heads, int32_t q_len,
                                 int32_t causal, void *out, int out_dtype, float *lse_out, void *workspace,
                                 size_t workspace_bytes, void *stream) {
  int r = attention_common_checks(cache, T, n_q_heads, q_len);
  if (r) return r;
  CQ_REQUIRE(out, CQ_ERR_INVALID, "cq_prefill_attend: out null");
  CQ_REQUIRE(out_dtype == CQ_F16 || out_dtype == CQ_BF16 || out_dtype == CQ_F32, CQ_ERR_UNSUPPORTED,
             "cq_prefill_attend: bad out dtype");
  return prefill_attend(*cache, T, n_q_heads, q_len, causal != 0, out, out_dtype, lse_out, workspace, workspace_bytes,
                        (cudaStream_t)stream);
}

extern "C" int cq_attention(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype, int32_t n_q_heads,
                            int32_t q_len, int32_t causal, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, void *out,
                            int out_dtype, float *lse_out, void *workspace, size_t workspace_bytes,
                            int32_t num_splits, void *stream) {
  int r = attention_common_checks(cache, T, n_q_heads, q_len);
  if (r) return r;
  CQ_REQUIRE(q && out, CQ_ERR_INVALID, "cq_attention: q/out null");
  CQ_REQUIRE(q_dtype == CQ_F16 || q_dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_attention: q dtype must be f16/bf16");
  CQ_REQUIRE(out_dtype == CQ_F16 || out_dtype == CQ_BF16 || out_dtype == CQ_F32, CQ_ERR_UNSUPPORTED,
             "cq_attention: bad out dtype");
  CacheView cv = make_view(*cache);
  cudaStream_t st = (cudaStream_t)stream;
  if (fast_decode_supported(*cache, n_q_heads, q_len))
    return run_fast_decode(*cache, cv, T, q, q_dtype, n_q_heads, q_sb, q_sh, scale, out, out_dtype, lse_out,
                           workspace, workspace_bytes, num_splits, st);
  if (prefill_supported(*cache, n_q_heads, q_len))
    return run_prefill(*cache, cv, T, q, q_dtype, n_q_heads, q_len, q_sb, q_sh, q_sq, scale, out, out_dtype, lse_out,
                       workspace, workspace_bytes, causal != 0, st);
  return run_generic(cv, T, q, q_dtype, n_q_heads, q_len, q_sb, q_sh, q_sq, scale, out, out_dtype, lse_out,
                     workspace, workspace_bytes, num_splits, st, MaskSpec(), causal != 0);
}

extern "C" int cq_attention_at(const cq_paged_cache *cache, const int64_t *len_dev, int64_t max_len, const void *q,
                               int q_dtype, int32_t n_q_heads, int64_t q_sb, int64_t q_sh, float scale, void *out,
                               int out_dtype, float *lse_out, void *workspace, size_t workspace_bytes, void *stream) {
  int r = attention_common_checks(cache, max_len, n_q_heads, 1);
  if (r) return r;
  CQ_REQUIRE(len_dev && q && out, CQ_ERR_INVALID, "cq_attention_at: null pointer");
  CQ_REQUIRE(q_dtype == CQ_F16 || q_dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_attention_at: q dtype must be f16/bf16");
  CQ_REQUIRE(out_dtype == CQ_F16 || out_dtype == CQ_BF16 || out_dtype == CQ_F32, CQ_ERR_UNSUPPORTED,
             "cq_attention_at: bad out dtype");
  CQ_REQUIRE(fast_decode_supported(*cache, n_q_heads, 1), CQ_ERR_UNSUPPORTED,
             "cq_attention_at: this cache layout or shape does not take the sm_100a decode kernel");
  return run_fast_decode(*cache, make_view(*cache), max_len, q, q_dtype, n_q_heads, q_sb, q_sh, scale, out,
                         out_dtype, lse_out, workspace, workspace_bytes, 0, (cudaStream_t)stream, len_dev);
}

extern "C" int cq_decode_step_at(const cq_paged_cache *cache, const void *keys, int64_t k_sb, int64_t k_sh,
                                 const void *values, int64_t v_sb, int64_t v_sh, int kv_dtype, int64_t *len_dev,
                                 int64_t max_len, const void *q, int q_dtype, int32_t n_q_heads, int64_t q_sb,
                                 int64_t q_sh, float scale, void *out, int out_dtype, float *lse_out, void *workspace,
                                 size_t workspace_bytes, void *stream) {
  int r = attention_common_checks(cache, max_len, n_q_heads, 1);
  if (r) return r;
  CQ_REQUIRE(keys && values && len_dev && q && out, CQ_ERR_INVALID, "cq_decode_step_at: null pointer");
  CQ_REQUIRE(kv_dtype == CQ_F16 || kv_dtype == CQ_BF16, CQ_ERR_UNSUPPORTED,
             "cq_decode_step_at: key/value dtype must be f16/bf16");
  CQ_REQUIRE(q_dtype == CQ_F16 || q_dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_decode_step_at: q dtype must be f16/bf16");
  CQ_REQUIRE(out_dtype == CQ_F16 || out_dtype == CQ_BF16 || out_dtype == CQ_F32, CQ_ERR_UNSUPPORTED,
             "cq_decode_step_at: bad out dtype");
  CQ_REQUIRE(fast_decode_supported(*cache, n_q_heads, 1), CQ_ERR_UNSUPPORTED,
             "cq_decode_step_at: this cache layout or shape does not take the sm_100a decode kernel");
  StepInputs in;
  in.x[0] = keys;
  in.x[1] = values;
  in.sb[0] = k_sb;
  in.sh[0] = k_sh;
  in.sb[1] = v_sb;
  in.sh[1] = v_sh;
  in.dtype = kv_dtype;
  in.len = len_dev;
  return run_fast_decode(*cache, make_view(*cache), max_len, q, q_dtype, n_q_heads, q_sb, q_sh, scale, out,
                         out_dtype, lse_out, workspace, workspace_bytes, 0, (cudaStream_t)stream, nullptr, &in);
}

extern "C" int cq_lse_merge(const float *lse, const float *o, int32_t n_parts, int64_t rows, int32_t dim, void *out,
                            int out_dtype, void *stream) {
  CQ_REQUIRE(lse && o && out, CQ_ERR_INVALID, "cq_lse_merge: null pointer");
  CQ_REQUIRE(n_parts >= 1 && rows >= 0 && dim >= 1, CQ_ERR_INVALID, "cq_lse_merge: bad sizes");
  CQ_REQUIRE(out_dtype == CQ_F16 || out_dtype == CQ_BF16 || out_dtype == CQ_F32, CQ_ERR_UNSUPPORTED,
             "cq_lse_merge: bad out dtype");
  if (rows == 0) return CQ_OK;
  int64_t blocks = (rows * 32 + 255) / 256;
  lse_merge_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(lse, o, n_parts, rows, dim, rows, rows * dim,
                                                                       out, out_dtype);
  return check_launch("lse_merge_kernel");
}

extern "C" int cq_lse_merge_packed(const float *parts, int32_t n_parts, int64_t rows, int32_t dim, void *out,
                                   int out_dtype, void *stream) {
  CQ_REQUIRE(parts && out, CQ_ERR_INVALID, "cq_lse_merge_packed: null pointer");
  CQ_REQUIRE(n_parts >= 1 && rows >= 0 && dim >= 1, CQ_ERR_INVALID, "cq_lse_merge_packed: bad sizes");
  CQ_REQUIRE(out_dtype == CQ_F16 || out_dtype == CQ_BF16 || out_dtype == CQ_F32, CQ_ERR_UNSUPPORTED,
             "cq_lse_merge_packed: bad out dtype");
  if (rows == 0) return CQ_OK;
  const int64_t ps = rows * ((int64_t)dim + 1);  // floats per part: [rows][dim] outputs, then [rows] lse
  int64_t blocks = (rows * 32 + 255) / 256;
  lse_merge_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(parts + rows * dim, parts, n_parts, rows, dim,
                                                                       ps, ps, out, out_dtype);
  return check_launch("lse_merge_kernel");
}

extern "C" int cq_sdpa_reference_layout(const float *q, int32_t n_q_heads, int32_t dim, const void *kf_k,
                                        int32_t n_kf_k, const uint32_t *packed_k, const void *scales_k,
                                        int32_t n_pf_k, const void *kf_v, int32_t n_kf_v, const uint32_t *packed_v,
                                        const void *scales_v, int32_t n_pf_v, int32_t n_kv_heads, int64_t seq_len,
                                        int32_t stride_k, int32_t stride_v, float *out, void *workspace,
                                        size_t workspace_bytes, void *stream) {
  CQ_REQUIRE(q && kf_k && kf_v && out, CQ_ERR_INVALID, "cq_sdpa_reference_layout: null pointer");
  CQ_REQUIRE(dim >= 1 && dim <= 256, CQ_ERR_UNSUPPORTED, "cq_sdpa_reference_layout: head_dim must be <= 256");
  CQ_REQUIRE(n_kv_heads >= 1 && n_q_heads % n_kv_heads == 0, CQ_ERR_INVALID,
             "cq_sdpa_reference_layout: n_q_heads must be a multiple of n_kv_heads");
  CQ_REQUIRE(stride_k >= 1 && stride_v >= 1 && seq_len >= 1, CQ_ERR_INVALID, "cq_sdpa_reference_layout: bad sizes");
  CQ_REQUIRE((seq_len - 1) / stride_k + 1 <= n_kf_k && (seq_len - 1) / stride_v + 1 <= n_kf_v, CQ_ERR_INVALID,
             "cq_sdpa_reference_layout: too few keyframes for seq_len");
  CQ_REQUIRE(seq_len - ((seq_len - 1) / stride_k + 1) <= n_pf_k && seq_len - ((seq_len - 1) / stride_v + 1) <= n_pf_v,
             CQ_ERR_INVALID, "cq_sdpa_reference_layout: too few P-frames for seq_len");
  // The reference views are one "page" per head that spans the whole sequence.
  CacheView cv;
  cv.B = 1;
  cv.H = n_kv_heads;
  cv.D = dim;
  cv.P = 1 << 30;  // one page: every token's page index is 0
  cv.max_pages = 1;
  cv.n_pages = 1;
  cv.block_table = nullptr;
  const void *kf[2] = {kf_k, kf_v};
  const uint32_t *pk[2] = {packed_k, packed_v};
  const void *sc[2] = {scales_k, scales_v};
  int nkf[2] = {n_kf_k, n_kf_v}, npf[2] = {n_pf_k, n_pf_v}, stv[2] = {stride_k, stride_v};
  for (int i = 0; i < 2; ++i) {
    cv.c[i].kf = (const __half *)kf[i];
    cv.c[i].codes = pk[i];
    cv.c[i].scales = (const __half *)sc[i];
    cv.c[i].stride = stv[i];
    cv.c[i].apg = nkf[i];
    cv.c[i].ppg = npf[i];
    cv.c[i].srow = npf[i];
    cv.c[i].order = CQ_ORDER_NATURAL;
    cv.c[i].stok = 0;
    cv.c[i].bits = 4;
    cv.c[i].dead_zone = 0.f;
    // one chunk spanning the whole view
    cv.c[i].ac = nkf[i] > 0 ? nkf[i] : 1;
    cv.c[i].pc = npf[i] > 0 ? npf[i] : 1;
    cv.c[i].scn = cv.c[i].pc;
    cv.c[i].kf_hs = (int64_t)nkf[i] * dim;
    cv.c[i].cd_hs = (int64_t)npf[i] * ((dim + 7) / 8);
    cv.c[i].sc_hs = npf[i];
    cv.c[i].kf_cs = cv.c[i].cd_cs = cv.c[i].sc_cs = 0;
  }
  CQ_REQUIRE(cv.P >= seq_len, CQ_ERR_UNSUPPORTED, "cq_sdpa_reference_layout: sequence too long");
  // padded code rows: words = ceil(dim/8)
  return run_generic(cv, seq_len, q, CQ_F32, n_q_heads, 1, (int64_t)n_q_heads * dim, dim, dim, 1.0f, out, CQ_F32,
                     nullptr, workspace, workspace_bytes, 0, (cudaStream_t)stream);
}

extern "C" int cq_attention_masked(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype,
                                   int32_t n_q_heads, int32_t q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq,
                                   float scale, const void *mask, int mask_kind, int mask_dtype, int64_t m_sb,
                                   int64_t m_sh, int64_t m_sq, int64_t m_st, void *out, int out_dtype,
                                   void *workspace, size_t workspace_bytes, int32_t num_splits, void *stream) {
  int r = attention_common_checks(cache, T, n_q_heads, q_len);
  if (r) return r;
  CQ_REQUIRE(q && out && mask, CQ_ERR_INVALID, "cq_attention_masked: null pointer");
  CQ_REQUIRE(q_dtype == CQ_F16 || q_dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_attention_masked: q dtype");
  CQ_REQUIRE(mask_kind == 1 || mask_kind == 2, CQ_ERR_INVALID, "cq_attention_masked: mask_kind must be 1 or 2");
  CQ_REQUIRE(out_dtype == CQ_F16 || out_dtype == CQ_BF16 || out_dtype == CQ_F32, CQ_ERR_UNSUPPORTED,
             "cq_attention_masked: bad out dtype");
  MaskSpec mk;
  mk.ptr = mask;
  mk.kind = mask_kind;
  mk.dtype = mask_dtype;
  mk.sb = m_sb;
  mk.sh = m_sh;
  mk.sq = m_sq;
  mk.st = m_st;
  return run_generic(make_view(*cache), T, q, q_dtype, n_q_heads, q_len, q_sb, q_sh, q_sq, scale, out, out_dtype,
                     nullptr, workspace, workspace_bytes, num_splits, (cudaStream_t)stream, mk);
}

extern "C" int cq_sdpa_reference_layout_workspace(int32_t n_q_heads, int32_t dim, int64_t seq_len, size_t *bytes) {
  CQ_REQUIRE(bytes && n_q_heads >= 1 && dim >= 1 && seq_len >= 1, CQ_ERR_INVALID,
             "cq_sdpa_reference_layout_workspace: bad arguments");
  *bytes = generic_workspace(n_q_heads, pick_splits(n_q_heads, seq_len, 0), dim);
  return CQ_OK;
}
