/*
 * chronoquant_b200.h -- C ABI of libchronoquant_b200.so (sm_100a).
 *
 * The drop-in boundary for ChronoQuant's KV-cache codec and fused
 * dequant-attention path.  Every entry point:
 *   - takes device pointers the caller allocated, plain sizes and a CUDA
 *     stream (cudaStream_t passed as void*; NULL = legacy default stream);
 *   - is stream-ordered, stateless and safe to call from any host thread;
 *   - returns CQ_OK (0) or a negative status, never aborts or throws;
 *     cq_last_error() returns the calling thread's last message.
 *
 * Reference interfaces replaced (gauravsaini/chronoquant_mlx):
 *   codec.py:23-65   ChronoQuantCodecMLX.quantize_delta   -> cq_quantize_delta
 *   codec.py:67-73   ChronoQuantCodecMLX.dequantize_delta -> cq_dequantize_delta
 *   kernels.py:34-54 pack_int4_codes (+ Metal kernels.py:9-29) -> cq_pack_int4
 *   kernels.py:57-61 unpack_int4_codes                   -> cq_unpack_int4
 *   cache.py:87-129  ChronoQuantCache._append_component   -> cq_append
 *   cache.py:131-160 _reconstruct_component               -> cq_reconstruct
 *   cache.py:220-255 state getter / setter                -> cq_export_state / cq_import_state
 *   kernels.py:248-279 chronoquant_sdpa_kernel (+ Metal kernels.py:79-228)
 *                                                          -> cq_sdpa_reference_layout
 *   attention.py:23-74 chronoquant_sdpa (fused + fallback) -> cq_attention
 *   attention.py:61-74 fallback branch (query chunks)     -> cq_prefill_prepare / cq_prefill_attend
 *   (no reference counterpart) seq-split partial merge     -> cq_lse_merge, cq_lse_merge_packed
 */
#ifndef CHRONOQUANT_B200_H
#define CHRONOQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CQ_ABI_VERSION 3

/* status codes */
#define CQ_OK 0
#define CQ_ERR_INVALID (-1)     /* bad argument (null pointer, size, stride) */
#define CQ_ERR_UNSUPPORTED (-2) /* valid but not supported (e.g. head_dim) */
#define CQ_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define CQ_ERR_WORKSPACE (-4)   /* workspace too small */

/* element types */
#define CQ_F16 0
#define CQ_BF16 1
#define CQ_F32 2

/* Scale indexing within a (page, head) row */
#define CQ_SCALE_BY_PFRAME 0 /* slot = P-frame ordinal (the reference layout, cache.py:116) */
#define CQ_SCALE_BY_TOKEN 1  /* slot = page-local token position, 0 at I-frames */

/* V-code nibble orders (the cache's own storage; the reference layout is order 0) */
#define CQ_ORDER_NATURAL 0 /* word w holds dims 8w..8w+7, LSB first (kernels.py:15-19) */
#define CQ_ORDER_MMA 1     /* word 2g+q, nibble j holds dim g + 64q + 8j (head_dim 128) */
/* Physical 3-bit codes (opt-in; bits <= 3, head_dim 128): a code row is 12
 * words, two bit planes holding v = code + 4 in [0, 8), in the decode
 * kernel's lane order: with g = d%8, k = d/8, the low two bits of dim d at
 * word g, bit 2k, the high bit at word 8 + g/2, bit 16*(g%2) + k.  No
 * reference counterpart: the reference stores 3-bit codes in INT4 lanes
 * (README.md:57); cq_export_state still produces that layout. */
#define CQ_ORDER_PLANES3 2
/* Physical 2-bit codes (opt-in; bits <= 2, head_dim 128): a code row is 8
 * words, v = code + 2 in [0, 4) at word g, bits 2k..2k+1 (the low plane of
 * CQ_ORDER_PLANES3). */
#define CQ_ORDER_PLANES2 3

/*
 * One compressed component (K or V) of a paged cache.  Token t of sequence b
 * lives in page pg = block_table[b*max_pages + t/page_tokens] at page-local
 * position tl = t % page_tokens; it is an I-frame iff tl % stride == 0 (anchor
 * slot tl/stride), else a P-frame in code row tl - tl/stride - 1 anchored on
 * slot tl/stride; its scale sits at that row index (CQ_SCALE_BY_PFRAME) or
 * at tl (CQ_SCALE_BY_TOKEN, whose I-frame slots hold 0).
 *
 * Addressing.  A page is cut into chunks of chunk_tokens tokens (a multiple
 * of the stride dividing page_tokens; 0 = the whole page).  A chunk holds
 * ac = chunk_tokens/stride anchor slots, pc = chunk_tokens - ac code rows and
 * sc = chunk_tokens (by token) or pc (by P-frame) scale slots; page-local
 * index i of an array falls in chunk i / (per-chunk count) at offset
 * i % (per-chunk count):
 *   keyframes fp16 + (pg*kv_heads + h)*keyframe_head_stride
 *                  + chunk*keyframe_chunk_stride + offset*head_dim
 *   codes     u32  + (pg*kv_heads + h)*code_head_stride
 *                  + chunk*code_chunk_stride + offset*ceil(head_dim/8)
 *   scales    fp16 + (pg*kv_heads + h)*scale_head_stride
 *                  + chunk*scale_chunk_stride + offset
 * Strides are in elements of each array; a head stride of 0 means the
 * contiguous [n_pages][kv_heads][...] layout (anchors_per_page*head_dim,
 * pframes_per_page*ceil(head_dim/8), scale_row).  The three arrays of both
 * components may share one allocation: the cache's own layout stores, per
 * (page, head, chunk), one block [K anchors][K codes][K scales][V anchors]
 * [V codes][V scales], which a decode step reads with a single bulk copy.
 */
typedef struct cq_component {
  int32_t stride;           /* I-frame period (cache.py:100) */
  int32_t bits;             /* residual bits 2..8, stored in INT4 lanes */
  float dead_zone;          /* dead-zone ratio (codec.py:36-45) */
  int32_t anchors_per_page; /* page_tokens / stride */
  int32_t pframes_per_page; /* page_tokens - anchors_per_page */
  int32_t scale_row;        /* scale slots per (page, head): >= page_tokens (by token) or pframes_per_page */
  int32_t code_order;       /* CQ_ORDER_* */
  int32_t scale_index;      /* CQ_SCALE_BY_* */
  void *keyframes;          /* fp16 */
  uint32_t *codes;
  void *scales;             /* fp16 */
  int64_t keyframe_head_stride, code_head_stride, scale_head_stride;    /* 0: contiguous */
  int32_t chunk_tokens;     /* 0: one chunk per page */
  int32_t reserved;
  int64_t keyframe_chunk_stride, code_chunk_stride, scale_chunk_stride;  /* unused with one chunk */
} cq_component;

typedef struct cq_paged_cache {
  int32_t batch;
  int32_t kv_heads;
  int32_t head_dim;    /* multiple of 8, <= 256 */
  int32_t page_tokens; /* multiple of lcm(stride_k, stride_v) */
  int32_t max_pages;   /* row length of block_table */
  int32_t n_pages;     /* pool capacity in pages */
  const int32_t *block_table; /* device int32 [batch][max_pages] */
  cq_component k;
  cq_component v;
} cq_paged_cache;

int cq_abi_version(void);
const char *cq_last_error(void);

/* Chunk size (tokens) in which a cache with these strides should store its
 * pages for the sm_100a decode kernel (one bulk copy per chunk block), or 0
 * when that kernel does not take these strides or head_dim (store one chunk
 * per page).  No reference counterpart: the reference stores flat arrays. */
int cq_decode_chunk_tokens(int32_t stride_k, int32_t stride_v, int32_t page_tokens, int32_t head_dim);

/* Device-side error word: set (non-zero) when a kernel gave up instead of
 * hanging or writing out of range: 1 = a bulk copy never landed (bounded
 * wait), 4 = a device-resident length outside [1, mapped tokens] (attention
 * wrote nothing), 5 = a device-resident append past the mapped pages (append
 * wrote nothing), 6 = the tensor-core query-chunk kernel gave up on a bounded
 * wait (its output is incomplete), 7 = (debug build with -DCQ_CHECKS only) a
 * page index outside the block-table row or the page pool, replaced by page 0
 * (results invalid), 9 = cq_peer_sum_norm gave up waiting for a peer rank
 * (its rows unwritten).  Synchronises the device; clear != 0 resets the word. */
int cq_device_error(int *code, int clear);

/* Row-parallel sum over NVLink peer memory, fused with the residual add and
 * RMSNorm that follow it in a tensor-parallel decode step (no reference
 * counterpart: the reference runs on one device).  Every rank allocates a
 * region of cq_peer_region_bytes(max_rows, dim, world) bytes with
 * cq_peer_region_alloc (zero-filled; its CUDA IPC handle, 64 bytes, goes to
 * the other ranks), and maps every other rank's region with
 * cq_peer_region_open, called with its own device current.  regions: host
 * array of the world regions' addresses as this rank sees them, in rank
 * order.  cq_peer_sum_norm pushes this rank's part [rows][dim] (local device
 * memory, dtype bf16 or f16) into every region, flags it, waits (bounded;
 * error 9 in cq_device_error when it gives up, rows unwritten) for every
 * rank's part, and computes per row x <- x + dtype(sum of the parts in rank
 * order), y <- dtype(x * rsqrt(mean(x^2) + eps)) * w.  parity alternates
 * between consecutive calls; counter: device int64[2], zero before the first
 * call of a region set.  Every rank makes the same calls in the same order;
 * rows <= max_rows <= 64, dim a multiple of 8, all pointers 16-byte aligned. */
int64_t cq_peer_region_bytes(int64_t max_rows, int32_t dim, int32_t world);
int cq_peer_region_alloc(int64_t bytes, void **ptr, void *ipc_handle);
int cq_peer_region_open(const void *ipc_handle, void **ptr);
int cq_peer_region_close(void *ptr);
int cq_peer_region_free(void *ptr);
int cq_peer_sum_norm(const uint64_t *regions, int32_t world, int32_t rank, int32_t parity, int64_t max_rows,
                     int64_t rows, int32_t dim, const void *part, void *x, const void *w, float eps, void *y,
                     int64_t *counter, int dtype, void *stream);

/* Encode S new tokens at absolute positions t0..t0+S-1 for K and V in one
 * launch (cache.py:87-129, codec.py:23-65).  keys/values: [batch][kv_heads]
 * [S][head_dim] with element strides (sb, sh, ss) and unit dim stride, of
 * type dtype (CQ_F16 or CQ_BF16).  Pages covering t0..t0+S-1 must be mapped
 * in block_table.  Anchors of P-frames that precede t0 are read from the
 * cache. */
int cq_append(const cq_paged_cache *cache, const void *keys, int64_t k_sb, int64_t k_sh, int64_t k_ss,
              const void *values, int64_t v_sb, int64_t v_sh, int64_t v_ss, int dtype, int64_t t0,
              int32_t S, void *stream);

/* Attention of q_len queries per sequence against the first T cached tokens
 * (attention.py:23-74).  q: [batch][n_q_heads][q_len][head_dim] with strides
 * (q_sb, q_sh, q_sq), dtype CQ_F16/CQ_BF16; the scores use q*scale rounded
 * to the query dtype (attention.py:46/65).  causal != 0 applies the causal
 * mask anchored at the end (attention.py:8-20; no effect when q_len == 1);
 * causal == 0 lets every query see all T keys (mask=None).  out: [batch][n_q_heads][q_len]
 * [head_dim] contiguous, out_dtype CQ_F16/CQ_BF16/CQ_F32.  workspace: device
 * memory of at least cq_attention_workspace() bytes (split-KV partials and
 * per-call-stamped completion words; its prior contents are ignored);
 * num_splits <= 0 picks a split count.  Query chunks (q_len >= 16, head_dim
 * 128, a GQA group that is a power of two <= 16) run on the tensor cores: the
 * history is reconstructed in fp16 (as cache.py:131-160) into the workspace
 * (16-byte aligned, as is out), whose size then covers 2*T*head_dim*2 bytes
 * per (sequence, kv-head) plus the query tiles.  lse_out (optional, may be NULL):
 * fp32 [batch][n_q_heads][q_len] log-sum-exp of the scaled scores (natural
 * log), for merging sequence shards. */
int cq_attention(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype, int32_t n_q_heads,
                 int32_t q_len, int32_t causal, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, void *out,
                 int out_dtype, float *lse_out, void *workspace, size_t workspace_bytes, int32_t num_splits,
                 void *stream);
int cq_attention_workspace(const cq_paged_cache *cache, int64_t T, int32_t n_q_heads, int32_t q_len,
                           int32_t num_splits, size_t *bytes);

/* The two halves of cq_attention's tensor-core query-chunk path, for callers
 * that schedule or time them apart (no reference counterpart; together they
 * are the fallback branch of attention.py:61-74).  cq_prefill_prepare
 * reconstructs the first T cached tokens in fp16 (cache.py:131-160) into the
 * workspace as tensor-core tile images and packs q*scale (rounded to the
 * query dtype, attention.py:65) into query tiles; cq_prefill_attend runs the
 * attention over those images.  Arguments and workspace as cq_attention;
 * CQ_ERR_UNSUPPORTED for shapes that do not take this path (head_dim != 128,
 * q_len < 16, GQA group not a power of two <= 16). */
int cq_prefill_prepare(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype, int32_t n_q_heads,
                       int32_t q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, void *workspace,
                       size_t workspace_bytes, void *stream);
int cq_prefill_attend(const cq_paged_cache *cache, int64_t T, int32_t n_q_heads, int32_t q_len, int32_t causal,
                      void *out, int out_dtype, float *lse_out, void *workspace, size_t workspace_bytes,
                      void *stream);

/* A decode step that a CUDA graph can replay at any length (no reference
 * counterpart: the reference steps eagerly from Python, cache.py:198-215 and
 * attention.py:23-74).  len_dev: device int64[2] = {tokens cached, arrival
 * counter}, zero-initialised by the caller; neither call reads the length on
 * the host.  cq_append_at encodes S tokens at positions len_dev[0].. (as
 * cq_append) and, when its grid completes, advances len_dev[0] by S and leaves
 * the counter at 0.  cq_attention_at is cq_attention for q_len 1 over
 * len_dev[0] tokens; its grid and workspace are sized for max_len tokens
 * (query cq_attention_workspace with T = max_len).  It needs the cache layout
 * of the sm_100a decode kernel (cq_decode_chunk_tokens) and answers
 * CQ_ERR_UNSUPPORTED otherwise.  A length outside the mapped pages makes the
 * kernels write nothing and set cq_device_error. */
int cq_append_at(const cq_paged_cache *cache, const void *keys, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                 const void *values, int64_t v_sb, int64_t v_sh, int64_t v_ss, int dtype, int64_t *len_dev,
                 int32_t S, void *stream);
int cq_attention_at(const cq_paged_cache *cache, const int64_t *len_dev, int64_t max_len, const void *q, int q_dtype,
                    int32_t n_q_heads, int64_t q_sb, int64_t q_sh, float scale, void *out, int out_dtype,
                    float *lse_out, void *workspace, size_t workspace_bytes, void *stream);

/* cq_append_at of one token per (sequence, kv-head) followed by
 * cq_attention_at, as one kernel launch: the warp that reads each unit's last
 * chunk first encodes the unit's new token (keys/values [batch][kv_heads][1]
 * [head_dim] at b*sb + h*sh, unit dim stride, kv_dtype f16/bf16) into the
 * cache and into its on-chip copy, the attention covers len_dev[0] + 1
 * tokens, and the grid's last CTA advances len_dev[0] by one (leaving the
 * arrival counter len_dev[1] at 0).  The cache bytes written equal
 * cq_append's.  Same requirements as cq_attention_at.  No reference
 * counterpart (the reference appends and attends in separate eager calls). */
int cq_decode_step_at(const cq_paged_cache *cache, const void *keys, int64_t k_sb, int64_t k_sh, const void *values,
                      int64_t v_sb, int64_t v_sh, int kv_dtype, int64_t *len_dev, int64_t max_len, const void *q,
                      int q_dtype, int32_t n_q_heads, int64_t q_sb, int64_t q_sh, float scale, void *out,
                      int out_dtype, float *lse_out, void *workspace, size_t workspace_bytes, void *stream);

/* cq_attention with an explicit mask instead of the implicit causal rule
 * (attention.py:8-20 for array masks): mask_kind 1 = boolean uint8 (nonzero
 * keeps the key; masked scores become finfo(score dtype).min as
 * attention.py:19 does), 2 = additive of mask_dtype.  Element (b, h, i, t) is
 * at b*m_sb + h*m_sh + i*m_sq + t*m_st (a 0 stride broadcasts). */
int cq_attention_masked(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype, int32_t n_q_heads,
                        int32_t q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, const void *mask,
                        int mask_kind, int mask_dtype, int64_t m_sb, int64_t m_sh, int64_t m_sq, int64_t m_st,
                        void *out, int out_dtype, void *workspace, size_t workspace_bytes, int32_t num_splits,
                        void *stream);

/* Merge attention outputs of the same rows computed over disjoint key shards
 * (sequence split): lse fp32 [n_parts][rows] (natural-log log-sum-exp of each
 * shard's scaled scores, -inf for an empty shard), o fp32 [n_parts][rows][dim]
 * (each shard's normalised output).  out[r] = sum_i exp(lse_i - L) o_i with
 * L = logsumexp_i lse_i; out: [rows][dim] in out_dtype. */
int cq_lse_merge(const float *lse, const float *o, int32_t n_parts, int64_t rows, int32_t dim, void *out,
                 int out_dtype, void *stream);

/* cq_lse_merge over partials packed one buffer per part, as a single
 * all-gather delivers them: parts fp32 [n_parts][rows*dim + rows], each part
 * its outputs [rows][dim] followed by its log-sum-exp [rows].  No reference
 * counterpart (the reference runs on one device). */
int cq_lse_merge_packed(const float *parts, int32_t n_parts, int64_t rows, int32_t dim, void *out, int out_dtype,
                        void *stream);

/* Decoded fp16 history of one component (0=K, 1=V) for tokens 0..T-1:
 * out [batch][kv_heads][T][head_dim].  mode 0 rounds like the reference's
 * fallback (fp16(code*scale), then fp16(anchor + that), cache.py:141-156);
 * mode 1 rounds the exact anchor + code*scale once. */
int cq_reconstruct(const cq_paged_cache *cache, int component, int64_t T, void *out, int mode, void *stream);

/* Reference-layout state (cache.py:220-234) of one component for tokens
 * 0..T-1: keyframes fp16 [batch][kv_heads][n_kf][head_dim], packed u32
 * [batch][kv_heads][n_pf][head_dim/8] (natural nibble order), scales fp16
 * [batch][kv_heads][n_pf].  cq_import_state is the inverse (cache.py:236-255). */
int cq_export_state(const cq_paged_cache *cache, int component, int64_t T, void *keyframes,
                    uint32_t *packed, void *scales, void *stream);
int cq_import_state(const cq_paged_cache *cache, int component, int64_t T, const void *keyframes,
                    const uint32_t *packed, const void *scales, void *stream);

/* Codec on a flat row set (codec.py:23-73).  delta: rows x dim of dtype;
 * codes int8 rows x dim; scales fp16 rows. */
int cq_quantize_delta(const void *delta, int dtype, int64_t rows, int32_t dim, int32_t bits, float dead_zone,
                      int8_t *codes, void *scales, void *stream);
int cq_dequantize_delta(const int8_t *codes, const void *scales, int64_t rows, int32_t dim, void *out,
                        void *stream);

/* INT4 packing in the reference layout (kernels.py:34-61): rows x dim int8
 * <-> rows x ceil(dim/8) uint32. */
int cq_pack_int4(const int8_t *codes, int64_t rows, int32_t dim, uint32_t *packed, void *stream);
int cq_unpack_int4(const uint32_t *packed, int64_t rows, int32_t dim, int8_t *codes, void *stream);

/* The fused decode kernel's reference-layout entry (kernels.py:248-279):
 * q fp32 [n_q_heads][dim] (already scaled), keyframes [kv_heads][n_kf][dim]
 * fp16, packed [kv_heads][n_pf][ceil(dim/8)] u32, scales [kv_heads][n_pf]
 * fp16, per K and V; out fp32 [n_q_heads][dim].  n_kf/n_pf are the first
 * dimension extents of the views (cache.py:162-190). */
int cq_sdpa_reference_layout(const float *q, int32_t n_q_heads, int32_t dim, const void *kf_k, int32_t n_kf_k,
                             const uint32_t *packed_k, const void *scales_k, int32_t n_pf_k, const void *kf_v,
                             int32_t n_kf_v, const uint32_t *packed_v, const void *scales_v, int32_t n_pf_v,
                             int32_t n_kv_heads, int64_t seq_len, int32_t stride_k, int32_t stride_v,
                             float *out, void *workspace, size_t workspace_bytes, void *stream);
int cq_sdpa_reference_layout_workspace(int32_t n_q_heads, int32_t dim, int64_t seq_len, size_t *bytes);

/* cq_attention without a workspace argument, for callers that cannot
 * allocate device memory at decode time (a runtime whose memory pool is owned
 * elsewhere, a thread that must not take an allocator's lock mid-step, a
 * binding that holds only plain pointers).  No reference counterpart: the
 * reference's attention (attention.py:23-74) allocates through MLX.
 *
 * The split-KV partials live in one fixed device array of
 * CQ_STATIC_SCRATCH_BYTES bytes per device inside the library; the call
 * allocates nothing.  A shape whose partials need more (cq_attention_workspace
 * reports the size) is rejected with CQ_ERR_WORKSPACE.  The first call on a
 * device, with that device current, looks up the array's address; make it
 * before any stream capture (resetting the device afterwards is not
 * supported).  Each call clears, on its stream, the few words of the array
 * the decode kernel counts in (they must start at zero; the rest is written
 * before it is read).  All calls on one device share the array: calls that
 * overlap on the device (other streams, other host threads) race and can
 * corrupt each other's results, so serialise them on one stream.  Arguments
 * and results are those of cq_attention. */
#define CQ_STATIC_SCRATCH_BYTES (8u << 20)
int cq_attention_static_scratch(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype,
                                int32_t n_q_heads, int32_t q_len, int32_t causal, int64_t q_sb, int64_t q_sh,
                                int64_t q_sq, float scale, void *out, int out_dtype, float *lse_out,
                                int32_t num_splits, void *stream);

/* Decoder helpers (no reference counterpart: the reference gets its model
 * from mlx_lm).  The elementwise steps of the decoder that drives the cache
 * end to end (bench config 5), each one kernel, rounding as the unfused
 * torch ops do:
 *   cq_rmsnorm       y[r] = dtype(x[r] * rsqrt(mean(x[r]^2) + eps)) * w, rows of dim;
 *   cq_qk_norm_rope  per head of fused QKV rows [batch][(Hq + 2 Hkv) * 128] (row
 *                    stride in elements): RMSNorm over head_dim with q_norm_w /
 *                    k_norm_w for the q / k heads, rotate-half RoPE at position
 *                    *pos with inv_freq[64] (fp32); q, k, v written contiguous
 *                    [batch][H][128];
 *   cq_silu_mul      y = dtype(silu(g)) * u for gu rows [gate (ffn) | up (ffn)].
 * dtype CQ_F16 or CQ_BF16 for every tensor argument except inv_freq and pos. */
int cq_rmsnorm(const void *x, const void *w, void *y, int64_t rows, int32_t dim, float eps, int dtype, void *stream);
int cq_qk_norm_rope(const void *qkv, int64_t row_stride, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                    int32_t head_dim, const void *q_norm_w, const void *k_norm_w, const float *inv_freq,
                    const int64_t *pos, float eps, void *q_out, void *k_out, void *v_out, int dtype, void *stream);
int cq_silu_mul(const void *gu, void *y, int64_t rows, int32_t ffn, int dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CHRONOQUANT_B200_H */
