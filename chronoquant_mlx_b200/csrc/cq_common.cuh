// cq_common.cuh -- shared device/host helpers for libchronoquant_b200.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/chronoquant_b200.h"

namespace cq {

// ---------------------------------------------------------------------------
// error reporting (thread-local message behind cq_last_error)
// ---------------------------------------------------------------------------
int set_error(int code, const std::string &msg);
int check_launch(const char *what);

#define CQ_REQUIRE(cond, code, msg)                  \
  do {                                               \
    if (!(cond)) return ::cq::set_error((code), (msg)); \
  } while (0)

// ---------------------------------------------------------------------------
// device view of a paged cache (copied by value into kernel parameters)
// ---------------------------------------------------------------------------
struct CompView {
  const __half *kf;
  const uint32_t *codes;
  const __half *scales;
  int stride;
  int apg;    // anchors per page
  int ppg;    // P-frames per page
  int srow;   // scale slots per (page, head)
  int order;  // CQ_ORDER_*
  int stok;   // scales indexed by token position (CQ_SCALE_BY_TOKEN)
  int bits;
  float dead_zone;
  // addressing (elements): per (page, head) block, per chunk, slots per chunk
  int64_t kf_hs, cd_hs, sc_hs;
  int64_t kf_cs, cd_cs, sc_cs;
  int ac, pc, scn;  // anchors, code rows, scale slots per chunk
};

struct CacheView {
  int B, H, D, P, max_pages, n_pages;
  const int32_t *block_table;  // nullptr -> page b*max_pages + logical page (reference layout)
  CompView c[2];
};

inline CacheView make_view(const cq_paged_cache &c) {
  CacheView v;
  v.B = c.batch;
  v.H = c.kv_heads;
  v.D = c.head_dim;
  v.P = c.page_tokens;
  v.max_pages = c.max_pages;
  v.n_pages = c.n_pages;
  v.block_table = c.block_table;
  const cq_component *src[2] = {&c.k, &c.v};
  for (int i = 0; i < 2; ++i) {
    v.c[i].kf = (const __half *)src[i]->keyframes;
    v.c[i].codes = src[i]->codes;
    v.c[i].scales = (const __half *)src[i]->scales;
    v.c[i].stride = src[i]->stride;
    v.c[i].apg = src[i]->anchors_per_page;
    v.c[i].ppg = src[i]->pframes_per_page;
    v.c[i].srow = src[i]->scale_row;
    v.c[i].order = src[i]->code_order;
    v.c[i].stok = src[i]->scale_index == CQ_SCALE_BY_TOKEN;
    v.c[i].bits = src[i]->bits;
    v.c[i].dead_zone = src[i]->dead_zone;
    const cq_component &k = *src[i];
    const int W = k.code_order == CQ_ORDER_PLANES3   ? 12
                  : k.code_order == CQ_ORDER_PLANES2 ? 8
                                                     : (c.head_dim + 7) >> 3;  // row words
    const int ct = k.chunk_tokens > 0 ? k.chunk_tokens : c.page_tokens;
    v.c[i].ac = ct / k.stride;
    v.c[i].pc = ct - v.c[i].ac;
    v.c[i].scn = k.scale_index == CQ_SCALE_BY_TOKEN ? ct : v.c[i].pc;
    const bool one = ct == c.page_tokens;
    v.c[i].kf_hs = k.keyframe_head_stride ? k.keyframe_head_stride : (int64_t)k.anchors_per_page * c.head_dim;
    v.c[i].cd_hs = k.code_head_stride ? k.code_head_stride : (int64_t)k.pframes_per_page * W;
    v.c[i].sc_hs = k.scale_head_stride ? k.scale_head_stride : (int64_t)k.scale_row;
    v.c[i].kf_cs = one ? 0 : k.keyframe_chunk_stride;
    v.c[i].cd_cs = one ? 0 : k.code_chunk_stride;
    v.c[i].sc_cs = one ? 0 : k.scale_chunk_stride;
    if (one) v.c[i].scn = k.scale_row;  // one chunk: the scale index never wraps
  }
  return v;
}

// Element addresses of anchor slot a, code row pf and scale slot si (all
// page-local) of (physical page pg, head h); see cq_component.
__host__ __device__ inline int64_t kf_index(const CompView &c, int H, int D, int64_t pg, int h, int a) {
  const int j = a / c.ac;
  return (pg * H + h) * c.kf_hs + j * c.kf_cs + (int64_t)(a - j * c.ac) * D;
}
__host__ __device__ inline int64_t code_index(const CompView &c, int H, int W, int64_t pg, int h, int pf) {
  const int j = pf / c.pc;
  return (pg * H + h) * c.cd_hs + j * c.cd_cs + (int64_t)(pf - j * c.pc) * W;
}
__host__ __device__ inline int64_t scale_index(const CompView &c, int H, int64_t pg, int h, int si) {
  const int j = si / c.scn;
  return (pg * H + h) * c.sc_hs + j * c.sc_cs + (si - j * c.scn);
}

int validate_cache(const cq_paged_cache *c);

__host__ __device__ inline int words_of(int D) { return (D + 7) >> 3; }
// Words of one code row in the cache's layout (the reference layout is words_of).
__host__ __device__ inline int row_words(int D, int order) {
  return order == CQ_ORDER_PLANES3 ? 12 : order == CQ_ORDER_PLANES2 ? 8 : words_of(D);  // planes: head_dim 128
}

// Position of dim d's nibble in a code row: word index and bit shift.
// NATURAL: word d/8, nibble d%8 (kernels.py:15-19).  MMA (head_dim multiple of
// 64): with g = d%8, k = d/8 (0..D/8-1), M4 = D/64: word g*M4 + k/8, nibble k%8.
__host__ __device__ inline void nibble_pos(int d, int D, int order, int &word, int &shift) {
  if (order == CQ_ORDER_MMA) {
    int g = d & 7, k = d >> 3, m4 = D >> 6;
    word = g * m4 + (k >> 3);
    shift = (k & 7) << 2;
  } else {
    word = d >> 3;
    shift = (d & 7) << 2;
  }
}

// Debug builds (-DCQ_CHECKS, libchronoquant_b200_checks.so): every page
// lookup is checked against the block-table row and the page pool.  A bad
// index is recorded in this translation unit's word (device error
// CQ_DEV_ERR_BOUNDS) and replaced by page 0, so the access stays inside the
// pool and the host reads an error code instead of a fault.  Release builds
// compile the checks out.
constexpr int CQ_DEV_ERR_BOUNDS = 7;
#ifdef CQ_CHECKS
static __device__ int g_bounds_error;
__device__ __forceinline__ bool bounds_ok(bool ok) {
  if (!ok) atomicExch(&g_bounds_error, CQ_DEV_ERR_BOUNDS);
  return ok;
}
#endif

// Physical page of logical page lp of sequence b.
__device__ __forceinline__ int64_t page_of(const CacheView &cv, int b, int64_t lp) {
#ifdef CQ_CHECKS
  if (!bounds_ok(b >= 0 && b < cv.B && lp >= 0 && lp < cv.max_pages)) return 0;
  const int64_t pg =
      cv.block_table ? (int64_t)cv.block_table[(int64_t)b * cv.max_pages + lp] : (int64_t)b * cv.max_pages + lp;
  return bounds_ok(pg >= 0 && pg < cv.n_pages) ? pg : 0;
#else
  return cv.block_table ? (int64_t)cv.block_table[(int64_t)b * cv.max_pages + lp] : (int64_t)b * cv.max_pages + lp;
#endif
}

// The same for a cache known to have a block table (the decode kernel's layout).
__device__ __forceinline__ int64_t table_page(const CacheView &cv, int b, int64_t lp) {
#ifdef CQ_CHECKS
  if (!bounds_ok(b >= 0 && b < cv.B && lp >= 0 && lp < cv.max_pages)) return 0;
  const int64_t pg = (int64_t)cv.block_table[(int64_t)b * cv.max_pages + lp];
  return bounds_ok(pg >= 0 && pg < cv.n_pages) ? pg : 0;
#else
  return (int64_t)cv.block_table[(int64_t)b * cv.max_pages + lp];
#endif
}

// Host: this translation unit's bounds-error word (0 in release builds).
static inline int read_bounds_error_here(int clear) {
#ifdef CQ_CHECKS
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_bounds_error, sizeof(int));
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_bounds_error, &z, sizeof(int));
  }
  return v;
#else
  (void)clear;
  return 0;
#endif
}

// Per translation unit readers, combined by cq_device_error.
int read_bounds_error_encode(int clear);
int read_bounds_error_layout(int clear);
int read_bounds_error_attention(int clear);
int read_bounds_error_prefill(int clear);
int read_bounds_error_decode(int clear);

// Locations of token t (absolute) of (b, h) in component comp.
struct TokLoc {
  const __half *anchor;   // fp16 [D]
  const uint32_t *codes;  // nullptr for an I-frame
  float scale;
  int tl;                 // page-local token position
};

__device__ __forceinline__ TokLoc locate(const CacheView &cv, int comp, int b, int h, int64_t t) {
  const CompView &c = cv.c[comp];
  int64_t lp = t / cv.P;
  int tl = (int)(t - lp * cv.P);
  int64_t pg = page_of(cv, b, lp);
  int a = tl / c.stride;
  TokLoc L;
  L.anchor = c.kf + kf_index(c, cv.H, cv.D, pg, h, a);
  L.tl = tl;
  if (tl - a * c.stride == 0) {
    L.codes = nullptr;
    L.scale = 0.f;
  } else {
    int pf = tl - a - 1;
    L.codes = c.codes + code_index(c, cv.H, row_words(cv.D, c.order), pg, h, pf);
    L.scale = __half2float(c.scales[scale_index(c, cv.H, pg, h, c.stok ? tl : pf)]);
  }
  return L;
}

__device__ __forceinline__ int nibble_at(const uint32_t *row, int d, int D, int order) {
  if (order == CQ_ORDER_PLANES3) {  // code + 4 from two planes (head_dim 128), returned as code + 8
    const int g = d & 7, k = d >> 3;
    const uint32_t lo = (row[g] >> (2 * k)) & 3u, hi = (row[8 + (g >> 1)] >> (16 * (g & 1) + k)) & 1u;
    return (int)(lo | (hi << 2)) + 4;
  }
  if (order == CQ_ORDER_PLANES2) return (int)((row[d & 7] >> (2 * (d >> 3))) & 3u) + 6;  // code + 2
  int w, s;
  nibble_pos(d, D, order, w, s);
  return (int)((row[w] >> s) & 0xFu);
}

// ORs the stored value of dim d (nib = code + 8, the INT4-lane value) into a
// code row being assembled in warp-shared words `sw` (zeroed beforehand).
__device__ __forceinline__ void pack_code(uint32_t *sw, int d, int D, int order, uint32_t nib) {
  if (order == CQ_ORDER_PLANES3) {  // head_dim 128
    const uint32_t v = nib - 4u;  // code + 4, in [0, 8) for codes of 3 bits or fewer
    const int g = d & 7, k = d >> 3;
    atomicOr(&sw[g], (v & 3u) << (2 * k));
    atomicOr(&sw[8 + (g >> 1)], (v >> 2) << (16 * (g & 1) + k));
    return;
  }
  if (order == CQ_ORDER_PLANES2) {  // head_dim 128: code + 2, in [0, 4) for codes of 2 bits
    atomicOr(&sw[d & 7], ((nib - 6u) & 3u) << (2 * (d >> 3)));
    return;
  }
  int w, s;
  nibble_pos(d, D, order, w, s);
  atomicOr(&sw[w], nib << s);
}

// ---------------------------------------------------------------------------
// scalar type helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void *p, int64_t i, int dtype) {
  if (dtype == CQ_F16) return __half2float(((const __half *)p)[i]);
  if (dtype == CQ_BF16) return __bfloat162float(((const __nv_bfloat16 *)p)[i]);
  return ((const float *)p)[i];
}

__device__ __forceinline__ void store_from_float(void *p, int64_t i, float v, int dtype) {
  if (dtype == CQ_F16)
    ((__half *)p)[i] = __float2half_rn(v);
  else if (dtype == CQ_BF16)
    ((__nv_bfloat16 *)p)[i] = __float2bfloat16_rn(v);
  else
    ((float *)p)[i] = v;
}

// Round a float to the arithmetic type of the token dtype (fp16 or bf16).
__device__ __forceinline__ float round_dt(float x, int dtype) {
  if (dtype == CQ_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  return __half2float(__float2half_rn(x));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

}  // namespace cq
