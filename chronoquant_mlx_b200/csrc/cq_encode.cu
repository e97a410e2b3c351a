// cq_encode.cu -- streaming encode of new K/V tokens into the paged cache.
//
// One warp per (component, sequence, kv-head, token); bulk appends at
// head_dim 128 take one warp per 8-token block (append_block_kernel).  A token at position t
// is an I-frame iff t % stride == 0 (cache.py:100-105): it is stored as fp16.
// Otherwise it is a P-frame anchored on the I-frame at (t/stride)*stride
// (cache.py:107-111); its residual against that anchor is quantised per token
// (codec.py:23-65) and packed into INT4 lanes (kernels.py:34-54).  Every step
// rounds to the token dtype exactly as the reference's fp16 (or bf16) MLX
// arithmetic does: fp32 arithmetic on dtype values followed by one rounding is
// the correctly rounded dtype result for + - * /.
#include "cq_encode.cuh"

namespace cq {

constexpr int kEncodeWarps = 8;

struct EncodeArgs {
  CacheView cv;
  const void *x[2];
  int64_t sb[2], sh[2], ss[2];
  int64_t t0;
  int S;
  // device-resident length (graph replays): t0 = len[0]; the last block to
  // finish advances len[0] by S and resets the arrival counter len[1]
  int64_t *len;
};

__device__ int g_append_error;
constexpr int ERR_APPEND_RANGE = 5;  // tokens past the mapped pages

template <int DTYPE>
__device__ __forceinline__ void encode_token(const EncodeArgs &A, int64_t t0, uint32_t *sw);

template <int DTYPE>
__global__ void __launch_bounds__(kEncodeWarps * 32) append_kernel(EncodeArgs A) {
  __shared__ uint32_t s_words[kEncodeWarps][32];
  __shared__ int64_t s_t0;
  // a programmatically dependent successor (the decode kernel) may be
  // scheduled now; it waits for this grid's completion before reading
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    int64_t t0 = A.t0;
    if (A.len) {
      t0 = *(volatile int64_t *)A.len;
      if (t0 < 0 || (t0 + A.S - 1) / A.cv.P >= A.cv.max_pages) {
        atomicExch(&g_append_error, ERR_APPEND_RANGE);
        t0 = -1;
      }
    }
    s_t0 = t0;
  }
  __syncthreads();
  const int64_t t0 = s_t0;
  if (t0 >= 0) encode_token<DTYPE>(A, t0, s_words[threadIdx.x >> 5]);
  if (A.len) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      unsigned long long *arrive = (unsigned long long *)(A.len + 1);
      if (atomicAdd(arrive, 1ull) == gridDim.x - 1) {  // every block has read the old length
        if (t0 >= 0) *(volatile int64_t *)A.len = t0 + A.S;
        *arrive = 0ull;
      }
    }
  }
}

// Encode the token of this warp: component, sequence, kv-head and position
// t0 + s from the warp index.
template <int DTYPE>
__device__ __forceinline__ void encode_token(const EncodeArgs &A, int64_t t0, uint32_t *sw) {
  const CacheView &cv = A.cv;
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int64_t warp = (int64_t)blockIdx.x * kEncodeWarps + wib;
  const int64_t total = 2LL * cv.B * cv.H * A.S;
  if (warp >= total) return;
  const int s = (int)(warp % A.S);
  int64_t r = warp / A.S;
  const int h = (int)(r % cv.H);
  r /= cv.H;
  const int b = (int)(r % cv.B);
  const int comp = (int)(r / cv.B);
  const CompView &c = cv.c[comp];
  const int D = cv.D;

  const int64_t t = t0 + s;
  const int64_t lp = t / cv.P;
  const int tl = (int)(t - lp * cv.P);
  const int64_t pg = page_of(cv, b, lp);
  const int a = tl / c.stride;
  const int phase = tl - a * c.stride;
  const int64_t xbase = b * A.sb[comp] + h * A.sh[comp];

  float xv[kMaxDimsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDimsPerLane; ++i) {
    int d = lane + 32 * i;
    xv[i] = (d < D) ? load_as_float(A.x[comp], xbase + s * A.ss[comp] + d, DTYPE) : 0.f;
  }

  __half *kf_row = const_cast<__half *>(c.kf) + kf_index(c, cv.H, D, pg, h, a);
  if (phase == 0) {  // I-frame: token.astype(float16) (cache.py:103-105)
#pragma unroll
    for (int i = 0; i < kMaxDimsPerLane; ++i) {
      int d = lane + 32 * i;
      if (d < D) kf_row[d] = __float2half_rn(xv[i]);
    }
    if (c.stok && lane == 0) const_cast<__half *>(c.scales)[scale_index(c, cv.H, pg, h, tl)] = __float2half_rn(0.f);
    return;
  }

  // Anchor token: in this call (read and convert the input, exactly as the
  // stored keyframe) or already in the cache (written by an earlier launch).
  const int64_t ta = t - phase;
  float av[kMaxDimsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDimsPerLane; ++i) {
    int d = lane + 32 * i;
    float v = 0.f;
    if (d < D) {
      if (ta >= t0)
        v = __half2float(__float2half_rn(load_as_float(A.x[comp], xbase + (ta - t0) * A.ss[comp] + d, DTYPE)));
      else
        v = __half2float(kf_row[d]);
    }
    av[i] = v;
  }

  const float scale = encode_residual<DTYPE>(xv, av, D, c.bits, c.dead_zone, c.order, sw, lane);
  const int W = row_words(D, c.order);
  const int pf = tl - a - 1;
  uint32_t *code_row = const_cast<uint32_t *>(c.codes) + code_index(c, cv.H, W, pg, h, pf);
  if (lane < W) code_row[lane] = sw[lane];
  if (lane == 0) {
    // scale.astype(float16) (codec.py:65, cache.py:116)
    const_cast<__half *>(c.scales)[scale_index(c, cv.H, pg, h, c.stok ? tl : pf)] = __float2half_rn(scale);
  }
}

// ---------------------------------------------------------------------------
// Bulk appends (head_dim 128, host-known position).  One warp per (component,
// sequence, kv-head, 8-token block aligned to multiples of 8); lane l encodes
// token l / 4 of the block, dims 32 j .. 32 j + 31 with j = l % 4.  A token's
// max and dead-zone max are two shuffles among its four lanes, a lane's 32
// values are independent of one another, and the code words are assembled in
// registers: in the natural order a lane's four words are whole, in the MMA
// order a word is two halves from neighbouring lanes, and a bit-plane word is
// an OR over the token's four lanes.  The codec and its rounding are
// encode_residual's; the quotients take one reciprocal per token
// (code_nibble_rcp) instead of a division per value.
constexpr int kBlockTokens = 8;

template <int DTYPE>
__device__ __forceinline__ void unpack8(uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 f;
    if (DTYPE == CQ_BF16)
      f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[k]));
    else
      f = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8_half(const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
    w[k] = *reinterpret_cast<const uint32_t *>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int DTYPE>
__global__ void __launch_bounds__(kEncodeWarps * 32) append_block_kernel(EncodeArgs A, int64_t blk0, int64_t nblk) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const CacheView &cv = A.cv;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * kEncodeWarps + (threadIdx.x >> 5);
  if (warp >= 2LL * cv.B * cv.H * nblk) return;  // whole warps
  const int64_t blk = blk0 + warp % nblk;
  int64_t r = warp / nblk;
  const int h = (int)(r % cv.H);
  r /= cv.H;
  const int b = (int)(r % cv.B);
  const int comp = (int)(r / cv.B);
  const CompView &c = cv.c[comp];
  const int j = lane & 3;
  const int64_t t = blk * kBlockTokens + (lane >> 2);
  const bool live = t >= A.t0 && t < A.t0 + A.S;
  // the block lies in one page and in one chunk of it
  const int64_t lp = blk * kBlockTokens / cv.P;
  const int tl = (int)(t - lp * cv.P);
  const int64_t pg = page_of(cv, b, lp);
  const int jc = (int)((blk * kBlockTokens - lp * cv.P) / (c.ac + c.pc));
  const int64_t hb = pg * cv.H + h;
  const int a = tl / c.stride, phase = tl - a * c.stride;
  __half *kf_row = const_cast<__half *>(c.kf) + hb * c.kf_hs + jc * c.kf_cs + (int64_t)(a - jc * c.ac) * 128 + 32 * j;
  __half *sc_base = const_cast<__half *>(c.scales) + hb * c.sc_hs + jc * c.sc_cs - (int64_t)jc * c.scn;
  const char *xp = (const char *)A.x[comp];
  const int64_t xb = b * A.sb[comp] + h * A.sh[comp] + 32 * j;
  float x[4][8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (live) {
      unpack8<DTYPE>(*reinterpret_cast<const uint4 *>(xp + 2 * (xb + (t - A.t0) * A.ss[comp] + 8 * k)), x[k]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[k][e] = 0.f;
    }
  }
  const bool iframe = live && phase == 0, pframe = live && phase != 0;
  if (iframe) {  // token.astype(float16) (cache.py:103-105)
#pragma unroll
    for (int k = 0; k < 4; ++k) reinterpret_cast<uint4 *>(kf_row)[k] = pack8_half(x[k]);
    if (c.stok && j == 0) sc_base[tl] = __float2half_rn(0.f);
  }
  // the anchor (its fp16 value): in this call's input, or stored by an earlier call
  float an[4][8];
  const int64_t ta = t - phase;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (pframe && ta >= A.t0) {
      unpack8<DTYPE>(*reinterpret_cast<const uint4 *>(xp + 2 * (xb + (ta - A.t0) * A.ss[comp] + 8 * k)), an[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) an[k][e] = __half2float(__float2half_rn(an[k][e]));
    } else if (pframe) {
      unpack8<CQ_F16>(reinterpret_cast<const uint4 *>(kf_row)[k], an[k]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) an[k][e] = 0.f;
    }
  }
  // delta = token - anchor.astype(token.dtype), in the token dtype (cache.py:113)
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float anv = (DTYPE == CQ_BF16) ? round_dt(an[k][e], CQ_BF16) : an[k][e];
      x[k][e] = pframe ? round_dt(x[k][e] - anv, DTYPE) : 0.f;
      amax = fmaxf(amax, fabsf(x[k][e]));
    }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const int hl_i = (1 << c.bits) / 2;
  const float hl = (float)hl_i, hlm1 = (float)(hl_i - 1);
  const float tiny = round_dt(1e-10f, DTYPE);  // 0 in fp16
  float scale = round_dt(__fdiv_rn(amax, hlm1), DTYPE);
  if (c.dead_zone > 0.f) {  // codec.py:36-45
    const float thr = round_dt(amax * round_dt(c.dead_zone, DTYPE), DTYPE);
    float amax_c = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (fabsf(x[k][e]) < thr) x[k][e] = 0.f;
        amax_c = fmaxf(amax_c, fabsf(x[k][e]));
      }
    amax_c = fmaxf(amax_c, __shfl_xor_sync(0xffffffffu, amax_c, 1));
    amax_c = fmaxf(amax_c, __shfl_xor_sync(0xffffffffu, amax_c, 2));
    scale = round_dt(__fdiv_rn((amax_c < tiny) ? amax : amax_c, hlm1), DTYPE);
  }
  const bool zero_scale = scale < tiny;
  const float scale_safe = zero_scale ? 1.f : scale;
  // one reciprocal per token; a bf16 scale so small that 1/scale overflows
  // is scaled up by 2^64 together with the residuals (exact, same quotients)
  float sc = scale_safe, rcp = __frcp_rn(scale_safe), up = 1.f;
  if (!(rcp < INFINITY)) {
    up = 0x1p64f;
    sc = scale_safe * up;
    rcp = __frcp_rn(sc);
  }
  uint32_t nib[4][8];
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) nib[k][e] = code_nibble_rcp<DTYPE>(x[k][e] * up, sc, rcp, hl, zero_scale);
  const int pf = tl - a - 1;
  const int W = row_words(128, c.order);
  uint32_t *row = const_cast<uint32_t *>(c.codes) + hb * c.cd_hs + jc * c.cd_cs + (int64_t)(pf - jc * c.pc) * W;
  if (c.order == CQ_ORDER_MMA) {
    // dim 32 j + 8 k + g -> word 2 g + j / 2, nibble 4 (j % 2) + k
    uint32_t m[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t v = 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) v |= nib[k][g] << (4 * (4 * (j & 1) + k));
      m[g] = v | __shfl_xor_sync(0xffffffffu, v, 1);
    }
    if (pframe) {
#pragma unroll
      for (int g = 0; g < 4; ++g) row[2 * (g + 4 * (j & 1)) + (j >> 1)] = (j & 1) ? m[g + 4] : m[g];
    }
  } else if (c.order == CQ_ORDER_PLANES3) {
    // v = code + 4: low bits of dim g + 8 k' in word g at bit 2 k', high bit in word 8 + g / 2 at
    // bit 16 (g % 2) + k', with k' = 4 j + k
    uint32_t w[12];
#pragma unroll
    for (int q = 0; q < 12; ++q) w[q] = 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const uint32_t v = nib[k][g] - 4u, kk = 4 * j + k;
        w[g] |= (v & 3u) << (2 * kk);
        w[8 + (g >> 1)] |= ((v >> 2) & 1u) << (16 * (g & 1) + kk);
      }
#pragma unroll
    for (int q = 0; q < 12; ++q) {
      w[q] |= __shfl_xor_sync(0xffffffffu, w[q], 1);
      w[q] |= __shfl_xor_sync(0xffffffffu, w[q], 2);
    }
    if (pframe) {
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        // word 3 j + q of the row, selected without local memory
        uint32_t o = w[q];
#pragma unroll
        for (int jj = 1; jj < 4; ++jj)
          if (j == jj) o = w[3 * jj + q];
        row[3 * j + q] = o;
      }
    }
  } else if (c.order == CQ_ORDER_PLANES2) {
    // v = code + 2: dim g + 8 k' in word g at bits 2 k', with k' = 4 j + k
    uint32_t w[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t v = 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) v |= ((nib[k][g] - 6u) & 3u) << (2 * (4 * j + k));
      v |= __shfl_xor_sync(0xffffffffu, v, 1);
      w[g] = v | __shfl_xor_sync(0xffffffffu, v, 2);
    }
    if (pframe) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        // word 2 j + q of the row, selected without local memory
        uint32_t o = w[q];
#pragma unroll
        for (int jj = 1; jj < 4; ++jj)
          if (j == jj) o = w[2 * jj + q];
        row[2 * j + q] = o;
      }
    }
  } else if (pframe) {  // natural: word 4 j + k holds dims 32 j + 8 k .. + 7, nibble g at bit 4 g
    uint32_t wd[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t v = 0u;
#pragma unroll
      for (int g = 0; g < 8; ++g) v |= nib[k][g] << (4 * g);
      wd[k] = v;
    }
    reinterpret_cast<uint4 *>(row)[j] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
  if (pframe && j == 0)  // scale.astype(float16) (codec.py:65, cache.py:116)
    sc_base[c.stok ? tl : pf] = __float2half_rn(scale);
}

// The bulk path's preconditions: head_dim 128, 8-token blocks that never
// straddle a page or a chunk, and 16-byte aligned token rows, anchor rows and
// code rows.
static bool block_path_ok(const cq_paged_cache *cache, const CacheView &cv, const void *keys, int64_t k_sb,
                          int64_t k_sh, int64_t k_ss, const void *values, int64_t v_sb, int64_t v_sh, int64_t v_ss) {
  if (cache->head_dim != 128 || cache->page_tokens % kBlockTokens) return false;
  const int64_t st[6] = {k_sb, k_sh, k_ss, v_sb, v_sh, v_ss};
  for (int64_t x : st)
    if (x % 8) return false;
  if (((uintptr_t)keys | (uintptr_t)values) & 15) return false;
  for (int i = 0; i < 2; ++i) {
    const CompView &c = cv.c[i];
    if ((c.ac + c.pc) % kBlockTokens) return false;
    if (((uintptr_t)c.kf & 15) || (c.kf_hs % 8) || (c.kf_cs % 8)) return false;
    if (((uintptr_t)c.codes & 15) || (c.cd_hs % 4) || (c.cd_cs % 4)) return false;
  }
  return true;
}

static int launch_append(const cq_paged_cache *cache, const void *keys, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                         const void *values, int64_t v_sb, int64_t v_sh, int64_t v_ss, int dtype, int64_t t0,
                         int64_t *len, int32_t S, void *stream, const char *who) {
  int r = validate_cache(cache);
  if (r) return r;
  CQ_REQUIRE(keys && values, CQ_ERR_INVALID, std::string(who) + ": keys/values null");
  CQ_REQUIRE(dtype == CQ_F16 || dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, std::string(who) + ": dtype must be f16 or bf16");
  CQ_REQUIRE(S >= 0 && t0 >= 0, CQ_ERR_INVALID, std::string(who) + ": negative S or t0");
  if (S == 0) return CQ_OK;
  if (!len) {
    int64_t last_page = (t0 + S - 1) / cache->page_tokens;
    CQ_REQUIRE(last_page < cache->max_pages, CQ_ERR_INVALID, std::string(who) + ": tokens beyond max_pages*page_tokens");
  }
  EncodeArgs A;
  A.cv = make_view(*cache);
  A.x[0] = keys;
  A.x[1] = values;
  A.sb[0] = k_sb; A.sh[0] = k_sh; A.ss[0] = k_ss;
  A.sb[1] = v_sb; A.sh[1] = v_sh; A.ss[1] = v_ss;
  A.t0 = t0;
  A.S = S;
  A.len = len;
  cudaStream_t st = (cudaStream_t)stream;
  if (!len && S > 1 && block_path_ok(cache, A.cv, keys, k_sb, k_sh, k_ss, values, v_sb, v_sh, v_ss)) {
    const int64_t blk0 = t0 / kBlockTokens, nblk = (t0 + S - 1) / kBlockTokens - blk0 + 1;
    const int64_t gw = 2LL * cache->batch * cache->kv_heads * nblk;
    const int64_t gb = (gw + kEncodeWarps - 1) / kEncodeWarps;
    CQ_REQUIRE(gb < (1LL << 31), CQ_ERR_INVALID, std::string(who) + ": too many tokens in one call");
    if (dtype == CQ_F16)
      append_block_kernel<CQ_F16><<<(unsigned)gb, kEncodeWarps * 32, 0, st>>>(A, blk0, nblk);
    else
      append_block_kernel<CQ_BF16><<<(unsigned)gb, kEncodeWarps * 32, 0, st>>>(A, blk0, nblk);
    return check_launch(who);
  }
  int64_t warps = 2LL * cache->batch * cache->kv_heads * S;
  int64_t blocks = (warps + kEncodeWarps - 1) / kEncodeWarps;
  CQ_REQUIRE(blocks < (1LL << 31), CQ_ERR_INVALID, std::string(who) + ": too many tokens in one call");
  if (dtype == CQ_F16)
    append_kernel<CQ_F16><<<(unsigned)blocks, kEncodeWarps * 32, 0, st>>>(A);
  else
    append_kernel<CQ_BF16><<<(unsigned)blocks, kEncodeWarps * 32, 0, st>>>(A);
  return check_launch(who);
}

// Read (and optionally clear) the append kernel's device error word.
int read_append_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_append_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_append_error, &z, sizeof(int));
  }
  return v;
}

int read_bounds_error_encode(int clear) { return read_bounds_error_here(clear); }

}  // namespace cq

using namespace cq;

extern "C" int cq_append(const cq_paged_cache *cache, const void *keys, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                         const void *values, int64_t v_sb, int64_t v_sh, int64_t v_ss, int dtype, int64_t t0,
                         int32_t S, void *stream) {
  return launch_append(cache, keys, k_sb, k_sh, k_ss, values, v_sb, v_sh, v_ss, dtype, t0, nullptr, S, stream,
                       "cq_append");
}

extern "C" int cq_append_at(const cq_paged_cache *cache, const void *keys, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                            const void *values, int64_t v_sb, int64_t v_sh, int64_t v_ss, int dtype, int64_t *len_dev,
                            int32_t S, void *stream) {
  CQ_REQUIRE(len_dev, CQ_ERR_INVALID, "cq_append_at: len_dev is null");
  return launch_append(cache, keys, k_sb, k_sh, k_ss, values, v_sb, v_sh, v_ss, dtype, 0, len_dev, S, stream,
                       "cq_append_at");
}
