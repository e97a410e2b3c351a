// cq_prefill.cu -- multi-token query chunks (chunked prefill) over the
// compressed cache on the sm_100a tensor cores.
//
// The reference answers a query chunk (q_len > 1) with its fallback path
// (attention.py:61-74): reconstruct the whole fp16 history (cache.py:131-160),
// then scores = q_scaled @ K^T, a causal mask aligned to the end of the keys
// (attention.py:8-20), softmax and weights @ V.  This file keeps that order
// with three kernels:
//
//   1. unpack_kernel   -- reconstructs K and V exactly as reconstruct_history
//      does (fp16 code*scale, then fp16 anchor + delta) into operand tile
//      images: per (sequence, kv-head, 128-key tile) one 32 KB image of K
//      (rows = keys, columns = head dims) and one of V transposed (rows = head
//      dims, columns = keys).
//   2. q_image_kernel  -- q * scale rounded to the query dtype (the reference's
//      q_scaled), as fp16, packed per (sequence, kv-head, query tile): the 128
//      rows of a tile are the GQA group's query heads x 128/G query tokens, so
//      one K/V tile serves every head of the group.
//   3. attn_kernel     -- flash attention over the images: tcgen05.mma computes
//      S = Q K^T and O += P V into tensor memory (fp16 operands, fp32
//      accumulation), one CTA per query tile, warp-specialised:
//        warps 0-3  softmax: one query row per thread (tensor-memory lane),
//                   base-2 online softmax with a lazy rescale of O, P as fp16
//                   into shared memory;
//        warp 4     copies: one bulk copy per 32 KB tile image into a 2-stage
//                   ring per operand (no multicast);
//        warp 5     MMA issue (one thread) and tensor-memory allocation.
//      S is double-buffered in tensor memory so the softmax of tile j overlaps
//      the MMAs of tiles j+1 (S) and j-1 (P V).
//
// An operand tile image is two 16 KB halves (64 columns each) of 128 rows x
// 128 bytes; the 16-byte chunk c of row r sits at position c ^ (r % 8) -- the
// 128-byte swizzle the tensor core's shared-memory descriptors read -- so one
// linear bulk copy into a 1024-byte aligned shared buffer gives an MMA
// operand with no bank conflicts.
//
// Every wait is bounded: on timeout the kernel records ERR_PREFILL_TIMEOUT in
// its device error word, lets its copies and MMAs in flight finish (bounded),
// frees its tensor memory and returns.
#include <algorithm>

#include "cq_common.cuh"
#include "cq_ptx.cuh"
#include "cq_tcgen05.cuh"

namespace cq {
namespace prefill {

constexpr int kTile = 128;          // keys per tile, query rows per tile, head_dim
constexpr int kImgBytes = 32768;    // one 128 x 128 fp16 tile image
constexpr int kHalfBytes = 16384;   // 64 columns x 128 rows
constexpr int kThreads = 192;       // 4 softmax warps, 1 copy warp, 1 MMA warp
constexpr int kMinRows = 16;        // shorter query chunks stay on the general kernel
constexpr uint32_t kTmemCols = 512; // S[0], S[1], O (128 columns each), rounded to a power of two
constexpr int kSmemTiles = 7 * kImgBytes;  // Q, K[2], V[2], P[2]
constexpr int kSmemBytes = kSmemTiles + 256 + 1024;  // + barriers, + alignment slack
constexpr long long kWaitBudget = 2000000000LL;      // clock cycles (about a second)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.f;  // log2 units: P stays <= 256 between rescales

__device__ int g_prefill_error;
constexpr int ERR_PREFILL_TIMEOUT = 6;

__device__ __forceinline__ float ptx_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// 1. unpack: grid (key tiles, B*H, 2 components), 256 threads
// ---------------------------------------------------------------------------
struct UnpackArgs {
  CacheView cv;
  int64_t T;
  int n_kt;
  uint8_t *img[2];  // K images, V^T images: [B*H][n_kt][32 KB]
};

__global__ void __launch_bounds__(256) unpack_kernel(UnpackArgs A) {
  // K: tile[key][dim]; V: tile[dim][key] (transposed while decoding); padded
  // rows (68 words) keep both the decode stores and the image reads spread
  // over the banks
  __shared__ __align__(16) __half tile[kTile][kTile + 8];
  __shared__ const __half *s_anchor[kTile];
  __shared__ const uint32_t *s_codes[kTile];
  __shared__ float s_scale[kTile];
  const int kt = blockIdx.x, bh = blockIdx.y, comp = blockIdx.z;
  const CacheView &cv = A.cv;
  const int b = bh / cv.H, h = bh - b * cv.H;
  const CompView &c = cv.c[comp];
  if (threadIdx.x < kTile) {
    const int r = threadIdx.x;
    const int64_t t = (int64_t)kt * kTile + r;
    const __half *an = nullptr;
    const uint32_t *cd = nullptr;
    float sc = 0.f;
    if (t < A.T) {
      const TokLoc L = locate(cv, comp, b, h, t);
      an = L.anchor;
      cd = L.codes;
      sc = L.scale;
    }
    s_anchor[r] = an;
    s_codes[r] = cd;
    s_scale[r] = sc;
  }
  __syncthreads();
  const bool natural = c.order != CQ_ORDER_MMA;
  // one item = (token, code word): the 8 dims whose nibbles share a u32
  for (int it = threadIdx.x; it < kTile * 16; it += 256) {
    const int r = it >> 4, w = it & 15;
    const __half *an = s_anchor[r];
    int dim[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) dim[j] = natural ? 8 * w + j : (w >> 1) + 64 * (w & 1) + 8 * j;
    __half v[8];
    if (an) {
      // reconstruct_history (cache.py:141-156): fp16(code) * scale in fp16, then anchor + that
      // in fp16.  I-frames read as code 0 with scale 0: anchor + (+0), which turns -0.0 into
      // +0.0 exactly as the reference's where(is_pframe, delta, 0) sum does.
      const uint32_t word = s_codes[r] ? s_codes[r][w] : 0x88888888u;
      const __half sh = __float2half_rn(s_scale[r]);
      __half a[8];
      if (natural && ((uintptr_t)(an + 8 * w) & 15) == 0) {
        *reinterpret_cast<uint4 *>(a) = *reinterpret_cast<const uint4 *>(an + 8 * w);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = an[dim[j]];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = __hadd_rn(a[j], __hmul_rn(__int2half_rn((int)((word >> (4 * j)) & 0xFu) - 8), sh));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __float2half_rn(0.f);
    }
    if (comp == 0 && natural) {
      *reinterpret_cast<uint4 *>(&tile[r][8 * w]) = *reinterpret_cast<const uint4 *>(v);
    } else if (comp == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) tile[r][dim[j]] = v[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) tile[dim[j]][r] = v[j];
    }
  }
  __syncthreads();
  // the image: chunk `ch` holds row `row`, columns col0..col0+7 (row = key for K, head dim for V)
  uint8_t *dst = A.img[comp] + ((int64_t)bh * A.n_kt + kt) * kImgBytes;
  for (int ch = threadIdx.x; ch < kImgBytes / 16; ch += 256) {
    const int half = ch >> 10, row = (ch >> 3) & 127, pos = ch & 7;
    const int col0 = half * 64 + ((pos ^ (row & 7)) << 3);
    *reinterpret_cast<uint4 *>(dst + (int64_t)ch * 16) = *reinterpret_cast<const uint4 *>(&tile[row][col0]);
  }
}

// ---------------------------------------------------------------------------
// 2. query images: grid (query tiles, B*Hkv), 256 threads
// ---------------------------------------------------------------------------
struct QArgs {
  const void *q;
  int q_dtype;
  int64_t sb, sh, sq;
  int Hkv, G, TQ, q_len, n_qt;
  float scale;  // the softmax scale rounded to the query dtype
  uint8_t *img; // [B*Hkv][n_qt][32 KB]
};

__global__ void __launch_bounds__(256) q_image_kernel(QArgs A) {
  const int qt = blockIdx.x, bh = blockIdx.y;
  const int b = bh / A.Hkv, h = bh - b * A.Hkv;
  uint8_t *dst = A.img + ((int64_t)bh * A.n_qt + qt) * kImgBytes;
  for (int ch = threadIdx.x; ch < kImgBytes / 16; ch += 256) {
    const int half = ch >> 10, row = (ch >> 3) & 127, pos = ch & 7;
    const int d0 = half * 64 + ((pos ^ (row & 7)) << 3);
    const int g = row / A.TQ, i = row - g * A.TQ;
    const int tok = qt * A.TQ + i;
    __half e[8];
    if (tok < A.q_len) {
      const int64_t base = (int64_t)b * A.sb + (int64_t)(h * A.G + g) * A.sh + (int64_t)tok * A.sq + d0;
      const uint16_t *src = (const uint16_t *)A.q + base;
      uint16_t raw[8];
      if (((uintptr_t)src & 15) == 0) {
        *reinterpret_cast<uint4 *>(raw) = *reinterpret_cast<const uint4 *>(src);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) raw[j] = src[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // q_scaled = queries * scale in the query dtype (attention.py:65), then fp16
        const float x = A.q_dtype == CQ_BF16 ? __bfloat162float(__ushort_as_bfloat16(raw[j]))
                                             : __half2float(__ushort_as_half(raw[j]));
        e[j] = __float2half_rn(round_dt(x * A.scale, A.q_dtype));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = __float2half_rn(0.f);
    }
    *reinterpret_cast<uint4 *>(dst + (int64_t)ch * 16) = *reinterpret_cast<const uint4 *>(e);
  }
}

// ---------------------------------------------------------------------------
// 3. attention
// ---------------------------------------------------------------------------
struct AttnParams {
  const uint8_t *kimg, *vimg, *qimg;
  int n_kt;  // key tiles per (b, h) in the images
  int64_t T;
  int q_len, G, TQ, n_qt, Hkv, Hq, causal;
  void *out;
  int out_dtype;
  float *lse;
};

// barrier slots
enum {
  BQ = 0,
  BKF = 1,   // [2] K tile landed
  BKE = 3,   // [2] K slot free (S MMA done)
  BVF = 5,   // [2] V tile landed
  BVE = 7,   // [2] V slot free (PV MMA done)
  BSF = 9,   // [2] S ready in tensor memory
  BSE = 11,  // [2] S read by all softmax threads
  BPF = 13,  // [2] P written by all softmax threads
  BPV = 15,  // [2] PV MMA of the tile done (O stable, P slot free)
  BDR = 17,  // drain: every MMA of the CTA done
  NBARS = 18
};

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (ptx::mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitBudget) {
      *abort_flag = 1;
      atomicExch(&g_prefill_error, ERR_PREFILL_TIMEOUT);
      return false;
    }
  }
}

// softmax warps: a wait that fails in any lane fails in the whole warp, so the
// warp-collective tensor-memory loads and stores stay convergent
__device__ __forceinline__ bool wait_rows(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  return __all_sync(0xffffffffu, wait_bar(bar, parity, abort_flag));
}

__device__ __forceinline__ void sts_u128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

__global__ void __launch_bounds__(kThreads, 1) attn_kernel(AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem_raw + NBARS * 8);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem_raw + NBARS * 8 + 4);
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t sbase = (raw + 256 + 1023) & ~1023u;  // 1024-byte aligned tile images
  const uint32_t sQ = sbase;
  auto sK = [&](int s) { return sbase + (uint32_t)(1 + s) * kImgBytes; };
  auto sV = [&](int s) { return sbase + (uint32_t)(3 + s) * kImgBytes; };
  auto sP = [&](int s) { return sbase + (uint32_t)(5 + s) * kImgBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x % p.n_qt;
  const int bh = blockIdx.x / p.n_qt;
  const int b = bh / p.Hkv, h = bh - b * p.Hkv;
  const int q0 = qt * p.TQ;
  const int qlast = min(q0 + p.TQ, p.q_len) - 1;
  const int64_t off = p.T - p.q_len;  // absolute position of query token 0
  const int64_t kend = p.causal ? (off + qlast + 1) : p.T;
  const int n = (int)((kend + kTile - 1) / kTile);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NBARS; ++i) {
      const bool by_rows = (i == BSE || i == BSE + 1 || i == BPF || i == BPF + 1);
      ptx::mbar_init(&bars[i], by_rows ? 128u : 1u);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 5) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS0 = tbase, tO = tbase + 256;

  if (warp == 4) {
    // ---------------------------------------------------------------- copies
    if (lane == 0) {
      const uint8_t *kimg = p.kimg + (int64_t)bh * p.n_kt * kImgBytes;
      const uint8_t *vimg = p.vimg + (int64_t)bh * p.n_kt * kImgBytes;
      ptx::mbar_arrive_expect_tx(&bars[BQ], kImgBytes);
      ptx::bulk_g2s_a(sQ, p.qimg + ((int64_t)bh * p.n_qt + qt) * kImgBytes, kImgBytes, &bars[BQ]);
      int nk = 0, nv = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (j >= 2 && !wait_bar(&bars[BKE + s], ph ^ 1, abort_flag)) break;
        ptx::mbar_arrive_expect_tx(&bars[BKF + s], kImgBytes);
        ptx::bulk_g2s_a(sK(s), kimg + (int64_t)j * kImgBytes, kImgBytes, &bars[BKF + s]);
        ++nk;
        if (j >= 2 && !wait_bar(&bars[BVE + s], ph ^ 1, abort_flag)) break;
        ptx::mbar_arrive_expect_tx(&bars[BVF + s], kImgBytes);
        ptx::bulk_g2s_a(sV(s), vimg + (int64_t)j * kImgBytes, kImgBytes, &bars[BVF + s]);
        ++nv;
      }
      // copies still in flight must land before the CTA's shared memory is released
      ptx::mbar_wait_bounded(&bars[BQ], 0, kWaitBudget);
      for (int i = std::max(0, nk - 2); i < nk; ++i) ptx::mbar_wait_bounded(&bars[BKF + (i & 1)], (i >> 1) & 1, kWaitBudget);
      for (int i = std::max(0, nv - 2); i < nv; ++i) ptx::mbar_wait_bounded(&bars[BVF + (i & 1)], (i >> 1) & 1, kWaitBudget);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(128, 128);
      bool ok = wait_bar(&bars[BQ], 0, abort_flag);
      auto pv = [&](int i) -> bool {
        const int s = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!wait_bar(&bars[BPF + s], ph, abort_flag)) return false;
        if (!wait_bar(&bars[BVF + s], ph, abort_flag)) return false;
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ko = (uint32_t)(k >> 2) * kHalfBytes + (uint32_t)(k & 3) * 32;
          tc::mma_f16_ss(tO, tc::desc_sw128(sP(s) + ko), tc::desc_sw128(sV(s) + ko), idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        tc::commit(&bars[BPV + s]);
        tc::commit(&bars[BVE + s]);
        return true;
      };
      for (int j = 0; ok && j < n; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!wait_bar(&bars[BKF + s], ph, abort_flag)) break;
        if (j >= 2 && !wait_bar(&bars[BSE + s], ph ^ 1, abort_flag)) break;
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ko = (uint32_t)(k >> 2) * kHalfBytes + (uint32_t)(k & 3) * 32;
          tc::mma_f16_ss(tS0 + (uint32_t)s * 128, tc::desc_sw128(sQ + ko), tc::desc_sw128(sK(s) + ko), idesc,
                         k > 0 ? 1u : 0u);
        }
        tc::commit(&bars[BSF + s]);
        tc::commit(&bars[BKE + s]);
        if (j >= 1 && !pv(j - 1)) {
          ok = false;
          break;
        }
        if (j == n - 1) ok = pv(j);
      }
      // every MMA issued by this thread completes before tensor memory and shared memory are released
      tc::commit(&bars[BDR]);
      ptx::mbar_wait_bounded(&bars[BDR], 0, kWaitBudget);
    }
  } else {
    // ---------------------------------------------------------------- softmax (one row per thread)
    const int r = threadIdx.x;  // 0..127 = tensor-memory lane = query row of the tile
    const int g = r / p.TQ, i = r - g * p.TQ;
    const int64_t lim = p.causal ? std::min(off + q0 + i + 1, p.T) : p.T;  // keys < lim are visible
    const uint32_t trow = (uint32_t)(warp * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!wait_rows(&bars[BSF + s], ph, abort_flag)) {
        ok = false;
        break;
      }
      tc::fence_after();
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::ld_32x32b_x32(tS0 + trow + (uint32_t)(s * 128 + c * 32), v[c]);
      tc::wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::after_wait(v[c]);
      tc::fence_before();
      ptx::mbar_arrive(&bars[BSE + s]);

      const int64_t k0 = (int64_t)j * kTile;
      if (k0 + kTile > lim) {  // causal edge or keys past T
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (k0 + c >= lim) v[c >> 5][c & 31] = __float_as_uint(-INFINITY);
      }
      // row max as a tree over 8 independent partial maxima (one thread owns the row)
      float pm[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) pm[t] = __uint_as_float(v[0][t]);
#pragma unroll
      for (int c = 8; c < 128; ++c) pm[c & 7] = fmaxf(pm[c & 7], __uint_as_float(v[c >> 5][c & 31]));
      const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) * kLog2e;
      if (mx > m + kRescaleThreshold) {
        const float f = ptx_exp2(m - mx);  // 0 while m = -inf
        if (j > 0) {
          // O holds tiles 0..j-1 at the old base: wait for the last PV, rescale in place
          if (!wait_rows(&bars[BPV + ((j - 1) & 1)], ((j - 1) >> 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc::fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tc::ld_32x32b_x32(tO + trow + (uint32_t)(c * 32), o);
            tc::wait_ld();
            tc::after_wait(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tc::st_32x32b_x32(tO + trow + (uint32_t)(c * 32), o);
          }
          tc::wait_st();
        }
        l *= f;
        m = mx;
      }
      // P slot s is free once the PV MMA of tile j-2 is done
      if (j >= 2 && !wait_rows(&bars[BPV + s], ph ^ 1, abort_flag)) {
        ok = false;
        break;
      }
      const uint32_t prow = sP(s) + (uint32_t)r * 128;
      float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // 8 independent partial row sums
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
        for (int kc = 0; kc < 8; ++kc) {
          float e[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const int c = hf * 64 + kc * 8 + t;
            e[t] = ptx_exp2(fmaf(__uint_as_float(v[c >> 5][c & 31]), kLog2e, -m));
            ps[t] += e[t];
          }
          sts_u128(prow + (uint32_t)hf * kHalfBytes + (uint32_t)((kc ^ (r & 7)) << 4), pack_h2(e[0], e[1]),
                   pack_h2(e[2], e[3]), pack_h2(e[4], e[5]), pack_h2(e[6], e[7]));
        }
      }
      l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      ptx::fence_proxy_async_smem();
      tc::fence_before();
      ptx::mbar_arrive(&bars[BPF + s]);
    }
    // ---------------------------------------------------------------- epilogue
    if (ok && wait_rows(&bars[BPV + ((n - 1) & 1)], ((n - 1) >> 1) & 1, abort_flag)) {
      tc::fence_after();
      const int tok = q0 + i;
      const bool live = tok < p.q_len;
      const int hq = h * p.G + g;
      const int64_t row = ((int64_t)b * p.Hq + hq) * p.q_len + tok;
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tc::ld_32x32b_x32(tO + trow + (uint32_t)(c * 32), o);
        tc::wait_ld();
        tc::after_wait(o);
        if (live) {
          if (p.out_dtype == CQ_F32) {
            float4 *dst = reinterpret_cast<float4 *>((float *)p.out + row * kTile + c * 32);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              dst[e] = make_float4(__uint_as_float(o[4 * e]) * inv, __uint_as_float(o[4 * e + 1]) * inv,
                                   __uint_as_float(o[4 * e + 2]) * inv, __uint_as_float(o[4 * e + 3]) * inv);
          } else {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float a = __uint_as_float(o[2 * e]) * inv, bb = __uint_as_float(o[2 * e + 1]) * inv;
              if (p.out_dtype == CQ_F16) {
                __half2 hv = __floats2half2_rn(a, bb);
                w[e] = *reinterpret_cast<uint32_t *>(&hv);
              } else {
                __nv_bfloat162 bv = __floats2bfloat162_rn(a, bb);
                w[e] = *reinterpret_cast<uint32_t *>(&bv);
              }
            }
            uint4 *dst = reinterpret_cast<uint4 *>((uint16_t *)p.out + row * kTile + c * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
          }
        }
      }
      if (live && p.lse) p.lse[row] = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : -INFINITY;
    }
  }

  tc::fence_before();
  __syncthreads();
  if (warp == 5) {
    tc::fence_after();
    tc::tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace prefill

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using namespace prefill;

bool prefill_supported(const cq_paged_cache &c, int n_q_heads, int q_len) {
  if (c.head_dim != kTile || q_len < kMinRows) return false;
  const int G = n_q_heads / c.kv_heads;
  return G >= 1 && G <= 16 && (G & (G - 1)) == 0;
}

static void prefill_shape(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int &n_kt, int &TQ,
                          int &n_qt) {
  const int G = n_q_heads / c.kv_heads;
  n_kt = (int)((T + kTile - 1) / kTile);
  TQ = kTile / G;
  n_qt = (q_len + TQ - 1) / TQ;
}

size_t prefill_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len) {
  if (!prefill_supported(c, n_q_heads, q_len)) return 0;
  int n_kt, TQ, n_qt;
  prefill_shape(c, T, n_q_heads, q_len, n_kt, TQ, n_qt);
  const size_t units = (size_t)c.batch * c.kv_heads;
  return units * (2 * (size_t)n_kt + (size_t)n_qt) * kImgBytes;
}

struct Plan {
  int n_kt, TQ, n_qt, units;
  uint8_t *kimg, *vimg, *qimg;
};

static int make_plan(const cq_paged_cache &cache, int64_t T, int Hq, int q_len, void *ws, size_t ws_bytes, Plan &pl) {
  CQ_REQUIRE(prefill_supported(cache, Hq, q_len), CQ_ERR_UNSUPPORTED,
             "query-chunk path: needs head_dim 128, q_len >= 16 and a GQA group that is a power of two <= 16");
  prefill_shape(cache, T, Hq, q_len, pl.n_kt, pl.TQ, pl.n_qt);
  const size_t need = prefill_workspace(cache, T, Hq, q_len);
  CQ_REQUIRE(ws && ws_bytes >= need, CQ_ERR_WORKSPACE, "cq_attention: workspace too small");
  CQ_REQUIRE(((uintptr_t)ws & 15) == 0, CQ_ERR_INVALID, "cq_attention: workspace must be 16-byte aligned for query chunks");
  pl.units = cache.batch * cache.kv_heads;
  CQ_REQUIRE((int64_t)pl.units * pl.n_qt < (1LL << 31), CQ_ERR_INVALID, "cq_attention: grid too large");
  pl.kimg = (uint8_t *)ws;
  pl.vimg = pl.kimg + (size_t)pl.units * pl.n_kt * kImgBytes;
  pl.qimg = pl.vimg + (size_t)pl.units * pl.n_kt * kImgBytes;
  return CQ_OK;
}

int prefill_prepare(const cq_paged_cache &cache, const CacheView &cv, int64_t T, const void *q, int q_dtype, int Hq,
                    int q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, void *ws, size_t ws_bytes,
                    cudaStream_t st) {
  Plan pl;
  int r = make_plan(cache, T, Hq, q_len, ws, ws_bytes, pl);
  if (r) return r;
  UnpackArgs U;
  U.cv = cv;
  U.T = T;
  U.n_kt = pl.n_kt;
  U.img[0] = pl.kimg;
  U.img[1] = pl.vimg;
  unpack_kernel<<<dim3((unsigned)pl.n_kt, (unsigned)pl.units, 2), 256, 0, st>>>(U);
  r = check_launch("prefill unpack_kernel");
  if (r) return r;

  QArgs Q;
  Q.q = q;
  Q.q_dtype = q_dtype;
  Q.sb = q_sb;
  Q.sh = q_sh;
  Q.sq = q_sq;
  Q.Hkv = cache.kv_heads;
  Q.G = Hq / cache.kv_heads;
  Q.TQ = pl.TQ;
  Q.q_len = q_len;
  Q.n_qt = pl.n_qt;
  // the scale is a weakly typed Python float: it multiplies in the query dtype
  Q.scale = (q_dtype == CQ_BF16) ? __bfloat162float(__float2bfloat16_rn(scale)) : __half2float(__float2half_rn(scale));
  Q.img = pl.qimg;
  q_image_kernel<<<dim3((unsigned)pl.n_qt, (unsigned)pl.units), 256, 0, st>>>(Q);
  return check_launch("prefill q_image_kernel");
}

int prefill_attend(const cq_paged_cache &cache, int64_t T, int Hq, int q_len, bool causal, void *out, int out_dtype,
                   float *lse_out, void *ws, size_t ws_bytes, cudaStream_t st) {
  Plan pl;
  int r = make_plan(cache, T, Hq, q_len, ws, ws_bytes, pl);
  if (r) return r;
  CQ_REQUIRE(((uintptr_t)out & 15) == 0, CQ_ERR_INVALID, "cq_attention: out must be 16-byte aligned for query chunks");
  AttnParams P;
  P.kimg = pl.kimg;
  P.vimg = pl.vimg;
  P.qimg = pl.qimg;
  P.n_kt = pl.n_kt;
  P.T = T;
  P.q_len = q_len;
  P.G = Hq / cache.kv_heads;
  P.TQ = pl.TQ;
  P.n_qt = pl.n_qt;
  P.Hkv = cache.kv_heads;
  P.Hq = Hq;
  P.causal = causal ? 1 : 0;
  P.out = out;
  P.out_dtype = out_dtype;
  P.lse = lse_out;
  cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return set_error(CQ_ERR_CUDA, std::string("prefill attn_kernel smem: ") + cudaGetErrorString(e));
  attn_kernel<<<(unsigned)(pl.units * pl.n_qt), kThreads, kSmemBytes, st>>>(P);
  return check_launch("prefill attn_kernel");
}

int run_prefill(const cq_paged_cache &cache, const CacheView &cv, int64_t T, const void *q, int q_dtype, int Hq,
                int q_len, int64_t q_sb, int64_t q_sh, int64_t q_sq, float scale, void *out, int out_dtype,
                float *lse_out, void *ws, size_t ws_bytes, bool causal, cudaStream_t st) {
  int r = prefill_prepare(cache, cv, T, q, q_dtype, Hq, q_len, q_sb, q_sh, q_sq, scale, ws, ws_bytes, st);
  if (r) return r;
  return prefill_attend(cache, T, Hq, q_len, causal, out, out_dtype, lse_out, ws, ws_bytes, st);
}

int read_prefill_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_prefill_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_prefill_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace cq
