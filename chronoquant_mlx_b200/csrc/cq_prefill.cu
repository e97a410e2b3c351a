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
//      accumulation).  One CTA takes a pair of query tiles (a, b) that read
//      the same K/V tiles, warp-specialised:
//        warps 0-3, 4-7  softmax of tile a, tile b: one query row per thread
//                   (tensor-memory lane), base-2 online softmax with a lazy
//                   rescale of O; P as fp16 into tensor memory over its own
//                   S columns, read there by the PV MMA;
//        warp 8     copies: one bulk copy per 32 KB tile image into a 5-slot
//                   K/V ring (each CTA loads its own tiles);
//        warp 9     MMA issue (one thread) and tensor-memory allocation.
//      The MMAs alternate between the tiles (PV_a, S_a, PV_b, S_b per key
//      tile), so one tile's softmax runs while the tensor core works for the
//      other, and each scheduler holds two softmax warps.
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
#include "cq_prefill.cuh"
#include "cq_ptx.cuh"
#include "cq_tcgen05.cuh"

namespace cq {
namespace prefill {

constexpr int kTile = 128;          // keys per tile, query rows per tile, head_dim
constexpr int kImgBytes = 32768;    // one 128 x 128 fp16 tile image
constexpr int kHalfBytes = 16384;   // 64 columns x 128 rows
constexpr int kThreads = 320;       // 2 x 4 softmax warps, 1 copy warp, 1 MMA warp
constexpr int kMinRows = 16;        // shorter query chunks stay on the general kernel
constexpr uint32_t kTmemCols = 512; // S_a, S_b, O_a, O_b (128 columns each)
constexpr int kRing = 5;            // K/V tile ring slots
constexpr int kSmemTiles = (2 + kRing) * kImgBytes;  // Q_a, Q_b, ring
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
  // key-range splits of each pair (whole waves of CTAs): with splits > 1 each
  // CTA writes its partial (m natural-log, l, unnormalised O) per row and split
  int splits;
  float *ws_m, *ws_l, *ws_o;
};

// barrier slots
enum {
  BQ = 0,                // both query tiles landed
  BFULL = 1,             // [kRing] ring slot landed
  BEMPTY = BFULL + kRing,  // [kRing] ring slot free (every MMA reading it done)
  BSF = BEMPTY + kRing,  // [2] S of query tile t ready in tensor memory
  BPF = BSF + 2,         // [2] P of query tile t written (over S_t) by its 128 softmax threads
  BPH = BPF + 2,         // [2] the first half of P_t (keys 0-63) written, O_t rescaled if needed
  BPV = BPH + 2,         // [2] PV MMA of query tile t done (O_t stable)
  BDR = BPV + 2,         // drain: every MMA of the CTA done
  NBARS = BDR + 1
};
static_assert(NBARS * 8 + 8 <= 256, "barriers, tensor-memory slot and abort flag fit in front of the tiles");

// Polls with try_wait (no suspend-time hint: a hinted wait woke hundreds of
// cycles after the phase completed, on the critical path of every key tile).
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(bar, parity)) return true;
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

// Packed fp32 pairs (sm_100 f32x2 arithmetic): one instruction for two lanes
// of a softmax row.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
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
  auto sQ = [&](int t) { return sbase + (uint32_t)t * kImgBytes; };        // query tiles a, b
  auto sR = [&](int L) { return sbase + (uint32_t)(2 + L % kRing) * kImgBytes; };  // ring slot of load L

  // one CTA = a pair of query tiles (2*TQ tokens) of one (sequence, kv-head):
  // both read the same K/V tiles
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_pairs = p.n_qt >> 1;
  const int split = blockIdx.x % p.splits;
  const int pr = (blockIdx.x / p.splits) % n_pairs;
  const int bh = blockIdx.x / p.splits / n_pairs;
  const int b = bh / p.Hkv, h = bh - b * p.Hkv;
  const int q0 = pr * 2 * p.TQ;  // first query token of tile a; tile b starts at q0 + TQ
  const int qlast = min(q0 + 2 * p.TQ, p.q_len) - 1;
  const int64_t off = p.T - p.q_len;  // absolute position of query token 0
  const int64_t kend = p.causal ? (off + qlast + 1) : p.T;
  const int n_all = (int)((kend + kTile - 1) / kTile);
  const int j0 = (int)((int64_t)split * n_all / p.splits);  // this CTA's key tiles: j0 .. j0+n-1
  const int n = (int)((int64_t)(split + 1) * n_all / p.splits) - j0;
  // loads in ring order: K_j is load 2j, V_j is load 2j+1
  auto full_parity = [](int L) { return (uint32_t)((L / kRing) & 1); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < NBARS; ++i) ptx::mbar_init(&bars[i], (i >= BPF && i < BPF + 4) ? 128u : 1u);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 9) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tbase = *tmem_slot;
  auto tS = [&](int t) { return tbase + (uint32_t)t * 128; };
  auto tO = [&](int t) { return tbase + 256 + (uint32_t)t * 128; };

  if (warp == 8) {
    // ---------------------------------------------------------------- copies
    if (lane == 0 && n > 0) {
      const uint8_t *kimg = p.kimg + ((int64_t)bh * p.n_kt + j0) * kImgBytes;
      const uint8_t *vimg = p.vimg + ((int64_t)bh * p.n_kt + j0) * kImgBytes;
      ptx::mbar_arrive_expect_tx(&bars[BQ], 2 * kImgBytes);  // the pair's two query tiles are adjacent
      ptx::bulk_g2s_a(sQ(0), p.qimg + ((int64_t)bh * p.n_qt + 2 * pr) * kImgBytes, 2 * kImgBytes, &bars[BQ]);
      int issued = 0;
      for (int L = 0; L < 2 * n; ++L) {
        const int slot = L % kRing;
        if (L >= kRing && !wait_bar(&bars[BEMPTY + slot], full_parity(L - kRing), abort_flag)) break;
        ptx::mbar_arrive_expect_tx(&bars[BFULL + slot], kImgBytes);
        ptx::bulk_g2s_a(sR(L), ((L & 1) ? vimg : kimg) + (int64_t)(L >> 1) * kImgBytes, kImgBytes,
                        &bars[BFULL + slot]);
        ++issued;
      }
      // copies still in flight must land before the CTA's shared memory is released
      ptx::mbar_wait_bounded(&bars[BQ], 0, kWaitBudget);
      for (int L = std::max(0, issued - kRing); L < issued; ++L)
        ptx::mbar_wait_bounded(&bars[BFULL + L % kRing], full_parity(L), kWaitBudget);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issue
    // order: S_a(0) S_b(0) | PV_a(j) S_a(j+1) PV_b(j) S_b(j+1) | ... so that the
    // softmax of one tile runs while the tensor core works on the other's
    if (lane == 0 && n > 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(128, 128);
      auto landed = [&](int L) { return wait_bar(&bars[BFULL + L % kRing], full_parity(L), abort_flag); };
      auto mma_s = [&](int t, int L) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ko = (uint32_t)(k >> 2) * kHalfBytes + (uint32_t)(k & 3) * 32;
          tc::mma_f16_ss(tS(t), tc::desc_sw128(sQ(t) + ko), tc::desc_sw128(sR(L) + ko), idesc, k > 0 ? 1u : 0u);
        }
      };
      auto mma_pv = [&](int t, int j, int L, int half) {  // P_t from tensor memory (columns 0-63 of S_t)
#pragma unroll
        for (int k = 4 * half; k < 4 * half + 4; ++k) {
          const uint32_t ko = (uint32_t)(k >> 2) * kHalfBytes + (uint32_t)(k & 3) * 32;
          tc::mma_f16_ts(tO(t), tS(t) + (uint32_t)k * 8, tc::desc_sw128(sR(L) + ko), idesc,
                         (j > 0 || k > 0) ? 1u : 0u);
        }
      };
      bool ok = wait_bar(&bars[BQ], 0, abort_flag) && landed(0);
      if (ok) {
        tc::fence_after();
        mma_s(0, 0);
        tc::commit(&bars[BSF + 0]);
        mma_s(1, 0);
        tc::commit(&bars[BSF + 1]);
        tc::commit(&bars[BEMPTY + 0]);
      }
      for (int j = 0; ok && j < n; ++j) {
        const int Lv = 2 * j + 1, Lk = 2 * j + 2;
        const bool more = j + 1 < n;
        // each PV in two halves of its keys: the first as soon as that half of P is written
        if (!wait_bar(&bars[BPH + 0], j & 1, abort_flag) || !landed(Lv)) break;
        tc::fence_after();
        mma_pv(0, j, Lv, 0);
        if (!wait_bar(&bars[BPF + 0], j & 1, abort_flag)) break;
        tc::fence_after();
        mma_pv(0, j, Lv, 1);
        tc::commit(&bars[BPV + 0]);
        if (more) {
          if (!landed(Lk)) break;
          tc::fence_after();
          mma_s(0, Lk);
          tc::commit(&bars[BSF + 0]);
        }
        if (!wait_bar(&bars[BPH + 1], j & 1, abort_flag)) break;
        tc::fence_after();
        mma_pv(1, j, Lv, 0);
        if (!wait_bar(&bars[BPF + 1], j & 1, abort_flag)) break;
        tc::fence_after();
        mma_pv(1, j, Lv, 1);
        tc::commit(&bars[BPV + 1]);
        tc::commit(&bars[BEMPTY + Lv % kRing]);
        if (more) {
          mma_s(1, Lk);
          tc::commit(&bars[BSF + 1]);
          tc::commit(&bars[BEMPTY + Lk % kRing]);
        }
      }
      // every MMA issued by this thread completes before tensor memory and shared memory are released
      tc::commit(&bars[BDR]);
      ptx::mbar_wait_bounded(&bars[BDR], 0, kWaitBudget);
    }
  } else {
    // ---------------------------------------------------------------- softmax (one row per thread)
    const int t = warp >> 2;            // query tile: warps 0-3 -> a, 4-7 -> b
    const int r = threadIdx.x & 127;    // tensor-memory lane = query row of the tile
    const int g = r / p.TQ, i = r - g * p.TQ;
    const int tok = q0 + t * p.TQ + i;  // query token of the row
    const int64_t lim = p.causal ? std::min(off + tok + 1, p.T) : p.T;  // keys < lim are visible
    const uint32_t trow = (uint32_t)((warp & 3) * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!wait_rows(&bars[BSF + t], j & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc::fence_after();
      const int64_t k0 = (int64_t)(j0 + j) * kTile;
      const bool edge = k0 + kTile > lim;  // causal edge or keys past T
      // Two passes over S_t: the row max (all 128 columns in one tensor-memory round
      // trip), then the exponentials 32 columns at a time (registers for P stay free).
      // row max as a tree over 8 independent partial maxima (one thread owns the row)
      float pm[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pm[u] = -INFINITY;
      {  // the whole row in one tensor-memory round trip (its registers are free again for pass 2)
        uint32_t v4[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::ld_32x32b_x32(tS(t) + trow + (uint32_t)(c * 32), v4[c]);
        tc::wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::after_wait(v4[c]);
        if (edge) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (k0 + c >= lim) v4[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c = 0; c < 64; ++c)
          pm[c & 7] = fmaxf(pm[c & 7], fmaxf(__uint_as_float(v4[c >> 5][c & 31]),
                                             __uint_as_float(v4[(c + 64) >> 5][(c + 64) & 31])));
      }
      const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) * kLog2e;
      float f = 1.f;  // rescale of O and l when the running max moves up by more than the threshold
      const bool rescale = mx > m + kRescaleThreshold;
      if (rescale) {
        f = ptx_exp2(m - mx);  // 0 while m = -inf
        l *= f;
        m = mx;
      }
      if (rescale && j > 0) {
        // O holds tiles 0..j-1 at the old base: once their last PV is done, scale it in
        // place (before the first half of P_t(j) is released, so before PV_t(j) starts)
        if (!wait_rows(&bars[BPV + t], (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc::fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tc::ld_32x32b_x32(tO(t) + trow + (uint32_t)(c * 32), o);
          tc::wait_ld();
          tc::after_wait(o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tc::st_32x32b_x32(tO(t) + trow + (uint32_t)(c * 32), o);
        }
      }
      // P_t (fp16 pairs) goes over columns 0-63 of S_t: half hf is written to
      // columns 32*hf.., inside the columns already read, and released on its own
      // (BPH, then BPF) so that the first half of PV_t(j) runs while the second
      // half of P is computed.  The PV MMA of key tile j-1 read the previous P_t
      // there before S_t(j) overwrote it: MMAs complete in issue order.
      const uint32_t tP = tS(t) + trow;
      // while no key of the row has been visible (m = -inf), every score is -inf and P is 0
      const float nm = (m == -INFINITY) ? 0.f : -m;
      const uint64_t l2e2 = f2_pack(kLog2e, kLog2e), nm2 = f2_pack(nm, nm);
      uint64_t ps[4] = {0ull, 0ull, 0ull, 0ull};  // 4 independent pair partial sums
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t w[32];
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {  // 32 columns at a time: no register spills
          uint32_t va[32];
          tc::ld_32x32b_x32(tS(t) + trow + (uint32_t)(hf * 64 + sub * 32), va);
          tc::wait_ld();
          tc::after_wait(va);
          if (edge) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (k0 + hf * 64 + sub * 32 + c >= lim) va[c] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int q = sub * 16; q < sub * 16 + 16; ++q) {
            const int c = (2 * q) & 31;
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(va[c]), __uint_as_float(va[c + 1])), l2e2, nm2), x0, x1);
            const float e0 = ptx_exp2(x0), e1 = ptx_exp2(x1);
            ps[q & 3] = f2_add(ps[q & 3], f2_pack(e0, e1));
            w[q] = pack_h2(e0, e1);
          }
        }
        tc::st_32x32b_x32(tP + (uint32_t)(hf * 32), w);
        tc::wait_st();
        tc::fence_before();
        ptx::mbar_arrive(&bars[(hf == 0 ? BPH : BPF) + t]);
      }
      float s0, s1, s2, s3;
      f2_unpack(f2_add(ps[0], ps[1]), s0, s1);
      f2_unpack(f2_add(ps[2], ps[3]), s2, s3);
      l += (s0 + s1) + (s2 + s3);
    }
    // ---------------------------------------------------------------- epilogue
    const bool live = tok < p.q_len;
    const int hq = h * p.G + g;
    const int64_t row = ((int64_t)b * p.Hq + hq) * p.q_len + tok;
    const int64_t prow = row * p.splits + split;  // partial slot of this row and split
    if (n == 0) {  // an empty key range: a partial with no mass
      if (live) {
        p.ws_m[prow] = -INFINITY;
        p.ws_l[prow] = 0.f;
      }
    } else if (ok && wait_rows(&bars[BPV + t], (n - 1) & 1, abort_flag)) {
      tc::fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tc::ld_32x32b_x32(tO(t) + trow + (uint32_t)(c * 32), o);
        tc::wait_ld();
        tc::after_wait(o);
        if (live && p.splits > 1) {
          float4 *dst = reinterpret_cast<float4 *>(p.ws_o + prow * kTile + c * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dst[e] = make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                                 __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
        } else if (live) {
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
      if (live && p.splits > 1) {
        p.ws_m[prow] = (m == -INFINITY) ? -INFINITY : m * 0.6931471805599453f;
        p.ws_l[prow] = l;
      } else if (live && p.lse) {
        p.lse[row] = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : -INFINITY;
      }
    }
  }

  tc::fence_before();
  __syncthreads();
  if (warp == 9) {
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
  // the tile images are built from INT4-lane code rows; bit-plane rows take the general kernel
  for (int o : {c.k.code_order, c.v.code_order})
    if (o == CQ_ORDER_PLANES3 || o == CQ_ORDER_PLANES2) return false;
  const int G = n_q_heads / c.kv_heads;
  return G >= 1 && G <= 16 && (G & (G - 1)) == 0;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    n = 0;
  return n > 0 ? n : 148;
}

struct Shape {
  int n_kt, TQ, n_qt, splits;
  int64_t rows;  // output rows B * Hq * q_len
};

// Tile counts, and the number of key-range splits per query-tile pair: the
// count (1..8, at least 4 key tiles each) whose CTAs fill whole waves of SMs
// best, each extra split charged 1.5 % for its pipeline fill and merge.
static Shape prefill_shape(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len) {
  Shape sh;
  const int G = n_q_heads / c.kv_heads;
  sh.n_kt = (int)((T + kTile - 1) / kTile);
  sh.TQ = kTile / G;
  sh.n_qt = ((q_len + sh.TQ - 1) / sh.TQ + 1) & ~1;  // whole pairs: the tail tile of an odd count is all padding
  sh.rows = (int64_t)c.batch * n_q_heads * q_len;
  const int64_t pairs = (int64_t)c.batch * c.kv_heads * (sh.n_qt / 2);
  const int nsm = sm_count();
  sh.splits = 1;
  double best = (double)((pairs + nsm - 1) / nsm);
  for (int s = 2; s <= 8 && sh.n_kt / s >= 4; ++s) {
    const double cost = (double)((pairs * s + nsm - 1) / nsm) / s * (1.0 + 0.015 * (s - 1));
    if (cost < best - 1e-9) {
      best = cost;
      sh.splits = s;
    }
  }
  return sh;
}

static size_t partial_bytes(const Shape &sh) {
  return sh.splits > 1 ? (size_t)sh.rows * sh.splits * (2 + kTile) * sizeof(float) : 0;
}

size_t prefill_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len) {
  if (!prefill_supported(c, n_q_heads, q_len)) return 0;
  const Shape sh = prefill_shape(c, T, n_q_heads, q_len);
  const size_t units = (size_t)c.batch * c.kv_heads;
  return units * (2 * (size_t)sh.n_kt + (size_t)sh.n_qt) * kImgBytes + partial_bytes(sh);
}

struct Plan {
  int n_kt, TQ, n_qt, units, splits;
  int64_t rows;
  uint8_t *kimg, *vimg, *qimg;
  float *ws_m, *ws_l, *ws_o;  // split partials (splits > 1)
};

static int make_plan(const cq_paged_cache &cache, int64_t T, int Hq, int q_len, void *ws, size_t ws_bytes, Plan &pl) {
  CQ_REQUIRE(prefill_supported(cache, Hq, q_len), CQ_ERR_UNSUPPORTED,
             "query-chunk path: needs head_dim 128, q_len >= 16 and a GQA group that is a power of two <= 16");
  const Shape sh = prefill_shape(cache, T, Hq, q_len);
  pl.n_kt = sh.n_kt;
  pl.TQ = sh.TQ;
  pl.n_qt = sh.n_qt;
  pl.splits = sh.splits;
  pl.rows = sh.rows;
  const size_t need = prefill_workspace(cache, T, Hq, q_len);
  CQ_REQUIRE(ws && ws_bytes >= need, CQ_ERR_WORKSPACE, "cq_attention: workspace too small");
  CQ_REQUIRE(((uintptr_t)ws & 15) == 0, CQ_ERR_INVALID, "cq_attention: workspace must be 16-byte aligned for query chunks");
  pl.units = cache.batch * cache.kv_heads;
  CQ_REQUIRE((int64_t)pl.units * pl.n_qt * pl.splits < (1LL << 31), CQ_ERR_INVALID, "cq_attention: grid too large");
  pl.kimg = (uint8_t *)ws;
  pl.vimg = pl.kimg + (size_t)pl.units * pl.n_kt * kImgBytes;
  pl.qimg = pl.vimg + (size_t)pl.units * pl.n_kt * kImgBytes;
  pl.ws_o = (float *)(pl.qimg + (size_t)pl.units * pl.n_qt * kImgBytes);  // first: 16-byte aligned rows
  pl.ws_m = pl.ws_o + pl.rows * pl.splits * kTile;
  pl.ws_l = pl.ws_m + pl.rows * pl.splits;
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
  P.splits = pl.splits;
  P.ws_m = pl.ws_m;
  P.ws_l = pl.ws_l;
  P.ws_o = pl.ws_o;
  cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return set_error(CQ_ERR_CUDA, std::string("prefill attn_kernel smem: ") + cudaGetErrorString(e));
  attn_kernel<<<(unsigned)(pl.units * (pl.n_qt / 2) * pl.splits), kThreads, kSmemBytes, st>>>(P);
  r = check_launch("prefill attn_kernel");
  if (r || pl.splits == 1) return r;
  return launch_split_combine(pl.ws_m, pl.ws_l, pl.ws_o, pl.rows, pl.splits, kTile, out, out_dtype, lse_out, st);
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

int read_bounds_error_prefill(int clear) { return read_bounds_error_here(clear); }

}  // namespace cq
