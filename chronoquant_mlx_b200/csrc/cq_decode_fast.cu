// cq_decode_fast.cu -- split-KV decode attention over the paged compressed
// cache, written for sm_100a.
//
// Replaces the reference's fused Metal decode kernel (kernels.py:79-228),
// which re-reads each kv-head stream once per query head and does scalar
// math.  Here a warp streams chunks (32 or 64 tokens) of one (sequence,
// kv-head) unit and serves every query head of the GQA group from one read.
//
// Every warp runs its own copy pipeline of 1-D bulk-async copies (the TMA
// engine) of chunk blocks -- the chunk's K/V anchors, code rows and per-token
// scales, stored contiguously by the cache -- completion counted on
// mbarriers.  For 32-token chunks a warp owns two slots, each filled with a
// whole block.  For 64-token chunks a warp owns one K buffer and one V buffer:
// the block's K part is refilled (with the next chunk's) as soon as the
// chunk's scores are done, while the V part is still being consumed, so a
// warp holds one block of buffers instead of two and 16 warps fit in shared
// memory.  A warp waits only for its own copies, never for other warps.  The kernel is instantiated per (stride_k, stride_v) pair,
// so the chunk geometry and every shared-memory offset are compile-time
// constants.  Per chunk:
//
//   q.anchor  for the chunk's K anchors, one tensor-core MMA tile (rows =
//             anchors), kept in a small per-warp table;
//   scores    S = q.anchor + scale_t * (q . codes_t)          (kernels.py:152-159)
//             q.codes as an MMA on the raw nibbles (fp16 1024+n / 1024+16n,
//             the query pre-divided by 16 on the 16n lanes) minus the same
//             product for the all-8 (code 0) word;
//   softmax   online, base 2, lazily rescaled (a new max is applied only when
//             it exceeds the running one by 8, so p <= 256);
//   output    O += anchor_v(t) * p_t + codes_v(t) * (p_t * scale_t), both as
//             MMAs with tokens as the reduction axis: V anchors are gathered
//             per token with ldmatrix.trans (32-token chunks), or P is summed
//             per anchor by an indicator MMA and the chunk's anchors applied
//             once (64-token chunks); V codes (MMA nibble order) enter
//             as the fp16 values 64 + n = code + 72 made by bit operations
//             alone, and 72 * sum_t(p_t * scale_t) -- one more MMA with the
//             same fp16 weights -- is subtracted when the partial is written;
//             P moves to the operand layout with movmatrix.trans, and
//             P * scale as one half2 product with two tokens' scales.
//
// Work: warp w of the grid takes the contiguous, balanced chunk range
// [w*tc/W, (w+1)*tc/W) of the unit-major chunk index and writes one partial
// (max, sum, unnormalised output) per unit its range touches, in slot w + unit
// (unique: ranges are increasing).  The CTA whose warps complete a unit
// (counted in a per-call stamped word) merges the unit's partials into the
// output rows -- one launch per decode step.
//
// Requirements (fast_decode_supported): q_len 1, head_dim 128, GQA group <= 8,
// power-of-two strides with stride_k in {16, 32, 64} and stride_v in
// {8, .., 64} (chunk = max(32, strides) tokens dividing page_tokens), the
// cache's chunk-block layout for that geometry, K codes in the natural and V
// codes in the MMA nibble order, token-indexed scales.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <numeric>
#include <string>

#include "cq_decode_fast.cuh"
#include "cq_prefill.cuh"
#include "cq_encode.cuh"
#include "cq_ptx.cuh"

namespace cq {
namespace fast {

constexpr int HD = 128;          // head_dim
constexpr int kMaxWarps = 16;    // warps per CTA (one CTA per SM)
constexpr float TAU = 8.0f;      // lazy-rescale threshold (log2 units)
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr long long WAIT_BUDGET = 1LL << 31;  // clock cycles (~1 s) before a wait gives up
constexpr int ERR_TIMEOUT_FULL = 1;
constexpr int ERR_LENGTH = 4;  // a device-resident length outside [1, mapped tokens]
constexpr int kQaBytes = 16 * 8 * 4;  // per-warp q.anchor table: 16 anchors x 8 heads, fp32
constexpr int kQnBytes = 8 * 32 * 8;  // per-warp natural-order query fragments
constexpr int kBarsPerWarp = 4;       // a warp's copy barriers (at most two slots, or one K and one V buffer)

constexpr int cx_log2(int x) { return x <= 1 ? 0 : 1 + cx_log2(x >> 1); }
constexpr int cx_up16(int x) { return (x + 15) & ~15; }
constexpr int cx_max(int a, int b) { return a > b ? a : b; }

// Compile-time geometry of one (stride_k, stride_v) pair: chunk tokens, tiles
// per chunk, anchors per chunk and the byte offsets of a chunk block's six
// segments [K anchors][K codes][K scales][V anchors][V codes][V scales]
// (each 16-byte aligned) -- the layout the cache stores and a slot mirrors.
template <int SK_, int SV_, int VP_ = 4>
struct Geo {
  static constexpr int SK = SK_, SV = SV_;
  // VP: bits per stored V code -- 4 (INT4 lanes, 64-byte rows), or bit planes of physical 3-bit
  // (CQ_ORDER_PLANES3, 48 bytes) or 2-bit codes (CQ_ORDER_PLANES2, 32 bytes)
  static constexpr int VP = VP_;
  static constexpr bool V3 = VP == 3, PL = VP < 4;
  static constexpr int VR = VP == 3 ? 48 : VP == 2 ? 32 : HD / 2;
  static constexpr int LSK = cx_log2(SK), LSV = cx_log2(SV);
  static constexpr int C = cx_max(32, cx_max(SK, SV));
  static constexpr int NT = C / 16;
  static constexpr int AK = C / SK, AV = C / SV;
  static constexpr int O_KF0 = 0;
  static constexpr int O_CD0 = cx_up16(O_KF0 + AK * HD * 2);
  static constexpr int O_SC0 = cx_up16(O_CD0 + (C - AK) * (HD / 2));
  static constexpr int O_KF1 = cx_up16(O_SC0 + C * 2);
  static constexpr int O_CD1 = cx_up16(O_KF1 + AV * HD * 2);
  static constexpr int O_SC1 = cx_up16(O_CD1 + (C - AV) * VR);
  static constexpr int SLOT = cx_up16(O_SC1 + C * 2);
  // 32-token chunks: two slots per warp, each filled with a whole block.
  // 64-token chunks (SPLIT): the K part [0, O_KF1) and the V part [O_KF1,
  // SLOT) of a block go to separate buffers, one of each per warp; the K
  // buffer is refilled as soon as the chunk's scores are done and the V
  // buffer once its output is accumulated, so a warp needs one block of
  // buffers instead of two and 16 warps fit in shared memory.
  static constexpr bool SPLIT = C == 64;
  static constexpr int KB = O_KF1, VB = SLOT - O_KF1;
  static constexpr int V_CD = O_CD1 - O_KF1, V_SC = O_SC1 - O_KF1;  // offsets inside the V part
  static constexpr int NSK = SPLIT ? 1 : 2;                         // buffer pairs (SPLIT) or slots
  static constexpr int BUF = NSK * SLOT;                            // a warp's copy buffers
  static_assert(SK >= 16 && SV >= 8 && C <= 64 && AK <= 16, "geometry outside the kernel's range");
  static_assert(KB % 16 == 0 && VB % 16 == 0, "bulk copies need 16-byte sizes");
};

struct Params {
  CacheView cv;
  const void *q;
  int q_dtype;
  int64_t q_sb, q_sh;
  float scale;
  int gqa;
  int64_t T;              // cached tokens (used when T_dev is null)
  const int64_t *T_dev;   // else: read from device memory at launch (graph replays)
  int C;         // tokens per chunk
  int cpp;       // chunks per page
  int nwarps;    // warps with work (<= tc)
  // shared memory: [mbarriers][per-warp regions: ns slots + q.anchor table]
  int off_fin, off_strad, off_warp, warp_bytes;
  const char *blk;                // chunk blocks: K keyframes base (bytes)
  int64_t phs;                    // bytes per (page, head)
  int nwc;                        // warps per CTA
  float *ws_m, *ws_l, *ws_o;      // warp partials: [nwarps + units][gqa], same, [nwarps + units][gqa][HD]
  float *cs_m, *cs_l, *cs_o;      // CTA partials: [grid + units][gqa], same, [grid + units][gqa][HD]
  unsigned long long *done;       // per unit: call stamp << 16 | CTAs that finished it
  unsigned long long stamp;       // this call's stamp (48 bits, never 0)
  int Hq;
  void *out;
  int out_dtype;
  float *lse_out;
  // in-step encode (graph decode steps): the kernel first stores token
  // *T_dev of every unit (inputs x[comp] at b*x_sb + h*x_sh, dtype x_dtype),
  // attends over *T_dev + 1 tokens and, when its grid ends, sets *len_rw to
  // that length (arrival counter len_rw[1], left at 0)
  int fuse;
  const void *x[2];
  int64_t x_sb[2], x_sh[2];
  int x_dtype;
  int64_t *len_rw;
};

__device__ __forceinline__ int64_t warp_of_chunk(int64_t x, int64_t tc, int nwarps) {
  return ((x + 1) * nwarps + tc - 1) / tc - 1;
}

// Length-dependent plan of one launch: cached tokens, chunks per unit, total
// chunks, and whether the range arithmetic fits 32 bits.  Fixed on the host,
// or derived at launch from a device-resident length (the grid and workspace
// are sized for the largest length the caller allows).
struct Len {
  int64_t T, tc;
  int cpu, small;
  int nw;  // warps with work: min(grid warps, tc), so every one of them owns at least one chunk
};

// Warp owning chunk x, first chunk of warp w, unit of chunk x -- in 32-bit
// arithmetic when the plan is small enough (the usual case).
__device__ __forceinline__ int warp_of(const Params &p, const Len &L, int64_t x) {
  if (L.small) return (int)(((uint32_t)x + 1u) * (uint32_t)L.nw + (uint32_t)L.tc - 1u) / (uint32_t)L.tc - 1;
  return (int)warp_of_chunk(x, L.tc, L.nw);
}
__device__ __forceinline__ int64_t first_chunk(const Params &p, const Len &L, int w) {
  if (L.small) return (int64_t)(((uint32_t)w * (uint32_t)L.tc) / (uint32_t)L.nw);
  return (int64_t)w * L.tc / L.nw;
}
__device__ __forceinline__ int unit_of(const Len &L, int64_t x) {
  if (L.small) return (int)((uint32_t)x / (uint32_t)L.cpu);
  return (int)(x / L.cpu);
}

__device__ int g_fast_error;

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float q_scaled(const Params &p, int b, int hq, int d) {
  const float sc = round_dt(p.scale, p.q_dtype);
  float v = load_as_float(p.q, b * p.q_sb + hq * p.q_sh + d, p.q_dtype) * sc;
  return round_dt(v, p.q_dtype);  // q * scale in the query dtype (attention.py:46)
}

// Walks a warp's chunk range with running counters (no per-chunk division).
struct Cursor {
  int unit, b, h, cu, lp, j;  // unit, its (sequence, head), chunk in unit, page in unit, chunk in page
  int64_t left;               // chunks left including the current one
  __device__ void init(const Params &p, const Len &L, int64_t first, int64_t last) {
    unit = (int)(first / L.cpu);
    cu = (int)(first - (int64_t)unit * L.cpu);
    lp = cu / p.cpp;
    j = cu - lp * p.cpp;
    b = unit / p.cv.H;
    h = unit - b * p.cv.H;
    left = last - first;
  }
  __device__ bool valid() const { return left > 0; }
  __device__ int nvalid(const Params &p, const Len &L) const {
    return (int)min((int64_t)p.C, L.T - (int64_t)cu * p.C);
  }
  __device__ void next(const Params &p, const Len &L) {
    ++cu;
    if (++j == p.cpp) {
      j = 0;
      ++lp;
    }
    if (cu == L.cpu) {
      cu = lp = j = 0;
      ++unit;
      if (++h == p.cv.H) {
        h = 0;
        ++b;
      }
    }
    --left;
  }
};

// One bulk copy of one part of a chunk's block (page `pg`): the K part
// (PART 0: K anchors, codes, scales), the V part (PART 1) or the whole block
// (PART 2) into `buf`, counted on `bar`, issued by lane 0.  The whole part is
// copied even for the last, partial chunk of a unit: the bytes past its valid
// tokens are masked.
template <class G, int PART>
__device__ __forceinline__ void issue_part(const Params &p, uint32_t buf, uint64_t *bar, const Cursor &c, int64_t pg,
                                           int lane) {
  if (lane != 0) return;
  constexpr int off = PART == 1 ? G::O_KF1 : 0, bytes = PART == 2 ? G::SLOT : (PART ? G::VB : G::KB);
  ptx::mbar_arrive_expect_tx(bar, (uint32_t)bytes);
  const char *src = p.blk + (pg * p.cv.H + c.h) * p.phs + (int64_t)c.j * G::SLOT + off;
  ptx::bulk_g2s_a(buf, src, (uint32_t)bytes, bar);
}

struct QFrag {
  uint32_t qb[4][4];  // query as B fragments in the K-code order (q/16 on the 16n lanes)
  float2 qc;          // q . (raw values of the all-8 word) for heads 2t, 2t+1
};

// Loads the unit's query: K-code-order fragments into registers, natural-order
// fragments (for the anchors) into the warp's table qn[8][32 lanes] (uint2).
__device__ void load_q(const Params &p, int b, int h, int lane, QFrag &f, uint2 *qn) {
  const int g = lane >> 2, t = lane & 3;
  const int hq = h * p.gqa + g;
  const bool real = g < p.gqa;
  float cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int J = 0; J < 4; ++J) {
    const int d0 = 32 * t + 8 * J;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = real ? q_scaled(p, b, hq, d0 + i) : 0.f;
    f.qb[J][0] = ptx::pack_half2(v[0], v[4]);
    f.qb[J][1] = ptx::pack_half2(v[1] * 0.0625f, v[5] * 0.0625f);
    f.qb[J][2] = ptx::pack_half2(v[2], v[6]);
    f.qb[J][3] = ptx::pack_half2(v[3] * 0.0625f, v[7] * 0.0625f);
    ptx::mma_f16_16816(cc, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_HI, ptx::RAW_CODE0_HI, f.qb[J][0],
                       f.qb[J][1]);
    ptx::mma_f16_16816(cc, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_HI, ptx::RAW_CODE0_HI, f.qb[J][2],
                       f.qb[J][3]);
  }
  f.qc = make_float2(cc[0], cc[1]);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d0 = 16 * kk + 2 * t;
    qn[kk * 32 + lane] =
        real ? make_uint2(ptx::pack_half2(q_scaled(p, b, hq, d0), q_scaled(p, b, hq, d0 + 1)),
                          ptx::pack_half2(q_scaled(p, b, hq, d0 + 8), q_scaled(p, b, hq, d0 + 9)))
             : make_uint2(0u, 0u);
  }
}

// q . anchor (log2 units) for the first nK (<= 16) K anchors of a slot, as
// one MMA tile with rows = anchors; table [16][8] fp32 at `qa`.
__device__ __forceinline__ void compute_qa(uint32_t kfK, float *qa, int nK, const uint2 *qn, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
  const int arow = min(rr + ((mi & 1) ? 8 : 0), nK - 1);
  const uint32_t base = kfK + arow * (HD * 2) + ((mi & 2) ? 16 : 0);
#pragma unroll
  for (int kk = 0; kk < 8; kk += 2) {
    uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
    ptx::ldmatrix_x4(a0, a1, a2, a3, base + kk * 32);
    ptx::ldmatrix_x4(b0, b1, b2, b3, base + kk * 32 + 32);
    const uint2 q0 = qn[kk * 32 + lane], q1 = qn[(kk + 1) * 32 + lane];
    ptx::mma_f16_16816(c0, a0, a1, a2, a3, q0.x, q0.y);
    ptx::mma_f16_16816(c1, b0, b1, b2, b3, q1.x, q1.y);
  }
  float *row0 = qa + g * 8 + 2 * t;
  *(float2 *)row0 = make_float2((c0[0] + c1[0]) * LOG2E, (c0[1] + c1[1]) * LOG2E);
  *(float2 *)(row0 + 64) = make_float2((c0[2] + c1[2]) * LOG2E, (c0[3] + c1[3]) * LOG2E);
}

// ---------------------------------------------------------------------------
// per-warp softmax state and one chunk of NT 16-token tiles
// ---------------------------------------------------------------------------
struct WarpState {
  float m[2];     // running max (log2 units) of heads 2t, 2t+1
  float l[2];     // this thread's partial sums
  float o[8][4];  // O^T fragments: [m-tile i][c0..c3]
  float vb[4];    // 72 * sum of the fp16 code weights P' (same fragment layout): the V code offset
  float ps[4];    // P summed per V anchor slot of the chunk (rows) and head
};

__device__ __forceinline__ void reset(WarpState &st) {
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
  st.vb[0] = st.vb[1] = st.vb[2] = st.vb[3] = 0.f;
  st.ps[0] = st.ps[1] = st.ps[2] = st.ps[3] = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[i][j] = 0.f;
}

// Per-lane shared-memory byte addresses into a K part.  Code rows are stored
// in P-frame order; the row of chunk-local token x is x - x/stride - 1 (an
// I-frame lands on the previous row, read harmlessly with scale 0).  For a
// 16-token tile at tb with stride_k >= 16 the K rows of tokens tb + x are
// (tb - tb/stride_k) + x - 1.
struct KAddr {
  uint32_t cdK;  // K code row of token g (tile base 0), word group t
  uint32_t scK;  // K scale of token g
  uint32_t qa;   // q.anchor table, heads 2t, 2t+1
  template <class G>
  __device__ __forceinline__ KAddr(G, uint32_t kb, uint32_t qa_base, int lane) {
    const int g = lane >> 2, t = lane & 3;
    cdK = kb + G::O_CD0 + (g - 1) * 64 + t * 16;
    scK = kb + G::O_SC0 + g * 2;
    qa = qa_base + t * 8;
  }
};

// Per-lane shared-memory byte addresses into a V part.
struct VAddr {
  uint32_t cdV;   // V code row of token 2t (tile base 0), words 2g, 2g+1
  uint32_t scV;   // V scales of tokens 2t, 2t+1 (one 32-bit word)
  uint32_t kfV;   // V anchor row of this lane's ldmatrix row (tile 0)
  uint32_t kfV0;  // V anchor row 0, same column half
  int dv8;        // V rows between tokens 2t and 2t+8
  template <class G>
  __device__ __forceinline__ VAddr(G, uint32_t vb, int lane) {
    const int g = lane >> 2, t = lane & 3, mi = lane >> 3;
    constexpr bool v8 = G::LSV == 3;
    cdV = vb + G::V_CD + (2 * t - 1) * G::VR + (G::PL ? 0 : g * 8);  // bit-plane rows: lane offsets at use
    dv8 = v8 ? 7 : 8;
    scV = vb + G::V_SC + t * 4;
    kfV0 = vb + ((mi & 1) ? 16 : 0);
    kfV = kfV0 + ((v8 ? (mi >> 1) : 0) * (HD * 2));
  }
};

__device__ __forceinline__ float lds_half_as_float(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return __half2float(__ushort_as_half(v));
}

// Scores of the two 16-token tiles at chunk-local token t0 and their softmax
// update; P of the two tiles in the MMA B-operand layout (a lane holds tokens
// 2t, 2t+1 (and 2t+8, 2t+9) of head g) into bp[0..1].  When the running max
// moves, the output state is rescaled and the function returns true with the
// factor for head g in `fh` (for the P of the chunk's earlier groups).
template <class G, bool MASK>
__device__ __forceinline__ bool k_group(WarpState &st, const KAddr &A, const QFrag &f, int t0, int nvalid, int lane,
                                        uint2 (&bp)[2], __half2 &fh) {
  constexpr int lsk = G::LSK;
  constexpr int NT = 2;
  const int g = lane >> 2;
  float s[NT][4];
  // ---------------- scores S^T[token][head] = scale_t * (q.codes_t) + q.anchor
#pragma unroll
  for (int tile = 0; tile < NT; ++tile) {
    const int tb = t0 + tile * 16;
    const uint32_t rk = (uint32_t)((tb - (tb >> lsk)) * 64);  // K rows before the tile
    const uint4 wk0 = ptx::lds_u128(A.cdK + rk);
    const uint4 wk1 = ptx::lds_u128(A.cdK + rk + 8 * 64);
    const float sk0 = lds_half_as_float(A.scK + tb * 2) * LOG2E;
    const float sk1 = lds_half_as_float(A.scK + (tb + 8) * 2) * LOG2E;
    const float2 qa = ptx::lds_f2(A.qa + (uint32_t)((tb >> lsk) * 32));  // one K anchor per tile (stride >= 16)
    // raw nibbles (1024+n, 1024+16n) against q (q/16 on the 16n lanes); the
    // accumulator starts at -q.(all-8 word), which removes the raw offset
    float ca[4] = {-f.qc.x, -f.qc.y, -f.qc.x, -f.qc.y}, cb[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t w0[4] = {wk0.x, wk0.y, wk0.z, wk0.w};
    const uint32_t w1[4] = {wk1.x, wk1.y, wk1.z, wk1.w};
#pragma unroll
    for (int J = 0; J < 4; ++J) {
      uint32_t h0[4], h1[4];
      ptx::nibbles_to_half2_raw(w0[J], h0);  // (d0,d4) (d1,d5) (d2,d6) (d3,d7)
      ptx::nibbles_to_half2_raw(w1[J], h1);
      ptx::mma_f16_16816(ca, h0[0], h1[0], h0[1], h1[1], f.qb[J][0], f.qb[J][1]);
      ptx::mma_f16_16816(cb, h0[2], h1[2], h0[3], h1[3], f.qb[J][2], f.qb[J][3]);
    }
    s[tile][0] = fmaf(sk0, ca[0] + cb[0], qa.x);
    s[tile][1] = fmaf(sk0, ca[1] + cb[1], qa.y);
    s[tile][2] = fmaf(sk1, ca[2] + cb[2], qa.x);
    s[tile][3] = fmaf(sk1, ca[3] + cb[3], qa.y);
    if (MASK) {
      // tokens past the end: score -inf (their buffer bytes are stale)
      if (tb + g >= nvalid) s[tile][0] = s[tile][1] = -INFINITY;
      if (tb + g + 8 >= nvalid) s[tile][2] = s[tile][3] = -INFINITY;
    }
  }
  // ---------------- online softmax (base 2), lazy rescale
  bool moved = false;
  {
    float mx0 = fmaxf(s[0][0], s[0][2]), mx1 = fmaxf(s[0][1], s[0][3]);
#pragma unroll
    for (int tile = 1; tile < NT; ++tile) {
      mx0 = fmaxf(mx0, fmaxf(s[tile][0], s[tile][2]));
      mx1 = fmaxf(mx1, fmaxf(s[tile][1], s[tile][3]));
    }
    const bool need = (mx0 > st.m[0] + TAU) || (mx1 > st.m[1] + TAU);
    if (__any_sync(0xffffffffu, need)) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float n0 = fmaxf(st.m[0], mx0), n1 = fmaxf(st.m[1], mx1);
      const float f0 = (n0 == -INFINITY) ? 1.f : fast_exp2(st.m[0] - n0);
      const float f1 = (n1 == -INFINITY) ? 1.f : fast_exp2(st.m[1] - n1);
      st.m[0] = n0;
      st.m[1] = n1;
      st.l[0] *= f0;
      st.l[1] *= f1;
      st.vb[0] *= f0;
      st.vb[1] *= f1;
      st.vb[2] *= f0;
      st.vb[3] *= f1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        st.o[i][0] *= f0;
        st.o[i][1] *= f1;
        st.o[i][2] *= f0;
        st.o[i][3] *= f1;
      }
      // the factor of head g (the operand layout's head) for the chunk's earlier P
      const float a = __shfl_sync(0xffffffffu, f0, g >> 1), b = __shfl_sync(0xffffffffu, f1, g >> 1);
      fh = __float2half2_rn((g & 1) ? b : a);
      moved = true;
    }
  }
#pragma unroll
  for (int tile = 0; tile < NT; ++tile) {
    // masked scores are -inf and the running max is finite here: ex2(-inf) = 0
    const float p0 = fast_exp2(s[tile][0] - st.m[0]);
    const float p1 = fast_exp2(s[tile][1] - st.m[1]);
    const float p2 = fast_exp2(s[tile][2] - st.m[0]);
    const float p3 = fast_exp2(s[tile][3] - st.m[1]);
    if (!G::SPLIT) {  // 64-token chunks sum P through the indicator MMA's all-ones row instead
      st.l[0] += p0 + p2;
      st.l[1] += p1 + p3;
    }
    bp[tile] = make_uint2(ptx::movmatrix_trans(ptx::pack_half2(p0, p1)), ptx::movmatrix_trans(ptx::pack_half2(p2, p3)));
  }
  return moved;
}

// Output of the 16-token tile at chunk-local token tb with its P (bP0, bP1).
template <class G, bool MASK>
__device__ __forceinline__ void v_tile(WarpState &st, const VAddr &A, int tb, uint32_t bP0, uint32_t bP1, int nvalid,
                                       int lane) {
  constexpr int lsv = G::LSV;
  // P' = P * scale_v: in the operand layout a lane holds tokens 2t, 2t+1 (and
  // 2t+8, 2t+9) of head g, whose V scales are one 32-bit word each
  uint32_t sw0 = ptx::lds_u32(A.scV + tb * 2), sw1 = ptx::lds_u32(A.scV + (tb + 8) * 2);
  if (MASK) {
    // scales past the end are stale bytes (P is 0 there, but 0 * inf is not)
    const int t2 = tb + 2 * (lane & 3);
    if (t2 >= nvalid) sw0 = 0u;
    else if (t2 + 1 >= nvalid) sw0 &= 0xffffu;
    if (t2 + 8 >= nvalid) sw1 = 0u;
    else if (t2 + 9 >= nvalid) sw1 &= 0xffffu;
  }
  const uint32_t bS0 = ptx::h22u(__hmul2(ptx::u2h2(bP0), ptx::u2h2(sw0)));
  const uint32_t bS1 = ptx::h22u(__hmul2(ptx::u2h2(bP1), ptx::u2h2(sw1)));
  if (G::SPLIT) {
    // 64-token chunks have few V anchors (2 for stride 32): P is summed per
    // anchor slot of the chunk (rows of ps) by one MMA with an indicator
    // matrix (row a, token k: 1 when token k belongs to anchor a), and the
    // anchors are applied once per chunk (see do_chunk) instead of gathered
    // for every token
    constexpr uint32_t ONE2 = 0x3C003C00u;
    const int gg = lane >> 2, t2 = 2 * (lane & 3);
    const int s0 = (tb + t2) >> lsv, s1 = (tb + t2 + 8) >> lsv;
    const uint32_t r15 = gg == 7 ? ONE2 : 0u;  // row 15: every token (the softmax denominator)
    ptx::mma_f16_16816(st.ps, gg == s0 ? ONE2 : 0u, r15, gg == s1 ? ONE2 : 0u, r15, bP0, bP1);
  } else
  // V anchors: O += A_v^T P, ldmatrix.trans gathers each token's anchor row
  {
    uint32_t base = A.kfV + (uint32_t)((tb >> lsv) * (HD * 2));
    if (MASK) {
      // rows past the copied anchors hold stale bytes: use anchor 0 (P is 0 there)
      const int mi = lane >> 3, r = lane & 7;
      if (tb + r + ((mi & 2) ? 8 : 0) >= nvalid) base = A.kfV0;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t a0, a1, a2, a3;
      ptx::ldmatrix_x4_trans(a0, a1, a2, a3, base + i * 32);
      ptx::mma_f16_16816(st.o[i], a0, a1, a2, a3, bP0, bP1);
    }
  }
  if constexpr (G::PL) {
    // bit-plane V codes: a row's low plane word g holds dims 8k + g (k = 0..15) at bits 2k; with
    // 3-bit codes a high plane half-word g holds the same dims' third bits at bit k
    // (CQ_ORDER_PLANES3, CQ_ORDER_PLANES2).  The fp16 operand 64 + v (v = code + 4, or code + 2)
    // gets the low bits at bits 4-5 and the high bit at bit 6 of each half
    constexpr uint32_t R = G::VR;  // bytes per row
    const int g = lane >> 2;
    const uint32_t r0 = A.cdV + (uint32_t)((tb - (tb >> lsv)) * R);
    const uint32_t r2 = r0 + (uint32_t)A.dv8 * R;
    const uint32_t lo = 4 * g, hi = 32 + 2 * g;
    const uint32_t la = ptx::lds_u32(r0 + lo), lb = ptx::lds_u32(r0 + R + lo);
    const uint32_t lc = ptx::lds_u32(r2 + lo), ld = ptx::lds_u32(r2 + R + lo);
    uint32_t hab = 0u, hcd = 0u;
    if constexpr (G::V3) {
      hab = __byte_perm(ptx::lds_u16(r0 + hi), ptx::lds_u16(r0 + R + hi), 0x5410u);
      hcd = __byte_perm(ptx::lds_u16(r2 + hi), ptx::lds_u16(r2 + R + hi), 0x5410u);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int bi = 2 * q + half;  // byte of the low plane (4 dims), nibble of the high plane
        const uint32_t sel = bi | (bi << 4) | ((4 + bi) << 8) | ((4 + bi) << 12);
        const uint32_t xab = __byte_perm(la, lb, sel), xcd = __byte_perm(lc, ld, sel);
        uint32_t xa[4], xc[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int sl = 4 - 2 * kk;  // low bits 2kk..2kk+1 -> 4..5; high bit kk -> 6
          const uint32_t pa = sl >= 0 ? xab << sl : xab >> -sl, pc = sl >= 0 ? xcd << sl : xcd >> -sl;
          xa[kk] = ptx::lop3_and_or(pa, 0x00300030u, 0x54005400u);
          xc[kk] = ptx::lop3_and_or(pc, 0x00300030u, 0x54005400u);
          if constexpr (G::V3) {
            const uint32_t yab = hab >> (4 * bi), ycd = hcd >> (4 * bi);
            xa[kk] = ptx::lop3_and_or(yab << (6 - kk), 0x00400040u, xa[kk]);
            xc[kk] = ptx::lop3_and_or(ycd << (6 - kk), 0x00400040u, xc[kk]);
          }
        }
        // dim index k = 8q + 4 half + kk <-> m-tile 4q + (4 half + kk)/2, row g (+8 when kk is odd)
        const int i0 = 4 * q + 2 * half;
        ptx::mma_f16_16816(st.o[i0], xa[0], xa[1], xc[0], xc[1], bS0, bS1);
        ptx::mma_f16_16816(st.o[i0 + 1], xa[2], xa[3], xc[2], xc[3], bS0, bS1);
      }
    }
    // the offset of every code value (68 or 66): offset * sum_t P'_t, exactly as the MMAs above weight it
    constexpr uint32_t OFF = G::V3 ? ptx::HALF2_68 : ptx::HALF2_66;
    ptx::mma_f16_16816(st.vb, OFF, OFF, OFF, OFF, bS0, bS1);
  } else
  // V codes: O += C_v^T P'  (tokens 2t,2t+1 | 2t+8,2t+9; words 2g, 2g+1)
  {
    // V rows of tokens tb+2t, +1, +8, +9 (stride 8: the I-frame at tb+8 sits between)
    const uint32_t rv = A.cdV + (uint32_t)((tb - (tb >> lsv)) * 64);
    const uint32_t rv8 = rv + (uint32_t)A.dv8 * 64;
    const uint2 va = ptx::lds_u64(rv);
    const uint2 vb = ptx::lds_u64(rv + 64);
    const uint2 vc = ptx::lds_u64(rv8);
    const uint2 vd = ptx::lds_u64(rv8 + 64);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint32_t wa = q ? va.y : va.x, wb = q ? vb.y : vb.x;
      const uint32_t wc = q ? vc.y : vc.x, wd = q ? vd.y : vd.x;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t sel = half ? 0x7632u : 0x5410u;
        uint32_t xa[4], xc[4];
        ptx::nibbles_to_half2_64(__byte_perm(wa, wb, sel), xa);  // nibbles 4*half + 0..3 of tokens (a, b)
        ptx::nibbles_to_half2_64(__byte_perm(wc, wd, sel), xc);
        // nibble j of word q <-> m-tile 4q + j/2, row g (+8 when j is odd)
        const int i0 = 4 * q + 2 * half;
        ptx::mma_f16_16816(st.o[i0], xa[0], xa[1], xc[0], xc[1], bS0, bS1);
        ptx::mma_f16_16816(st.o[i0 + 1], xa[2], xa[3], xc[2], xc[3], bS0, bS1);
      }
    }
    // the offset 72 of every code value: 72 * sum_t P'_t, exactly as the MMAs above weight it
    ptx::mma_f16_16816(st.vb, ptx::HALF2_72, ptx::HALF2_72, ptx::HALF2_72, ptx::HALF2_72, bS0, bS1);
  }
}

// Write the warp's state for one unit (real heads only) as a partial --
// max, sum and unnormalised output at pm[h], pl[h], po[h * HD + dim] -- and
// reset it.
__device__ void flush_to(const Params &p, WarpState &st, float *pm, float *pl, float *po, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int G = p.gqa;
  float l0 = st.l[0], l1 = st.l[1];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[i][j] -= st.vb[j];  // codes were 64 + n = (n - 8) + 72
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  const int h0 = 2 * t, h1 = 2 * t + 1;
  if (g == 0) {
    if (h0 < G) {
      pm[h0] = st.m[0];
      pl[h0] = l0;
    }
    if (h1 < G) {
      pm[h1] = st.m[1];
      pl[h1] = l1;
    }
  }
  if (h0 < G) {
    float *w0 = po + h0 * HD;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w0[16 * i + g] = st.o[i][0];
      w0[16 * i + g + 8] = st.o[i][2];
    }
  }
  if (h1 < G) {
    float *w1 = po + h1 * HD;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w1[16 * i + g] = st.o[i][1];
      w1[16 * i + g + 8] = st.o[i][3];
    }
  }
  reset(st);
}

// A unit change inside a warp's range: its partial goes to global slot wg + unit.
__device__ __forceinline__ void flush_global(const Params &p, WarpState &st, int64_t slot, int lane) {
  flush_to(p, st, p.ws_m + slot * p.gqa, p.ws_l + slot * p.gqa, p.ws_o + slot * p.gqa * HD, lane);
}

// Per-warp partial kept in shared memory at the end of the warp's range:
// [8] max, [8] sum, [8][HD] output (the warp's free copy slots hold it).
constexpr int kFinFloats = 16 + 8 * HD;
// Partials of the units a warp leaves inside its range (a unit boundary in
// the middle of a warp's range; one warp per boundary) stay on chip too, for
// the first kStrad units of the CTA's range; later ones go to global slots.
constexpr int kStrad = 2;

__device__ __forceinline__ int cta_first_unit(const Params &p, const Len &L, int cta) {
  return unit_of(L, first_chunk(p, L, cta * p.nwc));
}

// In-step encode of component COMP of token tnew of unit (b, h) by one warp,
// into the chunk's part in shared memory (already holding the part copied
// from the cache) and into the cache block itself (physical page pg).  The
// same codec as the append kernel.
template <class G, int DTYPE, int COMP>
__device__ void encode_new_token(const Params &p, unsigned char *part, int64_t pg, int b, int h, int64_t tnew,
                                 uint32_t *sw, int lane) {
  const int tl = (int)(tnew % p.cv.P);
  const int x = tl % G::C, j = tl / G::C;
  unsigned char *blk = const_cast<unsigned char *>((const unsigned char *)p.blk) + (pg * p.cv.H + h) * p.phs +
                       (int64_t)j * G::SLOT + (COMP ? G::O_KF1 : 0);
  const CompView &c = p.cv.c[COMP];
  constexpr int s = COMP ? G::SV : G::SK;
  constexpr int ocd = COMP ? G::V_CD : G::O_CD0, osc = COMP ? G::V_SC : G::O_SC0;  // offsets inside the part
  const int a = x / s, phase = x - a * s;
  const int64_t xb = b * p.x_sb[COMP] + h * p.x_sh[COMP];
  float xv[kMaxDimsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDimsPerLane; ++i) {
    const int d = lane + 32 * i;
    xv[i] = (d < HD) ? load_as_float(p.x[COMP], xb + d, DTYPE) : 0.f;
  }
  __half *arow_s = (__half *)(part + a * HD * 2), *arow_g = (__half *)(blk + a * HD * 2);
  if (phase == 0) {  // I-frame: token.astype(float16) (cache.py:103-105), scale slot 0
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) {
      const __half v = __float2half_rn(xv[i]);
      arow_s[lane + 32 * i] = v;
      arow_g[lane + 32 * i] = v;
    }
    if (lane == 0) {
      *(__half *)(part + osc + x * 2) = __float2half_rn(0.f);
      *(__half *)(blk + osc + x * 2) = __float2half_rn(0.f);
    }
  } else {
    float av[kMaxDimsPerLane];
#pragma unroll
    for (int i = 0; i < kMaxDimsPerLane; ++i) av[i] = (i < HD / 32) ? __half2float(arow_s[lane + 32 * i]) : 0.f;
    // the fast kernel's layouts: K codes in natural order, V codes in the MMA nibble order or bit planes
    constexpr int order =
        COMP ? (G::VP == 3 ? CQ_ORDER_PLANES3 : G::VP == 2 ? CQ_ORDER_PLANES2 : CQ_ORDER_MMA) : CQ_ORDER_NATURAL;
    const float scale = encode_residual<DTYPE>(xv, av, HD, c.bits, c.dead_zone, order, sw, lane);
    const int pf = x - a - 1;
    constexpr int rw = COMP ? G::VR / 4 : HD / 8;  // words of a code row
    if (lane < rw) {
      ((uint32_t *)(part + ocd + pf * rw * 4))[lane] = sw[lane];
      ((uint32_t *)(blk + ocd + pf * rw * 4))[lane] = sw[lane];
    }
    if (lane == 0) {
      *(__half *)(part + osc + x * 2) = __float2half_rn(scale);
      *(__half *)(blk + osc + x * 2) = __float2half_rn(scale);
    }
  }
  __syncwarp();
}

template <class G, int COMP>
__device__ __forceinline__ void encode_if_last(const Params &p, const Len &L, const Cursor &cc, unsigned char *part,
                                               uint32_t *sw, int lane) {
  if (!(p.fuse && cc.cu == L.cpu - 1)) return;  // this step's new token lies in the unit's last chunk
  const int64_t pg = table_page(p.cv, cc.b, cc.lp);
  if (p.x_dtype == CQ_BF16)
    encode_new_token<G, CQ_BF16, COMP>(p, part, pg, cc.b, cc.h, L.T - 1, sw, lane);
  else
    encode_new_token<G, CQ_F16, COMP>(p, part, pg, cc.b, cc.h, L.T - 1, sw, lane);
}

// One chunk: the K phase (scores and softmax of every 32-token group, P kept
// in registers), then the V phase (output of every tile).  With SPLIT the K
// buffer is refilled between the two phases and the V buffer after them;
// otherwise the whole slot is refilled at the end.  Returns false when a wait
// gave up.
template <class G, bool MASK>
__device__ __forceinline__ bool do_chunk(const Params &p, const Len &L, WarpState &st, const QFrag &f,
                                         const Cursor &cc, int nvalid, unsigned char *region, uint64_t *bar, int sk,
                                         uint32_t ph, Cursor &ci, int64_t pg_next, float *qa, const uint2 *qn,
                                         int lane) {
  constexpr int NG = G::NT / 2;  // 32-token groups per chunk
  const uint32_t ra = ptx::smem_u32(region);
  // K and V parts: separate buffers (SPLIT) or the two halves of slot sk
  const int koff = G::SPLIT ? 0 : sk * G::SLOT, voff = G::SPLIT ? G::KB : sk * G::SLOT + G::O_KF1;
  const uint32_t kb = ra + koff, vbuf = ra + voff;
  // ---- K phase
  if (!ptx::mbar_wait_bounded(&bar[sk], ph, WAIT_BUDGET)) return false;
  encode_if_last<G, 0>(p, L, cc, region + koff, (uint32_t *)qa, lane);
  compute_qa(kb + G::O_KF0, qa, MASK ? ((nvalid - 1) >> G::LSK) + 1 : G::AK, qn, lane);
  __syncwarp();
  uint2 bp[NG][2];
  {
    const KAddr A(G(), kb, ptx::smem_u32(qa), lane);
#pragma unroll
    for (int grp = 0; grp < NG; ++grp) {
      if (MASK && grp * 32 >= nvalid) break;
      __half2 fh;
      if (k_group<G, MASK>(st, A, f, grp * 32, nvalid, lane, bp[grp], fh)) {
        // this chunk's earlier P into the new frame
#pragma unroll
        for (int k = 0; k < grp; ++k)
#pragma unroll
          for (int tile = 0; tile < 2; ++tile) {
            bp[k][tile].x = ptx::h22u(__hmul2(ptx::u2h2(bp[k][tile].x), fh));
            bp[k][tile].y = ptx::h22u(__hmul2(ptx::u2h2(bp[k][tile].y), fh));
          }
      }
    }
  }
  if (G::SPLIT) {
    // every lane's reads of the K buffer (and of the q.anchor table) are done before the refill
    __syncwarp();
    ptx::fence_proxy_async_smem();
    if (ci.valid()) issue_part<G, 0>(p, kb, &bar[sk], ci, pg_next, lane);
    // ---- V phase: its own buffer
    if (!ptx::mbar_wait_bounded(&bar[G::NSK + sk], ph, WAIT_BUDGET)) return false;
  }
  encode_if_last<G, 1>(p, L, cc, region + voff, (uint32_t *)qa, lane);
  {
    const VAddr A(G(), vbuf, lane);
#pragma unroll
    for (int grp = 0; grp < NG; ++grp)
#pragma unroll
      for (int tile = 0; tile < 2; ++tile)
        if (!MASK || grp * 32 + tile * 16 < nvalid)
          v_tile<G, MASK>(st, A, grp * 32 + tile * 16, bp[grp][tile].x, bp[grp][tile].y, nvalid, lane);
    if (G::SPLIT) {
      // O += A_v^T PS: the chunk's V anchors (rows = slots; past the valid ones, the last valid one, weight 0)
      const int nA = MASK ? ((nvalid - 1) >> G::LSV) + 1 : G::AV;
      const uint32_t b0 = ptx::movmatrix_trans(ptx::pack_half2(st.ps[0], st.ps[1]));
      st.l[0] += st.ps[2];  // row 15 (lanes g == 7): this chunk's sum of P per head
      st.l[1] += st.ps[3];
      st.ps[0] = st.ps[1] = st.ps[2] = st.ps[3] = 0.f;
      const uint32_t base = vbuf + min(lane & 7, nA - 1) * (HD * 2) + (lane >> 3) * 16;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t a0, a1, a2, a3;
        ptx::ldmatrix_x4_trans(a0, a1, a2, a3, base + i * 64);
        ptx::mma_f16_16816(st.o[2 * i], a0, a1, 0u, 0u, b0, 0u);
        ptx::mma_f16_16816(st.o[2 * i + 1], a2, a3, 0u, 0u, b0, 0u);
      }
    }
  }
  // every lane's reads of the V part are done before the refill
  __syncwarp();
  ptx::fence_proxy_async_smem();
  if (ci.valid()) {
    if (G::SPLIT)
      issue_part<G, 1>(p, vbuf, &bar[G::NSK + sk], ci, pg_next, lane);
    else
      issue_part<G, 2>(p, kb, &bar[sk], ci, pg_next, lane);
    ci.next(p, L);
  }
  return true;
}

template <class G>
__device__ __forceinline__ void warp_main(const Params &p, const Len &L, unsigned char *smem, uint64_t *bar, int wg,
                                          int warp, int lane) {
  const int64_t first = first_chunk(p, L, wg);
  const int64_t last = first_chunk(p, L, wg + 1);
  unsigned char *region = smem + p.off_warp + warp * p.warp_bytes;
  const uint32_t region_a = ptx::smem_u32(region);
  const int u0 = cta_first_unit(p, L, blockIdx.x);
  float *qa = (float *)(region + G::BUF);
  uint2 *qn = (uint2 *)(region + G::BUF + kQaBytes);

  // the issue cursor runs NSK chunks ahead: a chunk's slot (or K and V
  // buffers) is refilled with the chunk NSK positions later
  Cursor ci, cc;
  cc.init(p, L, first, last);
  ci = cc;
  for (int s = 0; s < G::NSK && ci.valid(); ++s) {
    const int64_t pg = table_page(p.cv, ci.b, ci.lp);
    if (G::SPLIT) {
      issue_part<G, 0>(p, region_a, &bar[s], ci, pg, lane);
      issue_part<G, 1>(p, region_a + G::KB, &bar[G::NSK + s], ci, pg, lane);
    } else {
      issue_part<G, 2>(p, region_a + s * G::SLOT, &bar[s], ci, pg, lane);
    }
    ci.next(p, L);
  }

  WarpState st;
  reset(st);
  QFrag f;
  int cur_unit = -1;
  int sk = 0;  // slot (or buffer pair) of this chunk and its barrier phase
  uint32_t ph = 0;
  for (; cc.valid(); cc.next(p, L)) {
    // page of the next chunk to issue, loaded early so its latency hides under this chunk
    const int64_t pg_next = ci.valid() ? table_page(p.cv, ci.b, ci.lp) : 0;
    if (cc.unit != cur_unit) {
      if (cur_unit >= 0) {
        const int a = cur_unit - u0;
        if (a < kStrad) {
          float *sp = (float *)(smem + p.off_strad) + a * kFinFloats;
          flush_to(p, st, sp, sp + 8, sp + 16, lane);
        } else {
          flush_global(p, st, (int64_t)wg + cur_unit, lane);
        }
      }
      cur_unit = cc.unit;
      load_q(p, cc.b, cc.h, lane, f, qn);
      __syncwarp();
    }
    const int nvalid = cc.nvalid(p, L);
    const bool ok = (nvalid == G::C)
                        ? do_chunk<G, false>(p, L, st, f, cc, nvalid, region, bar, sk, ph, ci, pg_next, qa, qn, lane)
                        : do_chunk<G, true>(p, L, st, f, cc, nvalid, region, bar, sk, ph, ci, pg_next, qa, qn, lane);
    if (!ok) {
      // a copy never landed: record it and stop this warp (no hang, results invalid)
      atomicExch(&g_fast_error, ERR_TIMEOUT_FULL);
      return;
    }
    if (++sk == G::NSK) {
      sk = 0;
      ph ^= 1u;
    }
  }
  // the last unit's partial stays on chip for the CTA merge
  if (cur_unit >= 0) {
    float *fin = (float *)region;
    flush_to(p, st, fin, fin + 8, fin + 16, lane);
  }
  if (lane == 0) ((int *)(smem + p.off_fin))[warp] = cur_unit;
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// End of a CTA.  First the CTA merges, per unit its range touches, its warps'
// partials: the on-chip ones (each warp's last unit) and the global ones its
// warps wrote at a unit change.  A unit that lies entirely in this CTA's range
// goes straight to the output rows; otherwise the merge becomes CTA partial
// slot cta + unit, and the CTA counts itself in the unit's completion word
// stamp << 16 | count, where the stamp is this call's number: a word with any
// other stamp (left by an earlier call, or never written) counts as zero.
// The CTA that completes
// a unit merges the unit's CTA partials into the output rows of its query
// heads (and their log-sum-exp) while other CTAs may still be working.
__device__ void finish_units(const Params &p, const Len &L, unsigned char *smem) {
  __shared__ int s_n;
  __shared__ float s_w[kMaxWarps][8];  // per (warp, head): weight exp2(m_w - M)
  __shared__ float s_ML[8][2];         // per head: M, L
  __shared__ int s_glob[kMaxWarps];    // the warp's partial of this unit is in global memory
  __shared__ int s_src[kMaxWarps];     // else: float offset of its on-chip partial
  __shared__ const float *s_optr[kMaxWarps];  // output rows of the warp's partial (shared or global, generic)
  const int G = p.gqa;
  const int *fin_unit = (const int *)(smem + p.off_fin);
  const int w0 = blockIdx.x * p.nwc;
  const int w1 = min(w0 + p.nwc, L.nw) - 1;
  const int64_t cfirst = first_chunk(p, L, w0), clast = first_chunk(p, L, w1 + 1);
  if (clast <= cfirst) return;  // no chunks in this CTA's range (short cache, large grid)
  const int u0 = unit_of(L, cfirst), nu = unit_of(L, clast - 1) - u0 + 1;
  int *s_list = (int *)(smem + p.off_warp + 8192);  // warp 0's region, past its on-chip partial
  const int wstride = p.warp_bytes / 4;             // floats between two warps' on-chip partials
  const float *smf = (const float *)smem;

  // ---- CTA merge
  for (int k = 0; k < nu; ++k) {
    const int u = u0 + k;
    const int lo = warp_of(p, L, (int64_t)u * L.cpu);
    const int hi = warp_of(p, L, (int64_t)u * L.cpu + L.cpu - 1);
    const int wa = max(lo, w0), nw = min(hi, w1) - wa + 1;
    const bool whole = lo >= w0 && hi <= w1;
    const int fin0 = p.off_warp / 4 + (wa - w0) * wstride;  // float offset of warp wa's on-chip partial
    // where each warp's partial of u lives: its on-chip last-unit partial, the
    // CTA's on-chip boundary partial of u, or a global slot
    if (threadIdx.x < nw) {
      const int j = threadIdx.x, w = wa + j;
      int src = -1;  // float offset of the on-chip partial: [8] max, [8] sum, [8][HD] output
      if (fin_unit[w - w0] == u)
        src = fin0 + j * wstride;
      else if (k < kStrad)
        src = p.off_strad / 4 + k * kFinFloats;
      s_src[j] = src;
      s_glob[j] = src < 0;
      s_optr[j] = src >= 0 ? smf + src + 16 : p.ws_o + ((int64_t)wa + j + u) * G * HD;
    }
    __syncthreads();
    // per head: 16 lanes, one per warp (shuffle reductions stay inside each half-warp)
    if (threadIdx.x < ((G * 16 + 31) & ~31)) {  // whole warps: the shuffles use every lane
      const int hh = threadIdx.x >> 4, j = threadIdx.x & 15;
      float m = -INFINITY, l = 0.f;
      if (hh < G && j < nw) {
        if (s_glob[j]) {
          const int64_t i = ((int64_t)wa + j + u) * G + hh;
          m = p.ws_m[i];
          l = p.ws_l[i];
        } else {
          m = smf[s_src[j] + hh];
          l = smf[s_src[j] + 8 + hh];
        }
      }
      float M = m;
#pragma unroll
      for (int o = 8; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      const float f = (m == -INFINITY) ? 0.f : fast_exp2(m - M);
      float L = l * f;
#pragma unroll
      for (int o = 8; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
      if (hh < G) s_w[j][hh] = f;
      if (hh < G && j == 0) {
        s_ML[hh][0] = M;
        s_ML[hh][1] = L;
      }
    }
    __syncthreads();
    const int b = u / p.cv.H, h = u - b * p.cv.H;
    // four lanes per float4 of head dims, each summing a quarter of the warps' partials (one
    // generic load each, no branch on where the partial lives), combined by shuffles
    for (int base = 0; base < G * (HD / 4); base += blockDim.x >> 2) {
      const int item = base + (threadIdx.x >> 2), jq = threadIdx.x & 3;
      const bool valid = item < G * (HD / 4);
      const int hh = valid ? item / (HD / 4) : 0, d = valid ? (item - hh * (HD / 4)) * 4 : 0;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kMaxWarps / 4; ++r) {
        const int j = jq + 4 * r;
        if (valid && j < nw) {
          const float4 o = *reinterpret_cast<const float4 *>(s_optr[j] + hh * HD + d);
          const float w = s_w[j][hh];
          acc.x = fmaf(o.x, w, acc.x);
          acc.y = fmaf(o.y, w, acc.y);
          acc.z = fmaf(o.z, w, acc.z);
          acc.w = fmaf(o.w, w, acc.w);
        }
      }
#pragma unroll
      for (int x = 1; x < 4; x <<= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, x);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, x);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, x);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, x);
      }
      if (!valid || jq != 0) continue;
      const float M = s_ML[hh][0], L = s_ML[hh][1];
      if (whole) {
        const int64_t row = (int64_t)b * p.Hq + h * G + hh;
        const float inv = (L > 0.f) ? 1.f / L : 0.f;
        store_from_float(p.out, row * HD + d, acc.x * inv, p.out_dtype);
        store_from_float(p.out, row * HD + d + 1, acc.y * inv, p.out_dtype);
        store_from_float(p.out, row * HD + d + 2, acc.z * inv, p.out_dtype);
        store_from_float(p.out, row * HD + d + 3, acc.w * inv, p.out_dtype);
        if (p.lse_out && d == 0) p.lse_out[row] = (L > 0.f) ? (M + log2f(L)) * LN2 : -INFINITY;
      } else {
        const int64_t cs = ((int64_t)blockIdx.x + u) * G + hh;
        *reinterpret_cast<float4 *>(p.cs_o + cs * HD + d) = acc;
        if (d == 0) {
          p.cs_m[cs] = M;
          p.cs_l[cs] = L;
        }
      }
    }
    __syncthreads();
  }

  // ---- cross-CTA completion, in rounds of blockDim.x units
  for (int base = 0; base < nu; base += blockDim.x) {
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();  // the CTA's partial writes happen before the counting threads' release
    const int k = base + threadIdx.x;
    if (k < nu) {
      fence_acq_rel_gpu();  // release, cumulative over the barrier above
      const int u = u0 + k;
      const int c_lo = warp_of(p, L, (int64_t)u * L.cpu) / p.nwc;
      const int c_hi = warp_of(p, L, (int64_t)u * L.cpu + L.cpu - 1) / p.nwc;
      if (c_hi > c_lo) {
        // add first (one round trip when the word already carries this call's
        // stamp); a word with another stamp is reset to this call's by CAS,
        // and the add that hit it is recounted
        unsigned long long *w = p.done + u;
        const unsigned long long old = atomicAdd(w, 1ull);
        unsigned long long cnt = 0;
        if ((old >> 16) == p.stamp) {
          cnt = (old & 0xffffull) + 1;
        } else {
          unsigned long long cur = old + 1;
          for (int it = 0; it < (1 << 20); ++it) {
            const unsigned long long c = ((cur >> 16) == p.stamp) ? (cur & 0xffffull) : 0ull;
            const unsigned long long prev = atomicCAS(w, cur, (p.stamp << 16) | (c + 1));
            if (prev == cur) {
              cnt = c + 1;
              break;
            }
            cur = prev;
          }
        }
        if (cnt == (unsigned long long)(c_hi - c_lo + 1)) {
          s_list[atomicAdd(&s_n, 1)] = u;
          *w = 0ull;  // every CTA of u has counted: reset, so a replay of the same launch starts from zero
        }
      }
    }
    __syncthreads();
    const int n = s_n;
    if (n) fence_acq_rel_gpu();  // acquire: other CTAs' partials are read after their counts
    for (int e = 0; e < n; ++e) {
      const int u = s_list[e];
      const int c_lo = warp_of(p, L, (int64_t)u * L.cpu) / p.nwc;
      const int c_hi = warp_of(p, L, (int64_t)u * L.cpu + L.cpu - 1) / p.nwc;
      const int b = u / p.cv.H, h = u - b * p.cv.H;
      const int np = c_hi - c_lo + 1;
      for (int idx = threadIdx.x; idx < G * (HD / 4); idx += blockDim.x) {
        const int hh = idx / (HD / 4), d = (idx - hh * (HD / 4)) * 4;
        const int64_t i0 = ((int64_t)c_lo + u) * G + hh;
        float M = -INFINITY, L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        // all loads of up to 4 partials issued together, then merged (one float4 of dims per thread)
        for (int j0 = 0; j0 < np; j0 += 4) {
          float m[4], l[4];
          float4 o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const bool ok = j0 + j < np;
            const int64_t i = i0 + (int64_t)(j0 + j) * G;
            m[j] = ok ? __ldcg(p.cs_m + i) : -INFINITY;
            l[j] = ok ? __ldcg(p.cs_l + i) : 0.f;
            o[j] = ok ? __ldcg(reinterpret_cast<const float4 *>(p.cs_o + i * HD + d)) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          float Mn = M;
#pragma unroll
          for (int j = 0; j < 4; ++j) Mn = fmaxf(Mn, m[j]);
          const float fo = (M == -INFINITY) ? 0.f : fast_exp2(M - Mn);
          L *= fo;
          acc.x *= fo;
          acc.y *= fo;
          acc.z *= fo;
          acc.w *= fo;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float f = (m[j] == -INFINITY) ? 0.f : fast_exp2(m[j] - Mn);
            L += l[j] * f;
            acc.x = fmaf(o[j].x, f, acc.x);
            acc.y = fmaf(o[j].y, f, acc.y);
            acc.z = fmaf(o[j].z, f, acc.z);
            acc.w = fmaf(o[j].w, f, acc.w);
          }
          M = Mn;
        }
        const int64_t row = (int64_t)b * p.Hq + h * G + hh;
        const float inv = (L > 0.f) ? 1.f / L : 0.f;
        store_from_float(p.out, row * HD + d, acc.x * inv, p.out_dtype);
        store_from_float(p.out, row * HD + d + 1, acc.y * inv, p.out_dtype);
        store_from_float(p.out, row * HD + d + 2, acc.z * inv, p.out_dtype);
        store_from_float(p.out, row * HD + d + 3, acc.w * inv, p.out_dtype);
        if (p.lse_out && d == 0) p.lse_out[row] = (L > 0.f) ? (M + log2f(L)) * LN2 : -INFINITY;
      }
    }
    __syncthreads();
  }
}

template <class G>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwc = blockDim.x >> 5;
  uint64_t *bar = (uint64_t *)smem + warp * kBarsPerWarp;
  if (lane == 0) {
    for (int s = 0; s < kBarsPerWarp; ++s) ptx::mbar_init(&bar[s], 1);
    ptx::fence_mbar_init();
    ((int *)(smem + p.off_fin))[warp] = -1;  // warps without work contribute nothing
  }
  // inputs (query, block table, cache pages, the length) may come from the preceding kernel
  ptx::grid_dependency_wait();
  __shared__ Len s_len;
  if (threadIdx.x == 0) {
    Len L;
    L.T = (p.T_dev ? *p.T_dev : p.T) + (p.fuse ? 1 : 0);
    if (L.T < 1 || L.T > (int64_t)p.cv.max_pages * p.cv.P) {
      if (blockIdx.x == 0) atomicExch(&g_fast_error, ERR_LENGTH);
      L.T = 0;
    }
    L.cpu = (int)((L.T + p.C - 1) / p.C);
    L.tc = (int64_t)p.cv.B * p.cv.H * L.cpu;
    // A launch sized for a longer length (graph replays) has more warps than
    // this length has chunks: only the first tc of them take work, one chunk
    // or more each; every merge counts only those warps.
    L.nw = (int)(L.tc < (int64_t)p.nwarps ? (L.tc > 0 ? L.tc : 1) : (int64_t)p.nwarps);
    L.small = (uint64_t)L.tc * (uint64_t)(L.nw + 1) < (1ull << 32);
    s_len = L;
  }
  __syncthreads();
  const Len L = s_len;
  if (L.T == 0) return;  // no length: nothing written (the error word says why)
  const int wg = blockIdx.x * nwc + warp;
  if (wg < L.nw) warp_main<G>(p, L, smem, bar, wg, warp, lane);
  __syncthreads();
  finish_units(p, L, smem);
  if (p.len_rw) {  // every CTA has read the old length: the last one to finish advances it
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      unsigned long long *arrive = (unsigned long long *)(p.len_rw + 1);
      if (atomicAdd(arrive, 1ull) == gridDim.x - 1) {
        *(volatile int64_t *)p.len_rw = L.T;
        *arrive = 0ull;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static constexpr int kMaxSmem = 227 * 1024 - 1024;  // dynamic shared memory; the rest covers static use

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }
static int up128(int x) { return (x + 127) & ~127; }

using KernelFn = void (*)(Params);

// One supported (stride_k, stride_v) pair: its geometry and kernel.
struct GeoInfo {
  int sk, sv, vp, C, slot, buf;
  int off[6];  // K anchors, K codes, K scales, V anchors, V codes, V scales
  KernelFn fn;
};

template <int SK, int SV, int VP = 4>
static GeoInfo geo_info() {
  using G = Geo<SK, SV, VP>;
  return GeoInfo{SK, SV, VP, G::C, G::SLOT, G::BUF, {G::O_KF0, G::O_CD0, G::O_SC0, G::O_KF1, G::O_CD1, G::O_SC1},
                 decode_kernel<G>};
}

// Every pair the kernel takes: power-of-two strides, stride_k in {16, 32, 64}
// (one K anchor per 16-token tile), stride_v in {8, .., 64}; with physical
// 3-bit or 2-bit V rows (vp 3, 2), the Full-Throttle (64, 32) and Standard
// (32, 8) pairs.
static const GeoInfo *find_geo(int sk, int sv, int *index = nullptr, int vp = 4) {
  static const GeoInfo table[] = {
      geo_info<16, 8>(),  geo_info<16, 16>(), geo_info<16, 32>(), geo_info<16, 64>(),
      geo_info<32, 8>(),  geo_info<32, 16>(), geo_info<32, 32>(), geo_info<32, 64>(),
      geo_info<64, 8>(),  geo_info<64, 16>(), geo_info<64, 32>(), geo_info<64, 64>(),
      geo_info<64, 32, 3>(), geo_info<32, 8, 3>(), geo_info<64, 32, 2>(), geo_info<32, 8, 2>(),
  };
  for (int i = 0; i < (int)(sizeof(table) / sizeof(table[0])); ++i)
    if (table[i].sk == sk && table[i].sv == sv && table[i].vp == vp) {
      if (index) *index = i;
      return &table[i];
    }
  return nullptr;
}

// Chunk size of the fast kernel for these strides (0: not taken).
int fast_chunk_tokens(int stride_k, int stride_v, int page_tokens) {
  const GeoInfo *g = find_geo(stride_k, stride_v);
  if (!g || page_tokens % g->C) return 0;
  return g->C;
}

struct Layout {
  const GeoInfo *geo;
  int gi;  // index in the geometry table
  int C, nwc, warp_bytes, off_fin, off_strad, off_warp, total;
  int64_t phs;  // bytes per (page, head)
};

// The fast kernel reads the chunk-block layout: per (page, head, chunk) one
// block [K anchors][K codes][K scales][V anchors][V codes][V scales] of the
// kernel's geometry, the six arrays' base pointers pointing into the first
// block.  A slot is a byte image of one block.
static bool make_layout(const cq_paged_cache &c, Layout &L) {
  const int vp = c.v.code_order == CQ_ORDER_PLANES3 ? 3 : c.v.code_order == CQ_ORDER_PLANES2 ? 2 : 4;
  L.geo = find_geo(c.k.stride, c.v.stride, &L.gi, vp);
  if (!L.geo) return false;
  L.C = L.geo->C;
  if (c.page_tokens % L.C || c.k.chunk_tokens != L.C || c.v.chunk_tokens != L.C) return false;
  const cq_component *cc[2] = {&c.k, &c.v};
  const char *base = (const char *)c.k.keyframes;
  const int64_t cs = L.geo->slot;
  L.phs = c.k.keyframe_head_stride * 2;
  for (int i = 0; i < 2; ++i) {
    const cq_component &k = *cc[i];
    if (k.keyframe_chunk_stride * 2 != cs || k.code_chunk_stride * 4 != cs || k.scale_chunk_stride * 2 != cs)
      return false;
    if (k.keyframe_head_stride * 2 != L.phs || k.code_head_stride * 4 != L.phs || k.scale_head_stride * 2 != L.phs)
      return false;
    if ((const char *)k.keyframes - base != L.geo->off[3 * i] || (const char *)k.codes - base != L.geo->off[3 * i + 1] ||
        (const char *)k.scales - base != L.geo->off[3 * i + 2])
      return false;
  }
  if ((L.phs & 15) || L.phs < cs * (c.page_tokens / L.C)) return false;
  // a warp's copy slots later hold its on-chip partial; warp 0's also the unit list
  L.warp_bytes = std::max(L.geo->buf, 8192 + 4 * kMaxWarps * 32) + kQaBytes + kQnBytes;
  static_assert(kFinFloats * 4 <= 8192, "on-chip partial must fit below the unit list");
  L.off_fin = kMaxWarps * kBarsPerWarp * 8;  // after the mbarriers [warp][slot]: each warp's last unit
  L.off_strad = up128(L.off_fin + kMaxWarps * 4);
  L.off_warp = up128(L.off_strad + kStrad * kFinFloats * 4);
  if (L.warp_bytes & 15) return false;  // on-chip partials are read as float4
  L.nwc = std::min(kMaxWarps, (kMaxSmem - L.off_warp) / L.warp_bytes);
  L.total = L.off_warp + L.nwc * L.warp_bytes;
  return L.nwc >= 4;
}

bool fast_decode_supported(const cq_paged_cache &c, int n_q_heads, int q_len) {
  if (q_len != 1 || c.head_dim != HD) return false;
  if (n_q_heads % c.kv_heads) return false;
  const int gqa = n_q_heads / c.kv_heads;
  if (gqa < 1 || gqa > 8) return false;
  if (c.k.code_order != CQ_ORDER_NATURAL) return false;
  if (c.v.code_order != CQ_ORDER_MMA && c.v.code_order != CQ_ORDER_PLANES3 && c.v.code_order != CQ_ORDER_PLANES2)
    return false;
  if (c.k.scale_index != CQ_SCALE_BY_TOKEN || c.v.scale_index != CQ_SCALE_BY_TOKEN) return false;
  if (!aligned16(c.k.keyframes)) return false;
  Layout L;
  return make_layout(c, L);
}

static int sm_count() {
  static int n[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  if (!n[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) cudaGetLastError();
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

struct Plan {
  Layout L;
  int cpu, nwarps, grid;
  int64_t tc, units;
};

static Plan make_plan(const cq_paged_cache &c, int64_t T, int splits_req) {
  Plan pl;
  make_layout(c, pl.L);
  pl.cpu = (int)((T + pl.L.C - 1) / pl.L.C);
  pl.units = (int64_t)c.batch * c.kv_heads;
  pl.tc = pl.units * pl.cpu;
  int64_t w = (int64_t)sm_count() * pl.L.nwc;
  if (splits_req > 0) w = std::min<int64_t>(w, pl.units * splits_req);
  pl.nwarps = (int)std::max<int64_t>(1, std::min<int64_t>(w, pl.tc));
  pl.grid = (pl.nwarps + pl.L.nwc - 1) / pl.L.nwc;
  return pl;
}

size_t fast_decode_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req) {
  if (!fast_decode_supported(c, n_q_heads, q_len)) return 0;
  const Plan pl = make_plan(c, T, splits_req);
  const int G = n_q_heads / c.kv_heads;
  return (size_t)(pl.nwarps + pl.grid + 2 * pl.units) * G * (2 + HD) * sizeof(float) +
         (size_t)pl.units * sizeof(unsigned long long);
}

// Byte range of the per-unit completion words inside the workspace of
// run_fast_decode for this shape (0 bytes when the fast kernel does not take
// it).  A caller that reuses one workspace across shapes clears it so that
// stale partials cannot be read as this call's counts.
size_t fast_decode_done_words(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req,
                              size_t *offset) {
  *offset = 0;
  if (!fast_decode_supported(c, n_q_heads, q_len)) return 0;
  const Plan pl = make_plan(c, T, splits_req);
  const int G = n_q_heads / c.kv_heads;
  *offset = (size_t)(pl.nwarps + pl.grid + 2 * pl.units) * G * (2 + HD) * sizeof(float);
  return (size_t)pl.units * sizeof(unsigned long long);
}

int run_fast_decode(const cq_paged_cache &c, const CacheView &cv, int64_t T, const void *q, int q_dtype,
                    int n_q_heads, int64_t q_sb, int64_t q_sh, float scale, void *out, int out_dtype, float *lse_out,
                    void *ws, size_t ws_bytes, int splits_req, cudaStream_t st, const int64_t *T_dev,
                    const StepInputs *in) {
  Params p;
  p.T_dev = in ? in->len : T_dev;  // when set, T is the largest length the launch is sized for
  p.fuse = in != nullptr;
  p.len_rw = in ? in->len : nullptr;
  for (int i = 0; i < 2; ++i) {
    p.x[i] = in ? in->x[i] : nullptr;
    p.x_sb[i] = in ? in->sb[i] : 0;
    p.x_sh[i] = in ? in->sh[i] : 0;
  }
  p.x_dtype = in ? in->dtype : CQ_F16;
  p.cv = cv;
  p.q = q;
  p.q_dtype = q_dtype;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.scale = scale;
  p.gqa = n_q_heads / c.kv_heads;
  p.T = T;
  const Plan pl = make_plan(c, T, splits_req);
  const Layout &L = pl.L;
  p.C = L.C;
  p.cpp = c.page_tokens / L.C;
  p.nwarps = pl.nwarps;
  p.off_fin = L.off_fin;
  p.off_strad = L.off_strad;
  p.off_warp = L.off_warp;
  p.warp_bytes = L.warp_bytes;
  p.blk = (const char *)c.k.keyframes;
  p.phs = L.phs;
  p.nwc = L.nwc;
  const size_t slots = (size_t)(pl.nwarps + pl.units) * p.gqa;  // warp partials
  const size_t cslots = (size_t)(pl.grid + pl.units) * p.gqa;   // CTA partials
  const size_t need = (slots + cslots) * (2 + HD) * sizeof(float) + (size_t)pl.units * sizeof(unsigned long long);
  CQ_REQUIRE(ws && ws_bytes >= need, CQ_ERR_WORKSPACE, "cq_attention: workspace too small");
  CQ_REQUIRE(((uintptr_t)ws & 15) == 0, CQ_ERR_INVALID, "cq_attention: workspace must be 16-byte aligned");
  // output partials first: their rows stay 16-byte aligned for vector loads
  p.ws_o = (float *)ws;
  p.cs_o = p.ws_o + slots * HD;
  p.ws_m = p.cs_o + cslots * HD;
  p.ws_l = p.ws_m + slots;
  p.cs_m = p.ws_l + slots;
  p.cs_l = p.cs_m + cslots;
  p.done = (unsigned long long *)(p.cs_l + cslots);  // 8-byte aligned: 2 * (slots + cslots) floats precede it
  static std::atomic<unsigned long long> calls{0};
  p.stamp = (++calls) & 0xffffffffffffull;
  if (!p.stamp) p.stamp = (++calls) & 0xffffffffffffull;
  p.Hq = n_q_heads;
  p.out = out;
  p.out_dtype = out_dtype;
  p.lse_out = lse_out;

  static std::mutex mu;
  constexpr int kGeoSlots = 32;  // >= the entries of find_geo's table
  static bool attr_set[64][kGeoSlots] = {};
  const int v = L.gi;
  CQ_REQUIRE(v >= 0 && v < kGeoSlots, CQ_ERR_INVALID, "decode_kernel: geometry index out of range");
  {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev][v]) {
      cudaError_t e = cudaFuncSetAttribute(L.geo->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
      if (e != cudaSuccess)
        return set_error(CQ_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) attr_set[dev][v] = true;
    }
  }
  // launched as a programmatic dependent of the preceding kernel in the
  // stream: it may be scheduled while that kernel drains and waits
  // (griddepcontrol.wait) for its results before reading any input
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.grid);
  cfg.blockDim = dim3((unsigned)(L.nwc * 32));
  cfg.dynamicSmemBytes = (size_t)L.total;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, L.geo->fn, p);
  if (e != cudaSuccess) return set_error(CQ_ERR_CUDA, std::string("decode_kernel: ") + cudaGetErrorString(e));
  return check_launch("decode_kernel");
}

}  // namespace fast

bool fast_decode_supported(const cq_paged_cache &c, int n_q_heads, int q_len) {
  return fast::fast_decode_supported(c, n_q_heads, q_len);
}
size_t fast_decode_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req) {
  return fast::fast_decode_workspace(c, T, n_q_heads, q_len, splits_req);
}
size_t fast_decode_done_words(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req,
                              size_t *offset) {
  return fast::fast_decode_done_words(c, T, n_q_heads, q_len, splits_req, offset);
}
int run_fast_decode(const cq_paged_cache &c, const CacheView &cv, int64_t T, const void *q, int q_dtype, int n_q_heads,
                    int64_t q_sb, int64_t q_sh, float scale, void *out, int out_dtype, float *lse_out, void *ws,
                    size_t ws_bytes, int splits_req, cudaStream_t st, const int64_t *T_dev, const StepInputs *in) {
  return fast::run_fast_decode(c, cv, T, q, q_dtype, n_q_heads, q_sb, q_sh, scale, out, out_dtype, lse_out, ws,
                               ws_bytes, splits_req, st, T_dev, in);
}

// Read (and optionally clear) the device-side error word the fast kernel sets
// when a bounded wait gives up.  Synchronises the device.
int read_fast_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, fast::g_fast_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(fast::g_fast_error, &z, sizeof(int));
  }
  return v;
}

int read_bounds_error_decode(int clear) { return read_bounds_error_here(clear); }

}  // namespace cq

extern "C" int cq_decode_chunk_tokens(int32_t stride_k, int32_t stride_v, int32_t page_tokens, int32_t head_dim) {
  if (head_dim != cq::fast::HD || stride_k < 1 || stride_v < 1 || page_tokens < 1) return 0;
  return cq::fast::fast_chunk_tokens(stride_k, stride_v, page_tokens);
}

namespace cq {
int read_append_error(int clear);
namespace peer {
int read_peer_error(int clear);
}
}

extern "C" int cq_device_error(int *code, int clear) {
  if (!code) return cq::set_error(CQ_ERR_INVALID, "cq_device_error: code is null");
  const int a = cq::read_fast_error(clear), b = cq::read_append_error(clear), c = cq::read_prefill_error(clear);
  const int p = cq::peer::read_peer_error(clear);
  int d = 0;  // bounds checks of a CQ_CHECKS build
  for (int (*rd)(int) : {cq::read_bounds_error_encode, cq::read_bounds_error_layout, cq::read_bounds_error_attention,
                         cq::read_bounds_error_prefill, cq::read_bounds_error_decode}) {
    const int v = rd(clear);
    if (!d) d = v;
  }
  *code = a ? a : (b ? b : (c ? c : (p ? p : d)));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cq::set_error(CQ_ERR_CUDA, cudaGetErrorString(e));
  return CQ_OK;
}
