// cq_decode_fast.cu -- split-KV decode attention over the paged compressed
// cache, written for sm_100a.
//
// Replaces the reference's fused Metal decode kernel (kernels.py:79-228),
// which re-reads each kv-head stream once per query head and does scalar
// math.  Here one CTA streams pages of one (sequence, kv-head) unit and
// serves every query head of the GQA group from a single read:
//
//   producer warp:  1-D bulk-async copies (TMA engine) of a page's anchors,
//                   code rows and scales into a shared-memory stage, counted
//                   on an mbarrier (expect_tx); once a stage lands it computes
//                   q . K-anchor for every anchor of the page (tensor-core MMA)
//                   and releases the stage to the consumers;
//   8 consumer warps, 32 tokens each per page (the producer also expands the
//   page's per-token scales):
//     scores  S = q.anchor + scale_t * (q . codes_t)      (kernels.py:152-159)
//             q.codes: MMA with A = INT4 codes turned into exact fp16 integers
//             in registers, B = the query group;
//     softmax online, base 2, lazily rescaled (a new max is applied only when
//             it exceeds the running one by 8, so p <= 256);
//     output  O += anchor_v(t) * p_t + codes_v(t) * (p_t * scale_t)
//             both as MMAs with tokens as the reduction axis: V anchors are
//             gathered per token with ldmatrix.trans, V codes dequantise in
//             registers; P moves from the score layout to the operand layout
//             with movmatrix.trans.
//
// Work: every CTA of a persistent grid takes a balanced, contiguous range of
// the global page index (unit-major) and writes one partial (max, sum,
// unnormalised output) per unit its range touches; fast_combine merges the
// partials of each query head.
//
// Requirements (fast_decode_supported): q_len 1, head_dim 128, GQA group <= 8,
// page_tokens <= 256 and a multiple of 16, strides >= 2, V codes in the MMA
// nibble order, 16-byte aligned rows.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "cq_decode_fast.cuh"
#include "cq_ptx.cuh"

namespace cq {
namespace fast {

// consumer warps per CTA (template parameter NW): 16 (one CTA per SM) or 8
constexpr int kMaxNW = 16;
constexpr int HD = 128;             // head_dim
constexpr float TAU = 8.0f;         // lazy-rescale threshold (log2 units)
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr long long WAIT_BUDGET = 1LL << 31;  // clock cycles (~1 s) before a wait gives up
constexpr int ERR_TIMEOUT_FULL = 1, ERR_TIMEOUT_EMPTY = 2;

struct Params {
  CacheView cv;
  const void *q;
  int q_dtype;
  int64_t q_sb, q_sh;
  float scale;
  int gqa;
  int64_t T;
  int sub;            // tokens per sub-page (the pipeline unit)
  int nsub;           // sub-pages per page (1 or 2)
  int npu;            // sub-pages per (sequence, kv-head) unit
  int64_t tp;         // total sub-pages = units * npu
  int smax;           // partial slots per CTA (unit segments a CTA's page range can touch)
  int stages;
  int tpw;           // tiles (16 tokens) per consumer warp per page
  int qa_rows;       // q.anchor rows per stage (K anchors per sub-page rounded up to 16)
  // shared memory layout (bytes)
  int off_tab, off_qa, off_qb, off_merge, off_stage, stage_bytes;
  int st_kf[2], st_cd[2], st_sc[2];
  uint32_t full_bytes[6], full_total;  // bulk-copy sizes of a full sub-page
  int asub[2], rsub[2];                // anchors / code rows per full sub-page
  float *ws_m, *ws_l, *ws_o;  // [grid*smax][8], [grid*smax][8], [grid*smax][8][128]
};

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

// Per page-local token, two words of shared-memory byte offsets:
//   K: [code row offset:14][I-frame:1][0:1][q.anchor row offset:16]
//   V: [code row offset:14][I-frame:1][0:1][anchor row offset:16]
// I-frames point at code row 0; their scale is 0, so the row never counts.
constexpr uint32_t TAB_OFF = 0x3fffu, TAB_IFRAME = 0x4000u;

__device__ __forceinline__ uint2 tab_entry(int tl, int sk, int sv) {
  const int ak = tl / sk, av = tl / sv;
  const bool ik = (tl - ak * sk) == 0, iv = (tl - av * sv) == 0;
  const uint32_t ck = ik ? TAB_IFRAME : (uint32_t)((tl - ak - 1) * 64);
  const uint32_t cv = iv ? TAB_IFRAME : (uint32_t)((tl - av - 1) * 64);
  return make_uint2(ck | ((uint32_t)(ak * 32) << 16), cv | ((uint32_t)(av * 256) << 16));
}

struct CopyPlan {
  uint32_t bytes[6];
  uint32_t total;
};

// Bytes of the six bulk copies of a page holding `nvalid` tokens (only the
// anchors, code rows and 16-byte-rounded scales those tokens use).
__device__ __forceinline__ CopyPlan plan_page(const Params &p, int nvalid) {
  CopyPlan c;
  if (nvalid == p.sub) {
#pragma unroll
    for (int i = 0; i < 6; ++i) c.bytes[i] = p.full_bytes[i];
    c.total = p.full_total;
    return c;
  }
  c.total = 0;
  for (int comp = 0; comp < 2; ++comp) {
    const CompView &cc = p.cv.c[comp];
    const int a = (nvalid - 1) / cc.stride + 1;
    const int r = nvalid - a;
    c.bytes[comp * 3 + 0] = (uint32_t)a * HD * 2;
    c.bytes[comp * 3 + 1] = (uint32_t)r * (HD / 8) * 4;
    c.bytes[comp * 3 + 2] = (uint32_t)((nvalid * 2 + 15) & ~15);  // token-indexed scales
    c.total += c.bytes[comp * 3 + 0] + c.bytes[comp * 3 + 1] + c.bytes[comp * 3 + 2];
  }
  return c;
}

// Sub-pages [first, last) of the global page index (unit * npu + page) that this
// CTA processes: a contiguous, balanced share.
__device__ __forceinline__ void my_pages(const Params &p, int64_t &first, int64_t &last) {
  first = (int64_t)blockIdx.x * p.tp / gridDim.x;
  last = (int64_t)(blockIdx.x + 1) * p.tp / gridDim.x;
}

// Walks this CTA's pages in order with running counters (no per-page
// division): unit, its (sequence, head), page within the unit, partial-slot
// segment, pipeline stage and barrier phase.
struct Cursor {
  int unit, b, h, lp, seg, s;
  uint32_t ph;
  int64_t left;  // pages left including the current one
  __device__ void init(const Params &p, int64_t first, int64_t last) {
    unit = (int)(first / p.npu);
    lp = (int)(first - (int64_t)unit * p.npu);
    b = unit / p.cv.H;
    h = unit - b * p.cv.H;
    seg = 0;
    s = 0;
    ph = 0;
    left = last - first;
  }
  __device__ bool valid() const { return left > 0; }
  __device__ bool last_in_seg(const Params &p) const { return left == 1 || lp + 1 == p.npu; }
  __device__ int nvalid(const Params &p) const {
    return (int)min((int64_t)p.sub, p.T - (int64_t)lp * p.sub);
  }
  __device__ void next(const Params &p) {
    if (++lp == p.npu) {
      lp = 0;
      ++unit;
      ++seg;
      if (++h == p.cv.H) {
        h = 0;
        ++b;
      }
    }
    if (++s == p.stages) {
      s = 0;
      ph ^= 1u;
    }
    --left;
  }
};

// ---------------------------------------------------------------------------
// producer warp: bulk copies (lane 0) + q . K-anchor for each landed page
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t page_id(const Params &p, const Cursor &c) {
  return p.cv.block_table[(int64_t)c.b * p.cv.max_pages + (c.lp >> (p.nsub - 1))];
}

__device__ void issue_page(const Params &p, unsigned char *smem, uint64_t *full, const Cursor &c, int64_t pg) {
  const CacheView &cv = p.cv;
  const CopyPlan cp = plan_page(p, c.nvalid(p));
  const int sl = c.lp & (p.nsub - 1);  // which slice of the page
  unsigned char *stage = smem + p.off_stage + c.s * p.stage_bytes;
  ptx::mbar_arrive_expect_tx(&full[c.s], cp.total);
  for (int comp = 0; comp < 2; ++comp) {
    const CompView &cc = cv.c[comp];
    const int64_t ph = pg * cv.H + c.h;
    ptx::bulk_g2s(stage + p.st_kf[comp], cc.kf + (ph * cc.apg + (int64_t)sl * p.asub[comp]) * HD,
                  cp.bytes[comp * 3 + 0], &full[c.s]);
    if (cp.bytes[comp * 3 + 1])
      ptx::bulk_g2s(stage + p.st_cd[comp], cc.codes + (ph * cc.ppg + (int64_t)sl * p.rsub[comp]) * (HD / 8),
                    cp.bytes[comp * 3 + 1], &full[c.s]);
    ptx::bulk_g2s(stage + p.st_sc[comp], cc.scales + ph * cc.srow + (int64_t)sl * p.sub, cp.bytes[comp * 3 + 2],
                  &full[c.s]);
  }
}

// Copy warp (one thread): issues the bulk copies of every sub-page of this
// CTA's range, up to `stages` ahead of the consumers, and nothing else.
__device__ void copier(const Params &p, unsigned char *smem, uint64_t *full, uint64_t *empty) {
  int64_t first, last;
  my_pages(p, first, last);
  Cursor c;
  c.init(p, first, last);
  int64_t pg_next = c.valid() ? page_id(p, c) : 0;
  for (int64_t k = 0; c.valid(); ++k) {
    const int64_t pg = pg_next;
    if (k >= p.stages && !ptx::mbar_wait_bounded(&empty[c.s], c.ph ^ 1u, WAIT_BUDGET)) {
      atomicExch(&g_fast_error, ERR_TIMEOUT_EMPTY);
      // the consumers give up on their own bounded waits; copies already
      // issued complete into stages that stay resident until the CTA exits
      // only after the q.anchor warp and consumers drained them
      return;
    }
    issue_page(p, smem, full, c, pg);
    c.next(p);
    if (c.valid()) pg_next = page_id(p, c);  // next entry's load overlaps the wait above
  }
}

// q.anchor warp: once a sub-page lands, computes q . anchor for each of its
// K anchors (tensor-core MMA, rows = anchors) and marks the stage ready.
__device__ void qa_warp(const Params &p, unsigned char *smem, uint64_t *full, uint64_t *ready, int lane) {
  const CacheView &cv = p.cv;
  const int g = lane >> 2, t = lane & 3;
  int64_t first, last;
  my_pages(p, first, last);
  uint32_t qBn[8][2];
  int cur_unit = -1;
  Cursor rd;
  for (rd.init(p, first, last); rd.valid(); rd.next(p)) {
    if (rd.unit != cur_unit) {
      cur_unit = rd.unit;
      const int hq = rd.h * p.gqa + g;
      const bool real = g < p.gqa;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int d0 = 16 * kk + 2 * t;
        qBn[kk][0] = real ? ptx::pack_half2(q_scaled(p, rd.b, hq, d0), q_scaled(p, rd.b, hq, d0 + 1)) : 0u;
        qBn[kk][1] = real ? ptx::pack_half2(q_scaled(p, rd.b, hq, d0 + 8), q_scaled(p, rd.b, hq, d0 + 9)) : 0u;
      }
    }
    if (!ptx::mbar_wait_bounded(&full[rd.s], rd.ph, WAIT_BUDGET)) {
      atomicExch(&g_fast_error, ERR_TIMEOUT_FULL);
      return;
    }
    const int nvalid = rd.nvalid(p);
    const int nK = (nvalid == p.sub) ? p.asub[0] : (nvalid - 1) / cv.c[0].stride + 1;
    const unsigned char *kfK = smem + p.off_stage + rd.s * p.stage_bytes + p.st_kf[0];
    float *qa = (float *)(smem + p.off_qa) + rd.s * p.qa_rows * 8;
    const int mi = lane >> 3, rr = lane & 7;
    for (int mt = 0; mt * 16 < nK; ++mt) {
      // two accumulators halve the dependent MMA chain
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
      const int arow = min(mt * 16 + rr + ((mi & 1) ? 8 : 0), nK - 1);
      const uint32_t base = ptx::smem_u32(kfK + arow * (HD * 2) + ((mi & 2) ? 16 : 0));
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ptx::ldmatrix_x4(a0, a1, a2, a3, base + kk * 32);
        ptx::ldmatrix_x4(b0, b1, b2, b3, base + kk * 32 + 32);
        ptx::mma_f16_16816(c0, a0, a1, a2, a3, qBn[kk][0], qBn[kk][1]);
        ptx::mma_f16_16816(c1, b0, b1, b2, b3, qBn[kk + 1][0], qBn[kk + 1][1]);
      }
      float *row0 = qa + (mt * 16 + g) * 8 + 2 * t;
      row0[0] = (c0[0] + c1[0]) * LOG2E;
      row0[1] = (c0[1] + c1[1]) * LOG2E;
      row0[64] = (c0[2] + c1[2]) * LOG2E;
      row0[65] = (c0[3] + c1[3]) * LOG2E;
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&ready[rd.s]);
  }
}

// ---------------------------------------------------------------------------
// consumer warps
// ---------------------------------------------------------------------------
struct WarpState {
  float m[2];      // running max (log2 units) of heads 2t, 2t+1
  float l[2];      // this thread's partial sums
  float o[8][4];   // O^T fragments: [m-tile i][c0..c3]
};

__device__ __forceinline__ void reset(WarpState &st) {
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[i][j] = 0.f;
}

// Merge the consumer warps' states into one partial (real heads only) in
// slot `slot` of the workspace.
template <int NW>
__device__ void flush_partial(const Params &p, unsigned char *smem, WarpState &st, int64_t slot, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int G = p.gqa;
  float l0 = st.l[0], l1 = st.l[1];
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  float *wm = (float *)(smem + p.off_merge);  // [NW][8]
  float *wl = wm + NW * 8;                     // [NW][8]
  float *wo = wl + NW * 8;                     // [NW][G][HD]
  if (g == 0) {
    wm[warp * 8 + 2 * t] = st.m[0];
    wm[warp * 8 + 2 * t + 1] = st.m[1];
    wl[warp * 8 + 2 * t] = l0;
    wl[warp * 8 + 2 * t + 1] = l1;
  }
  if (2 * t < G) {
    float *w0 = wo + (warp * G + 2 * t) * HD;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w0[16 * i + g] = st.o[i][0];
      w0[16 * i + g + 8] = st.o[i][2];
    }
  }
  if (2 * t + 1 < G) {
    float *w1 = wo + (warp * G + 2 * t + 1) * HD;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w1[16 * i + g] = st.o[i][1];
      w1[16 * i + g + 8] = st.o[i][3];
    }
  }
  ptx::named_barrier_sync(1, NW * 32);
  for (int idx = threadIdx.x; idx < G * HD; idx += NW * 32) {
    const int hh = idx / HD, d = idx - (idx / HD) * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w * 8 + hh]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = wm[w * 8 + hh];
      const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
      L += wl[w * 8 + hh] * f;
      acc += wo[(w * G + hh) * HD + d] * f;
    }
    p.ws_o[(slot * 8 + hh) * HD + d] = acc;
    if (d == 0) {
      p.ws_m[slot * 8 + hh] = M;
      p.ws_l[slot * 8 + hh] = L;
    }
  }
  ptx::named_barrier_sync(1, NW * 32);
  reset(st);
}

// Shared-memory byte addresses a consumer thread uses for one page.
struct StageAddr {
  uint32_t tab;  // token table (uint2 per token)
  uint32_t scK, scV;  // token-indexed fp16 scales (0 on I-frames)
  uint32_t qa;   // q . anchor rows (8 floats per K anchor)
  uint32_t cdK, kfV, cdV;
  uint32_t qb;   // query fragments: [J][lane][4 words]
};

__device__ __forceinline__ float lds_half_as_float(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ void process_tile(WarpState &st, const StageAddr &A, float2 qc, int tb, int nvalid,
                                             int lane) {
  const int g = lane >> 2, t = lane & 3;
  // ---------------- scores S^T[token][head] = q.codes (MMA), then anchors + scale
  const uint32_t e0 = ptx::lds_u32(A.tab + (tb + g) * 8), e1 = ptx::lds_u32(A.tab + (tb + g + 8) * 8);
  const uint4 wk0 = ptx::lds_u128(A.cdK + (e0 & TAB_OFF) + t * 16);
  const uint4 wk1 = ptx::lds_u128(A.cdK + (e1 & TAB_OFF) + t * 16);
  // token-indexed scales (0 on I-frames): K in log2 units, V as stored
  const float2 sc0 = make_float2(lds_half_as_float(A.scK + (tb + g) * 2) * LOG2E, lds_half_as_float(A.scV + (tb + g) * 2));
  const float2 sc1 =
      make_float2(lds_half_as_float(A.scK + (tb + g + 8) * 2) * LOG2E, lds_half_as_float(A.scV + (tb + g + 8) * 2));
  const float2 qa0 = ptx::lds_f2(A.qa + (e0 >> 16) + t * 8);
  const float2 qa1 = ptx::lds_f2(A.qa + (e1 >> 16) + t * 8);
  float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
  {
    // raw nibble values (1024+n, 1024+16n) against q (q/16 on the 16n lanes):
    // q . codes = result - qc, qc = the same product for the all-8 word
    const uint32_t w0[4] = {wk0.x, wk0.y, wk0.z, wk0.w};
    const uint32_t w1[4] = {wk1.x, wk1.y, wk1.z, wk1.w};
#pragma unroll
    for (int J = 0; J < 4; ++J) {
      const uint4 qb = ptx::lds_u128(A.qb + J * 512);
      uint32_t h0[4], h1[4];
      ptx::nibbles_to_half2_raw(w0[J], h0);  // (d0,d4) (d1,d5) (d2,d6) (d3,d7)
      ptx::nibbles_to_half2_raw(w1[J], h1);
      ptx::mma_f16_16816(ca, h0[0], h1[0], h0[1], h1[1], qb.x, qb.y);
      ptx::mma_f16_16816(cb, h0[2], h1[2], h0[3], h1[3], qb.z, qb.w);
    }
  }
  float s0 = fmaf(sc0.x, (ca[0] + cb[0]) - qc.x, qa0.x), s1 = fmaf(sc0.x, (ca[1] + cb[1]) - qc.y, qa0.y);
  float s2 = fmaf(sc1.x, (ca[2] + cb[2]) - qc.x, qa1.x), s3 = fmaf(sc1.x, (ca[3] + cb[3]) - qc.y, qa1.y);
  if (tb + g >= nvalid) s0 = s1 = -INFINITY;
  if (tb + g + 8 >= nvalid) s2 = s3 = -INFINITY;

  // ---------------- online softmax (base 2), lazy rescale
  {
    float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
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
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        st.o[i][0] *= f0;
        st.o[i][1] *= f1;
        st.o[i][2] *= f0;
        st.o[i][3] *= f1;
      }
    }
  }
  // masked scores are -inf and the running max is finite here: ex2(-inf) = 0
  const float p0 = fast_exp2(s0 - st.m[0]);
  const float p1 = fast_exp2(s1 - st.m[1]);
  const float p2 = fast_exp2(s2 - st.m[0]);
  const float p3 = fast_exp2(s3 - st.m[1]);
  st.l[0] += p0 + p2;
  st.l[1] += p1 + p3;

  // ---------------- P (anchor term) and P' = P * scale_v (code term) as B operands
  const uint32_t bP0 = ptx::movmatrix_trans(ptx::pack_half2(p0, p1));
  const uint32_t bP1 = ptx::movmatrix_trans(ptx::pack_half2(p2, p3));
  const uint32_t bS0 = ptx::movmatrix_trans(ptx::pack_half2(p0 * sc0.y, p1 * sc0.y));
  const uint32_t bS1 = ptx::movmatrix_trans(ptx::pack_half2(p2 * sc1.y, p3 * sc1.y));

  // ---------------- V anchors: O += A_v^T P  (ldmatrix.trans gathers each token's anchor)
  {
    const int mi = lane >> 3, r = lane & 7;
    const int tok = tb + r + ((mi & 2) ? 8 : 0);
    const uint32_t aoff = (tok < nvalid) ? (ptx::lds_u32(A.tab + tok * 8 + 4) >> 16) : 0u;
    const uint32_t base = A.kfV + aoff + ((mi & 1) ? 16 : 0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t a0, a1, a2, a3;
      ptx::ldmatrix_x4_trans(a0, a1, a2, a3, base + i * 32);
      ptx::mma_f16_16816(st.o[i], a0, a1, a2, a3, bP0, bP1);
    }
  }
  // ---------------- V codes: O += C_v^T P'  (tokens 2t,2t+1 | 2t+8,2t+9; words 2g, 2g+1)
  {
    const uint4 ev = ptx::lds_u128(A.tab + (tb + 2 * t) * 8);      // entries of tokens 2t, 2t+1
    const uint4 ew = ptx::lds_u128(A.tab + (tb + 2 * t + 8) * 8);  // entries of tokens 2t+8, 2t+9
    const uint2 va = ptx::lds_u64(A.cdV + (ev.y & TAB_OFF) + g * 8);
    const uint2 vb = ptx::lds_u64(A.cdV + (ev.w & TAB_OFF) + g * 8);
    const uint2 vc = ptx::lds_u64(A.cdV + (ew.y & TAB_OFF) + g * 8);
    const uint2 vd = ptx::lds_u64(A.cdV + (ew.w & TAB_OFF) + g * 8);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint32_t wa = q ? va.y : va.x, wb = q ? vb.y : vb.x;
      const uint32_t wc = q ? vc.y : vc.x, wd = q ? vd.y : vd.x;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t sel = half ? 0x7632u : 0x5410u;
        uint32_t xa[4], xc[4];
        ptx::nibbles_to_half2(__byte_perm(wa, wb, sel), xa);  // nibbles 4*half + 0..3 of tokens (a, b)
        ptx::nibbles_to_half2(__byte_perm(wc, wd, sel), xc);
        // nibble j of word q <-> m-tile 4q + j/2, row g (+8 when j is odd)
        const int i0 = 4 * q + 2 * half;
        ptx::mma_f16_16816(st.o[i0], xa[0], xa[1], xc[0], xc[1], bS0, bS1);
        ptx::mma_f16_16816(st.o[i0 + 1], xa[2], xa[3], xc[2], xc[3], bS0, bS1);
      }
    }
  }
}

template <int NW>
__device__ void consumer(const Params &p, unsigned char *smem, uint64_t *full, uint64_t *empty, uint64_t *ready,
                         int warp, int lane) {
  const CacheView &cv = p.cv;
  const int g = lane >> 2, t = lane & 3;
  const int tile0 = warp * p.tpw;
  const int tile1 = min(tile0 + p.tpw, p.sub / 16);
  const uint32_t smem0 = ptx::smem_u32(smem);

  WarpState st;
  reset(st);
  int64_t first, last;
  my_pages(p, first, last);
  int cur_unit = -1;
  float2 qc = make_float2(0.f, 0.f);  // q . (raw values of code 0) for heads 2t, 2t+1
  StageAddr A;
  A.tab = smem0 + p.off_tab;
  A.qb = smem0 + p.off_qb + lane * 16;
  Cursor cu;
  for (cu.init(p, first, last); cu.valid(); cu.next(p)) {
    if (cu.unit != cur_unit) {
      // New query group.  Every warp writes the same fragments to the shared
      // copy (a unit changes only right after flush_partial's barriers, so no
      // warp still reads the previous group's).
      cur_unit = cu.unit;
      const int hq = cu.h * p.gqa + g;
      const bool real = g < p.gqa;
      float cc[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t *qbs = (uint32_t *)(smem + p.off_qb);
#pragma unroll
      for (int J = 0; J < 4; ++J) {
        const int d0 = 32 * t + 8 * J;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = real ? q_scaled(p, cu.b, hq, d0 + i) : 0.f;
        // query in the K-code order (k-permuted); lanes paired with 16n values carry q/16
        const uint32_t b0 = ptx::pack_half2(v[0], v[4]);
        const uint32_t b1 = ptx::pack_half2(v[1] * 0.0625f, v[5] * 0.0625f);
        const uint32_t b2 = ptx::pack_half2(v[2], v[6]);
        const uint32_t b3 = ptx::pack_half2(v[3] * 0.0625f, v[7] * 0.0625f);
        *(uint4 *)(qbs + (J * 32 + lane) * 4) = make_uint4(b0, b1, b2, b3);
        ptx::mma_f16_16816(cc, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_HI, ptx::RAW_CODE0_HI, b0, b1);
        ptx::mma_f16_16816(cc, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_LO, ptx::RAW_CODE0_HI, ptx::RAW_CODE0_HI, b2, b3);
      }
      qc = make_float2(cc[0], cc[1]);
      __syncwarp();
    }
    const int s = cu.s;
    // the bulk copies' own barrier makes their bytes visible to this thread;
    // `ready` adds the producer's q.anchor rows and per-token scales
    if (!ptx::mbar_wait_bounded(&full[s], cu.ph, WAIT_BUDGET) || !ptx::mbar_wait_bounded(&ready[s], cu.ph, WAIT_BUDGET)) {
      atomicExch(&g_fast_error, ERR_TIMEOUT_FULL);
      return;
    }
    const int nvalid = cu.nvalid(p);
    const uint32_t stage = smem0 + p.off_stage + s * p.stage_bytes;
    A.qa = smem0 + p.off_qa + s * p.qa_rows * 32;
    A.scK = stage + p.st_sc[0];
    A.scV = stage + p.st_sc[1];
    A.cdK = stage + p.st_cd[0];
    A.kfV = stage + p.st_kf[1];
    A.cdV = stage + p.st_cd[1];
    for (int tile = tile0; tile < tile1; ++tile) {
      const int tb = tile * 16;
      if (tb >= nvalid) break;
      process_tile(st, A, qc, tb, nvalid, lane);
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&empty[s]);
    if (cu.last_in_seg(p)) flush_partial<NW>(p, smem, st, (int64_t)blockIdx.x * p.smax + cu.seg, warp, lane);
  }
}

template <int NW>
__global__ void __launch_bounds__((NW + 2) * 32, NW == 8 ? 2 : 1) decode_kernel(const __grid_constant__ Params p) {
  constexpr int NT = (NW + 2) * 32;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t *full = (uint64_t *)smem;
  uint64_t *empty = full + p.stages;
  uint64_t *ready = empty + p.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], NW);
      ptx::mbar_init(&ready[s], 1);
    }
    ptx::fence_mbar_init();
  }
  uint2 *tab = (uint2 *)(smem + p.off_tab);
  for (int i = threadIdx.x; i < p.sub; i += NT) tab[i] = tab_entry(i, p.cv.c[0].stride, p.cv.c[1].stride);
  __syncthreads();
  if (warp == NW) {
    if (lane == 0) copier(p, smem, full, empty);
    return;
  }
  if (warp == NW + 1) {
    qa_warp(p, smem, full, ready, lane);
    return;
  }
  consumer<NW>(p, smem, full, empty, ready, warp, lane);
}

// Merge the partials of one (sequence, query head) row: one CTA of 128
// threads per row, thread = output dim.  The row's unit spans the page
// ranges of CTAs c_lo..c_hi; CTA c holds the unit's partial in slot
// c*smax + (unit - first unit of c).  Weights exp2(m_i - M) are computed once
// into shared memory, then every thread streams its dim with independent loads.
constexpr int kCombineMaxParts = 1024;

__device__ __forceinline__ int64_t cta_of_page(int64_t x, int64_t tp, int grid) {
  return ((x + 1) * grid + tp - 1) / tp - 1;
}

__global__ void __launch_bounds__(HD) fast_combine(const float *ws_m, const float *ws_l, const float *ws_o,
                                                   int64_t tp, int npu, int grid, int smax, int H, int gqa, int Hq,
                                                   void *out, int out_dtype, float *lse_out) {
  __shared__ float s_w[kCombineMaxParts];
  __shared__ int64_t s_slot[kCombineMaxParts];
  __shared__ float s_red[HD / 32];
  __shared__ float s_ML[2];
  const int row = blockIdx.x;  // b * Hq + hq
  const int b = row / Hq, hq = row - (row / Hq) * Hq;
  const int u = b * H + hq / gqa, hh = hq % gqa;
  const int64_t c_lo = cta_of_page((int64_t)u * npu, tp, grid);
  const int64_t c_hi = cta_of_page((int64_t)u * npu + npu - 1, tp, grid);
  const int np = (int)(c_hi - c_lo + 1);
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  // pass 1: slots and max
  float M = -INFINITY;
  for (int j = d; j < np; j += HD) {
    const int64_t c = c_lo + j;
    const int64_t first = c * tp / grid;
    const int64_t slot = c * smax + (u - first / npu);
    s_slot[j] = slot;
    M = fmaxf(M, ws_m[slot * 8 + hh]);
  }
  M = warp_max(M);
  if (lane == 0) s_red[warp] = M;
  __syncthreads();
  if (d == 0) {
    float v = s_red[0];
    for (int w = 1; w < HD / 32; ++w) v = fmaxf(v, s_red[w]);
    s_ML[0] = v;
  }
  __syncthreads();
  M = s_ML[0];
  // pass 2: weights and the denominator
  float L = 0.f;
  for (int j = d; j < np; j += HD) {
    const int64_t slot = s_slot[j];
    const float m = ws_m[slot * 8 + hh];
    const float f = (m == -INFINITY) ? 0.f : exp2f(m - M);
    s_w[j] = f;
    L += ws_l[slot * 8 + hh] * f;
  }
  L = warp_sum(L);
  __syncthreads();
  if (lane == 0) s_red[warp] = L;
  __syncthreads();
  if (d == 0) {
    float v = 0.f;
    for (int w = 0; w < HD / 32; ++w) v += s_red[w];
    s_ML[1] = v;
  }
  __syncthreads();
  L = s_ML[1];
  // pass 3: weighted sum of the partial outputs
  float a0 = 0.f, a1 = 0.f;
  int j = 0;
  for (; j + 2 <= np; j += 2) {
    a0 += ws_o[(s_slot[j] * 8 + hh) * HD + d] * s_w[j];
    a1 += ws_o[(s_slot[j + 1] * 8 + hh) * HD + d] * s_w[j + 1];
  }
  if (j < np) a0 += ws_o[(s_slot[j] * 8 + hh) * HD + d] * s_w[j];
  const float acc = a0 + a1;
  store_from_float(out, (int64_t)row * HD + d, (L > 0.f) ? acc / L : 0.f, out_dtype);
  if (lse_out && d == 0) lse_out[row] = (L > 0.f) ? (M + log2f(L)) * LN2 : -INFINITY;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Layout {
  int stages, stage_bytes, off_tab, off_qa, off_qb, off_merge, off_stage, total, qa_rows;
  int st_kf[2], st_cd[2], st_sc[2];
};

static inline int up128(int x) { return (x + 127) & ~127; }

// Sub-page size: 128 tokens when pages hold more and both strides divide 128.
static int sub_tokens(const cq_paged_cache &c) {
  if (c.page_tokens > 128 && c.page_tokens % 128 == 0 && 128 % c.k.stride == 0 && 128 % c.v.stride == 0) return 128;
  return c.page_tokens;
}

static Layout make_layout(const cq_paged_cache &c, int stages, int gqa, int NW) {
  Layout L;
  const int sub = sub_tokens(c);
  const cq_component *cc[2] = {&c.k, &c.v};
  int off = 0;
  for (int i = 0; i < 2; ++i) {
    const int a = sub / cc[i]->stride;
    L.st_kf[i] = off;
    off = up128(off + a * HD * 2);
    L.st_cd[i] = off;
    off = up128(off + (sub - a) * (HD / 8) * 4);
    L.st_sc[i] = off;
    off = up128(off + sub * 2);
  }
  L.stage_bytes = off;
  L.stages = stages;
  L.qa_rows = ((sub / c.k.stride + 15) / 16) * 16;
  L.off_tab = 128;  // mbarriers live in the first 128 bytes
  L.off_qa = up128(L.off_tab + sub * 8);
  L.off_qb = up128(L.off_qa + stages * L.qa_rows * 8 * 4);
  L.off_merge = up128(L.off_qb + 4 * 32 * 16);
  L.off_stage = up128(L.off_merge + (NW * 8 * 2 + NW * gqa * HD) * 4);
  L.total = L.off_stage + stages * L.stage_bytes;
  return L;
}

static constexpr int kMaxSmem = 227 * 1024;
static constexpr int kSmPerSm = 228 * 1024;

static int pick_stages(const cq_paged_cache &c, int gqa, int NW, int &per_sm) {
  if (NW == 8) {  // two CTAs per SM when they fit
    for (int s = 4; s >= 2; --s) {
      Layout L = make_layout(c, s, gqa, NW);
      if (2 * (L.total + 1024) <= kSmPerSm) {
        per_sm = 2;
        return s;
      }
    }
  }
  // one CTA per SM with the deepest pipeline that fits
  for (int s = 4; s >= 2; --s) {
    Layout L = make_layout(c, s, gqa, NW);
    if (L.total <= kMaxSmem) {
      per_sm = 1;
      return s;
    }
  }
  per_sm = 0;
  return 0;
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

bool fast_decode_supported(const cq_paged_cache &c, int n_q_heads, int q_len) {
  if (q_len != 1 || c.head_dim != HD) return false;
  if (n_q_heads % c.kv_heads) return false;
  const int gqa = n_q_heads / c.kv_heads;
  if (gqa < 1 || gqa > 8) return false;
  if (c.page_tokens > 256 || c.page_tokens % 16) return false;
  if (c.k.stride < 2 || c.v.stride < 2) return false;
  if (c.k.code_order != CQ_ORDER_NATURAL || c.v.code_order != CQ_ORDER_MMA) return false;
  if (c.k.scale_index != CQ_SCALE_BY_TOKEN || c.v.scale_index != CQ_SCALE_BY_TOKEN) return false;
  if (c.k.scale_row % 8 || c.v.scale_row % 8) return false;
  if (!aligned16(c.k.keyframes) || !aligned16(c.v.keyframes) || !aligned16(c.k.codes) || !aligned16(c.v.codes) ||
      !aligned16(c.k.scales) || !aligned16(c.v.scales))
    return false;
  int per_sm;
  return pick_stages(c, gqa, kMaxNW, per_sm) >= 2;
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
  int sub, npu, grid, smax, stages, per_sm, nw;
  int64_t tp;
};

// Consumer warps per CTA: 8 by default (two CTAs per SM); CQ_DECODE_WARPS=16
// selects one 16-warp CTA per SM (a tuning knob, same results).
static int pick_nw() {
  static int nw = 0;
  if (!nw) {
    const char *e = getenv("CQ_DECODE_WARPS");
    nw = (e && atoi(e) == 16) ? 16 : 8;
  }
  return nw;
}

static Plan make_plan(const cq_paged_cache &c, int64_t T, int gqa, int splits_req) {
  Plan pl;
  pl.sub = sub_tokens(c);
  pl.npu = (int)((T + pl.sub - 1) / pl.sub);
  const int64_t units = (int64_t)c.batch * c.kv_heads;
  pl.tp = units * pl.npu;
  pl.nw = pick_nw();
  pl.stages = pick_stages(c, gqa, pl.nw, pl.per_sm);
  int64_t g = (int64_t)sm_count() * std::max(1, pl.per_sm);
  if (splits_req > 0) g = std::min<int64_t>(g, units * splits_req);
  pl.grid = (int)std::max<int64_t>(1, std::min<int64_t>(g, pl.tp));
  const int64_t ppc = (pl.tp + pl.grid - 1) / pl.grid;  // sub-pages per CTA, at most
  pl.smax = (int)((ppc + pl.npu - 1) / pl.npu + 1);
  return pl;
}

size_t fast_decode_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req) {
  if (!fast_decode_supported(c, n_q_heads, q_len)) return 0;
  const Plan pl = make_plan(c, T, n_q_heads / c.kv_heads, splits_req);
  return (size_t)pl.grid * pl.smax * 8 * (2 + HD) * sizeof(float);
}

int run_fast_decode(const cq_paged_cache &c, const CacheView &cv, int64_t T, const void *q, int q_dtype,
                    int n_q_heads, int64_t q_sb, int64_t q_sh, float scale, void *out, int out_dtype, float *lse_out,
                    void *ws, size_t ws_bytes, int splits_req, cudaStream_t st) {
  Params p;
  p.cv = cv;
  p.q = q;
  p.q_dtype = q_dtype;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.scale = scale;
  p.gqa = n_q_heads / c.kv_heads;
  p.T = T;
  const Plan pl = make_plan(c, T, p.gqa, splits_req);
  p.sub = pl.sub;
  p.nsub = c.page_tokens / pl.sub;
  p.npu = pl.npu;
  p.tp = pl.tp;
  p.smax = pl.smax;
  Layout L = make_layout(c, pl.stages, p.gqa, pl.nw);
  p.stages = pl.stages;
  p.tpw = (pl.sub / 16 + pl.nw - 1) / pl.nw;
  p.qa_rows = L.qa_rows;
  p.off_tab = L.off_tab;
  p.off_qa = L.off_qa;
  p.off_qb = L.off_qb;
  p.off_merge = L.off_merge;
  p.off_stage = L.off_stage;
  p.stage_bytes = L.stage_bytes;
  for (int i = 0; i < 2; ++i) {
    p.st_kf[i] = L.st_kf[i];
    p.st_cd[i] = L.st_cd[i];
    p.st_sc[i] = L.st_sc[i];
  }
  {
    const cq_component *cc[2] = {&c.k, &c.v};
    p.full_total = 0;
    for (int i = 0; i < 2; ++i) {
      p.asub[i] = pl.sub / cc[i]->stride;
      p.rsub[i] = pl.sub - p.asub[i];
      p.full_bytes[i * 3 + 0] = (uint32_t)p.asub[i] * HD * 2;
      p.full_bytes[i * 3 + 1] = (uint32_t)p.rsub[i] * (HD / 8) * 4;
      p.full_bytes[i * 3 + 2] = (uint32_t)pl.sub * 2;
      for (int j = 0; j < 3; ++j) p.full_total += p.full_bytes[i * 3 + j];
    }
  }
  const size_t slots = (size_t)pl.grid * pl.smax;
  const size_t need = slots * 8 * (2 + HD) * sizeof(float);
  CQ_REQUIRE(ws && ws_bytes >= need, CQ_ERR_WORKSPACE, "cq_attention: workspace too small");
  p.ws_m = (float *)ws;
  p.ws_l = p.ws_m + slots * 8;
  p.ws_o = p.ws_l + slots * 8;

  static std::mutex mu;
  static bool attr_set[64][2] = {};
  {
    int dev = 0;
    cudaGetDevice(&dev);
    const int v = pl.nw == 8 ? 1 : 0;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev][v]) {
      cudaError_t e = v ? cudaFuncSetAttribute(decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)
                        : cudaFuncSetAttribute(decode_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
      if (e != cudaSuccess)
        return set_error(CQ_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) attr_set[dev][v] = true;
    }
  }
  if (pl.nw == 8)
    decode_kernel<8><<<pl.grid, (8 + 2) * 32, L.total, st>>>(p);
  else
    decode_kernel<16><<<pl.grid, (16 + 2) * 32, L.total, st>>>(p);
  int r = check_launch("decode_kernel");
  if (r) return r;
  fast_combine<<<c.batch * n_q_heads, HD, 0, st>>>(p.ws_m, p.ws_l, p.ws_o, pl.tp, pl.npu, pl.grid, pl.smax,
                                                    c.kv_heads, p.gqa, n_q_heads, out, out_dtype, lse_out);
  return check_launch("fast_combine");
}

}  // namespace fast

bool fast_decode_supported(const cq_paged_cache &c, int n_q_heads, int q_len) {
  return fast::fast_decode_supported(c, n_q_heads, q_len);
}
size_t fast_decode_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req) {
  return fast::fast_decode_workspace(c, T, n_q_heads, q_len, splits_req);
}
int run_fast_decode(const cq_paged_cache &c, const CacheView &cv, int64_t T, const void *q, int q_dtype, int n_q_heads,
                    int64_t q_sb, int64_t q_sh, float scale, void *out, int out_dtype, float *lse_out, void *ws,
                    size_t ws_bytes, int splits_req, cudaStream_t st) {
  return fast::run_fast_decode(c, cv, T, q, q_dtype, n_q_heads, q_sb, q_sh, scale, out, out_dtype, lse_out, ws,
                               ws_bytes, splits_req, st);
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

}  // namespace cq

extern "C" int cq_device_error(int *code, int clear) {
  if (!code) return cq::set_error(CQ_ERR_INVALID, "cq_device_error: code is null");
  *code = cq::read_fast_error(clear);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cq::set_error(CQ_ERR_CUDA, cudaGetErrorString(e));
  return CQ_OK;
}
