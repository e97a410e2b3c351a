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
//   8 consumer warps, 32 tokens each per page:
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
// Work is split into items of `ppi` pages of one unit; each CTA of a
// persistent grid takes a contiguous range of items and writes one partial
// (max, sum, unnormalised output) per item; fast_combine merges the partials
// of each query head.
//
// Requirements (fast_decode_supported): q_len 1, head_dim 128, GQA group <= 8,
// page_tokens <= 256 and a multiple of 16, strides >= 2, V codes in the MMA
// nibble order, 16-byte aligned rows.
#include <algorithm>
#include <mutex>
#include <string>

#include "cq_decode_fast.cuh"
#include "cq_ptx.cuh"

namespace cq {
namespace fast {

constexpr int NW = 8;               // consumer warps
constexpr int NT = (NW + 1) * 32;   // + one producer warp
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
  int n_pages_unit;  // pages per (sequence, kv-head) unit
  int ppi;           // pages per item
  int ipu;           // items per unit
  int n_items;
  int stages;
  int tpw;           // tiles (16 tokens) per consumer warp per page
  int qa_rows;       // q.anchor rows per stage (anchors per page rounded up to 16)
  // shared memory layout (bytes)
  int off_tab, off_qa, off_merge, off_stage, stage_bytes;
  int st_kf[2], st_cd[2], st_sc[2];
  float *ws_m, *ws_l, *ws_o;  // [n_items][8], [n_items][8], [n_items][8][128]
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

// Table entry per page-local token: [pfK:8][aK:8][pfV:8][aV:8], pf 255 = I-frame.
__device__ __forceinline__ uint32_t tab_entry(int tl, int sk, int sv) {
  const int ak = tl / sk, av = tl / sv;
  const int pk = (tl - ak * sk) ? (tl - ak - 1) : 255;
  const int pv = (tl - av * sv) ? (tl - av - 1) : 255;
  return (uint32_t)pk | ((uint32_t)ak << 8) | ((uint32_t)pv << 16) | ((uint32_t)av << 24);
}

struct CopyPlan {
  uint32_t bytes[6];
  uint32_t total;
};

__device__ __forceinline__ CopyPlan plan_page(const Params &p, int nvalid) {
  CopyPlan c;
  c.total = 0;
  for (int comp = 0; comp < 2; ++comp) {
    const CompView &cc = p.cv.c[comp];
    const int a = (nvalid - 1) / cc.stride + 1;
    const int r = nvalid - a;
    c.bytes[comp * 3 + 0] = (uint32_t)a * HD * 2;
    c.bytes[comp * 3 + 1] = (uint32_t)r * (HD / 8) * 4;
    c.bytes[comp * 3 + 2] = (uint32_t)((r * 2 + 15) & ~15);
    c.total += c.bytes[comp * 3 + 0] + c.bytes[comp * 3 + 1] + c.bytes[comp * 3 + 2];
  }
  return c;
}

// Items [first, last) of this CTA: a contiguous share of all items.
__device__ __forceinline__ void my_items(const Params &p, int &first, int &last) {
  first = (int)((int64_t)blockIdx.x * p.n_items / gridDim.x);
  last = (int)((int64_t)(blockIdx.x + 1) * p.n_items / gridDim.x);
}

struct PageRef {
  int item, unit, b, h, lp, last_in_item;
};

// Walk the pages of items [first, last) in order.
struct PageIter {
  const Params *p;
  int item, last, lp, lp1;
  __device__ void init(const Params &pp, int first, int last_) {
    p = &pp;
    item = first;
    last = last_;
    set_item();
  }
  __device__ void set_item() {
    if (item < last) {
      const int chunk = item % p->ipu;
      lp = chunk * p->ppi;
      lp1 = min(lp + p->ppi, p->n_pages_unit);
    }
  }
  __device__ bool valid() const { return item < last; }
  __device__ PageRef get() const {
    PageRef r;
    r.item = item;
    r.unit = item / p->ipu;
    r.b = r.unit / p->cv.H;
    r.h = r.unit - r.b * p->cv.H;
    r.lp = lp;
    r.last_in_item = (lp + 1 == lp1);
    return r;
  }
  __device__ void next() {
    if (++lp >= lp1) {
      ++item;
      set_item();
    }
  }
};

// ---------------------------------------------------------------------------
// producer warp: bulk copies (lane 0) + q . K-anchor for each landed page
// ---------------------------------------------------------------------------
__device__ void issue_page(const Params &p, unsigned char *smem, uint64_t *full, const PageRef &r, int s) {
  const CacheView &cv = p.cv;
  const int64_t pg = cv.block_table[(int64_t)r.b * cv.max_pages + r.lp];
  const int nvalid = (int)min((int64_t)cv.P, p.T - (int64_t)r.lp * cv.P);
  const CopyPlan cp = plan_page(p, nvalid);
  unsigned char *stage = smem + p.off_stage + s * p.stage_bytes;
  ptx::mbar_arrive_expect_tx(&full[s], cp.total);
  for (int comp = 0; comp < 2; ++comp) {
    const CompView &cc = cv.c[comp];
    const int64_t ph = pg * cv.H + r.h;
    ptx::bulk_g2s(stage + p.st_kf[comp], cc.kf + ph * cc.apg * HD, cp.bytes[comp * 3 + 0], &full[s]);
    if (cp.bytes[comp * 3 + 1]) {
      ptx::bulk_g2s(stage + p.st_cd[comp], cc.codes + ph * cc.ppg * (HD / 8), cp.bytes[comp * 3 + 1], &full[s]);
      ptx::bulk_g2s(stage + p.st_sc[comp], cc.scales + ph * cc.srow, cp.bytes[comp * 3 + 2], &full[s]);
    }
  }
}

__device__ void producer(const Params &p, unsigned char *smem, uint64_t *full, uint64_t *empty, uint64_t *ready,
                         int lane) {
  const CacheView &cv = p.cv;
  const int g = lane >> 2, t = lane & 3;
  int first, last;
  my_items(p, first, last);
  PageIter rd, pf;  // rd: page whose q.anchor is computed next; pf: next page to prefetch
  rd.init(p, first, last);
  pf.init(p, first, last);
  int it_pf = 0;
  bool ok = true;
  // prefetch distance stages-1
  for (; it_pf < p.stages - 1 && pf.valid(); ++it_pf, pf.next())
    if (lane == 0) issue_page(p, smem, full, pf.get(), it_pf % p.stages);

  uint32_t qBn[8][2];
  int cur_unit = -1;
  int it = 0;
  for (; rd.valid(); ++it, rd.next()) {
    const PageRef r = rd.get();
    const int s = it % p.stages;
    if (!ptx::mbar_wait_bounded(&full[s], (it / p.stages) & 1, WAIT_BUDGET)) {
      atomicExch(&g_fast_error, ERR_TIMEOUT_FULL);
      ok = false;
      break;
    }
    if (r.unit != cur_unit) {
      cur_unit = r.unit;
      const int hq = r.h * p.gqa + g;
      const bool real = g < p.gqa;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int d0 = 16 * kk + 2 * t;
        qBn[kk][0] = real ? ptx::pack_half2(q_scaled(p, r.b, hq, d0), q_scaled(p, r.b, hq, d0 + 1)) : 0u;
        qBn[kk][1] = real ? ptx::pack_half2(q_scaled(p, r.b, hq, d0 + 8), q_scaled(p, r.b, hq, d0 + 9)) : 0u;
      }
    }
    // q . anchor for every K anchor present in the page (rows = anchors)
    const int nvalid = (int)min((int64_t)cv.P, p.T - (int64_t)r.lp * cv.P);
    const int nK = (nvalid - 1) / cv.c[0].stride + 1;
    const unsigned char *kfK = smem + p.off_stage + s * p.stage_bytes + p.st_kf[0];
    float *qa = (float *)(smem + p.off_qa) + s * p.qa_rows * 8;
    const int mi = lane >> 3, rr = lane & 7;
    for (int mt = 0; mt * 16 < nK; ++mt) {
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      const int arow = min(mt * 16 + rr + ((mi & 1) ? 8 : 0), nK - 1);
      const uint32_t base = ptx::smem_u32(kfK + arow * (HD * 2) + ((mi & 2) ? 16 : 0));
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ptx::ldmatrix_x4(a0, a1, a2, a3, base + kk * 32);
        ptx::mma_f16_16816(c, a0, a1, a2, a3, qBn[kk][0], qBn[kk][1]);
      }
      float *row0 = qa + (mt * 16 + g) * 8 + 2 * t;
      row0[0] = c[0] * LOG2E;
      row0[1] = c[1] * LOG2E;
      row0[64] = c[2] * LOG2E;
      row0[65] = c[3] * LOG2E;
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&ready[s]);
    // prefetch: the stage of page it_pf was last used by page it_pf - stages = it - 1,
    // which the consumers are finishing while this page is ready for them
    if (pf.valid()) {
      const int s2 = it_pf % p.stages;
      if (lane == 0) {
        if (it_pf >= p.stages && !ptx::mbar_wait_bounded(&empty[s2], ((it_pf / p.stages) - 1) & 1, WAIT_BUDGET)) {
          atomicExch(&g_fast_error, ERR_TIMEOUT_EMPTY);
          ok = false;
        } else {
          issue_page(p, smem, full, pf.get(), s2);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        ++it;
        break;
      }
      ++it_pf;
      pf.next();
    }
  }
  if (!ok && lane == 0) {
    // drain: wait (bounded) for copies already issued into stages nobody will read
    for (int k = it; k < it_pf; ++k) ptx::mbar_wait_bounded(&full[k % p.stages], (k / p.stages) & 1, WAIT_BUDGET);
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

// Merge the consumer warps' states into one partial per item (real heads only).
__device__ void flush_item(const Params &p, unsigned char *smem, WarpState &st, int item, int warp, int lane) {
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
  // thread -> (head, dim): NW*32 = 256 threads cover 2 heads x 128 dims per round
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
    p.ws_o[((int64_t)item * 8 + hh) * HD + d] = acc;
    if (d == 0) {
      p.ws_m[(int64_t)item * 8 + hh] = M;
      p.ws_l[(int64_t)item * 8 + hh] = L;
    }
  }
  ptx::named_barrier_sync(1, NW * 32);
  reset(st);
}

__device__ __forceinline__ void process_tile(const Params &p, WarpState &st, const uint32_t *tab, const float *qa,
                                             const unsigned char *cdK, const __half *scK, const unsigned char *kfV,
                                             const unsigned char *cdV, const __half *scV, const uint32_t (&qB)[4][4],
                                             int tb, int nvalid, int lane) {
  const int g = lane >> 2, t = lane & 3;
  // ---------------- scores S^T[token][head] = q.codes (MMA), then anchors + scale
  const uint32_t e0 = tab[tb + g], e1 = tab[tb + g + 8];
  const int pk0 = e0 & 0xff, pk1 = e1 & 0xff;
  const int rk0 = (pk0 == 255) ? 0 : pk0, rk1 = (pk1 == 255) ? 0 : pk1;
  const uint4 wk0 = *(const uint4 *)(cdK + rk0 * 64 + t * 16);
  const uint4 wk1 = *(const uint4 *)(cdK + rk1 * 64 + t * 16);
  float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const uint32_t w0[4] = {wk0.x, wk0.y, wk0.z, wk0.w};
    const uint32_t w1[4] = {wk1.x, wk1.y, wk1.z, wk1.w};
#pragma unroll
    for (int J = 0; J < 4; ++J) {
      uint32_t h0[4], h1[4];
      ptx::nibbles_to_half2(w0[J], h0);  // (d0,d4) (d1,d5) (d2,d6) (d3,d7)
      ptx::nibbles_to_half2(w1[J], h1);
      ptx::mma_f16_16816(ca, h0[0], h1[0], h0[1], h1[1], qB[J][0], qB[J][1]);
      ptx::mma_f16_16816(cb, h0[2], h1[2], h0[3], h1[3], qB[J][2], qB[J][3]);
    }
  }
  const float sk0 = (pk0 == 255) ? 0.f : __half2float(scK[rk0]) * LOG2E;
  const float sk1 = (pk1 == 255) ? 0.f : __half2float(scK[rk1]) * LOG2E;
  const float2 qa0 = *(const float2 *)(qa + ((e0 >> 8) & 0xff) * 8 + 2 * t);
  const float2 qa1 = *(const float2 *)(qa + ((e1 >> 8) & 0xff) * 8 + 2 * t);
  float s0 = fmaf(sk0, ca[0] + cb[0], qa0.x), s1 = fmaf(sk0, ca[1] + cb[1], qa0.y);
  float s2 = fmaf(sk1, ca[2] + cb[2], qa1.x), s3 = fmaf(sk1, ca[3] + cb[3], qa1.y);
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
  const int pv0 = (e0 >> 16) & 0xff, pv1 = (e1 >> 16) & 0xff;
  const float sv0 = (pv0 == 255) ? 0.f : __half2float(scV[pv0]);
  const float sv1 = (pv1 == 255) ? 0.f : __half2float(scV[pv1]);
  const uint32_t bP0 = ptx::movmatrix_trans(ptx::pack_half2(p0, p1));
  const uint32_t bP1 = ptx::movmatrix_trans(ptx::pack_half2(p2, p3));
  const uint32_t bS0 = ptx::movmatrix_trans(ptx::pack_half2(p0 * sv0, p1 * sv0));
  const uint32_t bS1 = ptx::movmatrix_trans(ptx::pack_half2(p2 * sv1, p3 * sv1));

  // ---------------- V anchors: O += A_v^T P  (ldmatrix.trans gathers each token's anchor)
  {
    const int mi = lane >> 3, r = lane & 7;
    const int tok = tb + r + ((mi & 2) ? 8 : 0);
    const int av = (tok < nvalid) ? (int)(tab[tok] >> 24) : 0;
    const uint32_t base = ptx::smem_u32(kfV + av * (HD * 2) + ((mi & 1) ? 16 : 0));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t a0, a1, a2, a3;
      ptx::ldmatrix_x4_trans(a0, a1, a2, a3, base + i * 32);
      ptx::mma_f16_16816(st.o[i], a0, a1, a2, a3, bP0, bP1);
    }
  }
  // ---------------- V codes: O += C_v^T P'  (tokens 2t,2t+1 | 2t+8,2t+9; words 2g, 2g+1)
  {
    const uint2 ea = *(const uint2 *)(tab + tb + 2 * t);
    const uint2 ec = *(const uint2 *)(tab + tb + 2 * t + 8);
    int ra = (ea.x >> 16) & 0xff, rb = (ea.y >> 16) & 0xff;
    int rc = (ec.x >> 16) & 0xff, rd = (ec.y >> 16) & 0xff;
    ra = (ra == 255) ? 0 : ra;
    rb = (rb == 255) ? 0 : rb;
    rc = (rc == 255) ? 0 : rc;
    rd = (rd == 255) ? 0 : rd;
    const uint2 va = *(const uint2 *)(cdV + ra * 64 + g * 8);
    const uint2 vb = *(const uint2 *)(cdV + rb * 64 + g * 8);
    const uint2 vc = *(const uint2 *)(cdV + rc * 64 + g * 8);
    const uint2 vd = *(const uint2 *)(cdV + rd * 64 + g * 8);
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

__device__ void consumer(const Params &p, unsigned char *smem, uint64_t *full, uint64_t *empty, uint64_t *ready,
                         int warp, int lane) {
  const CacheView &cv = p.cv;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t *tab = (const uint32_t *)(smem + p.off_tab);
  const int tiles_page = cv.P / 16;
  const int tile0 = warp * p.tpw;
  const int tile1 = min(tile0 + p.tpw, tiles_page);

  WarpState st;
  reset(st);
  int first, last;
  my_items(p, first, last);
  PageIter pi;
  pi.init(p, first, last);
  int cur_unit = -1;
  uint32_t qB[4][4];  // query in the K-code order (k-permuted)
  for (int it = 0; pi.valid(); ++it, pi.next()) {
    const PageRef r = pi.get();
    if (r.unit != cur_unit) {
      cur_unit = r.unit;
      const int hq = r.h * p.gqa + g;
      const bool real = g < p.gqa;
#pragma unroll
      for (int J = 0; J < 4; ++J) {
        const int d0 = 32 * t + 8 * J;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = real ? q_scaled(p, r.b, hq, d0 + i) : 0.f;
        qB[J][0] = ptx::pack_half2(v[0], v[4]);
        qB[J][1] = ptx::pack_half2(v[1], v[5]);
        qB[J][2] = ptx::pack_half2(v[2], v[6]);
        qB[J][3] = ptx::pack_half2(v[3], v[7]);
      }
    }
    const int s = it % p.stages;
    // the bulk copies' own barrier makes their bytes visible to this thread;
    // `ready` adds the producer's q.anchor rows
    if (!ptx::mbar_wait_bounded(&full[s], (it / p.stages) & 1, WAIT_BUDGET) ||
        !ptx::mbar_wait_bounded(&ready[s], (it / p.stages) & 1, WAIT_BUDGET)) {
      atomicExch(&g_fast_error, ERR_TIMEOUT_FULL);
      return;
    }
    const int nvalid = (int)min((int64_t)cv.P, p.T - (int64_t)r.lp * cv.P);
    const unsigned char *stage = smem + p.off_stage + s * p.stage_bytes;
    const float *qa = (const float *)(smem + p.off_qa) + s * p.qa_rows * 8;
    for (int tile = tile0; tile < tile1; ++tile) {
      const int tb = tile * 16;
      if (tb >= nvalid) break;
      process_tile(p, st, tab, qa, stage + p.st_cd[0], (const __half *)(stage + p.st_sc[0]), stage + p.st_kf[1],
                   stage + p.st_cd[1], (const __half *)(stage + p.st_sc[1]), qB, tb, nvalid, lane);
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&empty[s]);
    if (r.last_in_item) flush_item(p, smem, st, r.item, warp, lane);
  }
}

__global__ void __launch_bounds__(NT, 2) decode_kernel(const __grid_constant__ Params p) {
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
  uint32_t *tab = (uint32_t *)(smem + p.off_tab);
  for (int i = threadIdx.x; i < p.cv.P; i += NT) tab[i] = tab_entry(i, p.cv.c[0].stride, p.cv.c[1].stride);
  __syncthreads();
  if (warp == NW) {
    producer(p, smem, full, empty, ready, lane);
    return;
  }
  consumer(p, smem, full, empty, ready, warp, lane);
}

// Merge the item partials of one (sequence, query head) row: one CTA of 128
// threads per row, thread = output dim.  The per-item weights exp2(m_i - M)/L
// are computed once into shared memory, then every thread streams its dim of
// the item outputs with independent loads.
constexpr int kCombineMaxItems = 1024;

__global__ void __launch_bounds__(HD) fast_combine(const float *ws_m, const float *ws_l, const float *ws_o, int ipu,
                                                   int H, int gqa, int Hq, void *out, int out_dtype, float *lse_out) {
  __shared__ float s_w[kCombineMaxItems];
  __shared__ float s_red[HD / 32];
  __shared__ float s_ML[2];
  const int row = blockIdx.x;  // b * Hq + hq
  const int b = row / Hq, hq = row - (row / Hq) * Hq;
  const int u = b * H + hq / gqa, hh = hq % gqa;
  const int64_t i0 = (int64_t)u * ipu;
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  // pass 1: max over items
  float M = -INFINITY;
  for (int j = d; j < ipu; j += HD) M = fmaxf(M, ws_m[(i0 + j) * 8 + hh]);
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
  for (int j = d; j < ipu; j += HD) {
    const float m = ws_m[(i0 + j) * 8 + hh];
    const float f = (m == -INFINITY) ? 0.f : exp2f(m - M);
    s_w[j] = f;
    L += ws_l[(i0 + j) * 8 + hh] * f;
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
  // pass 3: weighted sum of the item outputs
  const float *o = ws_o + (i0 * 8 + hh) * HD + d;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int j = 0;
  for (; j + 4 <= ipu; j += 4) {
    a0 += o[(int64_t)(j + 0) * 8 * HD] * s_w[j + 0];
    a1 += o[(int64_t)(j + 1) * 8 * HD] * s_w[j + 1];
    a2 += o[(int64_t)(j + 2) * 8 * HD] * s_w[j + 2];
    a3 += o[(int64_t)(j + 3) * 8 * HD] * s_w[j + 3];
  }
  for (; j < ipu; ++j) a0 += o[(int64_t)j * 8 * HD] * s_w[j];
  const float acc = (a0 + a1) + (a2 + a3);
  store_from_float(out, (int64_t)row * HD + d, (L > 0.f) ? acc / L : 0.f, out_dtype);
  if (lse_out && d == 0) lse_out[row] = (L > 0.f) ? (M + log2f(L)) * LN2 : -INFINITY;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Layout {
  int stages, stage_bytes, off_tab, off_qa, off_merge, off_stage, total, qa_rows;
  int st_kf[2], st_cd[2], st_sc[2];
};

static inline int up128(int x) { return (x + 127) & ~127; }

static Layout make_layout(const cq_paged_cache &c, int stages, int gqa) {
  Layout L;
  const cq_component *cc[2] = {&c.k, &c.v};
  int off = 0;
  for (int i = 0; i < 2; ++i) {
    L.st_kf[i] = off;
    off = up128(off + cc[i]->anchors_per_page * HD * 2);
    L.st_cd[i] = off;
    off = up128(off + cc[i]->pframes_per_page * (HD / 8) * 4);
    L.st_sc[i] = off;
    off = up128(off + cc[i]->scale_row * 2);
  }
  L.stage_bytes = off;
  L.stages = stages;
  L.qa_rows = ((c.k.anchors_per_page + 15) / 16) * 16;
  L.off_tab = 128;  // mbarriers live in the first 128 bytes
  L.off_qa = up128(L.off_tab + c.page_tokens * 4);
  L.off_merge = up128(L.off_qa + stages * L.qa_rows * 8 * 4);
  L.off_stage = up128(L.off_merge + (NW * 8 * 2 + NW * gqa * HD) * 4);
  L.total = L.off_stage + stages * L.stage_bytes;
  return L;
}

static constexpr int kMaxSmem = 227 * 1024;
static constexpr int kSmPerSm = 228 * 1024;

static int pick_stages(const cq_paged_cache &c, int gqa, int &per_sm) {
  // prefer two CTAs per SM (16 consumer warps), then the deepest pipeline
  for (int s = 4; s >= 2; --s) {
    Layout L = make_layout(c, s, gqa);
    if (2 * (L.total + 1024) <= kSmPerSm) {
      per_sm = 2;
      return s;
    }
  }
  for (int s = 4; s >= 2; --s) {
    Layout L = make_layout(c, s, gqa);
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
  if (c.k.scale_row % 8 || c.v.scale_row % 8) return false;
  if (!aligned16(c.k.keyframes) || !aligned16(c.v.keyframes) || !aligned16(c.k.codes) || !aligned16(c.v.codes) ||
      !aligned16(c.k.scales) || !aligned16(c.v.scales))
    return false;
  int per_sm;
  return pick_stages(c, gqa, per_sm) >= 2;
}

static int items_plan(const cq_paged_cache &c, int64_t T, int splits_req, int &ppi, int &ipu) {
  const int npu = (int)((T + c.page_tokens - 1) / c.page_tokens);
  ppi = 2;
  if (splits_req > 0) ppi = std::max(1, (npu + splits_req - 1) / splits_req);
  ppi = std::max(ppi, (npu + kCombineMaxItems - 1) / kCombineMaxItems);  // the combine holds <= 1024 weights
  ipu = (npu + ppi - 1) / ppi;
  return npu;
}

size_t fast_decode_workspace(const cq_paged_cache &c, int64_t T, int n_q_heads, int q_len, int splits_req) {
  if (!fast_decode_supported(c, n_q_heads, q_len)) return 0;
  int ppi, ipu;
  items_plan(c, T, splits_req, ppi, ipu);
  const size_t items = (size_t)c.batch * c.kv_heads * ipu;
  return items * 8 * (2 + HD) * sizeof(float);
}

static int sm_count() {
  static int n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
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
  p.n_pages_unit = items_plan(c, T, splits_req, p.ppi, p.ipu);
  p.n_items = c.batch * c.kv_heads * p.ipu;
  int per_sm = 0;
  const int stages = pick_stages(c, p.gqa, per_sm);
  Layout L = make_layout(c, stages, p.gqa);
  p.stages = stages;
  p.tpw = (c.page_tokens / 16 + NW - 1) / NW;
  p.qa_rows = L.qa_rows;
  p.off_tab = L.off_tab;
  p.off_qa = L.off_qa;
  p.off_merge = L.off_merge;
  p.off_stage = L.off_stage;
  p.stage_bytes = L.stage_bytes;
  for (int i = 0; i < 2; ++i) {
    p.st_kf[i] = L.st_kf[i];
    p.st_cd[i] = L.st_cd[i];
    p.st_sc[i] = L.st_sc[i];
  }
  const size_t need = (size_t)p.n_items * 8 * (2 + HD) * sizeof(float);
  CQ_REQUIRE(ws && ws_bytes >= need, CQ_ERR_WORKSPACE, "cq_attention: workspace too small");
  p.ws_m = (float *)ws;
  p.ws_l = p.ws_m + (size_t)p.n_items * 8;
  p.ws_o = p.ws_l + (size_t)p.n_items * 8;

  static std::mutex mu;
  static bool attr_set[64] = {};
  {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
      if (e != cudaSuccess)
        return set_error(CQ_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
  }
  const int grid = std::min(p.n_items, sm_count() * per_sm);
  decode_kernel<<<grid, NT, L.total, st>>>(p);
  int r = check_launch("decode_kernel");
  if (r) return r;
  fast_combine<<<c.batch * n_q_heads, HD, 0, st>>>(p.ws_m, p.ws_l, p.ws_o, p.ipu, c.kv_heads, p.gqa, n_q_heads,
                                                    out, out_dtype, lse_out);
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
