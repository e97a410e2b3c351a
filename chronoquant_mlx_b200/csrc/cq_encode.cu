// cq_encode.cu -- streaming encode of new K/V tokens into the paged cache.
//
// One warp per (component, sequence, kv-head, token).  A token at position t
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
  int64_t warps = 2LL * cache->batch * cache->kv_heads * S;
  int64_t blocks = (warps + kEncodeWarps - 1) / kEncodeWarps;
  CQ_REQUIRE(blocks < (1LL << 31), CQ_ERR_INVALID, std::string(who) + ": too many tokens in one call");
  cudaStream_t st = (cudaStream_t)stream;
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
