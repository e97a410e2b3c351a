// cq_decoder_ops.cu -- the elementwise steps of the decoder that drives the
// compressed cache end to end (bench config 5), fused so that a decode
// step is a handful of kernels per layer instead of dozens of small ones:
//
//   cq_rmsnorm        y = bf16(x * rsqrt(mean(x^2) + eps)) * w        (per row)
//   cq_qk_norm_rope   per head of a fused QKV row: RMSNorm over head_dim
//                     (q and k), then rotate-half RoPE at one position;
//                     q, k, v written as contiguous [B][H][D]
//   cq_silu_mul       y = bf16(silu(g)) * u                          (SwiGLU)
//
// Each keeps the rounding points of the equivalent torch expression in
// bf16/fp16: products in fp32, one rounding to the tensor dtype after each
// torch op.  Only the order of the fp32 sum of squares differs from torch's
// reduction, so a value can land one dtype ulp away.
#include "cq_common.cuh"

namespace cq {
namespace dec {

__device__ __forceinline__ float ld(const void *p, int64_t i, int dt) { return load_as_float(p, i, dt); }
__device__ __forceinline__ float rnd(float x, int dt) { return round_dt(x, dt); }

// one block per row, 256 threads
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void *x, const void *w, void *y, int dim, float eps,
                                                      int dt) {
  const int64_t row = blockIdx.x;
  const int64_t base = row * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += 256) {
    const float v = ld(x, base + i, dt);
    ss = fmaf(v, v, ss);
  }
  __shared__ float red[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += 256) {
    const float n = rnd(ld(x, base + i, dt) * r, dt);            // (x * rsqrt(...)).to(dtype)
    store_from_float(y, base + i, n * ld(w, i, dt), dt);         // * w  (one rounding)
  }
}

// one warp per (row b, head h) of the fused QKV row: heads [0, Hq) are q,
// [Hq, Hq+Hkv) k, [Hq+Hkv, Hq+2Hkv) v.  head_dim 128: lane l holds dims
// 4l..4l+3, the rotate-half partner of dim i < 64 is i + 64 (lane l ^ 16).
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const void *qkv, int64_t row_stride, int B, int Hq, int Hkv,
                                                           const void *wq, const void *wk, const float *inv_freq,
                                                           const int64_t *pos, float eps, void *q_out, void *k_out,
                                                           void *v_out, int dt) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int H = Hq + 2 * Hkv;
  if (gw >= (int64_t)B * H) return;
  const int b = (int)(gw / H), h = (int)(gw - (int64_t)b * H);
  constexpr int D = 128;
  const int64_t src = (int64_t)b * row_stride + (int64_t)h * D + 4 * lane;
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = ld(qkv, src + i, dt);
  if (h >= Hq + Hkv) {  // v: copied
    const int64_t dst = ((int64_t)b * Hkv + (h - Hq - Hkv)) * D + 4 * lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) store_from_float(v_out, dst + i, x[i], dt);
    return;
  }
  const bool is_q = h < Hq;
  const void *w = is_q ? wq : wk;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = rnd(rnd(x[i] * r, dt) * ld(w, 4 * lane + i, dt), dt);  // RMSNorm as above
  const float p = (float)*pos;
  const bool lo = lane < 16;
  float out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float partner = __shfl_xor_sync(0xffffffffu, n[i], 16);
    const int d = 4 * lane + i;
    const float ang = p * inv_freq[d & 63];
    const float rot = lo ? rnd(-partner, dt) : partner;  // cat(-x[64:], x[:64])
    out[i] = __fadd_rn(__fmul_rn(n[i], cosf(ang)), __fmul_rn(rot, sinf(ang)));  // x*cos + rot*sin, unfused
  }
  const int64_t dst = is_q ? ((int64_t)b * Hq + h) * D + 4 * lane : ((int64_t)b * Hkv + (h - Hq)) * D + 4 * lane;
  void *o = is_q ? q_out : k_out;
#pragma unroll
  for (int i = 0; i < 4; ++i) store_from_float(o, dst + i, out[i], dt);
}

// gu: [rows][2*ffn] (gate | up); y: [rows][ffn]
__global__ void silu_mul_kernel(const void *gu, void *y, int64_t rows, int ffn, int dt) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * ffn) return;
  const int64_t r = i / ffn, c = i - r * ffn;
  const float g = ld(gu, r * 2 * ffn + c, dt), u = ld(gu, r * 2 * ffn + ffn + c, dt);
  const float s = rnd(g / (1.f + expf(-g)), dt);  // silu(g) in the tensor dtype
  store_from_float(y, i, s * u, dt);
}

}  // namespace dec
}  // namespace cq

using namespace cq;

extern "C" int cq_rmsnorm(const void *x, const void *w, void *y, int64_t rows, int32_t dim, float eps, int dtype,
                          void *stream) {
  CQ_REQUIRE(x && w && y && rows >= 0 && dim >= 1, CQ_ERR_INVALID, "cq_rmsnorm: bad arguments");
  CQ_REQUIRE(dtype == CQ_F16 || dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_rmsnorm: dtype must be f16/bf16");
  if (rows == 0) return CQ_OK;
  CQ_REQUIRE(rows < (1LL << 31), CQ_ERR_INVALID, "cq_rmsnorm: too many rows");
  dec::rmsnorm_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(x, w, y, dim, eps, dtype);
  return check_launch("cq_rmsnorm");
}

extern "C" int cq_qk_norm_rope(const void *qkv, int64_t row_stride, int32_t batch, int32_t n_q_heads,
                               int32_t n_kv_heads, int32_t head_dim, const void *q_norm_w, const void *k_norm_w,
                               const float *inv_freq, const int64_t *pos, float eps, void *q_out, void *k_out,
                               void *v_out, int dtype, void *stream) {
  CQ_REQUIRE(qkv && q_norm_w && k_norm_w && inv_freq && pos && q_out && k_out && v_out, CQ_ERR_INVALID,
             "cq_qk_norm_rope: null pointer");
  CQ_REQUIRE(head_dim == 128, CQ_ERR_UNSUPPORTED, "cq_qk_norm_rope: head_dim must be 128");
  CQ_REQUIRE(dtype == CQ_F16 || dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_qk_norm_rope: dtype must be f16/bf16");
  CQ_REQUIRE(batch >= 1 && n_q_heads >= 1 && n_kv_heads >= 1, CQ_ERR_INVALID, "cq_qk_norm_rope: bad sizes");
  const int64_t warps = (int64_t)batch * (n_q_heads + 2 * n_kv_heads);
  dec::qk_norm_rope_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      qkv, row_stride, batch, n_q_heads, n_kv_heads, q_norm_w, k_norm_w, inv_freq, pos, eps, q_out, k_out, v_out,
      dtype);
  return check_launch("cq_qk_norm_rope");
}

extern "C" int cq_silu_mul(const void *gu, void *y, int64_t rows, int32_t ffn, int dtype, void *stream) {
  CQ_REQUIRE(gu && y && rows >= 0 && ffn >= 1, CQ_ERR_INVALID, "cq_silu_mul: bad arguments");
  CQ_REQUIRE(dtype == CQ_F16 || dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_silu_mul: dtype must be f16/bf16");
  const int64_t n = rows * ffn;
  if (n == 0) return CQ_OK;
  CQ_REQUIRE((n + 255) / 256 < (1LL << 31), CQ_ERR_INVALID, "cq_silu_mul: too large");
  dec::silu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(gu, y, rows, ffn, dtype);
  return check_launch("cq_silu_mul");
}
