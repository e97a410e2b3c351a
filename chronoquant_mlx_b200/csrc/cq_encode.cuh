// cq_encode.cuh -- the per-token residual codec (codec.py:23-65), shared by
// the append kernel and the decode kernel's in-step encode.  Every step rounds
// to the token dtype exactly as the reference's fp16 (or bf16) MLX arithmetic
// does: fp32 arithmetic on dtype values followed by one rounding is the
// correctly rounded dtype result for + - * /.
#pragma once

#include "cq_common.cuh"

namespace cq {

constexpr int kMaxDimsPerLane = 8;  // head_dim <= 256: lane holds dims lane + 32 i

// Quantise one residual value (codec.py:48-54).  `q` is the dtype-rounded
// quotient delta/scale_safe.
__device__ __forceinline__ int quantise_code(float q, float hl, bool zero_scale) {
  if (zero_scale || isnan(q)) return 0;  // NaN (0/0) is undefined in the reference; defined as 0
  float r = rintf(q);                    // mx.round: half to even
  r = fminf(fmaxf(r, -hl), hl - 1.f);
  return (int)r;
}

// The stored value (code + 8, kernels.py:40) of one residual: the quotient
// delta / scale rounded to the token dtype, then half to even and clipped
// (codec.py:48-54).
template <int DTYPE>
__device__ __forceinline__ uint32_t code_nibble(float dv, float scale_safe, float hl, bool zero_scale) {
  const float q = round_dt(__fdiv_rn(dv, scale_safe), DTYPE);
  const int code = quantise_code(q, hl, zero_scale);
  return (uint32_t)min(max(code + 8, 0), 15);
}

// code_nibble without a division per value, for many values sharing one
// scale: r is the correctly rounded 1/scale (finite; callers scale dv and
// scale by a power of two where it is not).  rint(round_dt(q))
// differs from rint(q) only when q rounds onto a half-integer m = k + 1/2;
// those are representable with an even significand (|m| < 64), so that
// happens exactly for q in [m - h, m + h], h half a dtype ulp at m.  q' = dv*r
// is within 2^-19 of q (|q| < 16), far less than h, so m = floor(q') + 1/2 is
// the only candidate, an FMA residual dv - (m -+ h) * scale (exact product,
// exact sign) settles membership, and outside the interval rint(q') = rint(q).
template <int DTYPE>
__device__ __forceinline__ uint32_t code_nibble_rcp(float dv, float scale_safe, float r, float hl,
                                                    bool zero_scale) {
  const float q = dv * r;
  const float m = floorf(q) + 0.5f;
  constexpr int fb = (DTYPE == CQ_BF16) ? 8 : 11;  // h = 2^(e - fb) for |m| in [2^e, 2^(e+1))
  const float h = __int_as_float((__float_as_int(m) & 0x7f800000) - (fb << 23));
  const bool on_half = fmaf(-(m - h), scale_safe, dv) >= 0.f && fmaf(-(m + h), scale_safe, dv) <= 0.f;
  const int code = quantise_code(on_half ? m : q, hl, zero_scale);  // rint(m): the even neighbour
  return (uint32_t)min(max(code + 8, 0), 15);
}

// Codes and scale of one P-frame token, computed by one warp.  xv: the
// token's values (exact in DTYPE), av: its anchor's fp16 values, for dims
// lane + 32 i.  Packs the nibbles (+8 bias, kernels.py:40) of the code row in
// `order` into sw[0 .. row_words(D, order)) (warp-private shared memory) and
// returns the scale in DTYPE precision (stored as fp16 by the caller,
// cache.py:116).
template <int DTYPE>
__device__ __forceinline__ float encode_residual(const float (&xv)[kMaxDimsPerLane],
                                                 const float (&av)[kMaxDimsPerLane], int D, int bits,
                                                 float dead_zone, int order, uint32_t *sw, int lane) {
  // delta = token - anchor.astype(token.dtype), in the token dtype (cache.py:113)
  float dv[kMaxDimsPerLane];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxDimsPerLane; ++i) {
    float an = (DTYPE == CQ_BF16) ? round_dt(av[i], CQ_BF16) : av[i];
    dv[i] = round_dt(xv[i] - an, DTYPE);
    amax = fmaxf(amax, fabsf(dv[i]));
  }
  amax = warp_max(amax);

  const int hl_i = (1 << bits) / 2;
  const float hl = (float)hl_i;
  const float hlm1 = (float)(hl_i - 1);
  const float tiny = round_dt(1e-10f, DTYPE);  // 0 in fp16
  float scale = round_dt(__fdiv_rn(amax, hlm1), DTYPE);
  if (dead_zone > 0.f) {  // codec.py:36-45
    const float ratio = round_dt(dead_zone, DTYPE);
    const float thr = round_dt(amax * ratio, DTYPE);
    float amax_c = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxDimsPerLane; ++i) {
      if (fabsf(dv[i]) < thr) dv[i] = 0.f;
      amax_c = fmaxf(amax_c, fabsf(dv[i]));
    }
    amax_c = warp_max(amax_c);
    const float amax_safe = (amax_c < tiny) ? amax : amax_c;
    scale = round_dt(__fdiv_rn(amax_safe, hlm1), DTYPE);
  }
  const bool zero_scale = scale < tiny;
  const float scale_safe = zero_scale ? 1.f : scale;

  sw[lane] = 0u;
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kMaxDimsPerLane; ++i) {
    int d = lane + 32 * i;
    if (d < D) pack_code(sw, d, D, order, code_nibble<DTYPE>(dv[i], scale_safe, hl, zero_scale));
  }
  __syncwarp();
  return scale;
}

}  // namespace cq
