// cq_layout.cu -- reconstruction, reference-layout state export/import and the
// flat codec / pack / unpack entry points (the reference's codec.py and
// kernels.py helpers on device buffers).
#include "cq_common.cuh"

namespace cq {

// ---------------------------------------------------------------------------
// reconstruct (cache.py:131-156): one warp per (b, h, t)
// ---------------------------------------------------------------------------
__global__ void reconstruct_kernel(CacheView cv, int comp, int64_t T, __half *out, int mode) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)cv.B * cv.H * T;
  if (row >= rows) return;
  const int64_t t = row % T;
  const int h = (int)((row / T) % cv.H);
  const int b = (int)(row / (T * cv.H));
  const CompView &c = cv.c[comp];
  TokLoc L = locate(cv, comp, b, h, t);
  for (int d = lane; d < cv.D; d += 32) {
    __half a = L.anchor[d];
    // I-frames: anchor + 0 as the reference's where(is_pframe, delta, 0) sum does (-0.0 becomes +0.0)
    __half v = __hadd_rn(a, __float2half_rn(0.f));
    if (L.codes) {
      int code = nibble_at(L.codes, d, cv.D, c.order) - 8;
      __half s = __float2half_rn(L.scale);
      if (mode == 0)  // fp16(code) * scale in fp16, then anchor + that in fp16 (two roundings, no FMA)
        v = __hadd_rn(a, __hmul_rn(__int2half_rn(code), s));
      else
        v = __float2half_rn(fmaf((float)code, L.scale, __half2float(a)));
    }
    out[row * cv.D + d] = v;
  }
}

// ---------------------------------------------------------------------------
// state export / import (cache.py:220-255), reference layout, natural order
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t pframe_token(int64_t j, int stride) {
  // j-th P-frame (0-based) in token order: each anchor group holds stride-1
  return (j / (stride - 1)) * stride + (j % (stride - 1)) + 1;
}

__global__ void export_kernel(CacheView cv, int comp, int64_t nkf, int64_t npf, __half *kf_out, uint32_t *pk_out,
                              __half *sc_out, int import_dir) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t per_bh = nkf + npf;
  const int64_t rows = (int64_t)cv.B * cv.H * per_bh;
  if (row >= rows) return;
  const int64_t i = row % per_bh;
  const int h = (int)((row / per_bh) % cv.H);
  const int b = (int)(row / (per_bh * cv.H));
  const CompView &c = cv.c[comp];
  const int D = cv.D, W = words_of(D);
  const int64_t bh = (int64_t)b * cv.H + h;
  if (i < nkf) {
    const int64_t t = i * c.stride;
    TokLoc L = locate(cv, comp, b, h, t);
    __half *dst = kf_out + (bh * nkf + i) * D;
    __half *cache_row = const_cast<__half *>(L.anchor);
    for (int d = lane; d < D; d += 32) {
      if (import_dir)
        cache_row[d] = dst[d];
      else
        dst[d] = cache_row[d];
    }
    return;
  }
  const int64_t j = i - nkf;
  const int64_t t = pframe_token(j, c.stride);
  const int64_t lp = t / cv.P;
  const int tl = (int)(t - lp * cv.P);
  const int64_t pg = page_of(cv, b, lp);
  const int a = tl / c.stride;
  const int pf = tl - a - 1;
  uint32_t *crow = const_cast<uint32_t *>(c.codes) + code_index(c, cv.H, row_words(D, c.order), pg, h, pf);
  __half *cscale = const_cast<__half *>(c.scales) + scale_index(c, cv.H, pg, h, c.stok ? tl : pf);
  uint32_t *rrow = pk_out + (bh * npf + j) * W;
  if (lane < W) {
    // natural word `lane` holds dims 8*lane .. 8*lane+7
    if (!import_dir) {
      uint32_t w = 0;
      for (int k = 0; k < 8; ++k) {
        int d = lane * 8 + k;
        if (d < D) w |= (uint32_t)nibble_at(crow, d, D, c.order) << (4 * k);
      }
      rrow[lane] = w;
    }
  }
  if (import_dir) {
    // gather the natural-order row, then write the cache-order row
    __shared__ uint32_t s_w[8][32];
    uint32_t *sw = s_w[(threadIdx.x >> 5) & 7];
    sw[lane] = 0u;
    __syncwarp();
    for (int d = lane; d < D; d += 32) {
      uint32_t nib = (rrow[d >> 3] >> ((d & 7) * 4)) & 0xFu;
      pack_code(sw, d, D, c.order, nib);
    }
    __syncwarp();
    if (lane < row_words(D, c.order)) crow[lane] = sw[lane];
    if (lane == 0) *cscale = sc_out[bh * npf + j];
  } else if (lane == 0) {
    sc_out[bh * npf + j] = *cscale;
  }
}

// ---------------------------------------------------------------------------
// flat codec (codec.py:23-73): one warp per row, any dim
// ---------------------------------------------------------------------------
__global__ void quantize_kernel(const void *delta, int dtype, int64_t rows, int dim, int bits, float dz,
                                int8_t *codes, __half *scales) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t base = row * dim;
  float amax = 0.f;
  for (int d = lane; d < dim; d += 32) amax = fmaxf(amax, fabsf(load_as_float(delta, base + d, dtype)));
  amax = warp_max(amax);
  const int hl_i = (1 << bits) / 2;
  const float hl = (float)hl_i, hlm1 = (float)(hl_i - 1);
  const float tiny = round_dt(1e-10f, dtype);
  float scale = round_dt(__fdiv_rn(amax, hlm1), dtype);
  float thr = -1.f;
  if (dz > 0.f) {
    thr = round_dt(amax * round_dt(dz, dtype), dtype);
    float amax_c = 0.f;
    for (int d = lane; d < dim; d += 32) {
      float v = load_as_float(delta, base + d, dtype);
      if (fabsf(v) < thr) v = 0.f;
      amax_c = fmaxf(amax_c, fabsf(v));
    }
    amax_c = warp_max(amax_c);
    scale = round_dt(__fdiv_rn((amax_c < tiny) ? amax : amax_c, hlm1), dtype);
  }
  const bool zero_scale = scale < tiny;
  const float ss = zero_scale ? 1.f : scale;
  for (int d = lane; d < dim; d += 32) {
    float v = load_as_float(delta, base + d, dtype);
    if (dz > 0.f && fabsf(v) < thr) v = 0.f;
    float q = round_dt(__fdiv_rn(v, ss), dtype);
    int code = 0;
    if (!zero_scale && !isnan(q)) code = (int)fminf(fmaxf(rintf(q), -hl), hl - 1.f);
    codes[base + d] = (int8_t)code;
  }
  if (lane == 0) scales[row] = __float2half_rn(scale);
}

__global__ void dequantize_kernel(const int8_t *codes, const __half *scales, int64_t rows, int dim, __half *out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * dim) return;
  out[i] = __hmul_rn(__int2half_rn((int)codes[i]), scales[i / dim]);
}

__global__ void pack_kernel(const int8_t *codes, int64_t rows, int dim, uint32_t *packed) {
  const int W = words_of(dim);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * W) return;
  const int64_t r = i / W;
  const int w = (int)(i - r * W);
  uint32_t v = 0;
  for (int k = 0; k < 8; ++k) {
    int d = w * 8 + k;
    if (d < dim) {
      int nib = min(max((int)codes[r * dim + d] + 8, 0), 15);  // kernels.py:40
      v |= (uint32_t)nib << (4 * k);
    }
  }
  packed[i] = v;
}

__global__ void unpack_kernel(const uint32_t *packed, int64_t rows, int dim, int8_t *codes) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * dim) return;
  const int64_t r = i / dim;
  const int d = (int)(i - r * dim);
  uint32_t w = packed[r * words_of(dim) + (d >> 3)];
  codes[i] = (int8_t)((int)((w >> ((d & 7) * 4)) & 0xFu) - 8);
}

inline unsigned blocks_for(int64_t threads, int bs) { return (unsigned)((threads + bs - 1) / bs); }

int read_bounds_error_layout(int clear) { return read_bounds_error_here(clear); }

}  // namespace cq

using namespace cq;

extern "C" int cq_reconstruct(const cq_paged_cache *cache, int component, int64_t T, void *out, int mode,
                              void *stream) {
  int r = validate_cache(cache);
  if (r) return r;
  CQ_REQUIRE(component == 0 || component == 1, CQ_ERR_INVALID, "cq_reconstruct: component must be 0 or 1");
  CQ_REQUIRE(out && T >= 0, CQ_ERR_INVALID, "cq_reconstruct: bad output");
  CQ_REQUIRE((T + cache->page_tokens - 1) / cache->page_tokens <= cache->max_pages, CQ_ERR_INVALID,
             "cq_reconstruct: T beyond mapped pages");
  if (T == 0) return CQ_OK;
  int64_t threads = (int64_t)cache->batch * cache->kv_heads * T * 32;
  reconstruct_kernel<<<blocks_for(threads, 256), 256, 0, (cudaStream_t)stream>>>(make_view(*cache), component, T,
                                                                                   (__half *)out, mode);
  return check_launch("reconstruct_kernel");
}

static int export_import(const cq_paged_cache *cache, int component, int64_t T, void *kf, uint32_t *pk, void *sc,
                         int dir, void *stream) {
  int r = validate_cache(cache);
  if (r) return r;
  CQ_REQUIRE(component == 0 || component == 1, CQ_ERR_INVALID, "state: component must be 0 or 1");
  CQ_REQUIRE(T >= 0, CQ_ERR_INVALID, "state: T < 0");
  CQ_REQUIRE((T + cache->page_tokens - 1) / cache->page_tokens <= cache->max_pages, CQ_ERR_INVALID,
             "state: T beyond mapped pages");
  if (T == 0) return CQ_OK;
  const cq_component &c = component ? cache->v : cache->k;
  int64_t nkf = (T - 1) / c.stride + 1;
  int64_t npf = T - nkf;
  CQ_REQUIRE(kf && (npf == 0 || (pk && sc)), CQ_ERR_INVALID, "state: null buffer");
  int64_t threads = (int64_t)cache->batch * cache->kv_heads * (nkf + npf) * 32;
  export_kernel<<<blocks_for(threads, 256), 256, 0, (cudaStream_t)stream>>>(make_view(*cache), component, nkf, npf,
                                                                              (__half *)kf, pk, (__half *)sc, dir);
  return check_launch("export_kernel");
}

extern "C" int cq_export_state(const cq_paged_cache *cache, int component, int64_t T, void *keyframes,
                               uint32_t *packed, void *scales, void *stream) {
  return export_import(cache, component, T, keyframes, packed, scales, 0, stream);
}

extern "C" int cq_import_state(const cq_paged_cache *cache, int component, int64_t T, const void *keyframes,
                               const uint32_t *packed, const void *scales, void *stream) {
  return export_import(cache, component, T, const_cast<void *>(keyframes), const_cast<uint32_t *>(packed),
                       const_cast<void *>(scales), 1, stream);
}

extern "C" int cq_quantize_delta(const void *delta, int dtype, int64_t rows, int32_t dim, int32_t bits,
                                 float dead_zone, int8_t *codes, void *scales, void *stream) {
  CQ_REQUIRE(delta && codes && scales, CQ_ERR_INVALID, "cq_quantize_delta: null pointer");
  CQ_REQUIRE(dtype == CQ_F16 || dtype == CQ_BF16, CQ_ERR_UNSUPPORTED, "cq_quantize_delta: dtype must be f16/bf16");
  CQ_REQUIRE(bits >= 2 && bits <= 8, CQ_ERR_INVALID, "cq_quantize_delta: bits must be in [2, 8]");
  CQ_REQUIRE(rows >= 0 && dim >= 1, CQ_ERR_INVALID, "cq_quantize_delta: bad sizes");
  if (rows == 0) return CQ_OK;
  quantize_kernel<<<blocks_for(rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(delta, dtype, rows, dim, bits,
                                                                                 dead_zone, codes, (__half *)scales);
  return check_launch("quantize_kernel");
}

extern "C" int cq_dequantize_delta(const int8_t *codes, const void *scales, int64_t rows, int32_t dim, void *out,
                                   void *stream) {
  CQ_REQUIRE(codes && scales && out, CQ_ERR_INVALID, "cq_dequantize_delta: null pointer");
  CQ_REQUIRE(rows >= 0 && dim >= 1, CQ_ERR_INVALID, "cq_dequantize_delta: bad sizes");
  if (rows == 0) return CQ_OK;
  dequantize_kernel<<<blocks_for(rows * dim, 256), 256, 0, (cudaStream_t)stream>>>(codes, (const __half *)scales,
                                                                                   rows, dim, (__half *)out);
  return check_launch("dequantize_kernel");
}

extern "C" int cq_pack_int4(const int8_t *codes, int64_t rows, int32_t dim, uint32_t *packed, void *stream) {
  CQ_REQUIRE(codes && packed, CQ_ERR_INVALID, "cq_pack_int4: null pointer");
  CQ_REQUIRE(rows >= 0 && dim >= 1, CQ_ERR_INVALID, "cq_pack_int4: bad sizes");
  if (rows == 0) return CQ_OK;
  pack_kernel<<<blocks_for(rows * words_of(dim), 256), 256, 0, (cudaStream_t)stream>>>(codes, rows, dim, packed);
  return check_launch("pack_kernel");
}

extern "C" int cq_unpack_int4(const uint32_t *packed, int64_t rows, int32_t dim, int8_t *codes, void *stream) {
  CQ_REQUIRE(codes && packed, CQ_ERR_INVALID, "cq_unpack_int4: null pointer");
  CQ_REQUIRE(rows >= 0 && dim >= 1, CQ_ERR_INVALID, "cq_unpack_int4: bad sizes");
  if (rows == 0) return CQ_OK;
  unpack_kernel<<<blocks_for(rows * dim, 256), 256, 0, (cudaStream_t)stream>>>(packed, rows, dim, codes);
  return check_launch("unpack_kernel");
}
