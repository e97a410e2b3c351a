// cq_static_scratch.cu -- cq_attention for callers that cannot allocate.
//
// cq_attention needs a caller-provided workspace for its split-KV partials
// (per-split running max, denominator and unnormalised output).  Some callers
// have no allocator to hand at decode time: an embedding runtime whose memory
// pool is owned elsewhere, a host thread that must not take the allocator's
// lock in the middle of a token step, or a foreign-language binding that can
// only pass plain pointers it already holds.  For them this entry point takes
// the partials from one fixed array of device memory declared in this file
// (CQ_STATIC_SCRATCH_BYTES bytes per device, part of the library's module
// image) and calls cq_attention with it.  Nothing here allocates: no
// cudaMalloc / cudaFree, no allocating library routine.
//
// Set-up: the first call on a device, made with that device current, looks up
// the array's device address (cudaGetSymbolAddress) and keeps it; later calls
// on that device reuse it.  Make that first call before any stream capture.
// The kept address belongs to the device's primary context: resetting the
// device (cudaDeviceReset) while the library stays loaded is not supported.
//
// The array keeps the last call's contents.  The split partials are written
// before they are read within each call, but the decode kernel counts its
// finished CTAs in per-unit completion words whose position depends on the
// shape, so an earlier call of another shape may have left partial values
// there: each call first clears those words (cudaMemsetAsync on the caller's
// stream, which allocates nothing).
//
// One array per device is shared by every call on it.  Two calls whose work
// overlaps on the device (different streams, or different host threads on the
// same device) race on the scratch and can corrupt each other's results;
// serialise them on one stream.
#include <mutex>
#include <string>

#include "cq_common.cuh"
#include "cq_decode_fast.cuh"

namespace cq {

static __device__ __align__(256) unsigned char g_static_scratch[CQ_STATIC_SCRATCH_BYTES];

constexpr int kMaxScratchDevices = 64;

// Device address of g_static_scratch for the current device (looked up once).
static int scratch_pointer(void **out) {
  static std::mutex mu;
  static void *ptrs[kMaxScratchDevices] = {};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return set_error(CQ_ERR_CUDA, std::string("cq_attention_static_scratch: cudaGetDevice: ") + cudaGetErrorString(e));
  CQ_REQUIRE(dev >= 0 && dev < kMaxScratchDevices, CQ_ERR_UNSUPPORTED,
             "cq_attention_static_scratch: device ordinal beyond 63");
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return set_error(CQ_ERR_CUDA, std::string("cq_attention_static_scratch: cudaGetSymbolAddress: ") +
                                        cudaGetErrorString(e));
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return CQ_OK;
}

}  // namespace cq

using namespace cq;

extern "C" int cq_attention_static_scratch(const cq_paged_cache *cache, int64_t T, const void *q, int q_dtype,
                                           int32_t n_q_heads, int32_t q_len, int32_t causal, int64_t q_sb,
                                           int64_t q_sh, int64_t q_sq, float scale, void *out, int out_dtype,
                                           float *lse_out, int32_t num_splits, void *stream) {
  size_t need = 0;
  int r = cq_attention_workspace(cache, T, n_q_heads, q_len, num_splits, &need);
  if (r) return r;
  if (need > (size_t)CQ_STATIC_SCRATCH_BYTES)
    return set_error(CQ_ERR_WORKSPACE, "cq_attention_static_scratch: this shape needs " + std::to_string(need) +
                                           " bytes of split-KV scratch, more than the fixed " +
                                           std::to_string((size_t)CQ_STATIC_SCRATCH_BYTES) +
                                           "; use cq_attention with a caller-provided workspace");
  void *ws = nullptr;
  r = scratch_pointer(&ws);
  if (r) return r;
  size_t off = 0;
  const size_t done = fast_decode_done_words(*cache, T, n_q_heads, q_len, num_splits, &off);
  if (done) {  // the decode kernel's completion words start at zero (see above)
    cudaError_t e = cudaMemsetAsync((char *)ws + off, 0, done, (cudaStream_t)stream);
    if (e != cudaSuccess)
      return set_error(CQ_ERR_CUDA, std::string("cq_attention_static_scratch: cudaMemsetAsync: ") +
                                        cudaGetErrorString(e));
  }
  return cq_attention(cache, T, q, q_dtype, n_q_heads, q_len, causal, q_sb, q_sh, q_sq, scale, out, out_dtype,
                      lse_out, ws, (size_t)CQ_STATIC_SCRATCH_BYTES, num_splits, stream);
}
