// cq_decode_fast.cu -- placeholder until the sm_100a decode kernel lands.
#include "cq_decode_fast.cuh"

namespace cq {

bool fast_decode_supported(const cq_paged_cache &, int, int) { return false; }
size_t fast_decode_workspace(const cq_paged_cache &, int64_t, int, int, int) { return 0; }
int run_fast_decode(const cq_paged_cache &, const CacheView &, int64_t, const void *, int, int, int64_t, int64_t,
                    float, void *, int, float *, void *, size_t, int, cudaStream_t) {
  return set_error(CQ_ERR_UNSUPPORTED, "fast decode not built");
}

}  // namespace cq
