// cq_common.cu -- error state and cache validation shared by all entry points.
#include <cstdio>
#include <string>

#include "cq_common.cuh"

namespace cq {

static thread_local std::string g_last_error;

int set_error(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(CQ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return CQ_OK;
}

static int validate_component(const cq_paged_cache *c, const cq_component &k, const char *name) {
  std::string n(name);
  CQ_REQUIRE(k.stride >= 1, CQ_ERR_INVALID, n + ": stride must be >= 1");
  CQ_REQUIRE(c->page_tokens % k.stride == 0, CQ_ERR_INVALID, n + ": page_tokens must be a multiple of the stride");
  CQ_REQUIRE(k.anchors_per_page == c->page_tokens / k.stride, CQ_ERR_INVALID,
             n + ": anchors_per_page != page_tokens/stride");
  CQ_REQUIRE(k.pframes_per_page == c->page_tokens - k.anchors_per_page, CQ_ERR_INVALID,
             n + ": pframes_per_page != page_tokens - anchors_per_page");
  CQ_REQUIRE(k.scale_index == CQ_SCALE_BY_PFRAME || k.scale_index == CQ_SCALE_BY_TOKEN, CQ_ERR_INVALID,
             n + ": scale_index must be CQ_SCALE_BY_PFRAME or CQ_SCALE_BY_TOKEN");
  CQ_REQUIRE(k.scale_row >= (k.scale_index == CQ_SCALE_BY_TOKEN ? c->page_tokens : k.pframes_per_page),
             CQ_ERR_INVALID, n + ": scale_row too small");
  CQ_REQUIRE(k.bits >= 2 && k.bits <= 8, CQ_ERR_INVALID, n + ": bits must be in [2, 8]");
  CQ_REQUIRE(k.code_order == CQ_ORDER_NATURAL || (k.code_order == CQ_ORDER_MMA && c->head_dim % 64 == 0) ||
                 (k.code_order == CQ_ORDER_PLANES3 && c->head_dim == 128 && k.bits <= 3) ||
                 (k.code_order == CQ_ORDER_PLANES2 && c->head_dim == 128 && k.bits <= 2),
             CQ_ERR_INVALID, n + ": code_order MMA needs head_dim % 64 == 0; PLANES3 (PLANES2) needs head_dim "
                                 "128 and bits <= 3 (<= 2)");
  if (k.chunk_tokens > 0 && k.chunk_tokens != c->page_tokens) {
    CQ_REQUIRE(c->page_tokens % k.chunk_tokens == 0 && k.chunk_tokens % k.stride == 0, CQ_ERR_INVALID,
               n + ": chunk_tokens must divide page_tokens and be a multiple of the stride");
    CQ_REQUIRE(k.keyframe_chunk_stride > 0 && k.code_chunk_stride > 0 && k.scale_chunk_stride > 0, CQ_ERR_INVALID,
               n + ": chunk strides must be positive with several chunks per page");
  }
  CQ_REQUIRE(k.keyframe_head_stride >= 0 && k.code_head_stride >= 0 && k.scale_head_stride >= 0, CQ_ERR_INVALID,
             n + ": negative head stride");
  CQ_REQUIRE(k.keyframes != nullptr, CQ_ERR_INVALID, n + ": keyframes is null");
  CQ_REQUIRE(k.pframes_per_page == 0 || (k.codes != nullptr && k.scales != nullptr), CQ_ERR_INVALID,
             n + ": codes/scales null");
  return CQ_OK;
}

int validate_cache(const cq_paged_cache *c) {
  CQ_REQUIRE(c != nullptr, CQ_ERR_INVALID, "cache descriptor is null");
  CQ_REQUIRE(c->batch >= 1 && c->kv_heads >= 1, CQ_ERR_INVALID, "batch and kv_heads must be >= 1");
  CQ_REQUIRE(c->head_dim >= 8 && c->head_dim <= 256 && c->head_dim % 8 == 0, CQ_ERR_UNSUPPORTED,
             "head_dim must be a multiple of 8 in [8, 256]");
  CQ_REQUIRE(c->page_tokens >= 1, CQ_ERR_INVALID, "page_tokens must be >= 1");
  CQ_REQUIRE(c->block_table != nullptr, CQ_ERR_INVALID, "block_table is null");
  CQ_REQUIRE(c->max_pages >= 1 && c->n_pages >= 1, CQ_ERR_INVALID, "max_pages and n_pages must be >= 1");
  int r = validate_component(c, c->k, "k");
  if (r) return r;
  return validate_component(c, c->v, "v");
}

}  // namespace cq

extern "C" int cq_abi_version(void) { return CQ_ABI_VERSION; }

extern "C" const char *cq_last_error(void) { return cq::g_last_error.c_str(); }
