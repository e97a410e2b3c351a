// cq_peer.cu -- the tensor-parallel decoder's row-parallel projection sum
// over NVLink peer memory, fused with the two operations that follow it in a
// decode step: the residual add and the next RMSNorm.
//
//   x <- x + dtype(sum_r part_r)         (every rank, the same rank order)
//   y <- dtype(x * rsqrt(mean(x^2) + eps)) * w
//
// Every rank owns one region of device memory (cq_peer_region_alloc) that
// every other rank maps through CUDA IPC (cq_peer_region_open, in the mapping
// process's own device context):
//   [flags: u32 per (row, source rank), kMaxRows x kMaxRanks]
//   [parts: parity (2) x source rank x rows x dim]
// For call e, block b of rank s pushes row b of its part (the projection's
// output, local memory) into slot s of every rank's region (NVLink stores),
// then stores e into flag (b, s) of every region (release, system scope).
// Block b of every rank waits until flags (b, 0..world-1) of its own region
// hold e or more (acquire), sums the slots of row b in rank order from local
// memory, and writes x and y.  Two part buffers alternate by call (parity): a
// rank writes a peer's buffer p again only two calls later, after the peer
// has flagged the call in between, which it does only after its reads of
// buffer p have finished (stream order).  e is a device counter advanced by
// the last block, so a captured graph replays with fresh epochs.  Waits are
// bounded: a wait that gives up records an error (cq_device_error 9) and the
// block writes nothing.
#include <cstring>
#include <string>

#include "cq_common.cuh"

namespace cq {
namespace peer {

constexpr int kMaxRanks = 8;
constexpr int kMaxRows = 64;
constexpr int kFlagBytes = kMaxRows * kMaxRanks * 4;
constexpr int kThreads = 256;
constexpr long long kSpinLimit = 1LL << 25;  // polls before giving up (seconds: the later ones sleep)
constexpr long long kBusyPolls = 1LL << 14;  // polls without sleeping: a peer a few ms late costs no sleep overshoot
constexpr int ERR_PEER_WAIT = 9;

__device__ int g_peer_error;

struct Regions {
  char *r[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 8 values of dtype dt (bf16 or fp16) from 16 bytes
__device__ __forceinline__ void unpack8(uint4 u, int dt, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 f;
    if (dt == CQ_BF16)
      f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[k]));
    else
      f = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8], int dt) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (dt == CQ_BF16) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
      w[k] = *reinterpret_cast<const uint32_t *>(&h);
    } else {
      const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
      w[k] = *reinterpret_cast<const uint32_t *>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// one block per row
__global__ void __launch_bounds__(kThreads) sum_norm_kernel(Regions R, int world, int rank, int parity,
                                                            int64_t part_bytes, int dim, const void *part, void *x,
                                                            const void *w, float eps, void *y, int64_t *ctr, int dt) {
  __shared__ uint32_t s_e;
  __shared__ int s_ok;
  __shared__ float red[kThreads / 32];
  if (threadIdx.x == 0) {
    s_e = (uint32_t)(*(volatile int64_t *)ctr + 1);
    s_ok = 1;
  }
  const int64_t row = blockIdx.x;
  const int n8 = dim / 8;
  // push this rank's row into slot `rank` of every region (parity buffer)
  const int64_t slot_off = kFlagBytes + ((int64_t)parity * world + rank) * part_bytes;
  const uint4 *src = reinterpret_cast<const uint4 *>(part) + row * n8;
  for (int c = threadIdx.x; c < n8; c += kThreads) {
    const uint4 v = src[c];
    for (int r = 0; r < world; ++r) reinterpret_cast<uint4 *>(R.r[r] + slot_off)[row * n8 + c] = v;
  }
  __syncthreads();
  const uint32_t e = s_e;
  if (threadIdx.x < world) {  // row `row` of this rank's part is in every region: flag it there
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(reinterpret_cast<uint32_t *>(R.r[threadIdx.x]) + row * kMaxRanks + rank, e);
    // wait for the row from source rank threadIdx.x in this rank's region
    const uint32_t *f = reinterpret_cast<const uint32_t *>(R.r[rank]) + row * kMaxRanks + threadIdx.x;
    long long it = 0;
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (++it > kSpinLimit) {
        atomicExch(&g_peer_error, ERR_PEER_WAIT);
        s_ok = 0;
        break;
      }
      if (it > kBusyPolls) __nanosleep(128);
    }
  }
  __syncthreads();
  if (s_ok) {
    float ss = 0.f;
    uint4 *xv = reinterpret_cast<uint4 *>(x) + row * n8;
    const char *mine = R.r[rank] + kFlagBytes + (int64_t)parity * world * part_bytes;
    for (int c = threadIdx.x; c < n8; c += kThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < world; ++r) {  // rank order: the same sum on every rank
        float v[8];
        unpack8(__ldcg(reinterpret_cast<const uint4 *>(mine + r * part_bytes) + row * n8 + c), dt, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += v[k];
      }
      float xo[8];
      unpack8(xv[c], dt, xo);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float sm = round_dt(acc[k], dt);  // the summed part, in the dtype
        xo[k] = round_dt(xo[k] + sm, dt);       // x + part (one rounding)
        ss = fmaf(xo[k], xo[k], ss);
      }
      xv[c] = pack8(xo, dt);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.f;
      t = warp_sum(t);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float rs = rsqrtf(red[0] / (float)dim + eps);
    const uint4 *wv = reinterpret_cast<const uint4 *>(w);
    uint4 *yv = reinterpret_cast<uint4 *>(y) + row * n8;
    for (int c = threadIdx.x; c < n8; c += kThreads) {
      float xo[8], wk[8], o[8];
      unpack8(xv[c], dt, xo);
      unpack8(wv[c], dt, wk);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = round_dt(xo[k] * rs, dt) * wk[k];  // (x * r).to(dtype) * w
      yv[c] = pack8(o, dt);
    }
  }
  // the last block to finish advances the epoch for the next call (every block has read it)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned long long *arrive = reinterpret_cast<unsigned long long *>(ctr + 1);
    if (atomicAdd(arrive, 1ull) == gridDim.x - 1) {
      *(volatile int64_t *)ctr = (int64_t)e;
      *arrive = 0ull;
    }
  }
}

int read_peer_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_peer_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_peer_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace peer
}  // namespace cq

using namespace cq;

static int64_t part_bytes_of(int64_t rows, int32_t dim) { return (rows * dim * 2 + 15) / 16 * 16; }

extern "C" int64_t cq_peer_region_bytes(int64_t max_rows, int32_t dim, int32_t world) {
  if (max_rows < 1 || max_rows > peer::kMaxRows || dim < 8 || world < 1 || world > peer::kMaxRanks) return 0;
  return peer::kFlagBytes + 2LL * world * part_bytes_of(max_rows, dim);
}

extern "C" int cq_peer_region_alloc(int64_t bytes, void **ptr, void *ipc_handle) {
  CQ_REQUIRE(ptr && ipc_handle && bytes > 0, CQ_ERR_INVALID, "cq_peer_region_alloc: bad arguments");
  *ptr = nullptr;
  void *p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return set_error(CQ_ERR_CUDA, "cq_peer_region_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return set_error(CQ_ERR_CUDA, "cq_peer_region_alloc: zero fill or IPC handle");
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return CQ_OK;
}

extern "C" int cq_peer_region_open(const void *ipc_handle, void **ptr) {
  CQ_REQUIRE(ptr && ipc_handle, CQ_ERR_INVALID, "cq_peer_region_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  // mapped into the calling thread's current device context, with peer access to the owner
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(CQ_ERR_CUDA, std::string("cq_peer_region_open: ") + cudaGetErrorString(e));
  return CQ_OK;
}

extern "C" int cq_peer_region_close(void *ptr) {
  if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) return set_error(CQ_ERR_CUDA, "cq_peer_region_close");
  return CQ_OK;
}

extern "C" int cq_peer_region_free(void *ptr) {
  if (ptr && cudaFree(ptr) != cudaSuccess) return set_error(CQ_ERR_CUDA, "cq_peer_region_free");
  return CQ_OK;
}

extern "C" int cq_peer_sum_norm(const uint64_t *regions, int32_t world, int32_t rank, int32_t parity, int64_t max_rows,
                                int64_t rows, int32_t dim, const void *part, void *x, const void *w, float eps, void *y,
                                int64_t *counter, int dtype, void *stream) {
  CQ_REQUIRE(regions && part && x && w && y && counter, CQ_ERR_INVALID, "cq_peer_sum_norm: null pointer");
  CQ_REQUIRE(world >= 1 && world <= peer::kMaxRanks && rank >= 0 && rank < world, CQ_ERR_INVALID,
             "cq_peer_sum_norm: need 1 <= world <= 8 and 0 <= rank < world");
  CQ_REQUIRE(parity == 0 || parity == 1, CQ_ERR_INVALID, "cq_peer_sum_norm: parity must be 0 or 1");
  CQ_REQUIRE(dtype == CQ_BF16 || dtype == CQ_F16, CQ_ERR_UNSUPPORTED, "cq_peer_sum_norm: dtype must be bf16 or f16");
  CQ_REQUIRE(dim >= 8 && dim % 8 == 0 && rows >= 1 && rows <= max_rows && max_rows <= peer::kMaxRows, CQ_ERR_INVALID,
             "cq_peer_sum_norm: dim must be a positive multiple of 8 and 1 <= rows <= max_rows <= 64");
  peer::Regions R{};
  for (int i = 0; i < world; ++i) {
    R.r[i] = reinterpret_cast<char *>(regions[i]);
    CQ_REQUIRE(R.r[i] && (regions[i] & 15) == 0, CQ_ERR_INVALID, "cq_peer_sum_norm: regions must be 16-byte aligned");
  }
  CQ_REQUIRE((((uintptr_t)part | (uintptr_t)x | (uintptr_t)w | (uintptr_t)y) & 15) == 0, CQ_ERR_INVALID,
             "cq_peer_sum_norm: part, x, w and y must be 16-byte aligned");
  peer::sum_norm_kernel<<<(unsigned)rows, peer::kThreads, 0, (cudaStream_t)stream>>>(
      R, world, rank, parity, part_bytes_of(max_rows, dim), dim, part, x, w, eps, y, counter, dtype);
  return check_launch("cq_peer_sum_norm");
}
