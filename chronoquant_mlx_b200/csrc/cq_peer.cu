// cq_peer.cu -- the tensor-parallel decoder's row-parallel projection sum
// over NVLink peer memory, fused with the two operations that follow it in a
// decode step: the residual add and the next RMSNorm.
//
//   x <- x + bf16(sum_r part_r)         (every rank, the same rank order)
//   y <- bf16(x * rsqrt(mean(x^2) + eps)) * w
//
// Every rank owns one region of device memory that the other ranks map (CUDA
// IPC, opened by the host): [flags: 64 x u32][part buffer 0][part buffer 1].
// A rank's projection GEMM writes its part into buffer (call parity) of its
// own region; the kernel then signals "part of call e ready" by storing e
// into flag slot `rank` of every peer's region (release, system scope), waits
// until every peer's slot in its own region holds e or more (acquire), reads
// the row from all regions over NVLink, and writes x and y locally.  Two part
// buffers alternate by call: a rank overwrites buffer p only two calls later,
// after every peer has signalled the call in between, which it does only once
// its reads of buffer p are done (stream order).  e is a device counter that
// the last block advances, so a captured graph replays with fresh epochs.
// Waits are bounded: a wait that gives up records an error (cq_device_error)
// and the block returns without writing.
#include "cq_common.cuh"

namespace cq {
namespace peer {

constexpr int kMaxRanks = 8;
constexpr int kFlagBytes = 256;
constexpr int kThreads = 256;
constexpr long long kSpinLimit = 1LL << 25;  // polls of 64 ns sleep: seconds, then give up
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
__global__ void __launch_bounds__(kThreads) sum_norm_kernel(Regions R, int world, int rank, int64_t part_off,
                                                            int dim, void *x, const void *w, float eps, void *y,
                                                            int64_t *ctr, int dt) {
  __shared__ uint32_t s_e;
  __shared__ int s_ok;
  __shared__ float red[kThreads / 32];
  if (threadIdx.x == 0) {
    s_e = (uint32_t)(*(volatile int64_t *)ctr + 1);
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_e;
  if (blockIdx.x == 0 && threadIdx.x < world) {
    // this rank's part of call e is complete (written before this kernel began): tell every rank
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(reinterpret_cast<uint32_t *>(R.r[threadIdx.x]) + rank, e);
  }
  if (threadIdx.x < world && threadIdx.x != rank) {
    const uint32_t *f = reinterpret_cast<const uint32_t *>(R.r[rank]) + threadIdx.x;
    long long it = 0;
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (++it > kSpinLimit) {
        atomicExch(&g_peer_error, ERR_PEER_WAIT);
        s_ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  const int64_t row = blockIdx.x;
  const int n8 = dim / 8;
  if (s_ok) {
    float ss = 0.f;
    uint4 *xv = reinterpret_cast<uint4 *>(x) + row * n8;
    for (int c = threadIdx.x; c < n8; c += kThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < world; ++r) {  // rank order: the same sum on every rank
        const uint4 *src = reinterpret_cast<const uint4 *>(R.r[r] + part_off) + row * n8 + c;
        float v[8];
        unpack8(__ldcv(src), dt, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += v[k];
      }
      float xo[8];
      unpack8(xv[c], dt, xo);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float s = round_dt(acc[k], dt);  // the all-reduced part, in the dtype
        xo[k] = round_dt(xo[k] + s, dt);       // x + part (one rounding)
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

extern "C" int cq_peer_sum_norm(const uint64_t *regions, int32_t world, int32_t rank, int32_t parity,
                                int64_t part_bytes, int64_t rows, int32_t dim, void *x, const void *w, float eps,
                                void *y, int64_t *counter, int dtype, void *stream) {
  CQ_REQUIRE(regions && x && w && y && counter, CQ_ERR_INVALID, "cq_peer_sum_norm: null pointer");
  CQ_REQUIRE(world >= 1 && world <= peer::kMaxRanks && rank >= 0 && rank < world, CQ_ERR_INVALID,
             "cq_peer_sum_norm: need 1 <= world <= 8 and 0 <= rank < world");
  CQ_REQUIRE(parity == 0 || parity == 1, CQ_ERR_INVALID, "cq_peer_sum_norm: parity must be 0 or 1");
  CQ_REQUIRE(dtype == CQ_BF16 || dtype == CQ_F16, CQ_ERR_UNSUPPORTED, "cq_peer_sum_norm: dtype must be bf16 or f16");
  CQ_REQUIRE(dim > 0 && dim % 8 == 0 && rows > 0 && rows < (1LL << 31), CQ_ERR_INVALID,
             "cq_peer_sum_norm: dim must be a positive multiple of 8, rows in [1, 2^31)");
  CQ_REQUIRE(rows * dim * 2 <= part_bytes && part_bytes % 16 == 0, CQ_ERR_INVALID,
             "cq_peer_sum_norm: a part (rows x dim) exceeds the region's part buffer");
  peer::Regions R{};
  for (int i = 0; i < world; ++i) {
    R.r[i] = reinterpret_cast<char *>(regions[i]);
    CQ_REQUIRE(R.r[i] && (regions[i] & 15) == 0, CQ_ERR_INVALID, "cq_peer_sum_norm: regions must be 16-byte aligned");
  }
  CQ_REQUIRE((((uintptr_t)x | (uintptr_t)w | (uintptr_t)y) & 15) == 0, CQ_ERR_INVALID,
             "cq_peer_sum_norm: x, w and y must be 16-byte aligned");
  const int64_t off = peer::kFlagBytes + (int64_t)parity * part_bytes;
  peer::sum_norm_kernel<<<(unsigned)rows, peer::kThreads, 0, (cudaStream_t)stream>>>(R, world, rank, off, dim, x, w,
                                                                                     eps, y, counter, dtype);
  return check_launch("cq_peer_sum_norm");
}

extern "C" int64_t cq_peer_region_bytes(int64_t part_bytes) {
  return part_bytes <= 0 ? 0 : peer::kFlagBytes + 2 * ((part_bytes + 15) / 16 * 16);
}
