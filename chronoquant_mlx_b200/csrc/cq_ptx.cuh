// cq_ptx.cuh -- inline-PTX wrappers: mbarriers, bulk-async copies (the TMA
// engine's 1-D form), warp-level tensor-core MMA, ldmatrix/movmatrix and the
// bit tricks that turn packed nibbles into fp16 pairs.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace cq {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the warp sleeps (up to `ns`) until the
// phase completes instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `budget` clock cycles and returns false.  The
// clock is read once per 16 suspended tries.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, long long budget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if (clock64() - t0 > budget) return false;
  }
}

// Orders this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk copy) accesses: needed before a bulk copy refills a
// buffer that plain loads just read.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch: wait until the preceding kernel in the
// stream has completed and its memory is visible (no-op when the launch has
// no programmatic dependency), and allow the next kernel to be scheduled.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 1-D bulk copy global -> shared (32-bit shared-memory address), completion
// counted on `bar` in bytes.  Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s_a(uint32_t dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_smem),
               "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- 32-bit shared-memory loads
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return (uint32_t)v;
}
__device__ __forceinline__ uint2 lds_u64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds_u128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float2 lds_f2(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- tensor-core fragments
// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                            uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                                  uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// ---------------------------------------------------------------- nibble -> fp16
// (a & b) | c in one LOP3
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ __half2 u2h2(uint32_t x) { return *reinterpret_cast<__half2 *>(&x); }
__device__ __forceinline__ uint32_t h22u(__half2 x) { return *reinterpret_cast<uint32_t *>(&x); }

// The 16-bit halves of x each hold four nibble lanes (stored value n = code +
// 8).  Returns, for nibbles {0,1,2,3} of each half, the fp16 pair
// (half lo, half hi) of code + 72 with no arithmetic: each nibble is moved to
// bits 4-7 of its half under the fp16 exponent of 64 (0x5400, one unit in the
// last place = 1/16), which reads as 64 + n = (n - 8) + 72.
__device__ __forceinline__ void nibbles_to_half2_64(uint32_t x, uint32_t (&out)[4]) {
  const uint32_t MAGIC = 0x54005400u;
  out[0] = lop3_and_or(x << 4, 0x00f000f0u, MAGIC);
  out[1] = lop3_and_or(x, 0x00f000f0u, MAGIC);
  out[2] = lop3_and_or(x >> 4, 0x00f000f0u, MAGIC);
  out[3] = lop3_and_or(x >> 8, 0x00f000f0u, MAGIC);
}
constexpr uint32_t HALF2_72 = 0x54805480u;  // (72, 72)
constexpr uint32_t HALF2_68 = 0x54405440u;  // (68, 68)
constexpr uint32_t HALF2_66 = 0x54205420u;  // (66, 66)

// Raw nibble values under the fp16 exponent of 1024 (0x6400, one unit in the
// last place = 1): out[0], out[2] hold 1024 + n (nibbles 0 and 2 of each
// 16-bit half), out[1], out[3] hold 1024 + 16n (nibbles 1 and 3).  A dot product with these values equals the dot product
// with the codes n - 8 plus a constant that does not depend on the codes; the
// caller removes that constant (computed from the all-8 nibble pattern).
__device__ __forceinline__ void nibbles_to_half2_raw(uint32_t x, uint32_t (&out)[4]) {
  const uint32_t MAGIC = 0x64006400u;
  out[0] = lop3_and_or(x, 0x000f000fu, MAGIC);
  out[1] = lop3_and_or(x, 0x00f000f0u, MAGIC);
  const uint32_t x8 = x >> 8;
  out[2] = lop3_and_or(x8, 0x000f000fu, MAGIC);
  out[3] = lop3_and_or(x8, 0x00f000f0u, MAGIC);
}

// The raw values of the all-8 nibble word (code 0): 1032 and 1152 = 1024 + 16*8.
constexpr uint32_t RAW_CODE0_LO = 0x64086408u, RAW_CODE0_HI = 0x64806480u;

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) { return h22u(__floats2half2_rn(lo, hi)); }

}  // namespace ptx
}  // namespace cq
