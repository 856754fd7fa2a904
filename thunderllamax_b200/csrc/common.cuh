// Device helpers shared by the verify-path kernels (sm_100a only).
//
// * 1-D bulk copies (cp.async.bulk, the TMA engine's untiled form) from HBM into
//   shared memory, completing on an mbarrier with a transaction count.  No
//   cluster multicast anywhere in this library.
// * Bounded mbarrier waits: every spin gives up after a fixed number of polls,
//   raises a bit in the caller's error word and lets the kernel finish
//   without touching the stage that never arrived.
// * fp16x2 helpers on raw 32-bit registers for the exact-integer dequantisers.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#ifndef __CUDA_ARCH__
#define TLX_HOST_ONLY 1
#endif

namespace tlx {

// error bits written to the workspace error word
enum : uint32_t {
  ERR_MBAR_TIMEOUT = 1u,   // a bulk copy never completed within the poll budget
  ERR_BAD_PARAM = 2u,      // device-side parameter check failed
  ERR_PEER_TIMEOUT = 4u,   // a peer's flag never arrived within the poll budget
};

constexpr uint32_t kMbarPollLimit = 1u << 22;  // polls of <= kTryWaitHintNs each: a few seconds at most

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// one poll; true once the phase with the given parity has completed.  A thread
// whose phase is still open is suspended for up to kTryWaitHintNs (it resumes as
// soon as the phase completes), so waiting warps leave the issue slots to others.
constexpr uint32_t kTryWaitHintNs = 1000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kTryWaitHintNs)
      : "memory");
  return ok != 0;
}

// bounded wait; returns false (and raises ERR_MBAR_TIMEOUT) if it gave up
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err) {
  for (uint32_t i = 0; i < kMbarPollLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, ERR_MBAR_TIMEOUT);
  return false;
}

// global -> shared bulk copy of `bytes` (multiple of 16, both ends 16-B aligned)
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// programmatic dependent launch: wait for the preceding grid in the stream to
// complete (and its memory to be visible); allow the next grid to start launching
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// order this thread's generic-proxy shared accesses before later async-proxy ones
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ uint2 lds64(const void* p) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ uint32_t lds32(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(smem_u32(p)));
  return v;
}

// ---- fp16x2 on raw registers (intrinsics, so the compiler can fold constants) ----
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) { return h2_bits(__hadd2(bits_h2(a), bits_h2(b))); }
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) { return h2_bits(__hmul2(bits_h2(a), bits_h2(b))); }
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  return h2_bits(__hfma2(bits_h2(a), bits_h2(b), bits_h2(c)));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- argmax keys ----
// key = order(v) << 32 | (0xFFFFFFFF - idx): u64 max picks the largest value and,
// among equal values, the LOWEST index.  Only v > -1e30 is a candidate (the
// reference scans start from best = -1e30 with a strict '>': NaN, -inf and
// anything <= -1e30 never win, and a row without a candidate yields index 0,
// engine/amx3.cu:124-128, engine/h_argmax.cu:20-24); those map to key 0.  -0 is
// folded onto +0 so signed zeros tie like they compare.
__device__ __forceinline__ uint64_t argmax_key(float v, uint32_t idx) {
  if (!(v > -1e30f)) return 0ull;
  v = v + 0.0f;
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ float key_value(uint64_t key) {
  if (key == 0ull) return __uint_as_float(0x7FC00000u);
  uint32_t u = static_cast<uint32_t>(key >> 32);
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(u);
}
__device__ __forceinline__ int32_t key_index(uint64_t key) {
  if (key == 0ull) return 0;
  return static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
}

}  // namespace tlx
