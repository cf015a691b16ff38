// tc.cuh - sm_100a tensor-core plumbing shared by the tcgen05 kernels: 2-D TMA loads through a tensor map,
// shared-memory matrix descriptors, tcgen05.mma / commit / fences, f16x2 arithmetic, and the driver entry point
// that encodes tensor maps (looked up once through the runtime, so the library links no libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"

namespace rb {

namespace mm4 {

// 2-D tiled TMA load global -> shared (this CTA), completion counted on `bar` in bytes. No multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load global -> shared (this CTA), completion counted on `bar` in bytes. No multicast.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory descriptor of a K-major SWIZZLE_128B operand: 8-row groups 1024 bytes apart, descriptor
// version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// cuTensorMapEncodeTiled from the driver, or nullptr. Host threads may race on the first lookup; they all
// store the same pointer.
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> fn{nullptr};
  PFN_cuTensorMapEncodeTiled_v12000 f = fn.load(std::memory_order_acquire);
  if (!f) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
      fn.store(f, std::memory_order_release);
    }
  }
  return f;
}

}  // namespace mm4

}  // namespace rb
