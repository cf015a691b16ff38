// common.cuh - sm_100a device helpers shared by the GEMV and prefill kernels: mbarriers with bounded
// waits, 1-D bulk async copies (TMA without a tensor map), programmatic-dependent-launch controls and the
// warp-level f16 MMA used as an fp32-accumulating dot-product engine.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <mutex>

namespace rb {

// Device-side error word: a kernel that gives up a bounded wait ORs a bit in here and returns early.
// The host reads and clears it with rb_get_device_error(). The library is one translation unit
// (rumik_b200.cu), so this single definition is shared by every kernel.
__device__ unsigned int g_device_error;

enum : unsigned int {
  ERR_GEMV4_FULL = 1u << 0,   // int4 GEMV consumer timed out waiting for a weight stage
  ERR_GEMV4_EMPTY = 1u << 1,  // int4 GEMV producer timed out waiting for a free slot
  ERR_GEMV8_FULL = 1u << 2,
  ERR_GEMV8_EMPTY = 1u << 3,
  ERR_MM4_WAIT = 1u << 4,     // prefill matmul timed out on an mbarrier
  ERR_MULTI_FULL = 1u << 5,   // multi-GEMV consumer timed out waiting for a tile
  ERR_MULTI_EMPTY = 1u << 6,  // multi-GEMV producer timed out waiting for ring space
  ERR_TC_WAIT = 1u << 7,      // tensor-core multi-GEMV timed out on an mbarrier
  ERR_TP_WAIT = 1u << 8,      // tensor-parallel reduction timed out waiting for a peer's flag
  ERR_ARG = 1u << 9,          // a device-side argument (a decode position) was out of range; nothing stored
  ERR_ATT_WAIT = 1u << 10,    // a fused-attention launch timed out waiting for the attention outputs
  ERR_STEP_WAIT = 1u << 11,   // the whole-step kernel gave up a wait (and aborted the launch)
};

// Upper bound on the wall time of one wait (an mbarrier phase, a peer's flag, a completion counter). Healthy
// waits here last microseconds (at most the duration of the previous GEMV when a kernel starts early under PDL);
// four seconds means the wait is hung. The limit in force is g_wait_limit_ns, per device, set by
// rb_set_wait_limit (a test lowers it to make a wait that nothing will satisfy run out quickly).
constexpr unsigned long long kMaxWaitNs = 4000000000ull;
__device__ unsigned long long g_wait_limit_ns = kMaxWaitNs;

// The limit, read once per wait that does not complete at its first test.
__device__ __forceinline__ unsigned long long wait_limit_ns() {
  return *const_cast<volatile unsigned long long*>(&g_wait_limit_ns);
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Arrive `count` times at once (release semantics at CTA scope, like the single arrive).
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(count)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Non-blocking test of an mbarrier phase (try_wait may suspend the thread until the phase completes or a time
// limit passes; test_wait returns at once): for a thread that polls several barriers in turn.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and sets `err_bit` in g_device_error) if the phase did
// not complete within the wait limit; the caller then skips its work and returns, so the context stays usable.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int err_bit) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns(), lim = wait_limit_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > lim) {
      atomicOr(&g_device_error, err_bit);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared (this CTA), completion counted on `bar` in bytes. dst, src and bytes
// must be multiples of 16. No tensor map, no multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch controls (no-ops when the kernel was launched without the attribute).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" :::);
}

// Named barrier among `nthreads` threads (multiple of 32) with id `id` (1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// D(16x8,f32) += A(16x16,f16) * B(16x8,f16); fragments in the standard m16n8k16 register layout:
// a0:(g, 2t..2t+1) a1:(g+8, 2t..) a2:(g, 2t+8..) a3:(g+8, 2t+8..), b0:(k=2t.., n=g) b1:(k=2t+8.., n=g),
// d0,d1:(g, 2t..2t+1) d2,d3:(g+8, 2t..2t+1), with g = lane/4, t = lane%4. A pure register operation (not
// volatile), so the compiler may interleave independent MMAs with other work.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B + C with C given as four separate (input-only) registers.
__device__ __forceinline__ void mma_f16_16816_c(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1, const float4& c) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c.x), "f"(c.y), "f"(c.z), "f"(c.w));
}

// Same with a zero accumulator input: D = A * B.
__device__ __forceinline__ void mma_f16_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// (a & b) | c in one LOP3. Callers pass b and c as runtime values (kernel parameters), not literals: with
// two immediate operands the compiler emits two instructions for this expression.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Shared-memory loads by 32-bit shared address. The "memory" clobber keeps them after the mbarrier wait that
// guards the data; ptxas still schedules them freely against the arithmetic.
__device__ __forceinline__ uint4 lds128_a(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ float4 lds128f_a(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a) : "memory");
  return v;
}
// Forms with a compile-time byte offset folded into the address (no separate address arithmetic).
template <int OFF>
__device__ __forceinline__ uint4 lds128_o(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4+%5];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a), "n"(OFF) : "memory");
  return v;
}
template <int OFF>
__device__ __forceinline__ float4 lds128f_o(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4+%5];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a), "n"(OFF) : "memory");
  return v;
}
template <int OFF>
__device__ __forceinline__ uint32_t lds32_o(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF) : "memory");
  return v;
}
template <int OFF>
__device__ __forceinline__ float lds_h2f_o(uint32_t a) {
  unsigned short h;
  asm volatile("ld.shared.u16 %0, [%1+%2];" : "=h"(h) : "r"(a), "n"(OFF) : "memory");
  return __half2float(__ushort_as_half(h));
}
// Predicated forms: lanes with on == 0 issue no shared-memory access and get zeros.
__device__ __forceinline__ uint4 lds128_pa(uint32_t a, uint32_t on) {
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %5, 0;\n\t@p ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n\t}"
               : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w) : "r"(a), "r"(on) : "memory");
  return v;
}
__device__ __forceinline__ float4 lds128f_pa(uint32_t a, uint32_t on) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %5, 0;\n\t@p ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n\t}"
               : "+f"(v.x), "+f"(v.y), "+f"(v.z), "+f"(v.w) : "r"(a), "r"(on) : "memory");
  return v;
}
__device__ __forceinline__ float2 lds64f_a(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds32_a(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ float lds_h2f_a(uint32_t a) {
  unsigned short h;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a) : "memory");
  return __half2float(__ushort_as_half(h));
}

// Shared-memory load as an ordinary C++ access, so the compiler orders it against the mbarrier waits
// (which clobber memory) and can still schedule it freely otherwise.
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Activation load that bypasses L1 (the producer of x may be the kernel that just finished).
__device__ __forceinline__ uint4 ldg_cg_128(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return static_cast<uint32_t>(__half_as_ushort(lo)) |
         (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

// 8 activations held in one 16-byte word (fp16 or bf16 storage) -> fp16.
__device__ __forceinline__ void raw_to_half8(const uint4 raw, bool is_bf16, __half (&h)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  if (is_bf16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xffff0000u);
      h[2 * i] = __float2half_rn(lo);
      h[2 * i + 1] = __float2half_rn(hi);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[2 * i] = __ushort_as_half(static_cast<unsigned short>(w[i] & 0xffffu));
      h[2 * i + 1] = __ushort_as_half(static_cast<unsigned short>(w[i] >> 16));
    }
  }
}

// 8 activations (one 16-byte load, bypassing L1) to fp16.
__device__ __forceinline__ void load8_as_half(const void* p, bool is_bf16, __half (&h)[8]) {
  raw_to_half8(ldg_cg_128(p), is_bf16, h);
}

// 8 activations held in one 16-byte word (fp16 or bf16 storage) -> fp32, exactly.
__device__ __forceinline__ void raw_to_f32(const uint4 raw, bool is_bf16, float (&v)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (is_bf16) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      v[2 * i] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] & 0xffffu)));
      v[2 * i + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] >> 16)));
    }
  }
}

// 8 activations (one 16-byte load, bypassing L1) to fp32, exactly.
__device__ __forceinline__ void load8_f32(const void* p, bool is_bf16, float (&v)[8]) {
  raw_to_f32(ldg_cg_128(p), is_bf16, v);
}

// v rounded to the 16-bit activation type (nearest even), back in fp32: the value a bf16/fp16 buffer holds.
// 8-bit double-quantised scales (rb_gemv_desc::s_row): a group's 16-bit word holds the scale code b (low byte)
// and the zero point z in 1/16 steps (high byte). They decode to the fp16 scale and min of the reference format:
// s = fp16(sc8(b) * s_row) with sc8(b) = 2^((b >> 4) - 15) * (1 + (b & 15) / 16), the fp32 whose bits are
// (b << 19) + 0x38000000 (exact), and m = fp16(-(z / 16) * s), each rounded to nearest even once.
// Two groups' words (low half first) -> their fp16 scales (s2) and mins (m2), packed the same way.
__device__ __forceinline__ void dq_scales8_f16x2(uint32_t words, float s_row, uint32_t& s2, uint32_t& m2) {
  uint32_t s_out = 0u, m_out = 0u;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t w = (words >> (16 * i)) & 0xFFFFu;
    const __half s = __float2half_rn(__uint_as_float(((w & 0xFFu) << 19) + 0x38000000u) * s_row);
    const __half m = __float2half_rn(-(static_cast<float>(w >> 8) * 0.0625f) * __half2float(s));
    s_out |= static_cast<uint32_t>(__half_as_ushort(s)) << (16 * i);
    m_out |= static_cast<uint32_t>(__half_as_ushort(m)) << (16 * i);
  }
  s2 = s_out;
  m2 = m_out;
}

__device__ __forceinline__ float round_act(float v, bool is_bf16) {
  return is_bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}

// One element of a bf16 or fp16 array, to fp32.
__device__ __forceinline__ float load_act(const void* p, int64_t idx, bool is_bf16) {
  const unsigned short u = reinterpret_cast<const unsigned short*>(p)[idx];
  return is_bf16 ? __uint_as_float(static_cast<uint32_t>(u) << 16) : __half2float(__ushort_as_half(u));
}

__device__ __forceinline__ void store_out(void* y, int64_t idx, float v, bool is_bf16) {
  if (is_bf16)
    reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device), not on every call, so that a call
// made while a CUDA graph is being captured issues nothing but the launch. Concurrent first calls may both
// set the attribute, which is harmless.
inline cudaError_t ensure_smem_limit(const void* kern, int bytes) {
  static const void* keys[64] = {};
  static unsigned long long done[64] = {};
  static std::mutex lock;  // host threads (e.g. one per GPU) may launch at the same time
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> hold(lock);
  int slot = -1;
  for (int i = 0; i < 64; ++i) {
    if (keys[i] == kern || keys[i] == nullptr) {
      keys[i] = kern;
      slot = i;
      break;
    }
  }
  const bool cacheable = slot >= 0 && dev >= 0 && dev < 64;
  if (cacheable && ((done[slot] >> dev) & 1ull)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && cacheable) done[slot] |= 1ull << dev;
  return e;
}

}  // namespace rb
