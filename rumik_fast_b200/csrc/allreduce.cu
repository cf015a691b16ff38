// allreduce.cu - the tensor-parallel decode step's per-layer reduction over NVLink peer memory (sm_100a).
//
// out = sum over ranks of (a + b), for the hidden vector of a row-parallel layer pair (o_proj partial a and
// down partial b of every rank). One CTA per rank, one launch per layer, replacing an add kernel and a
// collective call:
//  1. every thread adds its elements of a and b in fp32 and stores them, with plain stores over NVLink, into
//     slot [parity][this rank] of EVERY rank's symmetric buffer (the local one included);
//  2. after a CTA barrier and a system-scope fence, thread r < world publishes the call's epoch into flag
//     [this rank] of rank r's buffer (release store);
//  3. thread r < world waits (acquire loads, bounded by %globaltimer) until local flag [r] reaches the epoch;
//  4. every thread sums the world slots of its elements in rank order (the same order on every rank, so all
//     ranks hold bit-identical results) and writes fp16.
// Epochs come from a counter in the rank's own buffer, so a CUDA graph can replay the launch unchanged. Slots
// are double-buffered by epoch parity: a rank can only be one call ahead of any peer, because it cannot finish
// call e + 1 before every peer has published e + 1, which each does only after finishing call e.
// No multicast, no NVLS: peer loads and stores only.
#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace tpar {

constexpr int kMaxWorld = 8;
constexpr int kThreads = 1024;

struct ArParams {
  const __half* a;
  const __half* b;
  __half* out;
  uint8_t* buf[kMaxWorld];  // every rank's symmetric buffer; buf[rank] is this rank's
  int n, rank, world;
  uint32_t flag_off, counter_off;  // data at offset 0: [2][world][n] fp32
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads, 1) tp_allreduce_kernel(const __grid_constant__ ArParams p) {
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  uint32_t* counter = reinterpret_cast<uint32_t*>(p.buf[p.rank] + p.counter_off);
  griddep_wait();  // a and b come from the GEMV launch before
  if (tid == 0) s_epoch = *counter + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = static_cast<int>(e & 1u);
  const size_t slot = (static_cast<size_t>(par) * p.world + p.rank) * p.n;
  for (int i = tid; i < p.n; i += kThreads) {
    float v = __half2float(p.a[i]);
    if (p.b) v += __half2float(p.b[i]);
    for (int r = 0; r < p.world; ++r) reinterpret_cast<float*>(p.buf[r])[slot + i] = v;
  }
  __syncthreads();
  if (tid < p.world) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(p.buf[tid] + p.flag_off) + p.rank, e);
    const uint32_t* f = reinterpret_cast<const uint32_t*>(p.buf[p.rank] + p.flag_off) + tid;
    if (ld_acquire_sys(f) < e) {
      const unsigned long long t0 = globaltimer_ns(), lim = wait_limit_ns();
      while (ld_acquire_sys(f) < e) {
        if (globaltimer_ns() - t0 > lim) {
          atomicOr(&g_device_error, ERR_TP_WAIT);
          break;
        }
      }
    }
  }
  __syncthreads();
  const float* data = reinterpret_cast<const float*>(p.buf[p.rank]) + static_cast<size_t>(par) * p.world * p.n;
  for (int i = tid; i < p.n; i += kThreads) {
    float acc = 0.f;
    for (int r = 0; r < p.world; ++r) acc += data[static_cast<size_t>(r) * p.n + i];
    p.out[i] = __float2half_rn(acc);
  }
  if (tid == 0) *counter = e;
}

}  // namespace tpar

int launch_tp_allreduce(const __half* a, const __half* b, __half* out, int64_t n, void* const* bufs, int rank,
                        int world, uint32_t flag_off, uint32_t counter_off, int flags, cudaStream_t stream) {
  using namespace tpar;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || n <= 0 || n > (int64_t(1) << 24))
    return RB_ERR_SHAPE;
  ArParams p = {};
  p.a = a;
  p.b = b;
  p.out = out;
  for (int r = 0; r < world; ++r) {
    if (!bufs[r]) return RB_ERR_NULL;
    p.buf[r] = static_cast<uint8_t*>(bufs[r]);
  }
  p.n = static_cast<int>(n);
  p.rank = rank;
  p.world = world;
  p.flag_off = flag_off;
  p.counter_off = counter_off;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (flags & RB_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tp_allreduce_kernel, p) == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

}  // namespace rb
