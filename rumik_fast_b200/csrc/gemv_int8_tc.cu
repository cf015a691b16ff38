// gemv_int8_tc.cu - the int8 per-row GEMV (tied audio head), batch 1, on the tcgen05 tensor cores (sm_100a).
//
// y[n] = s[n] * sum_k v(q[n, k]) * x[k], the operation of rumik-fast's gemv_int8_kernel
// (kernels/cuda_gemv.py:141-186), v(q) = q - 128 for uint8 storage (quantize_int8_rows,
// kernels/cuda_gemv.py:234-242) or (int8)q for signed storage.
//
// The codes are already 8-bit integers, so they are the A operand of tcgen05.mma.kind::i8 as they arrive:
//  * warp 0 streams 128-row x 128-column tiles of q with 2-D TMA (128-byte swizzle, 16 KB) into a ring;
//  * warp 1 issues four tcgen05.mma (M=128, N=8, K=32) per tile straight from shared memory, accumulating a
//    whole row block in tensor memory (int32, exact), and frees each tile with tcgen05.commit;
//  * x is quantised once per CTA to 16-bit integers xi = rint(x / delta), delta = max|x| / 32639, split into
//    signed high and low bytes (B rows 0 and 1, as in gemv_int4_tc.cu);
//  * four warps read the row's two accumulator columns and write
//    y = s * delta * (256 * D0 + D1 - 128 * sum(xi))  (the last term only for uint8 storage).
// No dequantisation instruction runs at all; the kernel is a pure HBM stream. All waits are bounded.
#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace g8t {

constexpr int kRows = 128;
constexpr int kThreads = 6 * 32;          // producer, MMA issuer, four epilogue warps (also stage x)
constexpr uint32_t kStageBytes = kRows * 128;
constexpr int kMaxStages = 12;  // ring depth: as many 16 KB stages as fit beside the activation table (K <= 8192: 12)
constexpr uint32_t kXPad = 256;
constexpr uint32_t kTmemCols = 32;        // two 8-column int32 accumulators

struct __align__(64) H8Params {
  CUtensorMap qmap;                       // [N rows, K bytes], box 128 x 128, 128-byte swizzle
  const void* x;
  const void* s;
  void* y;
  int N, K, nblocks, x_bf16, y_bf16, s_f16, q_signed, prefetch, nst;
  uint32_t xs_off, bar_off, idesc;
};

__device__ __forceinline__ void umma_ss_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) gemv_int8_tc_kernel(const __grid_constant__ H8Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = gridDim.x, cta = blockIdx.x;
  const int nlocal = (p.nblocks - cta + C - 1) / C;
  const int nk = p.K / 128;
  const int nst = p.nst;  // ring depth of this launch
  uint8_t* xs = smem + p.xs_off;  // [K/16][32]: 16 high bytes, 16 low bytes per 16 columns; then reductions
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* full = bars;
  uint64_t* empty = bars + nst;
  uint64_t* dready = bars + 2 * nst;  // [2]
  uint64_t* dfree = dready + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfree + 2);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [4] per-warp maxima, [4] per-warp integer sums
  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&dready[b], 1);
      mbar_init(&dfree[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  mm4::tc_fence_before();
  __syncthreads();
  mm4::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      if (!p.prefetch) griddep_wait();
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nlocal && ok; ++j) {
        const int row0 = (cta + j * C) * kRows;
        for (int k = 0; k < nk; ++k) {
          const int slot = issued % nst;
          if (issued >= nst && !mbar_wait(&empty[slot], ((issued / nst) - 1) & 1, ERR_TC_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[slot], kStageBytes);
          mm4::tma_load_2d(smem + static_cast<size_t>(slot) * kStageBytes, &p.qmap, k * 128, row0, &full[slot]);
          ++issued;
        }
      }
      for (int t = max(0, issued - nst); t < issued; ++t)  // no retirement with copies in flight
        if (!mbar_wait(&full[t % nst], (t / nst) & 1, ERR_TC_WAIT)) break;
    }
  } else if (warp == 1) {
    named_bar_sync(1, 5 * 32);  // activation table staged
    if (lane == 0) {
      mm4::tc_fence_after();
      const uint32_t xtab = smem_u32(xs);
      int used = 0;
      bool ok = true;
      for (int j = 0; j < nlocal && ok; ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&dfree[b], ((j >> 1) - 1) & 1, ERR_TC_WAIT)) break;
        mm4::tc_fence_after();
        for (int k = 0; k < nk; ++k, ++used) {
          const int slot = used % nst;
          if (!mbar_wait(&full[slot], (used / nst) & 1, ERR_TC_WAIT)) {
            ok = false;
            break;
          }
          mm4::tc_fence_after();
          const uint32_t a_base = smem_u32(smem + static_cast<size_t>(slot) * kStageBytes);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            umma_ss_i8(tmem + b * 8, mm4::sw128_desc(a_base + 32 * i), g4t::x_desc<32>(xtab + k * 256 + 64 * i),
                       p.idesc, (k | i) != 0);
          mm4::umma_commit(&empty[slot]);  // the tile may be refilled once these MMAs have read it
        }
        if (ok) mm4::umma_commit(&dready[b]);
      }
    }
  } else {
    // ---------------- activation table, then epilogue ----------------
    const int et = tid - 64;  // 0..127
    griddep_wait();           // x may come from the previous kernel; y is written below
    // delta = max|x| / 32639 over the whole vector
    float mx = 0.f;
    for (int k = et * 8; k < p.K; k += 128 * 8) {
      __half h[8];
      load8_as_half(static_cast<const uint8_t*>(p.x) + static_cast<int64_t>(k) * 2, p.x_bf16, h);
#pragma unroll
      for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(__half2float(h[i])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp - 2] = mx;
    named_bar_sync(2, 128);
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float delta = mx > 0.f ? mx / 32639.f : 1.f;
    const float inv = 1.f / delta;
    int isum = 0;
    for (int k = et * 8; k < p.K; k += 128 * 8) {
      __half h[8];
      load8_as_half(static_cast<const uint8_t*>(p.x) + static_cast<int64_t>(k) * 2, p.x_bf16, h);
      uint32_t hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int xi = __float2int_rn(fminf(fmaxf(__half2float(h[i]) * inv, -32639.f), 32639.f));
        isum += xi;
        const int l = ((xi + 128) & 255) - 128;
        const int hh = (xi - l) >> 8;
        hi[i >> 2] |= (static_cast<uint32_t>(hh) & 255u) << (8 * (i & 3));
        lo[i >> 2] |= (static_cast<uint32_t>(l) & 255u) << (8 * (i & 3));
      }
      uint8_t* dst = xs + (k >> 4) * 32 + (k & 8);
      *reinterpret_cast<uint2*>(dst) = make_uint2(hi[0], hi[1]);
      *reinterpret_cast<uint2*>(dst + 16) = make_uint2(lo[0], lo[1]);
    }
    for (int i = et; i < static_cast<int>(kXPad / 16); i += 128)
      reinterpret_cast<uint4*>(xs + (p.K / 16) * 32)[i] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
    named_bar_sync(2, 128);  // everyone has read red[] (the maxima) before it is reused
    if (lane == 0) reinterpret_cast<int*>(red)[warp - 2] = isum;
    fence_proxy_async_smem();  // generic writes of the table -> visible to the tensor core
    named_bar_sync(1, 5 * 32);
    const int* ired = reinterpret_cast<const int*>(red);
    const float offset = p.q_signed ? 0.f : 128.f * static_cast<float>(ired[0] + ired[1] + ired[2] + ired[3]);
    const int quad = warp & 3;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    for (int j = 0; j < nlocal; ++j) {
      const int b = j & 1;
      if (ok) ok = mbar_wait(&dready[b], (j >> 1) & 1, ERR_TC_WAIT);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      mm4::tc_fence_after();
      int dh, dl;
      g4t::tmem_ld2(tq + b * 8, dh, dl);
      g4t::tmem_wait_ld(dh, dl);
      mm4::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dfree[b]);
      const int row = (cta + j * C) * kRows + quad * 32 + lane;
      if (row < p.N) {
        const float sr = p.s_f16 ? __half2float(reinterpret_cast<const __half*>(p.s)[row])
                                 : reinterpret_cast<const float*>(p.s)[row];
        const float v = sr * delta * ((256.f * static_cast<float>(dh) + static_cast<float>(dl)) - offset);
        store_out(p.y, row, v, p.y_bf16);
      }
    }
  }
  mm4::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mm4::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace g8t

// Batch 1, K % 128 == 0: the tensor-core path; returns RB_ERR_SHAPE for anything else (the caller then uses
// the warp-MMA kernel).
int launch_gemv_int8_tc(const GemvArgs& a, int num_sms, cudaStream_t stream) {
  using namespace g8t;
  if (a.batch != 1 || a.K % 128 != 0) return RB_ERR_SHAPE;
  auto encode = mm4::encode_fn();
  if (!encode) return RB_ERR_DEVICE;
  H8Params p;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.K), static_cast<cuuint64_t>(a.N)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.K)};
  const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(kRows)};
  const cuuint32_t es[2] = {1, 1};
  if (encode(&p.qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.q), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return RB_ERR_SHAPE;
  p.x = a.x;
  p.s = a.s_row;
  p.y = a.y;
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.nblocks = static_cast<int>((a.N + kRows - 1) / kRows);
  p.x_bf16 = a.x_dtype == RB_BF16;
  p.y_bf16 = a.y_dtype == RB_BF16;
  p.s_f16 = a.s_dtype == RB_F16;
  p.q_signed = a.q_signed ? 1 : 0;
  p.prefetch = (a.flags & RB_FLAG_PDL) && (a.flags & RB_FLAG_PREFETCH_WEIGHTS) ? 1 : 0;
  // instruction descriptor: D int32, A unsigned or signed 8-bit, B signed 8-bit, K-major, N = 8, M = 128
  p.idesc = (2u << 4) | ((p.q_signed ? 1u : 0u) << 7) | (1u << 10) | ((8u >> 3) << 17) |
            ((static_cast<uint32_t>(kRows) >> 4) << 24);
  constexpr uint32_t kSmemMax = 227 * 1024;
  const uint32_t xbytes = static_cast<uint32_t>(a.K / 16) * 32 + kXPad;
  const uint32_t fixed = 1024 + xbytes + 16 + (2 * kMaxStages + 4) * 8 + 16 + 32;
  p.nst = std::min(kMaxStages, static_cast<int>((kSmemMax - std::min(fixed, kSmemMax)) / kStageBytes));
  if (p.nst < 2) return RB_ERR_SHAPE;
  p.xs_off = static_cast<uint32_t>(p.nst) * kStageBytes;
  p.bar_off = (p.xs_off + xbytes + 15) & ~15u;
  const uint32_t smem = 1024 + p.bar_off + (2 * p.nst + 4) * 8 + 16 + 32;
  if (smem > kSmemMax) return RB_ERR_SHAPE;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(gemv_int8_tc_kernel), static_cast<int>(kSmemMax));
  if (e != cudaSuccess) return RB_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(num_sms, p.nblocks));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (a.flags & RB_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, gemv_int8_tc_kernel, p);
  return e == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

}  // namespace rb
