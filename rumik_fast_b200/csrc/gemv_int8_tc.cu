// gemv_int8_tc.cu - the int8 per-row GEMV (tied audio head), batch 1, on the tcgen05 tensor cores (sm_100a).
//
// y[n] = s[n] * sum_k v(q[n, k]) * x[k], the operation of rumik-fast's gemv_int8_kernel
// (kernels/cuda_gemv.py:141-186), v(q) = q - 128 for uint8 storage (quantize_int8_rows,
// kernels/cuda_gemv.py:234-242) or (int8)q for signed storage.
//
// The codes are already 8-bit integers, so they are the A operand of tcgen05.mma.kind::i8 as they arrive:
//  * warp 0 streams 128-row x 128-column tiles of q (one 128-column group each) with 2-D TMA (128-byte swizzle,
//    16 KB) into a ring;
//  * warp 1 issues four tcgen05.mma (M=128, N=8, K=32) per tile straight from shared memory into one of kDBufs
//    int32 accumulators in tensor memory (one per group, exact), frees the tile with tcgen05.commit and signals
//    the accumulator with another;
//  * x is quantised per 128-column group g to 16-bit integers xi = rint(x / delta_g), delta_g = max_g|x| / 32639,
//    split into signed high and low bytes (B rows 0 and 1): an outlier channel coarsens only its own group;
//  * four warps (thread = row) read each group's two accumulator columns and add
//    delta_g * (256 * D0 + D1 - 128 * sum_g(xi)) (the last term only for uint8 storage), combined in int32 so
//    that both storages give the same bits; y = s * sum.
// No dequantisation instruction runs at all; the kernel is a pure HBM stream. All waits are bounded.
#include "common.cuh"
#include "tc.cuh"
#include "kernels.h"

namespace rb {

namespace g8t {

constexpr int kRows = 128;
constexpr int kThreads = 6 * 32;          // producer, MMA issuer, four epilogue warps (also stage x)
constexpr uint32_t kStageBytes = kRows * 128;
constexpr int kMaxStages = 12;  // ring depth: as many 16 KB stages as fit beside the activation table (K <= 8192: 12)
constexpr uint32_t kXPad = 256;
constexpr int kDBufs = 8;                 // per-group accumulators in flight between the MMA issuer and epilogue
constexpr uint32_t kTmemCols = 64;        // kDBufs x 8 int32 columns

struct __align__(64) H8Params {
  CUtensorMap qmap;                       // [N rows, K bytes], box 128 x 128, 128-byte swizzle
  const void* x;
  const void* s;
  void* y;
  int N, K, nblocks, x_bf16, y_bf16, s_f16, q_signed, prefetch, nst;
  uint32_t xs_off, cst_off, bar_off, idesc;
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
  uint8_t* xs = smem + p.xs_off;  // [K/16][32]: 16 high bytes, 16 low bytes per 16 columns
  int2* cst = reinterpret_cast<int2*>(smem + p.cst_off);  // per group: {delta_g bits, sum_g(xi)}
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* full = bars;
  uint64_t* empty = bars + nst;
  uint64_t* dready = bars + 2 * nst;       // [kDBufs]
  uint64_t* dfree = dready + kDBufs;       // [kDBufs]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfree + kDBufs);
  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < kDBufs; ++b) {
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
      int u = 0;  // groups issued by this CTA: tile u % nst, accumulator u % kDBufs
      bool ok = true;
      for (int j = 0; j < nlocal && ok; ++j) {
        for (int k = 0; k < nk; ++k, ++u) {
          const int slot = u % nst, d = u % kDBufs;
          if (u >= kDBufs && !mbar_wait(&dfree[d], ((u / kDBufs) - 1) & 1, ERR_TC_WAIT)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&full[slot], (u / nst) & 1, ERR_TC_WAIT)) {
            ok = false;
            break;
          }
          mm4::tc_fence_after();
          const uint32_t a_base = smem_u32(smem + static_cast<size_t>(slot) * kStageBytes);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            umma_ss_i8(tmem + d * 8, mm4::sw128_desc(a_base + 32 * i), g4t::x_desc<32>(xtab + k * 256 + 64 * i),
                       p.idesc, i != 0);
          mm4::umma_commit(&empty[slot]);  // the tile may be refilled once these MMAs have read it
          mm4::umma_commit(&dready[d]);    // and the group's accumulator read
        }
      }
    }
  } else {
    // ---------------- activation table, then epilogue ----------------
    const int et = tid - 64;  // 0..127
    griddep_wait();           // x may come from the previous kernel; y is written below
    // chunk c = 8 columns; the 16 chunks of a group sit on 16 consecutive lanes (reduced with shuffles)
    const int nchunks = p.K / 8;
    for (int base = 0; base < nchunks; base += 128) {
      const int c = base + et;
      const bool valid = c < nchunks;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (valid) load8_f32(static_cast<const uint8_t*>(p.x) + static_cast<int64_t>(c) * 16, p.x_bf16, v);
      float mx = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float delta = mx > 0.f ? mx / 32639.f : 1.f;
      const float inv = 1.f / delta;
      int isum = 0;
      uint32_t hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int xi = __float2int_rn(fminf(fmaxf(v[i] * inv, -32639.f), 32639.f));
        isum += xi;
        const int l = ((xi + 128) & 255) - 128;
        const int hh = (xi - l) >> 8;
        hi[i >> 2] |= (static_cast<uint32_t>(hh) & 255u) << (8 * (i & 3));
        lo[i >> 2] |= (static_cast<uint32_t>(l) & 255u) << (8 * (i & 3));
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
      if (valid) {
        uint8_t* dst = xs + (c >> 1) * 32 + (c & 1) * 8;
        *reinterpret_cast<uint2*>(dst) = make_uint2(hi[0], hi[1]);
        *reinterpret_cast<uint2*>(dst + 16) = make_uint2(lo[0], lo[1]);
        if ((c & 15) == 0) cst[c >> 4] = make_int2(__float_as_int(delta), isum);
      }
    }
    for (int i = et; i < static_cast<int>(kXPad / 16); i += 128)
      reinterpret_cast<uint4*>(xs + (p.K / 16) * 32)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();  // generic writes of the table -> visible to the tensor core
    named_bar_sync(1, 5 * 32);
    const int quad = warp & 3;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const int off_mul = p.q_signed ? 0 : 128;
    bool ok = true;
    int u = 0;
    for (int j = 0; j < nlocal && ok; ++j) {
      float acc = 0.f;
      for (int k = 0; k < nk; ++k, ++u) {
        const int d = u % kDBufs;
        if (ok) ok = mbar_wait(&dready[d], (u / kDBufs) & 1, ERR_TC_WAIT);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        mm4::tc_fence_after();
        int dh, dl;
        g4t::tmem_ld2(tq + d * 8, dh, dl);
        g4t::tmem_wait_ld(dh, dl);
        mm4::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfree[d]);
        const int2 cg = cst[k];
        // sum over the group of v(q) * xi, exact in int32 (|value| <= 128 * 255 * 32639 < 2^31)
        const int t = dh * 256 + dl - off_mul * cg.y;
        acc = fmaf(__int_as_float(cg.x), static_cast<float>(t), acc);
      }
      const int row = (cta + j * C) * kRows + quad * 32 + lane;
      if (ok && row < p.N) {
        const float sr = p.s_f16 ? __half2float(reinterpret_cast<const __half*>(p.s)[row])
                                 : reinterpret_cast<const float*>(p.s)[row];
        store_out(p.y, row, sr * acc, p.y_bf16);
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
  const uint32_t cbytes = static_cast<uint32_t>(a.K / 128) * 8;
  const uint32_t fixed = 1024 + xbytes + cbytes + 32 + (2 * kMaxStages + 2 * kDBufs) * 8 + 16;
  p.nst = std::min(kMaxStages, static_cast<int>((kSmemMax - std::min(fixed, kSmemMax)) / kStageBytes));
  if (p.nst < 2) return RB_ERR_SHAPE;
  p.xs_off = static_cast<uint32_t>(p.nst) * kStageBytes;
  p.cst_off = (p.xs_off + xbytes + 15) & ~15u;
  p.bar_off = (p.cst_off + cbytes + 15) & ~15u;
  const uint32_t smem = 1024 + p.bar_off + (2 * p.nst + 2 * kDBufs) * 8 + 16;
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
