// mm_int4.cu - int4-weight matrix product for prefill on B200 tensor cores (tcgen05 / TMEM), sm_100a.
//
// Y[t, n] = sum_k X[t, k] * w[n, k] with w = code * s + m in the int4 group-128 layout; the operation of
// rumik-fast's Triton kernel _mm_int4 (kernels/mm_int4.py:24-46) and its wrapper mm_int4 (:59-73).
//
// One CTA computes a 128-weight-row x BT-token tile (UMMA M = 128, N = BT <= 256) with an fp32 accumulator
// in tensor memory, walking K one 128-column group per pipeline stage:
//  * warp 0 (producer): TMA loads of the stage's raw int4 codes (128 rows x 64 bytes, tensor map over q)
//    and of the two 64-column X atoms (tensor map over X, 128-byte swizzle), completing on ld_full.
//  * warps 2-9 (converters): turn the codes into fp16 w = code * s + m and write them straight into the
//    canonical K-major SWIZZLE_128B layout the UMMA descriptor reads (row r, 16-byte chunk c at
//    r * 128 + (c ^ (r & 7)) * 16 inside an 8-row, 1024-byte atom). Per code byte: one PRMT spreads it to
//    both fp16 lanes, one LOP3 ORs the nibbles under the fp16 magic numbers (1024 | low nibble,
//    64 | high nibble << 4), one HSUB2 removes the magic, one HFMA2 applies scale and min (single rounding).
//    Weights therefore never exist in HBM wider than int4. fp16 (not bf16) keeps the rounding of w at
//    ~2^-12 relative, far inside the 1e-3 tolerance.
//  * warp 1 (MMA): allocates the TMEM accumulator, and one elected thread issues eight
//    tcgen05.mma.cta_group::1.kind::f16 (K = 16 each) per stage, then tcgen05.commit frees the stage.
//  * the converter warps finally read the accumulator with tcgen05.ld (each warp its 32-lane quadrant)
//    and store Y (coalesced along n).
// All mbarrier waits are bounded; no multicast, no clusters.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace mm4 {

constexpr int kConvWarps = 8;
constexpr int kThreads = (2 + kConvWarps) * 32;
constexpr int kRows = 128;               // weight rows per tile (UMMA M)
constexpr int kAtomBytes = 128 * 128;    // one 128-row x 64-column fp16 swizzle atom
constexpr int kRawBytes = kRows * 64;    // one group of codes for 128 rows

struct MmParams {
  const uint16_t* s;
  const uint16_t* m;
  void* y;
  int64_t ldy;
  int M, N, K, G, BT;
  int y_bf16;
  int ns;
  uint32_t stage_bytes, b_off, raw_off;  // within a stage: A at 0, B at b_off, raw codes at raw_off
  uint32_t bar_off;                        // from the 1024-aligned base
  uint32_t idesc;
  uint32_t tmem_cols;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  // K-major, SWIZZLE_128B, stride between 8-row groups = 1024 bytes, descriptor version 1 (sm_100)
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

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

__global__ void __launch_bounds__(kThreads, 1)
    mm_int4_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ MmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * kRows, t0 = blockIdx.y * p.BT;
  const int nkb = p.G;
  uint64_t* ld_full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* a_full = ld_full + p.ns;
  uint64_t* st_empty = a_full + p.ns;
  uint64_t* acc_full = st_empty + p.ns;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  if (tid == 0) {
    for (int i = 0; i < p.ns; ++i) {
      mbar_init(&ld_full[i], 1);
      mbar_init(&a_full[i], kConvWarps);
      mbar_init(&st_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {  // TMEM accumulator: 128 lanes x tmem_cols fp32 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      griddep_wait();  // X may come from the previous kernel
      const uint32_t bytes = kRawBytes + 2 * p.BT * 128;
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % p.ns;
        if (kb >= p.ns && !mbar_wait(&st_empty[s], ((kb / p.ns) - 1) & 1, ERR_MM4_WAIT)) break;
        uint8_t* st = smem + static_cast<size_t>(s) * p.stage_bytes;
        mbar_arrive_expect_tx(&ld_full[s], bytes);
        tma_load_2d(st + p.raw_off, &qmap, kb * 64, n0, &ld_full[s]);
        tma_load_2d(st + p.b_off, &xmap, kb * 128, t0, &ld_full[s]);
        tma_load_2d(st + p.b_off + p.BT * 128, &xmap, kb * 128 + 64, t0, &ld_full[s]);
        issued = kb + 1;
      }
      for (int kb = max(0, issued - p.ns); kb < issued; ++kb)  // no retirement with copies in flight
        mbar_wait(&ld_full[kb % p.ns], (kb / p.ns) & 1, ERR_MM4_WAIT);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % p.ns;
        const uint32_t par = (kb / p.ns) & 1;
        ok = mbar_wait(&ld_full[s], par, ERR_MM4_WAIT) && mbar_wait(&a_full[s], par, ERR_MM4_WAIT);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + static_cast<size_t>(s) * p.stage_bytes);
        const uint32_t b_base = a_base + p.b_off;
#pragma unroll
        for (int k16 = 0; k16 < 8; ++k16) {
          const int atom = k16 >> 2, kk = k16 & 3;
          umma_f16(tmem, sw128_desc(a_base + atom * kAtomBytes + kk * 32),
                   sw128_desc(b_base + atom * p.BT * 128 + kk * 32), p.idesc, (kb | k16) != 0);
        }
        umma_commit(&st_empty[s]);  // stage s may be refilled once these MMAs have read it
      }
      umma_commit(acc_full);  // arrives when every MMA issued above has completed
    }
  } else {
    // ---------------- converters, then epilogue ----------------
    const int ct = tid - 64;                 // 0..255
    const int row = ct >> 1, half = ct & 1;  // A-tile row, 64-column atom
    const int n = n0 + row;
    const bool row_ok = n < p.N;
    const uint32_t k1024_64 = 0x54006400u;   // (fp16 1024 | low nibble, fp16 64 | high nibble << 4)
    const uint32_t sub_1024_64 = 0x54006400u;
    const uint32_t mask = 0x00F0000Fu;
    bool ok = true;
    uint16_t s_next = 0, m_next = 0;
    if (row_ok) {
      s_next = __ldg(p.s + static_cast<int64_t>(n) * p.G);
      m_next = __ldg(p.m + static_cast<int64_t>(n) * p.G);
    }
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % p.ns;
      const uint16_t s16 = s_next, m16 = m_next;
      if (row_ok && kb + 1 < nkb) {  // prefetch the next group's scale and min
        s_next = __ldg(p.s + static_cast<int64_t>(n) * p.G + kb + 1);
        m_next = __ldg(p.m + static_cast<int64_t>(n) * p.G + kb + 1);
      }
      if (ok) ok = mbar_wait(&ld_full[s], (kb / p.ns) & 1, ERR_MM4_WAIT);
      uint8_t* st = smem + static_cast<size_t>(s) * p.stage_bytes;
      if (ok) {
        const uint32_t s2 = static_cast<uint32_t>(s16) * 0x10001u, m2 = static_cast<uint32_t>(m16) * 0x10001u;
        const uint8_t* raw = st + p.raw_off + row * 64 + half * 32;
        uint4 w4[2];
        // the two 16-byte reads of a row pair go in opposite orders (fewer bank conflicts)
        const int first = (row >> 1) & 1;
        w4[first] = lds128(raw + first * 16);
        w4[first ^ 1] = lds128(raw + (first ^ 1) * 16);
        const uint32_t wv[8] = {w4[0].x, w4[0].y, w4[0].z, w4[0].w, w4[1].x, w4[1].y, w4[1].z, w4[1].w};
        uint8_t* arow = st + half * kAtomBytes + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // output chunk c = columns 8c..8c+7 of this atom = code word c
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t spread = __byte_perm(wv[c], 0u, 0x4040u | (0x0101u * j));
            const uint32_t t = and_or(spread, mask, k1024_64);  // (1024 + lo, 64 + hi) exact
            o[j] = hfma2_u(hsub2_u(t, sub_1024_64), s2, m2);    // (lo, hi) * s + m, one rounding
          }
          if (!row_ok) o[0] = o[1] = o[2] = o[3] = 0u;
          *reinterpret_cast<uint4*>(arow + ((c ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      fence_proxy_async_smem();  // generic writes of A -> visible to the tensor core (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
    }
    // ---- epilogue: TMEM -> registers -> Y ----
    if (ok) ok = mbar_wait(acc_full, 0, ERR_MM4_WAIT);
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective: decide per warp
    tc_fence_after();
    griddep_wait();  // Y may still be read by the previous kernel
    const int cw = warp - 2;                  // 0..7
    const int quad = warp & 3;                // TMEM lane quadrant this warp may access
    const int chalf = cw >> 2;                // which half of the token columns
    const int wrow = n0 + quad * 32 + lane;   // weight row = output column n
    const int cols = p.BT / 2;
    if (ok) {
      for (int c0 = chalf * cols; c0 < (chalf + 1) * cols; c0 += 8) {
        uint32_t v[8];
        const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int t = t0 + c0 + i;
          if (t < p.M && wrow < p.N) store_out(p.y, static_cast<int64_t>(t) * p.ldy + wrow, __uint_as_float(v[i]), p.y_bf16);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace mm4

int launch_mm_int4(const MmArgs& a, int num_sms, cudaStream_t stream) {
  using namespace mm4;
  (void)num_sms;
  if (a.x_dtype != RB_F16) return RB_ERR_DTYPE;  // the tensor-core operands are fp16 (see mm_int4.py)
  auto encode = encode_fn();
  if (!encode) return RB_ERR_DEVICE;
  const int M = static_cast<int>(a.M), N = static_cast<int>(a.N), K = static_cast<int>(a.K);
  // token tile: one tile up to 256 tokens, else equal tiles of <= 256 (multiples of 16)
  const int ntt = (M + 255) / 256;
  int BT = (M + ntt - 1) / ntt;
  BT = std::max(16, (BT + 15) / 16 * 16);
  const uint32_t b_bytes = 2u * BT * 128;
  const uint32_t stage_bytes = ((2u * kAtomBytes + b_bytes + kRawBytes) + 1023u) & ~1023u;
  constexpr uint32_t kSmemMax = 227 * 1024;
  int ns = static_cast<int>((kSmemMax - 1024 - 256) / stage_bytes);
  ns = std::min(ns, 4);
  if (ns < 2) return RB_ERR_SHAPE;
  MmParams p;
  p.s = a.s;
  p.m = a.m;
  p.y = a.Y;
  p.ldy = a.ldy;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = K / 128;
  p.BT = BT;
  p.y_bf16 = a.y_dtype == RB_BF16;
  p.ns = ns;
  p.stage_bytes = stage_bytes;
  p.b_off = 2u * kAtomBytes;
  p.raw_off = 2u * kAtomBytes + b_bytes;
  p.bar_off = static_cast<uint32_t>(ns) * stage_bytes;
  // instruction descriptor: D f32, A f16, B f16, both K-major, N = BT, M = 128
  p.idesc = (1u << 4) | (static_cast<uint32_t>(BT >> 3) << 17) | (static_cast<uint32_t>(kRows >> 4) << 24);
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(BT)) cols <<= 1;
  p.tmem_cols = cols;
  const uint32_t smem = 1024 + p.bar_off + (3 * ns + 1) * 8 + 16;

  CUtensorMap qmap, xmap;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(N)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K / 2)};
    const cuuint32_t box[2] = {64, kRows};
    const cuuint32_t es[2] = {1, 1};
    if (encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.q), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return RB_ERR_SHAPE;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.ldx) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(BT)};
    const cuuint32_t es[2] = {1, 1};
    if (encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.X), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return RB_ERR_SHAPE;
  }
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(mm_int4_kernel), kSmemMax);
  if (e != cudaSuccess) return RB_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + kRows - 1) / kRows, (M + BT - 1) / BT);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (a.flags & RB_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, mm_int4_kernel, qmap, xmap, p);
  return e == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

}  // namespace rb
