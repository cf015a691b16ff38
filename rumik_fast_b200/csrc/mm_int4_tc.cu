// mm_int4_tc.cu - the int4-weight prefill matmul Y[t, n] = sum_k X[t, k] w[n, k] on B200 tensor cores with
// the dequantised weights in tensor memory (sm_100a).
//
// The operation of rumik-fast's Triton kernel _mm_int4 (kernels/mm_int4.py:24-46) and its wrapper mm_int4
// (:59-73): w = code * s + m in the int4 group-128 layout, X fp16 or bf16 [M, K], fp32 accumulation. Both
// operands of a kind::f16 MMA share one type, and fp16 keeps the dequantised weight's rounding ~8x smaller than
// bf16, so a bf16 X is converted to fp16 in shared memory (the kernel instance with kBf16X: each converter set
// rewrites its stage's X atoms in place before it releases the group to the MMA issuer; exact for |x| <= 65504,
// as a torch cast of X to fp16 would be).
//
// Work items are (128-row weight block, token chunk of BT <= 128 tokens, K slice), block-major so that the CTAs working
// at the same time on the chunks of one block share its codes through L2; items are dealt round-robin to one
// CTA per SM. Both converter sets work on every item, set s on its groups g = s, s + 2, ..., each into its own
// accumulator; the epilogue adds the two in a fixed order. Per CTA:
//  * warp 0 (producer) streams, per item and group, the block's codes (TMA box 64 bytes x 128 rows, 64-byte
//    swizzle) and the chunk's two 64-column X atoms (TMA, 128-byte swizzle) into the set's ring;
//  * each converter set (four warps, thread = weight row = tensor-memory lane) dequantises its row's group
//    to fp16 (per code byte: PRMT, LOP3 to the fp16 magic numbers, HSUB2, HFMA2 with the row's scale and
//    min, one rounding) and writes the 64 columns to tensor memory (tcgen05.st);
//  * one thread per set issues eight tcgen05.mma.kind::f16 per group (M = 128, N = BT, K = 16): A from tensor
//    memory, B = the X atoms in shared memory, D = 128 x BT fp32 in tensor memory accumulating over all of K;
//  * the converter warps then read D0 + D1 (tcgen05.ld; set s takes every other 32-column chunk) and store Y,
//    or, when K is split into slices (a call with fewer row-block x chunk items than SMs), the slice's fp32
//    partial into a caller-provided workspace; mm_int4_reduce then adds the slices in slice order.
// All mbarrier waits are bounded; no multicast, no clusters.
#include "common.cuh"
#include "tc.cuh"
#include "kernels.h"

namespace rb {

namespace mm4t {

constexpr int kSets = 2;
constexpr int kRows = 128;
constexpr int kFirstConv = 1 + kSets;
constexpr int kThreads = (kFirstConv + 4 * kSets) * 32;
constexpr uint32_t kCodeBytes = kRows * 64;
constexpr int kNB = 2;                       // tensor-memory A buffers per set
constexpr uint32_t kACols = 64;
constexpr uint32_t kSetCols = 256;           // per set: A buffers (128 columns) + D (<= 128 columns)
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxStages = 6;

struct __align__(64) MmtParams {
  CUtensorMap qmap;  // [N rows, K/2 bytes], box 64 x 128, 64-byte swizzle
  CUtensorMap xmap;  // [M rows, K fp16], box 64 x BT, 128-byte swizzle
  const uint16_t* s;
  const uint16_t* m;
  void* y;
  int64_t ldy;
  float* ws;  // [kslices][M][N] fp32 partials when kslices > 1
  int M, N, K, G, BT, nchunks, kslices, gps, nitems, y_bf16, nst, prefetch;
  uint32_t stage_bytes, bar_off, idesc;
};

__device__ __forceinline__ void umma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];" : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]) : "r"(taddr) : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// bf16 -> fp16 of a pair of activations held in one 32-bit word (round to nearest even).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  const __half2 h = __floats2half2_rn(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool kBf16X>
__global__ void __launch_bounds__(kThreads, 1) mm_int4_tc_kernel(const __grid_constant__ MmtParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = gridDim.x, cta = blockIdx.x;
  const int nst = p.nst, G = p.G, BT = p.BT;
  const int nlocal = (p.nitems - cta + C - 1) / C;  // this CTA's items: cta + j * C
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  const int per_set = 2 * nst + 2 * kNB + 1;
  auto full = [&](int s, int i) { return bars + s * per_set + i; };
  auto empty = [&](int s, int i) { return bars + s * per_set + nst + i; };
  auto afull = [&](int s, int b) { return bars + s * per_set + 2 * nst + b; };
  auto mdone = [&](int s, int b) { return bars + s * per_set + 2 * nst + kNB + b; };
  auto dready = [&](int s) { return bars + s * per_set + 2 * nst + 2 * kNB; };
  uint64_t* dfree = bars + kSets * per_set;  // both sets' epilogues have read both accumulators
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfree + 1);
  auto stage_of = [&](int s, int slot) { return smem + (static_cast<size_t>(s) * nst + slot) * p.stage_bytes; };

  if (tid == 0) {
    for (int s = 0; s < kSets; ++s) {
      for (int i = 0; i < nst; ++i) {
        mbar_init(full(s, i), 1);
        mbar_init(empty(s, i), 5);  // four converter warps (codes read) + one MMA commit (X read)
      }
      for (int b = 0; b < kNB; ++b) {
        mbar_init(afull(s, b), 4);
        mbar_init(mdone(s, b), 1);
      }
      mbar_init(dready(s), 1);
    }
    mbar_init(dfree, 4 * kSets);
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
  const uint32_t stage_tx = kCodeBytes + 2u * BT * 128u;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      // The codes do not depend on the previous kernel: the first stages' code loads go out before
      // griddepcontrol.wait (overlapping the previous kernel's tail); X loads only after it.
      int pre[kSets] = {};
      for (int j = 0; j < nlocal; ++j) {
        const int item = cta + j * C;
        const int rem = item % (p.nchunks * p.kslices);
        const int row0 = (item / (p.nchunks * p.kslices)) * kRows;
        const int g0 = (rem % p.kslices) * p.gps, g1 = min(G, g0 + p.gps);
        bool room = false;
        for (int g = g0; g < g1; ++g) {
          const int s = (g - g0) % kSets;
          if (pre[s] >= nst) continue;
          room = true;
          const int slot = pre[s]++;
          mbar_arrive_expect_tx(full(s, slot), stage_tx);
          mm4::tma_load_2d(stage_of(s, slot), &p.qmap, g * 64, row0, full(s, slot));
        }
        if (!room) break;
      }
      griddep_wait();  // X may come from the previous kernel
      int issued[kSets] = {};
      bool ok = true;
      for (int j = 0; j < nlocal && ok; ++j) {
        const int item = cta + j * C;
        const int rem = item % (p.nchunks * p.kslices);
        const int row0 = (item / (p.nchunks * p.kslices)) * kRows, t0 = (rem / p.kslices) * BT;
        const int g0 = (rem % p.kslices) * p.gps, g1 = min(G, g0 + p.gps);
        for (int g = g0; g < g1 && ok; ++g) {
          const int s = (g - g0) % kSets;
          const int slot = issued[s] % nst;
          uint8_t* st = stage_of(s, slot);
          if (issued[s] >= pre[s]) {
            if (issued[s] >= nst && !mbar_wait(empty(s, slot), ((issued[s] / nst) - 1) & 1, ERR_MM4_WAIT)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full(s, slot), stage_tx);
            mm4::tma_load_2d(st, &p.qmap, g * 64, row0, full(s, slot));
          }
          mm4::tma_load_2d(st + kCodeBytes, &p.xmap, g * 128, t0, full(s, slot));
          mm4::tma_load_2d(st + kCodeBytes + BT * 128, &p.xmap, g * 128 + 64, t0, full(s, slot));
          ++issued[s];
        }
      }
      for (int s = 0; s < kSets; ++s)  // no retirement with copies in flight
        for (int t = max(0, issued[s] - nst); t < issued[s]; ++t)
          if (!mbar_wait(full(s, t % nst), (t / nst) & 1, ERR_MM4_WAIT)) break;
    }
  } else if (warp < kFirstConv) {
    // ---------------- MMA issuer of set s ----------------
    const int s = warp - 1;
    if (lane == 0) {
      const uint32_t d_col = tmem + s * kSetCols + kNB * kACols;
      int q = 0, used = 0;
      bool ok = true;
      for (int jj = 0; jj < nlocal && ok; ++jj) {
        if (jj >= 1 && !mbar_wait(dfree, (jj - 1) & 1, ERR_MM4_WAIT)) break;  // D read by the last epilogue
        const int item = cta + jj * C;
        const int g0 = (item % (p.nchunks * p.kslices) % p.kslices) * p.gps, g1 = min(G, g0 + p.gps);
        for (int gg = g0 + s; gg < g1; gg += kSets, ++q, ++used) {
          const int b = q % kNB, slot = used % nst;
          if (!mbar_wait(afull(s, b), (q / kNB) & 1, ERR_MM4_WAIT) ||
              !mbar_wait(full(s, slot), (used / nst) & 1, ERR_MM4_WAIT)) {
            ok = false;
            break;
          }
          mm4::tc_fence_after();
          const uint32_t xb = smem_u32(stage_of(s, slot) + kCodeBytes);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            umma_ts_f16(d_col, tmem + s * kSetCols + b * kACols + 8 * i,
                        mm4::sw128_desc(xb + (i >> 2) * BT * 128 + (i & 3) * 32), p.idesc, (gg - g0 >= kSets) || i != 0);
          mm4::umma_commit(mdone(s, b));     // A buffer b may be rewritten
          mm4::umma_commit(empty(s, slot));  // the stage's X atoms may be refilled
        }
        if (ok) mm4::umma_commit(dready(s));  // (with no group of this set in the item, arrives at once)
      }
    }
  } else {
    // ---------------- converters + epilogue of set s ----------------
    const int cw = warp - kFirstConv;
    const int s = cw >> 2;
    const int quad = warp & 3;
    const int rib = quad * 32 + lane;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t a_set = tq + s * kSetCols;
    const uint32_t magic = 0x54006400u, mask = 0x00F0000Fu;  // (1024 | low nibble, 64 | high nibble << 4)
    bool waited = false;  // griddepcontrol.wait before the first write of Y or of the workspace
    int q = 0, used = 0;
    bool ok = true;
    for (int jj = 0; jj < nlocal; ++jj) {
      const int item = cta + jj * C;
      const int rem = item % (p.nchunks * p.kslices);
      const int row = (item / (p.nchunks * p.kslices)) * kRows + rib, t0 = (rem / p.kslices) * BT;
      const int ks = rem % p.kslices, g0 = ks * p.gps, g1 = min(G, g0 + p.gps);
      const bool row_ok = row < p.N;
      const uint16_t* srow = p.s + static_cast<int64_t>(row_ok ? row : 0) * G;
      const uint16_t* mrow = p.m + static_cast<int64_t>(row_ok ? row : 0) * G;
      uint16_t s_next = 0, m_next = 0;
      if (g0 + s < g1) {
        s_next = __ldg(srow + g0 + s);
        m_next = __ldg(mrow + g0 + s);
      }
      for (int gg = g0 + s; gg < g1; gg += kSets, ++q, ++used) {
        const uint16_t s16 = s_next, m16 = m_next;
        if (gg + kSets < g1) {  // the set's next group's scale and min
          s_next = __ldg(srow + gg + kSets);
          m_next = __ldg(mrow + gg + kSets);
        }
        const int slot = used % nst;
        if (ok) ok = mbar_wait(full(s, slot), (used / nst) & 1, ERR_MM4_WAIT);
        uint4 w4[4];
        if (ok) {
          const uint8_t* rowp = stage_of(s, slot) + rib * 64;
#pragma unroll
          for (int c = 0; c < 4; ++c) w4[c] = lds128(rowp + ((c ^ ((rib >> 1) & 3)) << 4));
        }
        if constexpr (kBf16X) {
          // the stage's two X atoms (BT rows x 128 bytes each), bf16 -> fp16 in place; the MMA issuer reads them
          // only after this set's afull arrival below, and the proxy fence makes the writes visible to it
          if (ok) {
            uint8_t* xa = stage_of(s, slot) + kCodeBytes;
            for (int c = rib; c < BT * 16; c += 128) {
              uint4 v = *reinterpret_cast<const uint4*>(xa + c * 16);
              v.x = bf16x2_to_f16x2(v.x);
              v.y = bf16x2_to_f16x2(v.y);
              v.z = bf16x2_to_f16x2(v.z);
              v.w = bf16x2_to_f16x2(v.w);
              *reinterpret_cast<uint4*>(xa + c * 16) = v;
            }
            fence_proxy_async_smem();
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(s, slot));  // codes are in registers
        const uint32_t s2 = static_cast<uint32_t>(s16) * 0x10001u, m2 = static_cast<uint32_t>(m16) * 0x10001u;
        uint32_t o[64];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t wv[4] = {w4[c].x, w4[c].y, w4[c].z, w4[c].w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
#pragma unroll
            for (int bj = 0; bj < 4; ++bj) {  // byte bj of word: columns 2 bj, 2 bj + 1 of these 8
              const uint32_t spread = __byte_perm(wv[t], 0u, 0x4040u | (0x0101u * bj));
              const uint32_t tt = and_or(spread, mask, magic);  // (1024 + lo, 64 + hi), exact
              o[c * 16 + t * 4 + bj] = mm4::hfma2_u(mm4::hsub2_u(tt, magic), s2, m2);  // (lo, hi) * s + m
            }
          }
        }
        const int b = q % kNB;
        ok = __all_sync(0xffffffffu, ok);
        if (q >= kNB && ok) ok = __all_sync(0xffffffffu, mbar_wait(mdone(s, b), ((q / kNB) - 1) & 1, ERR_MM4_WAIT));
        if (ok) {
          mm4::tc_fence_after();
          g4t::tmem_st32(a_set + b * kACols, o);
          g4t::tmem_st32(a_set + b * kACols + 32, o + 32);
          g4t::tmem_wait_st();
          mm4::tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(afull(s, b));
      }
      // ---- epilogue of this item: D0 + D1 in that order; set s stores every other 32-column chunk ----
      if (!waited) {
        griddep_wait();  // Y (and a reused workspace) may still be read by the previous kernel
        waited = true;
      }
      for (int t = 0; t < kSets; ++t)
        if (ok) ok = mbar_wait(dready(t), jj & 1, ERR_MM4_WAIT);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        mm4::tc_fence_after();
        for (int c0 = 32 * s; c0 < BT; c0 += 32 * kSets) {
          float acc[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = 0.f;
          for (int t = 0; t < kSets; ++t) {
            if (t >= g1 - g0) break;  // that set had no group in this item
            uint32_t v[32];
            tmem_ld32(tq + t * kSetCols + kNB * kACols + c0, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] += __uint_as_float(v[i]);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int tok = t0 + c0 + i;  // columns past BT belong to no token of this chunk
            if (row_ok && c0 + i < BT && tok < p.M) {
              if (p.kslices == 1)
                store_out(p.y, static_cast<int64_t>(tok) * p.ldy + row, acc[i], p.y_bf16);
              else
                p.ws[(static_cast<int64_t>(ks) * p.M + tok) * p.N + row] = acc[i];
            }
          }
        }
        mm4::tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(dfree);
    }
  }
  mm4::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mm4::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Y[t, n] = sum over slices (in slice order) of ws[slice][t][n].
__global__ void __launch_bounds__(256) mm_int4_reduce_kernel(const float* ws, void* y, int64_t ldy, int M, int N,
                                                             int kslices, int y_bf16) {
  griddep_wait();
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t i = blockIdx.x * 256 + threadIdx.x; i < total; i += static_cast<int64_t>(gridDim.x) * 256) {
    float acc = 0.f;
    for (int k = 0; k < kslices; ++k) acc += ws[k * total + i];
    const int64_t t = i / N, n = i - t * N;
    store_out(y, t * ldy + n, acc, y_bf16);
  }
}

// Token chunking and K slicing of a call: chunks of <= 128 tokens; K is split into slices (>= 2 groups each)
// when the row-block x chunk items would leave SMs idle.
struct MmPlan {
  int BT, nchunks, kslices, gps;
};
inline MmPlan mm_plan(int64_t M, int64_t N, int64_t K, int num_sms) {
  MmPlan pl;
  const int64_t nch = (M + 127) / 128;
  const int64_t BT = (M + nch - 1) / nch;
  pl.BT = static_cast<int>(std::max<int64_t>(16, (BT + 15) / 16 * 16));
  pl.nchunks = static_cast<int>((M + pl.BT - 1) / pl.BT);
  const int G = static_cast<int>(K / 128);
  const int64_t items = (N + kRows - 1) / kRows * pl.nchunks;  // int64: M and N may each be up to 2^30
  int ks = 1;
  if (2 * items <= num_sms) ks = std::min(static_cast<int>(num_sms / items), G / 2);  // at most one wave of items
  ks = std::max(ks, 1);
  pl.gps = (G + ks - 1) / ks;
  pl.kslices = (G + pl.gps - 1) / pl.gps;
  return pl;
}

}  // namespace mm4t

// Scratch of the no-allocation entry point (rb_mm_int4_static): the split-K partials live in this file-scope
// array instead of a caller-provided workspace. 8 MiB bounds calls to kslices * M * N * 4 <= 8 MiB (e.g. the
// M = 34 prefill of every config-1 matrix needs at most 2.5 MiB). Every element a reduce reads is written by
// the same call first, so nothing needs to start at zero. The array is shared: calls that overlap in time
// (two streams, or two calls in flight without stream order) race on it.
constexpr int64_t kStaticScratchBytes = int64_t(8) << 20;
static __device__ __align__(256) float g_mm_scratch[kStaticScratchBytes / 4];

int64_t mm_int4_tc_workspace(int64_t M, int64_t N, int64_t K, int num_sms) {
  const mm4t::MmPlan pl = mm4t::mm_plan(M, N, K, num_sms);
  return pl.kslices > 1 ? static_cast<int64_t>(pl.kslices) * M * N * 4 : 0;
}

int launch_mm_int4_tc(const MmArgs& a, int num_sms, cudaStream_t stream) {
  using namespace mm4t;
  if (a.x_dtype != RB_F16 && a.x_dtype != RB_BF16) return RB_ERR_DTYPE;
  // the work-item count must fit the kernel's int arithmetic
  if ((a.N + kRows - 1) / kRows * ((a.M + 15) / 16) > (int64_t(1) << 30)) return RB_ERR_SHAPE;
  auto encode = mm4::encode_fn();
  if (!encode) return RB_ERR_DEVICE;
  const int M = static_cast<int>(a.M), N = static_cast<int>(a.N), K = static_cast<int>(a.K);
  MmPlan pl = mm_plan(M, N, K, num_sms);
  if (pl.kslices > 1 && (!a.ws || a.ws_bytes < static_cast<int64_t>(pl.kslices) * M * N * 4)) {
    pl.kslices = 1;  // no (or too small a) workspace: no split
    pl.gps = K / 128;
  }
  const int BT = pl.BT;
  MmtParams p;
  p.ws = a.ws;
  p.kslices = pl.kslices;
  p.gps = pl.gps;
  p.s = a.s;
  p.m = a.m;
  p.y = a.Y;
  p.ldy = a.ldy;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = K / 128;
  p.BT = BT;
  p.nchunks = pl.nchunks;
  p.nitems = ((N + kRows - 1) / kRows) * p.nchunks * p.kslices;
  p.y_bf16 = a.y_dtype == RB_BF16;
  p.prefetch = 0;
  p.stage_bytes = (kCodeBytes + 2u * BT * 128u + 1023u) & ~1023u;
  constexpr uint32_t kSmemMax = 227 * 1024;
  int nst = static_cast<int>((kSmemMax - 1024 - 512) / (kSets * p.stage_bytes));
  nst = std::min(nst, kMaxStages);
  if (nst < 2) return RB_ERR_SHAPE;
  p.nst = nst;
  p.bar_off = static_cast<uint32_t>(kSets * nst) * p.stage_bytes;
  // instruction descriptor: D f32, A f16, B f16, both K-major, N = BT, M = 128
  p.idesc = (1u << 4) | (static_cast<uint32_t>(BT >> 3) << 17) | (static_cast<uint32_t>(kRows >> 4) << 24);
  const uint32_t smem = 1024 + p.bar_off + (kSets * (2 * nst + 2 * kNB + 1) + 1) * 8 + 16;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(N)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K / 2)};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kRows)};
    const cuuint32_t es[2] = {1, 1};
    if (encode(&p.qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.q), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return RB_ERR_SHAPE;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.ldx) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(BT)};
    const cuuint32_t es[2] = {1, 1};
    const CUtensorMapDataType xt =
        a.x_dtype == RB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (encode(&p.xmap, xt, 2, const_cast<void*>(a.X), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return RB_ERR_SHAPE;
  }
  void (*kern)(MmtParams) = a.x_dtype == RB_BF16 ? mm_int4_tc_kernel<true> : mm_int4_tc_kernel<false>;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), kSmemMax);
  if (e != cudaSuccess) return RB_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(num_sms, p.nitems));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (a.flags & RB_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return RB_ERR_LAUNCH;
  if (p.kslices > 1) {
    cudaLaunchConfig_t rc = {};
    const int64_t total = static_cast<int64_t>(M) * N;
    rc.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 4 * num_sms)));
    rc.blockDim = dim3(256);
    rc.stream = stream;
    rc.attrs = attr;
    rc.numAttrs = 1;
    e = cudaLaunchKernelEx(&rc, mm_int4_reduce_kernel, static_cast<const float*>(p.ws), a.Y, a.ldy, M, N,
                           p.kslices, p.y_bf16);
    if (e != cudaSuccess) return RB_ERR_LAUNCH;
  }
  return RB_OK;
}

// rb_mm_int4_static: the split-K scratch from g_mm_scratch; allocates nothing. RB_ERR_SHAPE when the call's
// split would need more than kStaticScratchBytes.
int launch_mm_int4_tc_static(MmArgs a, int num_sms, cudaStream_t stream) {
  const int64_t need = mm_int4_tc_workspace(a.M, a.N, a.K, num_sms);
  if (need > kStaticScratchBytes) return RB_ERR_SHAPE;
  a.ws = nullptr;
  a.ws_bytes = 0;
  if (need > 0) {
    // the symbol's device address, looked up once per device (return code checked)
    static std::atomic<void*> addr[64] = {};  // host threads may race here; they all store the same address
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return RB_ERR_DEVICE;
    void* p = addr[dev].load(std::memory_order_acquire);
    if (!p) {
      if (cudaGetSymbolAddress(&p, g_mm_scratch) != cudaSuccess || !p) {
        (void)cudaGetLastError();
        return RB_ERR_DEVICE;
      }
      addr[dev].store(p, std::memory_order_release);
    }
    a.ws = static_cast<float*>(p);
    a.ws_bytes = kStaticScratchBytes;
  }
  return launch_mm_int4_tc(a, num_sms, stream);
}

}  // namespace rb
