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
// Work items are (128-row weight block, token chunk of BT <= 256 tokens, K slice), block-major so that the CTAs
// working at the same time on the chunks of one block share its codes through L2; items are dealt round-robin
// to one CTA per SM. Per CTA, for the groups of its items in order (a CTA-wide group sequence gq):
//  * warp 0 (producer) streams each group's codes (TMA box 64 bytes x 128 rows, 64-byte swizzle) and the chunk's
//    two 64-column X atoms (TMA, 128-byte swizzle) into one shared ring of stages;
//  * three converter sets (four warps each, thread = weight row = tensor-memory lane) take the groups in turn
//    (gq % 3): each dequantises its row's group to fp16 (per code byte: PRMT, LOP3 to the fp16 magic numbers,
//    HSUB2, HFMA2 with the row's scale and min, one rounding) and writes the 64 columns into the next of a ring
//    of tensor-memory A buffers (gq % NA; NA = 4..7 by the accumulator's width);
//  * ND MMA issuers (one thread each, warps 1..ND; ND = 3 for chunks of <= 64 tokens, 2 for <= 128, 1 for <= 256)
//    take the groups in turn (gq % ND): each issues eight tcgen05.mma.kind::f16 per group (M = 128, N = BT,
//    K = 16) in group order into ITS accumulator D_d = 128 x BT fp32 in tensor memory: A from the group's buffer,
//    B = the X atoms in shared memory. An MMA costs about 100 cycles to issue whatever its N (measured), so short
//    chunks spread their groups over several issuers, and up to 256 tokens share one dequantisation of the
//    weights;
//  * after the item's last group all twelve converter warps read D_0 + ... + D_{ND-1} in that order
//    (deterministic; tcgen05.ld, 32-column chunks dealt over the three warps of each lane quadrant) and store Y,
//    or, when K is split into slices (a call with fewer row-block x chunk items than SMs), the slice's fp32
//    partial into a caller-provided workspace; mm_int4_reduce then adds the slices in slice order. Chunks of
//    <= 128 tokens go through a 32 KB shared staging tile and one bulk-tensor store per round (per-thread
//    stores cost several times more); 256-token chunks store directly and keep shared memory for three stages.
//  * the producer brings a group's codes with one TMA copy and both of its X atoms with one 3-D copy.
// All mbarrier waits are bounded; no multicast, no clusters.
#include <new>

#include "common.cuh"
#include "tc.cuh"
#include "kernels.h"

namespace rb {

namespace mm4t {

constexpr int kSets = 3;
constexpr int kRows = 128;
constexpr int kMaxIssuers = 3;
constexpr int kFirstConv = 1 + kMaxIssuers;  // warp 0 producer, warps 1..3 MMA issuers (warp 1 owns tensor memory)
constexpr int kConvWarps = 4 * kSets;
constexpr int kThreads = (kFirstConv + kConvWarps) * 32;
constexpr uint32_t kCodeBytes = kRows * 64;
constexpr uint32_t kACols = 64;              // one group of fp16 weights: 128 lanes x 64 columns
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxStages = 12;
constexpr int kMaxBT = 256;
constexpr uint32_t kOutBytes = 32768;        // the epilogue's staging tile for bulk-tensor stores (BT <= 128)
constexpr int kBarEpi = 1;                   // named barrier of the twelve converter warps

// One matrix of a launch: its tensor maps, scales, output and the range of work items it owns.
struct __align__(64) MmEntry {
  CUtensorMap qmap;  // [N rows, K/2 bytes], box 64 x 128, 64-byte swizzle
  CUtensorMap xmap;  // x3d: {64 columns, M rows, K/64 atoms}, box 64 x BT x 2 (both atoms of a group in one copy);
                     // else [M rows, K fp16], box 64 x BT; 128-byte swizzle
  CUtensorMap omap;  // ostore 1: Y [M, N] (box 128 x tc); 2: the workspace [kslices, M, N] fp32 (box 128 x tc x 1)
  const uint16_t* s;
  const uint16_t* m;
  void* y;
  float* ws;  // [kslices][M][N] fp32 partials when kslices > 1
  int64_t ldy;
  int N, K, G, nchunks, kslices, gps, item_begin;
  int ostore, tc;  // epilogue: 0 plain stores, 1 / 2 bulk-tensor stores of Y / the workspace, tc tokens a round
  int x3d;
};

// A launch: kE entries (1 for rb_mm_int4*, up to kListEntries for rb_mm_int4_list) sharing M, the token chunk
// width BT and the shared-memory and tensor-memory layout.
template <int kE>
struct __align__(64) MmtParams {
  MmEntry e[kE];
  int count, M, BT, nitems, y_bf16, nst, na, nd;
  uint32_t stage_bytes, out_off, bar_off, idesc, dcols;  // dcols: columns per accumulator; A buffers from nd * dcols
};
constexpr int kListEntries = 52;
static_assert(sizeof(MmtParams<kListEntries>) <= 32000, "kernel parameter block too large");

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

// Bulk-tensor stores shared -> global through a tensor map (no multicast), their bulk group, and the waits: the
// source may be rewritten once `read` completes; the kernel ends only after the writes complete.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
               "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(map), "r"(x),
               "r"(y), "r"(z), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Item `item`: its entry, first weight row, first token and group range [g0, g1). Entries own consecutive item
// ranges and a role's items only increase, so the entry cursor `cur` only moves forward.
struct Item {
  int e, row0, t0, ks, g0, g1;
};
template <int kE>
__device__ __forceinline__ Item item_of(const MmtParams<kE>& p, int item, int& cur) {
  while (cur + 1 < p.count && item >= p.e[cur + 1].item_begin) ++cur;
  const MmEntry& E = p.e[cur];
  Item it;
  it.e = cur;
  const int li = item - E.item_begin;
  const int per_block = E.nchunks * E.kslices;
  const int rem = li % per_block;
  it.row0 = (li / per_block) * kRows;
  it.t0 = (rem / E.kslices) * p.BT;
  it.ks = rem % E.kslices;
  it.g0 = it.ks * E.gps;
  it.g1 = min(E.G, it.g0 + E.gps);
  return it;
}

template <bool kBf16X, int kE>
__global__ void __launch_bounds__(kThreads, 1) mm_int4_tc_kernel(const __grid_constant__ MmtParams<kE> p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = gridDim.x, cta = blockIdx.x;
  const int nst = p.nst, na = p.na, nd = p.nd, BT = p.BT;
  const uint32_t a_base = static_cast<uint32_t>(nd) * p.dcols;
  const int nlocal = (p.nitems - cta + C - 1) / C;  // this CTA's items: cta + j * C
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* full = bars;                 // [nst] producer -> converters (codes) and MMA issuer (X)
  uint64_t* empty = bars + nst;          // [nst] four converter warps + one MMA commit
  uint64_t* afull = bars + 2 * nst;      // [na] the converting set's four warps
  uint64_t* mdone = afull + na;          // [na] MMA commit: the A buffer may be rewritten
  uint64_t* dready = mdone + na;         // [kMaxIssuers] issuer d's commit after its last group of an item
  uint64_t* dfree = dready + kMaxIssuers;  // the twelve converter warps have read the accumulators
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfree + 1);
  auto stage_of = [&](int slot) { return smem + static_cast<size_t>(slot) * p.stage_bytes; };

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 5);
    }
    for (int b = 0; b < na; ++b) {
      mbar_init(afull + b, 4);
      mbar_init(mdone + b, 1);
    }
    for (int d = 0; d < kMaxIssuers; ++d) mbar_init(dready + d, 1);
    mbar_init(dfree, kConvWarps);
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
      int pre = 0, cur = 0;
      for (int j = 0; j < nlocal && pre < nst; ++j) {
        const Item it = item_of(p, cta + j * C, cur);
        for (int g = it.g0; g < it.g1 && pre < nst; ++g, ++pre) {
          mbar_arrive_expect_tx(full + pre, stage_tx);
          mm4::tma_load_2d(stage_of(pre), &p.e[it.e].qmap, g * 64, it.row0, full + pre);
        }
      }
      griddep_wait();  // X may come from the previous kernel
      int gq = 0;
      bool ok = true;
      cur = 0;
      for (int j = 0; j < nlocal && ok; ++j) {
        const Item it = item_of(p, cta + j * C, cur);
        const MmEntry& E = p.e[it.e];
        for (int g = it.g0; g < it.g1; ++g, ++gq) {
          const int slot = gq % nst;
          uint8_t* st = stage_of(slot);
          if (gq >= pre) {
            if (!mbar_wait(empty + slot, ((gq / nst) - 1) & 1, ERR_MM4_WAIT)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full + slot, stage_tx);
            mm4::tma_load_2d(st, &E.qmap, g * 64, it.row0, full + slot);
          }
          if (E.x3d) {
            mm4::tma_load_3d(st + kCodeBytes, &E.xmap, 0, it.t0, 2 * g, full + slot);
          } else {
            mm4::tma_load_2d(st + kCodeBytes, &E.xmap, g * 128, it.t0, full + slot);
            mm4::tma_load_2d(st + kCodeBytes + BT * 128, &E.xmap, g * 128 + 64, it.t0, full + slot);
          }
        }
      }
      // no retirement with copies in flight
      for (int t = max(0, gq - nst); t < gq; ++t)
        if (!mbar_wait(full + t % nst, (t / nst) & 1, ERR_MM4_WAIT)) break;
    }
  } else if (warp < kFirstConv) {
    // ---------------- MMA issuer d: the groups gq % nd == d, into accumulator d ----------------
    const int d = warp - 1;
    if (lane == 0 && d < nd) {
      int gq = 0, cur = 0;
      bool ok = true;
      const uint32_t dcol = tmem + static_cast<uint32_t>(d) * p.dcols;
      for (int jj = 0; jj < nlocal && ok; ++jj) {
        if (jj >= 1 && !mbar_wait(dfree, (jj - 1) & 1, ERR_MM4_WAIT)) break;  // read by the last epilogue
        mm4::tc_fence_after();
        const Item it = item_of(p, cta + jj * C, cur);
        bool first = true;
        for (int g = it.g0; g < it.g1; ++g, ++gq) {
          if (gq % nd != d) continue;
          const int b = gq % na, slot = gq % nst;
          if (!mbar_wait(afull + b, (gq / na) & 1, ERR_MM4_WAIT) ||
              !mbar_wait(full + slot, (gq / nst) & 1, ERR_MM4_WAIT)) {
            ok = false;
            break;
          }
          mm4::tc_fence_after();
          const uint32_t xb = smem_u32(stage_of(slot) + kCodeBytes);
          const uint32_t a = tmem + a_base + b * kACols;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            umma_ts_f16(dcol, a + 8 * i, mm4::sw128_desc(xb + (i >> 2) * BT * 128 + (i & 3) * 32), p.idesc,
                        !first || i != 0);
          first = false;
          mm4::umma_commit(mdone + b);     // A buffer b may be rewritten
          mm4::umma_commit(empty + slot);  // the stage's X atoms may be refilled
        }
        if (ok) mm4::umma_commit(dready + d);  // accumulator d holds its groups' sum (arrives at once if none)
      }
    }
  } else {
    // ---------------- converters (set s takes the groups gq % kSets == s) + epilogue ----------------
    const int cw = warp - kFirstConv;
    const int s = cw >> 2;
    const int quad = warp & 3;  // tensor-memory lane quadrant this warp may access
    const int rib = quad * 32 + lane;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t magic = 0x54006400u, mask = 0x00F0000Fu;  // (1024 | low nibble, 64 | high nibble << 4)
    bool waited = false;  // griddepcontrol.wait before the first write of Y or of the workspace
    int gq = 0, cur = 0;
    bool ok = true;
    for (int jj = 0; jj < nlocal; ++jj) {
      const Item it = item_of(p, cta + jj * C, cur);
      const MmEntry& E = p.e[it.e];
      const int row = it.row0 + rib;
      const bool row_ok = row < E.N;
      const uint16_t* srow = E.s + static_cast<int64_t>(row_ok ? row : 0) * E.G;
      const uint16_t* mrow = E.m + static_cast<int64_t>(row_ok ? row : 0) * E.G;
      // this set's first group of the item, and its scale and min fetched one of the set's groups ahead
      int g = it.g0 + ((s - gq % kSets) + kSets) % kSets;
      uint16_t s_next = 0, m_next = 0;
      if (g < it.g1) {
        s_next = __ldg(srow + g);
        m_next = __ldg(mrow + g);
      }
      for (; g < it.g1; g += kSets) {
        const int q = gq + (g - it.g0);  // this group's place in the CTA's sequence
        const uint16_t s16 = s_next, m16 = m_next;
        if (g + kSets < it.g1) {
          s_next = __ldg(srow + g + kSets);
          m_next = __ldg(mrow + g + kSets);
        }
        const int slot = q % nst;
        if (ok) ok = mbar_wait(full + slot, (q / nst) & 1, ERR_MM4_WAIT);
        uint4 w4[4];
        if (ok) {
          const uint8_t* rowp = stage_of(slot) + rib * 64;
#pragma unroll
          for (int c = 0; c < 4; ++c) w4[c] = lds128(rowp + ((c ^ ((rib >> 1) & 3)) << 4));
        }
        if constexpr (kBf16X) {
          // the stage's two X atoms (BT rows x 128 bytes each), bf16 -> fp16 in place; the MMA issuer reads them
          // only after this set's afull arrival below, and the proxy fence makes the writes visible to it
          if (ok) {
            uint8_t* xa = stage_of(slot) + kCodeBytes;
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
        if (lane == 0) mbar_arrive(empty + slot);  // codes are in registers
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
        const int b = q % na;
        ok = __all_sync(0xffffffffu, ok);
        if (q >= na && ok) ok = __all_sync(0xffffffffu, mbar_wait(mdone + b, ((q / na) - 1) & 1, ERR_MM4_WAIT));
        if (ok) {
          mm4::tc_fence_after();
          const uint32_t a = tq + a_base + b * kACols;
          g4t::tmem_st32(a, o);
          g4t::tmem_st32(a + 32, o + 32);
          g4t::tmem_wait_st();
          mm4::tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(afull + b);
      }
      gq += it.g1 - it.g0;
      // ---- epilogue of this item: 32-column chunks of D over the three warps of each lane quadrant ----
      if (!waited) {
        griddep_wait();  // Y (and a reused workspace) may still be read by the previous kernel
        waited = true;
      }
      for (int d = 0; d < nd; ++d)
        if (ok) ok = mbar_wait(dready + d, jj & 1, ERR_MM4_WAIT);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) mm4::tc_fence_after();
      const int gq0 = gq - (it.g1 - it.g0);  // the item's first group in the CTA's sequence
      // D_0 + ... + D_{nd-1} (issuers without a group in this item skipped) of the 32 columns from c0
      auto sum_d = [&](int c0, float (&acc)[32]) {
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        for (int d = 0; d < nd; ++d) {
          if ((d - gq0 % nd + nd) % nd >= it.g1 - it.g0) continue;
          uint32_t v[32];
          tmem_ld32(tq + static_cast<uint32_t>(d) * p.dcols + c0, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] += __uint_as_float(v[i]);
        }
      };
      if (E.ostore) {
        // rounds of tc tokens: every converter warp writes its 32-column chunks of D into the staging tile
        // [token][128 rows] in the output's type, then one thread stores the tile with one bulk-tensor copy (rows
        // past N and tokens past M are clipped by the tensor map). Every converter warp takes every barrier,
        // whatever `ok` is.
        uint8_t* out = smem + p.out_off;
        const int esz = E.ostore == 2 ? 4 : 2;
        const int ct = cw * 32 + lane;
        for (int tc0 = 0; tc0 < BT; tc0 += E.tc) {
          if (ct == 0) bulk_wait_read();  // the last store has read the staging tile
          named_bar_sync(kBarEpi, kConvWarps * 32);
          for (int c0 = tc0 + 32 * s; c0 < min(BT, tc0 + E.tc); c0 += 32 * kSets) {
            float acc[32];
            if (ok) {
              sum_d(c0, acc);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              uint8_t* dst = out + (static_cast<uint32_t>(c0 - tc0 + i) * kRows + rib) * esz;
              if (esz == 4)
                *reinterpret_cast<float*>(dst) = acc[i];
              else if (p.y_bf16)
                *reinterpret_cast<__nv_bfloat16*>(dst) = __float2bfloat16_rn(acc[i]);
              else
                *reinterpret_cast<__half*>(dst) = __float2half_rn(acc[i]);
            }
          }
          fence_proxy_async_smem();
          named_bar_sync(kBarEpi, kConvWarps * 32);
          if (ct == 0) {
            if (E.ostore == 2)
              tma_store_3d(&E.omap, smem_u32(out), it.row0, it.t0 + tc0, it.ks);
            else
              tma_store_2d(&E.omap, smem_u32(out), it.row0, it.t0 + tc0);
            bulk_commit();
          }
        }
      } else if (ok) {
        for (int c0 = 32 * s; c0 < BT; c0 += 32 * kSets) {
          float acc[32];
          sum_d(c0, acc);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int tok = it.t0 + c0 + i;  // columns past BT belong to no token of this chunk
            if (row_ok && c0 + i < BT && tok < p.M) {
              if (E.kslices == 1)
                store_out(E.y, static_cast<int64_t>(tok) * E.ldy + row, acc[i], p.y_bf16);
              else
                E.ws[(static_cast<int64_t>(it.ks) * p.M + tok) * E.N + row] = acc[i];
            }
          }
        }
      }
      if (ok) mm4::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dfree);
    }
  }
  if (warp == kFirstConv && lane == 0) bulk_wait_all();  // the epilogue's bulk stores have landed
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

// Token chunking and K slicing of a call. Chunks of up to `width` tokens (128 or 256: one dequantisation of a
// group then feeds up to 256 tokens); K is split into slices (>= 2 groups each) when the row-block x chunk items
// would leave SMs idle. Of the two widths the plan takes the one with the smaller estimated time of the busiest
// CTA: its items x (groups x the time of one group + the item's epilogue). Measured per group: about 1.05 us at
// 128 tokens and 1.2 us at 256 (the stage ring, not the tensor rate, paces it), i.e. (BT + 750) in units of one
// token-column; the epilogue about 1,700 units through the staging tile (BT <= 128) and 5,000 with plain stores.
struct MmPlan {
  int BT, nchunks, kslices, gps;
  int64_t cost;
};
inline MmPlan mm_plan_width(int64_t M, int64_t N, int64_t K, int num_sms, int64_t width) {
  MmPlan pl;
  const int64_t nch = (M + width - 1) / width;
  const int64_t BT = (M + nch - 1) / nch;
  // a multiple of 16 (the MMA's N); of 32 when there are several chunks, so that the epilogue's rounds of whole
  // 32-token pieces never reach into the next chunk's tokens
  const int64_t mult = nch > 1 ? 32 : 16;
  pl.BT = static_cast<int>(std::max<int64_t>(16, (BT + mult - 1) / mult * mult));
  pl.nchunks = static_cast<int>((M + pl.BT - 1) / pl.BT);
  const int G = static_cast<int>(K / 128);
  const int64_t items = (N + kRows - 1) / kRows * pl.nchunks;  // int64: M and N may each be up to 2^30
  int ks = 1;
  if (2 * items <= num_sms) ks = std::min(static_cast<int>(num_sms / items), G / 2);  // at most one wave of items
  ks = std::max(ks, 1);
  pl.gps = (G + ks - 1) / ks;
  pl.kslices = (G + pl.gps - 1) / pl.gps;
  const int64_t waves = (items * pl.kslices + num_sms - 1) / num_sms;
  pl.cost = waves * (static_cast<int64_t>(pl.gps) * (pl.BT + 750) + (pl.BT <= 128 ? 1700 : 5000));
  return pl;
}
inline MmPlan mm_plan(int64_t M, int64_t N, int64_t K, int num_sms) {
  const MmPlan a = mm_plan_width(M, N, K, num_sms, 128);
  if (M <= 128) return a;
  const MmPlan b = mm_plan_width(M, N, K, num_sms, kMaxBT);
  return b.cost < a.cost ? b : a;
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

namespace mm4t {

constexpr uint32_t kSmemMax = 227 * 1024;

// The launch-wide layout for chunks of BT tokens: accumulators (3 of 64 columns for chunks of <= 64 tokens: an
// MMA's issue cost, about 66 cycles, is above the tensor time of N <= 64; 2 of 128 for 65..127 tokens; 1 for
// 128..256, where one issuer reaches the tensor rate), the A buffers after them, the stage ring, the staging tile
// (chunks of <= 128 tokens; 256-token stages of 72 KB keep all of shared memory) and the barriers. Returns the
// dynamic shared-memory bytes, or 0 if two stages do not fit.
template <int kE>
uint32_t set_layout(MmtParams<kE>& p, int M, int BT, int y_dtype) {
  p.M = M;
  p.BT = BT;
  p.y_bf16 = y_dtype == RB_BF16;
  p.nd = BT <= 64 ? 3 : (BT < 128 ? 2 : 1);
  p.dcols = p.nd == 3 ? 64u : (BT <= 128 ? 128u : 256u);
  p.na = std::min(7, static_cast<int>((kTmemCols - p.nd * p.dcols) / kACols));
  p.stage_bytes = (kCodeBytes + 2u * BT * 128u + 1023u) & ~1023u;
  const uint32_t bar_bytes = (2 * kMaxStages + 2 * 7 + kMaxIssuers + 1) * 8 + 16;
  const uint32_t out_bytes = BT <= 128 ? kOutBytes : 0u;
  int nst = static_cast<int>((kSmemMax - 1024 - out_bytes - bar_bytes) / p.stage_bytes);
  nst = std::min(nst, kMaxStages);
  if (nst < 2) return 0;
  p.nst = nst;
  p.out_off = static_cast<uint32_t>(nst) * p.stage_bytes;
  p.bar_off = p.out_off + out_bytes;
  // instruction descriptor: D f32, A f16, B f16, both K-major, N = BT, M = 128
  p.idesc = (1u << 4) | (static_cast<uint32_t>(BT >> 3) << 17) | (static_cast<uint32_t>(kRows >> 4) << 24);
  return 1024 + p.bar_off + (2 * nst + 2 * p.na + kMaxIssuers + 1) * 8 + 16;
}

// One matrix's entry: tensor maps of its codes, of X and of its output; item range from `item_begin`.
int set_entry(MmEntry& E, const MmArgs& a, int M, int BT, int nchunks, int kslices, int gps, int item_begin,
              PFN_cuTensorMapEncodeTiled_v12000 encode) {
  const int N = static_cast<int>(a.N), K = static_cast<int>(a.K);
  E.s = a.s;
  E.m = a.m;
  E.y = a.Y;
  E.ws = a.ws;
  E.ldy = a.ldy;
  E.N = N;
  E.K = K;
  E.G = K / 128;
  E.nchunks = nchunks;
  E.kslices = kslices;
  E.gps = gps;
  E.item_begin = item_begin;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(N)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K / 2)};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kRows)};
    const cuuint32_t es[2] = {1, 1};
    if (encode(&E.qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.q), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return RB_ERR_SHAPE;
  }
  {
    // X as {64 columns, M rows, K/64 atoms of 64 columns}: one copy brings a group's two atoms, stacked as the MMA
    // descriptor reads them ([atom][token][64], each atom 1024-byte aligned since BT % 16 == 0). Every element
    // it addresses lies inside X. If the driver refuses the view, two 2-D copies per group.
    const CUtensorMapDataType xt =
        a.x_dtype == RB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint64_t dims3[3] = {64, static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(K / 64)};
    const cuuint64_t strides3[2] = {static_cast<cuuint64_t>(a.ldx) * 2, 128};
    const cuuint32_t box3[3] = {64, static_cast<cuuint32_t>(BT), 2};
    const cuuint32_t es3[3] = {1, 1, 1};
    E.x3d = encode(&E.xmap, xt, 3, const_cast<void*>(a.X), dims3, strides3, box3, es3, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    if (!E.x3d) {
      const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
      const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.ldx) * 2};
      const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(BT)};
      const cuuint32_t es[2] = {1, 1};
      if (encode(&E.xmap, xt, 2, const_cast<void*>(a.X), dims, strides, box, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return RB_ERR_SHAPE;
    }
  }
  // The epilogue's bulk-tensor store: Y when its rows start 16-byte aligned at a 16-byte multiple pitch, the fp32
  // workspace [kslices, M, N] when N % 4 == 0; otherwise plain stores. Tokens past M and rows past N are clipped.
  // A round stores tc tokens: all BT in fp16/bf16 (BT <= 128 fits the 32 KB tile); in fp32 BT when BT <= 64,
  // else 64 or 32 (BT is then a multiple of 32, or the chunk is the call's only one and tokens past M are clipped).
  E.ostore = 0;
  E.tc = 0;
  if (BT > 128) {
    // plain stores
  } else if (kslices == 1) {
    if ((reinterpret_cast<uintptr_t>(a.Y) & 15u) == 0 && (a.ldy * 2) % 16 == 0) {
      E.tc = BT;
      const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
      const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.ldy) * 2};
      const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRows), static_cast<cuuint32_t>(E.tc)};
      const cuuint32_t es[2] = {1, 1};
      const CUtensorMapDataType yt =
          a.y_dtype == RB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
      if (encode(&E.omap, yt, 2, a.Y, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
        E.ostore = 1;
    }
  } else if (N % 4 == 0 && (reinterpret_cast<uintptr_t>(a.ws) & 15u) == 0) {
    E.tc = BT <= 64 ? BT : (BT % 64 == 0 || nchunks == 1 ? 64 : 32);
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M),
                                static_cast<cuuint64_t>(kslices)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(N) * 4, static_cast<cuuint64_t>(M) * N * 4};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kRows), static_cast<cuuint32_t>(E.tc), 1};
    const cuuint32_t es[3] = {1, 1, 1};
    if (encode(&E.omap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a.ws, dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      E.ostore = 2;
  }
  return RB_OK;
}

template <int kE>
int launch_kernel(const MmtParams<kE>& p, int x_dtype, uint32_t smem, int num_sms, int flags, cudaStream_t stream) {
  void (*kern)(MmtParams<kE>) = x_dtype == RB_BF16 ? mm_int4_tc_kernel<true, kE> : mm_int4_tc_kernel<false, kE>;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), kSmemMax);
  if (e != cudaSuccess) return RB_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(num_sms, p.nitems));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (flags & RB_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

}  // namespace mm4t

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
  MmtParams<1> p;
  const uint32_t smem = set_layout(p, M, pl.BT, a.y_dtype);
  if (!smem) return RB_ERR_SHAPE;
  p.count = 1;
  p.nitems = ((N + kRows - 1) / kRows) * pl.nchunks * pl.kslices;
  int st = set_entry(p.e[0], a, M, pl.BT, pl.nchunks, pl.kslices, pl.gps, 0, encode);
  if (st != RB_OK) return st;
  st = launch_kernel(p, a.x_dtype, smem, num_sms, a.flags, stream);
  if (st != RB_OK) return st;
  if (pl.kslices > 1) {
    cudaLaunchConfig_t rc = {};
    const int64_t total = static_cast<int64_t>(M) * N;
    rc.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 4 * num_sms)));
    rc.blockDim = dim3(256);
    rc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (a.flags & RB_FLAG_PDL) ? 1 : 0;
    rc.attrs = attr;
    rc.numAttrs = 1;
    if (cudaLaunchKernelEx(&rc, mm_int4_reduce_kernel, static_cast<const float*>(a.ws), a.Y, a.ldy, M, N,
                           pl.kslices, p.y_bf16) != cudaSuccess)
      return RB_ERR_LAUNCH;
  }
  return RB_OK;
}

// A list of prefill matrices with one token count M in persistent launches of up to kListEntries entries each:
// items of all entries dealt round-robin to one CTA per SM, no K split (a list has items enough to fill the SMs).
// Chunk width: M <= 128 one chunk of roundup16(M) tokens; otherwise chunks of up to 256 (a multiple of 32).
int launch_mm_int4_list(const MmArgs* a, int count, int num_sms, cudaStream_t stream) {
  using namespace mm4t;
  if (count <= 0) return RB_OK;
  auto encode = mm4::encode_fn();
  if (!encode) return RB_ERR_DEVICE;
  const int M = static_cast<int>(a[0].M);
  const MmPlan pl = mm_plan_width(M, 1, 256, num_sms, M <= 128 ? 128 : kMaxBT);  // BT and chunks depend on M only
  for (int done = 0; done < count;) {
    const int n = std::min(count - done, kListEntries);
    auto* p = new (std::nothrow) MmtParams<kListEntries>;  // ~27 KB: not on the stack
    if (!p) return RB_ERR_LAUNCH;
    const uint32_t smem = set_layout(*p, M, pl.BT, a[done].y_dtype);
    if (!smem) {
      delete p;
      return RB_ERR_SHAPE;
    }
    int items = 0, st = RB_OK;
    for (int i = 0; i < n && st == RB_OK; ++i) {
      const MmArgs& x = a[done + i];
      if ((x.N + kRows - 1) / kRows * pl.nchunks + items > (int64_t(1) << 30)) st = RB_ERR_SHAPE;
      if (st == RB_OK)
        st = set_entry(p->e[i], x, M, pl.BT, pl.nchunks, 1, static_cast<int>(x.K / 128), items, encode);
      items += static_cast<int>((x.N + kRows - 1) / kRows) * pl.nchunks;
    }
    p->count = n;
    p->nitems = items;
    if (st == RB_OK) st = launch_kernel(*p, a[done].x_dtype, smem, num_sms, a[done].flags, stream);
    delete p;
    if (st != RB_OK) return st;
    done += n;
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
