// gemv_int4_multi.cu - one persistent launch for a list of independent int4 GEMVs (a decode step's
// projection set), batch 1, on B200 (sm_100a).
//
// A decode step issued as one kernel per GEMV pays a fixed cost per launch (launch, dependency wait,
// activation staging, tail) of several microseconds; 145 of them are as long as the whole step's HBM time.
// This kernel removes the boundaries for GEMVs whose inputs are all available at launch (the reference's
// projection-set benchmark, kernels/bench_gemv.py:83-113, and any set of independent projections):
//  * every activation vector of the list is converted to MMA B fragments once, at kernel start;
//  * the 16-row tiles of all matrices form one global list dealt round-robin to the CTAs (one per SM), so
//    every SM streams the same number of tiles, tile boundaries never stall the HBM stream, and one
//    producer warp keeps ~180 KB of tiles in flight per SM in a byte-granular FIFO ring (tiles of
//    different K have different sizes);
//  * each tile is split into work items for 16 consumer warps, which reuse the int4 GEMV's inner loop
//    (gemv4_load / gemv4_math: LOP3 magic-number dequantisation, m16n8k16 MMA as an fp32-accumulating dot
//    product) over all groups of the row and write its 8 outputs directly;
//  * full/empty mbarriers are per tile, reused modulo a window that is provably larger than any consumer's
//    lead over the oldest unreleased tile, so a waiting warp can never see a stale phase.
// Its per-launch cost is about half the tcgen05 multi-GEMV's (gemv_int4_tc.cu), so it runs the short lists: a
// decode layer's projections with the glue of glue.cuh (the add + LayerNorm prologue, the rope / KV and SwiGLU
// epilogues) and, optionally, the decode attention fused into the o_proj / down_proj launch (attn.cuh). The
// tcgen05 kernel runs the long, HBM-bound lists.
#include "common.cuh"
#include "glue.cuh"
#include "attn.cuh"
#include "kernels.h"

namespace rb {

namespace g4m {

// Build-time tuning (defaults measured best on B200): consumer warps, groups per work item, MMA chains per
// group.
#ifndef RB_MULTI_WARPS
#define RB_MULTI_WARPS 15
#endif
#ifndef RB_MULTI_SLICE_GROUPS
#define RB_MULTI_SLICE_GROUPS 12
#endif
#ifndef RB_MULTI_CHAINS
#define RB_MULTI_CHAINS 1
#endif
constexpr int kConsumerWarps = RB_MULTI_WARPS;
constexpr int kChains = RB_MULTI_CHAINS;
// Registers per thread for one CTA per SM: each of the SM's four sub-partitions has 16,384 registers and
// holds every fourth warp, allocated in multiples of 8 registers per thread.
constexpr int kWarpsPerPartition = (RB_MULTI_WARPS + 1 + 3) / 4;
constexpr int kMaxRegs = (16384 / (kWarpsPerPartition * 32)) / 8 * 8 > 255 ? 255
                                                                            : (16384 / (kWarpsPerPartition * 32)) / 8 * 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxEntries = 256;
constexpr int kMaxSlots = 8;
constexpr int kWindow = 128;       // barrier window (tiles)
constexpr int kRedSlots = 32;      // reduction slots (tiles), > kMaxOutstanding
constexpr int kMaxP = 8;           // K-slices per step at most
constexpr int kSliceGroups = RB_MULTI_SLICE_GROUPS;  // groups per work item at most
constexpr int kMaxOutstanding = 24;  // tiles in flight per CTA (window >= this + consumer warps)
// A tile's ring space is released when its empty barrier has counted kRelease arrivals: each work item
// arrives once with count 1, except the tile's last item, which arrives with kRelease - (ipt - 1).
constexpr int kRelease = 2 * kMaxP;

struct Entry {
  const uint8_t* q;
  const uint16_t* s;
  const uint16_t* m;
  void* y;
  int N, K, G, slot, tile_begin, pad;
  int epi, ep;  // epilogue kind (rb_epi_kind), index into MultiParams::epis
};

struct Slot {
  const void* x;  // activations; for the prologue slot (ln != 0) the residual stream of rb_add_ln
  const void* a;
  const void* b;
  const void* w;
  void* x_out;
  void* h_out;
  float eps;
  int ln;
  int K, G;
  uint32_t tab_off, cst_off;
  const int8_t* emb_q;  // prologue from a token's embedding row (rb_add_ln::emb_q)
  const void* emb_s;
  const int64_t* tok;
  int64_t vocab;
  int emb_f16;
  int att;  // the vector is the attention output computed inside the launch (staged once it is complete)
};

// Per-entry data kept in shared memory for the whole launch (per-tile lookups must not go to the
// parameter block: it is indexed dynamically, and its misses in the constant cache stalled the producer).
// What the producer needs:
struct __align__(16) EntryP {
  const uint8_t* q;
  const uint8_t* s;
  const uint8_t* m;
  int N, G, tile_begin;
  uint32_t tbytes, row_bytes, sblk;  // tile bytes in the ring, code bytes per row, bytes of one s (or m) block
};
// What the consumers need, plus this CTA's share of the entry: its tiles are the local tiles
// [jlo, jlo + n) and their work items are the CTA-local items [ib, ib + n * ipt). An extra entry after the
// last holds ib = the CTA's total item count.
struct __align__(16) EntryC {
  void* y;
  int N, tile_begin;
  int G, rs;                     // groups per row, code bytes per row
  uint32_t sblk, tab_off_x;      // s block bytes (the m block follows it); x table of its slot
  uint32_t cst_off_x;
  int P, gps, ipt;               // K-slices per 8-row step, groups per slice, items per tile (steps * P)
  int jlo, ib;
  uint32_t mag_ipt, mag_p;       // ceil(2^32 / ipt), ceil(2^32 / P): division by multiply-high
  int epi, ep;                   // epilogue kind and its index into MultiParams::epis
};

struct MultiParams {
  int count, nslots, total_tiles, x_bf16, y_bf16, prefetch;
  int maxp;  // largest K-slice count of the launch's entries (sizes the reduction area)
  uint32_t ring_bytes, ring_off, bar_off, start_off, zero_off, ent_off, red_off;
  uint32_t m_lo, m_hi, k1024, k64, ln_off;
  Slot slots[kMaxSlots];
  Entry e[kMaxEntries];
  EpiP epis[4];
  // decode attention fused into the launch (rb_attn_src): CTAs < att_ctas compute key-value head
  // cta / att.nsplit, split cta % att.nsplit with consumer warps 0-3; entries from att_entry on read its output
  attn::AttnParams att;
  int att_on, att_ctas, att_rep, att_entry, att_nkv;
  uint32_t att_off;
};

// A tile of TR rows (16, or 8 when the largest K needs smaller tiles) arrives as two contiguous copies of
// TR/2 rows each, the second placed 64 bytes (mod 128) further on.
__host__ __device__ __forceinline__ uint32_t tile_bytes(int TR, int K, int G) {
  return ((static_cast<uint32_t>(TR) * (K / 2) + 64u + 2u * (2u * TR * G + 16u)) + 127u) & ~127u;
}

// One 128-column group of an 8-row MMA step for this lane: w = its 32 codes (row prow, 16 bytes at qd*16
// in the group), b01/b23 = the activation B fragments, c = {-offset, sum x, ., .} of the group. MMA row R
// carries the row's columns 0-63 in rows 0-7 and 64-127 in rows 8-15; B column 0 carries x for the first
// half and column 1 for the second, so D[r][0] + D[r+8][1] (d[0] + d[3] in lanes with qd = 0) is the row's
// dot product. Lanes 8-31 load duplicates of lanes 0-7's activation fragments: their B columns 2-7 only
// produce D columns that are never read. Returns acc + s * (dot - offset) + m * sum x.
__device__ __forceinline__ float group_dot(const uint4& w4, const uint4& b01, const uint4& b23, const float4& c,
                                           float s, float m, const g4::DequantK& k, const float4& zq,
                                           float acc) {
  const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
  uint32_t a[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t w = wv[j], w8 = __umulhi(wv[j], 1u << 24);  // w >> 8 on the FMA pipe
    a[j][0] = and_or(w, k.m_lo, k.k1024);
    a[j][1] = and_or(w8, k.m_lo, k.k1024);
    a[j][2] = and_or(w, k.m_hi, k.k64);
    a[j][3] = and_or(w8, k.m_hi, k.k64);
  }
  float dot;
  if (kChains == 2) {
    float d0[4], d1[4];
    mma_f16_16816_c(d0, a[0][0], a[0][1], a[0][2], a[0][3], b01.x, b01.y, c);
    mma_f16_16816_c(d1, a[1][0], a[1][1], a[1][2], a[1][3], b01.z, b01.w, zq);
    mma_f16_16816(d0, a[2][0], a[2][1], a[2][2], a[2][3], b23.x, b23.y);
    mma_f16_16816(d1, a[3][0], a[3][1], a[3][2], a[3][3], b23.z, b23.w);
    dot = (d0[0] + d0[3]) + (d1[0] + d1[3]);
  } else {
    float d0[4];
    mma_f16_16816_c(d0, a[0][0], a[0][1], a[0][2], a[0][3], b01.x, b01.y, c);
    mma_f16_16816(d0, a[1][0], a[1][1], a[1][2], a[1][3], b01.z, b01.w);
    mma_f16_16816(d0, a[2][0], a[2][1], a[2][2], a[2][3], b23.x, b23.y);
    mma_f16_16816(d0, a[3][0], a[3][1], a[3][2], a[3][3], b23.z, b23.w);
    dot = d0[0] + d0[3];
  }
  return fmaf(s, dot, fmaf(m, c.y, acc));
}

// Shared-memory addresses of one work item (8 rows x groups [g, g1)), advanced group by group.
struct ItemAddr {
  uint32_t w;  // this lane's 16 code bytes of group g
  uint32_t x;  // activation fragments of group g (b01 at +0, b23 at +128; 256 bytes per group)
  uint32_t c;  // constants of group g (16 bytes per group)
  uint32_t s;  // scale of (row, g); the min is m_off bytes further
};

__device__ __forceinline__ float item_single(ItemAddr& A, uint32_t m_off, const g4::DequantK& k,
                                             const float4& zq, float acc) {
  const uint4 w = lds128_o<0>(A.w);
  const uint4 b01 = lds128_o<0>(A.x), b23 = lds128_o<128>(A.x);
  const float4 c = lds128f_o<0>(A.c);
  const float s = lds_h2f_o<0>(A.s), m = lds_h2f_o<0>(A.s + m_off);
  A.w += 64;
  A.x += 256;
  A.c += 16;
  A.s += 2;
  return group_dot(w, b01, b23, c, s, m, k, zq, acc);
}

// Operands of a pair of groups (g, g+1).
struct PairOps {
  uint32_t s2, m2;
  uint4 w0, w1, x0, y0, x1, y1;
  float4 c0, c1;
};

__device__ __forceinline__ void load_pair(const ItemAddr& A, uint32_t ma, PairOps& o) {
  o.s2 = lds32_o<0>(A.s);
  o.m2 = lds32_o<0>(ma);
  o.w0 = lds128_o<0>(A.w);
  o.w1 = lds128_o<64>(A.w);
  o.x0 = lds128_o<0>(A.x);
  o.y0 = lds128_o<128>(A.x);
  o.x1 = lds128_o<256>(A.x);
  o.y1 = lds128_o<384>(A.x);
  o.c0 = lds128f_o<0>(A.c);
  o.c1 = lds128f_o<16>(A.c);
}

__device__ __forceinline__ void pair_math(const PairOps& o, const g4::DequantK& k, const float4& zq, float& acc0,
                                          float& acc1) {
  const float2 sf = __half22float2(*reinterpret_cast<const __half2*>(&o.s2));
  const float2 mf = __half22float2(*reinterpret_cast<const __half2*>(&o.m2));
  acc0 = group_dot(o.w0, o.x0, o.y0, o.c0, sf.x, mf.x, k, zq, acc0);
  acc1 = group_dot(o.w1, o.x1, o.y1, o.c1, sf.y, mf.y, k, zq, acc1);
}

// Dot products of this lane's row over groups [g0, g1) (scaled, offset-corrected, fp32).
__device__ __forceinline__ float item_dot(ItemAddr A, uint32_t m_off, int G, int g0, int g1,
                                          const g4::DequantK& k, const float4& zq) {
  float acc0 = 0.f, acc1 = 0.f;
  int g = g0;
  if ((G & 1) == 0) {
    // scale/min pairs (g, g+1) are 4-byte aligned for even g: one load each per pair
    if (g & 1) {
      acc1 = item_single(A, m_off, k, zq, acc1);
      ++g;
    }
    uint32_t ma = A.s + m_off;
    for (; g + 1 < g1; g += 2) {
      PairOps o;
      load_pair(A, ma, o);
      A.w += 128;
      A.x += 512;
      A.c += 32;
      A.s += 4;
      ma += 4;
      pair_math(o, k, zq, acc0, acc1);
    }
  }
  for (; g < g1; ++g) acc0 = item_single(A, m_off, k, zq, acc0);
  return acc0 + acc1;
}

// x of every slot -> fp16 B fragments [g][2][8 lanes][16 B] and constants {-offset, sum, 0, 0} per group
// One 8-activation chunk (it = 16 g + 4 qq + j: elements 32 qq + 8 j .. + 7 of group g) of a slot's table:
// fp16 B fragments and, summed over the group's 16 chunks (16 consecutive lanes), the group's constants.
__device__ __forceinline__ void table_chunk(const __half (&h)[8], bool valid, int it, uint8_t* xs, float4* cst) {
  float off = 0.f, sum = 0.f;
  if (valid) {
    const int g = it >> 4, qq = (it >> 2) & 3, j = it & 3;
    uint8_t* tab = xs + static_cast<size_t>((g * 2 + (j >> 1)) * 8) * 16;
    uint32_t* l1 = reinterpret_cast<uint32_t*>(tab + qq * 16) + (j & 1) * 2;
    uint32_t* l2 = reinterpret_cast<uint32_t*>(tab + (4 + qq) * 16) + (j & 1) * 2;
    l1[0] = pack_half2(h[0], h[4]);
    l1[1] = pack_half2(h[1], h[5]);
    l2[0] = pack_half2(h[2], h[6]);
    l2[1] = pack_half2(h[3], h[7]);
    const float ev = __half2float(h[0]) + __half2float(h[2]) + __half2float(h[4]) + __half2float(h[6]);
    const float od = __half2float(h[1]) + __half2float(h[3]) + __half2float(h[5]) + __half2float(h[7]);
    off = 1024.f * ev + 64.f * od;
    sum = ev + od;
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    off += __shfl_xor_sync(0xffffffffu, off, o);
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  if (valid && (it & 15) == 0) cst[it >> 4] = make_float4(-off, sum, 0.f, 0.f);
}

// Tabulate the slots' activations: att_phase 0 every slot except the fused attention's output, 1 only that one.
__device__ void stage_all_x(const MultiParams& p, uint8_t* smem, int tid, int att_phase) {
  for (int sl = 0; sl < p.nslots; ++sl) {
    const Slot& S = p.slots[sl];
    if (S.att != att_phase) continue;
    const int items = S.G * 16;
    uint8_t* xs = smem + S.tab_off;
    float4* cst = reinterpret_cast<float4*>(smem + S.cst_off);
    if (S.ln) {  // the add + LayerNorm prologue (engine/fused.py:29-40) produces this slot's vector
      LnSrc L;
      L.x = S.x;
      L.a = S.a;
      L.b = S.b;
      L.w = S.w;
      L.x_out = S.x_out;
      L.h_out = S.h_out;
      L.eps = S.eps;
      L.K = S.K;
      L.emb_q = S.emb_q;
      L.emb_s = S.emb_s;
      L.tok = S.tok;
      L.vocab = S.vocab;
      L.emb_f16 = S.emb_f16;
      stage_ln<4>(L, p.x_bf16 != 0, reinterpret_cast<float*>(smem + p.ln_off), 2, tid, kConsumerWarps * 32,
                  blockIdx.x == 0, [&](const float (&v)[8], bool valid, int it) {
                    __half h[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(v[i]);
                    table_chunk(h, valid, it, xs, cst);
                  });
      continue;
    }
    for (int base = 0; base < items; base += kConsumerWarps * 32) {
      const int it = base + tid;
      const bool valid = it < items;
      __half h[8];
      if (valid) load8_as_half(static_cast<const uint8_t*>(S.x) + static_cast<int64_t>(it) * 16, p.x_bf16, h);
      table_chunk(h, valid, it, xs, cst);
    }
  }
}

// Producer (lane 0 of the producer warp): streams this CTA's tiles into the ring in order.
template <int TR>
__device__ void multi_produce(const MultiParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                              uint32_t* start) {
  const EntryP* ent = reinterpret_cast<const EntryP*>(smem + p.ent_off);
  const int C = gridDim.x, cta = blockIdx.x;
  const int ntiles = (p.total_tiles - cta + C - 1) / C;
  uint8_t* ring = smem + p.ring_off;
  uint32_t head = 0, tail = 0;  // FIFO ring: outstanding tiles occupy [tail, head) or, wrapped, [tail, end) + [0, head)
  int old = 0;                  // oldest unreclaimed local tile
  int e = 0;
  bool ok = true;
  int j = 0;
  for (; j < ntiles && ok; ++j) {
    const int gt = cta + j * C;
    while (e + 1 < p.count && gt >= ent[e + 1].tile_begin) ++e;
    const EntryP& E = ent[e];
    const uint32_t b = E.tbytes;
    // allocate b bytes, reclaiming the oldest tiles (in order) until the space is free
    uint32_t pos = 0;
    for (;;) {
      const int n_out = j - old;
      if (n_out == 0) {
        head = tail = 0;
      }
      bool fits = false;
      if (n_out < kMaxOutstanding) {
        // strict comparisons: head == tail must only ever mean "empty"
        if (tail <= head) {
          if (head + b <= p.ring_bytes) { pos = head; fits = true; }
          else if (b < tail || n_out == 0) { pos = 0; fits = true; }
        } else if (head + b < tail) {
          pos = head;
          fits = true;
        }
      }
      if (fits) break;
      if (!mbar_wait(&empty[old % kWindow], (old / kWindow) & 1, ERR_MULTI_EMPTY)) { ok = false; break; }
      ++old;
      tail = (j - old > 0) ? start[old % kWindow] : head;
    }
    if (!ok) break;
    start[j % kWindow] = pos;
    head = pos + b;
    const int row0 = (gt - E.tile_begin) * TR;
    const int nr = min(TR, E.N - row0);
    const uint32_t row_bytes = E.row_bytes;
    const uint32_t rs = row_bytes, sblk = E.sblk;
    uint8_t* sb = ring + pos;
    const int64_t sm_total = static_cast<int64_t>(E.N) * E.G * 2;
    const int64_t b0 = static_cast<int64_t>(row0) * E.G * 2;
    const int64_t b1 = b0 + static_cast<int64_t>(nr) * E.G * 2;
    const int64_t a0 = b0 & ~int64_t(15);
    const int64_t want_end = (b1 + 15) & ~int64_t(15);
    const int64_t end = want_end < sm_total ? want_end : sm_total;
    const uint32_t tma = static_cast<uint32_t>((end & ~int64_t(15)) - a0);
    uint8_t* s_dst = sb + TR * rs + 64;
    uint8_t* m_dst = s_dst + sblk;
    if (a0 + tma < end) {
      for (int64_t bb = a0 + tma; bb < end; bb += 2) {
        reinterpret_cast<uint16_t*>(s_dst)[(bb - a0) >> 1] = *reinterpret_cast<const uint16_t*>(E.s + bb);
        reinterpret_cast<uint16_t*>(m_dst)[(bb - a0) >> 1] = *reinterpret_cast<const uint16_t*>(E.m + bb);
      }
      fence_proxy_async_smem();
    }
    uint64_t* fb = &full[j % kWindow];
    mbar_arrive_expect_tx(fb, nr * row_bytes + 2 * tma);  // also publishes start[] (release)
    const uint8_t* qsrc = E.q + static_cast<int64_t>(row0) * row_bytes;
    constexpr int H = TR / 2;
    bulk_g2s(sb, qsrc, min(nr, H) * row_bytes, fb);
    if (nr > H) bulk_g2s(sb + H * rs + 64, qsrc + H * row_bytes, (nr - H) * row_bytes, fb);
    if (tma) {
      bulk_g2s(s_dst, E.s + a0, tma, fb);
      bulk_g2s(m_dst, E.m + a0, tma, fb);
    }
  }
  // no retirement with copies in flight
  for (int t = old; t < j; ++t)
    if (!mbar_wait(&full[t % kWindow], (t / kWindow) & 1, ERR_MULTI_FULL)) break;
}

// Number of this CTA's local tiles j (global tile cta + j * C) that lie below global tile T.
__device__ __forceinline__ int local_tiles_below(int T, int cta, int C) { return T > cta ? (T - cta + C - 1) / C : 0; }

// n / d for 0 <= n < 2^24 and 1 <= d <= 2^8 with mag = ceil(2^32 / d) (exact in that range); d == 1 apart.
__device__ __forceinline__ int fdiv(int n, int d, uint32_t mag) {
  return d == 1 ? n : static_cast<int>(__umulhi(static_cast<uint32_t>(n), mag));
}
__host__ __device__ __forceinline__ uint32_t div_magic(uint32_t d) {
  return d <= 1 ? 0u : static_cast<uint32_t>((0xFFFFFFFFull + d) / d);
}

template <int TR, bool kAtt>  // kAtt: the launch computes the fused decode attention (rb_attn_src)
__global__ void __maxnreg__(kMaxRegs) gemv_int4_multi_kernel(const __grid_constant__ MultiParams p) {
  constexpr int ST = TR / 8, H = TR / 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = gridDim.x, cta = blockIdx.x;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + kWindow;
  uint32_t* start = reinterpret_cast<uint32_t*>(smem + p.start_off);
  if (tid < kWindow) {  // one barrier pair per thread: 256 serial inits would cost a microsecond per launch
    mbar_init(&full[tid], 1);
    mbar_init(&empty[tid], kRelease);
    fence_mbar_init();
  }
  if (tid < 16) reinterpret_cast<uint32_t*>(smem + p.zero_off)[tid] = 0u;
  int* cnt = reinterpret_cast<int*>(smem + p.red_off);  // [kRedSlots][ST]: arrivals of the K-slices of a step
  for (int i = tid; i < kRedSlots * ST; i += kThreads) cnt[i] = 0;
  EntryP* entp = reinterpret_cast<EntryP*>(smem + p.ent_off);
  EntryC* entc = reinterpret_cast<EntryC*>(smem + p.ent_off + p.count * sizeof(EntryP));
  for (int i = tid; i < p.count; i += kThreads) {
    const Entry& E = p.e[i];
    const Slot& S = p.slots[E.slot];
    EntryP a;
    a.q = E.q;
    a.s = reinterpret_cast<const uint8_t*>(E.s);
    a.m = reinterpret_cast<const uint8_t*>(E.m);
    a.N = E.N;
    a.G = E.G;
    a.tile_begin = E.tile_begin;
    a.tbytes = tile_bytes(TR, E.K, E.G);
    a.row_bytes = static_cast<uint32_t>(E.K / 2);
    a.sblk = 2u * TR * E.G + 16u;
    entp[i] = a;
    EntryC c;
    c.y = E.y;
    c.N = E.N;
    c.tile_begin = E.tile_begin;
    c.G = E.G;
    c.rs = E.K / 2;
    c.sblk = a.sblk;
    c.tab_off_x = S.tab_off;
    c.cst_off_x = S.cst_off;
    c.P = min(kMaxP, (E.G + kSliceGroups - 1) / kSliceGroups);
    c.gps = (E.G + c.P - 1) / c.P;
    c.ipt = ST * c.P;
    const int tile_end = i + 1 < p.count ? p.e[i + 1].tile_begin : p.total_tiles;
    c.jlo = local_tiles_below(E.tile_begin, cta, C);
    c.ib = (local_tiles_below(tile_end, cta, C) - c.jlo) * c.ipt;  // this entry's items; prefix-summed below
    c.mag_ipt = div_magic(c.ipt);
    c.mag_p = div_magic(c.P);
    c.epi = E.epi;
    c.ep = E.ep;
    entc[i] = c;
  }
  __syncthreads();
  griddep_launch_dependents();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (!p.prefetch) griddep_wait();
      multi_produce<TR>(p, smem, full, empty, start);
    }
    return;
  }

  if (warp == 0) {
    // exclusive prefix sum of the item counts over the entries (and the total into the extra entry)
    int carry = 0;
    for (int base = 0; base <= p.count; base += 32) {
      const int i = base + lane;
      const int v = i < p.count ? entc[i].ib : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (i <= p.count) entc[i].ib = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  griddep_wait();
  stage_all_x(p, smem, tid, 0);
  named_bar_sync(1, kConsumerWarps * 32);
  if (kAtt && warp < attn::kWarps && cta < p.att_ctas) {
    // the fused decode attention: this CTA's (key-value head, split) with warps 0-3, while warps 4.. start
    // streaming the entries that do not need it
    float* sa = reinterpret_cast<float*>(smem + p.att_off);
    int* last = reinterpret_cast<int*>(sa + attn::kWarps * 4 * (2 + attn::kHd));
    const int g = cta / p.att.nsplit, sp = cta - g * p.att.nsplit;
    switch (p.att_rep) {
#define RB_ATT_CASE(R)                                                                                          \
  case R:                                                                                                       \
    attn::attn_cta<R, true>(p.att, g, sp, tid, 3, reinterpret_cast<float(*)[R]>(sa),                            \
                            reinterpret_cast<float(*)[R]>(sa + attn::kWarps * R),                               \
                            reinterpret_cast<float(*)[R][attn::kHd]>(sa + 2 * attn::kWarps * R), last);         \
    break;
      RB_ATT_CASE(1)
      RB_ATT_CASE(2)
      RB_ATT_CASE(3)
      RB_ATT_CASE(4)
#undef RB_ATT_CASE
      default:
        break;
    }
  }

  const int r = lane >> 2, qd = lane & 3;
  const int prow0 = (r & 1) * H + (r >> 1);  // tile row of this lane's MMA row in step 0 (step t: + 4t)
  const uint32_t zero_a = smem_u32(smem + p.zero_off);
  const float4 zq = lds128f_a(zero_a);
  const g4::DequantK dk = {p.m_lo, p.m_hi, p.k1024, p.k64};
  const uint8_t* ring = smem + p.ring_off;
  float* red = reinterpret_cast<float*>(cnt + kRedSlots * ST);  // [kRedSlots][ST][maxp][8] slice partials
  const int total_items = entc[p.count].ib;
  bool dead = false;
  // CTA-local work items in order (tile by tile, item it = step * P + slice within a tile); warp w takes
  // items w, w + kConsumerWarps, ...; the entry of an item is found by scanning forward (items only grow)
  int e = -1, next_ib = 0;
  // items of the entries that read the fused attention's output come last: they start once every CTA has seen
  // all key-value heads complete and has tabulated that output
  const int n_pre = kAtt ? entc[p.att_entry].ib : total_items;
  // in the CTAs that compute attention, warps 0-3 (the attention warps) leave the entries that do not need it
  // to warps 4.. and go straight to the wait
  const bool att_cta = kAtt && cta < p.att_ctas;
  const int w0 = att_cta ? attn::kWarps : 0, nw0 = kConsumerWarps - w0;
  int I = warp >= w0 ? warp - w0 : n_pre;
  int stride = nw0;
  for (int phase = 0; phase < 2; ++phase) {
    if (phase == 1) {
      if (!kAtt) break;
      if (tid == 0) {
        const int64_t pos = *p.att.pos;
        if (pos >= 0 && pos < p.att.S) {  // otherwise no head completes (the attention reported ERR_ARG)
          const unsigned long long t0 = globaltimer_ns(), lim = wait_limit_ns();
          unsigned int done = 0;
          for (;;) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(done) : "l"(p.att.heads_done) : "memory");
            // signed: a counter the caller left below zero (a workspace not zeroed) never completes, and the
            // wait runs out instead of passing at once
            if (static_cast<int>(done) >= p.att_nkv) break;
            if (globaltimer_ns() - t0 > lim) {
              atomicOr(&g_device_error, ERR_ATT_WAIT);
              break;
            }
            __nanosleep(64);
          }
        }
        // the launch's last CTA past this point resets the counters for the next launch (which starts after
        // this one has completed)
        unsigned int* passed = p.att.heads_done + 1;
        if (atomicAdd(passed, 1u) == gridDim.x - 1) {
          *p.att.heads_done = 0u;
          *passed = 0u;
        }
      }
      named_bar_sync(1, kConsumerWarps * 32);
      stage_all_x(p, smem, tid, 1);
      named_bar_sync(1, kConsumerWarps * 32);
      I = n_pre + warp;
      stride = kConsumerWarps;
    }
    const int i_end = phase == 0 ? n_pre : total_items;
  for (; I < i_end; I += stride) {
    while (I >= next_ib) {
      ++e;
      next_ib = entc[e + 1].ib;
    }
    const EntryC E = entc[e];  // re-read per item (four 16-byte loads): cheaper than holding it in registers
    const int local = I - E.ib;
    const int jj = fdiv(local, E.ipt, E.mag_ipt);
    const int it = local - jj * E.ipt;
    const int t = fdiv(it, E.P, E.mag_p);
    const int sl = it - t * E.P;
    const int j = E.jlo + jj;
    const int gt = cta + j * C;
    const int slot = j % kRedSlots;
    if (!dead && !mbar_wait(&full[j % kWindow], (j / kWindow) & 1, ERR_MULTI_FULL)) dead = true;
    if (dead) continue;
    const int row0 = (gt - E.tile_begin) * TR;
    const uint8_t* sq = ring + start[j % kWindow];
    const int rs = E.rs, G = E.G;
    const int g0 = sl * E.gps, g1 = min(G, g0 + E.gps);
    ItemAddr A;
    A.w = smem_u32(sq + (r & 1) * (H * rs + 64) + ((r >> 1) + 4 * t) * rs + qd * 16) + g0 * 64;
    A.s = smem_u32(sq + TR * rs + 64) + ((prow0 + 4 * t) * G + g0) * 2;
    A.x = smem_u32(smem + E.tab_off_x) + (lane & 7) * 16 + g0 * 256;
    A.c = smem_u32(smem + E.cst_off_x) + g0 * 16;
    const float v = item_dot(A, E.sblk, G, g0, g1, dk, zq);
    const int row = row0 + prow0 + 4 * t;
    float out = v;
    bool store = E.P == 1;
    if (E.P > 1) {
      // K-sliced: the last slice of this step to finish adds the P partials in slice order (deterministic)
      float* rp = red + ((slot * ST + t) * p.maxp) * 8;
      if (qd == 0) rp[sl * 8 + r] = v;
      __syncwarp();
      int prior = 0;
      if (lane == 0) {
        __threadfence_block();
        prior = atomicAdd(&cnt[slot * ST + t], 1);
      }
      prior = __shfl_sync(0xffffffffu, prior, 0);
      if (prior == E.P - 1) {
        __threadfence_block();
        if (qd == 0) {
          out = 0.f;
          for (int k = 0; k < E.P; ++k) out += rp[k * 8 + r];
        }
        if (lane == 0) cnt[slot * ST + t] = 0;
        store = true;
      }
    }
    __syncwarp();
    // every item releases its share of the tile's ring space (the tile's reduction slot is reused only after
    // the whole tile is reclaimed). The arrive has release semantics: it waits until this thread's earlier
    // memory operations are performed, so the global store of y comes after it.
    if (lane == 0) mbar_arrive_cnt(&empty[j % kWindow], it == E.ipt - 1 ? kRelease - (E.ipt - 1) : 1);
    if (E.epi == RB_EPI_STORE) {
      if (store && qd == 0 && row < E.N) store_out(E.y, row, out, p.y_bf16);
    } else if (store) {  // routed as the engine's post kernel would (engine/fused.py:43-84); store is warp-uniform
      const EpiP& P = p.epis[E.ep];
      const float rr = round_act(out, p.y_bf16);             // what the engine's y buffer would hold
      const float pr = __shfl_xor_sync(0xffffffffu, rr, 8);  // row ^ 1 is MMA row r ^ 2: lane ^ 8
      int64_t pos = 0;
      bool pos_ok = true;
      if (E.epi == RB_EPI_ROPE_KV) {
        pos = *P.pos;
        pos_ok = pos >= 0 && pos < P.S;
        if (!pos_ok && lane == 0) atomicOr(&g_device_error, ERR_ARG);
      }
      if (qd == 0 && row < E.N) {
        if (E.y) store_out(E.y, row, out, p.y_bf16);
        if (pos_ok) route_row(P, E.epi, row, rr, pr, pos, p.y_bf16);
      }
    }
  }
  }
}

}  // namespace g4m

int launch_gemv_int4_multi(const rb_gemv_desc* d, int count, int x_dtype, int y_dtype, int flags, int num_sms,
                           cudaStream_t stream, const rb_gemv_epi* epi, const rb_add_ln* ln, const rb_attn_src* attn) {
  using namespace g4m;
  constexpr uint32_t kSmemMax = 227 * 1024;
  // shared memory of the fused attention's CTA merge: max, sum and 128 outputs per warp and head (rep <= 4)
  const uint32_t att_bytes = attn ? attn::kWarps * 4 * (2 + attn::kHd) * 4 + 16 : 0u;
  // 16-row tiles halve the per-tile producer work; lists with a K too large for two 16-row tiles (plus
  // the activation tables) in shared memory use 8-row tiles
  int64_t kmax = 0;
  for (int i = 0; i < count; ++i) {
    // 8-bit double-quantised scales, int8 entries: the tcgen05 kernel only
    if (d[i].s_row || d[i].w8 != RB_W8_NONE) return RB_ERR_SHAPE;
    kmax = std::max(kmax, d[i].K);
  }
  const int TR = (2u * tile_bytes(16, static_cast<int>(kmax), static_cast<int>(kmax / 128)) +
                  static_cast<uint32_t>(kmax / 128) * 272u + 48u * 1024u <= kSmemMax) ? 16 : 8;
  int done = 0;
  while (done < count) {
    const int n = std::min(count - done, kMaxEntries);
    MultiParams p;  // ~15 KB, built on the host and passed by value in the launch
    p.count = n;
    p.x_bf16 = x_dtype == RB_BF16;
    p.y_bf16 = y_dtype == RB_BF16;
    p.prefetch = (flags & RB_FLAG_PDL) && (flags & RB_FLAG_PREFETCH_WEIGHTS) ? 1 : 0;
    p.m_lo = 0x000F000Fu;
    p.m_hi = 0x00F000F0u;
    p.k1024 = 0x64006400u;
    p.k64 = 0x54005400u;
    // distinct activation vectors -> slots; stop adding entries when the next one would not fit
    // (activation tables + two of the largest tiles must fit in shared memory)
    constexpr uint32_t kFixed = 64 + 16 + 2 * kLnMaxGroups * 4 + kMaxEntries * (sizeof(EntryP) + sizeof(EntryC)) + sizeof(EntryC) +
                                kWindow * 4 + 16 + kRedSlots * 2 * 4 + kRedSlots * 2 * kMaxP * 8 * 4 +
                                2 * kWindow * 8 + 128;
    int nslots = 0, tiles = 0, nepis = 0;
    uint32_t x_bytes = 0, max_tile = 0;
    int take = 0;
    for (; take < n; ++take) {
      const rb_gemv_desc& D = d[done + take];
      const uint32_t G = static_cast<uint32_t>(D.K / 128);
      const uint32_t tb = tile_bytes(TR, static_cast<int>(D.K), static_cast<int>(G));
      const bool from_ln = D.x == nullptr;  // multiplies the prologue's normalised vector
      const int kind = epi ? epi[done + take].kind : RB_EPI_STORE;
      if (from_ln && !ln) return RB_ERR_NULL;
      int slot = -1;
      for (int i = 0; i < nslots; ++i)
        if (p.slots[i].ln == (from_ln ? 1 : 0) && (from_ln || p.slots[i].x == D.x) &&
            p.slots[i].K == static_cast<int>(D.K))
          slot = i;
      const uint32_t add_x = slot < 0 ? G * (256u + 16u) : 0u;
      if (slot < 0 && nslots == kMaxSlots) break;
      if (x_bytes + add_x + kFixed + att_bytes + 2u * std::max(max_tile, tb) > kSmemMax) break;
      if (kind != RB_EPI_STORE && nepis == 4) break;
      if (slot < 0) {
        slot = nslots++;
        Slot& S = p.slots[slot];
        S = Slot{};
        S.x = from_ln ? ln->x : D.x;
        S.att = attn && !from_ln && D.x == attn->out ? 1 : 0;
        if (from_ln) {
          S.ln = 1;
          S.a = ln->a;
          S.b = ln->b;
          S.w = ln->w;
          S.x_out = ln->x_out;
          S.h_out = ln->h_out;
          S.eps = ln->eps;
          S.emb_q = ln->emb_q;
          S.emb_s = ln->emb_s;
          S.tok = ln->tok;
          S.vocab = ln->vocab;
          S.emb_f16 = ln->emb_s_dtype == RB_F16;
        }
        S.K = static_cast<int>(D.K);
        S.G = static_cast<int>(G);
        x_bytes += add_x;
      }
      Entry& E = p.e[take];
      E.q = D.q;
      E.s = D.s;
      E.m = D.m;
      E.y = D.y;
      E.N = static_cast<int>(D.N);
      E.K = static_cast<int>(D.K);
      E.G = static_cast<int>(G);
      E.slot = slot;
      E.tile_begin = tiles;
      E.epi = kind;
      E.ep = 0;
      if (kind != RB_EPI_STORE) {
        const rb_gemv_epi& X = epi[done + take];
        EpiP& P = p.epis[nepis];
        P.pos = X.pos;
        P.cos = X.cos;
        P.sin = X.sin;
        P.q_out = X.q_out;
        P.k_cache = X.k_cache;
        P.v_cache = X.v_cache;
        P.act = X.act_out;
        P.S = X.cache_len;
        P.rope = X.rope;
        P.nq = X.n_q_heads;
        P.nkv = X.n_kv_heads;
        P.hd = X.head_dim;
        E.ep = nepis++;
      }
      tiles += static_cast<int>((D.N + TR - 1) / TR);
      max_tile = std::max(max_tile, tb);
    }
    if (take == 0) return RB_ERR_SHAPE;
    if ((epi || ln || attn) && take < count) return RB_ERR_SHAPE;  // the fused glue needs one launch
    p.count = take;
    p.nslots = nslots;
    p.total_tiles = tiles;
    p.att_on = 0;
    p.att_ctas = p.att_rep = p.att_entry = p.att_nkv = 0;
    if (attn) {
      // entries reading the attention output must be the last ones (their items run after the wait)
      int first = -1;
      for (int i = 0; i < take; ++i) {
        const bool a = p.slots[p.e[i].slot].att != 0;
        if (a && first < 0) first = i;
        if (!a && first >= 0) return RB_ERR_SHAPE;
      }
      const int grid = std::min(num_sms, std::max(1, tiles));
      const int nkv = attn->n_kv_heads;
      const int nsplit = std::min(static_cast<int>(attn::nsplit_for(nkv, num_sms)), grid / nkv);
      if (first < 0 || nsplit < 1) return RB_ERR_SHAPE;
      attn::AttnParams& A = p.att;
      uint8_t* w = static_cast<uint8_t*>(attn->ws);
      A.q = attn->q;
      A.kc = attn->k_cache;
      A.vc = attn->v_cache;
      A.pos = attn->pos;
      A.out = attn->out;
      A.ticket = reinterpret_cast<unsigned int*>(w);
      A.heads_done = reinterpret_cast<unsigned int*>(w + attn::kHeadsDoneOff);  // the passed counter follows
      A.po = reinterpret_cast<float*>(w + attn::kTicketBytes);
      A.pm = A.po + static_cast<int64_t>(attn->n_q_heads) * nsplit * attn::kHd;
      A.pl = A.pm + static_cast<int64_t>(attn->n_q_heads) * nsplit;
      A.S = attn->cache_len;
      A.scale = attn->scale;
      A.nsplit = nsplit;
      A.bf16 = x_dtype == RB_BF16;
      p.att_on = 1;
      p.att_ctas = nkv * nsplit;
      p.att_rep = attn->n_q_heads / nkv;
      p.att_entry = first;
      p.att_nkv = nkv;
    }
    p.maxp = 1;
    for (int i = 0; i < take; ++i)
      p.maxp = std::max(p.maxp, std::min(kMaxP, (p.e[i].G + kSliceGroups - 1) / kSliceGroups));
    // layout: [x tables + constants][zero][start offsets][barriers][ring]
    uint32_t off = 0;
    for (int i = 0; i < nslots; ++i) {
      p.slots[i].tab_off = off;
      off += static_cast<uint32_t>(p.slots[i].G) * 256u;
      p.slots[i].cst_off = off;
      off += static_cast<uint32_t>(p.slots[i].G) * 16u;
    }
    p.zero_off = off;
    off += 64;
    p.ln_off = off;  // the prologue's group sums (2 x kLnMaxGroups floats)
    off += 2 * kLnMaxGroups * 4;
    off = (off + 15) & ~15u;
    p.att_off = off;
    off += att_bytes;
    p.ent_off = off;
    off += static_cast<uint32_t>(take) * sizeof(EntryP) + static_cast<uint32_t>(take + 1) * sizeof(EntryC);
    p.start_off = off;
    off += kWindow * 4;
    off = (off + 15) & ~15u;
    p.red_off = off;
    off += kRedSlots * 2 * 4 + (p.maxp > 1 ? kRedSlots * 2 * p.maxp * 8 * 4 : 0);
    off = (off + 7) & ~7u;
    p.bar_off = off;
    off += 2 * kWindow * 8;
    off = (off + 127) & ~127u;
    p.ring_off = off;
    if (off + 2 * max_tile > kSmemMax) return RB_ERR_SHAPE;
    p.ring_bytes = kSmemMax - off;
    void (*kern)(MultiParams) = p.att_on ? (TR == 16 ? gemv_int4_multi_kernel<16, true> : gemv_int4_multi_kernel<8, true>)
                                         : (TR == 16 ? gemv_int4_multi_kernel<16, false> : gemv_int4_multi_kernel<8, false>);
    cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), kSmemMax);
    if (e != cudaSuccess) return RB_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(num_sms, std::max(1, tiles)));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemMax;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (flags & RB_FLAG_PDL) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return RB_ERR_LAUNCH;
    done += take;
  }
  return RB_OK;
}

}  // namespace rb
