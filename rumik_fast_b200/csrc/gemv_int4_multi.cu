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
#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace g4m {

constexpr int kConsumerWarps = 16;  // work items need ~80 registers: 16 warps fit without spills
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxEntries = 256;
constexpr int kMaxSlots = 8;
constexpr int kWindow = 128;       // barrier window (tiles)
constexpr int kRedSlots = 32;      // reduction slots (tiles), > kMaxOutstanding
constexpr int kMaxP = 8;           // K-slices per step at most
constexpr int kSliceGroups = 24;   // groups per work item at most (~12 KB of codes for 8 rows)
constexpr int kMaxOutstanding = 24;  // tiles in flight per CTA (window >= this + consumer warps)

struct Entry {
  const uint8_t* q;
  const uint16_t* s;
  const uint16_t* m;
  void* y;
  int N, K, G, slot, tile_begin, pad;
};

struct Slot {
  const void* x;
  int K, G;
  uint32_t tab_off, cst_off;
};

// Entry as kept in shared memory for the whole launch (per-tile lookups must not go to the parameter
// block: it is indexed dynamically, and its misses in the constant cache stalled the producer).
struct __align__(16) EntryS {
  const uint8_t* q;
  const uint8_t* s;
  const uint8_t* m;
  void* y;
  int N, K, G, tile_begin;
  uint32_t tbytes, row_bytes, sblk, tab_off_x;  // tile bytes in the ring; x table offset of its slot
  uint32_t cst_off_x;
  int P, gps, ipt;  // K-slices per 8-row step, groups per slice, work items per tile (= steps * P)
};

struct MultiParams {
  int count, nslots, total_tiles, x_bf16, y_bf16, prefetch;
  uint32_t ring_bytes, ring_off, bar_off, start_off, zero_off, ent_off, red_off;
  uint32_t m_lo, m_hi, k1024, k64;
  Slot slots[kMaxSlots];
  Entry e[kMaxEntries];
};

// A tile of TR rows (16, or 8 when the largest K needs smaller tiles) arrives as two contiguous copies of
// TR/2 rows each, the second placed 64 bytes (mod 128) further on.
__host__ __device__ __forceinline__ uint32_t tile_bytes(int TR, int K, int G) {
  return ((static_cast<uint32_t>(TR) * (K / 2) + 64u + 2u * (2u * TR * G + 16u)) + 127u) & ~127u;
}

// Operands of one 128-column group for the TR/8 eight-row MMA steps of a tile. MMA row R of step t carries
// tile row (R & 1) * TR/2 + t * 4 + R / 2, so the two rows a warp reads in one shared-memory phase come from
// the two copies (64 bytes apart modulo 128) and hit disjoint banks.
template <int ST>
struct Ops16 {
  uint4 w[ST];
  float s[ST], m[ST];
  uint4 b01, b23;
  float4 c;
};

// Scales and mins of a pair of groups (g, g+1) for every step, loaded as half2: with 16-row tiles the
// scale block of a tile starts 16-byte aligned, so for even G the pair is 4-byte aligned. Halves the
// scale/min load instructions (and their bank conflicts: rows of one step share banks when G*2 is a
// multiple of 128 bytes).
template <int ST>
struct SM2 {
  uint32_t s[ST], m[ST];
};

template <int ST>
__device__ __forceinline__ void load_sm2(uint32_t a_s, uint32_t s_step, uint32_t m_off, SM2<ST>& o) {
#pragma unroll
  for (int t = 0; t < ST; ++t) {
    o.s[t] = lds32_a(a_s + t * s_step);
    o.m[t] = lds32_a(a_s + m_off + t * s_step);
  }
}

template <int ST>
__device__ __forceinline__ void split_sm2(const SM2<ST>& v, Ops16<ST>& o0, Ops16<ST>& o1) {
#pragma unroll
  for (int t = 0; t < ST; ++t) {
    const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(&v.s[t]));
    const float2 m2 = __half22float2(*reinterpret_cast<const __half2*>(&v.m[t]));
    o0.s[t] = s2.x;
    o1.s[t] = s2.y;
    o0.m[t] = m2.x;
    o1.m[t] = m2.y;
  }
}

struct Addr16 {
  uint32_t w, s, x, c;   // step-0 code bytes, step-0 scale, activation fragments, constants
  uint32_t xon, con;
};

template <int ST>
__device__ __forceinline__ void load16(const Addr16& a, uint32_t w_step, uint32_t s_step, uint32_t m_off,
                                       uint32_t xhalf, Ops16<ST>& o) {
#pragma unroll
  for (int t = 0; t < ST; ++t) {
    o.w[t] = lds128_a(a.w + t * w_step);
    o.s[t] = lds_h2f_a(a.s + t * s_step);
    o.m[t] = lds_h2f_a(a.s + m_off + t * s_step);
  }
  o.b01 = lds128_pa(a.x, a.xon);
  o.b23 = lds128_pa(a.x + xhalf, a.xon);
  o.c = lds128f_pa(a.c, a.con);
}

// Codes, activation fragments and constants of one group (scales and mins come from load_sm2).
template <int ST>
__device__ __forceinline__ void load16w(const Addr16& a, uint32_t w_step, uint32_t xhalf, Ops16<ST>& o) {
#pragma unroll
  for (int t = 0; t < ST; ++t) o.w[t] = lds128_a(a.w + t * w_step);
  o.b01 = lds128_pa(a.x, a.xon);
  o.b23 = lds128_pa(a.x + xhalf, a.xon);
  o.c = lds128f_pa(a.c, a.con);
}

template <int ST>
__device__ __forceinline__ void math16(const Ops16<ST>& o, const float4& zq, const g4::DequantK& k,
                                       float (&acc)[ST]) {
#pragma unroll
  for (int t = 0; t < ST; ++t) {
    const uint32_t wv[4] = {o.w[t].x, o.w[t].y, o.w[t].z, o.w[t].w};
    uint32_t a[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w = wv[j], w8 = __umulhi(wv[j], 1u << 24);  // w >> 8 on the FMA pipe
      a[j][0] = and_or(w, k.m_lo, k.k1024);
      a[j][1] = and_or(w8, k.m_lo, k.k1024);
      a[j][2] = and_or(w, k.m_hi, k.k64);
      a[j][3] = and_or(w8, k.m_hi, k.k64);
    }
    float d0[4], d1[4];
    mma_f16_16816_c(d0, a[0][0], a[0][1], a[0][2], a[0][3], o.b01.x, o.b01.y, o.c);
    mma_f16_16816_c(d1, a[1][0], a[1][1], a[1][2], a[1][3], o.b01.z, o.b01.w, zq);
    mma_f16_16816(d0, a[2][0], a[2][1], a[2][2], a[2][3], o.b23.x, o.b23.y);
    mma_f16_16816(d1, a[3][0], a[3][1], a[3][2], a[3][3], o.b23.z, o.b23.w);
    const float dot = (d0[0] + d0[3]) + (d1[0] + d1[3]);
    acc[t] = fmaf(o.s[t], dot, fmaf(o.m[t], o.c.y, acc[t]));
  }
}

// x of every slot -> fp16 B fragments [g][2][8 lanes][16 B] and constants {-offset, sum, 0, 0} per group
__device__ void stage_all_x(const MultiParams& p, uint8_t* smem, int tid) {
  for (int sl = 0; sl < p.nslots; ++sl) {
    const Slot& S = p.slots[sl];
    const int items = S.G * 16;
    uint8_t* xs = smem + S.tab_off;
    float4* cst = reinterpret_cast<float4*>(smem + S.cst_off);
    for (int base = 0; base < items; base += kConsumerWarps * 32) {
      const int it = base + tid;
      const bool valid = it < items;
      float off = 0.f, sum = 0.f;
      if (valid) {
        const int g = it >> 4, qq = (it >> 2) & 3, j = it & 3;
        __half h[8];
        load8_as_half(static_cast<const uint8_t*>(S.x) + (static_cast<int64_t>(g) * 128 + 32 * qq + 8 * j) * 2,
                      p.x_bf16, h);
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
  }
}

template <int TR>
__device__ void multi_produce(const MultiParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                              uint32_t* start) {
  const EntryS* ent = reinterpret_cast<const EntryS*>(smem + p.ent_off);
  const int C = gridDim.x, cta = blockIdx.x;
  const int ntiles = (p.total_tiles - cta + C - 1) / C;
  uint8_t* ring = smem + p.ring_off;
  uint32_t head = 0, tail = 0;  // FIFO ring: outstanding tiles occupy [tail, head) or, wrapped, [tail, end) + [0, head)
  int old = 0;                  // oldest unreleased local tile
  int e = 0;
  bool ok = true;
  int j = 0;
  for (; j < ntiles && ok; ++j) {
    const int gt = cta + j * C;
    while (e + 1 < p.count && gt >= ent[e + 1].tile_begin) ++e;
    const EntryS& E = ent[e];
    const uint32_t b = E.tbytes;
    // allocate b bytes, releasing the oldest tiles (in order) until the space is free
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
  for (int t = old; t < j; ++t) mbar_wait(&full[t % kWindow], (t / kWindow) & 1, ERR_MULTI_FULL);
}

template <int TR>
__global__ void __launch_bounds__(kThreads, 1) gemv_int4_multi_kernel(const __grid_constant__ MultiParams p) {
  constexpr int ST = TR / 8, H = TR / 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + kWindow;
  uint32_t* start = reinterpret_cast<uint32_t*>(smem + p.start_off);
  if (tid == 0) {
    for (int i = 0; i < kWindow; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
  }
  if (tid < 16) reinterpret_cast<uint32_t*>(smem + p.zero_off)[tid] = 0u;
  int* cnt = reinterpret_cast<int*>(smem + p.red_off);  // [kRedSlots][ST + 1]: per-step and per-tile counters
  for (int i = tid; i < kRedSlots * (ST + 1); i += kThreads) cnt[i] = 0;
  EntryS* ent = reinterpret_cast<EntryS*>(smem + p.ent_off);
  for (int i = tid; i < p.count; i += kThreads) {
    const Entry& E = p.e[i];
    const Slot& S = p.slots[E.slot];
    EntryS v;
    v.q = E.q;
    v.s = reinterpret_cast<const uint8_t*>(E.s);
    v.m = reinterpret_cast<const uint8_t*>(E.m);
    v.y = E.y;
    v.N = E.N;
    v.K = E.K;
    v.G = E.G;
    v.tile_begin = E.tile_begin;
    v.tbytes = tile_bytes(TR, E.K, E.G);
    v.row_bytes = static_cast<uint32_t>(E.K / 2);
    v.sblk = 2u * TR * E.G + 16u;
    v.tab_off_x = S.tab_off;
    v.cst_off_x = S.cst_off;
    v.P = min(kMaxP, (E.G + kSliceGroups - 1) / kSliceGroups);
    v.gps = (E.G + v.P - 1) / v.P;
    v.ipt = ST * v.P;
    ent[i] = v;
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

  griddep_wait();
  stage_all_x(p, smem, tid);
  named_bar_sync(1, kConsumerWarps * 32);

  const int C = gridDim.x, cta = blockIdx.x;
  const int ntiles = (p.total_tiles - cta + C - 1) / C;
  const int r = lane >> 2, qd = lane & 3;
  const int prow0 = (r & 1) * H + (r >> 1);  // tile row of this lane's MMA row in step 0 (step t: + 4t)
  const uint32_t zero_a = smem_u32(smem + p.zero_off);
  const float4 zq = lds128f_a(zero_a);
  const g4::DequantK dk = {p.m_lo, p.m_hi, p.k1024, p.k64};
  const bool xl = lane < 8;   // batch 1: lanes 0-7 carry the activation columns
  const bool cl = qd == 0;
  const uint32_t xhalf = xl ? 8u * 16u : 0u;
  const uint32_t xstep = xl ? 2u * 8u * 16u : 0u;
  const uint32_t cstep = cl ? 16u : 0u;
  const uint8_t* ring = smem + p.ring_off;
  float* red = reinterpret_cast<float*>(cnt + kRedSlots * (ST + 1));  // [kRedSlots][ST][kMaxP][8]
  bool dead = false;
  // work items of this CTA, in order: tile j, item it = step * P + slice; warp w takes items w, w + 8, ...
  int e = 0, j = 0, it = warp;
  auto entry_of = [&](int jj) -> const EntryS& {
    const int gt = cta + jj * C;
    while (e + 1 < p.count && gt >= ent[e + 1].tile_begin) ++e;
    return ent[e];
  };
  while (j < ntiles && it >= entry_of(j).ipt) { it -= entry_of(j).ipt; ++j; }
  while (j < ntiles) {
    const EntryS& E = entry_of(j);
    const int gt = cta + j * C;
    const int P = E.P, t = it / P, sl = it - t * P;
    const int slot = j % kRedSlots;
    if (!dead && !mbar_wait(&full[j % kWindow], (j / kWindow) & 1, ERR_MULTI_FULL)) dead = true;
    float acc0[1] = {0.f}, acc1[1] = {0.f};
    const int row0 = (gt - E.tile_begin) * TR;
    if (!dead) {
      const uint8_t* sq = ring + start[j % kWindow];
      const int rs = E.K / 2, G = E.G;
      const int g0 = sl * E.gps, g1 = min(G, g0 + E.gps);
      const int shift = static_cast<int>((static_cast<int64_t>(row0) * G * 2) & 15) >> 1;
      Addr16 A;
      A.w = smem_u32(sq + (r & 1) * (H * rs + 64) + ((r >> 1) + 4 * t) * rs + qd * 16) + g0 * 64;
      A.s = smem_u32(sq + TR * rs + 64) + (shift + (prow0 + 4 * t) * G + g0) * 2;
      A.x = (xl ? smem_u32(smem + E.tab_off_x) + lane * 16 : zero_a) + g0 * xstep;
      A.c = (cl ? smem_u32(smem + E.cst_off_x) : zero_a) + g0 * cstep;
      A.xon = xl;
      A.con = cl;
      const uint32_t m_off = E.sblk;
      int g = g0;
      if (((G | g0) & 1) == 0 && TR == 16) {  // scale/min pairs 4-byte aligned: one half2 load per pair
        for (; g + 1 < g1; g += 2) {
          Ops16<1> o0, o1;
          SM2<1> sm2;
          load_sm2<1>(A.s, 0u, m_off, sm2);
          load16w<1>(A, 0u, xhalf, o0);
          A.w += 64; A.x += xstep; A.c += cstep;
          load16w<1>(A, 0u, xhalf, o1);
          A.w += 64; A.s += 4; A.x += xstep; A.c += cstep;
          split_sm2<1>(sm2, o0, o1);
          math16<1>(o0, zq, dk, acc0);
          math16<1>(o1, zq, dk, acc1);
        }
      }
      for (; g + 1 < g1; g += 2) {
        Ops16<1> o0, o1;
        load16<1>(A, 0u, 0u, m_off, xhalf, o0);
        A.w += 64; A.s += 2; A.x += xstep; A.c += cstep;
        load16<1>(A, 0u, 0u, m_off, xhalf, o1);
        A.w += 64; A.s += 2; A.x += xstep; A.c += cstep;
        math16<1>(o0, zq, dk, acc0);
        math16<1>(o1, zq, dk, acc1);
      }
      if (g < g1) {
        Ops16<1> o0;
        load16<1>(A, 0u, 0u, m_off, xhalf, o0);
        math16<1>(o0, zq, dk, acc0);
      }
      const int row = row0 + prow0 + 4 * t;
      const float v = acc0[0] + acc1[0];
      if (P == 1) {
        if (qd == 0 && row < E.N) store_out(E.y, row, v, p.y_bf16);
      } else {
        // K-sliced: the last slice of this step to finish adds the P partials in slice order
        float* rp = red + ((slot * ST + t) * kMaxP) * 8;
        if (qd == 0) rp[sl * 8 + r] = v;
        __syncwarp();
        int old = 0;
        if (lane == 0) {
          __threadfence_block();
          old = atomicAdd(&cnt[slot * (ST + 1) + t], 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == P - 1) {
          __threadfence_block();
          if (qd == 0) {
            float sum = 0.f;
            for (int k = 0; k < P; ++k) sum += rp[k * 8 + r];
            if (row < E.N) store_out(E.y, row, sum, p.y_bf16);
          }
          if (lane == 0) cnt[slot * (ST + 1) + t] = 0;
        }
      }
      // the last item of the tile releases its ring space (and its reduction slot)
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        const int done_items = atomicAdd(&cnt[slot * (ST + 1) + ST], 1);
        if (done_items == E.ipt - 1) {
          cnt[slot * (ST + 1) + ST] = 0;
          mbar_arrive(&empty[j % kWindow]);
        }
      }
    }
    it += kConsumerWarps;
    while (j < ntiles && it >= entry_of(j).ipt) { it -= entry_of(j).ipt; ++j; }
  }
}

}  // namespace g4m

int launch_gemv_int4_multi(const rb_gemv_desc* d, int count, int x_dtype, int y_dtype, int flags, int num_sms,
                           cudaStream_t stream) {
  using namespace g4m;
  constexpr uint32_t kSmemMax = 227 * 1024;
  // 16-row tiles halve the per-tile producer work; lists with a K too large for two 16-row tiles (plus
  // the activation tables) in shared memory use 8-row tiles
  int64_t kmax = 0;
  for (int i = 0; i < count; ++i) kmax = std::max(kmax, d[i].K);
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
    constexpr uint32_t kFixed = 64 + 16 + kMaxEntries * sizeof(EntryS) + kWindow * 4 + 16 +
                                kRedSlots * 3 * 4 + kRedSlots * 2 * kMaxP * 8 * 4 + 2 * kWindow * 8 + 128;
    int nslots = 0, tiles = 0;
    uint32_t x_bytes = 0, max_tile = 0;
    int take = 0;
    for (; take < n; ++take) {
      const rb_gemv_desc& D = d[done + take];
      const uint32_t G = static_cast<uint32_t>(D.K / 128);
      const uint32_t tb = tile_bytes(TR, static_cast<int>(D.K), static_cast<int>(G));
      int slot = -1;
      for (int i = 0; i < nslots; ++i)
        if (p.slots[i].x == D.x && p.slots[i].K == static_cast<int>(D.K)) slot = i;
      const uint32_t add_x = slot < 0 ? G * (256u + 16u) : 0u;
      if (slot < 0 && nslots == kMaxSlots) break;
      if (x_bytes + add_x + kFixed + 2u * std::max(max_tile, tb) > kSmemMax) break;
      if (slot < 0) {
        slot = nslots++;
        p.slots[slot].x = D.x;
        p.slots[slot].K = static_cast<int>(D.K);
        p.slots[slot].G = static_cast<int>(G);
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
      tiles += static_cast<int>((D.N + TR - 1) / TR);
      max_tile = std::max(max_tile, tb);
    }
    if (take == 0) return RB_ERR_SHAPE;
    p.count = take;
    p.nslots = nslots;
    p.total_tiles = tiles;
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
    off = (off + 15) & ~15u;
    p.ent_off = off;
    off += static_cast<uint32_t>(take) * sizeof(EntryS);
    p.start_off = off;
    off += kWindow * 4;
    off = (off + 15) & ~15u;
    p.red_off = off;
    off += kRedSlots * 3 * 4 + kRedSlots * 2 * kMaxP * 8 * 4;
    off = (off + 7) & ~7u;
    p.bar_off = off;
    off += 2 * kWindow * 8;
    off = (off + 127) & ~127u;
    p.ring_off = off;
    if (off + 2 * max_tile > kSmemMax) return RB_ERR_SHAPE;
    p.ring_bytes = kSmemMax - off;
    void (*kern)(MultiParams) = TR == 16 ? gemv_int4_multi_kernel<16> : gemv_int4_multi_kernel<8>;
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
