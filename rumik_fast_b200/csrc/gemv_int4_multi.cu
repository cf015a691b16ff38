// gemv_int4_multi.cu - one persistent launch for a list of independent int4 GEMVs (a decode step's
// projection set), batch 1, on B200 (sm_100a).
//
// A decode step issued as one kernel per GEMV pays a fixed cost per launch (launch, dependency wait,
// activation staging, tail) of several microseconds; 145 of them are as long as the whole step's HBM time.
// This kernel removes the boundaries for GEMVs whose inputs are all available at launch (the reference's
// projection-set benchmark, kernels/bench_gemv.py:83-113, and any set of independent projections):
//  * every activation vector of the list is converted to MMA B fragments once, at kernel start;
//  * the 8-row tiles of all matrices form one global list dealt round-robin to the CTAs (one per SM), so
//    every SM streams the same number of tiles, tile boundaries never stall the HBM stream, and one
//    producer warp keeps ~180 KB of tiles in flight per SM in a byte-granular FIFO ring (tiles of
//    different K have different sizes);
//  * each tile is one work item for one of 16 consumer warps, which reuse the int4 GEMV's inner loop
//    (gemv4_load / gemv4_math: LOP3 magic-number dequantisation, m16n8k16 MMA as an fp32-accumulating dot
//    product) over all groups of the row and write its 8 outputs directly;
//  * full/empty mbarriers are per tile, reused modulo a window that is provably larger than any consumer's
//    lead over the oldest unreleased tile, so a waiting warp can never see a stale phase.
#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace g4m {

constexpr int kConsumerWarps = 16;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxEntries = 256;
constexpr int kMaxSlots = 8;
constexpr int kWindow = 128;       // barrier window (tiles)
constexpr int kMaxOutstanding = 64; // tiles in flight per CTA (window >= this + consumer warps)

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

struct MultiParams {
  int count, nslots, total_tiles, x_bf16, y_bf16, prefetch;
  uint32_t ring_bytes, ring_off, bar_off, start_off, zero_off;
  uint32_t m_lo, m_hi, k1024, k64;
  Slot slots[kMaxSlots];
  Entry e[kMaxEntries];
};

__device__ __forceinline__ uint32_t tile_bytes(int K, int G) {
  return ((8u * (K / 2) + 64u + 2u * (16u * G + 16u)) + 127u) & ~127u;
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

__device__ void multi_produce(const MultiParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                              uint32_t* start) {
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
    while (e + 1 < p.count && gt >= p.e[e + 1].tile_begin) ++e;
    const Entry& E = p.e[e];
    const uint32_t b = tile_bytes(E.K, E.G);
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
    const int row0 = (gt - E.tile_begin) * 8;
    const int nr = min(8, E.N - row0);
    const uint32_t row_bytes = static_cast<uint32_t>(E.K / 2);
    const uint32_t rs = row_bytes, sblk = 16u * E.G + 16u;
    uint8_t* sb = ring + pos;
    const int64_t sm_total = static_cast<int64_t>(E.N) * E.G * 2;
    const int64_t b0 = static_cast<int64_t>(row0) * E.G * 2;
    const int64_t b1 = b0 + static_cast<int64_t>(nr) * E.G * 2;
    const int64_t a0 = b0 & ~int64_t(15);
    const int64_t want_end = (b1 + 15) & ~int64_t(15);
    const int64_t end = want_end < sm_total ? want_end : sm_total;
    const uint32_t tma = static_cast<uint32_t>((end & ~int64_t(15)) - a0);
    uint8_t* s_dst = sb + 8 * rs + 64;
    uint8_t* m_dst = s_dst + sblk;
    if (a0 + tma < end) {
      for (int64_t bb = a0 + tma; bb < end; bb += 2) {
        reinterpret_cast<uint16_t*>(s_dst)[(bb - a0) >> 1] = E.s[bb >> 1];
        reinterpret_cast<uint16_t*>(m_dst)[(bb - a0) >> 1] = E.m[bb >> 1];
      }
      fence_proxy_async_smem();
    }
    uint64_t* fb = &full[j % kWindow];
    mbar_arrive_expect_tx(fb, nr * row_bytes + 2 * tma);  // also publishes start[] (release)
    const uint8_t* qsrc = E.q + static_cast<int64_t>(row0) * row_bytes;
    bulk_g2s(sb, qsrc, min(nr, 4) * row_bytes, fb);
    if (nr > 4) bulk_g2s(sb + 4 * rs + 64, qsrc + 4 * row_bytes, (nr - 4) * row_bytes, fb);
    if (tma) {
      bulk_g2s(s_dst, reinterpret_cast<const uint8_t*>(E.s) + a0, tma, fb);
      bulk_g2s(m_dst, reinterpret_cast<const uint8_t*>(E.m) + a0, tma, fb);
    }
  }
  // no retirement with copies in flight
  for (int t = old; t < j; ++t) mbar_wait(&full[t % kWindow], (t / kWindow) & 1, ERR_MULTI_FULL);
}

__global__ void __launch_bounds__(kThreads, 1) gemv_int4_multi_kernel(const __grid_constant__ MultiParams p) {
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
  __syncthreads();
  griddep_launch_dependents();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (!p.prefetch) griddep_wait();
      multi_produce(p, smem, full, empty, start);
    }
    return;
  }

  griddep_wait();
  stage_all_x(p, smem, tid);
  named_bar_sync(1, kConsumerWarps * 32);

  const int C = gridDim.x, cta = blockIdx.x;
  const int ntiles = (p.total_tiles - cta + C - 1) / C;
  const int r = lane >> 2, qd = lane & 3;
  const int prow = (r & 1) * 4 + (r >> 1);
  const uint32_t zero_a = smem_u32(smem + p.zero_off);
  const float4 zq = lds128f_a(zero_a);
  const g4::DequantK dk = {p.m_lo, p.m_hi, p.k1024, p.k64};
  const bool xl = lane < 8;   // batch 1: lanes 0-7 carry the activation columns
  const bool cl = qd == 0;
  const uint32_t xhalf[1] = {xl ? 8u * 16u : 0u};
  const int xstep[1] = {xl ? 2 * 8 * 16 : 0};
  const int cstep[1] = {cl ? 16 : 0};
  const uint8_t* ring = smem + p.ring_off;
  bool dead = false;
  int e = 0;
  for (int j = warp; j < ntiles; j += kConsumerWarps) {
    const int gt = cta + j * C;
    while (e + 1 < p.count && gt >= p.e[e + 1].tile_begin) ++e;
    const Entry& E = p.e[e];
    if (!dead && !mbar_wait(&full[j % kWindow], (j / kWindow) & 1, ERR_MULTI_FULL)) dead = true;
    float acc0[1] = {0.f}, acc1[1] = {0.f};
    const int row0 = (gt - E.tile_begin) * 8;
    if (!dead) {
      const uint8_t* sq = ring + start[j % kWindow];
      const int rs = E.K / 2, G = E.G;
      const int shift = static_cast<int>((static_cast<int64_t>(row0) * G * 2) & 15) >> 1;
      const Slot& S = p.slots[E.slot];
      g4::Gemv4Addr<1> A;
      A.w = smem_u32(sq + (r & 1) * (4 * rs + 64) + (r >> 1) * rs + qd * 16);
      A.s = smem_u32(sq + 8 * rs + 64) + (shift + prow * G) * 2;
      A.m = A.s + 16u * G + 16u;
      A.x[0] = xl ? smem_u32(smem + S.tab_off) + lane * 16 : zero_a;
      A.c[0] = cl ? smem_u32(smem + S.cst_off) : zero_a;
      A.xon[0] = xl;
      A.con[0] = cl;
      int g = 0;
      for (; g + 1 < G; g += 2) {
        g4::Gemv4Ops<1> o0, o1;
        g4::gemv4_load<1>(A, xhalf, o0);
        g4::gemv4_step<1>(A, xstep, cstep);
        g4::gemv4_load<1>(A, xhalf, o1);
        g4::gemv4_step<1>(A, xstep, cstep);
        g4::gemv4_math<1>(o0, zq, dk, acc0);
        g4::gemv4_math<1>(o1, zq, dk, acc1);
      }
      if (g < G) {
        g4::Gemv4Ops<1> o0;
        g4::gemv4_load<1>(A, xhalf, o0);
        g4::gemv4_math<1>(o0, zq, dk, acc0);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[j % kWindow]);
      const int row = row0 + prow;
      if (qd == 0 && row < E.N) store_out(E.y, row, acc0[0] + acc1[0], p.y_bf16);
    }
  }
}

}  // namespace g4m

int launch_gemv_int4_multi(const rb_gemv_desc* d, int count, int x_dtype, int y_dtype, int flags, int num_sms,
                           cudaStream_t stream) {
  using namespace g4m;
  constexpr uint32_t kSmemMax = 227 * 1024;
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
    constexpr uint32_t kFixed = 64 + kWindow * 4 + 8 + 2 * kWindow * 8 + 128;
    int nslots = 0, tiles = 0;
    uint32_t x_bytes = 0, max_tile = 0;
    int take = 0;
    for (; take < n; ++take) {
      const rb_gemv_desc& D = d[done + take];
      const uint32_t G = static_cast<uint32_t>(D.K / 128);
      const uint32_t tb = ((8u * static_cast<uint32_t>(D.K / 2) + 64u + 2u * (16u * G + 16u)) + 127u) & ~127u;
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
      tiles += static_cast<int>((D.N + 7) / 8);
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
    p.start_off = off;
    off += kWindow * 4;
    off = (off + 7) & ~7u;
    p.bar_off = off;
    off += 2 * kWindow * 8;
    off = (off + 127) & ~127u;
    p.ring_off = off;
    if (off + 2 * max_tile > kSmemMax) return RB_ERR_SHAPE;
    p.ring_bytes = kSmemMax - off;
    cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(gemv_int4_multi_kernel), kSmemMax);
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
    e = cudaLaunchKernelEx(&cfg, gemv_int4_multi_kernel, p);
    if (e != cudaSuccess) return RB_ERR_LAUNCH;
    done += take;
  }
  return RB_OK;
}

}  // namespace rb
