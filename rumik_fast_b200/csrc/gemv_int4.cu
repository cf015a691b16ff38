// gemv_int4.cu - int4 group-128 GEMV for batch-1..16 decode on B200 (sm_100a).
//
// Computes y[b, n] = sum_k (code[n,k] * s[n,k/128] + m[n,k/128]) * x[b, k], the operation of rumik-fast's
// gemv_int4_kernel (kernels/cuda_gemv.py:38-115), in the weight layout of kernels/int4_gemv.py:1-3.
//
// Design (B200-first, not a translation of the reference kernel):
//  * Persistent grid, one CTA per SM; CTA b owns the contiguous row band [N*b/C, N*(b+1)/C), so every SM
//    streams the same number of bytes (+-1 row) and each band is one sequential HBM range.
//  * A producer warp streams the band in stages of 8 rows with 1-D bulk async copies (cp.async.bulk, the
//    TMA engine without a tensor map) into a ring of shared-memory slots guarded by mbarriers: 70-100 KB in
//    flight per SM, which is what HBM3e needs (bytes-in-flight = bandwidth x latency). The 8 code rows of a
//    stage are one contiguous range in HBM and move as TWO copies (rows 0-3, rows 4-7 placed 64 bytes
//    further on): the number of bulk copies an SM keeps in flight is limited, so per-row copies of 1.5 KB
//    capped a K=3072 stream at ~2.8 TB/s. MMA row R carries stage row (R&1)*4 + R/2, so the two rows a
//    warp reads in one shared-memory phase come from different halves and hit disjoint banks.
//  * Consumer work items are (stage, K-slice) pairs: a stage's 128-column groups are cut into P slices so
//    that a CTA always has >= 16 items for its consumer warps, whatever its number of stages. Warps take
//    items round-robin with no barrier between stages; partial sums go to shared memory and one
//    fixed-order reduction at the end writes y (deterministic).
//  * Dequantisation is two LOP3 per four codes: (w & 0x000F000F) | 0x64006400 gives the fp16 pair
//    (1024 + c_even), and (w & 0x00F000F0) | 0x54005400 gives (64 + c_odd) - exact fp16 integers with an
//    offset and no subtraction. The products and the fp32 accumulation run on the warp-level MMA
//    (m16n8k16, f16 in, f32 accumulate) used as a dot-product engine: ~1.2 instructions per weight
//    instead of the ~2 of an HFMA2 chain, and fp32 accumulation inside each group (the reference's fp16
//    partial sums alone cost ~1e-3 relative L2 error). The per-group offset sum_k off_k x_k is subtracted
//    in fp32 together with the affine terms: y += s * (dot - off) + m * sum(x).
//  * One MMA covers 8 rows x 32 columns: the 16 MMA rows are 8 weight rows twice, rows 0-7 carrying one
//    half of each row's columns (S1) and rows 8-15 the other half (S2); B column 2b carries batch b's
//    S1 activations and column 2b+1 its S2 activations, so D[r][2b] + D[r+8][2b+1] is row r, batch b.
//    Four batch rows share every MMA; batches 5-16 reuse the dequantised A fragments for more MMAs.
//  * Programmatic dependent launch: with RB_FLAG_PREFETCH_WEIGHTS the producer starts streaming weights
//    before griddepcontrol.wait, so the next GEMV's weights load while the previous kernel finishes;
//    x is read and y written only after the wait.
#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace g4 {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageRows = 8;

struct Gemv4Params {
  const void* x;
  const uint8_t* q;
  const uint16_t* s;
  const uint16_t* m;
  void* y;
  int64_t ldx, ldy;
  int N, K, G, batch;
  int x_bf16, y_bf16, prefetch;
  int ns;           // ring slots
  int nfull;        // full barriers = stages of the largest row band
  int rs;           // shared-memory pitch of a code row within a half stage (bytes, = K/2)
  int stage_bytes;  // bytes per ring slot
  int sblk;         // bytes reserved for the scale block (and again for the min block) in a slot
  int lp;           // lanes per entry of the activation-fragment table (8 per batch row, <= 32)
  int P;            // K-slices per stage
  int gps;          // groups per slice
  uint32_t xs_off, cst_off, zero_off, red_off, bar_off;
  // dequantisation masks and fp16 magic numbers, passed at run time so each mask-and-or is one LOP3:
  // 0x000F000F, 0x00F000F0, 0x64006400 (fp16 1024 | low nibble), 0x54005400 (fp16 64 | high nibble)
  uint32_t m_lo, m_hi, k1024, k64;
};

struct DequantK {
  uint32_t m_lo, m_hi, k1024, k64;
};

// Producer: one thread streams this CTA's row band, stage by stage, into the ring.
__device__ void gemv4_produce(const Gemv4Params& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                              int row_begin, int row_end) {
  const int nst = (row_end - row_begin + kStageRows - 1) / kStageRows;
  const int64_t sm_total = static_cast<int64_t>(p.N) * p.G * 2;  // bytes of s (and of m)
  const uint32_t row_bytes = static_cast<uint32_t>(p.K / 2);
  int issued = 0;
  for (int st = 0; st < nst; ++st) {
    const int slot = st % p.ns;
    if (st >= p.ns && !mbar_wait(&empty[slot], ((st / p.ns) - 1) & 1, ERR_GEMV4_EMPTY)) break;
    const int r0 = row_begin + st * kStageRows;
    const int nr = min(kStageRows, row_end - r0);
    uint8_t* sb = smem + static_cast<size_t>(slot) * p.stage_bytes;
    // scale/min byte range of these rows, widened to 16-byte boundaries for the bulk copy; bytes past the
    // last 16-byte boundary of the tensor are copied with plain loads instead.
    const int64_t b0 = static_cast<int64_t>(r0) * p.G * 2;
    const int64_t b1 = b0 + static_cast<int64_t>(nr) * p.G * 2;
    const int64_t a0 = b0 & ~int64_t(15);
    const int64_t want_end = (b1 + 15) & ~int64_t(15);
    const int64_t end = want_end < sm_total ? want_end : sm_total;
    const uint32_t tma = static_cast<uint32_t>((end & ~int64_t(15)) - a0);
    uint8_t* s_dst = sb + kStageRows * p.rs + 64;
    uint8_t* m_dst = s_dst + p.sblk;
    if (a0 + tma < end) {
      for (int64_t b = a0 + tma; b < end; b += 2) {
        reinterpret_cast<uint16_t*>(s_dst)[(b - a0) >> 1] = p.s[b >> 1];
        reinterpret_cast<uint16_t*>(m_dst)[(b - a0) >> 1] = p.m[b >> 1];
      }
      fence_proxy_async_smem();  // order these generic stores before later bulk copies into the slot
    }
    mbar_arrive_expect_tx(&full[st], nr * row_bytes + 2 * tma);
    const uint8_t* qsrc = p.q + static_cast<int64_t>(r0) * row_bytes;
    // rows 0-3 and rows 4-7 as two contiguous copies, the second 64 bytes further on, so a warp reading
    // one row of each half in the same shared-memory phase hits disjoint banks
    bulk_g2s(sb, qsrc, min(nr, 4) * row_bytes, &full[st]);
    if (nr > 4) bulk_g2s(sb + 4 * p.rs + 64, qsrc + 4 * row_bytes, (nr - 4) * row_bytes, &full[st]);
    if (tma) {
      bulk_g2s(s_dst, reinterpret_cast<const uint8_t*>(p.s) + a0, tma, &full[st]);
      bulk_g2s(m_dst, reinterpret_cast<const uint8_t*>(p.m) + a0, tma, &full[st]);
    }
    issued = st + 1;
  }
  // Do not let the CTA retire with bulk copies still in flight: wait (bounded) for the last stages.
  for (int st = max(0, issued - p.ns); st < issued; ++st)
    mbar_wait(&full[st], 0, ERR_GEMV4_FULL);
}

// Activations -> fp16 MMA B fragments in shared memory, plus per (batch, group) constants
// (offset sum = sum_k off_k x_k with off = 1024 for even and 64 for odd columns, and sum_k x_k).
__device__ void gemv4_stage_x(const Gemv4Params& p, uint8_t* smem, int tid) {
  constexpr int U = 4;  // loads issued together before any is used (one L2 round trip, not U)
  const int items = p.batch * p.G * 16;
  uint8_t* xs = smem + p.xs_off;
  float4* cst = reinterpret_cast<float4*>(smem + p.cst_off);
  for (int base = 0; base < items; base += U * kConsumerWarps * 32) {
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = base + u * kConsumerWarps * 32 + tid;
      raw[u] = make_uint4(0, 0, 0, 0);
      if (it < items) {
        const int b = it / (p.G * 16), rem = it - b * p.G * 16;
        const int64_t col = static_cast<int64_t>(rem >> 4) * 128 + 32 * ((rem >> 2) & 3) + 8 * (rem & 3);
        raw[u] = ldg_cg_128(static_cast<const uint8_t*>(p.x) + (b * p.ldx + col) * 2);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = base + u * kConsumerWarps * 32 + tid;
      const bool valid = it < items;
      float off = 0.f, sum = 0.f;
      int b = 0, g = 0;
      if (valid) {
        b = it / (p.G * 16);
        const int rem = it - b * p.G * 16;
        g = rem >> 4;
        const int qq = (rem >> 2) & 3, j = rem & 3;
        __half h[8];
        raw_to_half8(raw[u], p.x_bf16, h);
        const int pp = b >> 2, bs = b & 3;
        uint8_t* tab = xs + static_cast<size_t>(((pp * p.G + g) * 2 + (j >> 1)) * p.lp) * 16;
        uint32_t* l1 = reinterpret_cast<uint32_t*>(tab + ((2 * bs) * 4 + qq) * 16) + (j & 1) * 2;
        uint32_t* l2 = reinterpret_cast<uint32_t*>(tab + ((2 * bs + 1) * 4 + qq) * 16) + (j & 1) * 2;
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
      if (valid && (it & 15) == 0) cst[b * p.G + g] = make_float4(-off, sum, 0.f, 0.f);
    }
  }
}

// Per-thread 32-bit shared addresses of one work item, each advanced by a fixed stride per group: this
// thread's code bytes (row r, lane quad qd), its row's scale and min, and per batch pass the activation
// fragments and (offset, sum) constants. Lanes whose batch column is unused read a zero block with
// stride 0, so the inner loop has no predicates and no 64-bit address arithmetic.
template <int NP>
struct Gemv4Addr {
  uint32_t w, s, m;
  uint32_t x[NP], c[NP];
  uint32_t xon[NP], con[NP];  // this lane's batch column is in use (else no load, zeros)
};

template <int NP>
struct Gemv4Ops {
  uint4 w;
  float s, m;
  uint4 b01[NP], b23[NP];
  float4 c[NP];  // {-offset sum, sum x, 0, 0}: the first MMA chain starts from it
};

template <int NP>
__device__ __forceinline__ void gemv4_load(const Gemv4Addr<NP>& a, const uint32_t (&xhalf)[NP], Gemv4Ops<NP>& o) {
  o.w = lds128_a(a.w);
  o.s = lds_h2f_a(a.s);
  o.m = lds_h2f_a(a.m);
#pragma unroll
  for (int pp = 0; pp < NP; ++pp) {
    o.b01[pp] = lds128_pa(a.x[pp], a.xon[pp]);
    o.b23[pp] = lds128_pa(a.x[pp] + xhalf[pp], a.xon[pp]);
    o.c[pp] = lds128f_pa(a.c[pp], a.con[pp]);
  }
}

template <int NP>
__device__ __forceinline__ void gemv4_step(Gemv4Addr<NP>& a, const int (&xstep)[NP], const int (&cstep)[NP]) {
  a.w += 64;
  a.s += 2;
  a.m += 2;
#pragma unroll
  for (int pp = 0; pp < NP; ++pp) {
    a.x[pp] += xstep[pp];
    a.c[pp] += cstep[pp];
  }
}

// The dot products of one 128-column group for this thread's (row r, batch lanes), accumulated into acc.
template <int NP>
__device__ __forceinline__ void gemv4_math(const Gemv4Ops<NP>& o, const float4& zq, const DequantK& k,
                                           float (&acc)[NP]) {
  const uint32_t wv[4] = {o.w.x, o.w.y, o.w.z, o.w.w};
  uint32_t a[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t w = wv[j], w8 = wv[j] >> 8;
    a[j][0] = and_or(w, k.m_lo, k.k1024);   // (1024 + c0, 1024 + c4)   row r,   k 2t..2t+1
    a[j][1] = and_or(w8, k.m_lo, k.k1024);  // (1024 + c2, 1024 + c6)   row r+8, k 2t..2t+1
    a[j][2] = and_or(w, k.m_hi, k.k64);     // (64 + c1, 64 + c5)       row r,   k 2t+8..
    a[j][3] = and_or(w8, k.m_hi, k.k64);    // (64 + c3, 64 + c7)       row r+8, k 2t+8..
  }
#pragma unroll
  for (int pp = 0; pp < NP; ++pp) {
    // two short MMA chains; the first starts from -offset (so d0 + d1 is sum_k c_k x_k directly), the
    // second from the zero quad
    float d0[4], d1[4];
    mma_f16_16816_c(d0, a[0][0], a[0][1], a[0][2], a[0][3], o.b01[pp].x, o.b01[pp].y, o.c[pp]);
    mma_f16_16816_c(d1, a[1][0], a[1][1], a[1][2], a[1][3], o.b01[pp].z, o.b01[pp].w, zq);
    mma_f16_16816(d0, a[2][0], a[2][1], a[2][2], a[2][3], o.b23[pp].x, o.b23[pp].y);
    mma_f16_16816(d1, a[3][0], a[3][1], a[3][2], a[3][3], o.b23[pp].z, o.b23[pp].w);
    const float dot = (d0[0] + d0[3]) + (d1[0] + d1[3]);
    acc[pp] = fmaf(o.s, dot, fmaf(o.m, o.c[pp].y, acc[pp]));
  }
}

template <int NP>
__global__ void __launch_bounds__(kThreads, 1) gemv_int4_kernel(const __grid_constant__ Gemv4Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // one full barrier per stage (used for a single phase), one empty barrier per ring slot
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + p.nfull;
  const int row_begin = static_cast<int>(static_cast<int64_t>(p.N) * blockIdx.x / gridDim.x);
  const int row_end = static_cast<int>(static_cast<int64_t>(p.N) * (blockIdx.x + 1) / gridDim.x);
  const int nst = (row_end - row_begin + kStageRows - 1) / kStageRows;

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) mbar_init(&full[i], 1);
    for (int i = 0; i < p.ns; ++i) {
      mbar_init(&empty[i], p.P);  // one arrival per K-slice item of the stage
    }
    fence_mbar_init();
  }
  if (tid < 16) reinterpret_cast<uint32_t*>(smem + p.zero_off)[tid] = 0u;  // 64-byte zero block
  __syncthreads();
  griddep_launch_dependents();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (!p.prefetch) griddep_wait();
      gemv4_produce(p, smem, full, empty, row_begin, row_end);
    }
    return;
  }

  // ---- consumers ----
  griddep_wait();
  gemv4_stage_x(p, smem, tid);
  named_bar_sync(1, kConsumerWarps * 32);

  const int r = lane >> 2, qd = lane & 3;
  const int prow = (r & 1) * 4 + (r >> 1);  // the stage row this lane's MMA row carries
  const uint8_t* xs = smem + p.xs_off;
  const float4* cst = reinterpret_cast<const float4*>(smem + p.cst_off);
  float* red = reinterpret_cast<float*>(smem + p.red_off);
  // per-lane constant parts of the addresses; lanes of unused batch columns point at the zero block
  uint32_t x0[NP], c0[NP], xhalf[NP];
  int xstep[NP], cstep[NP];
  const uint32_t zero_a = smem_u32(smem + p.zero_off);
#pragma unroll
  for (int pp = 0; pp < NP; ++pp) {
    const bool xl = lane < 8 * min(4, p.batch - 4 * pp);   // this lane's batch column is in use
    const int b = 4 * pp + qd;
    x0[pp] = xl ? smem_u32(xs + static_cast<size_t>(pp * p.G * 2 * p.lp + lane) * 16) : zero_a;
    xstep[pp] = xl ? 2 * p.lp * 16 : 0;
    xhalf[pp] = xl ? p.lp * 16 : 0;  // offset of the second fragment pair (0 inside the zero block)
    c0[pp] = b < p.batch ? smem_u32(cst + b * p.G) : zero_a;
    cstep[pp] = b < p.batch ? 16 : 0;
  }
  const float4 zq = lds128f_a(zero_a);  // loop-invariant zero accumulator input
  const DequantK dk = {p.m_lo, p.m_hi, p.k1024, p.k64};
  bool dead = false;
  const int n_items = nst * p.P;
  for (int it = warp; it < n_items; it += kConsumerWarps) {
    const int st = it / p.P, sl = it - st * p.P;
    const int slot = st % p.ns;
    const int r0 = row_begin + st * kStageRows;
    if (!dead && !mbar_wait(&full[st], 0, ERR_GEMV4_FULL)) dead = true;
    float acc0[NP], acc1[NP];
#pragma unroll
    for (int pp = 0; pp < NP; ++pp) acc0[pp] = acc1[pp] = 0.f;
    if (!dead) {
      const uint8_t* sq = smem + static_cast<size_t>(slot) * p.stage_bytes;
      const int shift = static_cast<int>((static_cast<int64_t>(r0) * p.G * 2) & 15) >> 1;
      const int g0 = sl * p.gps, g1 = min(p.G, g0 + p.gps);
      Gemv4Addr<NP> A;
      A.w = smem_u32(sq + (r & 1) * (4 * p.rs + 64) + (r >> 1) * p.rs + qd * 16) + g0 * 64;
      A.s = smem_u32(sq + kStageRows * p.rs + 64) + (shift + prow * p.G + g0) * 2;
      A.m = A.s + p.sblk;
#pragma unroll
      for (int pp = 0; pp < NP; ++pp) {
        A.x[pp] = x0[pp] + g0 * xstep[pp];
        A.c[pp] = c0[pp] + g0 * cstep[pp];
        A.xon[pp] = xstep[pp] != 0;
        A.con[pp] = cstep[pp] != 0;
      }
      int g = g0;
      for (; g + 1 < g1; g += 2) {  // two independent groups: all loads first, then both groups' math
        Gemv4Ops<NP> o0, o1;
        gemv4_load<NP>(A, xhalf, o0);
        gemv4_step<NP>(A, xstep, cstep);
        gemv4_load<NP>(A, xhalf, o1);
        gemv4_step<NP>(A, xstep, cstep);
        gemv4_math<NP>(o0, zq, dk, acc0);
        gemv4_math<NP>(o1, zq, dk, acc1);
      }
      if (g < g1) {
        Gemv4Ops<NP> o0;
        gemv4_load<NP>(A, xhalf, o0);
        gemv4_math<NP>(o0, zq, dk, acc0);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
#pragma unroll
    for (int pp = 0; pp < NP; ++pp) red[((st * p.P + sl) * NP + pp) * 32 + lane] = acc0[pp] + acc1[pp];
  }
  named_bar_sync(1, kConsumerWarps * 32);
  // fixed-order reduction over the K-slices of every stage, then the stores
  for (int o = tid; o < nst * NP * 32; o += kConsumerWarps * 32) {
    const int st = o / (NP * 32), rem = o - st * NP * 32, pp = rem >> 5, l = rem & 31;
    float v = 0.f;
    for (int sl = 0; sl < p.P; ++sl) v += red[((st * p.P + sl) * NP + pp) * 32 + l];
    const int row = row_begin + st * kStageRows + ((l >> 2) & 1) * 4 + (l >> 3), b = pp * 4 + (l & 3);
    if (!dead && row < row_end && b < p.batch) store_out(p.y, b * p.ldy + row, v, p.y_bf16);
  }
}

}  // namespace g4

int launch_gemv_int4(const GemvArgs& a, int num_sms, cudaStream_t stream) {
  using namespace g4;
  const int G = static_cast<int>(a.K / 128);
  const int ctas = static_cast<int>(std::min<int64_t>((a.N + kStageRows - 1) / kStageRows, num_sms));
  const int64_t rows_max = (a.N + ctas - 1) / ctas;
  const int nst_max = static_cast<int>((rows_max + kStageRows - 1) / kStageRows);
  // K-slices per stage: enough items for two rounds of the consumer warps, at least 2 groups per slice
  int P = 1;
  while (P < 8 && nst_max * P < 2 * kConsumerWarps && G / (2 * P) >= 2) P *= 2;
  const int gps = (G + P - 1) / P;
  const int half_k = static_cast<int>(a.K / 2);
  const int rs = half_k;  // rows packed as in HBM within each half of a stage
  const int sblk = 16 * G + 16;
  const int stage_bytes = ((kStageRows * rs + 64 + 2 * sblk) + 127) & ~127;
  constexpr int kSmemMax = 227 * 1024;
  constexpr int kCoResident = 110 * 1024;  // two CTAs per SM: this kernel and the next one (PDL)

  // Split the batch into launches whose activation tables fit in shared memory next to >= 2 ring slots.
  int64_t done = 0;
  while (done < a.batch) {
    int bc = static_cast<int>(std::min<int64_t>(16, a.batch - done));
    int np = 0, lp = 0, ns = 0;
    uint32_t xs_off = 0, cst_off = 0, zero_off = 0, red_off = 0, bar_off = 0, total = 0;
    for (;; --bc) {
      if (bc < 1) return RB_ERR_SHAPE;
      np = (bc + 3) / 4;
      if (np == 3) np = 4;
      lp = 8 * std::min(4, bc);
      const uint32_t xs_bytes = static_cast<uint32_t>(np) * G * 2 * lp * 16;
      const uint32_t cst_bytes = static_cast<uint32_t>(bc) * G * 16;
      const uint32_t red_bytes = static_cast<uint32_t>(nst_max) * P * np * 32 * 4;
      const uint32_t fixed = xs_bytes + cst_bytes + 64 + red_bytes + (nst_max + 8) * 8 + 256;
      int slots = static_cast<int>((static_cast<int64_t>(kCoResident) - fixed) / stage_bytes);
      slots = std::max(2, std::min(slots, 8));
      slots = std::min(slots, std::max(1, nst_max));
      uint32_t need = static_cast<uint32_t>(slots) * stage_bytes + fixed;
      while (need > static_cast<uint32_t>(kSmemMax) && slots > 1) {
        --slots;
        need -= stage_bytes;
      }
      if (need > static_cast<uint32_t>(kSmemMax)) continue;
      ns = slots;
      xs_off = static_cast<uint32_t>(ns) * stage_bytes;
      cst_off = xs_off + xs_bytes;
      zero_off = cst_off + ((cst_bytes + 15) & ~15u);
      red_off = zero_off + 64;
      bar_off = red_off + red_bytes;
      total = bar_off + (nst_max + ns) * 8;
      break;
    }
    Gemv4Params p;
    p.x = static_cast<const uint8_t*>(a.x) + done * a.ldx * 2;
    p.q = a.q;
    p.s = a.s;
    p.m = a.m;
    p.y = static_cast<uint8_t*>(a.y) + done * a.ldy * 2;
    p.ldx = a.ldx;
    p.ldy = a.ldy;
    p.N = static_cast<int>(a.N);
    p.K = static_cast<int>(a.K);
    p.G = G;
    p.batch = bc;
    p.x_bf16 = a.x_dtype == RB_BF16;
    p.y_bf16 = a.y_dtype == RB_BF16;
    p.prefetch = (a.flags & RB_FLAG_PDL) && (a.flags & RB_FLAG_PREFETCH_WEIGHTS) ? 1 : 0;
    p.ns = ns;
    p.nfull = nst_max;
    p.rs = rs;
    p.stage_bytes = stage_bytes;
    p.sblk = sblk;
    p.lp = lp;
    p.P = P;
    p.gps = gps;
    p.xs_off = xs_off;
    p.cst_off = cst_off;
    p.zero_off = zero_off;
    p.red_off = red_off;
    p.bar_off = bar_off;
    p.m_lo = 0x000F000Fu;
    p.m_hi = 0x00F000F0u;
    p.k1024 = 0x64006400u;
    p.k64 = 0x54005400u;

    void (*kern)(Gemv4Params) = np == 1 ? gemv_int4_kernel<1> : np == 2 ? gemv_int4_kernel<2> : gemv_int4_kernel<4>;
    cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), kSmemMax);
    if (e != cudaSuccess) return RB_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (a.flags & RB_FLAG_PDL) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return RB_ERR_LAUNCH;
    done += bc;
  }
  return RB_OK;
}

}  // namespace rb
