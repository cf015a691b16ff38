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
//    flight per SM, which is what HBM3e needs (bytes-in-flight = bandwidth x latency).
//  * Code rows land in shared memory with a row pitch = 64 (mod 128) bytes, so the 8 rows a warp reads in
//    one step hit disjoint banks.
//  * Eight consumer warps split the 128-column groups of a stage. Dequantisation is two LOP3 per four
//    codes: (w & 0x000F000F) | 0x64006400 gives the fp16 pair (1024 + c_even), and
//    (w & 0x00F000F0) | 0x54005400 gives (64 + c_odd) - exact fp16 integers with an offset and no
//    subtraction. The products and the fp32 accumulation run on the warp-level MMA (m16n8k16, f16 in,
//    f32 accumulate) used as a dot-product engine: ~1.1 instructions per weight instead of the ~2 of an
//    HFMA2 chain, and fp32 accumulation inside each group (the reference's fp16 partial sums alone
//    cost ~1e-3 relative L2 error). The per-group offset sum_k off_k x_k is subtracted in fp32 together
//    with the affine terms: y += s * (dot - off) + m * sum(x).
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
  int rs;           // shared-memory pitch of a code row in a stage (bytes, = 64 mod 128)
  int stage_bytes;  // bytes per ring slot
  int sblk;         // bytes reserved for the scale block (and again for the min block) in a slot
  int lp;           // lanes per entry of the activation-fragment table (8 per batch row, <= 32)
  uint32_t xs_off, cst_off, red_off, bar_off;
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
    uint8_t* s_dst = sb + kStageRows * p.rs;
    uint8_t* m_dst = s_dst + p.sblk;
    if (a0 + tma < end) {
      for (int64_t b = a0 + tma; b < end; b += 2) {
        reinterpret_cast<uint16_t*>(s_dst)[(b - a0) >> 1] = p.s[b >> 1];
        reinterpret_cast<uint16_t*>(m_dst)[(b - a0) >> 1] = p.m[b >> 1];
      }
      fence_proxy_async_smem();  // order these generic stores before later bulk copies into the slot
    }
    mbar_arrive_expect_tx(&full[slot], nr * row_bytes + 2 * tma);
    const uint8_t* qsrc = p.q + static_cast<int64_t>(r0) * row_bytes;
    for (int rr = 0; rr < nr; ++rr) bulk_g2s(sb + rr * p.rs, qsrc + rr * row_bytes, row_bytes, &full[slot]);
    if (tma) {
      bulk_g2s(s_dst, reinterpret_cast<const uint8_t*>(p.s) + a0, tma, &full[slot]);
      bulk_g2s(m_dst, reinterpret_cast<const uint8_t*>(p.m) + a0, tma, &full[slot]);
    }
    issued = st + 1;
  }
  // Do not let the CTA retire with bulk copies still in flight: wait (bounded) for the last stages.
  for (int st = max(0, issued - p.ns); st < issued; ++st)
    mbar_wait(&full[st % p.ns], (st / p.ns) & 1, ERR_GEMV4_FULL);
}

// Activations -> fp16 MMA B fragments in shared memory, plus per (batch, group) constants
// (offset sum = sum_k off_k x_k with off = 1024 for even and 64 for odd columns, and sum_k x_k).
__device__ void gemv4_stage_x(const Gemv4Params& p, uint8_t* smem, int tid) {
  const int items = p.batch * p.G * 16;
  uint8_t* xs = smem + p.xs_off;
  float2* cst = reinterpret_cast<float2*>(smem + p.cst_off);
  const size_t esz = 2;
  for (int base = 0; base < items; base += kConsumerWarps * 32) {
    const int it = base + tid;
    const bool valid = it < items;
    float off = 0.f, sum = 0.f;
    int b = 0, g = 0;
    if (valid) {
      b = it / (p.G * 16);
      const int rem = it - b * p.G * 16;
      g = rem >> 4;
      const int qq = (rem >> 2) & 3, j = rem & 3;
      __half h[8];
      const int64_t col = static_cast<int64_t>(g) * 128 + 32 * qq + 8 * j;
      load8_as_half(static_cast<const uint8_t*>(p.x) + (b * p.ldx + col) * esz, p.x_bf16, h);
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
    if (valid && (it & 15) == 0) cst[b * p.G + g] = make_float2(off, sum);
  }
}

template <int NP>
__global__ void __launch_bounds__(kThreads, 1) gemv_int4_kernel(const __grid_constant__ Gemv4Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + p.ns;
  const int row_begin = static_cast<int>(static_cast<int64_t>(p.N) * blockIdx.x / gridDim.x);
  const int row_end = static_cast<int>(static_cast<int64_t>(p.N) * (blockIdx.x + 1) / gridDim.x);
  const int nst = (row_end - row_begin + kStageRows - 1) / kStageRows;

  if (tid == 0) {
    for (int i = 0; i < p.ns; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
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
  const uint8_t* xs = smem + p.xs_off;
  const float2* cst = reinterpret_cast<const float2*>(smem + p.cst_off);
  bool dead = false;
  for (int st = 0; st < nst; ++st) {
    const int slot = st % p.ns;
    const int r0 = row_begin + st * kStageRows;
    const int nr = min(kStageRows, row_end - r0);
    if (!dead && !mbar_wait(&full[slot], (st / p.ns) & 1, ERR_GEMV4_FULL)) dead = true;
    float acc[NP];
#pragma unroll
    for (int pp = 0; pp < NP; ++pp) acc[pp] = 0.f;
    if (!dead) {
      const uint8_t* sq = smem + static_cast<size_t>(slot) * p.stage_bytes;
      const int shift = static_cast<int>((static_cast<int64_t>(r0) * p.G * 2) & 15) >> 1;
      const uint16_t* ss = reinterpret_cast<const uint16_t*>(sq + kStageRows * p.rs) + shift;
      const uint16_t* sm = reinterpret_cast<const uint16_t*>(sq + kStageRows * p.rs + p.sblk) + shift;
      const uint8_t* wrow = sq + r * p.rs + qd * 16;
      for (int g = warp; g < p.G; g += kConsumerWarps) {
        const uint4 wq = lds128(wrow + g * 64);
        const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
        uint32_t a[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t w = wv[j], w8 = wv[j] >> 8;
          a[j][0] = (w & 0x000F000Fu) | 0x64006400u;   // (1024 + c0, 1024 + c4)   row r,   k 2t..2t+1
          a[j][1] = (w8 & 0x000F000Fu) | 0x64006400u;  // (1024 + c2, 1024 + c6)   row r+8, k 2t..2t+1
          a[j][2] = (w & 0x00F000F0u) | 0x54005400u;   // (64 + c1, 64 + c5)       row r,   k 2t+8..
          a[j][3] = (w8 & 0x00F000F0u) | 0x54005400u;  // (64 + c3, 64 + c7)       row r+8, k 2t+8..
        }
        const float sc = __half2float(__ushort_as_half(ss[r * p.G + g]));
        const float mn = __half2float(__ushort_as_half(sm[r * p.G + g]));
#pragma unroll
        for (int pp = 0; pp < NP; ++pp) {
          const int lanes_p = 8 * min(4, p.batch - 4 * pp);
          uint4 b01 = make_uint4(0, 0, 0, 0), b23 = make_uint4(0, 0, 0, 0);
          if (lane < lanes_p) {
            const uint8_t* e = xs + static_cast<size_t>((pp * p.G + g) * 2 * p.lp + lane) * 16;
            b01 = lds128(e);
            b23 = lds128(e + p.lp * 16);
          }
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_f16_16816(d, a[0][0], a[0][1], a[0][2], a[0][3], b01.x, b01.y);
          mma_f16_16816(d, a[1][0], a[1][1], a[1][2], a[1][3], b01.z, b01.w);
          mma_f16_16816(d, a[2][0], a[2][1], a[2][2], a[2][3], b23.x, b23.y);
          mma_f16_16816(d, a[3][0], a[3][1], a[3][2], a[3][3], b23.z, b23.w);
          const int b = 4 * pp + qd;
          const float2 c = (b < p.batch) ? cst[b * p.G + g] : make_float2(0.f, 0.f);
          acc[pp] = fmaf(sc, (d[0] + d[3]) - c.x, fmaf(mn, c.y, acc[pp]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // cross-warp reduction of this stage's 8 rows (double-buffered by stage parity)
    float* red = reinterpret_cast<float*>(smem + p.red_off) + (st & 1) * kConsumerWarps * NP * 32;
#pragma unroll
    for (int pp = 0; pp < NP; ++pp) red[(warp * NP + pp) * 32 + lane] = acc[pp];
    named_bar_sync(1, kConsumerWarps * 32);
    if (!dead && warp < NP) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) v += red[(w * NP + warp) * 32 + lane];
      const int b = warp * 4 + qd;
      if (r < nr && b < p.batch) store_out(p.y, b * p.ldy + r0 + r, v, p.y_bf16);
    }
  }
}

}  // namespace g4

int launch_gemv_int4(const GemvArgs& a, int num_sms, cudaStream_t stream) {
  using namespace g4;
  const int G = static_cast<int>(a.K / 128);
  const int ctas = static_cast<int>(std::min<int64_t>((a.N + kStageRows - 1) / kStageRows, num_sms));
  const int64_t rows_max = (a.N + ctas - 1) / ctas;
  const int nst_max = static_cast<int>((rows_max + kStageRows - 1) / kStageRows);
  const int half_k = static_cast<int>(a.K / 2);
  const int rs = half_k + ((half_k % 128) == 0 ? 64 : 0);
  const int sblk = 16 * G + 16;
  const int stage_bytes = ((kStageRows * rs + 2 * sblk) + 127) & ~127;
  constexpr int kSmemMax = 227 * 1024;
  constexpr int kCoResident = 110 * 1024;  // two CTAs per SM: this kernel and the next one (PDL)

  // Split the batch into launches whose activation tables fit in shared memory next to >= 2 ring slots.
  int64_t done = 0;
  while (done < a.batch) {
    int bc = static_cast<int>(std::min<int64_t>(16, a.batch - done));
    int np = 0, lp = 0, ns = 0;
    uint32_t xs_off = 0, cst_off = 0, red_off = 0, bar_off = 0, total = 0;
    for (;; --bc) {
      if (bc < 1) return RB_ERR_SHAPE;
      np = (bc + 3) / 4;
      if (np == 3) np = 4;
      lp = 8 * min(4, bc);
      const uint32_t xs_bytes = static_cast<uint32_t>(np) * G * 2 * lp * 16;
      const uint32_t cst_bytes = static_cast<uint32_t>(bc) * G * 8;
      const uint32_t red_bytes = 2 * kConsumerWarps * np * 32 * 4;
      const uint32_t fixed = xs_bytes + cst_bytes + red_bytes + 2 * 8 * 8 + 256;
      int slots = static_cast<int>((static_cast<int64_t>(kCoResident) - fixed) / stage_bytes);
      slots = max(2, min(slots, 8));
      slots = min(slots, max(1, nst_max));
      uint32_t need = static_cast<uint32_t>(slots) * stage_bytes + fixed;
      while (need > static_cast<uint32_t>(kSmemMax) && slots > 1) {
        --slots;
        need -= stage_bytes;
      }
      if (need > static_cast<uint32_t>(kSmemMax)) continue;
      ns = slots;
      xs_off = static_cast<uint32_t>(ns) * stage_bytes;
      cst_off = xs_off + xs_bytes;
      red_off = cst_off + ((cst_bytes + 15) & ~15u);
      bar_off = red_off + red_bytes;
      total = bar_off + 2 * ns * 8;
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
    p.rs = rs;
    p.stage_bytes = stage_bytes;
    p.sblk = sblk;
    p.lp = lp;
    p.xs_off = xs_off;
    p.cst_off = cst_off;
    p.red_off = red_off;
    p.bar_off = bar_off;

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
