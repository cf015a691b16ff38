// gemv_int8.cu - int8 per-row-scale GEMV (the tied audio head) for batch-1..16 decode on B200 (sm_100a).
//
// Computes y[b, n] = s[n] * sum_k v(q[n,k]) * x[b, k], the operation of rumik-fast's gemv_int8_kernel
// (kernels/cuda_gemv.py:141-186), with v(q) = q - 128 for the uint8 storage that quantize_int8_rows writes
// (kernels/cuda_gemv.py:234-242) or v(q) = (int8)q for signed storage.
//
// Same streaming skeleton as the int4 GEMV (persistent row bands, 8-row stages moved by 1-D bulk async
// copies into an mbarrier ring, producer warp + 8 consumer warps, PDL weight prefetch). Dequantisation is
// one PRMT per two weights: prmt(w, 0x64646464, 0x4140) = fp16 pair (1024 + u0, 1024 + u1); signed storage
// first flips the sign bits (u = b ^ 0x80 = b + 128). The MMA accumulates sum_k (1024 + u_k) x_k over the
// whole row in fp32; the epilogue subtracts 1152 * sum_k x_k and applies the row scale. Any N is accepted
// (the reference needs N % 16 == 0 and pads the 16,385 head rows to 16,400).
#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace g8 {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageRows = 8;

struct Gemv8Params {
  const void* x;
  const uint8_t* q;
  const void* s;
  void* y;
  int64_t ldx, ldy;
  int N, K, C, batch;  // C = K / 64 chunks per row
  int x_bf16, y_bf16, s_f32, q_signed, prefetch;
  int ns, rs, stage_bytes, lp;
  int nfull;  // full barriers = stages of the largest row band
  int P, cps;  // K-slices per stage and 64-column chunks per slice
  uint32_t xs_off, xsum_off, part_off, red_off, bar_off;
};

__device__ void gemv8_produce(const Gemv8Params& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                              int row_begin, int row_end) {
  const int nst = (row_end - row_begin + kStageRows - 1) / kStageRows;
  const uint32_t row_bytes = static_cast<uint32_t>(p.K);
  int issued = 0;
  for (int st = 0; st < nst; ++st) {
    const int slot = st % p.ns;
    if (st >= p.ns && !mbar_wait(&empty[slot], ((st / p.ns) - 1) & 1, ERR_GEMV8_EMPTY)) break;
    const int r0 = row_begin + st * kStageRows;
    const int nr = min(kStageRows, row_end - r0);
    uint8_t* sb = smem + static_cast<size_t>(slot) * p.stage_bytes;
    mbar_arrive_expect_tx(&full[st], nr * row_bytes);
    const uint8_t* qsrc = p.q + static_cast<int64_t>(r0) * row_bytes;
    bulk_g2s(sb, qsrc, nr * row_bytes, &full[st]);  // the stage's rows are one contiguous range
    issued = st + 1;
  }
  for (int st = max(0, issued - p.ns); st < issued; ++st)
    mbar_wait(&full[st], 0, ERR_GEMV8_FULL);
}

// Activations -> fp16 B fragments: for chunk ch (64 columns) and lane quad qq, the S1 lane of batch b
// holds x[c..c+3], x[c+8..c+11] and the S2 lane x[c+4..c+7], x[c+12..c+15], c = 64 ch + 16 qq.
__device__ void gemv8_stage_x(const Gemv8Params& p, uint8_t* smem, int tid) {
  const int items = p.batch * p.C * 4;
  uint8_t* xs = smem + p.xs_off;
  float* xsum = reinterpret_cast<float*>(smem + p.xsum_off);
  float* part = reinterpret_cast<float*>(smem + p.part_off);
  for (int base = 0; base < items; base += kConsumerWarps * 32) {
    const int it = base + tid;
    const bool valid = it < items;
    float sum = 0.f;
    int b = 0;
    if (valid) {
      b = it / (p.C * 4);
      const int rem = it - b * p.C * 4;
      const int ch = rem >> 2, qq = rem & 3;
      const int64_t col = static_cast<int64_t>(ch) * 64 + 16 * qq;
      const uint8_t* src = static_cast<const uint8_t*>(p.x) + (b * p.ldx + col) * 2;
      __half h[16];
      load8_as_half(src, p.x_bf16, *reinterpret_cast<__half(*)[8]>(&h[0]));
      load8_as_half(src + 16, p.x_bf16, *reinterpret_cast<__half(*)[8]>(&h[8]));
      const int pp = b >> 2, bs = b & 3;
      uint8_t* tab = xs + static_cast<size_t>((pp * p.C + ch) * p.lp) * 16;
      uint32_t* l1 = reinterpret_cast<uint32_t*>(tab + ((2 * bs) * 4 + qq) * 16);
      uint32_t* l2 = reinterpret_cast<uint32_t*>(tab + ((2 * bs + 1) * 4 + qq) * 16);
      l1[0] = pack_half2(h[0], h[1]);
      l1[1] = pack_half2(h[2], h[3]);
      l1[2] = pack_half2(h[8], h[9]);
      l1[3] = pack_half2(h[10], h[11]);
      l2[0] = pack_half2(h[4], h[5]);
      l2[1] = pack_half2(h[6], h[7]);
      l2[2] = pack_half2(h[12], h[13]);
      l2[3] = pack_half2(h[14], h[15]);
#pragma unroll
      for (int i = 0; i < 16; ++i) sum += __half2float(h[i]);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (valid && (it & 3) == 0) part[it >> 2] = sum;  // = part[b * C + ch]
  }
  named_bar_sync(1, kConsumerWarps * 32);
  // fixed-order total per batch row, so results do not depend on thread timing
  if (tid < p.batch) {
    float t = 0.f;
    for (int ch = 0; ch < p.C; ++ch) t += part[tid * p.C + ch];
    xsum[tid] = t;
  }
}

template <int NP>
__global__ void __launch_bounds__(kThreads, 1) gemv_int8_kernel(const __grid_constant__ Gemv8Params p) {
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
      mbar_init(&empty[i], p.P);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch_dependents();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (!p.prefetch) griddep_wait();
      gemv8_produce(p, smem, full, empty, row_begin, row_end);
    }
    return;
  }

  griddep_wait();
  gemv8_stage_x(p, smem, tid);
  named_bar_sync(1, kConsumerWarps * 32);

  const int r = lane >> 2, qd = lane & 3;
  const uint8_t* xs = smem + p.xs_off;
  const float* xsum = reinterpret_cast<const float*>(smem + p.xsum_off);
  float* red = reinterpret_cast<float*>(smem + p.red_off);
  const uint32_t flip = p.q_signed ? 0x80808080u : 0u;
  bool dead = false;
  const int n_items = nst * p.P;
  for (int it = warp; it < n_items; it += kConsumerWarps) {
    const int st = it / p.P, sl = it - st * p.P;
    const int slot = st % p.ns;
    if (!dead && !mbar_wait(&full[st], 0, ERR_GEMV8_FULL)) dead = true;
    float d[NP][2][4];  // two independent MMA chains per pass
#pragma unroll
    for (int pp = 0; pp < NP; ++pp)
#pragma unroll
      for (int h = 0; h < 2; ++h) d[pp][h][0] = d[pp][h][1] = d[pp][h][2] = d[pp][h][3] = 0.f;
    if (!dead) {
      const uint8_t* wrow = smem + static_cast<size_t>(slot) * p.stage_bytes + r * p.rs + qd * 16;
      const int c0 = sl * p.cps, c1 = min(p.C, c0 + p.cps);
      for (int ch = c0; ch < c1; ++ch) {
        const uint4 wq = lds128(wrow + ch * 64);
        const uint32_t wv[4] = {wq.x ^ flip, wq.y ^ flip, wq.z ^ flip, wq.w ^ flip};
        uint32_t a[2][4];
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          a[jj][0] = __byte_perm(wv[2 * jj], 0x64646464u, 0x4140);      // (1024+u0, 1024+u1) row r
          a[jj][2] = __byte_perm(wv[2 * jj], 0x64646464u, 0x4342);      // (1024+u2, 1024+u3) row r
          a[jj][1] = __byte_perm(wv[2 * jj + 1], 0x64646464u, 0x4140);  // (1024+u4, 1024+u5) row r+8
          a[jj][3] = __byte_perm(wv[2 * jj + 1], 0x64646464u, 0x4342);  // (1024+u6, 1024+u7) row r+8
        }
#pragma unroll
        for (int pp = 0; pp < NP; ++pp) {
          const int lanes_p = 8 * min(4, p.batch - 4 * pp);
          uint4 bb = make_uint4(0, 0, 0, 0);
          if (lane < lanes_p) bb = lds128(xs + static_cast<size_t>((pp * p.C + ch) * p.lp + lane) * 16);
          mma_f16_16816(d[pp][0], a[0][0], a[0][1], a[0][2], a[0][3], bb.x, bb.y);
          mma_f16_16816(d[pp][1], a[1][0], a[1][1], a[1][2], a[1][3], bb.z, bb.w);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
#pragma unroll
    for (int pp = 0; pp < NP; ++pp)
      red[((st * p.P + sl) * NP + pp) * 32 + lane] = (d[pp][0][0] + d[pp][0][3]) + (d[pp][1][0] + d[pp][1][3]);
  }
  named_bar_sync(1, kConsumerWarps * 32);
  // fixed-order reduction over the K-slices of every stage, then scale and store
  for (int o = tid; o < nst * NP * 32; o += kConsumerWarps * 32) {
    const int st = o / (NP * 32), rem = o - st * NP * 32, pp = rem >> 5, l = rem & 31;
    const int row = row_begin + st * kStageRows + (l >> 2), b = pp * 4 + (l & 3);
    if (dead || row >= row_end || b >= p.batch) continue;
    float v = 0.f;
    for (int sl = 0; sl < p.P; ++sl) v += red[((st * p.P + sl) * NP + pp) * 32 + l];
    const float srow = p.s_f32 ? __ldg(static_cast<const float*>(p.s) + row)
                               : __half2float(__ldg(static_cast<const __half*>(p.s) + row));
    store_out(p.y, b * p.ldy + row, srow * (v - 1152.f * xsum[b]), p.y_bf16);
  }
}

}  // namespace g8

int launch_gemv_int8(const GemvArgs& a, int num_sms, cudaStream_t stream) {
  using namespace g8;
  const int C = static_cast<int>(a.K / 64);
  const int ctas = static_cast<int>(std::min<int64_t>((a.N + kStageRows - 1) / kStageRows, num_sms));
  const int64_t rows_max = (a.N + ctas - 1) / ctas;
  const int nst_max = static_cast<int>((rows_max + kStageRows - 1) / kStageRows);
  int P = 1;
  while (P < 8 && nst_max * P < 2 * kConsumerWarps && C / (2 * P) >= 4) P *= 2;
  const int cps = (C + P - 1) / P;
  const int K = static_cast<int>(a.K);
  const int rs = K;  // rows packed as in HBM: one bulk copy per stage
  const int stage_bytes = (kStageRows * rs + 127) & ~127;
  constexpr int kSmemMax = 227 * 1024;
  constexpr int kCoResident = 110 * 1024;

  int64_t done = 0;
  while (done < a.batch) {
    int bc = static_cast<int>(std::min<int64_t>(16, a.batch - done));
    int np = 0, lp = 0, ns = 0;
    uint32_t xs_off = 0, xsum_off = 0, part_off = 0, red_off = 0, bar_off = 0, total = 0;
    for (;; --bc) {
      if (bc < 1) return RB_ERR_SHAPE;
      np = (bc + 3) / 4;
      if (np == 3) np = 4;
      lp = 8 * min(4, bc);
      const uint32_t xs_bytes = static_cast<uint32_t>(np) * C * lp * 16;
      const uint32_t red_bytes = static_cast<uint32_t>(nst_max) * P * np * 32 * 4;
      const uint32_t part_bytes = static_cast<uint32_t>(bc) * C * 4;
      const uint32_t fixed = xs_bytes + 64 + part_bytes + red_bytes + (nst_max + 8) * 8 + 256;
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
      xsum_off = xs_off + xs_bytes;
      part_off = xsum_off + 64;
      red_off = part_off + ((part_bytes + 15) & ~15u);
      bar_off = red_off + red_bytes;
      total = bar_off + (nst_max + ns) * 8;
      break;
    }
    Gemv8Params p;
    p.x = static_cast<const uint8_t*>(a.x) + done * a.ldx * 2;
    p.q = a.q;
    p.s = a.s_row;
    p.y = static_cast<uint8_t*>(a.y) + done * a.ldy * 2;
    p.ldx = a.ldx;
    p.ldy = a.ldy;
    p.N = static_cast<int>(a.N);
    p.K = K;
    p.C = C;
    p.batch = bc;
    p.x_bf16 = a.x_dtype == RB_BF16;
    p.y_bf16 = a.y_dtype == RB_BF16;
    p.s_f32 = a.s_dtype == RB_F32;
    p.q_signed = a.q_signed ? 1 : 0;
    p.prefetch = (a.flags & RB_FLAG_PDL) && (a.flags & RB_FLAG_PREFETCH_WEIGHTS) ? 1 : 0;
    p.ns = ns;
    p.nfull = nst_max;
    p.rs = rs;
    p.stage_bytes = stage_bytes;
    p.lp = lp;
    p.P = P;
    p.cps = cps;
    p.xs_off = xs_off;
    p.xsum_off = xsum_off;
    p.part_off = part_off;
    p.red_off = red_off;
    p.bar_off = bar_off;

    void (*kern)(Gemv8Params) = np == 1 ? gemv_int8_kernel<1> : np == 2 ? gemv_int8_kernel<2> : gemv_int8_kernel<4>;
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
