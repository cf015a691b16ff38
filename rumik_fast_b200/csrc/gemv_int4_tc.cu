// gemv_int4_tc.cu - a list of independent int4 group-128 GEMVs (batch 1) in one persistent launch on the
// tcgen05 tensor cores of B200 (sm_100a), with the dequantised weights in tensor memory.
//
// y_i = W_i x_i for every entry, the operation of rumik-fast's gemv_int4_kernel (kernels/cuda_gemv.py:38-115)
// applied to a decode step's projection set (kernels/bench_gemv.py:83-113).
//
// Work is cut into blocks of 128 weight rows (one UMMA M, one tensor-memory lane per row); the blocks of all
// matrices are dealt round-robin to the CTAs, one CTA per SM. Per CTA:
//  * warp 0 (producer) streams each block's int4 codes two groups (128 columns x 2) at a time with 2-D TMA
//    (box 128 bytes x 128 rows, 128-byte swizzle, 16 KB) into a ring per converter set;
//  * each converter set (four warps, one per tensor-memory lane quadrant, thread = weight row) unpacks one
//    group of its row to unsigned 8-bit codes (even columns as the code, odd columns as 16 x the code: two
//    instructions per eight codes, no dequantisation at all) and writes the 32 columns to tensor memory
//    (tcgen05.st);
//  * one thread per set issues four tcgen05.mma.kind::i8 per group (K = 32 each), eight per pair of groups
//    (one TMA stage, the unit in which converters and MMA issuers synchronise): A = the codes in tensor
//    memory (128 rows), B = the group's activations quantised to 16-bit integers and split into a signed
//    high byte and a signed low byte, each in one B row for the even columns and one for the odd columns
//    (B rows 0-3), read from shared memory by a K-major, no-swizzle descriptor; D = 128 x 8 int32 in tensor
//    memory (columns 0-3 used), exact;
//  * two pairs later the converter reads its row's four accumulator columns per group (tcgen05.ld) and adds
//    s * delta / 16 * (4096 D0 + 16 D1 + 256 D2 + D3) in fp32; m * sum(x) is added when the group is unpacked.
// The activations are quantised per 128-column group with delta = max|x| / 32639 (relative error below
// 2e-5 of the group's largest activation); the weights are used exactly. All mbarrier waits are bounded;
// no multicast, no clusters.
#include "common.cuh"
#include "tc.cuh"
#include "glue.cuh"
#include "kernels.h"

namespace rb {

namespace g4t {

#ifndef RB_TC_SETS
#define RB_TC_SETS 3
#endif
constexpr int kSets = RB_TC_SETS;          // converter sets (four warps each); sets take alternate blocks
constexpr int kRows = 128;                 // rows per block = UMMA M = tensor-memory lanes
constexpr int kConvWarps = 4 * kSets;
constexpr int kFirstConv = 1 + kSets;      // warp 0 producer, warps 1..kSets the MMA issuers of the sets
constexpr int kThreads = (kFirstConv + kConvWarps) * 32;
constexpr uint32_t kStageBytes = kRows * 128;  // two groups of codes for 128 rows
constexpr int kMaxStages = 6;              // ring stages per set
constexpr int kMaxEntries = 160;
constexpr int kMaxSlots = 8;
constexpr int kNP = 2;  // tensor-memory buffers per set, each for a PAIR of groups (one TMA stage): the epilogue
                        // reads a pair's results two pairs after writing its codes
constexpr uint32_t kACols = 64, kDCols = 16, kSetCols = kNP * (kACols + kDCols);  // group 0 | group 1 halves
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kXPad = 256;            // bytes the B descriptor's unused rows read past a table
// Activation table per group: 8 chunks of 16 positions, each 4 B rows of 16 bytes: the high and low bytes of x at
// the even-column positions (zero at the odd ones), then those at the odd-column positions. The odd-column codes
// then stay in their high nibble (16 x code): one instruction per 8 codes fewer than shifting them down.
constexpr uint32_t kXGroupBytes = 512;
constexpr uint32_t kXChunkBytes = 64;

constexpr int kMaxEpis = 4;                // routed (non-store) epilogues per launch
constexpr int kLnIter = 4;                 // prologue: 8-element chunks per converter thread (H <= 4 x 384 x 8)
constexpr int kBarLn = 2 + kSets;          // named barriers: 1 = tables staged, 2 + s = set s, kBarLn = prologue
enum : int { kEpiStore = RB_EPI_STORE, kEpiRopeKv = RB_EPI_ROPE_KV, kEpiSwiglu = RB_EPI_SWIGLU };

struct Entry {
  const uint16_t* s;  // fp16 scales [N, G]; 8-bit scales (s8): the packed (scale code, zero point) pairs [N, G]
  const void* m;      // fp16 mins [N, G]; s8: the fp32 per-row scale factors [N]
  void* y;
  int N, G, slot, block_begin;
  int epi, ep;  // epilogue kind, index into TcParams::epis
  // K split: each 128-row block is cut into `ks` slices of `ppk` pairs of groups (the last may be shorter);
  // work item i of this entry (i from item_begin) is block i / ks, slice i % ks
  int ks, ppk, item_begin;
  int fmt;  // kFmt* bits: the weight and scale format (fills the struct's padding)
};
// Entry::fmt. kFmtS8: int4 codes with 8-bit double-quantised scales (rb_gemv_desc::s_row set). kFmtW8: int8
// rows (rb_gemv_desc::w8): q int8 [N, K], one scale per row (s: fp16 [N]; m: fp32 [N] with kFmtRowF32), a stage
// holds ONE group and the item's "pairs" are its groups. kFmtOffset: the codes are stored as uint8 = int8 + 128.
constexpr int kFmtS8 = 1, kFmtW8 = 2, kFmtOffset = 4, kFmtRowF32 = 8;
constexpr uint32_t kIdescASigned = 1u << 7;  // instruction descriptor, kind::i8: A signed 8-bit
// Stages (16 KB: 128 bytes of every row) per 128-row block of an entry: two int4 groups or one int8 group each.
__host__ __device__ __forceinline__ int entry_pairs(int G, int fmt) { return (fmt & kFmtW8) ? G : (G + 1) / 2; }

struct Slot {
  const void* x;  // activations; for the prologue slot the residual stream
  const void* a;  // prologue (ln != 0): x + a + b -> LayerNorm with weight w
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
};

struct __align__(64) TcParams {
  CUtensorMap maps[kMaxEntries];  // codes of each entry: [N rows, K/2 bytes], box 128 x 128, 128B swizzle
  Entry e[kMaxEntries];
  Slot slots[kMaxSlots];
  EpiP epis[kMaxEpis];
  int count, nslots, total_blocks, total_items, x_bf16, y_bf16, prefetch, nst;
  uint32_t xs_off, bar_off, aux_off, idesc;
  float* ws_part;           // split K: fp32 partial results, 128 per work item
  unsigned int* ws_ticket;  // split K: slices finished per block (global block index), zero between launches
};
static_assert(sizeof(TcParams) <= 32000, "kernel parameter block too large");

// Auxiliary shared memory: the prologue's two arrays of group sums, then per set the split-K "last slice" flag.
constexpr uint32_t kAuxBytes = 2 * kLnMaxGroups * 4 + 16;

// Split-K workspace: one completion counter per 128-row block (rounded up to 256 bytes), then the partials.
inline int64_t split_ticket_bytes(int blocks) { return (static_cast<int64_t>(blocks) * 4 + 255) / 256 * 256; }

// B operand descriptor over an activation table: K-major, no swizzle, 16-byte rows at a 16-byte pitch, the next
// 16 K-elements of a row kChunk bytes further on (leading byte offset), 8-row groups 128 bytes apart (unused with
// N = 8), descriptor version 1 (sm_100). This kernel's tables: kChunk = 64 (rows 0-3 of a chunk; B rows 4-7 read
// the next chunk, their D columns are never read). The int8 head's: kChunk = 32 (rows 0-1).
template <uint32_t kChunk = kXChunkBytes>
__device__ __forceinline__ uint64_t x_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(kChunk >> 4) << 16) |
         (static_cast<uint64_t>(128 >> 4) << 32) | (static_cast<uint64_t>(1) << 46);
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::i8 (A unsigned, B signed, D int32), one CTA.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Accumulator columns 0 and 1 of this thread's lane; the registers are valid only after tmem_wait_ld, which
// takes them as operands so that no use can be scheduled before it.
__device__ __forceinline__ void tmem_ld2(uint32_t taddr, int& h, int& l) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(h), "=r"(l) : "r"(taddr) : "memory");
}
// Accumulator columns 0-3 (rows 0-3 of B: even-column high / low, odd-column high / low) of this lane; valid only
// after tmem_wait_ld4, which takes them as operands so that no use can be scheduled before it.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, int (&d)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld4(int (&d)[4]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3]) : : "memory");
}
// 16 x a group's integer dot product from its accumulators; exact in int32 (|value| < 1.02e9).
__device__ __forceinline__ float group_dot16(const int (&d)[4]) {
  return static_cast<float>((d[0] << 12) + (d[1] << 4) + (d[2] << 8) + d[3]);
}
// The same for an int8 group, whose odd-column codes are not scaled by 16 in tensor memory: 16 x (256 (D0 + D2)
// + D1 + D3). The int32 sum is exact (|value| <= 128 * 127 * 32767 < 2^29); its conversion rounds to 24 bits.
__device__ __forceinline__ float group_dot16_w8(const int (&d)[4]) {
  return static_cast<float>(((d[0] + d[2]) << 8) + d[1] + d[3]) * 16.f;
}
__device__ __forceinline__ float h2f_lo(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
}
__device__ __forceinline__ float h2f_hi(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}
__device__ __forceinline__ void tmem_wait_ld(int& h, int& l) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(h), "+r"(l) : : "memory");
}

// Activation tables: for every slot and 128-column group, x quantised to 16-bit integers
// xi = rint(x / delta), delta = max|x| / 32639, split as xi = 256 * hi + lo with hi, lo signed bytes, in the
// order in which a converter thread writes a group's codes to tensor memory (within each 8 columns: the four
// even columns, then the four odd ones), stored per 16 positions as four 16-byte B rows (kXChunkBytes); plus per
// group {delta / 16, sum(x)}.
//
// One chunk: positions 8c .. 8c + 7 of a slot. All 32 lanes call this together (a group is 16 chunks = 16
// consecutive threads, reduced with shuffles); lanes with valid == false contribute zeros and write nothing.
__device__ __forceinline__ void quant_chunk(const float (&v)[8], bool valid, int c, uint8_t* tab, float2* cst) {
  float mx = 0.f, sum = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mx = fmaxf(mx, fabsf(v[i]));
    sum += v[i];
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  const float delta = mx > 0.f ? mx / 32639.f : 1.f;
  const float inv = 1.f / delta;
  if (valid) {
    uint32_t hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
#pragma unroll
    for (int jp = 0; jp < 8; ++jp) {  // table position jp <- column (jp < 4 ? 2 jp : 2 (jp - 4) + 1)
      const int col = jp < 4 ? 2 * jp : 2 * (jp - 4) + 1;
      const int xi = __float2int_rn(fminf(fmaxf(v[col] * inv, -32639.f), 32639.f));
      const int l = ((xi + 128) & 255) - 128;
      const int h = (xi - l) >> 8;
      hi[jp >> 2] |= (static_cast<uint32_t>(h) & 255u) << (8 * (jp & 3));
      lo[jp >> 2] |= (static_cast<uint32_t>(l) & 255u) << (8 * (jp & 3));
    }
    // positions 8 * (c % 16) .. + 7 of the group: 16-position chunk (c % 16) / 2, half (c & 1)
    uint8_t* dst = tab + (c >> 4) * kXGroupBytes + ((c & 15) >> 1) * kXChunkBytes + (c & 1) * 8;
    *reinterpret_cast<uint2*>(dst) = make_uint2(hi[0], 0u);       // B row 0: even-column x, high bytes
    *reinterpret_cast<uint2*>(dst + 16) = make_uint2(lo[0], 0u);  // B row 1: even-column x, low bytes
    *reinterpret_cast<uint2*>(dst + 32) = make_uint2(0u, hi[1]);  // B row 2: odd-column x, high bytes
    *reinterpret_cast<uint2*>(dst + 48) = make_uint2(0u, lo[1]);  // B row 3: odd-column x, low bytes
    // 4096 D0 + 16 D1 + 256 D2 + D3 is 16 x the group's dot product in units of delta
    if ((c & 15) == 0) cst[c >> 4] = make_float2(delta * 0.0625f, sum);
  }
}

__device__ __forceinline__ LnSrc ln_src(const Slot& S) {
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
  return L;
}

// The same add + LayerNorm on its own (the final norm in front of the head): one CTA; bit-identical to the
// prologue of the fused launches (the prologue's sums do not depend on the thread count).
__global__ void __launch_bounds__(kConvWarps * 32, 1) add_ln_kernel(const __grid_constant__ Slot S, int bf) {
  __shared__ float gsum[2 * kLnMaxGroups];
  griddep_wait();
  stage_ln<kLnIter>(ln_src(S), bf != 0, gsum, 1, threadIdx.x, kConvWarps * 32, true,
                    [](const float (&)[8], bool, int) {});
  griddep_launch_dependents();
}

constexpr int kPreChunks = 8;  // chunks of 8 activations a converter thread loads before it quantises any

__device__ void stage_x_tables(const TcParams& p, uint8_t* xs, float* red, int ct, int nthreads) {
  // The plain slots' activations were written by the previous kernel: issue every load first (up to
  // kPreChunks per thread, one round trip to memory), then quantise. Lists with more activations per thread
  // load the rest chunk by chunk.
  uint4 pre[kPreChunks];
#pragma unroll
  for (int i = 0; i < kPreChunks; ++i) {  // the i-th chunk this thread will quantise (constant index: registers)
    int rem = i, c = -1;
    const void* src = nullptr;
    for (int sl = 0; sl < p.nslots; ++sl) {
      const Slot& S = p.slots[sl];
      if (S.ln) continue;
      const int iters = (S.K / 8 + nthreads - 1) / nthreads;
      if (rem < iters) {
        c = rem * nthreads + ct;
        src = c < S.K / 8 ? S.x : nullptr;
        break;
      }
      rem -= iters;
    }
    pre[i] = src ? ldg_cg_128(static_cast<const uint8_t*>(src) + static_cast<int64_t>(c) * 16)
                 : make_uint4(0u, 0u, 0u, 0u);
  }
  int n = 0;
  for (int sl = 0; sl < p.nslots; ++sl) {
    const Slot& S = p.slots[sl];
    uint8_t* tab = xs + S.tab_off;
    float2* cst = reinterpret_cast<float2*>(xs + S.cst_off);
    if (S.ln) {
      stage_ln<kLnIter>(ln_src(S), p.x_bf16 != 0, red, kBarLn, ct, nthreads, blockIdx.x == 0,
                        [&](const float (&h)[8], bool valid, int c) { quant_chunk(h, valid, c, tab, cst); });
    } else {
      const int chunks = S.K / 8;  // 16 per group
      for (int base = 0; base < chunks; base += nthreads, ++n) {
        const int c = base + ct;
        const bool valid = c < chunks;
        uint4 raw = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int i = 0; i < kPreChunks; ++i)
          if (i == n) raw = pre[i];
        if (n >= kPreChunks && valid) raw = ldg_cg_128(static_cast<const uint8_t*>(S.x) + static_cast<int64_t>(c) * 16);
        float v[8];
        raw_to_f32(raw, p.x_bf16, v);
        quant_chunk(v, valid, c, tab, cst);
      }
    }
    for (int i = ct; i < static_cast<int>(kXPad / 16); i += nthreads)
      reinterpret_cast<uint4*>(tab + S.G * kXGroupBytes)[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Block (within its entry) and pair range [p0, p1) of global work item gi of entry E (for int8 entries the
// "pairs" are single groups: one stage each).
__device__ __forceinline__ void item_range(const Entry& E, int gi, int& blk, int& p0, int& p1) {
  const int li = gi - E.item_begin;
  blk = li / E.ks;
  p0 = (li - blk * E.ks) * E.ppk;
  p1 = min(p0 + E.ppk, entry_pairs(E.G, E.fmt));
}

// The entry of global work item gi (entries hold consecutive item ranges; e only moves forward).
__device__ __forceinline__ const Entry& entry_of(const TcParams& p, int gi, int& e) {
  while (e + 1 < p.count && gi >= p.e[e + 1].item_begin) ++e;
  return p.e[e];
}

// kS8: the launch has entries with 8-bit scales (each entry's format is then checked where its scales are read).
// Launches without any run the instance with kS8 = false, which has no trace of the decoder: carrying it costs
// the fp16 path about 4 % (same-box A/B). kW8: the launch has int8 entries (checked per work item).
template <bool kS8, bool kW8>
__global__ void __launch_bounds__(kThreads, 1) gemv_int4_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = gridDim.x, cta = blockIdx.x;
  const int nst = p.nst;
  const int nlocal = (p.total_items - cta + C - 1) / C;  // this CTA's work items: cta + j * C
  uint8_t* xs = smem + p.xs_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  // per set: full[nst], empty[nst], afull[kNP], mdone[kNP]
  const int per_set = 2 * nst + 2 * kNP;
  auto full = [&](int s, int i) { return bars + s * per_set + i; };
  auto empty = [&](int s, int i) { return bars + s * per_set + nst + i; };
  auto afull = [&](int s, int b) { return bars + s * per_set + 2 * nst + b; };
  auto mdone = [&](int s, int b) { return bars + s * per_set + 2 * nst + kNP + b; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kSets * per_set);
  float* aux = reinterpret_cast<float*>(smem + p.aux_off);  // prologue group sums, then split-K flags

  if (tid == 0) {
    for (int s = 0; s < kSets; ++s) {
      for (int i = 0; i < nst; ++i) {
        mbar_init(full(s, i), 1);
        mbar_init(empty(s, i), 4);
      }
      for (int b = 0; b < kNP; ++b) {
        mbar_init(afull(s, b), 4);
        mbar_init(mdone(s, b), 1);
      }
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
    // ---------------- producer ----------------
    if (lane == 0) {
      if (!p.prefetch) griddep_wait();
      int j[kSets], k[kSets], nk[kSets], e[kSets], row0[kSets], issued[kSets];
      bool live[kSets];
      for (int s = 0; s < kSets; ++s) {
        e[s] = 0;
        j[s] = s;
        k[s] = 0;
        issued[s] = 0;
        live[s] = j[s] < nlocal;
        if (live[s]) {
          const int gi = cta + j[s] * C;
          const Entry& E = entry_of(p, gi, e[s]);
          int blk;
          item_range(E, gi, blk, k[s], nk[s]);
          row0[s] = blk * kRows;
        }
      }
      bool ok = true;
      bool any = true;
      while (any && ok) {
        any = false;
        for (int s = 0; s < kSets && ok; ++s) {
          if (!live[s]) continue;
          any = true;
          const int slot = issued[s] % nst;
          if (issued[s] >= nst && !mbar_wait(empty(s, slot), ((issued[s] / nst) - 1) & 1, ERR_TC_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full(s, slot), kStageBytes);
          mm4::tma_load_2d(smem + (static_cast<size_t>(s) * nst + slot) * kStageBytes, &p.maps[e[s]], k[s] * 128,
                           row0[s], full(s, slot));
          ++issued[s];
          if (++k[s] == nk[s]) {
            j[s] += kSets;
            live[s] = j[s] < nlocal;
            if (live[s]) {
              const int gi = cta + j[s] * C;
              const Entry& E = entry_of(p, gi, e[s]);
              int blk;
              item_range(E, gi, blk, k[s], nk[s]);
              row0[s] = blk * kRows;
            }
          }
        }
      }
      // no retirement with copies in flight
      for (int s = 0; s < kSets; ++s)
        for (int t = max(0, issued[s] - nst); t < issued[s]; ++t)
          if (!mbar_wait(full(s, t % nst), (t / nst) & 1, ERR_TC_WAIT)) break;
    }
  } else if (warp < kFirstConv) {
    // ---------------- MMA issuer of set s ----------------
    const int s = warp - 1;
    named_bar_sync(1, (kSets + kConvWarps) * 32);  // activation tables staged
    if (lane == 0) {
      mm4::tc_fence_after();
      int e = 0, q = 0;
      bool ok = true;
      for (int jj = s; jj < nlocal && ok; jj += kSets) {
        const int gi = cta + jj * C;
        const Entry& E = entry_of(p, gi, e);
        int blk, p0, p1;
        item_range(E, gi, blk, p0, p1);
        const uint32_t xtab = smem_u32(xs + p.slots[E.slot].tab_off);
        const bool w8 = kW8 && (E.fmt & kFmtW8);  // one group per stage, A signed
        const uint32_t idesc = w8 ? p.idesc | kIdescASigned : p.idesc;
        for (int pp = p0; pp < p1; ++pp, ++q) {
          const int b = q % kNP;
          if (!mbar_wait(afull(s, b), (q / kNP) & 1, ERR_TC_WAIT)) {
            ok = false;
            break;
          }
          mm4::tc_fence_after();
          const uint32_t acol = s * kSetCols + b * kACols, dcol = s * kSetCols + kNP * kACols + b * kDCols;
          const int g = w8 ? pp : 2 * pp;
          const int ng = w8 ? 1 : min(2, E.G - g);
          for (int h = 0; h < ng; ++h)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              umma_ts(tmem + dcol + 8 * h, tmem + acol + 32 * h + 8 * i,
                      x_desc(xtab + (g + h) * kXGroupBytes + 2 * kXChunkBytes * i), idesc, i > 0);
          mm4::umma_commit(mdone(s, b));
        }
      }
    }
  } else {
    // ---------------- converters + epilogue of set s ----------------
    const int cw = warp - kFirstConv;        // 0 .. kConvWarps-1
    const int s = cw >> 2;
    const int quad = warp & 3;               // tensor-memory lane quadrant this warp may access
    const int rib = quad * 32 + lane;        // row in block = tensor-memory lane
    griddep_wait();                          // x may come from the previous kernel; y is written below
    stage_x_tables(p, xs, aux, tid - kFirstConv * 32, kConvWarps * 32);
    fence_proxy_async_smem();                // generic writes of the tables -> visible to the tensor core
    named_bar_sync(1, (kSets + kConvWarps) * 32);
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    int e = 0, q = 0, st = 0;
    bool ok = true;
    for (int jj = s; jj < nlocal; jj += kSets) {
      const int gi = cta + jj * C;
      const Entry& E = entry_of(p, gi, e);
      const int G = E.G;
      const bool w8 = kW8 && (E.fmt & kFmtW8);  // int8 rows: one group per stage
      int blk, p0, p1;
      item_range(E, gi, blk, p0, p1);
      const int row = blk * kRows + rib;
      const bool row_ok = row < E.N;
      const uint16_t* srow = E.s + static_cast<int64_t>(row_ok ? row : 0) * G;
      const float2* cst = reinterpret_cast<const float2*>(xs + p.slots[E.slot].cst_off);
      float acc = 0.f;
      // s * delta of the two groups of each pair whose results are pending, oldest pair first (0 for a missing
      // second group: its accumulator columns hold stale finite integers, which the zero scale cancels)
      float pa[kNP] = {0.f, 0.f}, pb[kNP] = {0.f, 0.f};
      const int qp0 = q;  // pair counter of this set at the item's first pair
      const uint32_t a_set = tq + s * kSetCols, d_set = tq + s * kSetCols + kNP * kACols;
      const int npairs = p1 - p0;  // pairs of this item: p0 .. p1 - 1 of the block
      // codes of the next pair (both groups of one stage), software-pipelined one pair ahead
      uint4 wn[8];
      auto load_codes = [&](int k) {
        const int slot = st % nst;
        if (ok) ok = mbar_wait(full(s, slot), (st / nst) & 1, ERR_TC_WAIT);
        if (ok) {
          const uint8_t* rowp = smem + (static_cast<size_t>(s) * nst + slot) * kStageBytes + rib * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) wn[c] = lds128(rowp + ((c ^ (rib & 7)) << 4));
        }
        (void)k;
      };
      auto unpack = [&](const uint4* w, uint32_t* o) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            o[c * 8 + t * 2 + 0] = wv[t] & 0x0F0F0F0Fu;         // even columns of these 8
            o[c * 8 + t * 2 + 1] = wv[t] & 0xF0F0F0F0u;         // odd columns, as 16 x code
          }
        }
      };
      // int8 codes of one group (the stage's 128 bytes of this row) in the order unpack gives the int4 codes:
      // within every 8 columns the four even ones, then the four odd ones (stored uint8 = int8 + 128: the top
      // bit flipped gives the int8 code)
      auto order8 = [&](const uint4* w, uint32_t* o) {
        const uint32_t flip = (E.fmt & kFmtOffset) ? 0x80808080u : 0u;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t a0 = w[c].x ^ flip, a1 = w[c].y ^ flip, a2 = w[c].z ^ flip, a3 = w[c].w ^ flip;
          o[4 * c + 0] = __byte_perm(a0, a1, 0x6420);
          o[4 * c + 1] = __byte_perm(a0, a1, 0x7531);
          o[4 * c + 2] = __byte_perm(a2, a3, 0x6420);
          o[4 * c + 3] = __byte_perm(a2, a3, 0x7531);
        }
      };
      auto dot16 = [&](const int (&d)[4]) { return w8 ? group_dot16_w8(d) : group_dot16(d); };
      // the item's pair k (groups g, g + 1 of the block; for int8 rows the one group g): codes into tensor
      // memory, results of the pair kNP back
      auto step = [&](int k, float s0, float m0, float s1, float m1) {
        const int g = w8 ? p0 + k : 2 * (p0 + k);
        const bool two = !w8 && g + 1 < G;
        const uint4 w[8] = {wn[0], wn[1], wn[2], wn[3], wn[4], wn[5], wn[6], wn[7]};
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(s, st % nst));  // both groups of this stage are in registers
        ++st;
        const float2 ca = cst[g];
        const float2 cb = two ? cst[g + 1] : make_float2(0.f, 0.f);
        acc = fmaf(m0, ca.y, acc);
        if (two) acc = fmaf(m1, cb.y, acc);
        const int qq = qp0 + k, b = qq % kNP;
        const bool epi = k >= kNP;
        int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};
        ok = __all_sync(0xffffffffu, ok);  // tcgen05 loads / stores are warp-collective
        if (epi && ok) {  // the pair kNP back used this buffer: fetch its results once its MMAs are done
          ok = __all_sync(0xffffffffu, mbar_wait(mdone(s, b), ((qq / kNP) - 1) & 1, ERR_TC_WAIT));
          if (ok) mm4::tc_fence_after();
        }
        if (ok) {
          uint32_t o[32];
          if (w8) {
            order8(w, o);
            tmem_st32(a_set + b * kACols, o);
          } else {
            unpack(w, o);
            tmem_st32(a_set + b * kACols, o);
            unpack(w + 4, o);
            tmem_st32(a_set + b * kACols + 32, o);
          }
          if (epi) {  // issued after the codes, so that the accumulators are not live across the unpack
            tmem_ld4(d_set + b * kDCols, d0);
            tmem_ld4(d_set + b * kDCols + 8, d1);
          }
        }
        if (k + 1 < npairs) load_codes(k + 1);  // overlaps the tensor-memory traffic above
        ok = __all_sync(0xffffffffu, ok);
        if (epi && ok) {
          tmem_wait_ld4(d0);
          tmem_wait_ld4(d1);
          acc = fmaf(pa[0], dot16(d0), acc);
          acc = fmaf(pb[0], group_dot16(d1), acc);  // 0 for int8 rows
        }
        if (epi) {
          pa[0] = pa[1];
          pb[0] = pb[1];
          pa[1] = s0 * ca.x;
          pb[1] = two ? s1 * cb.x : 0.f;
        } else if (k == 0) {
          pa[0] = s0 * ca.x;
          pb[0] = two ? s1 * cb.x : 0.f;
        } else {
          pa[1] = s0 * ca.x;
          pb[1] = two ? s1 * cb.x : 0.f;
        }
        if (ok) {
          tmem_wait_st();
          mm4::tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(afull(s, b));
      };
      load_codes(0);
      const int g0 = 2 * p0, g1 = min(2 * p1, G);  // this item's groups
      // 8-bit scales: each chunk of (scale code, zero point) words is expanded to the fp16 scale / min pairs that
      // the fp16 format stores, and both formats then run the same code. The format, the mins' row and the row's
      // scale factor are read from the kernel parameters when used, not held in registers across the chunk.
      const int64_t r0 = row_ok ? row : 0;
      auto mins_at = [&](int g) { return static_cast<const uint16_t*>(E.m) + r0 * G + g; };
      auto expand = [&](uint32_t& sw, uint32_t& mw) {
        dq_scales8_f16x2(sw, __ldg(static_cast<const float*>(E.m) + r0), sw, mw);
      };
      if (w8) {
        // int8 rows: one scale per row, no min (16 x the scale: dot16 is 16 x the dot in units of delta / 16)
        const float sr = (E.fmt & kFmtRowF32) ? __ldg(static_cast<const float*>(E.m) + r0)
                                              : __half2float(__ushort_as_half(__ldg(E.s + r0)));
        for (int k = 0; k < npairs; ++k) step(k, sr, 0.f, 0.f, 0.f);
      } else if ((G & 7) == 0) {
        // scales and mins of 4 groups (2 pairs) per 8-byte load, fetched one iteration (about 2.7 us) ahead; two
        // pair steps per iteration, so the pair step is inlined twice rather than four times (fewer
        // instruction-fetch stalls: +1.1 % on the whole-step list, same-box A/B; fully rolled, one step per
        // iteration, is 0.4 % slower; fetching 8 groups a chunk ahead instead spilled and was no faster). With
        // G % 8 == 0 every item starts on a multiple of 8 groups and holds a multiple of 8 groups (slices are a
        // multiple of 4 pairs), so both pairs of an iteration exist and the loads are 8-byte aligned.
        uint2 sn = __ldg(reinterpret_cast<const uint2*>(srow + g0));
        uint2 mn = (kS8 && (E.fmt & kFmtS8)) ? sn : __ldg(reinterpret_cast<const uint2*>(mins_at(g0)));
#pragma unroll 1
        for (int g4 = g0; g4 < g1; g4 += 4) {
          uint32_t sw0 = sn.x, sw1 = sn.y, mw0 = mn.x, mw1 = mn.y;
          if (g4 + 4 < g1) {
            sn = __ldg(reinterpret_cast<const uint2*>(srow + g4 + 4));
            mn = (kS8 && (E.fmt & kFmtS8)) ? sn : __ldg(reinterpret_cast<const uint2*>(mins_at(g4 + 4)));
          }
          if (kS8 && (E.fmt & kFmtS8)) {
            expand(sw0, mw0);
            expand(sw1, mw1);
          }
          const int k0 = (g4 - g0) >> 1;
          step(k0, h2f_lo(sw0), h2f_lo(mw0), h2f_hi(sw0), h2f_hi(mw0));
          step(k0 + 1, h2f_lo(sw1), h2f_lo(mw1), h2f_hi(sw1), h2f_hi(mw1));
        }
      } else {
        for (int k = 0; k < npairs; ++k) {
          const int g = 2 * (p0 + k);
          const bool two = g + 1 < G;
          uint32_t sw = __ldg(srow + g) | (two ? static_cast<uint32_t>(__ldg(srow + g + 1)) << 16 : 0u), mw = sw;
          if (kS8 && (E.fmt & kFmtS8))
            expand(sw, mw);
          else
            mw = __ldg(mins_at(g)) | (two ? static_cast<uint32_t>(__ldg(mins_at(g + 1))) << 16 : 0u);
          step(k, h2f_lo(sw), h2f_lo(mw), two ? h2f_hi(sw) : 0.f, two ? h2f_hi(mw) : 0.f);
        }
      }
      q += npairs;
      // drain this block's last (up to) kNP pairs, oldest first
      const int nd = min(npairs, kNP);
#pragma unroll
      for (int i = 0; i < kNP; ++i) {
        if (i < nd) {
          const int qq = q - nd + i;
          const int b = qq % kNP;
          if (ok) ok = mbar_wait(mdone(s, b), (qq / kNP) & 1, ERR_TC_WAIT);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            mm4::tc_fence_after();
            int d0[4], d1[4];
            tmem_ld4(d_set + b * kDCols, d0);
            tmem_ld4(d_set + b * kDCols + 8, d1);
            tmem_wait_ld4(d0);
            tmem_wait_ld4(d1);
            acc = fmaf(pa[i], dot16(d0), acc);
            acc = fmaf(pb[i], group_dot16(d1), acc);
          }
        }
      }
      // ---- split K: every slice leaves its partial sums; the block's last slice to finish (an atomic ticket)
      // adds them in slice order (the same result whichever slice finishes last) and runs the epilogue
      if (E.ks > 1) {
        p.ws_part[static_cast<int64_t>(gi) * kRows + rib] = acc;
        __threadfence();
        named_bar_sync(2 + s, 128);
        volatile int* last = reinterpret_cast<volatile int*>(aux + 2 * kLnMaxGroups) + s;
        if (rib == 0)
          *last = atomicAdd(p.ws_ticket + E.block_begin + blk, 1u) == static_cast<unsigned int>(E.ks - 1) ? 1 : 0;
        named_bar_sync(2 + s, 128);
        if (!*last) continue;
        __threadfence();
        const float* parts = p.ws_part + static_cast<int64_t>(E.item_begin + blk * E.ks) * kRows + rib;
        acc = 0.f;
#pragma unroll 4
        for (int k = 0; k < E.ks; ++k) acc += __ldcg(parts + k * kRows);
        if (rib == 0) p.ws_ticket[E.block_begin + blk] = 0u;  // ready for the next launch
      }
      // ---- the block's results: stored, or routed as the engine's post kernel would (engine/fused.py:43-84)
      if (E.epi == kEpiStore) {
        if (ok && row_ok) store_out(E.y, row, acc, p.y_bf16);
      } else {
        const EpiP& P = p.epis[E.ep];
        if (E.y && ok && row_ok) store_out(E.y, row, acc, p.y_bf16);
        const float r = round_act(acc, p.y_bf16);               // what the engine's y buffer would hold
        const float pr = __shfl_xor_sync(0xffffffffu, r, 1);    // the partner row (rotary pair / up channel)
        int64_t pos = 0;
        bool pos_ok = true;
        if (E.epi == kEpiRopeKv) {
          pos = *P.pos;
          pos_ok = pos >= 0 && pos < P.S;
          if (!pos_ok && rib == 0) atomicOr(&g_device_error, ERR_ARG);
        }
        if (ok && row_ok && pos_ok) route_row(P, E.epi, row, r, pr, pos, p.y_bf16);
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

}  // namespace g4t

int launch_add_ln(const rb_add_ln* ln, int dtype, int flags, cudaStream_t stream) {
  using namespace g4t;
  Slot S = {};
  S.x = ln->x;
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
  S.ln = 1;
  S.K = static_cast<int>(ln->H);
  S.G = static_cast<int>(ln->H / 128);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kConvWarps * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (flags & RB_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, add_ln_kernel, S, dtype == RB_BF16 ? 1 : 0) == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

namespace g4t {

// Split-K plan of one launch. A converter set finishes about one pair of groups per microsecond, so a launch
// with fewer 128-row blocks than num_sms x kSets sets (a decode layer's projections, 18-35 MB) would leave most
// sets idle; its blocks are cut into slices of about ppk pairs so that about one item per set runs (a multiple
// of 4 pairs where K % 1024 == 0, so that the 8-group scale loads stay aligned). Sets every entry's ks / ppk /
// item_begin and p.total_items, and returns the workspace bytes the plan needs (0 without a split). Without
// that much workspace the launch is not split.
int64_t plan_split(TcParams& p, int num_sms, int64_t ws_bytes) {
  int64_t pairs = 0;
  int maxnp = 1;
  for (int i = 0; i < p.count; ++i) {
    const int np = entry_pairs(p.e[i].G, p.e[i].fmt), nb = (p.e[i].N + kRows - 1) / kRows;
    pairs += static_cast<int64_t>(np) * nb;
    maxnp = std::max(maxnp, np);
  }
  auto assign = [&](int ppk) -> int64_t {
    int items = 0;
    bool split = false;
    for (int i = 0; i < p.count; ++i) {
      Entry& E = p.e[i];
      const int np = entry_pairs(E.G, E.fmt), nb = (E.N + kRows - 1) / kRows;
      const int pk = (E.G & 7) == 0 && !(E.fmt & kFmtW8) ? (ppk + 3) & ~3 : ppk;
      E.ks = pk >= np ? 1 : (np + pk - 1) / pk;
      E.ppk = E.ks == 1 ? np : pk;
      E.item_begin = items;
      items += nb * E.ks;
      split |= E.ks > 1;
    }
    p.total_items = items;
    return split ? split_ticket_bytes(p.total_blocks) + static_cast<int64_t>(items) * kRows * 4 : 0;
  };
  const int64_t sets = static_cast<int64_t>(num_sms) * kSets;
  if (ws_bytes > 0 && p.total_blocks < sets) {
    const int64_t t = std::max<int64_t>(2, (pairs + sets - 1) / sets);
    if (t < maxnp) {
      const int64_t need = assign(static_cast<int>(t));
      if (need <= ws_bytes) return need;
    }
  }
  return assign(maxnp);
}

}  // namespace g4t

int launch_gemv_int4_tc(const rb_gemv_desc* d, int count, int x_dtype, int y_dtype, int flags, int num_sms,
                        cudaStream_t stream, const rb_gemv_epi* epi, const rb_add_ln* ln, void* ws,
                        int64_t ws_bytes, int64_t* query) {
  using namespace g4t;
  if (query) *query = 0;
  constexpr uint32_t kSmemMax = 227 * 1024;
  auto encode = mm4::encode_fn();
  if (!encode) return RB_ERR_DEVICE;
  TcParams p;  // ~27 KB, built on the host and passed by value in the launch
  int done = 0;
  while (done < count) {
    const int n = std::min(count - done, kMaxEntries);
    p.x_bf16 = x_dtype == RB_BF16;
    p.y_bf16 = y_dtype == RB_BF16;
    p.prefetch = (flags & RB_FLAG_PDL) && (flags & RB_FLAG_PREFETCH_WEIGHTS) ? 1 : 0;
    // instruction descriptor: D int32, A unsigned 8-bit, B signed 8-bit, both K-major, N = 8, M = 128 (the int8
    // entries' MMAs add kIdescASigned)
    p.idesc = (2u << 4) | (0u << 7) | (1u << 10) | ((8u >> 3) << 17) | ((static_cast<uint32_t>(kRows) >> 4) << 24);
    const uint32_t kBars = kSets * (2 * kMaxStages + 2 * kNP) * 8 + 16 + 16 + kAuxBytes;
    int nslots = 0, blocks = 0, take = 0, nepis = 0;
    uint32_t x_bytes = 0;
    for (; take < n; ++take) {
      const rb_gemv_desc& D = d[done + take];
      const uint32_t G = static_cast<uint32_t>(D.K / 128);
      const bool from_ln = D.x == nullptr;  // multiplies the prologue's normalised vector
      const int kind = epi ? epi[done + take].kind : kEpiStore;
      if (from_ln && !ln) return RB_ERR_NULL;
      int slot = -1;
      for (int i = 0; i < nslots; ++i)
        if (p.slots[i].ln == (from_ln ? 1 : 0) && (from_ln || p.slots[i].x == D.x) &&
            p.slots[i].K == static_cast<int>(D.K))
          slot = i;
      const uint32_t add_x = slot < 0 ? (G * kXGroupBytes + kXPad + ((G * 8 + 15) & ~15u)) : 0u;
      if (slot < 0 && nslots == kMaxSlots) break;
      if (1024 + kSets * 2 * kStageBytes + x_bytes + add_x + kBars > kSmemMax) break;
      if (kind != kEpiStore && nepis == kMaxEpis) break;
      if (slot < 0) {
        slot = nslots++;
        Slot& S = p.slots[slot];
        S = Slot{};
        S.x = from_ln ? ln->x : D.x;
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
      const bool w8 = D.w8 != RB_W8_NONE;
      if (w8 && kind != kEpiStore) return RB_ERR_SHAPE;  // int8 rows: the store epilogue only
      E.s = D.s;
      E.fmt = w8 ? kFmtW8 | (D.w8 == RB_W8_OFFSET ? kFmtOffset : 0) | (D.s_row ? kFmtRowF32 : 0)
                 : (D.s_row ? kFmtS8 : 0);
      E.m = D.s_row ? static_cast<const void*>(D.s_row) : static_cast<const void*>(D.m);
      E.y = D.y;
      E.N = static_cast<int>(D.N);
      E.G = static_cast<int>(G);
      E.slot = slot;
      E.block_begin = blocks;
      E.epi = kind;
      E.ep = 0;
      if (kind != kEpiStore) {
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
      blocks += static_cast<int>((D.N + kRows - 1) / kRows);
      const int64_t row_bytes = w8 ? D.K : D.K / 2;  // int8 codes [N, K] or packed int4 codes [N, K/2]
      const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(D.N)};
      const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
      const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(kRows)};
      const cuuint32_t es[2] = {1, 1};
      if (encode(&p.maps[take], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(D.q), dims, strides, box, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return RB_ERR_SHAPE;
    }
    if (take == 0) return RB_ERR_SHAPE;
    if ((epi || ln) && take < count) return RB_ERR_SHAPE;  // the fused glue needs the whole list in one launch
    p.count = take;
    p.nslots = nslots;
    p.total_blocks = blocks;
    const int64_t need = plan_split(p, num_sms, query ? INT64_MAX : (ws ? ws_bytes : 0));
    if (query) {
      *query = std::max(*query, need);
      done += take;
      continue;
    }
    p.ws_ticket = static_cast<unsigned int*>(ws);
    p.ws_part = need ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + split_ticket_bytes(blocks)) : nullptr;
    // layout (from a 1024-aligned base): [stages: kSets x nst x 16 KB][activation tables][barriers][tmem slot]
    uint32_t off = 0;
    for (int i = 0; i < nslots; ++i) {
      p.slots[i].tab_off = off;
      off += static_cast<uint32_t>(p.slots[i].G) * kXGroupBytes + kXPad;
      p.slots[i].cst_off = off;
      off += (static_cast<uint32_t>(p.slots[i].G) * 8 + 15) & ~15u;
    }
    const uint32_t xtot = off;
    int nst = static_cast<int>((kSmemMax - 1024 - xtot - kBars) / (kSets * kStageBytes));
    nst = std::min(nst, kMaxStages);
    if (nst < 2) return RB_ERR_SHAPE;
    p.nst = nst;
    p.xs_off = static_cast<uint32_t>(kSets * nst) * kStageBytes;
    p.bar_off = (p.xs_off + xtot + 15) & ~15u;
    p.aux_off = (p.bar_off + kSets * (2 * nst + 2 * kNP) * 8 + 16 + 15) & ~15u;
    const uint32_t smem = 1024 + p.aux_off + kAuxBytes;
    bool any8 = false, anyw8 = false;
    for (int i = 0; i < take; ++i) {
      any8 = any8 || (p.e[i].fmt & kFmtS8);
      anyw8 = anyw8 || (p.e[i].fmt & kFmtW8);
    }
    void (*kern)(TcParams) = any8 ? (anyw8 ? gemv_int4_tc_kernel<true, true> : gemv_int4_tc_kernel<true, false>)
                                  : (anyw8 ? gemv_int4_tc_kernel<false, true> : gemv_int4_tc_kernel<false, false>);
    cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), static_cast<int>(kSmemMax));
    if (e != cudaSuccess) return RB_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(num_sms, std::max(1, p.total_items)));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
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
