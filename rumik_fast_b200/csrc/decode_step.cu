// decode_step.cu - the transformer layers of a decode step as ONE persistent launch on B200 (sm_100a).
//
// rumik-fast runs each decode layer as a chain of launches (engine/rumik_fused.py:97-121): add_ln -> GEMV(w_in)
// -> post (rope, KV write, silu * up) -> attention -> GEMV(w_o), GEMV(w_down). This kernel runs every layer
// of a step in one cooperative launch of one CTA per SM, so the weight stream never stops at a launch boundary:
// a CTA's producer warp keeps streaming the codes of its next work while its converters wait for the data the
// work depends on. Per layer l there are three phases, each a set of int4 group-128 GEMVs on the tcgen05
// tensor cores (the arithmetic of gemv_int4_tc.cu: codes unpacked into tensor memory as the A operand of
// kind::i8 MMAs, activations quantised per 128-column group to 16-bit integers, exact int32 partial dots):
//   A  h = LayerNorm(x + o + d) (every CTA computes it; CTA 0 stores the new residual x), then QKV and gate_up
//      of h; their epilogues rotate q and k and write q, k and v (the cache slot at *pos), and silu(gate) * up;
//   B  the decode attention (the CTA routine of attn.cuh) on one converter set of each of the first
//      n_kv_heads x nsplit CTAs, and down_proj of silu(gate) * up on every other converter set;
//   C  o_proj of the attention output.
// Work is balanced "stream-K": a phase's (block, pair of groups) units are laid out block by block and cut into
// equal contiguous ranges, one per converter set, so a 128-row block can be shared by a few sets; each share
// leaves an fp32 partial and the block's last share (an atomic ticket) adds the shares in order (deterministic)
// and runs the epilogue. Dependencies between phases are release/acquire counters in a workspace: a CTA's
// converter warps meet at the end of each phase, wait (bounded) for the counter the next phase needs, and build
// that phase's activation table. Buffers written per layer alternate between two copies by layer parity, so a
// layer never overwrites what a slower CTA may still be reading from the layer before. Every wait is bounded;
// one that runs out sets a bit in the device error word and an abort flag, and every CTA then skips the rest of
// its work and returns. The last CTA to finish zeroes the counters, so the workspace is ready for the next call.
// No multicast, no clusters.
#include "attn.cuh"
#include "common.cuh"
#include "glue.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace rb {

namespace dstep {

using g4t::kXChunkBytes;
using g4t::kXGroupBytes;

constexpr int kSets = 3;
constexpr int kRows = 128;
constexpr int kConvWarps = 4 * kSets;
constexpr int kFirstConv = 1 + kSets;
constexpr int kThreads = (kFirstConv + kConvWarps) * 32;
constexpr int kConvThreads = kConvWarps * 32;
constexpr uint32_t kStageBytes = kRows * 128;  // one pair of groups (256 columns) of 128 rows
constexpr int kNst = 3;                        // ring stages per set
constexpr int kNP = 2;                         // tensor-memory buffers per set (one pair each)
constexpr uint32_t kACols = 64, kDCols = 16, kSetCols = kNP * (kACols + kDCols);
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kXPad = 256;
constexpr int kMaxLayers = 36;
constexpr int kBarConv = 1;  // named barrier of all converter warps; 2 + s: the four warps of set s
constexpr int kLnIter = 2;   // the prologue's 8-element chunks per converter thread: H <= 2 x 384 x 8 = 6144
constexpr int kRegsIssue = 56, kRegsConv = 152;  // registers per thread of warpgroup 0 / the converter warpgroups
enum : int { kQKV = 0, kGU = 1, kDown = 2, kO = 3 };
enum : int { kPhA = 0, kPhD = 1, kPhO = 2 };
// per-layer counters (workspace words, 8 per layer)
enum : int { kCtrQkv = 0, kCtrAct = 1, kCtrAtt = 2, kCtrOut = 3, kCtrResid = 4 };
constexpr int kCtrPerLayer = 8;

struct LayerP {
  const uint16_t* s[4];
  const uint16_t* m[4];
  const void* ln_w;
  void* kc;
  void* vc;
  int rope;
};

struct __align__(64) DsParams {
  CUtensorMap maps[4 * kMaxLayers];  // codes of QKV, gate_up, down, o per layer: box 128 B x 128 rows, SW128
  LayerP L[kMaxLayers];
  int nl, l0, H, I, nq, nkv, hd;
  int nb[4], np[4];   // 128-row blocks and pairs of groups per block, per entry kind
  int T[3];           // pairs per phase
  int S;              // converter sets in the grid
  int natt, nsplit;   // attention sets (set 0 of CTAs 0 .. natt-1) and splits per key-value head
  int bf16, emb_f16;
  int64_t cache_len, vocab;
  float eps, scale;
  uint32_t idesc;
  const int64_t* pos;
  const void* cos;
  const void* sin;
  const int8_t* emb_q;
  const void* emb_s;
  const int64_t* tok;
  void* resid[2];
  void* q_out[2];
  void* ob[2];
  void* act[2];
  void* bo[2];
  void* bd[2];
  unsigned int* ctr;     // [nl][kCtrPerLayer]
  unsigned int* misc;    // [0] CTAs finished, [1] abort
  unsigned int* ticket;  // per phase block: [nb QKV + nb GU | nb down | nb o]
  unsigned int* att_ticket;
  float* att_po;
  float* att_pm;
  float* att_pl;
  float* part[3];        // split-K partials per phase: [T][128], indexed by the share's first pair
  uint32_t tab[3], cst[3];  // activation tables of h (A), act (D), attention output (C): smem offsets
  uint32_t bar_off, aux_off, att_off;
};
static_assert(sizeof(DsParams) <= 32000, "kernel parameter block too large");

// ---- the static schedule (the same arithmetic in every role) ----
// Participating sets of a phase: all S sets, except in phase D the attention sets.
__device__ __forceinline__ int phase_sets(const DsParams& p, int ph) { return ph == kPhD ? p.S - p.natt : p.S; }
// Rank of converter set sigma (= cta * kSets + s) in phase ph, or -1 when it takes no pairs of the phase.
__device__ __forceinline__ int phase_rank(const DsParams& p, int ph, int sigma) {
  if (ph != kPhD) return sigma;
  if (sigma % kSets == 0 && sigma / kSets < p.natt) return -1;
  return sigma - min(p.natt, (sigma + kSets - 1) / kSets);
}
// First pair of rank rho's range in phase ph (range rho = [first(rho), first(rho + 1))). 32-bit arithmetic: the
// host checks T x S < 2^31.
__device__ __forceinline__ int range_first(const DsParams& p, int ph, int rho) {
  return static_cast<int>(static_cast<unsigned int>(p.T[ph] * rho) / static_cast<unsigned int>(phase_sets(p, ph)));
}
// Rank owning pair t of phase ph.
__device__ __forceinline__ int owner(const DsParams& p, int ph, int t) {
  return static_cast<int>(static_cast<unsigned int>((t + 1) * phase_sets(p, ph) - 1) / static_cast<unsigned int>(p.T[ph]));
}
// The shares of a block whose pairs are [t0, t0 + np): with at least as many pairs as sets in the phase every range
// is non-empty and the block's shares are the ranges of its first to last owner; with fewer, every range holds at
// most one pair and each pair is a share. first_of(k): the first pair of share k.
struct Shares {
  int n, o0, t0, per_pair;
};
__device__ __forceinline__ Shares block_shares(const DsParams& p, int ph, int t0, int np) {
  Shares r;
  r.t0 = t0;
  r.per_pair = p.T[ph] < phase_sets(p, ph);
  r.o0 = owner(p, ph, t0);
  r.n = r.per_pair ? np : owner(p, ph, t0 + np - 1) - r.o0 + 1;
  return r;
}
__device__ __forceinline__ int share_first(const DsParams& p, int ph, const Shares& sh, int k) {
  return sh.per_pair ? sh.t0 + k : max(sh.t0, range_first(p, ph, sh.o0 + k));
}
// Entry kind, block (within the entry), pair (within the block), the block's first pair in the phase, and the
// block's index among the phase's blocks, of pair t of phase ph.
struct PairAt {
  int e, blk, k, t0, gb;
};
__device__ __forceinline__ PairAt pair_at(const DsParams& p, int ph, int t) {
  PairAt r;
  int e0 = ph == kPhA ? kQKV : ph == kPhD ? kDown : kO;
  int base = 0, gbase = 0;
  if (ph == kPhA && t >= p.nb[kQKV] * p.np[kQKV]) {
    base = p.nb[kQKV] * p.np[kQKV];
    gbase = p.nb[kQKV];
    e0 = kGU;
  }
  const int np = p.np[e0];
  r.e = e0;
  r.blk = (t - base) / np;
  r.k = t - base - r.blk * np;
  r.t0 = base + r.blk * np;
  r.gb = gbase + r.blk;
  return r;
}
__device__ __forceinline__ int entry_rows(const DsParams& p, int e) {
  return e == kQKV ? (p.nq + 2 * p.nkv) * p.hd : e == kGU ? 2 * p.I : p.H;
}
__device__ __forceinline__ int ticket_base(const DsParams& p, int ph) {
  return ph == kPhA ? 0 : ph == kPhD ? p.nb[kQKV] + p.nb[kGU] : p.nb[kQKV] + p.nb[kGU] + p.nb[kDown];
}

// ---- waits on the workspace counters ----
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool aborted(const DsParams& p) {
  return *const_cast<volatile unsigned int*>(p.misc + 1) != 0u;
}
__device__ __noinline__ void set_abort(const DsParams& p, unsigned int err) {
  atomicOr(&g_device_error, err);
  atomicExch(p.misc + 1, 1u);
}
// Wait until *c >= target (acquire). False when the launch was aborted or the wait ran out (which aborts it).
__device__ bool wait_count(const DsParams& p, const unsigned int* c, unsigned int target) {
  if (ld_acquire_gpu(c) >= target) return true;
  const unsigned long long t0 = globaltimer_ns(), lim = wait_limit_ns();
  for (;;) {
    if (ld_acquire_gpu(c) >= target) return true;
    if (aborted(p)) return false;
    if (globaltimer_ns() - t0 > lim) {
      set_abort(p, ERR_STEP_WAIT);
      return false;
    }
    __nanosleep(32);
  }
}
// An mbarrier wait that also gives up when another CTA aborted the launch.
__device__ bool mbar_wait_ab(const DsParams& p, uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns(), lim = wait_limit_ns();
  int n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 63) == 0) {
      if (aborted(p)) return false;
      if (globaltimer_ns() - t0 > lim) {
        set_abort(p, ERR_STEP_WAIT);
        return false;
      }
    }
  }
  return true;
}

// A pair's 128 code bytes of one row (two groups, as the swizzled stage holds them) -> the unsigned 8-bit A
// operand: even columns as the code, odd columns as 16 x the code (gemv_int4_tc.cu's layout).
__device__ __forceinline__ void unpack_codes(const uint4* w, uint32_t* o) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      o[c * 8 + t * 2 + 0] = wv[t] & 0x0F0F0F0Fu;
      o[c * 8 + t * 2 + 1] = wv[t] & 0xF0F0F0F0u;
    }
  }
}

// The MMA issuer's wait for a set's converters: between polls it sleeps, so that an idle issuer (a phase boundary,
// the attention) takes no issue slots from the converter warps of its SM sub-partition.
__device__ bool mbar_wait_idle(const DsParams& p, uint64_t* bar, uint32_t parity) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns(), lim = wait_limit_ns();
  for (int n = 1;; ++n) {
    __nanosleep(64);
    if (mbar_test_wait(bar, parity)) return true;
    if ((n & 15) == 0) {
      if (aborted(p)) return false;
      if (globaltimer_ns() - t0 > lim) {
        set_abort(p, ERR_STEP_WAIT);
        return false;
      }
    }
  }
}

// ---- activation tables (the layout of gemv_int4_tc.cu) ----
__device__ void build_plain(const void* src, int K, bool bf, uint8_t* tab, float2* cst, int ct) {
  const int chunks = K / 8;
  for (int base = 0; base < chunks; base += kConvThreads) {
    const int c = base + ct;
    const bool valid = c < chunks;
    float v[8];
    raw_to_f32(valid ? ldg_cg_128(static_cast<const uint8_t*>(src) + static_cast<int64_t>(c) * 16)
                     : make_uint4(0u, 0u, 0u, 0u),
               bf, v);
    g4t::quant_chunk(v, valid, c, tab, cst);
  }
  for (int i = ct; i < static_cast<int>(kXPad / 16); i += kConvThreads)
    reinterpret_cast<uint4*>(tab + (K / 128) * kXGroupBytes)[i] = make_uint4(0u, 0u, 0u, 0u);
}

template <int REP>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ DsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = blockIdx.x;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  constexpr int per_set = 2 * kNst + 2 * kNP;  // full[kNst], empty[kNst], afull[kNP], mdone[kNP]
  auto full = [&](int s, int i) { return bars + s * per_set + i; };
  auto empty = [&](int s, int i) { return bars + s * per_set + kNst + i; };
  auto afull = [&](int s, int b) { return bars + s * per_set + 2 * kNst + b; };
  auto mdone = [&](int s, int b) { return bars + s * per_set + 2 * kNst + kNP + b; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kSets * per_set);
  float* aux = reinterpret_cast<float*>(smem + p.aux_off);  // LN group sums [2][kLnMaxGroups], then flags
  volatile int* last_flag = reinterpret_cast<volatile int*>(aux + 2 * kLnMaxGroups);  // [kSets]
  volatile int* dead_flag = last_flag + kSets;

  if (tid == 0) {
    for (int s = 0; s < kSets; ++s) {
      for (int i = 0; i < kNst; ++i) {
        mbar_init(full(s, i), 1);
        mbar_init(empty(s, i), 4);
      }
      for (int b = 0; b < kNP; ++b) {
        mbar_init(afull(s, b), 4);
        mbar_init(mdone(s, b), 1);
      }
    }
    *dead_flag = 0;
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
  // Register split: warpgroup 0 (producer + MMA issuers) gives registers to the three converter warpgroups. The
  // shares add up to the launch's 128 per thread: 4 x 32 x kRegsIssue + 12 x 32 x kRegsConv = 512 x 128.
  // Each role's code sits inside the branch that sets its limit, so that the compiler allocates it accordingly.
  static_assert(4 * 32 * kRegsIssue + kConvWarps * 32 * kRegsConv == kThreads * 128, "register split");
  // the token's position: every CTA makes the same decision, so an invalid one skips the whole launch
  const int64_t pos = __ldcg(p.pos);
  const bool pos_ok = pos >= 0 && pos < p.cache_len;
  if (!pos_ok && tid == 0 && cta == 0) atomicOr(&g_device_error, ERR_ARG);

  if (warp < kFirstConv) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsIssue));
  if (!pos_ok) {
    // nothing to do
  } else if (warp == 0) {
    // ---------------- producer: the codes of every set's pairs, in each set's order ----------------
    if (lane == 0) {
      int l[kSets] = {0, 0, 0}, ph[kSets] = {0, 0, 0}, t[kSets] = {0, 0, 0}, t1[kSets] = {0, 0, 0};
      int issued[kSets] = {0, 0, 0};
      bool live[kSets] = {false, false, false};
      auto open = [&](int s) {  // move set s to its next non-empty range at or after (l, ph)
        const int sigma = cta * kSets + s;
        while (l[s] < p.nl) {
          const int rho = phase_rank(p, ph[s], sigma);
          if (rho >= 0) {
            t[s] = range_first(p, ph[s], rho);
            t1[s] = range_first(p, ph[s], rho + 1);
            if (t[s] < t1[s]) return;
          }
          if (++ph[s] == 3) {
            ph[s] = 0;
            ++l[s];
          }
        }
      };
#pragma unroll
      for (int s = 0; s < kSets; ++s) {
        l[s] = 0;
        ph[s] = 0;
        issued[s] = 0;
        open(s);
        live[s] = l[s] < p.nl;
      }
      unsigned long long idle_since = 0;
      int spins = 0;
      bool ok = true;
      while (ok && (live[0] || live[1] || live[2])) {
        bool progress = false;
#pragma unroll
        for (int s = 0; s < kSets; ++s) {
          if (!live[s]) continue;
          const int slot = issued[s] % kNst;
          // non-blocking: a full ring (a set waiting for its phase's inputs) must not hold up the others
          if (issued[s] >= kNst && !mbar_test_wait(empty(s, slot), ((issued[s] / kNst) - 1) & 1)) continue;
          const PairAt a = pair_at(p, ph[s], t[s]);
          mbar_arrive_expect_tx(full(s, slot), kStageBytes);
          mm4::tma_load_2d(smem + (static_cast<size_t>(s) * kNst + slot) * kStageBytes, &p.maps[4 * l[s] + a.e],
                           a.k * 128, a.blk * kRows, full(s, slot));
          ++issued[s];
          progress = true;
          if (++t[s] == t1[s]) {
            if (++ph[s] == 3) {
              ph[s] = 0;
              ++l[s];
            }
            open(s);
            live[s] = l[s] < p.nl;
          }
        }
        // no set had ring space: bounded by the wait limit without progress, and by the abort flag
        if (progress) {
          idle_since = 0;
        } else {
          // every ring full: sleep rather than poll, so that this warp takes no issue slots from the converter
          // warps of its SM sub-partition (a stage takes about a microsecond to consume)
          __nanosleep(128);
        }
        if (!progress && (++spins & 15) == 0) {
          if (aborted(p)) ok = false;
          const unsigned long long now = globaltimer_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > wait_limit_ns()) {
            set_abort(p, ERR_STEP_WAIT);
            ok = false;
          }
        }
      }
      // no retirement with copies in flight
      for (int s = 0; s < kSets; ++s)
        for (int u = max(0, issued[s] - kNst); u < issued[s]; ++u)
          if (!mbar_wait(full(s, u % kNst), (u / kNst) & 1, ERR_STEP_WAIT)) break;
    }
  } else if (warp < kFirstConv) {
    // ---------------- MMA issuer of set s: eight kind::i8 MMAs per pair ----------------
    const int s = warp - 1;
    if (lane == 0) {
      const int sigma = cta * kSets + s;
      int q = 0;
      bool ok = true;
      for (int l = 0; l < p.nl && ok; ++l) {
        for (int ph = 0; ph < 3 && ok; ++ph) {
          const int rho = phase_rank(p, ph, sigma);
          if (rho < 0) continue;
          const int ta = range_first(p, ph, rho), tb = range_first(p, ph, rho + 1);
          const uint32_t xtab = smem_u32(smem + p.tab[ph]);
          for (int t = ta; t < tb; ++t, ++q) {
            const int b = q % kNP;
            if (!mbar_wait_idle(p, afull(s, b), (q / kNP) & 1)) {
              ok = false;
              break;
            }
            mm4::tc_fence_after();
            const PairAt a = pair_at(p, ph, t);
            const uint32_t acol = s * kSetCols + b * kACols, dcol = s * kSetCols + kNP * kACols + b * kDCols;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int i = 0; i < 4; ++i)
                g4t::umma_ts(tmem + dcol + 8 * h, tmem + acol + 32 * h + 8 * i,
                             g4t::x_desc(xtab + (2 * a.k + h) * kXGroupBytes + 2 * kXChunkBytes * i), p.idesc, i > 0);
            mm4::umma_commit(mdone(s, b));
          }
        }
      }
      if (q > 0) (void)mbar_wait_ab(p, mdone(s, (q - 1) % kNP), ((q - 1) / kNP) & 1);  // no MMA in flight at exit
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsConv));
  if (pos_ok) {
    // ---------------- converters, epilogues, tables and attention ----------------
    const int ct = tid - kFirstConv * 32;  // 0 .. kConvThreads - 1
    const int cw = warp - kFirstConv;
    const int s = cw >> 2;
    const int quad = warp & 3;
    const int rib = quad * 32 + lane;      // row in block = tensor-memory lane
    const int sigma = cta * kSets + s;
    const bool bf = p.bf16 != 0;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t a_set = tq + s * kSetCols, d_set = tq + s * kSetCols + kNP * kACols;
    const int sbar = 2 + s;
    bool dead = false;
    int q = 0, st = 0;  // pairs of this set so far (tensor-memory buffer q % kNP), ring stages consumed
    // The two pairs whose results are pending (issued, not read yet), older first: sa / sb = scale * delta / 16 of
    // their two groups, mt = their min terms; `last`: the pair ends its segment (share) [t, t1). Results are read
    // in pair order, so one accumulator holds the segment being read; a phase ends with a drain, so rd_l / rd_ph
    // (the layer and phase of the pending pairs) are per phase.
    struct Pend {
      float sa, sb, mt;
      int last, t, t1;
    };
    Pend po = {0.f, 0.f, 0.f, 0, 0, 0}, pn = po;
    int npend = 0, rd_l = 0, rd_ph = 0;
    float acc = 0.f;

    // The end of a share [t, t1) of phase ph in layer l with sum r: the row's result (a whole block), or an fp32
    // partial whose block's last share adds all shares in order. Then the epilogue and the block's completion count.
    auto finalize = [&](int l, int ph, int t, int t1, float r) {
      const PairAt a = pair_at(p, ph, t);
      const int np = p.np[a.e];
      const int N = entry_rows(p, a.e);
      const int row = a.blk * kRows + rib;
      const bool row_ok = row < N;
      bool have = true;
      if (!(t == a.t0 && t1 == a.t0 + np)) {  // shared block
        // Every thread stores its partial; the barrier orders those stores before thread 0's acq_rel ticket add
        // (which releases them at GPU scope), and the last share's loads follow its acquire through the barrier.
        p.part[ph][static_cast<int64_t>(t) * kRows + rib] = r;
        const Shares sh = block_shares(p, ph, a.t0, np);
        named_bar_sync(sbar, 128);
        if (rib == 0) {
          unsigned int prev;
          asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                       : "=r"(prev)
                       : "l"(p.ticket + ticket_base(p, ph) + a.gb)
                       : "memory");
          last_flag[s] = prev == static_cast<unsigned int>(sh.n - 1) ? 1 : 0;
        }
        named_bar_sync(sbar, 128);
        have = last_flag[s] != 0;
        if (have) {
          r = 0.f;
          for (int k = 0; k < sh.n; ++k)  // the shares in pair order, each stored at its first pair
            r += __ldcg(p.part[ph] + static_cast<int64_t>(share_first(p, ph, sh, k)) * kRows + rib);
          if (rib == 0) p.ticket[ticket_base(p, ph) + a.gb] = 0u;  // ready for the next layer
        }
      }
      if (!have) return;
      const int par = (p.l0 + l) & 1;
      if (a.e == kQKV || a.e == kGU) {
        EpiP P;
        P.pos = p.pos;
        P.cos = p.cos;
        P.sin = p.sin;
        P.q_out = p.q_out[par];
        P.k_cache = p.L[l].kc;
        P.v_cache = p.L[l].vc;
        P.act = p.act[par];
        P.S = p.cache_len;
        P.rope = p.L[l].rope;
        P.nq = p.nq;
        P.nkv = p.nkv;
        P.hd = p.hd;
        const float rr = round_act(r, bf);
        const float pr = __shfl_xor_sync(0xffffffffu, rr, 1);  // rotary pair / up channel
        if (row_ok && !dead) route_row(P, a.e == kQKV ? RB_EPI_ROPE_KV : RB_EPI_SWIGLU, row, rr, pr, pos, bf);
      } else if (row_ok && !dead) {
        store_out(a.e == kDown ? p.bd[par] : p.bo[par], row, r, bf);
      }
      named_bar_sync(sbar, 128);  // every row stored: the release below publishes them (barrier cumulativity)
      if (rib == 0) {
        const int c = a.e == kQKV ? kCtrQkv : a.e == kGU ? kCtrAct : kCtrOut;
        red_release_gpu(p.ctr + l * kCtrPerLayer + c, 1u);
      }
    };

    // Results of pending pair e, in tensor-memory buffer b and issued as this set's pair qq: its two groups'
    // accumulators into the segment sum; the segment's last pair finalizes it.
    auto read_pair = [&](const Pend& e, int b, uint32_t qq) {
      int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};
      bool ok = !dead && mbar_wait_ab(p, mdone(s, b), (qq / kNP) & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        mm4::tc_fence_after();
        g4t::tmem_ld4(d_set + b * kDCols, d0);
        g4t::tmem_ld4(d_set + b * kDCols + 8, d1);
        g4t::tmem_wait_ld4(d0);
        g4t::tmem_wait_ld4(d1);
      } else {
        dead = true;
      }
      acc += e.mt + e.sa * g4t::group_dot16(d0) + e.sb * g4t::group_dot16(d1);
      if (e.last) {
        finalize(rd_l, rd_ph, e.t, e.t1, acc);
        acc = 0.f;
      }
    };

    // Drain: every pending pair's results, oldest first.
    auto drain = [&]() {
      if (npend >= 1) read_pair(po, (q - npend) % kNP, static_cast<uint32_t>(q - npend));
      if (npend == 2) read_pair(pn, (q - 1) % kNP, static_cast<uint32_t>(q - 1));
      npend = 0;
    };

    // The set's pairs [ta, tb) of phase ph in layer l.
    auto run_pairs = [&](int l, int ph, int ta, int tb) {
      const float2* cst = reinterpret_cast<const float2*>(smem + p.cst[ph]);
      rd_l = l;
      rd_ph = ph;
      uint4 wn[8];
      auto load_codes = [&]() {
        const int slot = st % kNst;
        bool ok = !dead && mbar_wait_ab(p, full(s, slot), (st / kNst) & 1);
        if (!__all_sync(0xffffffffu, ok)) {
          dead = true;
          return;
        }
        const uint8_t* rowp = smem + (static_cast<size_t>(s) * kNst + slot) * kStageBytes + rib * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) wn[c] = lds128(rowp + ((c ^ (rib & 7)) << 4));
      };
      // the scale and min words of pair t (two groups each) of this thread's row; loaded a pair ahead
      auto scale_words = [&](int t, uint32_t& sw, uint32_t& mw) {
        const PairAt a = pair_at(p, ph, t);
        const int G = p.np[a.e] * 2;
        const int row = a.blk * kRows + rib;
        const int64_t off = static_cast<int64_t>(row < entry_rows(p, a.e) ? row : 0) * G + 2 * a.k;
        sw = __ldg(reinterpret_cast<const uint32_t*>(p.L[l].s[a.e] + off));
        mw = __ldg(reinterpret_cast<const uint32_t*>(p.L[l].m[a.e] + off));
      };
      uint32_t sw_n = 0u, mw_n = 0u;
      if (ta < tb) {
        scale_words(ta, sw_n, mw_n);
        load_codes();
      }
      int seg_t = ta;
      for (int t = ta; t < tb; ++t) {
        const PairAt a = pair_at(p, ph, t);
        const uint32_t sw = sw_n, mw = mw_n;
        if (t + 1 < tb) scale_words(t + 1, sw_n, mw_n);
        const uint4 w[8] = {wn[0], wn[1], wn[2], wn[3], wn[4], wn[5], wn[6], wn[7]};
        __syncwarp();
        if (lane == 0 && !dead) mbar_arrive(empty(s, st % kNst));  // both groups of this stage are in registers
        ++st;
        const int b = q % kNP;
        // the pair kNP back used buffer b: its results first (this may finish its segment)
        if (npend == kNP) {
          read_pair(po, b, static_cast<uint32_t>(q - kNP));
          po = pn;
          npend = 1;
        }
        if (a.k == 0) seg_t = t;  // a block's first pair starts a new segment (so does the range's first pair)
        const float2 ca = cst[2 * a.k], cb = cst[2 * a.k + 1];
        Pend e;
        e.sa = g4t::h2f_lo(sw) * ca.x;
        e.sb = g4t::h2f_hi(sw) * cb.x;
        e.mt = g4t::h2f_lo(mw) * ca.y + g4t::h2f_hi(mw) * cb.y;
        e.t = seg_t;
        e.t1 = min(tb, a.t0 + p.np[a.e]);
        e.last = t + 1 == e.t1;
        if (npend == 0)
          po = e;
        else
          pn = e;
        ++npend;
        if (!dead) {
          uint32_t o[32];
          unpack_codes(w, o);
          g4t::tmem_st32(a_set + b * kACols, o);
          unpack_codes(w + 4, o);
          g4t::tmem_st32(a_set + b * kACols + 32, o);
        }
        if (t + 1 < tb) load_codes();  // overlaps the tensor-memory traffic above
        if (!dead) {
          g4t::tmem_wait_st();
          mm4::tc_fence_before();
        }
        __syncwarp();
        if (lane == 0 && !dead) mbar_arrive(afull(s, b));
        ++q;
      }
    };

    // The converter warps of the CTA meet; ct 0 waits for `c` >= target (if c); all then build a table.
    auto meet = [&](const unsigned int* c, unsigned int target, const unsigned int* c2, unsigned int target2) {
      drain();
      named_bar_sync(kBarConv, kConvThreads);
      if (ct == 0) {
        bool ok = !dead && !aborted(p);
        if (ok && c) ok = wait_count(p, c, target);
        if (ok && c2) ok = wait_count(p, c2, target2);
        *dead_flag = ok ? 0 : 1;
      }
      named_bar_sync(kBarConv, kConvThreads);
      dead = dead || *dead_flag != 0;
    };

    const int GH = p.H / 128;
    for (int l = 0; l < p.nl; ++l) {
      const int g = p.l0 + l, par = g & 1;
      unsigned int* ctr = p.ctr + l * kCtrPerLayer;
      // ---- phase A: h = LayerNorm(x + o + d) (or the token's embedding row), QKV and gate_up ----
      if (l == 0)
        meet(nullptr, 0, nullptr, 0);
      else
        meet(ctr - kCtrPerLayer + kCtrOut, p.nb[kO] + p.nb[kDown], ctr - kCtrPerLayer + kCtrResid, 1);
      if (!dead) {
        LnSrc S;
        S.w = p.L[l].ln_w;
        S.x_out = p.resid[par];
        S.h_out = nullptr;
        S.eps = p.eps;
        S.K = p.H;
        S.emb_q = nullptr;
        S.emb_s = nullptr;
        S.tok = nullptr;
        S.vocab = 0;
        S.emb_f16 = 0;
        S.x = S.a = S.b = nullptr;
        if (g == 0) {
          S.emb_q = p.emb_q;
          S.emb_s = p.emb_s;
          S.tok = p.tok;
          S.vocab = p.vocab;
          S.emb_f16 = p.emb_f16;
        } else {
          S.x = p.resid[par ^ 1];
          S.a = p.bo[par ^ 1];
          S.b = p.bd[par ^ 1];
        }
        uint8_t* tab = smem + p.tab[kPhA];
        float2* cstp = reinterpret_cast<float2*>(smem + p.cst[kPhA]);
        stage_ln<kLnIter>(S, bf, aux, kBarConv, ct, kConvThreads, cta == 0,
                               [&](const float (&h)[8], bool valid, int c) { g4t::quant_chunk(h, valid, c, tab, cstp); });
        for (int i = ct; i < static_cast<int>(kXPad / 16); i += kConvThreads)
          reinterpret_cast<uint4*>(tab + GH * kXGroupBytes)[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      named_bar_sync(kBarConv, kConvThreads);
      if (cta == 0 && ct == 0 && !dead) {  // the new residual is stored: publish it to the next layer's prologue
        __threadfence();
        red_release_gpu(ctr + kCtrResid, 1u);
      }
      {
        const int rho = phase_rank(p, kPhA, sigma);
        run_pairs(l, kPhA, range_first(p, kPhA, rho), range_first(p, kPhA, rho + 1));
      }
      // ---- phase B: the table of silu(gate) * up; down_proj, or the attention on an attention set ----
      meet(ctr + kCtrAct, p.nb[kGU], nullptr, 0);
      if (!dead)
        build_plain(p.act[par], p.I, bf, smem + p.tab[kPhD], reinterpret_cast<float2*>(smem + p.cst[kPhD]), ct);
      fence_proxy_async_smem();
      named_bar_sync(kBarConv, kConvThreads);
      const int rhoD = phase_rank(p, kPhD, sigma);
      if (rhoD >= 0) {
        run_pairs(l, kPhD, range_first(p, kPhD, rhoD), range_first(p, kPhD, rhoD + 1));
      } else {
        // attention unit cta = (key-value head, split): q, k and v of this layer must all be written
        if (rib == 0) *(last_flag + s) = (!dead && wait_count(p, ctr + kCtrQkv, p.nb[kQKV])) ? 1 : 0;
        named_bar_sync(sbar, 128);
        if (last_flag[s] == 0) {
          dead = true;
        } else {
          attn::AttnParams ap;
          ap.q = p.q_out[par];
          ap.kc = p.L[l].kc;
          ap.vc = p.L[l].vc;
          ap.pos = p.pos;
          ap.out = p.ob[par];
          ap.ticket = p.att_ticket;
          ap.po = p.att_po;
          ap.pm = p.att_pm;
          ap.pl = p.att_pl;
          ap.heads_done = ctr + kCtrAtt;
          ap.S = p.cache_len;
          ap.scale = p.scale;
          ap.nsplit = p.nsplit;
          ap.bf16 = p.bf16;
          float* sa = reinterpret_cast<float*>(smem + p.att_off);
          attn::attn_cta<REP, true, true>(ap, cta / p.nsplit, cta % p.nsplit, rib, sbar,
                                          reinterpret_cast<float(*)[REP]>(sa),
                                          reinterpret_cast<float(*)[REP]>(sa + attn::kWarps * REP),
                                          reinterpret_cast<float(*)[REP][attn::kHd]>(sa + 2 * attn::kWarps * REP),
                                          reinterpret_cast<int*>(sa + 2 * attn::kWarps * REP +
                                                                 attn::kWarps * REP * attn::kHd));
        }
      }
      // ---- phase C: the attention output's table; o_proj ----
      meet(ctr + kCtrAtt, p.nkv, nullptr, 0);
      if (!dead)
        build_plain(p.ob[par], p.nq * p.hd, bf, smem + p.tab[kPhO], reinterpret_cast<float2*>(smem + p.cst[kPhO]),
                    ct);
      fence_proxy_async_smem();
      named_bar_sync(kBarConv, kConvThreads);
      {
        const int rho = phase_rank(p, kPhO, sigma);
        run_pairs(l, kPhO, range_first(p, kPhO, rho), range_first(p, kPhO, rho + 1));
      }
    }
    drain();
  }
  }

  mm4::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mm4::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  // the last CTA to finish zeroes the counters for the next launch (which starts after this one completes)
  if (tid == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(p.misc, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      for (int i = 0; i < p.nl * kCtrPerLayer; ++i) p.ctr[i] = 0u;
      // tickets are zero after a complete launch; an aborted one may leave some set
      const int nt = p.nb[kQKV] + p.nb[kGU] + p.nb[kDown] + p.nb[kO];
      for (int i = 0; i < nt; ++i) p.ticket[i] = 0u;
      for (int i = 0; i < p.nkv; ++i) p.att_ticket[i] = 0u;
      p.misc[1] = 0u;
      p.misc[0] = 0u;
    }
  }
}

}  // namespace dstep
}  // namespace rb

namespace rb {

namespace dstep {

struct WsLayout {
  int64_t ctr, misc, ticket, att, part[3], total;
};

inline WsLayout ws_layout(int nl, int nblocks, int nq, int nkv, const int (&T)[3]) {
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  WsLayout w;
  w.ctr = 0;
  w.misc = up(static_cast<int64_t>(nl) * kCtrPerLayer * 4);
  w.ticket = w.misc + 256;
  w.att = w.ticket + up(static_cast<int64_t>(nblocks) * 4);
  int64_t off = w.att + up(attn_decode_workspace(nq, nkv, attn::kHd));
  for (int ph = 0; ph < 3; ++ph) {
    w.part[ph] = off;
    off += up(static_cast<int64_t>(T[ph]) * kRows * 4);
  }
  w.total = off;
  return w;
}

}  // namespace dstep

// Validation and the plan of a call; fills p (all but the tensor maps) when given. Returns an rb_status, or the
// workspace bytes through *ws_need.
static int decode_plan(const rb_decode_step* d, int num_sms, dstep::DsParams* p, dstep::WsLayout* wl) {
  using namespace dstep;
  if (!d || !d->layers) return RB_ERR_NULL;
  if (d->n_layers < 1 || d->n_layers > kMaxLayers || d->first_layer < 0) return RB_ERR_SHAPE;
  if (d->head_dim != attn::kHd || d->n_kv_heads < 1 || d->n_q_heads % d->n_kv_heads != 0) return RB_ERR_SHAPE;
  const int rep = d->n_q_heads / d->n_kv_heads;
  if (rep < 1 || rep > 4 || d->n_kv_heads > attn::kMaxKv) return RB_ERR_SHAPE;
  const int64_t H = d->H, I = d->I, QD = static_cast<int64_t>(d->n_q_heads) * d->head_dim;
  if (H < 256 || H % 256 || H > kLnIter * kConvThreads * 8 || I < 256 || I % 256 || I > 16384 || QD % 256 || QD > 16384)
    return RB_ERR_SHAPE;
  if (d->cache_len < 1 || d->cache_len > (int64_t(1) << 31) || !(d->eps >= 0.f)) return RB_ERR_SHAPE;
  int nb[4], np[4];
  nb[kQKV] = static_cast<int>(((d->n_q_heads + 2 * d->n_kv_heads) * d->head_dim + kRows - 1) / kRows);
  nb[kGU] = static_cast<int>((2 * I + kRows - 1) / kRows);
  nb[kDown] = static_cast<int>((H + kRows - 1) / kRows);
  nb[kO] = nb[kDown];
  np[kQKV] = np[kGU] = static_cast<int>(H / 256);
  np[kDown] = static_cast<int>(I / 256);
  np[kO] = static_cast<int>(QD / 256);
  int T[3] = {nb[kQKV] * np[kQKV] + nb[kGU] * np[kGU], nb[kDown] * np[kDown], nb[kO] * np[kO]};
  const int S = num_sms * kSets;
  const int nsplit = static_cast<int>(std::min<int64_t>(attn::nsplit_for(d->n_kv_heads, num_sms), num_sms / d->n_kv_heads));
  const int natt = d->n_kv_heads * nsplit;
  if (nsplit < 1 || natt > num_sms) return RB_ERR_SHAPE;
  // every set takes pairs in phase A and every non-attention set in phase D: what makes the per-parity buffers
  // safe to reuse two layers later (the module comment)
  if (T[kPhA] < S || T[kPhD] < S - natt) return RB_ERR_SHAPE;
  for (int ph = 0; ph < 3; ++ph)  // the kernel's schedule arithmetic is 32-bit
    if (static_cast<int64_t>(T[ph] + 1) * S >= (int64_t(1) << 31)) return RB_ERR_SHAPE;
  *wl = ws_layout(d->n_layers, nb[0] + nb[1] + nb[2] + nb[3], d->n_q_heads, d->n_kv_heads, T);
  if (!p) return RB_OK;
  for (int i = 0; i < 4; ++i) {
    p->nb[i] = nb[i];
    p->np[i] = np[i];
  }
  for (int i = 0; i < 3; ++i) p->T[i] = T[i];
  p->nl = d->n_layers;
  p->l0 = d->first_layer;
  p->H = static_cast<int>(H);
  p->I = static_cast<int>(I);
  p->nq = d->n_q_heads;
  p->nkv = d->n_kv_heads;
  p->hd = d->head_dim;
  p->S = S;
  p->natt = natt;
  p->nsplit = nsplit;
  p->cache_len = d->cache_len;
  p->vocab = d->vocab;
  p->eps = d->eps;
  p->scale = d->attn_scale;
  return RB_OK;
}

int64_t decode_layers_workspace(const rb_decode_step* d, int num_sms) {
  dstep::WsLayout wl;
  const int st = decode_plan(d, num_sms, nullptr, &wl);
  return st == RB_OK ? wl.total : -st;
}

int launch_decode_layers(const rb_decode_step* d, int dtype, int flags, int num_sms, cudaStream_t stream) {
  using namespace dstep;
  (void)flags;
  static DsParams p;  // ~23 KB: built on the host per call, passed by value in the launch
  static std::mutex lock;
  std::lock_guard<std::mutex> hold(lock);
  WsLayout wl;
  int st = decode_plan(d, num_sms, &p, &wl);
  if (st != RB_OK) return st;
  if (!d->ws || d->ws_bytes < wl.total) return RB_ERR_SHAPE;
  if (!d->pos || !d->cos || !d->sin) return RB_ERR_NULL;
  if (d->first_layer == 0 && (!d->emb_q || !d->emb_s || !d->tok || d->vocab < 1)) return RB_ERR_NULL;
  if (d->first_layer == 0 && d->emb_s_dtype != RB_F32 && d->emb_s_dtype != RB_F16) return RB_ERR_DTYPE;
  for (int i = 0; i < 2; ++i)
    if (!d->resid[i] || !d->q_out[i] || !d->attn_out[i] || !d->act[i] || !d->o_out[i] || !d->down_out[i])
      return RB_ERR_NULL;
  auto encode = mm4::encode_fn();
  if (!encode) return RB_ERR_DEVICE;
  p.bf16 = dtype == RB_BF16;
  p.emb_f16 = d->emb_s_dtype == RB_F16;
  p.idesc = (2u << 4) | (0u << 7) | (1u << 10) | ((8u >> 3) << 17) | ((static_cast<uint32_t>(kRows) >> 4) << 24);
  p.pos = d->pos;
  p.cos = d->cos;
  p.sin = d->sin;
  p.emb_q = d->emb_q;
  p.emb_s = d->emb_s;
  p.tok = d->tok;
  for (int i = 0; i < 2; ++i) {
    p.resid[i] = d->resid[i];
    p.q_out[i] = d->q_out[i];
    p.ob[i] = d->attn_out[i];
    p.act[i] = d->act[i];
    p.bo[i] = d->o_out[i];
    p.bd[i] = d->down_out[i];
  }
  uint8_t* w = static_cast<uint8_t*>(d->ws);
  p.ctr = reinterpret_cast<unsigned int*>(w + wl.ctr);
  p.misc = reinterpret_cast<unsigned int*>(w + wl.misc);
  p.ticket = reinterpret_cast<unsigned int*>(w + wl.ticket);
  p.att_ticket = reinterpret_cast<unsigned int*>(w + wl.att);
  p.att_po = reinterpret_cast<float*>(w + wl.att + attn::kTicketBytes);
  p.att_pm = p.att_po + static_cast<int64_t>(d->n_q_heads) * p.nsplit * attn::kHd;
  p.att_pl = p.att_pm + static_cast<int64_t>(d->n_q_heads) * p.nsplit;
  for (int ph = 0; ph < 3; ++ph) p.part[ph] = reinterpret_cast<float*>(w + wl.part[ph]);
  const int64_t Ns[4] = {static_cast<int64_t>(d->n_q_heads + 2 * d->n_kv_heads) * d->head_dim, 2 * d->I, d->H, d->H};
  const int64_t Ks[4] = {d->H, d->H, d->I, static_cast<int64_t>(d->n_q_heads) * d->head_dim};
  for (int l = 0; l < d->n_layers; ++l) {
    const rb_decode_layer& Ly = d->layers[l];
    const rb_gemv_desc* g[4] = {&Ly.qkv, &Ly.gate_up, &Ly.down, &Ly.o_proj};
    if (!Ly.ln_w || !Ly.k_cache || !Ly.v_cache) return RB_ERR_NULL;
    for (int e = 0; e < 4; ++e) {
      if (!g[e]->q || !g[e]->s || !g[e]->m) return RB_ERR_NULL;
      if (g[e]->s_row || g[e]->w8 != RB_W8_NONE) return RB_ERR_SHAPE;  // int4 codes with fp16 scales only
      if (g[e]->N != Ns[e] || g[e]->K != Ks[e]) return RB_ERR_SHAPE;
      if ((reinterpret_cast<uintptr_t>(g[e]->q) | reinterpret_cast<uintptr_t>(g[e]->s) |
           reinterpret_cast<uintptr_t>(g[e]->m)) & 15u)
        return RB_ERR_ALIGN;
      p.L[l].s[e] = g[e]->s;
      p.L[l].m[e] = g[e]->m;
      const cuuint64_t dims[2] = {static_cast<cuuint64_t>(Ks[e] / 2), static_cast<cuuint64_t>(Ns[e])};
      const cuuint64_t strides[1] = {static_cast<cuuint64_t>(Ks[e] / 2)};
      const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(kRows)};
      const cuuint32_t es[2] = {1, 1};
      if (encode(&p.maps[4 * l + e], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(g[e]->q), dims, strides,
                 box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return RB_ERR_SHAPE;
    }
    p.L[l].ln_w = Ly.ln_w;
    p.L[l].kc = Ly.k_cache;
    p.L[l].vc = Ly.v_cache;
    p.L[l].rope = Ly.rope;
  }
  // shared memory: [rings][tables h | act | attention output][barriers, tmem slot][LN sums, flags][attention]
  constexpr uint32_t kSmemMax = 227 * 1024;
  uint32_t off = static_cast<uint32_t>(kSets * kNst) * kStageBytes;
  const int Gs[3] = {p.H / 128, p.I / 128, p.nq * p.hd / 128};
  for (int ph = 0; ph < 3; ++ph) {
    p.tab[ph] = off;
    off += static_cast<uint32_t>(Gs[ph]) * kXGroupBytes + kXPad;
    p.cst[ph] = off;
    off += (static_cast<uint32_t>(Gs[ph]) * 8 + 15) & ~15u;
  }
  p.bar_off = off;
  off += kSets * (2 * kNst + 2 * kNP) * 8 + 16;
  p.aux_off = (off + 15) & ~15u;
  off = p.aux_off + 2 * kLnMaxGroups * 4 + 32;
  const int rep = d->n_q_heads / d->n_kv_heads;
  p.att_off = (off + 15) & ~15u;
  off = p.att_off + static_cast<uint32_t>(2 * attn::kWarps * rep + attn::kWarps * rep * attn::kHd + 4) * 4;
  const uint32_t smem = 1024 + off;
  if (smem > kSmemMax) return RB_ERR_SHAPE;
  void (*kern)(DsParams) = nullptr;
  switch (rep) {
    case 1: kern = decode_step_kernel<1>; break;
    case 2: kern = decode_step_kernel<2>; break;
    case 3: kern = decode_step_kernel<3>; break;
    case 4: kern = decode_step_kernel<4>; break;
    default: return RB_ERR_SHAPE;
  }
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), static_cast<int>(kSmemMax));
  if (e != cudaSuccess) return RB_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: they wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  return e == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

}  // namespace rb
