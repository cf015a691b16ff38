// attn.cuh - decode attention of one token over the KV cache (grouped-query heads): the CTA-level routine shared
// by the standalone kernel (attn_decode.cu) and the attention phase fused into the warp-MMA GEMV launch of a
// layer's o_proj / down_proj (gemv_int4_multi.cu). rumik-fast's decode attention: engine/fused.py:92-200.
#pragma once

#include "common.cuh"

namespace rb {

namespace attn {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kHd = 128;       // head_dim: 4 dimensions per lane
constexpr int kStep = 8;       // slots per warp step
constexpr int kMaxRep = 8;
constexpr int kMaxSplit = 64;
constexpr int kMaxKv = 64;
// workspace: per key-value head completion counters, then (fused use) the heads-done and passed counters, then
// the partials
constexpr int64_t kTicketBytes = 512;
constexpr int64_t kHeadsDoneOff = kMaxKv * 4, kPassedOff = kMaxKv * 4 + 4;

struct AttnParams {
  const void* q;
  const void* kc;
  const void* vc;
  const int64_t* pos;
  void* out;
  unsigned int* ticket;  // [n_kv_heads], zero between calls
  float* po;             // [n_q_heads, nsplit, 128] partial accumulators
  float* pm;             // [n_q_heads, nsplit] partial maxima
  float* pl;             // [n_q_heads, nsplit] partial sums
  unsigned int* heads_done;  // fused use: key-value heads whose outputs are written (null: standalone)
  int64_t S;
  float scale;
  int nsplit, bf16;
  // standalone kernel only: issue the position load and the K/V rows of slots before the position ahead of the
  // dependency wait (griddepcontrol.wait); only q and the position's own slot wait for the preceding kernel
  int pre;
};

__device__ __forceinline__ void unpack4(uint2 u, bool bf, float (&f)[4]) {
  if (bf) {
    f[0] = __uint_as_float(u.x << 16);
    f[1] = __uint_as_float(u.x & 0xffff0000u);
    f[2] = __uint_as_float(u.y << 16);
    f[3] = __uint_as_float(u.y & 0xffff0000u);
  } else {
    f[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(u.x & 0xffffu)));
    f[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(u.x >> 16)));
    f[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(u.y & 0xffffu)));
    f[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(u.y >> 16)));
  }
}

// Sum of s[j] over the 32 lanes for 8 values at once: afterwards lane l holds the sum for slot j = l >> 2.
__device__ __forceinline__ float reduce8(const float (&s)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float k1[4], k2[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? s[i] : s[i + 4];
    k1[i] = (b4 ? s[i + 4] : s[i]) + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? k1[i] : k1[i + 2];
    k2[i] = (b3 ? k1[i + 2] : k1[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float send = b2 ? k2[0] : k2[1];
  float v = (b2 ? k2[1] : k2[0]) + __shfl_xor_sync(0xffffffffu, send, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}

// One step's online-softmax update for one query head: s = this lane's 8 partial dot products (one per slot of
// the step), vr = the step's V rows (4 dimensions per lane). Folds the step into m (running max), l (running sum,
// per lane: the 4 lanes of a slot hold the same value) and o (this lane's 4 output dimensions).
template <int REP>
__device__ __forceinline__ void online_step(const float (&s)[kStep], bool mine_in, int lane, const uint2 (&vr)[kStep],
                                            bool bf, float& m, float& l, float (&o)[4]) {
  float sc = reduce8(s, lane);
  if (!mine_in) sc = -INFINITY;
  float mx = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 4));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
  const float m_new = fmaxf(m, mx);         // finite: the step's first slot is always in range
  const float alpha = __expf(m - m_new);    // 0 on the first step (m = -inf)
  const float pj = __expf(sc - m_new);      // 0 for slots past the end
  l = l * alpha + pj;
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] *= alpha;
#pragma unroll
  for (int j = 0; j < kStep; ++j) {
    const float pb = __shfl_sync(0xffffffffu, pj, 4 * j);
    float vf[4];
    unpack4(vr[j], bf, vf);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = fmaf(pb, vf[i], o[i]);
  }
  m = m_new;
}

// One CTA's share of the decode attention: key-value head g, split sp, with kThreads threads (tid) that meet at
// named barrier bar_id. Writes its partial (or, when one split holds every slot, the output); the last split of
// the head to finish merges the partials and writes the head group's outputs (and, when p.heads_done is set,
// adds 1 to it with release semantics). sm_*: shared memory of the CTA merge; is_last: one shared int.
// Cache rows: through the read-only path, or (kCoherent) through L2 only, for a launch that itself writes the
// token's slot (the whole-step kernel, where another CTA's epilogue stores it earlier in the same launch).
template <bool kCoherent>
__device__ __forceinline__ uint2 ld_row8(const uint8_t* p) {
  if constexpr (kCoherent)
    return __ldcg(reinterpret_cast<const uint2*>(p));
  else
    return __ldg(reinterpret_cast<const uint2*>(p));
}

// kPre (standalone launch with programmatic dependent launch): the CTA reads the position and the K/V rows of its
// first step's slots before the position BEFORE it waits for the preceding kernel (griddepcontrol.wait, called
// here), then q and the position's own slot. Valid when the preceding kernels write only q and that slot (the
// decode step: the layer's input launch writes q and the token's K/V slot).
// kCluster (standalone launch in clusters of nsplit CTAs, one cluster per key-value head): the CTA leaves its merged
// partial in shared memory - the accumulator in sm_o[0], the maximum and the sum in cml[r] and cml[REP + r] - for
// the cluster's merge through distributed shared memory, instead of the global partials and the ticket.
// Returns the number of splits with slots (the same in every CTA of the launch), or -1 for a position outside
// the cache (nothing written).
// W: warps of the CTA (kWarps, or more in the cluster form: threads past the first kHd take part in the slots but
// not in the CTA's merge).
template <int REP, bool kLean, bool kCoherent = false, bool kPre = false, bool kCluster = false, int W = kWarps>
__device__ int attn_cta(const AttnParams& p, int g, int sp, int tid, int bar_id, float (*sm_m)[REP],
                        float (*sm_l)[REP], float (*sm_o)[REP][kHd], int* is_last, float* cml = nullptr) {
  static_assert(!((kPre || kCluster) && (kLean || kCoherent)), "the early loads are the standalone kernel's");
  static_assert(W == kWarps || kCluster, "other CTA widths only in the cluster form");
  static_assert(W >= kWarps, "a merge thread per dimension");
  const int warp = tid >> 5, lane = tid & 31;
  const bool bf = p.bf16 != 0;
  uint2 qraw[REP];  // issued together with the position load: one round trip for both
  auto load_q = [&]() {
#pragma unroll
    for (int r = 0; r < REP; ++r)
      qraw[r] = __ldcg(reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(p.q) +
                                                      (static_cast<int64_t>(g * REP + r) * kHd + 4 * lane) * 2));
  };
  if constexpr (!kPre) load_q();
  const int64_t pos = __ldcg(p.pos);
  if (pos < 0 || pos >= p.S) {  // the same decision in every CTA: none takes a ticket
    if (tid == 0 && blockIdx.x == 0) atomicOr(&g_device_error, ERR_ARG);
    return -1;
  }
  const int64_t n = pos + 1;
  const int64_t ch = ((n + p.nsplit - 1) / p.nsplit + W * kStep - 1) / (W * kStep) * (W * kStep);
  const int active = static_cast<int>((n + ch - 1) / ch);  // splits with slots; the others leave at once
  if (sp >= active) return active;
  const int64_t start = static_cast<int64_t>(sp) * ch, end = start + ch < n ? start + ch : n;

  const uint8_t* kb = static_cast<const uint8_t*>(p.kc) + static_cast<int64_t>(g) * p.S * kHd * 2 + lane * 8;
  const uint8_t* vb = static_cast<const uint8_t*>(p.vc) + static_cast<int64_t>(g) * p.S * kHd * 2 + lane * 8;
  uint2 kr[kStep], vr[kStep];  // the non-lean path's first step
  auto load_rows = [&](int64_t t, uint2 (&kk)[kStep], uint2 (&vv)[kStep], int64_t lim) {
#pragma unroll
    for (int j = 0; j < kStep; ++j) {
      const bool in = t + j < lim;
      kk[j] = in ? ld_row8<kCoherent>(kb + (t + j) * kHd * 2) : make_uint2(0u, 0u);
      vv[j] = in ? ld_row8<kCoherent>(vb + (t + j) * kHd * 2) : make_uint2(0u, 0u);
    }
  };
  if constexpr (kPre) {
    const int64_t t0 = start + warp * kStep, lim = end < pos ? end : pos;
    load_rows(t0, kr, vr, lim);  // slots before the position: not written by the launches before
    {  // the warp's later steps of such slots into L2: one 128-byte line per lane and step (slot lane / 4, K or V,
       // half of the 256-byte row); a plain prefetch, nothing to wait for
      const int j = lane >> 2;
      const uint8_t* line = ((lane >> 1) & 1 ? vb : kb) - lane * 8 + (lane & 1) * 128;
      for (int64_t t = t0 + W * kStep; t < lim; t += W * kStep)
        if (t + j < lim) asm volatile("prefetch.global.L2 [%0];" ::"l"(line + (t + j) * kHd * 2));
    }
    griddep_wait();  // q and the position's slot come from the previous kernel
    load_q();
#pragma unroll
    for (int j = 0; j < kStep; ++j)
      if (t0 + j == pos) {  // end == pos + 1 in the split that holds the position
        kr[j] = ld_row8<kCoherent>(kb + pos * kHd * 2);
        vr[j] = ld_row8<kCoherent>(vb + pos * kHd * 2);
      }
  } else if constexpr (!kLean) {
    load_rows(start + warp * kStep, kr, vr, end);
  }

  float qv[REP][4], m[REP], l[REP], o[REP][4];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    unpack4(qraw[r], bf, qv[r]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      qv[r][i] *= p.scale;
      o[r][i] = 0.f;
    }
    m[r] = -INFINITY;
    l[r] = 0.f;
  }
  const int jl = lane >> 2;  // the slot of the step whose score this lane ends up holding
  if constexpr (kLean) {  // one step's rows at a time, keys unpacked per head: fits 128 registers
    for (int64_t t0 = start + warp * kStep; t0 < end; t0 += W * kStep) {
      uint2 kr[kStep], vr[kStep];
#pragma unroll
      for (int j = 0; j < kStep; ++j) {
        const bool in = t0 + j < end;
        kr[j] = in ? ld_row8<kCoherent>(kb + (t0 + j) * kHd * 2) : make_uint2(0u, 0u);
        vr[j] = in ? ld_row8<kCoherent>(vb + (t0 + j) * kHd * 2) : make_uint2(0u, 0u);
      }
      const bool mine_in = t0 + jl < end;
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        float s[kStep];
#pragma unroll
        for (int j = 0; j < kStep; ++j) {
          float kf[4];
          unpack4(kr[j], bf, kf);
          s[j] = qv[r][0] * kf[0] + qv[r][1] * kf[1] + qv[r][2] * kf[2] + qv[r][3] * kf[3];
        }
        online_step<REP>(s, mine_in, lane, vr, bf, m[r], l[r], o[r]);
      }
    }
  } else {
    // kr / vr: this step's K and V rows (loaded above); the next step's are loaded before this one's math
    for (int64_t t0 = start + warp * kStep; t0 < end; t0 += W * kStep) {
      uint2 kn[kStep], vn[kStep];
      load_rows(t0 + W * kStep, kn, vn, end);  // past the end: nothing loaded
      float kf[kStep][4];
  #pragma unroll
      for (int j = 0; j < kStep; ++j) unpack4(kr[j], bf, kf[j]);
      const bool mine_in = t0 + jl < end;
  #pragma unroll
      for (int r = 0; r < REP; ++r) {
        float s[kStep];
  #pragma unroll
        for (int j = 0; j < kStep; ++j)
          s[j] = qv[r][0] * kf[j][0] + qv[r][1] * kf[j][1] + qv[r][2] * kf[j][2] + qv[r][3] * kf[j][3];
        online_step<REP>(s, mine_in, lane, vr, bf, m[r], l[r], o[r]);
      }
  #pragma unroll
      for (int j = 0; j < kStep; ++j) {
        kr[j] = kn[j];
        vr[j] = vn[j];
      }
    }
  }
  // merge the warps of this CTA
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float lt = l[r] + __shfl_xor_sync(0xffffffffu, l[r], 4);  // one lane per slot group of the step
    lt += __shfl_xor_sync(0xffffffffu, lt, 8);
    lt += __shfl_xor_sync(0xffffffffu, lt, 16);
    if (lane == 0) {
      sm_m[warp][r] = m[r];
      sm_l[warp][r] = lt;
    }
    *reinterpret_cast<float4*>(&sm_o[warp][r][4 * lane]) = make_float4(o[r][0], o[r][1], o[r][2], o[r][3]);
  }
  named_bar_sync(bar_id, W * 32);
  if (W > kWarps && tid >= kHd) return active;  // the CTA's merge: one thread per dimension
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, sm_m[w][r]);
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float e = __expf(sm_m[w][r] - M);
        O = fmaf(e, sm_o[w][r][tid], O);
        L = fmaf(e, sm_l[w][r], L);
      }
    }
    if (active == 1) {  // one split holds every slot: no partials, no merge
      store_out(p.out, static_cast<int64_t>(g * REP + r) * kHd + tid, O / L, bf);
      continue;
    }
    if constexpr (kCluster) {  // each thread rewrites only its own column of sm_o[0]
      sm_o[0][r][tid] = O;
      if (tid == 0) {
        cml[r] = M;
        cml[REP + r] = L;
      }
      continue;
    }
    const int64_t hs = static_cast<int64_t>(g * REP + r) * p.nsplit + sp;
    p.po[hs * kHd + tid] = O;
    if (tid == 0) {
      p.pm[hs] = M;
      p.pl[hs] = L;
    }
  }
  if (active == 1) {
    if (p.heads_done) {  // fused use: this head group is complete
      named_bar_sync(bar_id, kThreads);
      if (tid == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.heads_done) : "memory");
    }
    return active;
  }
  if constexpr (kCluster) return active;
  // The counter add releases this CTA's partial (the barrier orders every thread's stores before thread 0's
  // release) and, for the last CTA, acquires the others' (its loads follow the barrier after the acquire).
  named_bar_sync(bar_id, kThreads);
  if (tid == 0) {
    unsigned int prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.ticket + g) : "memory");
    *is_last = prev == static_cast<unsigned int>(active - 1);
  }
  named_bar_sync(bar_id, kThreads);
  if (!*is_last) return active;
  // The last CTA of key-value head g merges the active partials of its query heads. Warp w takes splits
  // w, w + 4, ... and every lane 4 dimensions (16-byte loads), merging with an online rescale (running max) so
  // that all loads of a warp - maxima, sums and accumulators of its splits for every head - are independent
  // and in flight together; the four warps' results are then merged through shared memory in warp order.
  const int64_t hg = static_cast<int64_t>(g * REP) * p.nsplit;
  {
    float Mw[REP], Lw[REP], Ow[REP][4];
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      Mw[r] = -INFINITY;
      Lw[r] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) Ow[r][i] = 0.f;
    }
#pragma unroll 4
    for (int s = warp; s < active; s += kWarps) {
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        const int64_t hs = hg + r * p.nsplit + s;
        const float ms = __ldcg(p.pm + hs), ls = __ldcg(p.pl + hs);
        const float4 os = __ldcg(reinterpret_cast<const float4*>(p.po + hs * kHd) + lane);
        const float Mn = fmaxf(Mw[r], ms);
        const float a = __expf(Mw[r] - Mn), w = __expf(ms - Mn);  // a = 0 for the warp's first split
        Lw[r] = fmaf(Lw[r], a, w * ls);
        Ow[r][0] = fmaf(Ow[r][0], a, w * os.x);
        Ow[r][1] = fmaf(Ow[r][1], a, w * os.y);
        Ow[r][2] = fmaf(Ow[r][2], a, w * os.z);
        Ow[r][3] = fmaf(Ow[r][3], a, w * os.w);
        Mw[r] = Mn;
      }
    }
    named_bar_sync(bar_id, kThreads);  // the CTA-merge arrays are free again
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      if (lane == 0) {
        sm_m[warp][r] = Mw[r];
        sm_l[warp][r] = Lw[r];
      }
      *reinterpret_cast<float4*>(&sm_o[warp][r][4 * lane]) = make_float4(Ow[r][0], Ow[r][1], Ow[r][2], Ow[r][3]);
    }
  }
  named_bar_sync(bar_id, kThreads);
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w][r]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float e = sm_m[w][r] == -INFINITY ? 0.f : __expf(sm_m[w][r] - M);  // a warp without splits
      O = fmaf(e, sm_o[w][r][tid], O);
      L = fmaf(e, sm_l[w][r], L);
    }
    store_out(p.out, static_cast<int64_t>(g * REP + r) * kHd + tid, O / L, bf);
  }
  if (tid == 0) p.ticket[g] = 0u;  // ready for the next call
  if (p.heads_done) {  // fused use: publish this key-value head's outputs to the waiting CTAs of the launch
    named_bar_sync(bar_id, kThreads);
    if (tid == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.heads_done) : "memory");
  }
  return active;
}

// Splits per key-value head: about one CTA per SM over all heads.
inline int64_t nsplit_for(int nkv, int sms) { return std::max(1, std::min(kMaxSplit, sms / nkv)); }

}  // namespace attn

}  // namespace rb
