// glue.cuh - the decode-layer glue shared by the GEMV kernels (tensor-core and warp-MMA): the add + LayerNorm
// prologue that produces a launch's activations (rumik-fast engine/fused.py:29-40) and the row routing of the
// epilogues (rotary embedding + KV-cache write, SiLU-gated MLP activation; engine/fused.py:43-84).
#pragma once

#include "common.cuh"

namespace rb {

// Where a routed entry's rows go (rb_gemv_epi).
struct EpiP {
  const int64_t* pos;
  const void* cos;
  const void* sin;
  void* q_out;
  void* k_cache;
  void* v_cache;
  void* act;
  int64_t S;
  int rope, nq, nkv, hd;
};

// Sources of the add + LayerNorm prologue (rb_add_ln): h = LayerNorm(round(x + a + b)) * w.
struct LnSrc {
  const void* x;
  const void* a;
  const void* b;
  const void* w;
  void* x_out;
  void* h_out;
  float eps;
  int K;
  const int8_t* emb_q;  // token-embedding source (x, a, b unused): round(emb_q[tok] * emb_s[tok])
  const void* emb_s;
  const int64_t* tok;
  int64_t vocab;
  int emb_f16;          // emb_s is fp16 (else fp32)
};

constexpr int kLnMaxGroups = 96;  // H <= 12288: 128-element groups of the prologue vector

__device__ __forceinline__ void store8_act(void* p, const float (&v)[8], bool is_bf16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (is_bf16) {
      w[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i]))) |
             (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1]))) << 16);
    } else {
      w[i] = pack_half2(__float2half_rn(v[2 * i]), __float2half_rn(v[2 * i + 1]));
    }
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Sum over the 16 chunks (8 elements each) of every 128-element group, written by the group's first lane to
// gsum[group]: chunk c of the vector is held by thread c mod nthreads, so a group is 16 consecutive lanes of
// one warp (nthreads a multiple of 32). All 32 lanes call this.
__device__ __forceinline__ void group_sums(float cs, bool valid, int c, int ct, float* gsum) {
  cs += __shfl_xor_sync(0xffffffffu, cs, 8);
  cs += __shfl_xor_sync(0xffffffffu, cs, 4);
  cs += __shfl_xor_sync(0xffffffffu, cs, 2);
  cs += __shfl_xor_sync(0xffffffffu, cs, 1);
  if (valid && (ct & 15) == 0) gsum[c >> 4] = cs;
}

// The add + LayerNorm of rumik-fast's add_ln (engine/fused.py:29-40), computed by every CTA from global
// memory with `nthreads` threads (ids ct): s = (x + a) + b in fp32 rounded to the activation type,
// h = (s - mean) * rsqrt(var + eps) * w rounded likewise, mean and var over the K elements in two passes as the
// reference. The sums run per 128-element group (fixed lane order) and then over the groups in order, so the
// result is bit-identical for any thread count (the tensor-core and warp-MMA prologues, and the standalone
// kernel). `writer_cta` also stores s (x_out) and h (h_out); write(h[8], valid, chunk) tabulates each chunk
// for the GEMV (all 32 lanes of every warp call it together). gsum: 2 x kLnMaxGroups floats of shared memory;
// bar_id: a named barrier of the nthreads threads.
template <int kIter, class Writer>
__device__ void stage_ln(const LnSrc& S, bool bf, float* gsum, int bar_id, int ct, int nthreads, bool writer_cta,
                         Writer&& write) {
  const int chunks = S.K / 8, G = S.K / 128;
  float v[kIter][8];
  uint4 wraw[kIter];  // the LayerNorm weight, loaded with x, a and b
  // token-embedding source (engine/fused.py:18-27): the token's int8 row and its scale
  const int8_t* erow = nullptr;
  float escale = 0.f;
  if (S.emb_q) {
    int64_t tok = *S.tok;
    if (tok < 0 || tok >= S.vocab) {
      if (ct == 0 && writer_cta) atomicOr(&g_device_error, ERR_ARG);
      tok = 0;
    }
    erow = S.emb_q + tok * S.K;
    escale = S.emb_f16 ? __half2float(reinterpret_cast<const __half*>(S.emb_s)[tok])
                       : reinterpret_cast<const float*>(S.emb_s)[tok];
  }
#pragma unroll
  for (int it = 0; it < kIter; ++it) {
    const int c = it * nthreads + ct;
    const bool valid = c < chunks;
    wraw[it] = valid ? ldg_cg_128(static_cast<const uint8_t*>(S.w) + static_cast<int64_t>(c) * 16)
                     : make_uint4(0u, 0u, 0u, 0u);
    float cs = 0.f;
    if (valid && erow) {
      const uint2 q8 = __ldg(reinterpret_cast<const uint2*>(erow + static_cast<int64_t>(c) * 8));
      const uint32_t qw[2] = {q8.x, q8.y};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int8_t qi = static_cast<int8_t>((qw[i >> 2] >> (8 * (i & 3))) & 0xFFu);
        v[it][i] = round_act(static_cast<float>(qi) * escale, bf);
        cs += v[it][i];
      }
    } else if (valid) {
      load8_f32(static_cast<const uint8_t*>(S.x) + static_cast<int64_t>(c) * 16, bf, v[it]);
      float t[8];
      if (S.a) {
        load8_f32(static_cast<const uint8_t*>(S.a) + static_cast<int64_t>(c) * 16, bf, t);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] += t[i];
      }
      if (S.b) {
        load8_f32(static_cast<const uint8_t*>(S.b) + static_cast<int64_t>(c) * 16, bf, t);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] += t[i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[it][i] = round_act(v[it][i], bf);
        cs += v[it][i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[it][i] = 0.f;
    }
    if (it * nthreads < chunks) group_sums(cs, valid, c, ct, gsum);  // uniform over the threads
  }
  named_bar_sync(bar_id, nthreads);
  const float inv_h = 1.f / static_cast<float>(S.K);
  float tot = 0.f;
  for (int g = 0; g < G; ++g) tot += gsum[g];
  const float mean = tot * inv_h;
#pragma unroll
  for (int it = 0; it < kIter; ++it) {
    const int c = it * nthreads + ct;
    float cs = 0.f;
    if (c < chunks) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[it][i] - mean;
        cs += d * d;
      }
    }
    if (it * nthreads < chunks) group_sums(cs, c < chunks, c, ct, gsum + kLnMaxGroups);
  }
  named_bar_sync(bar_id, nthreads);
  float sq = 0.f;
  for (int g = 0; g < G; ++g) sq += gsum[kLnMaxGroups + g];
  const float rstd = rsqrtf(sq * inv_h + S.eps);
#pragma unroll
  for (int it = 0; it < kIter; ++it) {
    if (it * nthreads >= chunks) break;  // uniform over the threads
    const int c = it * nthreads + ct;
    const bool valid = c < chunks;
    float h[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (valid) {
      float w[8];
      raw_to_f32(wraw[it], bf, w);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = round_act((v[it][i] - mean) * rstd * w[i], bf);
      if (writer_cta && S.x_out) store8_act(static_cast<uint8_t*>(S.x_out) + static_cast<int64_t>(c) * 16, v[it], bf);
      if (writer_cta && S.h_out) store8_act(static_cast<uint8_t*>(S.h_out) + static_cast<int64_t>(c) * 16, h, bf);
    }
    write(h, valid, c);
  }
}

// Route one output row of a RB_EPI_ROPE_KV / RB_EPI_SWIGLU entry (engine/fused.py:43-84). r: the row's result
// rounded to the output type (what the engine's y buffer would hold); pr: that of its partner row (row ^ 1:
// the other element of a rotary pair, or the up channel of a gate row); pos: the token's position, already
// checked to lie in [0, S).
__device__ __forceinline__ void route_row(const EpiP& P, int epi, int row, float r, float pr, int64_t pos,
                                          bool bf) {
  if (epi == RB_EPI_ROPE_KV) {
    const int head = row / P.hd, dd = row - head * P.hd;
    float o = r;
    if (P.rope && head < P.nq + P.nkv) {  // pairs (2j, 2j + 1) rotated by pos * theta_j
      const int64_t ci = pos * P.hd + (dd & ~1);
      const float c = load_act(P.cos, ci, bf), sn = load_act(P.sin, ci, bf);
      o = (dd & 1) ? r * c + pr * sn : r * c - pr * sn;
    }
    if (head < P.nq)
      store_out(P.q_out, static_cast<int64_t>(head) * P.hd + dd, o, bf);
    else if (head < P.nq + P.nkv)
      store_out(P.k_cache, (static_cast<int64_t>(head - P.nq) * P.S + pos) * P.hd + dd, o, bf);
    else
      store_out(P.v_cache, (static_cast<int64_t>(head - P.nq - P.nkv) * P.S + pos) * P.hd + dd, o, bf);
  } else if ((row & 1) == 0) {  // RB_EPI_SWIGLU: row 2c = gate channel c, row 2c + 1 = its up channel
    store_out(P.act, row >> 1, r / (1.f + __expf(-r)) * pr, bf);
  }
}

}  // namespace rb
