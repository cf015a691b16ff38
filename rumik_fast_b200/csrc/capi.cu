// capi.cu - the extern "C" boundary (include/rumik_b200.h). Validates arguments on the host (before any
// CUDA call), picks the launch shape for the device's SM count and forwards to the kernel files.
#include <cuda_runtime.h>

#include "common.cuh"
#include <vector>

#include "kernels.h"

#include <cstring>

namespace {

constexpr int kVersion = 100;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool act_dtype_ok(int d) { return d == RB_F16 || d == RB_BF16; }

int device_sms(int* sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RB_ERR_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return RB_ERR_DEVICE;
  if (major != 10) return RB_ERR_DEVICE;  // the cubins are sm_100a only
  if (cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return RB_ERR_DEVICE;
  return RB_OK;
}

// Shared checks of the activation / output side of a GEMV-shaped call.
int check_act(const void* x, int x_dtype, int64_t ldx, const void* y, int y_dtype, int64_t ldy, int64_t K,
              int64_t N, int64_t batch) {
  if (!x || !y) return RB_ERR_NULL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(y_dtype)) return RB_ERR_DTYPE;
  if (batch > 1 && (ldx < K || ldy < N)) return RB_ERR_SHAPE;
  if (!aligned16(x) || (batch > 1 && (ldx % 8) != 0)) return RB_ERR_ALIGN;
  return RB_OK;
}

}  // namespace

extern "C" {

int rb_version(void) { return kVersion; }

const char* rb_status_string(int status) {
  switch (status) {
    case RB_OK: return "ok";
    case RB_ERR_NULL: return "a required pointer is NULL";
    case RB_ERR_SHAPE: return "unsupported shape";
    case RB_ERR_DTYPE: return "unsupported dtype";
    case RB_ERR_ALIGN: return "pointer not 16-byte aligned or row stride not a multiple of 8 elements";
    case RB_ERR_LAUNCH: return "CUDA kernel launch failed";
    case RB_ERR_DEVICE: return "no usable sm_100 CUDA device";
    case RB_ERR_TIMEOUT: return "a kernel gave up a bounded wait";
    default: return "unknown status";
  }
}

int rb_gemv_int4(const void* x, int x_dtype, int64_t ldx, const uint8_t* q, const uint16_t* s, const uint16_t* m,
                 void* y, int y_dtype, int64_t ldy, int64_t N, int64_t K, int64_t batch, int flags, void* stream) {
  if (N < 0 || K <= 0 || batch < 0) return RB_ERR_SHAPE;
  if (K % 128 != 0 || K > 16384 || N > (int64_t(1) << 30)) return RB_ERR_SHAPE;
  if (N == 0 || batch == 0) return RB_OK;
  if (!q || !s || !m) return RB_ERR_NULL;
  int st = check_act(x, x_dtype, ldx, y, y_dtype, ldy, K, N, batch);
  if (st != RB_OK) return st;
  if (!aligned16(q) || !aligned16(s) || !aligned16(m)) return RB_ERR_ALIGN;
  int sms = 0;
  if ((st = device_sms(&sms)) != RB_OK) return st;
  rb::GemvArgs a = {};
  a.x = x; a.x_dtype = x_dtype; a.ldx = batch > 1 ? ldx : K;
  a.q = q; a.s = s; a.m = m;
  a.y = y; a.y_dtype = y_dtype; a.ldy = batch > 1 ? ldy : N;
  a.N = N; a.K = K; a.batch = batch; a.flags = flags;
  // batch 1 with at least one 128-row block per SM: the tensor-core kernel (a one-entry list). Smaller
  // matrices keep the warp-MMA kernel, which spreads 8-row stages over every SM.
  if (batch == 1 && N >= static_cast<int64_t>(sms) * 128) {
    rb_gemv_desc d = {x, y, q, s, m, N, K};
    st = rb::launch_gemv_int4_tc(&d, 1, x_dtype, y_dtype, flags, sms, static_cast<cudaStream_t>(stream));
    if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
    return st;
  }
  st = rb::launch_gemv_int4(a, sms, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int rb_gemv_int8(const void* x, int x_dtype, int64_t ldx, const uint8_t* q, int q_signed, const void* s,
                 int s_dtype, void* y, int y_dtype, int64_t ldy, int64_t N, int64_t K, int64_t batch, int flags,
                 void* stream) {
  if (N < 0 || K <= 0 || batch < 0) return RB_ERR_SHAPE;
  if (K % 64 != 0 || K > 16384 || N > (int64_t(1) << 30)) return RB_ERR_SHAPE;
  if (N == 0 || batch == 0) return RB_OK;
  if (!q || !s) return RB_ERR_NULL;
  if (s_dtype != RB_F32 && s_dtype != RB_F16) return RB_ERR_DTYPE;
  int st = check_act(x, x_dtype, ldx, y, y_dtype, ldy, K, N, batch);
  if (st != RB_OK) return st;
  if (!aligned16(q)) return RB_ERR_ALIGN;
  int sms = 0;
  if ((st = device_sms(&sms)) != RB_OK) return st;
  rb::GemvArgs a = {};
  a.x = x; a.x_dtype = x_dtype; a.ldx = batch > 1 ? ldx : K;
  a.q = q; a.q_signed = q_signed; a.s_row = s; a.s_dtype = s_dtype;
  a.y = y; a.y_dtype = y_dtype; a.ldy = batch > 1 ? ldy : N;
  a.N = N; a.K = K; a.batch = batch; a.flags = flags;
  // batch 1 with K % 128 == 0 runs on the tensor cores; other shapes on the warp-MMA kernel
  st = rb::launch_gemv_int8_tc(a, sms, static_cast<cudaStream_t>(stream));
  if (st == RB_ERR_SHAPE) st = rb::launch_gemv_int8(a, sms, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

// The min / per-row-factor pointer of a descriptor: fp16 mins 16-byte aligned, or (8-bit scales) fp32 factors
// 4-byte aligned.
static bool scales_aligned(const rb_gemv_desc& d) {
  return d.s_row ? (reinterpret_cast<uintptr_t>(d.s_row) & 3u) == 0 : aligned16(d.m);
}

static bool any_scales8(const rb_gemv_desc* d, int count) {
  for (int i = 0; i < count; ++i)
    if (d[i].s_row && d[i].w8 == RB_W8_NONE) return true;
  return false;
}

// int8 entries (rb_gemv_desc::w8): the tcgen05 list kernel only.
static bool any_w8(const rb_gemv_desc* d, int count) {
  for (int i = 0; i < count; ++i)
    if (d[i].w8 != RB_W8_NONE) return true;
  return false;
}

// An int8 entry's pointers: x, y, q (16-byte aligned) and its row scales, s_row (fp32, 4-byte aligned) or s (fp16).
static int check_w8(const rb_gemv_desc& d) {
  if (d.w8 != RB_W8_SIGNED && d.w8 != RB_W8_OFFSET) return RB_ERR_SHAPE;
  if (!d.x || !d.y || !d.q || (!d.s_row && !d.s)) return RB_ERR_NULL;
  const uintptr_t sp = d.s_row ? reinterpret_cast<uintptr_t>(d.s_row) : reinterpret_cast<uintptr_t>(d.s);
  if (!aligned16(d.x) || !aligned16(d.q) || (sp & (d.s_row ? 3u : 1u))) return RB_ERR_ALIGN;
  return RB_OK;
}

static int check_multi(const rb_gemv_desc* descs, int count, int x_dtype, int y_dtype) {
  if (!descs) return RB_ERR_NULL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(y_dtype)) return RB_ERR_DTYPE;
  for (int i = 0; i < count; ++i) {
    const rb_gemv_desc& d = descs[i];
    if (d.N < 1 || d.K <= 0 || d.K % 128 != 0 || d.K > 16384 || d.N > (int64_t(1) << 30)) return RB_ERR_SHAPE;
    if (d.w8 != RB_W8_NONE) {
      const int st = check_w8(d);
      if (st != RB_OK) return st;
      continue;
    }
    if (!d.x || !d.y || !d.q || !d.s || (!d.m && !d.s_row)) return RB_ERR_NULL;
    if (!aligned16(d.x) || !aligned16(d.q) || !aligned16(d.s) || !scales_aligned(d)) return RB_ERR_ALIGN;
  }
  return RB_OK;
}

// Lists whose int4 codes total less than this run on the warp-MMA multi-GEMV (gemv_int4_multi.cu): a decode
// layer's projections (18-35 MB) are latency-bound, and its per-launch cost is about half the tensor-core
// kernel's. Longer lists (a whole step's projections, 1.9 GB) are HBM-bound and run on the tcgen05 kernel.
#ifndef RB_SMALL_LIST_BYTES
#define RB_SMALL_LIST_BYTES (int64_t(128) << 20)
#endif
// A list with 8-bit scales or int8 entries cannot be forced onto the warp-MMA kernel, which has no path for them.
static bool kernel_ok(const rb_gemv_desc* d, int count, int flags) {
  return !((flags & RB_FLAG_KERNEL_MMA) && (any_scales8(d, count) || any_w8(d, count)));
}

static bool small_list(const rb_gemv_desc* d, int count, int flags) {
  if (flags & RB_FLAG_KERNEL_TC) return false;
  // 8-bit scales, int8 entries: the tcgen05 kernel only (kernel_ok refuses MMA)
  if (any_scales8(d, count) || any_w8(d, count)) return false;
  if (flags & RB_FLAG_KERNEL_MMA) return true;
  int64_t bytes = 0;
  for (int i = 0; i < count; ++i) bytes += d[i].N * (d[i].K / 2);
  return bytes < RB_SMALL_LIST_BYTES;
}

static int multi_impl(const rb_gemv_desc* descs, int count, void* ws, int64_t ws_bytes, int x_dtype, int y_dtype,
                      int flags, void* stream) {
  if (count < 0) return RB_ERR_SHAPE;
  if (count == 0) return RB_OK;
  int st = check_multi(descs, count, x_dtype, y_dtype);
  if (st != RB_OK) return st;
  if (!kernel_ok(descs, count, flags)) return RB_ERR_SHAPE;
  if (ws && !aligned16(ws)) return RB_ERR_ALIGN;
  int sms = 0;
  st = device_sms(&sms);
  if (st != RB_OK) return st;
  if (small_list(descs, count, flags))
    st = rb::launch_gemv_int4_multi(descs, count, x_dtype, y_dtype, flags, sms, static_cast<cudaStream_t>(stream));
  else
    st = rb::launch_gemv_int4_tc(descs, count, x_dtype, y_dtype, flags, sms, static_cast<cudaStream_t>(stream),
                                 nullptr, nullptr, ws, ws_bytes);
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int rb_gemv_int4_multi(const rb_gemv_desc* descs, int count, int x_dtype, int y_dtype, int flags, void* stream) {
  return multi_impl(descs, count, nullptr, 0, x_dtype, y_dtype, flags, stream);
}

int rb_gemv_int4_multi_ws(const rb_gemv_desc* descs, int count, void* ws, int64_t ws_bytes, int x_dtype,
                          int y_dtype, int flags, void* stream) {
  return multi_impl(descs, count, ws, ws_bytes, x_dtype, y_dtype, flags, stream);
}

int64_t rb_gemv_int4_workspace(const rb_gemv_desc* descs, int count, int flags) {
  if (count < 0) return -RB_ERR_SHAPE;
  if (count == 0) return 0;
  if (!descs) return -RB_ERR_NULL;
  for (int i = 0; i < count; ++i) {
    const rb_gemv_desc& d = descs[i];
    if (d.N < 1 || d.K <= 0 || d.K % 128 != 0 || d.K > 16384 || d.N > (int64_t(1) << 30)) return -RB_ERR_SHAPE;
    if (d.w8 < RB_W8_NONE || d.w8 > RB_W8_OFFSET) return -RB_ERR_SHAPE;
    if (!d.q) return -RB_ERR_NULL;
  }
  if (!kernel_ok(descs, count, flags)) return -RB_ERR_SHAPE;
  if (small_list(descs, count, flags)) return 0;  // the warp-MMA kernel splits K inside each CTA
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return -st;
  // entries with x == NULL read a prologue's vector: only the slot bookkeeping looks at it here
  static const uint8_t dummy[16] = {};
  rb_add_ln ln = {};
  ln.x = dummy;
  ln.w = dummy;
  bool from_ln = false;
  for (int i = 0; i < count; ++i) from_ln |= descs[i].x == nullptr;
  int64_t need = 0;
  st = rb::launch_gemv_int4_tc(descs, count, RB_F16, RB_F16, 0, sms, nullptr, nullptr, from_ln ? &ln : nullptr,
                               nullptr, 0, &need);
  return st == RB_OK ? need : -st;
}

static bool ranges_overlap(const void* a, int64_t abytes, const void* b, int64_t bbytes) {
  if (!a || !b) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + static_cast<uintptr_t>(bbytes) && b0 < a0 + static_cast<uintptr_t>(abytes);
}

static int check_add_ln(const rb_add_ln* ln) {
  if (ln->emb_q) {  // the token-embedding source replaces x + a + b
    if (ln->x || ln->a || ln->b) return RB_ERR_SHAPE;
    if (!ln->emb_s || !ln->tok || !ln->w) return RB_ERR_NULL;
    if (ln->vocab < 1) return RB_ERR_SHAPE;
    if (ln->emb_s_dtype != RB_F32 && ln->emb_s_dtype != RB_F16) return RB_ERR_DTYPE;
    if (!aligned16(ln->emb_q)) return RB_ERR_ALIGN;
  } else if (!ln->x || !ln->w) {
    return RB_ERR_NULL;
  }
  if (ln->H < 128 || ln->H % 128 != 0 || ln->H > 12288) return RB_ERR_SHAPE;
  if (!(ln->eps >= 0.f)) return RB_ERR_SHAPE;
  const void* in[4] = {ln->x, ln->a, ln->b, ln->w};
  const void* out[2] = {ln->x_out, ln->h_out};
  for (const void* v : in)
    if (v && !aligned16(v)) return RB_ERR_ALIGN;
  for (const void* v : out)
    if (v && !aligned16(v)) return RB_ERR_ALIGN;
  const int64_t bytes = ln->H * 2;
  for (const void* o : out)
    for (const void* v : in)
      if (ranges_overlap(o, bytes, v, bytes)) return RB_ERR_SHAPE;
  if (ranges_overlap(ln->x_out, bytes, ln->h_out, bytes)) return RB_ERR_SHAPE;
  return RB_OK;
}

int rb_add_layernorm(const rb_add_ln* ln, int dtype, int flags, void* stream) {
  if (!ln) return RB_ERR_NULL;
  if (!act_dtype_ok(dtype)) return RB_ERR_DTYPE;
  int st = check_add_ln(ln);
  if (st != RB_OK) return st;
  int sms = 0;
  st = device_sms(&sms);
  if (st != RB_OK) return st;
  st = rb::launch_add_ln(ln, dtype, flags, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int64_t rb_sample_workspace(int nz) { return nz < 1 ? -RB_ERR_SHAPE : rb::sample_workspace(nz); }

int rb_sample(const rb_sampler* s, int flags, void* stream) {
  if (!s) return RB_ERR_NULL;
  if (s->n_vocab < 1 || s->n_vocab > 32768 || s->top_k < 1 || s->top_k > 32 || s->top_k > s->n_vocab)
    return RB_ERR_SHAPE;
  if (s->H < 1 || s->H > 8192 || s->nz < 1 || s->out_len < 0 || !(s->inv_temp == s->inv_temp)) return RB_ERR_SHAPE;
  if (!s->logits || !s->ids || !s->u || !s->h || !s->ln_w || !s->ln_b || !s->w1 || !s->b1 || !s->w2 || !s->b2 ||
      !s->step || !s->tok || !s->ws || (s->out_len > 0 && !s->out))
    return RB_ERR_NULL;
  if (!aligned16(s->w1) || !aligned16(s->ws)) return RB_ERR_ALIGN;
  const int dts[3] = {s->logits_dtype, s->h_dtype, s->w1_dtype};
  for (int d : dts)
    if (d != RB_F16 && d != RB_BF16 && d != RB_F32) return RB_ERR_DTYPE;
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return st;
  st = rb::launch_sample(s, flags, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int64_t rb_attn_decode_workspace(int n_q_heads, int n_kv_heads, int head_dim) {
  return rb::attn_decode_workspace(n_q_heads, n_kv_heads, head_dim);
}

int rb_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                   int n_q_heads, int n_kv_heads, int head_dim, int64_t cache_len, float scale, void* ws,
                   int64_t ws_bytes, int dtype, int flags, void* stream) {
  const int64_t need = rb::attn_decode_workspace(n_q_heads, n_kv_heads, head_dim);
  if (need < 0 || cache_len < 1 || cache_len > (int64_t(1) << 31)) return RB_ERR_SHAPE;
  if (!q || !k_cache || !v_cache || !pos || !out || !ws) return RB_ERR_NULL;
  if (!act_dtype_ok(dtype)) return RB_ERR_DTYPE;
  if (!(scale == scale)) return RB_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) || !aligned16(ws))
    return RB_ERR_ALIGN;
  if (ws_bytes < need) return RB_ERR_SHAPE;
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return st;
  st = rb::launch_attn_decode(q, k_cache, v_cache, pos, out, n_q_heads, n_kv_heads, cache_len, scale, ws, dtype, flags,
                              sms, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int rb_gemv_int4_fused(const rb_gemv_desc* descs, const rb_gemv_epi* epis, int count, const rb_add_ln* ln,
                       const rb_attn_src* attn, void* ws, int64_t ws_bytes, int x_dtype, int y_dtype, int flags,
                       void* stream) {
  if (count < 0 || count > 160) return RB_ERR_SHAPE;
  if (count == 0) return RB_OK;
  if (!descs) return RB_ERR_NULL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(y_dtype)) return RB_ERR_DTYPE;
  if (ln) {
    const int st = check_add_ln(ln);
    if (st != RB_OK) return st;
  }
  int routed = 0;
  for (int i = 0; i < count; ++i) {
    const rb_gemv_desc& d = descs[i];
    const int kind = epis ? epis[i].kind : RB_EPI_STORE;
    if (d.N < 1 || d.K <= 0 || d.K % 128 != 0 || d.K > 16384 || d.N > (int64_t(1) << 30)) return RB_ERR_SHAPE;
    if (d.w8 != RB_W8_NONE) return RB_ERR_SHAPE;  // int8 entries: rb_gemv_int4_multi(_ws) only
    if (!d.q || !d.s || (!d.m && !d.s_row)) return RB_ERR_NULL;
    if (!d.x && !ln) return RB_ERR_NULL;
    if (!d.x && d.K != ln->H) return RB_ERR_SHAPE;
    if ((d.x && !aligned16(d.x)) || !aligned16(d.q) || !aligned16(d.s) || !scales_aligned(d)) return RB_ERR_ALIGN;
    if (kind == RB_EPI_STORE) {
      if (!d.y) return RB_ERR_NULL;
      continue;
    }
    ++routed;
    const rb_gemv_epi& e = epis[i];
    if (kind == RB_EPI_ROPE_KV) {
      if (e.head_dim < 2 || e.head_dim % 2 != 0 || e.n_q_heads < 0 || e.n_kv_heads < 0 || e.cache_len < 1)
        return RB_ERR_SHAPE;
      if (d.N != static_cast<int64_t>(e.n_q_heads + 2 * e.n_kv_heads) * e.head_dim) return RB_ERR_SHAPE;
      if (!e.pos || (e.n_q_heads > 0 && !e.q_out) || (e.n_kv_heads > 0 && (!e.k_cache || !e.v_cache)))
        return RB_ERR_NULL;
      if (e.rope && (!e.cos || !e.sin)) return RB_ERR_NULL;
    } else if (kind == RB_EPI_SWIGLU) {
      if (d.N % 2 != 0) return RB_ERR_SHAPE;
      if (!e.act_out) return RB_ERR_NULL;
    } else {
      return RB_ERR_SHAPE;
    }
  }
  if (routed > 4) return RB_ERR_SHAPE;
  if (!kernel_ok(descs, count, flags)) return RB_ERR_SHAPE;
  if (ws && !aligned16(ws)) return RB_ERR_ALIGN;
  if (attn) {
    const int64_t need = rb::attn_decode_workspace(attn->n_q_heads, attn->n_kv_heads, attn->head_dim);
    if (need < 0 || attn->n_q_heads / attn->n_kv_heads > 4) return RB_ERR_SHAPE;
    if (attn->cache_len < 1 || attn->cache_len > (int64_t(1) << 31) || !(attn->scale == attn->scale))
      return RB_ERR_SHAPE;
    if (!attn->q || !attn->k_cache || !attn->v_cache || !attn->pos || !attn->out || !attn->ws) return RB_ERR_NULL;
    if (!aligned16(attn->q) || !aligned16(attn->k_cache) || !aligned16(attn->v_cache) || !aligned16(attn->out) ||
        !aligned16(attn->ws))
      return RB_ERR_ALIGN;
    if (attn->ws_bytes < need) return RB_ERR_SHAPE;
    if (flags & RB_FLAG_KERNEL_TC) return RB_ERR_SHAPE;  // fused attention runs on the warp-MMA kernel
    if (any_scales8(descs, count)) return RB_ERR_SHAPE;  // which has no 8-bit scales
    bool any = false;
    for (int i = 0; i < count; ++i) {
      if (descs[i].x != attn->out) continue;
      any = true;
      if (descs[i].K != static_cast<int64_t>(attn->n_q_heads) * attn->head_dim) return RB_ERR_SHAPE;
    }
    if (!any) return RB_ERR_SHAPE;
  }
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return st;
  if (attn || small_list(descs, count, flags))
    st = rb::launch_gemv_int4_multi(descs, count, x_dtype, y_dtype, flags, sms, static_cast<cudaStream_t>(stream), epis,
                                    ln, attn);
  else
    st = rb::launch_gemv_int4_tc(descs, count, x_dtype, y_dtype, flags, sms, static_cast<cudaStream_t>(stream), epis,
                                 ln, ws, ws_bytes);
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

static int mm_int4_impl(const void* X, int x_dtype, int64_t ldx, const uint8_t* q, const uint16_t* s,
                        const uint16_t* m, void* Y, int y_dtype, int64_t ldy, int64_t M, int64_t N, int64_t K,
                        void* ws, int64_t ws_bytes, int flags, void* stream, bool static_scratch = false) {
  if (M < 0 || N < 0 || K <= 0) return RB_ERR_SHAPE;
  if (K % 128 != 0 || N > (int64_t(1) << 30) || M > (int64_t(1) << 30)) return RB_ERR_SHAPE;
  if (M == 0 || N == 0) return RB_OK;
  if (!X || !Y || !q || !s || !m) return RB_ERR_NULL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(y_dtype)) return RB_ERR_DTYPE;
  if (ldx < K || ldy < N) return RB_ERR_SHAPE;
  if (!aligned16(X) || !aligned16(Y) || (ldx % 8) != 0 || (ldy % 8) != 0) return RB_ERR_ALIGN;
  if (!aligned16(q) || !aligned16(s) || !aligned16(m)) return RB_ERR_ALIGN;
  if (ws && !aligned16(ws)) return RB_ERR_ALIGN;
  // one token is a GEMV: the GEMV kernels stream the weights faster than the prefill's per-item pipeline
  // (measured: 1.33 against 2.06 ms for the 36-layer projection set)
  if (M == 1 && K <= 16384) return rb_gemv_int4(X, x_dtype, K, q, s, m, Y, y_dtype, N, N, K, 1, flags, stream);
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return st;
  rb::MmArgs a = {};
  a.X = X; a.x_dtype = x_dtype; a.ldx = ldx;
  a.q = q; a.s = s; a.m = m;
  a.Y = Y; a.y_dtype = y_dtype; a.ldy = ldy;
  a.M = M; a.N = N; a.K = K; a.flags = flags;
  a.ws = static_cast<float*>(ws); a.ws_bytes = ws ? ws_bytes : 0;
  if (static_scratch) {
    st = rb::launch_mm_int4_tc_static(a, sms, static_cast<cudaStream_t>(stream));
    if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
    return st;
  }
  st = rb::launch_mm_int4_tc(a, sms, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int rb_mm_int4(const void* X, int x_dtype, int64_t ldx, const uint8_t* q, const uint16_t* s, const uint16_t* m,
               void* Y, int y_dtype, int64_t ldy, int64_t M, int64_t N, int64_t K, int flags, void* stream) {
  return mm_int4_impl(X, x_dtype, ldx, q, s, m, Y, y_dtype, ldy, M, N, K, nullptr, 0, flags, stream);
}

int64_t rb_mm_int4_workspace(int64_t M, int64_t N, int64_t K) {
  int sms = 0;
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || device_sms(&sms) != RB_OK) return 0;
  return rb::mm_int4_tc_workspace(M, N, K, sms);
}

int rb_mm_int4_ws(const void* X, int x_dtype, int64_t ldx, const uint8_t* q, const uint16_t* s, const uint16_t* m,
                  void* Y, int y_dtype, int64_t ldy, int64_t M, int64_t N, int64_t K, void* ws, int64_t ws_bytes,
                  int flags, void* stream) {
  return mm_int4_impl(X, x_dtype, ldx, q, s, m, Y, y_dtype, ldy, M, N, K, ws, ws_bytes, flags, stream);
}

int rb_mm_int4_static(const void* X, int x_dtype, int64_t ldx, const uint8_t* q, const uint16_t* s, const uint16_t* m,
                      void* Y, int y_dtype, int64_t ldy, int64_t M, int64_t N, int64_t K, int flags, void* stream) {
  if (x_dtype != RB_F16 && x_dtype != RB_BF16) return RB_ERR_DTYPE;
  return mm_int4_impl(X, x_dtype, ldx, q, s, m, Y, y_dtype, ldy, M, N, K, nullptr, 0, flags, stream, true);
}

int rb_mm_int4_list(const rb_mm_desc* descs, int count, int64_t M, int x_dtype, int y_dtype, int flags,
                    void* stream) {
  if (count < 0 || M < 0 || M > (int64_t(1) << 30)) return RB_ERR_SHAPE;
  if (count == 0 || M == 0) return RB_OK;
  if (!descs) return RB_ERR_NULL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(y_dtype)) return RB_ERR_DTYPE;
  std::vector<rb::MmArgs> args;
  args.reserve(count);
  for (int i = 0; i < count; ++i) {
    const rb_mm_desc& d = descs[i];
    if (d.N < 1 || d.K <= 0 || d.K % 128 != 0 || d.N > (int64_t(1) << 30)) return RB_ERR_SHAPE;
    if (!d.X || !d.Y || !d.q || !d.s || !d.m) return RB_ERR_NULL;
    if (d.ldx < d.K || d.ldy < d.N) return RB_ERR_SHAPE;
    if (!aligned16(d.X) || !aligned16(d.Y) || (d.ldx % 8) != 0 || (d.ldy % 8) != 0) return RB_ERR_ALIGN;
    if (!aligned16(d.q) || !aligned16(d.s) || !aligned16(d.m)) return RB_ERR_ALIGN;
    rb::MmArgs a = {};
    a.X = d.X; a.x_dtype = x_dtype; a.ldx = d.ldx;
    a.q = d.q; a.s = d.s; a.m = d.m;
    a.Y = d.Y; a.y_dtype = y_dtype; a.ldy = d.ldy;
    a.M = M; a.N = d.N; a.K = d.K; a.flags = flags;
    args.push_back(a);
  }
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return st;
  st = rb::launch_mm_int4_list(args.data(), count, sms, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int rb_tp_allreduce_f16(const void* a, const void* b, void* out, int64_t n, void* const* bufs, int rank, int world,
                        uint32_t flag_off, uint32_t counter_off, int flags, void* stream) {
  if (!a || !out || !bufs) return RB_ERR_NULL;
  if (n <= 0 || world < 1 || world > 8 || rank < 0 || rank >= world) return RB_ERR_SHAPE;
  if ((flag_off % 4) != 0 || (counter_off % 4) != 0) return RB_ERR_ALIGN;
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return st;
  st = rb::launch_tp_allreduce(static_cast<const __half*>(a), static_cast<const __half*>(b), static_cast<__half*>(out),
                               n, bufs, rank, world, flag_off, counter_off, flags, static_cast<cudaStream_t>(stream));
  if (st == RB_OK && cudaGetLastError() != cudaSuccess) st = RB_ERR_LAUNCH;
  return st;
}

int rb_ipc_alloc(uint64_t bytes, void** ptr, void* handle_out) {
  if (!ptr || !handle_out) return RB_ERR_NULL;
  if (bytes == 0) return RB_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return RB_ERR_DEVICE;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(p);
    return RB_ERR_DEVICE;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return RB_OK;
}

int rb_ipc_free(void* ptr) {
  if (!ptr) return RB_ERR_NULL;
  return cudaFree(ptr) == cudaSuccess ? RB_OK : RB_ERR_DEVICE;
}

int rb_ipc_open(const void* handle, uint64_t offset, void** base, void** ptr) {
  if (!handle || !base || !ptr) return RB_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  if (cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    (void)cudaGetLastError();
    return RB_ERR_DEVICE;
  }
  *base = b;
  *ptr = static_cast<char*>(b) + offset;
  return RB_OK;
}

int rb_ipc_close(void* base) {
  if (!base) return RB_ERR_NULL;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    (void)cudaGetLastError();
    return RB_ERR_DEVICE;
  }
  return RB_OK;
}

int64_t rb_decode_layers_workspace(const rb_decode_step* st) {
  int sms = 0, s = device_sms(&sms);
  if (s != RB_OK) return -s;
  return rb::decode_layers_workspace(st, sms);
}

int rb_decode_layers(const rb_decode_step* st, int dtype, int flags, void* stream) {
  if (!st) return RB_ERR_NULL;
  if (!act_dtype_ok(dtype)) return RB_ERR_DTYPE;
  int sms = 0, s = device_sms(&sms);
  if (s != RB_OK) return s;
  s = rb::launch_decode_layers(st, dtype, flags, sms, static_cast<cudaStream_t>(stream));
  if (s == RB_OK && cudaGetLastError() != cudaSuccess) s = RB_ERR_LAUNCH;
  return s;
}

int rb_set_wait_limit(uint64_t ns, void* stream) {
  if (ns == 0) ns = rb::kMaxWaitNs;
  if (ns < 1000 || ns > 60000000000ull) return RB_ERR_SHAPE;
  int sms = 0, st = device_sms(&sms);
  if (st != RB_OK) return st;
  const unsigned long long v = ns;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyToSymbolAsync(rb::g_wait_limit_ns, &v, sizeof(v), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return RB_ERR_DEVICE;
  return RB_OK;
}

int rb_get_device_error(unsigned int* out, void* stream) {
  if (!out) return RB_ERR_NULL;
  unsigned int zero = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyFromSymbolAsync(out, rb::g_device_error, sizeof(unsigned int), 0, cudaMemcpyDeviceToHost, s) !=
      cudaSuccess)
    return RB_ERR_DEVICE;
  if (cudaMemcpyToSymbolAsync(rb::g_device_error, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, s) !=
      cudaSuccess)
    return RB_ERR_DEVICE;
  if (cudaStreamSynchronize(s) != cudaSuccess) return RB_ERR_DEVICE;
  return RB_OK;
}

}  // extern "C"
