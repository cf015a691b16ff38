/*
 * rumik_b200.h - C ABI of the B200 (sm_100a) weight-only quantised linear-layer kernels.
 *
 * These entry points are the native boundary that replaces rumik-fast's torch extension
 * (kernels/cuda_gemv.py:214-218, load_inline(... functions=["gemv_int4", "gemv_int8"])) and its Triton
 * prefill matmul (kernels/mm_int4.py:59-73). They take plain device pointers, sizes, dtype codes and a
 * cudaStream_t passed as void*. They never allocate, never synchronise, and are safe to call while a CUDA
 * graph is being captured on `stream`. Every function returns an rb_status code (0 = success); argument
 * checks run before any CUDA call, so a bad argument is reported without touching the device.
 * Several host threads may call them at once (for example one per GPU): the library's only process-wide host
 * state, a per-kernel cache of the shared-memory attribute and the static scratch's address per device, is
 * guarded. Device buffers that two calls share (a workspace, the static scratch) must be ordered by the caller.
 *
 * Weight format (kernels/int4_gemv.py:1-3, modal_export_int4.py:48-59):
 *   q  uint8 [N, K/2]   two 4-bit codes per byte, low nibble = even column, high nibble = odd column
 *   s  fp16  [N, K/128] per-group scale
 *   m  fp16  [N, K/128] per-group min;            w[n,k] = code[n,k] * s[n,k/128] + m[n,k/128]
 * int8 head (kernels/cuda_gemv.py:234-242): q uint8 [N, K] = int8 + 128 (or signed int8), one scale per row.
 *
 * Alignment: every base pointer must be 16-byte aligned, and the activation row strides (ldx) must be a
 * multiple of 8 elements; the kernels move weights with 16-byte bulk copies.
 */
#ifndef RUMIK_B200_H
#define RUMIK_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference raises RuntimeError through TORCH_CHECK (kernels/cuda_gemv.py:121,135,190);
 * the Python layer of this library turns a non-zero status into the same exception type. */
enum rb_status {
  RB_OK = 0,
  RB_ERR_NULL = 1,    /* a required pointer is NULL */
  RB_ERR_SHAPE = 2,   /* unsupported N / K / M / batch (e.g. K % 128 != 0) */
  RB_ERR_DTYPE = 3,   /* unsupported dtype code */
  RB_ERR_ALIGN = 4,   /* a pointer is not 16-byte aligned or a stride is not a multiple of 8 elements */
  RB_ERR_LAUNCH = 5,  /* the CUDA launch failed (error reported by cudaGetLastError) */
  RB_ERR_DEVICE = 6,  /* no usable sm_100 device, or a device query failed */
  RB_ERR_TIMEOUT = 7  /* a kernel gave up a bounded wait (reported by rb_get_device_error) */
};

/* Element type codes for activations, outputs and scales. */
enum rb_dtype { RB_F16 = 0, RB_BF16 = 1, RB_F32 = 2 };

/* Launch flags. */
enum rb_flags {
  /* Launch with programmatic dependent launch: the kernel may start while the previous kernel on the
   * stream is still running; it waits for that kernel (griddepcontrol.wait) before touching x or y. */
  RB_FLAG_PDL = 1,
  /* With RB_FLAG_PDL: also stream the weights (q, s, m) into shared memory BEFORE that wait. Only valid
   * when the weights are not written by the kernel immediately before this one on the stream, which holds
   * for inference weights loaded once. This is what lets a chain of GEMVs keep HBM busy across kernel
   * boundaries. rb_attn_decode with this flag reads the position and the K/V rows of the slots before it
   * ahead of the wait, and only q and the position's own slot after it: valid when the kernels just before it
   * on the stream write neither the position nor any other slot of the caches (a decode step's input launch
   * writes q and the token's slot). */
  RB_FLAG_PREFETCH_WEIGHTS = 2,
  /* GEMV lists (rb_gemv_int4_multi / _multi_ws / _fused): run on the tcgen05 kernel, or on the warp-MMA kernel,
   * whatever the list's size. Without either, lists whose codes total less than 128 MiB (a decode layer's
   * projections, latency-bound) run on the warp-MMA kernel and longer lists on the tcgen05 kernel. */
  RB_FLAG_KERNEL_TC = 4,
  RB_FLAG_KERNEL_MMA = 8,
  /* rb_attn_decode: merge the splits through global partials and a per-head ticket (the form that needs no
   * thread-block clusters) even where the device can run the cluster form. */
  RB_FLAG_ATTN_TICKET = 16
};

/*
 * int4 group-128 GEMV, batch 1..16:  y[b, n] = sum_k w[n, k] * x[b, k]   (fp32 accumulation).
 * Replaces gemv_int4(x, q, s, m, y, warps, rows) (kernels/cuda_gemv.py:130-136) and its kernel
 * gemv_int4_kernel (kernels/cuda_gemv.py:38-115); the Python wrapper gemv_int4_cuda (:226-231) calls this.
 *   x       [batch, K] activations (x_dtype RB_F16 or RB_BF16), row stride ldx elements
 *   y       [batch, N] output (y_dtype RB_F16 or RB_BF16), row stride ldy elements
 *   N >= 1, K % 128 == 0, 128 <= K <= 16384, 1 <= batch <= 16 (batch 0 or N 0: no-op)
 */
int rb_gemv_int4(const void* x, int x_dtype, int64_t ldx,
                 const uint8_t* q, const uint16_t* s, const uint16_t* m,
                 void* y, int y_dtype, int64_t ldy,
                 int64_t N, int64_t K, int64_t batch, int flags, void* stream);

/*
 * int8 per-row GEMV (tied audio head), batch 1..16:  y[b, n] = s[n] * sum_k v(q[n, k]) * x[b, k]
 *   v(q) = q - 128 for q_signed == 0 (uint8 storage of int8 + 128, as quantize_int8_rows writes it),
 *   v(q) = (int8)q  for q_signed != 0.
 * Replaces gemv_int8(x, q, s, y) (kernels/cuda_gemv.py:188-195) and gemv_int8_kernel (:141-186); the
 * Python wrapper gemv_int8_cuda (:245-249) calls this. s_dtype RB_F32 (engine) or RB_F16 (configs).
 *   N >= 1 (no padding to 16 required), K % 64 == 0, 64 <= K <= 16384, 1 <= batch <= 16
 * Batch 1 with K % 128 == 0 runs on the tcgen05 tensor cores (the codes are the 8-bit A operand, x is
 * quantised per 128-column group to 16-bit integers, delta_g = max_g|x| / 32639, each group's integer dot
 * product combined exactly in int32); other shapes on the warp-level MMA kernel.
 */
int rb_gemv_int8(const void* x, int x_dtype, int64_t ldx,
                 const uint8_t* q, int q_signed, const void* s, int s_dtype,
                 void* y, int y_dtype, int64_t ldy,
                 int64_t N, int64_t K, int64_t batch, int flags, void* stream);

/*
 * int4-weight matrix product (prefill) on tcgen05 tensor cores:  Y[t, n] = sum_k X[t, k] * w[n, k].
 * Replaces mm_int4(x, q, s, m) (kernels/mm_int4.py:59-73) and its Triton kernel _mm_int4 (:24-46).
 *   X [M, K] fp16 or bf16, row stride ldx;  Y [M, N] fp16 or bf16, row stride ldy.
 *   Each 128-row weight block is dequantised per group to fp16 straight into tensor memory, the A operand of
 *   tcgen05.mma.kind::f16 (the weights never exist wider than int4 in HBM or shared memory); X tiles arrive by
 *   TMA and a bf16 X is converted to fp16 in shared memory (exact for |x| <= 65504). fp32 accumulation.
 *   M == 1 is a GEMV and runs as rb_gemv_int4. This entry point never splits K (no workspace); see
 *   rb_mm_int4_ws and rb_mm_int4_static for the split that fills idle SMs on calls with few tiles.
 *   M >= 1, N >= 1, K % 128 == 0.
 */
int rb_mm_int4(const void* X, int x_dtype, int64_t ldx,
               const uint8_t* q, const uint16_t* s, const uint16_t* m,
               void* Y, int y_dtype, int64_t ldy,
               int64_t M, int64_t N, int64_t K, int flags, void* stream);

/*
 * The same product with a caller-provided fp32 workspace, which lets a call whose 128-row x token-chunk tiles
 * would leave SMs idle (small N or few tokens) split K into slices: every slice writes its fp32 partial to the
 * workspace and a second kernel adds the slices in slice order into Y (deterministic). rb_mm_int4_workspace
 * returns the bytes this needs for (M, N, K) on the current device (0: no split, ws may be NULL); a smaller
 * workspace runs the call without a split.
 */
int64_t rb_mm_int4_workspace(int64_t M, int64_t N, int64_t K);

/*
 * rb_mm_int4_ws for callers that cannot allocate device memory: the split-K partials go to a file-scope
 * `static __device__` scratch array of 8 MiB (8,388,608 bytes) inside this library, so the call allocates
 * nothing. Returns RB_ERR_SHAPE when the split it would use needs more than 8 MiB
 * (rb_mm_int4_workspace(M, N, K) > 8 MiB); nothing in the scratch needs to start at zero. The scratch is one
 * per device and shared by every call: calls that overlap in time (on two streams, or otherwise not ordered
 * one after the other) race on it. Consecutive calls on one stream are safe. The scratch's device address is
 * looked up (cudaGetSymbolAddress) on the first call that splits on each device and kept for the life of the
 * process: do not use this entry point across a cudaDeviceReset of that device.
 */
int rb_mm_int4_static(const void* X, int x_dtype, int64_t ldx,
                      const uint8_t* q, const uint16_t* s, const uint16_t* m,
                      void* Y, int y_dtype, int64_t ldy,
                      int64_t M, int64_t N, int64_t K, int flags, void* stream);
int rb_mm_int4_ws(const void* X, int x_dtype, int64_t ldx,
                  const uint8_t* q, const uint16_t* s, const uint16_t* m,
                  void* Y, int y_dtype, int64_t ldy,
                  int64_t M, int64_t N, int64_t K, void* ws, int64_t ws_bytes, int flags, void* stream);

/* One prefill product of a list: Y [M, N] = X [M, K] * w^T, the layout of rb_mm_int4 (M is the list's). */
typedef struct rb_mm_desc {
  const void* X;        /* [M, K], row stride ldx elements (multiple of 8), 16-byte aligned */
  int64_t ldx;
  const uint8_t* q;     /* codes [N, K/2] */
  const uint16_t* s;    /* fp16 scales [N, K/128] */
  const uint16_t* m;    /* fp16 mins [N, K/128] */
  void* Y;              /* [M, N], row stride ldy elements (multiple of 8), 16-byte aligned */
  int64_t ldy;
  int64_t N;            /* >= 1 */
  int64_t K;            /* multiple of 128 */
} rb_mm_desc;

/*
 * A list of independent prefill products with one token count M (one x dtype, one y dtype) in persistent
 * launches of up to 52 products each: the work items of every product (128-row weight block x token chunk) are
 * dealt round-robin to one CTA per SM, so the list pays one launch, one pipeline fill and one tail instead of one
 * per product, and needs no split-K workspace. The arithmetic is rb_mm_int4's. No reference counterpart as a
 * single call: it runs what rumik-fast's prefill benchmark issues as one mm_int4 per matrix
 * (kernels/mm_int4.py:94-101), or a layer's products that share their input (QKV and gate_up). `descs` is a host
 * array read during the call; every X must be ready and no Y may alias another product's inputs.
 */
int rb_mm_int4_list(const rb_mm_desc* descs, int count, int64_t M, int x_dtype, int y_dtype, int flags,
                    void* stream);

/* One int4 GEMV of a list (host-side description, read by rb_gemv_int4_multi during the call). */
typedef struct rb_gemv_desc {
  const void* x;        /* activations [K] (dtype x_dtype of the call), 16-byte aligned */
  void* y;              /* output [N] (dtype y_dtype of the call) */
  const uint8_t* q;     /* codes [N, K/2] */
  const uint16_t* s;    /* fp16 scales [N, K/128] */
  const uint16_t* m;    /* fp16 mins [N, K/128]; unused (may be NULL) when s_row is set */
  int64_t N;            /* >= 1 */
  int64_t K;            /* multiple of 128, <= 16384 */
  /* NULL: s and m are the reference's fp16 scales and mins. Set: 8-bit double-quantised scales - s holds one
   * 16-bit word per group [N, K/128] (low byte b: scale code, high byte z: zero point in 1/16 steps) and s_row
   * the fp32 per-row scale factors [N] (4-byte aligned). They decode to the fp16 scale and min of the fp16
   * format: scale = fp16(2^((b >> 4) - 15) * (1 + (b & 15) / 16) * s_row[n]), min = fp16(-(z / 16) * scale)
   * (rumik_fast_b200/scales8.py packs them). Such entries run on the tcgen05
   * kernel only (with RB_FLAG_KERNEL_MMA or fused attention: RB_ERR_SHAPE). No reference counterpart: the
   * byte saving rumik-fast names as its next step (engine/README.md:192-193). */
  const float* s_row;
  /* 0: an int4 entry as above. RB_W8_SIGNED / RB_W8_OFFSET: an int8 entry, y = s * (q @ x) - the int8 head
   * (gemv_int8, kernels/cuda_gemv.py:138-195) streamed as more rows of the same launch. q holds int8 codes
   * [N, K] (RB_W8_OFFSET: uint8 = int8 + 128, quantize_int8_rows' storage), 16-byte aligned; the per-row scales
   * [N] are s_row (fp32, 4-byte aligned) or, when s_row is NULL, s (fp16); m is unused. Such entries run on the
   * tcgen05 kernel only, with the store epilogue (RB_FLAG_KERNEL_MMA or another epilogue: RB_ERR_SHAPE). */
  int w8;
} rb_gemv_desc;
enum rb_w8 { RB_W8_NONE = 0, RB_W8_SIGNED = 1, RB_W8_OFFSET = 2 };

/*
 * A list of independent int4 GEMVs (batch 1) in one persistent launch: y_i = W_i x_i for every entry.
 * No reference counterpart as a single call: it executes what rumik-fast's projection-set benchmark
 * (kernels/bench_gemv.py:83-113) issues as one gemv_int4 launch per matrix, without the per-launch cost.
 * Runs on the tcgen05 tensor cores: the int4 codes are the unsigned 8-bit A operand in tensor memory and each
 * x_i is quantised per 128-column group to 16-bit integers (delta = max|x| / 32639; error below 2e-5 of the
 * group's largest |x|) split into two signed bytes. Every x_i must be ready when the launch starts and no y_i
 * may alias another entry's inputs. `descs` is a host array, copied into the launch (at most 160 entries and 8
 * distinct activation vectors per launch; longer lists are split into several launches).
 */
int rb_gemv_int4_multi(const rb_gemv_desc* descs, int count, int x_dtype, int y_dtype, int flags, void* stream);

/*
 * The same list with a caller-provided workspace that lets a launch with few 128-row blocks (fewer than
 * 3 x the SM count: a decode layer's projections, 18-35 MB, rather than a whole step's) split K. Each block's
 * pairs of groups are cut into slices run by different converter sets; every slice writes its fp32 partial sums
 * to the workspace, and the block's last slice to finish (a per-block counter in the workspace) adds them in slice
 * order - the result does not depend on which finishes last - and stores the rows.
 * rb_gemv_int4_workspace returns the bytes a list needs on the current device with those launch flags (0: no
 * split, e.g. a list that runs on the warp-MMA kernel, which splits K inside each CTA; negative: -status).
 * The workspace must be 16-byte aligned and zero before its first use; every launch leaves it zero again
 * (except after a device error, when it must be cleared). A smaller workspace runs the list unsplit. Calls
 * sharing a workspace must not overlap in time (one stream).
 */
int64_t rb_gemv_int4_workspace(const rb_gemv_desc* descs, int count, int flags);
int rb_gemv_int4_multi_ws(const rb_gemv_desc* descs, int count, void* ws, int64_t ws_bytes, int x_dtype, int y_dtype,
                          int flags, void* stream);

/*
 * Decode-layer glue fused into the GEMV launch (rumik-fast engine/fused.py): an add + LayerNorm prologue that
 * produces the activations of the GEMVs, and per-entry epilogues that route each GEMV's rows to where the
 * engine's next kernels read them. One call replaces, per layer, the engine's
 *     add_ln (engine/fused.py:29-40)  ->  gemv(w_in) (engine/rumik_fused.py:84)  ->  post (engine/fused.py:43-84)
 * launch sequence (engine/rumik_fused.py:84-87,115-116).
 *
 * Prologue (rb_add_ln), engine/fused.py:29-40:  s = x + a + b in fp32, rounded to the activation dtype
 * (the new residual, written to x_out), then h = (s - mean(s)) * rsqrt(var(s) + eps) * w, rounded to the
 * activation dtype (Cohere LayerNorm: centred, no bias). Entries whose `x` is NULL multiply h. H % 128 == 0,
 * H <= 12288. x_out (and h_out, optional) must not overlap x, a, b or w: every CTA reads x while one writes
 * x_out, so the residual stream alternates between two buffers.
 *
 * Epilogues (rb_gemv_epi), engine/fused.py:43-84, on the GEMV result rounded to the output dtype as the
 * engine's y buffer would hold it:
 *   RB_EPI_STORE    y[n] (as rb_gemv_int4_multi).
 *   RB_EPI_ROPE_KV  rows are n_q_heads query heads, n_kv_heads key heads, n_kv_heads value heads of head_dim
 *                   rows each (N = (n_q_heads + 2 n_kv_heads) head_dim, head_dim even). With `rope`, query and
 *                   key heads are rotated by the interleaved rotary embedding at position *pos (pairs (2j, 2j+1),
 *                   cos/sin [cache_len, head_dim] at [pos, 2j]); queries go to q_out [n_q_heads, head_dim],
 *                   keys and values to slot *pos of k_cache / v_cache [n_kv_heads, cache_len, head_dim].
 *   RB_EPI_SWIGLU   rows hold gate and up channels in pairs: row 2c = gate channel c, row 2c + 1 = up channel c
 *                   (Python helper interleave_gate_up); act_out[c] = silu(gate[c]) * up[c], N / 2 channels,
 *                   N even.
 * cos, sin, q_out, the caches and act_out are in the output dtype. `y` may be NULL for ROPE_KV and SWIGLU
 * (when given, the plain result is stored as well). *pos is read on the device (int64); a position outside
 * [0, cache_len) stores no query, key or value and sets the RB_DEVERR_ARG bit of the device error word.
 * At most 160 entries and 8 activation vectors (the whole call is one launch), at most 4 ROPE_KV / SWIGLU
 * entries.
 */
typedef struct rb_add_ln {
  const void* x;        /* residual stream [H] (activation dtype) */
  const void* a;        /* added term [H] or NULL (e.g. the o_proj output) */
  const void* b;        /* added term [H] or NULL (e.g. the down_proj output) */
  const void* w;        /* LayerNorm weight [H] (activation dtype) */
  void* x_out;          /* new residual x + a + b [H], or NULL */
  void* h_out;          /* the normalised vector [H], or NULL */
  int64_t H;
  float eps;
  /* Token-embedding source (engine/fused.py:18-27, embed_ln): with emb_q non-NULL the residual is the token's
   * int8 embedding row times its scale, s = round(emb_q[tok, :] * emb_s[tok]), instead of x + a + b (x, a, b
   * must then be NULL). emb_q int8 [vocab, H]; emb_s [vocab] of dtype emb_s_dtype (RB_F32 or RB_F16); tok a
   * device pointer to the int64 token id. A token outside [0, vocab) reads row 0 and sets RB_DEVERR_ARG. */
  const int8_t* emb_q;
  const void* emb_s;
  const int64_t* tok;
  int64_t vocab;
  int emb_s_dtype;
} rb_add_ln;

enum rb_epi_kind { RB_EPI_STORE = 0, RB_EPI_ROPE_KV = 1, RB_EPI_SWIGLU = 2 };

typedef struct rb_gemv_epi {
  int kind;                  /* rb_epi_kind */
  int rope;                  /* RB_EPI_ROPE_KV: rotate the query and key heads (0 = copy only) */
  int n_q_heads, n_kv_heads, head_dim;
  int64_t cache_len;         /* slots per head in k_cache / v_cache */
  const int64_t* pos;        /* device pointer to the position */
  const void* cos;           /* [cache_len, head_dim] */
  const void* sin;
  void* q_out;               /* [n_q_heads, head_dim] */
  void* k_cache;             /* [n_kv_heads, cache_len, head_dim] */
  void* v_cache;
  void* act_out;             /* RB_EPI_SWIGLU: [N / 2] */
} rb_gemv_epi;

/* Device error bit set by rb_gemv_int4_fused when *pos is outside [0, cache_len). */
#define RB_DEVERR_ARG (1u << 9)

/*
 * Decode attention fused into a GEMV launch (the o_proj input of a layer; rb_attn_decode's attention, in the
 * same launch as the layer's o_proj and down_proj). Entries whose `x` equals `out` read the attention output,
 * which the launch computes and also stores to `out`; they must come last in the list. The other entries (the
 * down_proj of the layer, whose input is ready at launch) stream while the attention runs. Fields as
 * rb_attn_decode; ws: rb_attn_decode_workspace(...) bytes, its first 512 bytes zero before the first use (every
 * launch leaves them zero). 1 <= n_q_heads / n_kv_heads <= 4. Such a launch always runs on the warp-MMA kernel
 * (RB_FLAG_KERNEL_TC: RB_ERR_SHAPE) and the whole list must fit one launch.
 */
typedef struct rb_attn_src {
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const int64_t* pos;
  void* out;
  int n_q_heads, n_kv_heads, head_dim;
  int64_t cache_len;
  float scale;
  void* ws;
  int64_t ws_bytes;
} rb_attn_src;

/* descs[i], epis[i] (epis may be NULL: all RB_EPI_STORE); ln may be NULL (no entry may then have x == NULL);
 * attn may be NULL. ws / ws_bytes: the split-K workspace of rb_gemv_int4_multi_ws
 * (rb_gemv_int4_workspace(descs, count, flags) bytes), or NULL / 0. A split entry runs its epilogue in the last
 * slice of each block. */
int rb_gemv_int4_fused(const rb_gemv_desc* descs, const rb_gemv_epi* epis, int count, const rb_add_ln* ln,
                       const rb_attn_src* attn, void* ws, int64_t ws_bytes, int x_dtype, int y_dtype, int flags,
                       void* stream);

/* The add + LayerNorm alone (engine/fused.py:29-40 as launched at engine/rumik_fused.py:115-116 for the final
 * norm in front of the head): one CTA; results bit-identical to rb_gemv_int4_fused's prologue. dtype is the
 * activation dtype of every vector. */
int rb_add_layernorm(const rb_add_ln* ln, int dtype, int flags, void* stream);

/*
 * Decode attention of one token over the KV cache, grouped-query heads, ONE launch. Replaces rumik-fast's
 * flash-decoding pair attn_split + attn_combine (engine/fused.py:120-200, launched at
 * engine/rumik_fused.py:88-94) and its single-kernel form attn (engine/fused.py:92-118):
 *   out[h] = sum_{t <= *pos} softmax_t(q[h] . k_cache[h / rep, t] * scale) v_cache[h / rep, t]
 *   q [n_q_heads, head_dim], k_cache / v_cache [n_kv_heads, cache_len, head_dim], out [n_q_heads, head_dim], all
 *   in `dtype` (RB_F16 / RB_BF16); *pos on the device (int64), 0 <= *pos < cache_len, else nothing is written
 *   and the RB_DEVERR_ARG bit of the device error word is set. head_dim == 128, rep = n_q_heads / n_kv_heads
 *   in 1..8, n_kv_heads <= 64. Scores, softmax and the weighted sum are fp32.
 *   Where the device can schedule them, one thread-block cluster of 8 CTAs of 8 warps per key-value head splits the slots
 *   and merges its splits through distributed shared memory (the workspace is then untouched); otherwise, or
 *   with RB_FLAG_ATTN_TICKET, about SMs / n_kv_heads CTAs per head merge through fp32 partials in the workspace.
 *   ws: rb_attn_decode_workspace(...) bytes of device memory, 16-byte aligned; its first 256 bytes (per-head
 *   completion counters) must be zero before the first call and are zero again after each call. Calls that
 *   share a workspace must not overlap in time (one stream).
 */
/*
 * The sampling tail of a decode step (rumik-fast engine/sample.py, the same maths as
 * engine/rumik_int4.py:174-198): the stop predictor, top-k over the audio head's logits, a Gumbel-max draw and the
 * device-side counters, in two launches:
 *   stop  = W2 . gelu(W1 . LayerNorm(h; ln_w, ln_b, eps 1e-5) + b1) + b2 > 0    (counted once *step >= min_new)
 *   token = ids[argmax_{j < top_k}(top_j * inv_temp - log(-log(clamp(u_j, 1e-10, 1))))]
 * where top_j is the j-th largest logit (ties: the higher row first) with row end_idx masked to -inf while
 * *step < min_new; then out[*step] = token (if *step < out_len), *tok = token, *step += 1. The first of equal
 * scores wins. u: top_k uniforms drawn by the caller (the reference draws them with torch.rand).
 * logits [n_vocab] (RB_F16 / RB_BF16 / RB_F32), n_vocab <= 32768, 1 <= top_k <= 32; h [H] (H <= 8192);
 * w1 [nz, H] (any of the three dtypes, 16-byte aligned); ln_w, ln_b [H], b1, w2 [nz], b2 [1] fp32;
 * ws: rb_sample_workspace(nz) bytes of device scratch, 16-byte aligned.
 */
typedef struct rb_sampler {
  const void* logits;
  int logits_dtype;
  int64_t n_vocab;
  int64_t end_idx;
  const int64_t* ids;
  int top_k;
  float inv_temp;
  const float* u;
  const void* h;
  int h_dtype;
  int64_t H;
  const float* ln_w;
  const float* ln_b;
  const void* w1;
  int w1_dtype;
  int nz;
  const float* b1;
  const float* w2;
  const float* b2;
  int64_t end_id;
  int64_t min_new;
  int64_t* step;
  int64_t* tok;
  int64_t* out;
  int64_t out_len;
  void* ws;
} rb_sampler;

int64_t rb_sample_workspace(int nz);
int rb_sample(const rb_sampler* s, int flags, void* stream);

int64_t rb_attn_decode_workspace(int n_q_heads, int n_kv_heads, int head_dim);
int rb_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                   int n_q_heads, int n_kv_heads, int head_dim, int64_t cache_len, float scale, void* ws,
                   int64_t ws_bytes, int dtype, int flags, void* stream);

/*
 * Tensor-parallel per-layer reduction over NVLink peer memory:  out[i] = sum over ranks of (a[i] + b[i]).
 * Replaces the add + all-reduce that follows a row-parallel layer pair (o_proj and down partials) in a
 * tensor-parallel decode step; no reference counterpart (the reference engine runs on one GPU).
 *   a, b, out  fp16 [n] on this rank's device (b may be NULL); 1 <= n <= 2^24
 *   bufs       the `world` ranks' symmetric buffers (device pointers mapped into this process, bufs[rank] the
 *              local one), each at least 8 * world * n bytes of data at offset 0, `world` uint32 flags at
 *              flag_off and one uint32 counter at counter_off, all zero before the first call
 * Every rank must make the same sequence of calls. A peer that does not arrive within the wait limit (4 s unless
 * rb_set_wait_limit changed it) sets a bit in the device error word (rb_get_device_error). 1 <= world <= 8.
 */
int rb_tp_allreduce_f16(const void* a, const void* b, void* out, int64_t n, void* const* bufs, int rank, int world,
                        uint32_t flag_off, uint32_t counter_off, int flags, void* stream);

/*
 * Setup for rb_tp_allreduce_f16 (not part of the GEMV path, which never allocates): a zeroed device buffer of
 * `bytes` on the current device from cudaMalloc, and its 64-byte cudaIpcMemHandle_t in handle_out for the
 * other ranks. Release with rb_ipc_free.
 */
int rb_ipc_alloc(uint64_t bytes, void** ptr, void* handle_out);
int rb_ipc_free(void* ptr);

/*
 * Map another process's device buffer (a 64-byte cudaIpcMemHandle_t of its allocation plus the buffer's byte
 * offset in it) into this process for the CURRENT device, with peer access enabled between the current device
 * and the buffer's device. *base receives the mapped allocation (pass it to rb_ipc_close), *ptr the buffer.
 * Setup for rb_tp_allreduce_f16; no kernel is launched.
 */
int rb_ipc_open(const void* handle, uint64_t offset, void** base, void** ptr);
int rb_ipc_close(void* base);

/* One transformer layer of a decode step (rb_decode_layers). The GEMV descriptors' x and y are not used. */
typedef struct rb_decode_layer {
  rb_gemv_desc qkv;      /* q|k|v rows: N = (n_q_heads + 2 n_kv_heads) head_dim, K = H (fp16 scales) */
  rb_gemv_desc gate_up;  /* gate and up rows interleaved (row 2c = gate c, 2c + 1 = up c): N = 2 I, K = H */
  rb_gemv_desc o_proj;   /* N = H, K = n_q_heads head_dim */
  rb_gemv_desc down;     /* N = H, K = I */
  const void* ln_w;      /* LayerNorm weight [H] of this layer's input */
  void* k_cache;         /* [n_kv_heads, cache_len, head_dim]: slot *pos is written */
  void* v_cache;
  int rope;              /* rotary embedding of q and k (0: none) */
} rb_decode_layer;

/* A decode step's layers and the buffers they pass on. Buffers marked [2] alternate by layer: the layer with step
 * index g (first_layer + its index in layers) writes copy g & 1 and reads what layer g - 1 wrote in copy
 * (g - 1) & 1. All activation buffers have the call's dtype. */
typedef struct rb_decode_step {
  const rb_decode_layer* layers;
  int n_layers;          /* 1 .. 36 per call; a longer step is several calls, first_layer advancing */
  int first_layer;       /* step index of layers[0]; 0: its input is the token's int8 embedding row */
  int64_t H, I;          /* hidden size, MLP channels: multiples of 256 */
  int n_q_heads, n_kv_heads, head_dim;  /* head_dim 128; 1 .. 4 query heads per key-value head */
  int64_t cache_len;
  float eps;             /* LayerNorm epsilon */
  float attn_scale;      /* softmax scale of q . k */
  const int64_t* pos;    /* device: the token's position (its cache slot) */
  const void* cos;       /* [cache_len, head_dim] rotary tables (engine/rumik_int4.py:107-109) */
  const void* sin;
  const int8_t* emb_q;   /* first_layer == 0: int8 token embeddings [vocab, H] */
  const void* emb_s;     /* their per-row scales, dtype emb_s_dtype (RB_F32 or RB_F16) */
  int emb_s_dtype;
  const int64_t* tok;    /* device: the token id */
  int64_t vocab;
  void* resid[2];        /* residual stream x [H] */
  void* q_out[2];        /* rotated queries [n_q_heads * head_dim] */
  void* attn_out[2];     /* attention output [n_q_heads * head_dim] */
  void* act[2];          /* silu(gate) * up [I] */
  void* o_out[2];        /* o_proj output [H] */
  void* down_out[2];     /* down_proj output [H] */
  void* ws;              /* rb_decode_layers_workspace() bytes, zeroed once; every call leaves it zeroed */
  int64_t ws_bytes;
} rb_decode_step;

/*
 * A decode step's transformer layers as ONE persistent launch (one CTA per SM, cooperative): per layer
 * h = LayerNorm(x + o_out + down_out) (layer 0: the token's embedding row), x stored to resid; QKV and gate_up
 * of h with rope, the KV-cache write at *pos and silu(gate) * up; the decode attention; down_proj and o_proj.
 * The same results as the per-layer launches (rb_gemv_int4_fused for the input side, rb_attn_decode,
 * rb_gemv_int4_multi for o_proj + down_proj) up to the order of fp32 additions. Replaces the per-layer
 * launch sequence of engine/rumik_fused.py:97-121 (the add_ln / gemv / post / attention / gemv calls). After
 * it the step's final add + LayerNorm (rb_add_layernorm on resid, o_out, down_out of the last layer) and the
 * head follow. dtype: RB_F16 or RB_BF16. A wait that runs out sets bit 11 (0x800) of the device error word and
 * aborts the launch (rb_get_device_error).
 */
int64_t rb_decode_layers_workspace(const rb_decode_step* st);
int rb_decode_layers(const rb_decode_step* st, int dtype, int flags, void* stream);

/* Human-readable text for a status code (static storage). */
const char* rb_status_string(int status);

/* Library ABI version (major * 100 + minor). */
int rb_version(void);

/* Read and clear the device-side error word of the current device (bit set by a kernel that gave up a
 * bounded wait). Synchronises `stream`. *out receives the word; returns RB_OK or RB_ERR_DEVICE. */
int rb_get_device_error(unsigned int* out, void* stream);

/* Set the longest a kernel of this library waits on the CURRENT device for anything another thread, CTA or rank
 * must provide (an mbarrier phase, a peer's flag, a completion counter) before it gives up: it then sets its bit
 * in the device error word, skips the work that depended on the wait and returns, so the context stays usable.
 * ns = 0 restores the default of 4 s; otherwise 1000 <= ns <= 6e10. Affects kernels launched after the call
 * (it synchronises `stream`). A short limit is for tests that let a wait run out on purpose. No reference
 * counterpart (the reference's kernels do not wait on one another). */
int rb_set_wait_limit(uint64_t ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RUMIK_B200_H */
