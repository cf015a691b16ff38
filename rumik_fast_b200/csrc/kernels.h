// kernels.h - internal launcher interface between the C ABI (capi.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/rumik_b200.h"

namespace rb {

// Arguments of one GEMV call after validation (sizes in elements; strides in elements of x/y).
struct GemvArgs {
  const void* x;
  int x_dtype;
  int64_t ldx;
  const uint8_t* q;
  const uint16_t* s;  // int4: per-group scale; int8: unused
  const uint16_t* m;  // int4: per-group min;   int8: unused
  const void* s_row;  // int8: per-row scale (fp32 or fp16)
  int s_dtype;        // int8: RB_F32 or RB_F16
  int q_signed;       // int8: codes are signed int8
  void* y;
  int y_dtype;
  int64_t ldy;
  int64_t N, K, batch;
  int flags;
};

struct MmArgs {
  const void* X;
  int x_dtype;
  int64_t ldx;
  const uint8_t* q;
  const uint16_t* s;
  const uint16_t* m;
  void* Y;
  int y_dtype;
  int64_t ldy;
  int64_t M, N, K;
  int flags;
  float* ws;          // split-K partials [kslices][M][N] fp32, or NULL (no split)
  int64_t ws_bytes;
};

int launch_gemv_int4(const GemvArgs& a, int num_sms, cudaStream_t stream);
int launch_gemv_int8(const GemvArgs& a, int num_sms, cudaStream_t stream);
int launch_gemv_int8_tc(const GemvArgs& a, int num_sms, cudaStream_t stream);
int launch_mm_int4_tc(const MmArgs& a, int num_sms, cudaStream_t stream);
// count products with one M, one x dtype and one y dtype, in persistent launches of up to 52 matrices each
int launch_mm_int4_list(const MmArgs* a, int count, int num_sms, cudaStream_t stream);
int64_t mm_int4_tc_workspace(int64_t M, int64_t N, int64_t K, int num_sms);
int launch_mm_int4_tc_static(MmArgs a, int num_sms, cudaStream_t stream);
int launch_tp_allreduce(const __half* a, const __half* b, __half* out, int64_t n, void* const* bufs, int rank,
                        int world, uint32_t flag_off, uint32_t counter_off, int flags, cudaStream_t stream);
int launch_gemv_int4_multi(const rb_gemv_desc* d, int count, int x_dtype, int y_dtype, int flags, int num_sms,
                           cudaStream_t stream, const rb_gemv_epi* epi = nullptr, const rb_add_ln* ln = nullptr,
                           const rb_attn_src* attn = nullptr);
// The sampling tail (sample.cu): stop predictor, top-k, Gumbel-max pick, counters.
int launch_sample(const rb_sampler* s, int flags, cudaStream_t stream);
int64_t sample_workspace(int nz);
// Decode attention (attn_decode.cu): workspace bytes (-1: unsupported shape) and the launch.
int64_t attn_decode_workspace(int nq, int nkv, int hd);
int64_t decode_layers_workspace(const rb_decode_step* d, int num_sms);
int launch_decode_layers(const rb_decode_step* d, int dtype, int flags, int num_sms, cudaStream_t stream);
int launch_attn_decode(const void* q, const void* kc, const void* vc, const int64_t* pos, void* out, int nq, int nkv,
                       int64_t S, float scale, void* ws, int dtype, int flags, int num_sms, cudaStream_t stream);
// The add + LayerNorm of rb_add_layernorm (one CTA), bit-identical to the prologue of rb_gemv_int4_fused.
int launch_add_ln(const rb_add_ln* ln, int dtype, int flags, cudaStream_t stream);
// epi (per entry, may be null) and ln (may be null): the fused decode-layer glue of rb_gemv_int4_fused; a call
// with either must fit one launch (RB_ERR_SHAPE otherwise).
// ws / ws_bytes: split-K workspace (may be null: no split). With `query` non-null nothing is launched and
// *query receives the workspace bytes the launches of this list would use.
int launch_gemv_int4_tc(const rb_gemv_desc* d, int count, int x_dtype, int y_dtype, int flags, int num_sms,
                        cudaStream_t stream, const rb_gemv_epi* epi = nullptr, const rb_add_ln* ln = nullptr,
                        void* ws = nullptr, int64_t ws_bytes = 0, int64_t* query = nullptr);

}  // namespace rb
