// attn_decode.cu - decode attention of one token over the KV cache (grouped-query heads), one launch on B200.
//
// o_h = sum_{t <= pos} softmax_t(q_h . k_t * scale) v_t for every query head h, k/v from key-value head
// h / rep: rumik-fast's decode attention (engine/fused.py:92-118, split as :120-200, launched at
// engine/rumik_fused.py:88-97; eager form engine/rumik_int4.py:163-171,217).
//
// Grid = n_kv_heads x nsplit CTAs (nsplit ~ SMs / n_kv_heads); the filled slots 0..pos are cut into nsplit
// chunks whose length is computed from *pos on the device (one CUDA graph serves every position). A CTA reads
// its chunk of K and V once for all `rep` query heads of its key-value head. Each warp takes 8 slots per step
// (the next step's rows are loaded during this step's math):
// every lane holds 4 of the 128 dimensions of each row (8-byte loads, one 256-byte row per warp-load), the 8
// x rep partial dot products are reduced across the warp with a butterfly that sums 8 values in 9 shuffles,
// and an online softmax (running max, running sum, rescaled accumulator) folds them in. The CTA merges its
// warps and writes an fp32 partial (acc, max, sum); the last CTA of each key-value head to finish (an atomic
// ticket) merges the nsplit partials in split order and writes the heads' outputs, so no second launch.
// HBM-bound at long contexts: 2 x (pos + 1) x 256 bytes per key-value head.
// With programmatic dependent launch and RB_FLAG_PREFETCH_WEIGHTS, a CTA loads the position and its first step's
// K/V rows of the slots before the position ahead of griddepcontrol.wait, so that round trip overlaps the tail of
// the launch before it (the layer's input launch, which writes only q and the position's slot); q and that slot
// are read after the wait.
#include "attn.cuh"
#include "kernels.h"

namespace rb {

namespace attn {

template <int REP>
__global__ void __launch_bounds__(kThreads) attn_decode_kernel(const __grid_constant__ AttnParams p) {
  __shared__ float sm_m[kWarps][REP], sm_l[kWarps][REP];
  __shared__ __align__(16) float sm_o[kWarps][REP][kHd];
  __shared__ int is_last;
  griddep_launch_dependents();
  if (p.pre) {  // the early loads, then the wait (inside)
    attn_cta<REP, false, false, true>(p, blockIdx.x / p.nsplit, blockIdx.x % p.nsplit, threadIdx.x, 0, sm_m, sm_l,
                                      sm_o, &is_last);
  } else {
    griddep_wait();  // q and the cache slot of this token come from the previous kernel
    attn_cta<REP, false>(p, blockIdx.x / p.nsplit, blockIdx.x % p.nsplit, threadIdx.x, 0, sm_m, sm_l, sm_o,
                         &is_last);
  }
}


}  // namespace attn

int64_t attn_decode_workspace(int nq, int nkv, int hd) {
  using namespace attn;
  if (hd != kHd || nkv < 1 || nkv > kMaxKv || nq < nkv || nq % nkv != 0 || nq / nkv > kMaxRep) return -1;
  return kTicketBytes + static_cast<int64_t>(nq) * kMaxSplit * (kHd + 2) * 4;
}

int launch_attn_decode(const void* q, const void* kc, const void* vc, const int64_t* pos, void* out, int nq, int nkv,
                       int64_t S, float scale, void* ws, int dtype, int flags, int num_sms, cudaStream_t stream) {
  using namespace attn;
  AttnParams p;
  p.q = q;
  p.kc = kc;
  p.vc = vc;
  p.pos = pos;
  p.out = out;
  p.S = S;
  p.scale = scale;
  p.bf16 = dtype == RB_BF16;
  p.nsplit = static_cast<int>(nsplit_for(nkv, num_sms));
  p.pre = (flags & RB_FLAG_PDL) && (flags & RB_FLAG_PREFETCH_WEIGHTS) ? 1 : 0;
  uint8_t* w = static_cast<uint8_t*>(ws);
  p.ticket = reinterpret_cast<unsigned int*>(w);
  p.heads_done = nullptr;
  p.po = reinterpret_cast<float*>(w + kTicketBytes);
  p.pm = p.po + static_cast<int64_t>(nq) * p.nsplit * kHd;
  p.pl = p.pm + static_cast<int64_t>(nq) * p.nsplit;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nkv * p.nsplit);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (flags & RB_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (nq / nkv) {
    case 1: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<1>, p); break;
    case 2: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<2>, p); break;
    case 3: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<3>, p); break;
    case 4: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<4>, p); break;
    case 5: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<5>, p); break;
    case 6: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<6>, p); break;
    case 7: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<7>, p); break;
    case 8: e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<8>, p); break;
    default: return RB_ERR_SHAPE;
  }
  return e == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

}  // namespace rb
