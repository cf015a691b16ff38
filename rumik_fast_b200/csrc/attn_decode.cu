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
//
// Cluster form (the default where the device can co-schedule it): one cluster of kClusterSplits CTAs of
// kClusterWarps warps per key-value head. Each CTA stores its merged partial of query head r straight into the shared memory of CTA r of
// the cluster (distributed shared-memory stores); after one cluster barrier (release / acquire) CTA r merges head r
// from its own shared memory and writes it. No global partials, no ticket, no workspace traffic.
#include <atomic>

#include <cooperative_groups.h>

#include "attn.cuh"
#include "kernels.h"

namespace rb {

namespace attn {

// Splits per key-value head = CTAs per cluster, and warps per CTA: 8 x 8 measured faster than 16 x 4 (same warps
// per head and slots per warp, half the SMs, so more of the next launch's CTAs start beside it) and needs no
// non-portable cluster size.
#ifndef RB_ATTN_CLUSTER
#define RB_ATTN_CLUSTER 8
#endif
constexpr int kClusterSplits = RB_ATTN_CLUSTER;
#ifndef RB_ATTN_CLUSTER_WARPS
#define RB_ATTN_CLUSTER_WARPS 8
#endif
constexpr int kClusterWarps = RB_ATTN_CLUSTER_WARPS;  // warps per CTA of the cluster form
constexpr int kClusterThreads = kClusterWarps * 32;

template <int REP>
__global__ void __launch_bounds__(kClusterThreads) attn_cluster_kernel(const __grid_constant__ AttnParams p) {
  static_assert(REP <= kClusterSplits, "one merging CTA per query head of the group");
  namespace cg = cooperative_groups;
  __shared__ float sm_m[kClusterWarps][REP], sm_l[kClusterWarps][REP];
  __shared__ __align__(16) float sm_o[kClusterWarps][REP][kHd];
  __shared__ float cml[2 * REP];
  __shared__ int is_last;
  // the merging CTA's inbox (CTA r merges query head r of the group): every split's accumulator, maximum and sum
  __shared__ __align__(16) float in_o[kClusterSplits][kHd];
  __shared__ float in_m[kClusterSplits], in_l[kClusterSplits];
  griddep_launch_dependents();
  cg::cluster_group cl = cg::this_cluster();
  // Cluster barrier phase 1, split: arrive now, wait just before the first store into another CTA's shared memory,
  // so that no store reaches a CTA of the cluster that has not started. Every thread of every CTA takes both
  // phases whatever its path, so that no CTA can wait for one that took another path.
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  const int g = blockIdx.x / kClusterSplits, sp = static_cast<int>(cl.block_rank()), tid = threadIdx.x;
  int active;
  if (p.pre) {
    active = attn_cta<REP, false, false, true, true, kClusterWarps>(p, g, sp, tid, 0, sm_m, sm_l, sm_o, &is_last, cml);
  } else {
    griddep_wait();
    active = attn_cta<REP, false, false, false, true, kClusterWarps>(p, g, sp, tid, 0, sm_m, sm_l, sm_o, &is_last,
                                                                     cml);
  }
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  // active <= 1: the position is outside the cache, or one split wrote the outputs. Otherwise every split with
  // slots pushes its partial of head r into CTA r's inbox (each thread its own column, written by itself above).
  if (active > 1 && sp < active && tid < kHd) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      cl.map_shared_rank(&in_o[0][0], r)[sp * kHd + tid] = sm_o[0][r][tid];
      if (tid == 0) {
        cl.map_shared_rank(in_m, r)[sp] = cml[r];
        cl.map_shared_rank(in_l, r)[sp] = cml[REP + r];
      }
    }
  }
  cl.sync();  // phase 2 (release / acquire): the pushed partials are visible; no shared-memory access crosses CTAs
              // after it, so every CTA may leave
  if (active > 1 && sp < REP && tid < kHd) {
    float M = in_m[0];
#pragma unroll
    for (int s = 1; s < kClusterSplits; ++s)
      if (s < active) M = fmaxf(M, in_m[s]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int s = 0; s < kClusterSplits; ++s) {
      if (s < active) {  // in split order
        const float e = __expf(in_m[s] - M);
        O = fmaf(e, in_o[s][tid], O);
        L = fmaf(e, in_l[s], L);
      }
    }
    store_out(p.out, static_cast<int64_t>(g * REP + sp) * kHd + tid, O / L, p.bf16 != 0);
  }
}

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

namespace attn {

// Whether clusters of kClusterSplits CTAs of attn_cluster_kernel<REP> can be scheduled on the current device
// (checked once per device and group size; the non-portable cluster size is enabled on the way).
template <int REP>
bool cluster_ok(int dev) {
  static std::atomic<int> state[64] = {};  // 0 unknown, 1 yes, 2 no
  if (dev < 0 || dev >= 64) return false;
  int st = state[dev].load(std::memory_order_acquire);
  if (st == 0) {
    st = 2;
    if (cudaFuncSetAttribute(attn_cluster_kernel<REP>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
        cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(kClusterSplits);
      cfg.blockDim = dim3(kClusterThreads);
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = kClusterSplits;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, attn_cluster_kernel<REP>, &cfg) == cudaSuccess && n >= 1) st = 1;
    }
    (void)cudaGetLastError();
    state[dev].store(st, std::memory_order_release);
  }
  return st == 1;
}

template <int REP>
cudaError_t launch_rep(AttnParams p, int nkv, int num_sms, int flags, cudaStream_t stream) {
  int dev = 0;
  const bool cluster = !(flags & RB_FLAG_ATTN_TICKET) && cudaGetDevice(&dev) == cudaSuccess && cluster_ok<REP>(dev);
  p.nsplit = cluster ? kClusterSplits : static_cast<int>(nsplit_for(nkv, num_sms));
  p.pm = p.po + static_cast<int64_t>(nkv) * REP * p.nsplit * kHd;
  p.pl = p.pm + static_cast<int64_t>(nkv) * REP * p.nsplit;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nkv * p.nsplit);
  cfg.blockDim = dim3(cluster ? kClusterThreads : kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (flags & RB_FLAG_PDL) ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kClusterSplits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster ? 2 : 1;
  return cluster ? cudaLaunchKernelEx(&cfg, attn_cluster_kernel<REP>, p) : cudaLaunchKernelEx(&cfg, attn_decode_kernel<REP>, p);
}

}  // namespace attn

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
  p.pre = (flags & RB_FLAG_PDL) && (flags & RB_FLAG_PREFETCH_WEIGHTS) ? 1 : 0;
  uint8_t* w = static_cast<uint8_t*>(ws);
  p.ticket = reinterpret_cast<unsigned int*>(w);
  p.heads_done = nullptr;
  p.po = reinterpret_cast<float*>(w + kTicketBytes);
  cudaError_t e;
  switch (nq / nkv) {
    case 1: e = launch_rep<1>(p, nkv, num_sms, flags, stream); break;
    case 2: e = launch_rep<2>(p, nkv, num_sms, flags, stream); break;
    case 3: e = launch_rep<3>(p, nkv, num_sms, flags, stream); break;
    case 4: e = launch_rep<4>(p, nkv, num_sms, flags, stream); break;
    case 5: e = launch_rep<5>(p, nkv, num_sms, flags, stream); break;
    case 6: e = launch_rep<6>(p, nkv, num_sms, flags, stream); break;
    case 7: e = launch_rep<7>(p, nkv, num_sms, flags, stream); break;
    case 8: e = launch_rep<8>(p, nkv, num_sms, flags, stream); break;
    default: return RB_ERR_SHAPE;
  }
  return e == cudaSuccess ? RB_OK : RB_ERR_LAUNCH;
}

}  // namespace rb
