// sample.cu - the decode step's sampling tail on B200: the stop predictor, top-k over the audio head's logits and
// a Gumbel-max draw, with the step counters updated on the device (rumik-fast engine/sample.py:1-140, the same
// maths as engine/rumik_int4.py:174-198):
//   stop  = W2 . gelu(W1 . LayerNorm(h) + b1) + b2 > 0            (sigmoid > 0.5; only once step >= min_new)
//   token = ids[argmax_{j < top_k}(top_j / T + g_j)],  g_j = -log(-log(clamp(u_j, 1e-10, 1)))
// with the </audio> row masked while step < min_new. Two launches: the stop predictor's hidden layer (one warp per
// W1 row, every CTA recomputing the cheap LayerNorm) together with every 512-logit chunk's top 32, then one warp
// that merges the chunk lists and picks. The top-k packs
// each logit with its row into one 64-bit key whose integer order is the float order (negative floats have
// their 31 value bits flipped), so keys sort values and carry the row, ties going to the higher row.
#include "common.cuh"
#include "kernels.h"

namespace rb {

namespace smp {

constexpr int kStopWarps = 8;        // threads / 32 of the first launch's CTAs: W1 rows per CTA (one per warp)
constexpr int kChunk = 512;          // logits per CTA of the first launch (2 per thread)
constexpr int kMaxChunks = 64;       // n_vocab <= 64 x 512 = 32768: the pick warp merges 64 lists, two per lane
constexpr int kTop = 32;             // candidates kept per warp and per chunk, and overall (>= top_k)
constexpr int kMaxH = 8192;
static_assert(kStopWarps * 32 * 2 == kChunk, "two logits per thread of the first launch");

struct SampleParams {
  const void* logits;
  const int64_t* ids;
  const float* u;
  const void* h;
  const float* ln_w;
  const float* ln_b;
  const void* w1;
  const float* b1;
  const float* w2;
  const float* b2;
  float* z1;
  long long* keys;  // [kMaxChunks][kTop] every chunk's top 32, best first
  int64_t* step;
  int64_t* tok;
  int64_t* out;
  int64_t n_vocab, end_idx, end_id, min_new, out_len, H;
  float inv_temp;
  int logits_dtype, h_dtype, w1_dtype, top_k, nz;
};

__device__ __forceinline__ float load_any(const void* p, int64_t i, int dtype) {
  if (dtype == RB_F32) return reinterpret_cast<const float*>(p)[i];
  return load_act(p, i, dtype == RB_BF16);
}

__device__ __forceinline__ long long sort_key(float x, int64_t row) {
  const int b = __float_as_int(x);
  const int k32 = b ^ ((b >> 31) & 0x7FFFFFFF);
  return (static_cast<long long>(k32) << 32) | static_cast<long long>(static_cast<uint32_t>(row));
}

__device__ __forceinline__ float key_value(long long key) {
  const int k32 = static_cast<int>(key >> 32);
  return __int_as_float(k32 ^ ((k32 >> 31) & 0x7FFFFFFF));
}

// The largest key of the warp, in every lane: the largest high word (signed, the value's order), then among the
// lanes holding it the largest low word (unsigned, the row) - the 64-bit signed maximum, in two warp-wide integer
// reductions instead of five rounds of 64-bit shuffles and compares.
__device__ __forceinline__ long long warp_max_key(long long v) {
  const int hi = static_cast<int>(v >> 32);
  const unsigned lo = static_cast<unsigned>(v & 0xFFFFFFFFll);
  const int mh = __reduce_max_sync(0xffffffffu, hi);
  const unsigned ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
  return static_cast<long long>((static_cast<unsigned long long>(static_cast<unsigned>(mh)) << 32) | ml);
}

// ---- first launch: the stop predictor's hidden layer, z1[row] = gelu(W1[row] . LayerNorm(h) + b1[row]) (exact
// GELU, erf; CTAs below ceil(nz / 8), one W1 row per warp), and every 512-logit chunk's top 32 (CTAs below
// ceil(n_vocab / 512)): two keys per thread, each warp's top 32 by 32 rounds of "largest head among the lanes",
// then warp 0 merges the 8 warps' lists.
__device__ void chunk_top(const SampleParams& p, int chunk, bool early) {
  __shared__ long long wl[kStopWarps][kTop];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  long long k0, k1;
  {
    const int64_t r0 = static_cast<int64_t>(chunk) * kChunk + tid, r1 = r0 + kStopWarps * 32;
    float x0 = r0 < p.n_vocab ? load_any(p.logits, r0, p.logits_dtype) : -INFINITY;
    float x1 = r1 < p.n_vocab ? load_any(p.logits, r1, p.logits_dtype) : -INFINITY;
    if (early && r0 == p.end_idx) x0 = -INFINITY;  // no </audio> in the first min_new tokens
    if (early && r1 == p.end_idx) x1 = -INFINITY;
    k0 = r0 < p.n_vocab ? sort_key(x0, r0) : LLONG_MIN;
    k1 = r1 < p.n_vocab ? sort_key(x1, r1) : LLONG_MIN;
    if (k1 > k0) {
      const long long t = k0;
      k0 = k1;
      k1 = t;
    }
  }
  for (int r = 0; r < kTop; ++r) {
    const long long best = warp_max_key(k0);
    if (lane == 0) wl[warp][r] = best;
    if (k0 == best) {  // keys carry the row, so one lane pops (or all, once every list is exhausted)
      k0 = k1;
      k1 = LLONG_MIN;
    }
  }
  __syncthreads();
  if (warp == 0) {
    int head = 0;
    for (int r = 0; r < kTop; ++r) {
      const long long v = lane < kStopWarps && head < kTop ? wl[lane][head] : LLONG_MIN;
      const long long best = warp_max_key(v);
      if (v == best && best != LLONG_MIN) ++head;
      if (lane == 0) p.keys[chunk * kTop + r] = best;
    }
  }
}

__global__ void __launch_bounds__(kStopWarps * 32) sample_stage1_kernel(const __grid_constant__ SampleParams p) {
  griddep_wait();
  const bool early = *p.step < p.min_new;
  if (blockIdx.x * kChunk < p.n_vocab) chunk_top(p, blockIdx.x, early);
  if (blockIdx.x * kStopWarps >= p.nz) {
    griddep_launch_dependents();
    return;
  }
  __shared__ float z[kMaxH];
  __shared__ float red[2][kStopWarps];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = static_cast<int>(p.H);
  float s = 0.f;
  for (int i = tid; i < H; i += kStopWarps * 32) {
    const float v = load_any(p.h, i, p.h_dtype);
    z[i] = v;
    s += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) red[0][warp] = s;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < kStopWarps; ++w) tot += red[0][w];
  const float mean = tot / static_cast<float>(H);
  float q = 0.f;
  for (int i = tid; i < H; i += kStopWarps * 32) {
    const float d = z[i] - mean;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  if (lane == 0) red[1][warp] = q;
  __syncthreads();
  float var = 0.f;
  for (int w = 0; w < kStopWarps; ++w) var += red[1][w];
  const float rstd = rsqrtf(var / static_cast<float>(H) + 1e-5f);
  for (int i = tid; i < H; i += kStopWarps * 32) z[i] = (z[i] - mean) * rstd * p.ln_w[i] + p.ln_b[i];
  __syncthreads();
  const int row = blockIdx.x * kStopWarps + warp;
  if (row < p.nz) {
    float acc = 0.f;
    if (p.w1_dtype != RB_F32 && (H & 7) == 0) {
      // 8 weights per lane per 16-byte load, all of the row's loads independent
      const uint8_t* wr = static_cast<const uint8_t*>(p.w1) + static_cast<int64_t>(row) * H * 2;
#pragma unroll 4
      for (int i = lane * 8; i < H; i += 256) {
        float w[8];
        raw_to_f32(__ldg(reinterpret_cast<const uint4*>(wr + static_cast<int64_t>(i) * 2)), p.w1_dtype == RB_BF16, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(w[j], z[i + j], acc);
      }
    } else {
      for (int i = lane; i < H; i += 32)
        acc = fmaf(load_any(p.w1, static_cast<int64_t>(row) * H + i, p.w1_dtype), z[i], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const float y = acc + p.b1[row];
      p.z1[row] = 0.5f * y * (1.f + erff(y * 0.70710678118654752f));
    }
  }
  griddep_launch_dependents();
}

// ---- second launch (one warp): merge the chunks' lists into the overall top 32, the Gumbel-max pick, the stop
// rule and the counters
__global__ void __launch_bounds__(32) pick_kernel(const __grid_constant__ SampleParams p) {
  const int lane = threadIdx.x;
  griddep_wait();  // the chunk lists and the stop predictor's hidden layer come from the first launch
  const int64_t step = *p.step;
  const bool early = step < p.min_new;
  const int nchunks = static_cast<int>((p.n_vocab + kChunk - 1) / kChunk);
  // the chunk lists into shared memory first: independent, coalesced loads instead of one dependent load per round
  __shared__ long long lists[kMaxChunks * kTop];
#pragma unroll 8
  for (int i = lane; i < nchunks * kTop; i += 32) lists[i] = __ldcg(p.keys + i);
  __syncwarp();
  // lane l reads lists l and l + 32, best first; 32 rounds of "largest head"
  int ha = 0, hb = 0;
  long long mine = LLONG_MIN;  // lane j ends up holding the j-th best key
  for (int r = 0; r < kTop; ++r) {
    const long long va = lane < nchunks && ha < kTop ? lists[lane * kTop + ha] : LLONG_MIN;
    const long long vb = lane + 32 < nchunks && hb < kTop ? lists[(lane + 32) * kTop + hb] : LLONG_MIN;
    const long long v = va > vb ? va : vb;
    const long long best = warp_max_key(v);
    if (v == best && best != LLONG_MIN) {
      if (va >= vb) ++ha;
      else ++hb;
    }
    if (lane == r) mine = best;
  }
  // Gumbel-max over the top_k (engine/rumik_int4.py:185-190): the first of equal scores wins
  const float val = key_value(mine);
  const int row = static_cast<int>(mine & 0xFFFFFFFFll);
  float score = -INFINITY;
  if (lane < p.top_k) {
    const float uu = fminf(fmaxf(p.u[lane], 1e-10f), 1.f);
    score = val * p.inv_temp - logf(-logf(uu));
  }
  int best_lane = lane;
  float best_score = score;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float s2 = __shfl_xor_sync(0xffffffffu, best_score, o);
    const int l2 = __shfl_xor_sync(0xffffffffu, best_lane, o);
    if (s2 > best_score || (s2 == best_score && l2 < best_lane)) {
      best_score = s2;
      best_lane = l2;
    }
  }
  const int choice = __shfl_sync(0xffffffffu, row, best_lane);
  // the stop predictor's output (engine/rumik_int4.py:179): sigmoid(s) > 0.5  <=>  s > 0
  float s = 0.f;
  for (int i = lane; i < p.nz; i += 32) s = fmaf(p.z1[i], p.w2[i], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    s += p.b2[0];
    int64_t next = p.ids[choice];
    if (s > 0.f && !early) next = p.end_id;
    if (step >= 0 && step < p.out_len) p.out[step] = next;
    *p.tok = next;
    *p.step = step + 1;
  }
}

}  // namespace smp

int64_t sample_keys_offset(int nz) { return (static_cast<int64_t>(nz) * 4 + 255) / 256 * 256; }
int64_t sample_workspace(int nz) { return sample_keys_offset(nz) + smp::kMaxChunks * smp::kTop * 8; }

int launch_sample(const rb_sampler* s, int flags, cudaStream_t stream) {
  using namespace smp;
  SampleParams p;
  p.logits = s->logits;
  p.ids = s->ids;
  p.u = s->u;
  p.h = s->h;
  p.ln_w = s->ln_w;
  p.ln_b = s->ln_b;
  p.w1 = s->w1;
  p.b1 = s->b1;
  p.w2 = s->w2;
  p.b2 = s->b2;
  p.z1 = reinterpret_cast<float*>(s->ws);
  p.keys = reinterpret_cast<long long*>(static_cast<uint8_t*>(s->ws) + sample_keys_offset(s->nz));
  p.step = s->step;
  p.tok = s->tok;
  p.out = s->out;
  p.n_vocab = s->n_vocab;
  p.end_idx = s->end_idx;
  p.end_id = s->end_id;
  p.min_new = s->min_new;
  p.out_len = s->out_len;
  p.H = s->H;
  p.inv_temp = s->inv_temp;
  p.logits_dtype = s->logits_dtype;
  p.h_dtype = s->h_dtype;
  p.w1_dtype = s->w1_dtype;
  p.top_k = s->top_k;
  p.nz = s->nz;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (flags & RB_FLAG_PDL) ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int g1 = std::max((s->nz + kStopWarps - 1) / kStopWarps, static_cast<int>((s->n_vocab + kChunk - 1) / kChunk));
  cfg.gridDim = dim3(g1);
  cfg.blockDim = dim3(kStopWarps * 32);
  if (cudaLaunchKernelEx(&cfg, sample_stage1_kernel, p) != cudaSuccess) return RB_ERR_LAUNCH;
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  if (cudaLaunchKernelEx(&cfg, pick_kernel, p) != cudaSuccess) return RB_ERR_LAUNCH;
  return RB_OK;
}

}  // namespace rb
