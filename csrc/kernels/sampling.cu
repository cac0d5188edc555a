// Filtered sampling (top-k and / or top-p with temperature) over materialised logits, one CTA per row.
//
// The temperature-only path samples inside the LM-head GEMM epilogue (gemm.cu / gemm_small.cu) and never
// writes logits. With a top-k or top-p filter the kept set depends on the whole row, so the logits
// [B, V] fp32 come from the tcgen05 GEMM first and this kernel does the rest on the device:
//
//   1. z = logits / T, row max;
//   2. top-k: the k-th largest z found exactly by a 32-step binary search over the order-preserving
//      integer image of the floats (count of z >= candidate, block-reduced each step); tokens below it are
//      dropped, ties with it kept -- the same set as masking ``z < kth`` after ``torch.topk``;
//   3. top-p: with p = softmax over the kept tokens, the smallest probability threshold tau such that the
//      mass strictly above tau is <= top_p (binary search over the bit patterns of non-negative floats);
//      tokens with p >= tau are kept, i.e. a token survives when the mass ranked before it is <= top_p;
//   4. a Gumbel-max draw over the kept tokens (Philox noise keyed by seed, step, row, token) and the
//      token's log-probability under the filtered, tempered distribution.
//
// Temperature 0 is greedy (log-prob 0). No host synchronisation: a decode step with this sampler can be
// captured in a CUDA graph.
#include <cuda_runtime.h>

#include "../include/common.cuh"
#include "misc.h"

namespace meshy {

namespace {

constexpr int kSampThreads = 1024;

// float -> uint32 that orders like the float (negative values flipped)
__device__ __forceinline__ uint32_t fkey(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = (threadIdx.x < blockDim.x / 32) ? sh[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) sh[32] = t;
  __syncthreads();
  return sh[32];
}

__device__ __forceinline__ float block_max(float v, float* sh) {
  v = warp_max(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = (threadIdx.x < blockDim.x / 32) ? sh[threadIdx.x] : -INFINITY;
  if (w == 0) t = warp_max(t);
  if (threadIdx.x == 0) sh[32] = t;
  __syncthreads();
  return sh[32];
}

__global__ void __launch_bounds__(kSampThreads)
    filtered_sample_kernel(const float* __restrict__ logits, int V, float temperature, int top_k, float top_p,
                           uint64_t seed, const int64_t* __restrict__ step_ptr, int64_t* __restrict__ tok,
                           float* __restrict__ lp) {
  __shared__ float sh[33];
  __shared__ float shv[32];
  __shared__ int shi[32];
  const int row = blockIdx.x;
  const float* z = logits + (size_t)row * V;
  const bool greedy = !(temperature > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temperature;
  // 1. row max of z / T
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, z[i] * inv_t);
  mx = block_max(mx, sh);
  // 2. top-k threshold (exact k-th largest value)
  uint32_t kth = 0u;  // keep every key >= kth
  if (!greedy && top_k > 0 && top_k < V) {
    uint32_t lo = 0u, hi = 0xFFFFFFFFu;  // largest key with count(key >= k) >= top_k
    for (int it = 0; it < 32; ++it) {
      const uint32_t mid = lo + ((hi - lo) >> 1) + ((hi - lo) & 1u);
      float c = 0.f;
      for (int i = threadIdx.x; i < V; i += blockDim.x) c += (fkey(z[i] * inv_t) >= mid) ? 1.f : 0.f;
      c = block_sum(c, sh);
      if (c >= (float)top_k) lo = mid;
      else hi = mid - 1u;
      if (lo >= hi) break;
    }
    kth = lo;
  }
  // normaliser of the top-k-filtered tempered distribution
  float se = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = z[i] * inv_t;
    se += (fkey(v) >= kth) ? __expf(v - mx) : 0.f;
  }
  se = block_sum(se, sh);
  // 3. top-p threshold on probabilities p = exp(v - mx) / se (non-negative: bit patterns order like values)
  float tau = 0.f;
  if (!greedy && top_p < 1.f) {
    uint32_t lo = 0u, hi = 0x3F800000u;  // [0, 1]
    // smallest tau with mass(p > tau) <= top_p
    for (int it = 0; it < 32 && lo < hi; ++it) {
      const uint32_t mid = lo + ((hi - lo) >> 1);
      const float t = __uint_as_float(mid);
      float m = 0.f;
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = z[i] * inv_t;
        if (fkey(v) < kth) continue;
        const float p = __expf(v - mx) / se;
        if (p > t) m += p;
      }
      m = block_sum(m, sh);
      if (m <= top_p) hi = mid;
      else lo = mid + 1u;
    }
    tau = __uint_as_float(lo);
  }
  // 4. draw (Gumbel-max over kept tokens) and the kept-set normaliser
  const uint64_t step = step_ptr ? (uint64_t)*step_ptr : 0ull;
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32) ^ (uint32_t)step);
  float best = -INFINITY, bestz = 0.f, kept = 0.f;
  int besti = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = z[i] * inv_t;
    const bool keep = fkey(v) >= kth && (tau <= 0.f || __expf(v - mx) / se >= tau);
    if (!keep) continue;
    kept += __expf(v - mx);
    float score = v;
    if (!greedy) {
      const uint4 r = Philox::gen(make_uint4((uint32_t)i, (uint32_t)row, (uint32_t)(step >> 32), 0x7A11u), key);
      score = v + gumbel(r.x);
    }
    if (score > best || (score == best && i < besti)) {
      best = score;
      besti = i;
      bestz = v;
    }
  }
  kept = block_sum(kept, sh);
  // block argmax of (best, index)
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    const float oz = __shfl_xor_sync(0xffffffffu, bestz, o);
    if (ob > best || (ob == best && oi < besti)) {
      best = ob;
      besti = oi;
      bestz = oz;
    }
  }
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) {
    shv[w] = best;
    shi[w] = besti;
    sh[w] = bestz;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -INFINITY, bz = 0.f;
    int bi = 0x7fffffff;
    for (int q = 0; q < (int)(blockDim.x / 32); ++q) {
      if (shv[q] > b || (shv[q] == b && shi[q] < bi)) {
        b = shv[q];
        bi = shi[q];
        bz = sh[q];
      }
    }
    if (bi == 0x7fffffff) bi = 0;  // an all -inf row
    tok[row] = bi;
    lp[row] = greedy ? 0.f : (bz - mx - __logf(fmaxf(kept, 1e-30f)));
  }
}

}  // namespace

void filtered_sample(const float* logits, int B, int V, float temperature, int top_k, float top_p, uint64_t seed,
                     const int64_t* step_ptr, int64_t* tok, float* lp, cudaStream_t st) {
  if (B == 0) return;
  MESHY_CHECK(V > 0, "filtered_sample: empty vocabulary");
  filtered_sample_kernel<<<B, kSampThreads, 0, st>>>(logits, V, temperature, top_k, top_p, seed, step_ptr, tok, lp);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
