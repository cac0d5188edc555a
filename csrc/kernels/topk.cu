// Top-K distillation kernels (sm_100a).
//
//   topk_logprobs   per row of fp32 logits z [T, V]: the K largest entries (sorted, largest first) and their
//                   log-probabilities z - logsumexp(z). One CTA per row. The K-th largest value is found
//                   exactly by a 4-pass radix select over the order-preserving integer image of the floats
//                   (8-bit digits, 256-bin shared-memory histograms with warp-aggregated counts; the first
//                   pass also folds the row's max and sum of exponentials), then one pass collects the K
//                   winners and a bitonic sort in shared memory orders them. For K <= 8 one read of the row
//                   suffices: per-thread register lists of the 8 largest, merged by warp maxima.
//   gather_logprobs z[t, ids[t, k]] - lse[t] without the logits: one warp per (t, k) takes the dot product of
//                   the hidden row and the vocabulary row of the weight (fp32 accumulation of bf16 products).
//   scatter_add_rows  dz[t, ids[t, k]] += g[t, k] in bf16 (one thread per row, so repeated ids in a row add
//                   up without races); the backward of the gather on top of dz = -G p from the LM-head GEMM.
#include <cuda_runtime.h>

#include "../include/common.cuh"
#include "misc.h"

namespace meshy {

namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMax = 1024;

__device__ __forceinline__ uint32_t okey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One element's share of a radix pass: the row's online max / sum of exponentials on the first pass, and a
// count in the histogram bin of its digit when it still matches the selected prefix. Lanes of a warp whose
// elements fall in the same bin add once, through their lowest lane: logits occupy few exponent bins, so
// one shared-memory atomic per lane would serialise up to 32-fold on one address. All 32 lanes call this
// together (``valid`` false for the lanes past the row's end).
__device__ __forceinline__ void radix_count(float v, bool valid, bool first, uint32_t prefix, uint32_t pmask,
                                            int shift, float& m, float& s, unsigned* hist, int lane) {
  bool take = false;
  uint32_t bin = 0u;
  if (valid) {
    if (first) {
      if (v > m) {
        s = s * __expf(m - v) + 1.f;
        m = v;
      } else {
        s += __expf(v - m);
      }
    }
    const uint32_t u = okey(v);
    take = (u & pmask) == prefix;
    bin = (u >> shift) & 255u;
  }
  const unsigned takers = __ballot_sync(0xffffffffu, take);
  if (take) {
    const unsigned peers = __match_any_sync(takers, bin);
    if (__ffs(peers) - 1 == lane) atomicAdd(&hist[bin], (unsigned)__popc(peers));
  }
}

__global__ void __launch_bounds__(kTopkThreads)
    topk_logprobs_kernel(const float* __restrict__ z, long long ldz, int V, int K, int64_t* __restrict__ ids,
                         float* __restrict__ lp, float* __restrict__ lse_out) {
  __shared__ unsigned hist[256];
  __shared__ float cv[kTopkMax];
  __shared__ int ci[kTopkMax];
  __shared__ float red_m[32], red_s[32];
  __shared__ uint32_t sel_digit;
  __shared__ int sel_above;
  __shared__ int n_gt, n_eq;
  const int row = blockIdx.x;
  const float* zr = z + (size_t)row * ldz;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;

  uint32_t prefix = 0u, pmask = 0u;
  int kr = K;  // how many of the remaining candidates (those matching the prefix) are still to be taken
  float m = -INFINITY, s = 0.f;
  // 16-byte loads when the rows allow them (blockDim.x is a multiple of 32, so every warp runs the same
  // number of iterations and stays converged at the warp votes in radix_count)
  const bool vec = (ldz % 4 == 0) && (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(z) & 15u) == 0u);
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    const bool first = shift == 24;
    if (vec) {
      const float4* z4 = reinterpret_cast<const float4*>(zr);
      const int V4 = V / 4;
      for (int j0 = 0; j0 < V4; j0 += blockDim.x) {
        const int j = j0 + tid;
        const bool ok = j < V4;
        const float4 q = ok ? z4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        radix_count(q.x, ok, first, prefix, pmask, shift, m, s, hist, lane);
        radix_count(q.y, ok, first, prefix, pmask, shift, m, s, hist, lane);
        radix_count(q.z, ok, first, prefix, pmask, shift, m, s, hist, lane);
        radix_count(q.w, ok, first, prefix, pmask, shift, m, s, hist, lane);
      }
    } else {
      for (int i0 = 0; i0 < V; i0 += blockDim.x) {
        const int i = i0 + tid;
        const bool ok = i < V;
        radix_count(ok ? zr[i] : 0.f, ok, first, prefix, pmask, shift, m, s, hist, lane);
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255 - 8 l ... 248 - 8 l (descending); counts above a bin come from a suffix scan
      unsigned c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        tot += c[j];
      }
      unsigned incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      unsigned above = incl - tot;  // candidates in bins owned by lower lanes (larger digits)
      if (above < (unsigned)kr && (unsigned)kr <= incl) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (above < (unsigned)kr && (unsigned)kr <= above + c[j]) {
            sel_digit = 255u - 8u * lane - j;
            sel_above = (int)above;
          }
          above += c[j];
        }
      }
    }
    __syncthreads();
    kr -= sel_above;
    prefix |= sel_digit << shift;
    pmask |= 255u << shift;
    __syncthreads();  // sel_* are rewritten by the next pass
  }
  // row log-sum-exp
  {
    float mm = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
    float ss = (m == -INFINITY) ? 0.f : s * __expf(m - mm);
    ss = warp_sum(ss);
    if (lane == 0) {
      red_m[warp] = mm;
      red_s[warp] = ss;
    }
  }
  if (tid == 0) {
    n_gt = 0;
    n_eq = 0;
  }
  __syncthreads();
  float gm = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x / 32); ++w) gm = fmaxf(gm, red_m[w]);
  float gs = 0.f;
  for (int w = 0; w < (int)(blockDim.x / 32); ++w) gs += (red_m[w] == -INFINITY) ? 0.f : red_s[w] * __expf(red_m[w] - gm);
  const float lse = gm + __logf(gs);
  // collect: keys above the K-th go to slots [0, K - kr), ties with it fill [K - kr, K)
  const uint32_t kth = prefix;
  const int n_above = K - kr;
  for (int i = tid; i < V; i += blockDim.x) {
    const float v = zr[i];
    const uint32_t u = okey(v);
    if (u > kth) {
      const int slot = atomicAdd(&n_gt, 1);
      if (slot < n_above) {
        cv[slot] = v;
        ci[slot] = i;
      }
    } else if (u == kth) {
      const int e = atomicAdd(&n_eq, 1);
      if (e < kr) {
        cv[n_above + e] = v;
        ci[n_above + e] = i;
      }
    }
  }
  int P = 1;
  while (P < K) P <<= 1;
  for (int i = K + tid; i < P; i += blockDim.x) {
    cv[i] = -INFINITY;
    ci[i] = 0x7fffffff;
  }
  __syncthreads();
  // bitonic sort, descending by value, ascending index among equal values
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float a = cv[i], b = cv[j];
          const int ia = ci[i], ib = ci[j];
          const bool a_first = a > b || (a == b && ia < ib);
          if (desc != a_first) {
            cv[i] = b;
            cv[j] = a;
            ci[i] = ib;
            ci[j] = ia;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < K; j += blockDim.x) {
    ids[(size_t)row * K + j] = ci[j];
    lp[(size_t)row * K + j] = cv[j] - lse;
  }
  if (lse_out && tid == 0) lse_out[row] = lse;
}

// ---------------------------------------------------------------------------------------------------------
// Small K (K <= kSmallK): one read of the row. Every thread keeps the kSmallK largest of the elements it visits
// as 64-bit keys (order-preserving image of the value in the high half, 0x7fffffff - index in the low half,
// so equal values rank by ascending index and every key is unique), then warps and finally warp 0 merge the
// per-thread lists by repeated warp maxima. The row's log-sum-exp is folded into the same read.

constexpr int kSmallK = 8;

__device__ __forceinline__ unsigned long long topk_key(float v, int i) {
  return (static_cast<unsigned long long>(okey(v)) << 32) | static_cast<unsigned>(0x7fffffff - i);
}

__device__ __forceinline__ float key_value(unsigned long long k) {
  const uint32_t u = static_cast<uint32_t>(k >> 32);
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

__device__ __forceinline__ void small_visit(float v, int i, float& m, float& s, unsigned long long (&keys)[kSmallK]) {
  if (v > m) {
    s = s * __expf(m - v) + 1.f;
    m = v;
  } else {
    s += __expf(v - m);
  }
  unsigned long long k = topk_key(v, i);
  if (k > keys[kSmallK - 1]) {  // rare once the list has filled: insert, carrying the displaced key down
#pragma unroll
    for (int j = 0; j < kSmallK; ++j) {
      if (k > keys[j]) {
        const unsigned long long t = keys[j];
        keys[j] = k;
        k = t;
      }
    }
  }
}

// The warp's kSmallK largest keys (each lane's list sorted descending) into out[0..kSmallK) by lane 0.
__device__ __forceinline__ void warp_merge_keys(unsigned long long (&keys)[kSmallK], unsigned long long* out,
                                                int lane) {
#pragma unroll
  for (int r = 0; r < kSmallK; ++r) {
    unsigned long long best = keys[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) out[r] = best;
    if (best != 0ull && keys[0] == best) {  // keys are unique: exactly one lane pops its head
#pragma unroll
      for (int j = 0; j < kSmallK - 1; ++j) keys[j] = keys[j + 1];
      keys[kSmallK - 1] = 0ull;
    }
  }
}

__global__ void __launch_bounds__(kTopkThreads)
    topk_small_kernel(const float* __restrict__ z, long long ldz, int V, int K, int64_t* __restrict__ ids,
                      float* __restrict__ lp, float* __restrict__ lse_out) {
  __shared__ unsigned long long wtop[32][kSmallK];
  __shared__ unsigned long long top[kSmallK];
  __shared__ float red_m[32], red_s[32];
  const int row = blockIdx.x;
  const float* zr = z + (size_t)row * ldz;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32, nwarps = blockDim.x / 32;
  unsigned long long keys[kSmallK];
#pragma unroll
  for (int j = 0; j < kSmallK; ++j) keys[j] = 0ull;  // below every real key (okey(-inf) > 0)
  float m = -INFINITY, s = 0.f;
  if ((ldz % 4 == 0) && (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(z) & 15u) == 0u)) {
    const float4* z4 = reinterpret_cast<const float4*>(zr);
    for (int j = tid; j < V / 4; j += blockDim.x) {
      const float4 q = z4[j];
      small_visit(q.x, 4 * j, m, s, keys);
      small_visit(q.y, 4 * j + 1, m, s, keys);
      small_visit(q.z, 4 * j + 2, m, s, keys);
      small_visit(q.w, 4 * j + 3, m, s, keys);
    }
  } else {
    for (int i = tid; i < V; i += blockDim.x) small_visit(zr[i], i, m, s, keys);
  }
  warp_merge_keys(keys, wtop[warp], lane);
  {
    float mm = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
    float ss = (m == -INFINITY) ? 0.f : s * __expf(m - mm);
    ss = warp_sum(ss);
    if (lane == 0) {
      red_m[warp] = mm;
      red_s[warp] = ss;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  unsigned long long k2[kSmallK];
#pragma unroll
  for (int j = 0; j < kSmallK; ++j) k2[j] = lane < nwarps ? wtop[lane][j] : 0ull;
  warp_merge_keys(k2, top, lane);
  float gm = -INFINITY;
  for (int w = 0; w < nwarps; ++w) gm = fmaxf(gm, red_m[w]);
  float gs = 0.f;
  for (int w = 0; w < nwarps; ++w) gs += (red_m[w] == -INFINITY) ? 0.f : red_s[w] * __expf(red_m[w] - gm);
  const float lse = gm + __logf(gs);
  __syncwarp();
  if (lane < K) {
    const unsigned long long k = top[lane];
    ids[(size_t)row * K + lane] = 0x7fffffff - static_cast<int>(k & 0xffffffffull);
    lp[(size_t)row * K + lane] = key_value(k) - lse;
  }
  if (lse_out && lane == 0) lse_out[row] = lse;
}

__global__ void gather_logprobs_kernel(const bf16* __restrict__ h, long long ldh, const bf16* __restrict__ w,
                                       long long ldw, int D, int V, const int64_t* __restrict__ ids, int TK,
                                       int K, const float* __restrict__ lse, float* __restrict__ lp) {
  const int pair = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (pair >= TK) return;
  const int t = pair / K;
  const int64_t id = ids[pair];
  float acc = 0.f;
  if (id >= 0 && id < V) {
    const bf16* hr = h + (size_t)t * ldh;
    const bf16* wr = w + (size_t)id * ldw;
    for (int c = lane * 8; c < D; c += 32 * 8) {
      const uint4 a = *reinterpret_cast<const uint4*>(hr + c);
      const uint4 b = *reinterpret_cast<const uint4*>(wr + c);
      const uint32_t qa[4] = {a.x, a.y, a.z, a.w}, qb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = unpack_bf16x2(qa[j]), y = unpack_bf16x2(qb[j]);
        acc += x.x * y.x + x.y * y.y;
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) lp[pair] = (id >= 0 && id < V) ? acc - lse[t] : -INFINITY;
}

__global__ void scatter_add_rows_kernel(bf16* __restrict__ dz, long long ldz, int T, int V,
                                        const int64_t* __restrict__ ids, const float* __restrict__ g, int K) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  for (int k = 0; k < K; ++k) {
    const int64_t id = ids[(size_t)t * K + k];
    const float gv = g[(size_t)t * K + k];
    if (id < 0 || id >= V || gv == 0.f) continue;
    bf16* p = dz + (size_t)t * ldz + id;
    *p = __float2bfloat16(__bfloat162float(*p) + gv);
  }
}

}  // namespace

void topk_logprobs(const float* z, long long ldz, int T, int V, int K, int64_t* ids, float* lp, float* lse,
                   cudaStream_t st) {
  MESHY_CHECK(K >= 1 && K <= kTopkMax && K <= V, "topk_logprobs: need 1 <= K <= min(1024, V)");
  if (T == 0) return;
  if (K <= kSmallK)
    topk_small_kernel<<<T, kTopkThreads, 0, st>>>(z, ldz, V, K, ids, lp, lse);
  else
    topk_logprobs_kernel<<<T, kTopkThreads, 0, st>>>(z, ldz, V, K, ids, lp, lse);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void gather_logprobs(const bf16* h, long long ldh, const bf16* w, long long ldw, int T, int D, int V,
                     const int64_t* ids, int K, const float* lse, float* lp, cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0 && ldh % 8 == 0 && ldw % 8 == 0, "gather_logprobs: rows must be 16-byte aligned");
  const int TK = T * K;
  if (TK == 0) return;
  const int warps = 8;
  gather_logprobs_kernel<<<(TK + warps - 1) / warps, warps * 32, 0, st>>>(h, ldh, w, ldw, D, V, ids, TK, K, lse, lp);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void scatter_add_rows(bf16* dz, long long ldz, int T, int V, const int64_t* ids, const float* g, int K,
                      cudaStream_t st) {
  if (T == 0 || K == 0) return;
  scatter_add_rows_kernel<<<(T + 127) / 128, 128, 0, st>>>(dz, ldz, T, V, ids, g, K);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
