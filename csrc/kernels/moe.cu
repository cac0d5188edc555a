// Mixture-of-experts token routing kernels (sm_100a): router softmax + top-k, the device-side plan that
// sorts (token, slot) assignments by expert into 128-row-aligned segments, the gather into those
// segments, and the weighted combine -- plus their backward passes. Together with the grouped tcgen05
// GEMM (gemm.cu, GRP_M / GRP_K) a MoE layer runs without a host synchronisation: every size the expert
// GEMMs need (segment offsets, counts) stays on the device.
//
// Layout of the dispatched rows: expert e owns rows [off[e], off[e + 1]) of the padded buffer, of which
// the first cnt[e] hold its assignments in (token, slot) order and the rest are zero. off[e] is a
// multiple of 128, so a GEMM tile never spans two experts, and zero padding rows add nothing to the
// weight-gradient contractions.
#include <cuda_runtime.h>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "moe.h"

namespace meshy {

namespace {

constexpr int kPlaceThreads = 1024;

// ─── router ────────────────────────────────────────────────────────────────
// One warp per token: softmax over E <= 256 logits (EPL = E / 32 per lane, padded with -inf), then k
// rounds of warp argmax (lower expert index wins a tie), then the optional renormalisation.
template <int EPL>
__global__ void route_kernel(const bf16* __restrict__ logits, int T, int E, int k, int norm,
                             float* __restrict__ probs, float* __restrict__ weights, int* __restrict__ experts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  const bf16* z = logits + (size_t)warp * E;
  float v[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __bfloat162float(z[e]) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    v[i] = (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
    s += v[i];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    v[i] *= inv;
    const int e = lane + 32 * i;
    if (e < E) probs[(size_t)warp * E + e] = v[i];
  }
  // top-k: taken entries are marked by a negative value (probabilities are >= 0)
  float picked_sum = 0.f;
  float my_w = 0.f;
  int my_e = -1;
  for (int j = 0; j < k; ++j) {
    float best = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && v[i] >= 0.f && (v[i] > best || (v[i] == best && e < bi))) {
        best = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    // the owner lane marks it taken
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i == bi) v[i] = -1.f;
    picked_sum += best;
    if (lane == j) {
      my_w = best;
      my_e = bi;
    }
  }
  if (lane < k) {
    const float w = norm ? my_w / fmaxf(picked_sum, 1e-20f) : my_w;
    weights[(size_t)warp * k + lane] = w;
    experts[(size_t)warp * k + lane] = my_e;
  }
}

// d logits of the router: p = softmax(z); selected set S; w_j = p_{e_j} (/ sum_S p with norm).
//   norm:    dp_i = (dw_i - <dw, w>) / sum_S p   for i in S, else 0
//   no norm: dp_i = dw_i for i in S, else 0
//   dz = p * (dp - <dp, p>)
template <int EPL>
__global__ void route_bwd_kernel(const float* __restrict__ dw, const float* __restrict__ probs,
                                 const float* __restrict__ weights, const int* __restrict__ experts, int T, int E,
                                 int k, int norm, bf16* __restrict__ dlogits) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  const float* p = probs + (size_t)warp * E;
  // lanes < k hold one selection each
  float g = 0.f, w = 0.f, ps = 0.f;
  int e_sel = -1;
  if (lane < k) {
    g = dw[(size_t)warp * k + lane];
    w = weights[(size_t)warp * k + lane];
    e_sel = experts[(size_t)warp * k + lane];
    ps = p[e_sel];
  }
  const float sum_s = warp_sum(ps);
  const float gw = warp_sum(g * w);
  float dp_sel = 0.f;
  if (lane < k) dp_sel = norm ? (g - gw) / fmaxf(sum_s, 1e-20f) : g;
  // <dp, p> over the selected set
  const float dpp = warp_sum(dp_sel * ps);
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    float dpe = 0.f;
    for (int j = 0; j < k; ++j) {  // every lane shuffles (uniform trip counts), lanes past E write nothing
      const int ej = __shfl_sync(0xffffffffu, e_sel, j);
      const float dj = __shfl_sync(0xffffffffu, dp_sel, j);
      if (ej == e) dpe += dj;
    }
    if (e < E) dlogits[(size_t)warp * E + e] = __float2bfloat16(p[e] * (dpe - dpp));
  }
}

// Block-wide exclusive scan of 0/1 flags (blockDim = kPlaceThreads); returns this thread's rank and the
// block total through ``total``.
__device__ __forceinline__ int block_rank(bool flag, int* warp_tot, int& total) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const unsigned m = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(m & ((1u << lane) - 1u));
  if (lane == 0) warp_tot[warp] = __popc(m);
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    int x = lane < nw ? warp_tot[lane] : 0;
    int incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane < nw) warp_tot[lane] = incl - x;  // exclusive prefix
    if (lane == 31) warp_tot[32] = incl;
  }
  __syncthreads();
  const int r = warp_tot[warp] + in_warp;
  total = warp_tot[32];
  __syncthreads();
  return r;
}

// CTA e counts the assignments to expert e.
__global__ void __launch_bounds__(kPlaceThreads) count_kernel(const int* __restrict__ experts, int n, int* cnt) {
  __shared__ int warp_tot[33];
  const int e = blockIdx.x;
  int c = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int tot;
    block_rank(i < n && experts[i] == e, warp_tot, tot);
    c += tot;
  }
  if (threadIdx.x == 0) cnt[e] = c;
}

// CTA e: its segment offset (sum of the padded counts before it), a stable placement of its assignments
// (slot_of[i] = destination row of assignment i = t * k + j; row_src[row] = i), the gather of their token
// rows (one warp per row, coalesced) and the zero padding. CTA 0 also writes off[E]. A plan that would
// not fit ``rows_cap`` rows sets the error word and writes nothing past the buffer.
__global__ void __launch_bounds__(kPlaceThreads)
    place_kernel(const int* __restrict__ experts, int n, int k, int E, const int* __restrict__ cnt, int* off,
                 int* slot_of, int* row_src, const bf16* __restrict__ x, int D, bf16* __restrict__ xp, int rows_cap,
                 int* err) {
  __shared__ int warp_tot[33];
  __shared__ int s_off;
  const int e = blockIdx.x;
  pdl_wait();
  if (threadIdx.x == 0) {
    int o = 0, total = 0;
    for (int q = 0; q < E; ++q) {
      const int pad = (cnt[q] + 127) / 128 * 128;
      if (q < e) o += pad;
      total += pad;
    }
    s_off = o;
    off[e] = o;
    if (e == 0) off[E] = total;
    if (total > rows_cap && err) atomicCAS(err, 0, kErrBadArg);
  }
  __syncthreads();
  const int o = s_off;
  const int c = cnt[e];
  const int padded = (c + 127) / 128 * 128;
  if (o + padded > rows_cap) return;  // reported above
  int seen = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool mine = i < n && experts[i] == e;
    int tot;
    const int r = block_rank(mine, warp_tot, tot);
    if (mine) {
      slot_of[i] = o + seen + r;
      row_src[o + seen + r] = i;
    }
    seen += tot;
  }
  for (int r = o + c + threadIdx.x; r < o + padded; r += blockDim.x) row_src[r] = -1;
  if (xp == nullptr) return;
  __syncthreads();  // row_src of this segment is complete
  const int vpr = D / 8;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  for (int r = warp; r < padded; r += nwarps) {
    uint4* d = reinterpret_cast<uint4*>(xp + (size_t)(o + r) * D);
    if (r < c) {
      const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(row_src[o + r] / k) * D);
      for (int v = lane; v < vpr; v += 32) d[v] = src[v];
    } else {
      for (int v = lane; v < vpr; v += 32) d[v] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Zero rows [off[e] + cnt[e], off[e + 1]) of a [rows, C] bf16 buffer (CTA per expert).
__global__ void zero_pad_kernel(const int* __restrict__ off, const int* __restrict__ cnt, bf16* buf, int C) {
  const int e = blockIdx.x;
  pdl_wait();
  const int r0 = off[e] + cnt[e], r1 = off[e + 1];
  const int vpr = C / 8;
  uint4* p = reinterpret_cast<uint4*>(buf + (size_t)r0 * C);
  const int nv = (r1 - r0) * vpr;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) p[v] = make_uint4(0, 0, 0, 0);
}

// out[t] = sum_j w[t, j] * y[slot_of[t * k + j]] (w == nullptr: weight 1). One CTA per token, 8 columns per
// thread step, fp32 accumulation.
__global__ void combine_kernel(const bf16* __restrict__ y, int rows, const int* __restrict__ slot_of,
                               const float* __restrict__ w, int k, int D, bf16* __restrict__ out) {
  const int t = blockIdx.x;
  pdl_wait();
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int s = slot_of[(size_t)t * k + j];
      if (s < 0 || s >= rows) continue;  // an unplaced assignment (never produced by a valid plan)
      const float wj = w ? w[(size_t)t * k + j] : 1.f;
      const uint4 u = *reinterpret_cast<const uint4*>(y + (size_t)s * D + c);
      const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), cc = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
      acc[0] += wj * a.x; acc[1] += wj * a.y; acc[2] += wj * b.x; acc[3] += wj * b.y;
      acc[4] += wj * cc.x; acc[5] += wj * cc.y; acc[6] += wj * d.x; acc[7] += wj * d.y;
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * D + c) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
}

// Backward of the combine: dy[slot] = w[t, j] * dout[t] (bf16) and dw[t, j] = <dout[t], y[slot]> (fp32).
__global__ void combine_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ y, int rows,
                                   const int* __restrict__ slot_of, const float* __restrict__ w, int k, int D,
                                   bf16* __restrict__ dy, float* __restrict__ dw) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  pdl_wait();
  for (int j = 0; j < k; ++j) {
    const int s = slot_of[(size_t)t * k + j];
    const bool ok = s >= 0 && s < rows;  // block-uniform
    const float wj = w[(size_t)t * k + j];
    float dot = 0.f;
    for (int c = threadIdx.x * 8; ok && c < D; c += blockDim.x * 8) {
      const uint4 g = *reinterpret_cast<const uint4*>(dout + (size_t)t * D + c);
      const uint4 u = *reinterpret_cast<const uint4*>(y + (size_t)s * D + c);
      const uint32_t gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {u.x, u.y, u.z, u.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 gg = unpack_bf16x2(gs[q]), yy = unpack_bf16x2(us[q]);
        dot += gg.x * yy.x + gg.y * yy.y;
        o[q] = pack_bf16x2(wj * gg.x, wj * gg.y);
      }
      *reinterpret_cast<uint4*>(dy + (size_t)s * D + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    dot = warp_sum(dot);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = dot;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) dw[(size_t)t * k + j] = v;
    }
    __syncthreads();
  }
}

}  // namespace

void moe_route(const bf16* logits, int T, int E, int k, bool norm, float* probs, float* weights, int* experts,
               cudaStream_t st) {
  MESHY_CHECK(E > 0 && E <= 256 && k > 0 && k <= 32 && k <= E, "moe_route: need 0 < k <= min(E, 32), E <= 256");
  if (T == 0) return;
  const int threads = 256, per = threads / 32;
  const int grid = (T + per - 1) / per;
  const int epl = (E + 31) / 32;
  if (epl <= 1) route_kernel<1><<<grid, threads, 0, st>>>(logits, T, E, k, norm, probs, weights, experts);
  else if (epl <= 2) route_kernel<2><<<grid, threads, 0, st>>>(logits, T, E, k, norm, probs, weights, experts);
  else if (epl <= 4) route_kernel<4><<<grid, threads, 0, st>>>(logits, T, E, k, norm, probs, weights, experts);
  else route_kernel<8><<<grid, threads, 0, st>>>(logits, T, E, k, norm, probs, weights, experts);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void moe_route_bwd(const float* dw, const float* probs, const float* weights, const int* experts, int T, int E, int k,
                   bool norm, bf16* dlogits, cudaStream_t st) {
  MESHY_CHECK(E > 0 && E <= 256 && k > 0 && k <= 32, "moe_route_bwd: E <= 256, k <= 32");
  if (T == 0) return;
  const int threads = 256, per = threads / 32;
  const int grid = (T + per - 1) / per;
  const int epl = (E + 31) / 32;
  if (epl <= 1) route_bwd_kernel<1><<<grid, threads, 0, st>>>(dw, probs, weights, experts, T, E, k, norm, dlogits);
  else if (epl <= 2) route_bwd_kernel<2><<<grid, threads, 0, st>>>(dw, probs, weights, experts, T, E, k, norm, dlogits);
  else if (epl <= 4) route_bwd_kernel<4><<<grid, threads, 0, st>>>(dw, probs, weights, experts, T, E, k, norm, dlogits);
  else route_bwd_kernel<8><<<grid, threads, 0, st>>>(dw, probs, weights, experts, T, E, k, norm, dlogits);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void moe_plan(const int* experts, int n, int k, int E, int* cnt, int* off, int* slot_of, int* row_src, const bf16* x,
              int D, bf16* xp, int rows_cap, int* err, cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0, "moe_plan: D must be a multiple of 8");
  MESHY_CHECK(E > 0, "moe_plan: no experts");
  count_kernel<<<E, kPlaceThreads, 0, st>>>(experts, n, cnt);
  MESHY_CUDA_CHECK(cudaGetLastError());
  launch_pdl(place_kernel, dim3(E), dim3(kPlaceThreads), 0, st, experts, n, k, E, (const int*)cnt, off, slot_of,
             row_src, x, D, xp, rows_cap, err);
}

void moe_zero_pad(const int* off, const int* cnt, int E, bf16* buf, int C, cudaStream_t st) {
  MESHY_CHECK(C % 8 == 0, "moe_zero_pad: C must be a multiple of 8");
  launch_pdl(zero_pad_kernel, dim3(E), dim3(256), 0, st, off, cnt, buf, C);
}

void moe_combine(const bf16* y, int rows, const int* slot_of, const float* w, int T, int k, int D, bf16* out,
                 cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0, "moe_combine: D must be a multiple of 8");
  if (T == 0) return;
  launch_pdl(combine_kernel, dim3(T), dim3(std::min(256, std::max(32, D / 8))), 0, st, y, rows, slot_of, w, k, D, out);
}

void moe_combine_bwd(const bf16* dout, const bf16* y, int rows, const int* slot_of, const float* w, int T, int k,
                     int D, bf16* dy, float* dw, cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0, "moe_combine_bwd: D must be a multiple of 8");
  if (T == 0) return;
  const int threads = std::min(256, std::max(32, (D / 8 + 31) / 32 * 32));
  launch_pdl(combine_bwd_kernel, dim3(T), dim3(threads), 0, st, dout, y, rows, slot_of, w, k, D, dy, dw);
}

}  // namespace meshy
