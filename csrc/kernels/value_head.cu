// Critic value head fused with the clipped value loss (sm_100a).
//
//   forward  (one warp per token): v_t = h_t . w + b in fp32 from bf16 h; the clipped squared error against
//            the returns (PPO value clipping around the old values when given); the window-loss numerator
//            sum(err * mask) (block partials, one atomic per block); and dL/dv_t = mask_t * d err_t / dv_t
//            / denom, kept for the backward;
//   backward (CTAs over 128-column slices x 1024-token chunks): dh[t, c] = dv_t * w[c] (bf16) and
//            dw[c] += sum_t dv_t * h[t, c], db += sum_t dv_t (fp32; one atomic per column and chunk).
//
// The value head is a GEMV (N = 1), so it belongs on the CUDA cores; what the fusion saves is the [T]
// values round trip, the separate loss kernels and the dv / dh / dw passes as individual ops.
#include <cuda_runtime.h>

#include "../include/common.cuh"
#include "misc.h"

namespace meshy {

namespace {

__global__ void value_fwd_kernel(const bf16* __restrict__ h, const float* __restrict__ w, const float* __restrict__ b,
                                 int T, int D,
                                 const float* __restrict__ ret, const float* __restrict__ mask,
                                 const float* __restrict__ old, float clip, float inv_denom, float* __restrict__ v,
                                 float* __restrict__ dv, float* __restrict__ num) {
  __shared__ float part[32];
  const int warps = blockDim.x / 32;
  const int t = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  float contrib = 0.f;
  if (t < T) {
    const bf16* row = h + (size_t)t * D;
    float acc = 0.f;
    for (int c = lane * 8; c < D; c += 32 * 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + c);
      const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = unpack_bf16x2(q[j]);
        acc += x.x * w[c + 2 * j] + x.y * w[c + 2 * j + 1];
      }
    }
    acc = warp_sum(acc) + *b;
    if (lane == 0) {
      const float r = ret[t], m = mask[t];
      float err = (acc - r) * (acc - r);
      float g = 2.f * (acc - r);
      if (old != nullptr && clip > 0.f) {
        const float o = old[t];
        const float d = fminf(fmaxf(acc - o, -clip), clip);
        const float vc = o + d;
        const float errc = (vc - r) * (vc - r);
        // d vc / d v is 1 inside the clip band, 0 outside
        if (errc > err) {
          err = errc;
          g = (acc - o > -clip && acc - o < clip) ? 2.f * (vc - r) : 0.f;
        }
      }
      v[t] = acc;
      dv[t] = g * m * inv_denom;
      contrib = err * m;
    }
  }
  contrib = warp_sum(contrib);
  if (lane == 0) part[threadIdx.x / 32] = contrib;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < warps; ++i) s += part[i];
    atomicAdd(num, s);
  }
}

// CTA (x, y) handles columns [128 x, 128 x + 128) of tokens [kTokChunk y, kTokChunk (y + 1)): every thread owns
// one column, walks the chunk, writes dh and adds its partial of dw (one atomic per column and chunk).
constexpr int kTokChunk = 1024;

__global__ void value_bwd_kernel(const bf16* __restrict__ h, const float* __restrict__ w,
                                 const float* __restrict__ dv, int T, int D, bf16* __restrict__ dh,
                                 float* __restrict__ dw, float* __restrict__ db) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int t0 = blockIdx.y * kTokChunk, t1 = min(T, t0 + kTokChunk);
  if (c < D) {
    const float wc = w[c];
    float acc = 0.f;
    for (int t = t0; t < t1; ++t) {
      const float g = dv[t];
      acc += g * __bfloat162float(h[(size_t)t * D + c]);
      dh[(size_t)t * D + c] = __float2bfloat16(g * wc);
    }
    atomicAdd(dw + c, acc);
  }
  if (blockIdx.x == 0 && threadIdx.x < 32) {
    float acc = 0.f;
    for (int t = t0 + threadIdx.x; t < t1; t += 32) acc += dv[t];
    acc = warp_sum(acc);
    if (threadIdx.x == 0) atomicAdd(db, acc);
  }
}

}  // namespace

void value_head_fwd(const bf16* h, const float* w, const float* b, int T, int D, const float* ret, const float* mask,
                    const float* old, float clip, float inv_denom, float* v, float* dv, float* num, cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0, "value head: hidden size must be a multiple of 8");
  if (T == 0) return;
  const int threads = 256, warps = threads / 32;
  value_fwd_kernel<<<(T + warps - 1) / warps, threads, 0, st>>>(h, w, b, T, D, ret, mask, old, clip, inv_denom, v,
                                                                  dv, num);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void value_head_bwd(const bf16* h, const float* w, const float* dv, int T, int D, bf16* dh, float* dw, float* db,
                    cudaStream_t st) {
  if (T == 0) return;
  dim3 grid((D + 127) / 128, (T + kTokChunk - 1) / kTokChunk);
  value_bwd_kernel<<<grid, 128, 0, st>>>(h, w, dv, T, D, dh, dw, db);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
