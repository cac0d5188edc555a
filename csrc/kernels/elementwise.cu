// Memory-bound kernels: RMSNorm fwd/bwd, QKV split + QK-norm + RoPE fwd/bwd,
// SwiGLU backward, embedding fwd/bwd, dtype cast copies.
//
// All are one pass over HBM with 16-byte vector accesses; reductions stay in
// registers/warps; weight gradients are accumulated in fp32 per block and
// flushed with one atomicAdd per column per block.
#include "../include/common.cuh"
#include "elementwise.h"

namespace meshy {

// ─── RMSNorm ────────────────────────────────────────────────────────────────
// One warp per row; lane owns columns {8*lane + 256*j .. +8}.
template <int VPT>  // 8-element vectors per lane
__global__ void rmsnorm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ y,
                                   float* __restrict__ rstd, int rows, int D, float eps) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  pdl_wait();
  pdl_trigger();
  for (int r = blockIdx.x * warps + threadIdx.x / 32; r < rows; r += gridDim.x * warps) {
    const bf16* xr = x + (size_t)r * D;
    float v[VPT * 8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int c = (j * 32 + lane) * 8;
      if (c < D) {
        uint4 u = *reinterpret_cast<const uint4*>(xr + c);
        uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 f = unpack_bf16x2(uu[t]);
          v[j * 8 + 2 * t] = f.x;
          v[j * 8 + 2 * t + 1] = f.y;
          ss += f.x * f.x + f.y * f.y;
        }
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / D + eps);
    if (lane == 0 && rstd) rstd[r] = rs;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int c = (j * 32 + lane) * 8;
      if (c < D) {
        uint4 wu = *reinterpret_cast<const uint4*>(w + c);
        uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
        uint32_t o[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 wf = unpack_bf16x2(ww[t]);
          o[t] = pack_bf16x2(v[j * 8 + 2 * t] * rs * wf.x, v[j * 8 + 2 * t + 1] * rs * wf.y);
        }
        *reinterpret_cast<uint4*>(y + (size_t)r * D + c) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

template <int VPT>
__global__ void rmsnorm_bwd_kernel(const bf16* __restrict__ gy, const bf16* __restrict__ x, const bf16* __restrict__ w,
                                   const float* __restrict__ rstd, bf16* __restrict__ gx, float* __restrict__ gw,
                                   int rows, int D) {
  // Two passes over the row (the second hits L1): pass 1 forms mean(dxh * xh),
  // pass 2 writes gx.  dw accumulates in registers for D <= 2048, else in smem.
  constexpr bool kRegDw = VPT <= 8;
  extern __shared__ float sdw[];
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  float dw[kRegDw ? VPT * 8 : 1];
  if (kRegDw) {
#pragma unroll
    for (int i = 0; i < (kRegDw ? VPT * 8 : 1); ++i) dw[i] = 0.f;
  }
  for (int i = threadIdx.x; i < D; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  for (int r = blockIdx.x * warps + threadIdx.x / 32; r < rows; r += gridDim.x * warps) {
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int c = (j * 32 + lane) * 8;
      if (c < D) {
        uint4 xu = *reinterpret_cast<const uint4*>(x + (size_t)r * D + c);
        uint4 gu = *reinterpret_cast<const uint4*>(gy + (size_t)r * D + c);
        uint4 wu = *reinterpret_cast<const uint4*>(w + c);
        uint32_t xx[4] = {xu.x, xu.y, xu.z, xu.w}, gg[4] = {gu.x, gu.y, gu.z, gu.w}, ww[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 xf = unpack_bf16x2(xx[t]), gf = unpack_bf16x2(gg[t]), wf = unpack_bf16x2(ww[t]);
          dot += gf.x * wf.x * xf.x * rs + gf.y * wf.y * xf.y * rs;
        }
      }
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int c = (j * 32 + lane) * 8;
      if (c < D) {
        uint4 xu = *reinterpret_cast<const uint4*>(x + (size_t)r * D + c);
        uint4 gu = *reinterpret_cast<const uint4*>(gy + (size_t)r * D + c);
        uint4 wu = *reinterpret_cast<const uint4*>(w + c);
        uint32_t xx[4] = {xu.x, xu.y, xu.z, xu.w}, gg[4] = {gu.x, gu.y, gu.z, gu.w}, ww[4] = {wu.x, wu.y, wu.z, wu.w};
        uint32_t o[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 xf = unpack_bf16x2(xx[t]), gf = unpack_bf16x2(gg[t]), wf = unpack_bf16x2(ww[t]);
          float xh0 = xf.x * rs, xh1 = xf.y * rs;
          o[t] = pack_bf16x2(rs * (gf.x * wf.x - xh0 * dot), rs * (gf.y * wf.y - xh1 * dot));
          if (kRegDw) {
            dw[(j * 8 + 2 * t) % (kRegDw ? VPT * 8 : 1)] += gf.x * xh0;
            dw[(j * 8 + 2 * t + 1) % (kRegDw ? VPT * 8 : 1)] += gf.y * xh1;
          } else {
            atomicAdd(&sdw[c + 2 * t], gf.x * xh0);
            atomicAdd(&sdw[c + 2 * t + 1], gf.y * xh1);
          }
        }
        *reinterpret_cast<uint4*>(gx + (size_t)r * D + c) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  if (kRegDw) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      int c = (j * 32 + lane) * 8;
      if (c < D)
#pragma unroll
        for (int t = 0; t < 8; ++t) atomicAdd(&sdw[c + t], dw[(j * 8 + t) % (kRegDw ? VPT * 8 : 1)]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) atomicAdd(&gw[i], sdw[i]);
}

static int grid_for(int rows, int warps_per_block) {
  int blocks = (rows + warps_per_block - 1) / warps_per_block;
  return std::max(1, std::min(blocks, 148 * 8));
}

void rmsnorm_fwd(const bf16* x, const bf16* w, bf16* y, float* rstd, int rows, int D, float eps, cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0 && D <= 8192, "rmsnorm: D must be a multiple of 8 and <= 8192");
  const int vpt = (D + 255) / 256;
  dim3 block(256);
  int grid = grid_for(rows, 8);
#define RMS_F(V) launch_pdl(rmsnorm_fwd_kernel<V>, dim3(grid), block, 0, st, x, w, y, rstd, rows, D, eps)
  if (vpt <= 1) RMS_F(1);
  else if (vpt <= 2) RMS_F(2);
  else if (vpt <= 4) RMS_F(4);
  else if (vpt <= 8) RMS_F(8);
  else if (vpt <= 16) RMS_F(16);
  else RMS_F(32);
#undef RMS_F
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(const bf16* gy, const bf16* x, const bf16* w, const float* rstd, bf16* gx, float* gw, int rows, int D,
                 cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0 && D <= 8192, "rmsnorm: D must be a multiple of 8 and <= 8192");
  const int vpt = (D + 255) / 256;
  dim3 block(256);
  int grid = std::max(1, std::min((rows + 7) / 8, 148 * 2));
  size_t sm = D * sizeof(float);
#define RMS_B(V) rmsnorm_bwd_kernel<V><<<grid, block, sm, st>>>(gy, x, w, rstd, gx, gw, rows, D)
  if (vpt <= 1) RMS_B(1);
  else if (vpt <= 2) RMS_B(2);
  else if (vpt <= 4) RMS_B(4);
  else if (vpt <= 8) RMS_B(8);
  else if (vpt <= 16) RMS_B(16);
  else RMS_B(32);
#undef RMS_B
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── QKV split + QK-norm + RoPE ─────────────────────────────────────────────
// One warp per (token, head) of the fused qkv row; lane l owns dims
// {2l, 2l+1} of the first half and their rotate-half partners {2l+hd/2, ...}.
// head_dim 64 or 128 (hd/4 lanes active for hd 64).
__global__ void qkv_rope_fwd_kernel(const bf16* __restrict__ qkv, const int* __restrict__ pos,
                                    const bf16* __restrict__ qn, const bf16* __restrict__ kn,
                                    const float* __restrict__ inv_freq, bf16* __restrict__ q, bf16* __restrict__ k,
                                    bf16* __restrict__ v, int T, int Hq, int Hkv, int hd, float eps,
                                    bf16* __restrict__ kc, bf16* __restrict__ vc, const int64_t* __restrict__ slots,
                                    int page) {
  const int H = Hq + 2 * Hkv;
  const int lane = threadIdx.x % 32;
  const long long gw = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  pdl_wait();
  pdl_trigger();
  if (gw >= (long long)T * H) return;
  const int t = (int)(gw / H), h = (int)(gw % H);
  const int half = hd / 2;
  // paged-cache row of this token for head hh: [n_pages, Hkv, page, hd]
  auto cache_row = [&](bf16* base, int hh) -> bf16* {
    const int64_t slot = slots[t];
    return base + (((size_t)(slot / page) * Hkv + hh) * page + (size_t)(slot % page)) * hd;
  };
  const bf16* src = qkv + (size_t)t * H * hd + (size_t)h * hd;
  const int i0 = 2 * lane;
  const bool act = i0 < half;
  float a0 = 0, a1 = 0, b0 = 0, b1 = 0;
  if (act) {
    float2 fa = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + i0));
    float2 fb = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + i0 + half));
    a0 = fa.x; a1 = fa.y; b0 = fb.x; b1 = fb.y;
  }
  if (h >= Hq + Hkv) {  // V: plain copy (to the v tensor and/or the paged cache)
    if (act) {
      const uint32_t lo = pack_bf16x2(a0, a1), hi = pack_bf16x2(b0, b1);
      if (v) {
        bf16* dst = v + ((size_t)t * Hkv + (h - Hq - Hkv)) * hd;
        *reinterpret_cast<uint32_t*>(dst + i0) = lo;
        *reinterpret_cast<uint32_t*>(dst + i0 + half) = hi;
      }
      if (vc) {
        bf16* dst = cache_row(vc, h - Hq - Hkv);
        *reinterpret_cast<uint32_t*>(dst + i0) = lo;
        *reinterpret_cast<uint32_t*>(dst + i0 + half) = hi;
      }
    }
    return;
  }
  const bool is_q = h < Hq;
  const bf16* nw = is_q ? qn : kn;
  if (nw) {
    float ss = warp_sum(a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1);
    float rs = rsqrtf(ss / hd + eps);
    if (act) {
      // round-trip through bf16 like the unfused path (norm output is bf16)
      a0 = __bfloat162float(__float2bfloat16(a0 * rs * __bfloat162float(nw[i0])));
      a1 = __bfloat162float(__float2bfloat16(a1 * rs * __bfloat162float(nw[i0 + 1])));
      b0 = __bfloat162float(__float2bfloat16(b0 * rs * __bfloat162float(nw[i0 + half])));
      b1 = __bfloat162float(__float2bfloat16(b1 * rs * __bfloat162float(nw[i0 + half + 1])));
    }
  }
  if (!act) return;
  const float p = (float)pos[t];
  float s0, c0, s1, c1;
  sincosf(p * inv_freq[i0], &s0, &c0);
  sincosf(p * inv_freq[i0 + 1], &s1, &c1);
  float o_a0 = a0 * c0 - b0 * s0, o_b0 = b0 * c0 + a0 * s0;
  float o_a1 = a1 * c1 - b1 * s1, o_b1 = b1 * c1 + a1 * s1;
  const uint32_t lo = pack_bf16x2(o_a0, o_a1), hi = pack_bf16x2(o_b0, o_b1);
  bf16* dst = is_q ? q + ((size_t)t * Hq + h) * hd : (k ? k + ((size_t)t * Hkv + (h - Hq)) * hd : nullptr);
  if (dst) {
    *reinterpret_cast<uint32_t*>(dst + i0) = lo;
    *reinterpret_cast<uint32_t*>(dst + i0 + half) = hi;
  }
  if (!is_q && kc) {
    bf16* c = cache_row(kc, h - Hq);
    *reinterpret_cast<uint32_t*>(c + i0) = lo;
    *reinterpret_cast<uint32_t*>(c + i0 + half) = hi;
  }
}

__global__ void qkv_rope_bwd_kernel(const bf16* __restrict__ qkv, const int* __restrict__ pos,
                                    const bf16* __restrict__ qn, const bf16* __restrict__ kn,
                                    const float* __restrict__ inv_freq, const bf16* __restrict__ gq,
                                    const bf16* __restrict__ gk, const bf16* __restrict__ gv, bf16* __restrict__ gqkv,
                                    float* __restrict__ gqn, float* __restrict__ gkn, int T, int Hq, int Hkv, int hd,
                                    float eps) {
  const int H = Hq + 2 * Hkv;
  const int lane = threadIdx.x % 32;
  const long long gwid = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (gwid >= (long long)T * H) return;
  const int t = (int)(gwid / H), h = (int)(gwid % H);
  const int half = hd / 2;
  const int i0 = 2 * lane;
  const bool act = i0 < half;
  bf16* dst = gqkv + (size_t)t * H * hd + (size_t)h * hd;
  if (h >= Hq + Hkv) {
    if (act) {
      const bf16* g = gv + ((size_t)t * Hkv + (h - Hq - Hkv)) * hd;
      *reinterpret_cast<uint32_t*>(dst + i0) = *reinterpret_cast<const uint32_t*>(g + i0);
      *reinterpret_cast<uint32_t*>(dst + i0 + half) = *reinterpret_cast<const uint32_t*>(g + i0 + half);
    }
    return;
  }
  const bool is_q = h < Hq;
  const bf16* g = is_q ? gq + ((size_t)t * Hq + h) * hd : gk + ((size_t)t * Hkv + (h - Hq)) * hd;
  float ga0 = 0, ga1 = 0, gb0 = 0, gb1 = 0;
  if (act) {
    float2 fa = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(g + i0));
    float2 fb = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(g + i0 + half));
    const float p = (float)pos[t];
    float s0, c0, s1, c1;
    sincosf(p * inv_freq[i0], &s0, &c0);
    sincosf(p * inv_freq[i0 + 1], &s1, &c1);
    // inverse rotation (transpose of the forward 2x2 rotation)
    ga0 = fa.x * c0 + fb.x * s0;
    gb0 = fb.x * c0 - fa.x * s0;
    ga1 = fa.y * c1 + fb.y * s1;
    gb1 = fb.y * c1 - fa.y * s1;
  }
  const bf16* nw = is_q ? qn : kn;
  if (nw) {
    const bf16* src = qkv + (size_t)t * H * hd + (size_t)h * hd;
    float x0 = 0, x1 = 0, y0 = 0, y1 = 0;
    if (act) {
      float2 fa = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + i0));
      float2 fb = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + i0 + half));
      x0 = fa.x; x1 = fa.y; y0 = fb.x; y1 = fb.y;
    }
    float ss = warp_sum(x0 * x0 + x1 * x1 + y0 * y0 + y1 * y1);
    float rs = rsqrtf(ss / hd + eps);
    float w0 = act ? __bfloat162float(nw[i0]) : 0.f, w1 = act ? __bfloat162float(nw[i0 + 1]) : 0.f;
    float w2 = act ? __bfloat162float(nw[i0 + half]) : 0.f, w3 = act ? __bfloat162float(nw[i0 + half + 1]) : 0.f;
    float xh0 = x0 * rs, xh1 = x1 * rs, yh0 = y0 * rs, yh1 = y1 * rs;
    float d0 = ga0 * w0, d1 = ga1 * w1, d2 = gb0 * w2, d3 = gb1 * w3;
    float dot = warp_sum(d0 * xh0 + d1 * xh1 + d2 * yh0 + d3 * yh1) / hd;
    if (act) {
      float* gw = is_q ? gqn : gkn;
      atomicAdd(&gw[i0], ga0 * xh0);
      atomicAdd(&gw[i0 + 1], ga1 * xh1);
      atomicAdd(&gw[i0 + half], gb0 * yh0);
      atomicAdd(&gw[i0 + half + 1], gb1 * yh1);
    }
    ga0 = rs * (d0 - xh0 * dot);
    ga1 = rs * (d1 - xh1 * dot);
    gb0 = rs * (d2 - yh0 * dot);
    gb1 = rs * (d3 - yh1 * dot);
  }
  if (act) {
    *reinterpret_cast<uint32_t*>(dst + i0) = pack_bf16x2(ga0, ga1);
    *reinterpret_cast<uint32_t*>(dst + i0 + half) = pack_bf16x2(gb0, gb1);
  }
}

void qkv_rope_fwd(const bf16* qkv, const int* pos, const bf16* qn, const bf16* kn, const float* inv_freq, bf16* q,
                  bf16* k, bf16* v, int T, int Hq, int Hkv, int hd, float eps, cudaStream_t st, bf16* kc, bf16* vc,
                  const int64_t* slots, int page) {
  MESHY_CHECK(hd % 4 == 0 && hd <= 128, "qkv_rope: head_dim must be <= 128 and a multiple of 4");
  MESHY_CHECK((kc == nullptr) == (vc == nullptr) && (kc == nullptr || (slots != nullptr && page > 0)),
              "qkv_rope: cache write needs both caches, the slot map and the page size");
  MESHY_CHECK((k != nullptr || kc != nullptr) && (v != nullptr || vc != nullptr), "qkv_rope: K/V have no destination");
  long long warps = (long long)T * (Hq + 2 * Hkv);
  int grid = (int)((warps + 7) / 8);
  if (grid == 0) return;
  launch_pdl(qkv_rope_fwd_kernel, dim3(grid), dim3(256), 0, st, qkv, pos, qn, kn, inv_freq, q, k, v, T, Hq, Hkv, hd,
             eps, kc, vc, slots, page);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void qkv_rope_bwd(const bf16* qkv, const int* pos, const bf16* qn, const bf16* kn, const float* inv_freq,
                  const bf16* gq, const bf16* gk, const bf16* gv, bf16* gqkv, float* gqn, float* gkn, int T, int Hq,
                  int Hkv, int hd, float eps, cudaStream_t st) {
  long long warps = (long long)T * (Hq + 2 * Hkv);
  int grid = (int)((warps + 7) / 8);
  if (grid == 0) return;
  qkv_rope_bwd_kernel<<<grid, 256, 0, st>>>(qkv, pos, qn, kn, inv_freq, gq, gk, gv, gqkv, gqn, gkn, T, Hq, Hkv, hd,
                                            eps);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── SwiGLU backward (block-interleaved gate/up, block 64) ──────────────────
__global__ void swiglu_bwd_kernel(const bf16* __restrict__ h, const bf16* __restrict__ ga, bf16* __restrict__ dh,
                                  long long T, int F, int blk) {
  // one thread per 8 output columns
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long per_row = F / 8;
  if (idx >= T * per_row) return;
  long long t = idx / per_row;
  int f = (int)(idx % per_row) * 8;
  int b = f / blk, o = f % blk;
  const bf16* hr = h + t * 2 * F;
  size_t gi = (size_t)b * 2 * blk + o, ui = gi + blk;
  uint4 gu = *reinterpret_cast<const uint4*>(hr + gi);
  uint4 uu = *reinterpret_cast<const uint4*>(hr + ui);
  uint4 au = *reinterpret_cast<const uint4*>(ga + t * F + f);
  uint32_t g4[4] = {gu.x, gu.y, gu.z, gu.w}, u4[4] = {uu.x, uu.y, uu.z, uu.w}, a4[4] = {au.x, au.y, au.z, au.w};
  uint32_t dg[4], du[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 g = unpack_bf16x2(g4[i]), u = unpack_bf16x2(u4[i]), a = unpack_bf16x2(a4[i]);
    float s0 = 1.f / (1.f + __expf(-g.x)), s1 = 1.f / (1.f + __expf(-g.y));
    float sl0 = g.x * s0, sl1 = g.y * s1;
    dg[i] = pack_bf16x2(a.x * u.x * s0 * (1.f + g.x * (1.f - s0)), a.y * u.y * s1 * (1.f + g.y * (1.f - s1)));
    du[i] = pack_bf16x2(a.x * sl0, a.y * sl1);
  }
  bf16* dr = dh + t * 2 * F;
  *reinterpret_cast<uint4*>(dr + gi) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
  *reinterpret_cast<uint4*>(dr + ui) = make_uint4(du[0], du[1], du[2], du[3]);
}

void swiglu_bwd(const bf16* h, const bf16* ga, bf16* dh, long long T, int F, int blk, cudaStream_t st) {
  MESHY_CHECK(F % blk == 0 && blk % 8 == 0, "swiglu_bwd: bad block");
  long long n = T * (F / 8);
  if (n == 0) return;
  swiglu_bwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(h, ga, dh, T, F, blk);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── embedding ─────────────────────────────────────────────────────────────
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ w, bf16* __restrict__ out,
                                     long long T, int D, long long V) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long per = D / 8;
  pdl_wait();
  pdl_trigger();
  if (idx >= T * per) return;
  long long t = idx / per;
  int c = (int)(idx % per) * 8;
  long long id = ids[t];
  uint4 val = make_uint4(0, 0, 0, 0);
  if (id >= 0 && id < V) val = *reinterpret_cast<const uint4*>(w + id * D + c);
  *reinterpret_cast<uint4*>(out + t * D + c) = val;
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ g, float* __restrict__ gw,
                                     long long T, int D, long long V) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long per = D / 2;
  if (idx >= T * per) return;
  long long t = idx / per;
  int c = (int)(idx % per) * 2;
  long long id = ids[t];
  if (id < 0 || id >= V) return;
  float2 f = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(g + t * D + c));
  atomicAdd(gw + id * D + c, f.x);
  atomicAdd(gw + id * D + c + 1, f.y);
}

void embedding_fwd(const int64_t* ids, const bf16* w, bf16* out, long long T, int D, long long V, cudaStream_t st) {
  long long n = T * (D / 8);
  if (n == 0) return;
  launch_pdl(embedding_fwd_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, ids, w, out, T, D, V);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void embedding_bwd(const int64_t* ids, const bf16* g, float* gw, long long T, int D, long long V, cudaStream_t st) {
  long long n = T * (D / 2);
  if (n == 0) return;
  embedding_bwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, g, gw, T, D, V);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── casts ─────────────────────────────────────────────────────────────────
__global__ void cast_f32_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, long long n) {
  long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i + 8 <= n) {
    float4 a = *reinterpret_cast<const float4*>(src + i);
    float4 b = *reinterpret_cast<const float4*>(src + i + 4);
    *reinterpret_cast<uint4*>(dst + i) =
        make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
  } else {
    for (; i < n; ++i) dst[i] = __float2bfloat16(src[i]);
  }
}

void cast_f32_bf16(const float* src, bf16* dst, long long n, cudaStream_t st) {
  if (n == 0) return;
  long long threads = (n + 7) / 8;
  cast_f32_bf16_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(src, dst, n);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
