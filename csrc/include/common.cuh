// Shared helpers for the kernel library: checks, bf16 packing, warp reductions.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <utility>

#define MESHY_CUDA_CHECK(expr)                                                                  \
  do {                                                                                          \
    cudaError_t _e = (expr);                                                                    \
    if (_e != cudaSuccess)                                                                      \
      throw std::runtime_error(std::string("CUDA error ") + cudaGetErrorString(_e) + " at " + \
                               __FILE__ + ":" + std::to_string(__LINE__));                      \
  } while (0)

#define MESHY_CHECK(cond, msg)                                                  \
  do {                                                                          \
    if (!(cond)) throw std::runtime_error(std::string("meshy_b200: ") + (msg)); \
  } while (0)

namespace meshy {

using bf16 = __nv_bfloat16;

// ─── programmatic dependent launch (PDL) ────────────────────────────────────
// Kernels of the decode step are launched with programmatic stream
// serialisation: a kernel may start (prologue, barrier init, TMEM alloc, weight
// prefetch) while its predecessor in the stream finishes, and calls pdl_wait()
// before it touches anything the predecessor wrote.  pdl_trigger() lets the
// successor start early.  Both are no-ops for a kernel launched normally.
bool pdl_enabled();  // env MESHY_PDL (default on)

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("CUDA error ") + cudaGetErrorString(e) + " in launch_pdl");
}

#if defined(__CUDACC__)

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(h);
}

// Counter-based random numbers: Philox4x32-10 (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011), implemented from
// the paper's round function and its published multipliers / Weyl constants.
struct Philox {
  __device__ __forceinline__ static uint4 round(uint4 c, uint2 k) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
    uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    return make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  __device__ __forceinline__ static uint4 gen(uint4 ctr, uint2 key) {
    const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int i = 0; i < 10; ++i) {
      ctr = round(ctr, key);
      key.x += W0;
      key.y += W1;
    }
    return ctr;
  }
};

// Uniform in (0, 1): 23 random bits, offset by half a step so 0 and 1 never occur. (With 24 bits the
// top value 2^24 - 0.5 is not a float and rounds to 2^24, i.e. u = 1 exactly and log(u) = 0.)
__device__ __forceinline__ float u01(uint32_t x) { return ((x >> 9) + 0.5f) * (1.0f / 8388608.0f); }

// Standard Gumbel variate -log(-log(u)) from 32 random bits. The inner -log(u) must be accurate relative
// to its value: u can lie within 2^-24 of 1, where -log(u) is ~6e-8 and the fast __logf's absolute error
// (~1e-7) could make it zero or negative -- an infinite or NaN perturbation that hands the draw to an
// arbitrary token (a few draws in 10^7, a few percent of the rows of a 152k-entry vocabulary). Near 1 it
// is the Taylor series -log(1 - v) = v + v^2/2 + v^3/3 + v^4/4 (v = 1 - u is exact, truncation < v^5/5);
// elsewhere |log u| > 0.01 and the fast log's relative error stays below 2e-5.
__device__ __forceinline__ float gumbel(uint32_t bits) {
  const float u = u01(bits);
  const float v = 1.0f - u;
  const float e = v < 0.01f ? v * (1.0f + v * (0.5f + v * (1.0f / 3.0f + v * 0.25f))) : -__logf(u);
  return -__logf(e);
}
#endif  // __CUDACC__

}  // namespace meshy
