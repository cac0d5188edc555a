// Symmetric peer memory and the fused data-parallel optimiser step over NVLink.
//
// Symmetric heap: every rank of a single-node process group cudaMalloc's a
// buffer of the same size, exports a CUDA IPC handle, and maps every peer's
// buffer into its address space (cudaIpcOpenMemHandle; NVLink peer access
// through NVSwitch).  Kernels then load from and store to peer pointers
// directly (plain ld/st.global; no TMA, no multicast).
//
// Fused DP optimiser step (one rank owns shard [lo, hi) of the flat buffers):
//
//   1. symm_barrier          every rank's gradient is final (release/acquire
//                            flags, bounded spin)
//   2. symm_rs_sumsq         reduce-scatter: sum this shard of the gradient
//                            over all ranks straight from their buffers (P2P
//                            loads), write it into the local gradient shard,
//                            accumulate its squared norm
//   3. symm_norm_exchange    push the shard norm to every peer, wait for all,
//                            global gradient norm (fixed summation order, so
//                            every rank computes the identical value)
//   4. symm_adamw_push       clip + AdamW on the shard (moments stay local,
//                            ZeRO-1 style), then all-gather by P2P stores.
//                            With a bf16 compute copy the fp32 master is
//                            sharded too: the shard is written locally and
//                            only the bf16 values go to every rank (2 bytes
//                            per parameter cross NVLink instead of 6); with
//                            fp32 compute the master itself is pushed
//   5. symm_barrier          nobody reuses its gradient or parameters before
//                            every peer has finished reading and writing.
//
// The AdamW arithmetic is the same as adamw_kernel (misc.cu), so the fused
// path and the NCCL path produce the same update.
//
// Every spin is bounded by a clock64 deadline: on timeout the kernel records
// kErrTimeoutPeer in the error word, skips its remaining work and returns; the
// host reads the word and raises.  A rank never waits on a flag that only a
// kernel on the same GPU could set.
#include <cuda_runtime.h>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "symm.h"

namespace meshy {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One CTA; thread p < world signals peer p and waits for peer p's signal.
__global__ void symm_barrier_kernel(const unsigned long long* __restrict__ flag_ptrs, int rank, int world,
                                    unsigned int epoch, long long timeout_cycles, int* err) {
  const int p = threadIdx.x;
  if (p < world) {
    // flags of rank q: world u32 slots, slot r = last epoch rank r reached
    unsigned int* peer_flags = reinterpret_cast<unsigned int*>(flag_ptrs[p]);
    __threadfence_system();
    st_release_sys(peer_flags + rank, epoch);
    const unsigned int* mine = reinterpret_cast<const unsigned int*>(flag_ptrs[rank]) + p;
    long long t0 = clock64();
    while ((int)(ld_acquire_sys(mine) - epoch) < 0) {
      if (clock64() - t0 > timeout_cycles) {
        atomicCAS(err, 0, (int)kErrTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
}

// grad shard [lo, hi): out = sum over ranks q of grad_q[i] (rank order), sumsq += out^2
__global__ void symm_rs_sumsq_kernel(const unsigned long long* __restrict__ grad_ptrs, int world, long long lo,
                                     long long hi, float* __restrict__ local_grad, float* __restrict__ sumsq,
                                     const int* __restrict__ err) {
  if (*err) return;
  __shared__ float sh[32];
  float acc = 0.f;
  const long long n = hi - lo;
  const long long n4 = n / 4;  // lo and the shard length are multiples of 4 (host checks)
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = lo + 4 * i;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < world; ++q) {
      const float4 g = __ldcv(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(grad_ptrs[q]) + e));
      s.x += g.x; s.y += g.y; s.z += g.z; s.w += g.w;
    }
    *reinterpret_cast<float4*>(local_grad + e) = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  acc = warp_sum(acc);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) sh[w] = acc;
  __syncthreads();
  if (w == 0) {
    acc = (l < (int)(blockDim.x / 32)) ? sh[l] : 0.f;
    acc = warp_sum(acc);
    if (l == 0) atomicAdd(sumsq, acc);
  }
}

// One CTA: publish this rank's shard sum of squares into every peer's slot array, wait for all,
// write sqrt(sum over ranks in rank order) to *norm.
__global__ void symm_norm_exchange_kernel(const unsigned long long* __restrict__ slot_ptrs,
                                          const unsigned long long* __restrict__ flag_ptrs, int rank, int world,
                                          unsigned int epoch, const float* __restrict__ sumsq, float* __restrict__ norm,
                                          long long timeout_cycles, int* err) {
  const int p = threadIdx.x;
  __shared__ int failed;
  if (p == 0) failed = 0;
  __syncthreads();
  if (p < world && !*err) {
    float* peer_slots = reinterpret_cast<float*>(slot_ptrs[p]);
    peer_slots[rank] = *sumsq;
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned int*>(flag_ptrs[p]) + rank, epoch);
    const unsigned int* mine = reinterpret_cast<const unsigned int*>(flag_ptrs[rank]) + p;
    long long t0 = clock64();
    while ((int)(ld_acquire_sys(mine) - epoch) < 0) {
      if (clock64() - t0 > timeout_cycles) {
        atomicCAS(err, 0, (int)kErrTimeoutPeer);
        failed = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (p == 0) {
    float total = 0.f;
    const volatile float* slots = reinterpret_cast<const volatile float*>(slot_ptrs[rank]);
    for (int q = 0; q < world; ++q) total += slots[q];
    *norm = (failed || *err) ? 0.f : sqrtf(total);
  }
}

__global__ void symm_adamw_push_kernel(const unsigned long long* __restrict__ master_ptrs,
                                       const unsigned long long* __restrict__ compute_ptrs,
                                       float* __restrict__ master_local, int world, long long lo,
                                       long long hi, const float* __restrict__ g, float* __restrict__ m,
                                       float* __restrict__ v, const float* __restrict__ norm, float max_norm, float lr,
                                       float b1, float b2, float eps, float wd, float bc1, float bc2,
                                       const int* __restrict__ err) {
  if (*err) return;
  float coef = 1.f;
  if (max_norm > 0.f) coef = fminf(1.f, max_norm / (*norm + 1e-6f));
  const float step = lr / bc1, inv_bc2 = 1.f / bc2, decay = 1.f - lr * wd;
  const long long n4 = (hi - lo) / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = lo + 4 * i;
    float4 pp = *reinterpret_cast<const float4*>(master_local + e);
    const float4 gg = *reinterpret_cast<const float4*>(g + e);
    // moments hold only this rank's shard [lo, hi)
    float4 mm = *reinterpret_cast<const float4*>(m + 4 * i), vv = *reinterpret_cast<const float4*>(v + 4 * i);
    float* P = &pp.x;
    const float* G = &gg.x;
    float* Mv = &mm.x;
    float* Vv = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float gk = G[k] * coef;
      Mv[k] = b1 * Mv[k] + (1.f - b1) * gk;
      Vv[k] = b2 * Vv[k] + (1.f - b2) * gk * gk;
      P[k] = P[k] * decay - step * Mv[k] / (sqrtf(Vv[k] * inv_bc2) + eps);
    }
    *reinterpret_cast<float4*>(m + 4 * i) = mm;
    *reinterpret_cast<float4*>(v + 4 * i) = vv;
    const uint2 packed = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
    if (master_ptrs == nullptr) {
      // master weights sharded like the moments: the fp32 shard stays here, only bf16 crosses NVLink
      *reinterpret_cast<float4*>(master_local + e) = pp;
      for (int q = 0; q < world; ++q)
        *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(compute_ptrs[q]) + e) = packed;
    } else {
      for (int q = 0; q < world; ++q) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(master_ptrs[q]) + e) = pp;
        if (compute_ptrs) *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(compute_ptrs[q]) + e) = packed;
      }
    }
  }
}

}  // namespace

// ═══════════════════════════════ host ══════════════════════════════════════

void* symm_malloc(size_t bytes) {
  void* p = nullptr;
  MESHY_CUDA_CHECK(cudaMalloc(&p, bytes));
  MESHY_CUDA_CHECK(cudaMemset(p, 0, bytes));
  return p;
}

void symm_free(void* p) {
  if (p) MESHY_CUDA_CHECK(cudaFree(p));
}

std::string symm_export(void* p) {
  cudaIpcMemHandle_t h;
  MESHY_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void* symm_import(const std::string& handle) {
  MESHY_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "symm_import: bad handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  MESHY_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void symm_close(void* p) {
  if (p) MESHY_CUDA_CHECK(cudaIpcCloseMemHandle(p));
}

// The SM clock rate is read once per device: the attribute query costs milliseconds of host time on this
// driver, which stalled every optimiser step (and every barrier) while the GPU waited for the next launch.
static long long cycles_for(double seconds) {
  static int khz_of[64] = {};
  int dev = 0;
  MESHY_CUDA_CHECK(cudaGetDevice(&dev));
  int& khz = khz_of[dev & 63];
  if (khz == 0) MESHY_CUDA_CHECK(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev));
  return (long long)(seconds * (double)khz * 1000.0);
}

void symm_barrier(const unsigned long long* flag_ptrs, int rank, int world, unsigned int epoch, double timeout_s,
                  int* err, cudaStream_t st) {
  MESHY_CHECK(world >= 1 && world <= 32, "symm_barrier: 1..32 ranks");
  symm_barrier_kernel<<<1, 32, 0, st>>>(flag_ptrs, rank, world, epoch, cycles_for(timeout_s), err);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void symm_dp_adamw_step(const SymmAdamWArgs& a, cudaStream_t st) {
  MESHY_CHECK(a.world >= 1 && a.world <= 32, "fused DP step: 1..32 ranks");
  MESHY_CHECK(a.lo % 4 == 0 && (a.hi - a.lo) % 4 == 0, "fused DP step: shard bounds must be multiples of 4");
  const long long cyc = cycles_for(a.timeout_s);
  symm_barrier_kernel<<<1, 32, 0, st>>>(a.flag_ptrs, a.rank, a.world, a.epoch, cyc, a.err);
  MESHY_CUDA_CHECK(cudaMemsetAsync(a.sumsq, 0, sizeof(float), st));
  const long long n4 = (a.hi - a.lo) / 4;
  const int grid = (int)std::max<long long>(1, std::min<long long>((n4 + 255) / 256, 148 * 8));
  if (n4 > 0)
    symm_rs_sumsq_kernel<<<grid, 256, 0, st>>>(a.grad_ptrs, a.world, a.lo, a.hi, a.local_grad, a.sumsq, a.err);
  symm_norm_exchange_kernel<<<1, 32, 0, st>>>(a.slot_ptrs, a.flag_ptrs, a.rank, a.world, a.epoch + 1, a.sumsq,
                                              a.norm, cyc, a.err);
  const float bc1 = 1.f - powf(a.b1, (float)a.step), bc2 = 1.f - powf(a.b2, (float)a.step);
  if (n4 > 0)
    symm_adamw_push_kernel<<<grid, 256, 0, st>>>(a.master_ptrs, a.compute_ptrs, a.master_local, a.world, a.lo, a.hi,
                                                 a.local_grad,
                                                 a.exp_avg, a.exp_avg_sq, a.norm, a.max_norm, a.lr, a.b1, a.b2, a.eps,
                                                 a.wd, bc1, bc2, a.err);
  symm_barrier_kernel<<<1, 32, 0, st>>>(a.flag_ptrs, a.rank, a.world, a.epoch + 2, cyc, a.err);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
