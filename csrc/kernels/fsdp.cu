// Sharded-parameter collectives over NVLink peer memory (sm_100a), for one process per GPU on one node.
//
//   fsdp_gather   every rank's shard of one unit -> this rank's full-size buffer: CTA row y reads rank y's
//                 shard through its IPC mapping (16-byte loads over NVLink) and writes it to [y * n, (y + 1) * n)
//                 of the local buffer. The shards are only rewritten by the optimiser step, which the host
//                 brackets with a device barrier, so the copy needs no flags of its own.
//   fsdp_reduce   this rank's shard of the summed gradient: dst[j] += sum_r grad_r[rank * n + j], the peers'
//                 full-size fp32 gradient buffers read in rank order (the same order on every rank, so the sum
//                 is deterministic). The host puts a device barrier before it (every rank's gradients of the
//                 unit are complete) and after it (every rank has read this rank's buffer before it is zeroed).
//
// Only plain loads and stores touch peer memory; no TMA and no multicast.
#include <cuda_runtime.h>

#include "../include/common.cuh"
#include "symm.h"

namespace meshy {

namespace {

__global__ void fsdp_gather_kernel(const unsigned long long* __restrict__ ptrs, long long off_bytes, long long n16,
                                   uint4* __restrict__ dst) {
  const int r = blockIdx.y;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(ptrs[r]) + off_bytes);
  uint4* out = dst + (size_t)r * n16;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  // four independent loads in flight per thread before the stores
  for (; j + 3 * stride < n16; j += 4 * stride) {
    const uint4 a = src[j], b = src[j + stride], c = src[j + 2 * stride], d = src[j + 3 * stride];
    out[j] = a;
    out[j + stride] = b;
    out[j + 2 * stride] = c;
    out[j + 3 * stride] = d;
  }
  for (; j < n16; j += stride) out[j] = src[j];
}

__global__ void fsdp_reduce_kernel(const unsigned long long* __restrict__ ptrs, long long off_bytes, long long n4,
                                   int rank, int world, float4* __restrict__ dst) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < n4; j += stride) {
    float4 v[kMaxPeers];
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r < world) {
        const float4* src =
            reinterpret_cast<const float4*>(reinterpret_cast<const char*>(ptrs[r]) + off_bytes) + (size_t)rank * n4;
        v[r] = src[j];
      }
    }
    float4 acc = dst[j];
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r < world) {
        acc.x += v[r].x;
        acc.y += v[r].y;
        acc.z += v[r].z;
        acc.w += v[r].w;
      }
    }
    dst[j] = acc;
  }
}

int sm_count_fsdp() {
  static int n = 0;
  if (!n) {
    int dev;
    MESHY_CUDA_CHECK(cudaGetDevice(&dev));
    MESHY_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

}  // namespace

void fsdp_gather(const unsigned long long* ptrs, long long off_bytes, long long bytes, int world, void* dst,
                 cudaStream_t st) {
  MESHY_CHECK(world >= 1 && world <= kMaxPeers, "fsdp_gather: 1 <= world <= 8");
  MESHY_CHECK(off_bytes % 16 == 0 && bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
              "fsdp_gather: 16-byte aligned offsets and sizes");
  const long long n16 = bytes / 16;
  if (n16 == 0) return;
  const int per_rank = std::max(1, std::min<int>(2 * sm_count_fsdp() / world, (int)((n16 + 1023) / 1024)));
  fsdp_gather_kernel<<<dim3(per_rank, world), 256, 0, st>>>(ptrs, off_bytes, n16, reinterpret_cast<uint4*>(dst));
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void fsdp_reduce(const unsigned long long* ptrs, long long off_bytes, long long n, int rank, int world, float* dst,
                 cudaStream_t st) {
  MESHY_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "fsdp_reduce: rank / world");
  MESHY_CHECK(off_bytes % 16 == 0 && n % 4 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
              "fsdp_reduce: 16-byte aligned offsets and sizes");
  const long long n4 = n / 4;
  if (n4 == 0) return;
  const int blocks = std::max(1, std::min<int>(2 * sm_count_fsdp(), (int)((n4 + 255) / 256)));
  fsdp_reduce_kernel<<<blocks, 256, 0, st>>>(ptrs, off_bytes, n4, rank, world, reinterpret_cast<float4*>(dst));
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
