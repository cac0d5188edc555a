// Symmetric peer memory (CUDA IPC over NVLink) and the fused data-parallel optimiser step (symm.cu).
#pragma once
#include <cuda_runtime.h>

#include <string>

#include "../include/common.cuh"

namespace meshy {

void* symm_malloc(size_t bytes);
void symm_free(void* p);
std::string symm_export(void* p);          // cudaIpcMemHandle bytes
void* symm_import(const std::string& h);   // peer pointer in this process
void symm_close(void* p);

// One-CTA barrier over the ranks' flag arrays (bounded spin; err := kErrTimeoutPeer on timeout).
void symm_barrier(const unsigned long long* flag_ptrs, int rank, int world, unsigned int epoch, double timeout_s,
                  int* err, cudaStream_t st);

struct SymmAdamWArgs {
  const unsigned long long* grad_ptrs = nullptr;     // [world] device table
  const unsigned long long* master_ptrs = nullptr;   // [world], or null: master sharded (needs compute_ptrs)
  const unsigned long long* compute_ptrs = nullptr;  // [world] or null (no bf16 copy)
  const unsigned long long* flag_ptrs = nullptr;     // [world] u32[world] flag arrays
  const unsigned long long* slot_ptrs = nullptr;     // [world] f32[world] norm slots
  float* master_local = nullptr;
  float* local_grad = nullptr;
  float* exp_avg = nullptr;     // AdamW moments of this rank's shard only: [hi - lo]
  float* exp_avg_sq = nullptr;  // (ZeRO-1: every rank keeps 1/world of the optimiser state)
  float* sumsq = nullptr;  // device scratch scalar
  float* norm = nullptr;   // device scalar: global gradient norm (output)
  int* err = nullptr;
  int rank = 0, world = 1;
  long long lo = 0, hi = 0;  // this rank's shard
  unsigned int epoch = 0;    // uses epoch, epoch + 1, epoch + 2
  float max_norm = 1.f, lr = 0.f, b1 = 0.9f, b2 = 0.999f, eps = 1e-8f, wd = 0.f;
  int step = 1;
  double timeout_s = 10.0;
};

void symm_dp_adamw_step(const SymmAdamWArgs& a, cudaStream_t st);

// Sharded-parameter collectives over peer memory (fsdp.cu); ``ptrs`` is the [world] device table of the
// ranks' heap addresses of one symmetric region, ``off_bytes`` an offset inside it.
constexpr int kMaxPeers = 8;
// dst[r * bytes .. (r + 1) * bytes) = rank r's bytes at off_bytes, for every rank r.
void fsdp_gather(const unsigned long long* ptrs, long long off_bytes, long long bytes, int world, void* dst,
                 cudaStream_t st);
// dst[j] += sum_r (rank r's fp32 region at off_bytes)[rank * n + j], j < n.
void fsdp_reduce(const unsigned long long* ptrs, long long off_bytes, long long n, int rank, int world, float* dst,
                 cudaStream_t st);

}  // namespace meshy
