#pragma once
#include "../include/common.cuh"
namespace meshy {
void rmsnorm_fwd(const bf16* x, const bf16* w, bf16* y, float* rstd, int rows, int D, float eps, cudaStream_t st);
void rmsnorm_bwd(const bf16* gy, const bf16* x, const bf16* w, const float* rstd, bf16* gx, float* gw, int rows, int D,
                 cudaStream_t st);
// k / v may be null when kc / vc (paged caches [n_pages, Hkv, page, hd]) receive them at ``slots``.
void qkv_rope_fwd(const bf16* qkv, const int* pos, const bf16* qn, const bf16* kn, const float* inv_freq, bf16* q,
                  bf16* k, bf16* v, int T, int Hq, int Hkv, int hd, float eps, cudaStream_t st, bf16* kc = nullptr,
                  bf16* vc = nullptr, const int64_t* slots = nullptr, int page = 0);
void qkv_rope_bwd(const bf16* qkv, const int* pos, const bf16* qn, const bf16* kn, const float* inv_freq,
                  const bf16* gq, const bf16* gk, const bf16* gv, bf16* gqkv, float* gqn, float* gkn, int T, int Hq,
                  int Hkv, int hd, float eps, cudaStream_t st);
void swiglu_bwd(const bf16* h, const bf16* ga, bf16* dh, long long T, int F, int blk, cudaStream_t st);
void embedding_fwd(const int64_t* ids, const bf16* w, bf16* out, long long T, int D, long long V, cudaStream_t st);
void embedding_bwd(const int64_t* ids, const bf16* g, float* gw, long long T, int D, long long V, cudaStream_t st);
void cast_f32_bf16(const float* src, bf16* dst, long long n, cudaStream_t st);
}  // namespace meshy
