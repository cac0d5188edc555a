#pragma once
#include "../include/common.cuh"
namespace meshy {
void flash_attn_fwd(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, bf16* o, float* lse, int T,
                    int max_seqlen, int Hq, int Hkv, int hd, float scale, cudaStream_t st);
void flash_attn_bwd(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, const bf16* o,
                    const bf16* dout, const float* lse, float* dvec, bf16* dq, bf16* dk, bf16* dv, int T,
                    int max_seqlen, int Hq, int Hkv, int hd, float scale, cudaStream_t st);
int paged_decode_splits(int B, int Hkv, int max_pages);
void paged_decode(const bf16* q, const bf16* kc, const bf16* vc, const int* bt, const int* seq_lens, bf16* o,
                  float* part, int B, int Hq, int Hkv, int hd, int page, int max_pages, int n_split, float scale,
                  cudaStream_t st);
// TMA-pipelined split-KV decode (decode_attn.cu). Up to kMaxClusterSplits splits reduce
// through distributed shared memory; more splits need ``part`` [B, Hq, n_split, hd + 2] fp32.
constexpr int kMaxClusterSplits = 8;
int paged_decode_tma_splits(int B, int Hkv, int max_pages);
void paged_decode_force_splits(int n);  // tests: 0 restores the heuristic
void paged_decode_tma(const bf16* q, const bf16* kc, const bf16* vc, int n_cache_pages, const int* bt,
                      const int* seq_lens, bf16* o, float* part, int B, int Hq, int Hkv, int hd, int page,
                      int max_pages, int n_split, float scale, int* err, cudaStream_t st);
void paged_decode_combine(const float* part, bf16* o, int B, int Hq, int hd, int n_split, cudaStream_t st);
void kv_write(const bf16* k, const bf16* v, bf16* kc, bf16* vc, const int64_t* slots, int n, int Hkv, int hd, int page,
              cudaStream_t st);
}  // namespace meshy
