#pragma once
#include "../include/common.cuh"
namespace meshy {
void sq_norm(const float* x, long long n, float* out, cudaStream_t st);
void adamw_flat(float* p, const float* g, float* m, float* v, bf16* out, bf16* mirror, const float* norm, long long n,
                float max_norm, float lr, float b1, float b2, float eps, float wd, int step, cudaStream_t st);
void ppo_loss_fused(const float* new_lp, const float* old_lp, const float* adv, const float* mask, const float* roll,
                    const float* inv, const float* posw, const float* ent, const int64_t* doc, float* grad, float* sums,
                    float* seg, long long T, float lo, float hi, int use_tis, int use_icepop, float tmin, float tmax,
                    float pcoef, int train_old, cudaStream_t st);
void gae_scan(const float* x, const float* d, const float* valid, float* out, int rows, int S, cudaStream_t st);
void lse_merge(const float* part, int n_tiles, int bn, const int64_t* labels, float* lp, float* lse, float* ent,
               int64_t* tok, float* tok_lp, int rows, cudaStream_t st);
void decode_advance(const int64_t* tok, const float* lp, int64_t* tok_in, int* pos, int* seq_lens, int* gen,
                    const int* max_new, int* done, int64_t* slot, const int* bt, const int* req, int64_t* out_tok,
                    float* out_lp, const int64_t* eos, int n_eos, int B, int max_pages, int cap, int page,
                    cudaStream_t st);
// Merge of the small-M sampler's partials ([B][n_parts][8]) fused with decode_advance; also adds 1 to
// ``step`` (the sampler's noise key) when given.
void sample_advance(const float* part, int n_parts, int64_t* tok_in, int* pos, int* seq_lens, int* gen,
                    const int* max_new, int* done, int64_t* slot, const int* bt, const int* req, int64_t* out_tok,
                    float* out_lp, const int64_t* eos, int n_eos, int B, int max_pages, int cap, int page,
                    int64_t* step, cudaStream_t st);
// Top-k / top-p (and temperature) sampling over fp32 logits [B, V], one CTA per row (sampling.cu): token and
// its log-probability under the filtered, tempered distribution; temperature 0 is greedy.
void filtered_sample(const float* logits, int B, int V, float temperature, int top_k, float top_p, uint64_t seed,
                     const int64_t* step_ptr, int64_t* tok, float* lp, cudaStream_t st);

// Critic value head fused with the clipped value loss (value_head.cu). fwd: v = h w + b, num += sum(err *
// mask), dv = mask * d err / dv / denom; bwd: dh = dv w^T (bf16), dw += dv^T h, db += sum dv (fp32).
void value_head_fwd(const bf16* h, const float* w, const float* b, int T, int D, const float* ret, const float* mask,
                    const float* old, float clip, float inv_denom, float* v, float* dv, float* num, cudaStream_t st);
void value_head_bwd(const bf16* h, const float* w, const float* dv, int T, int D, bf16* dh, float* dw, float* db,
                    cudaStream_t st);

// Top-K distillation (topk.cu): the K largest fp32 logits of each row (sorted) with their log-probabilities
// and the row's log-sum-exp; log-probabilities of given ids from the hidden rows and the LM-head weight
// (needs lse); dz[t, ids[t, k]] += g[t, k] on bf16 logit gradients.
void topk_logprobs(const float* z, long long ldz, int T, int V, int K, int64_t* ids, float* lp, float* lse,
                   cudaStream_t st);
void gather_logprobs(const bf16* h, long long ldh, const bf16* w, long long ldw, int T, int D, int V,
                     const int64_t* ids, int K, const float* lse, float* lp, cudaStream_t st);
void scatter_add_rows(bf16* dz, long long ldz, int T, int V, const int64_t* ids, const float* g, int K,
                      cudaStream_t st);

}  // namespace meshy
