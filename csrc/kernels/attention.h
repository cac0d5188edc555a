#pragma once
#include "../include/common.cuh"
namespace meshy {
// Causal GQA flash attention over packed documents.  Document d's queries are rows [cu[d], cu[d+1])
// of q; its keys are rows [cu_k[d], cu_k[d+1]) of k/v (cu_k null: the same rows) and its first query
// sits at key position q_off[d] (null: 0), so query i attends keys [0, q_off[d] + i].  The second
// form is what context parallelism uses: local query chunks against the gathered sequence.
void flash_attn_fwd(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, bf16* o, float* lse, int T,
                    int max_seqlen, int Hq, int Hkv, int hd, float scale, cudaStream_t st,
                    const int* cu_k = nullptr, const int* q_off = nullptr, int Tk = -1, int* err = nullptr);
// head_dim 128 on the tcgen05 tensor cores (attention_tc.cu); Tk = rows of k / v. flash_attn_fwd
// dispatches here unless MESHY_FA_TC=0.
void flash_attn_fwd_tc(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, bf16* o, float* lse,
                       int T, int Tk, int max_seqlen, int Hq, int Hkv, float scale, cudaStream_t st, const int* cu_k,
                       const int* q_off, int* err);
// Context-parallel forward without an all-gather (tcgen05, head_dim 128): query chunks ``q`` of this rank
// (documents ``cu``, ``docs_per_row`` of them per sequence row, causal offsets ``q_off``) against the
// whole rows, whose K / V are read in place from every CP rank's local buffer (``k_ranks[r]`` /
// ``v_ranks[r]``: rank r's [rows * 2 chunk, Hkv * 128] head and tail chunks, mapped into this process).
// The buffers must stay unchanged until the kernel has finished on every rank.
constexpr int kFaMaxCp = 8;
void flash_attn_fwd_tc_cp(const bf16* q, const bf16* const* k_ranks, const bf16* const* v_ranks, int cp, int rows,
                          int chunk, const int* cu, int n_docs, int docs_per_row, const int* q_off, bf16* o, float* lse,
                          int T, int max_seqlen, int Hq, int Hkv, float scale, cudaStream_t st, int* err);
bool flash_attn_tc_enabled();
// dk / dv are written for every key row of every key document (zero where no query attends).
void flash_attn_bwd(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, const bf16* o,
                    const bf16* dout, const float* lse, float* dvec, bf16* dq, bf16* dk, bf16* dv, int T,
                    int max_seqlen, int Hq, int Hkv, int hd, float scale, cudaStream_t st,
                    const int* cu_k = nullptr, const int* q_off = nullptr, int max_seqlen_k = 0, int Tk = -1,
                    int* err = nullptr);
// head_dim 128 on tcgen05 (attention_tc.cu): dK/dV and dQ kernels after the D = rowsum(dO * O) prep.
void flash_attn_bwd_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* dout, const float* lse,
                       const float* dvec, const int* cu, int n_docs, bf16* dq, bf16* dk, bf16* dv, int T, int Tk,
                       int max_seqlen, int max_seqlen_k, int Hq, int Hkv, float scale, cudaStream_t st,
                       const int* cu_k, const int* q_off, int* err);
int paged_decode_splits(int B, int Hkv, int max_pages);
void paged_decode(const bf16* q, const bf16* kc, const bf16* vc, const int* bt, const int* seq_lens, bf16* o,
                  float* part, int B, int Hq, int Hkv, int hd, int page, int max_pages, int n_split, float scale,
                  cudaStream_t st);
// TMA-pipelined split-KV decode (decode_attn.cu). Up to kMaxClusterSplits splits reduce
// through distributed shared memory (above 8 a non-portable cluster size); more splits need
// ``part`` [B, Hq, n_split, hd + 2] fp32.
constexpr int kMaxClusterSplits = 16;
int paged_decode_tma_splits(int B, int Hkv, int max_pages);
int paged_decode_max_cluster();  // kMaxClusterSplits, or 8 where the device cannot place 16-CTA clusters
void paged_decode_force_splits(int n);  // tests: 0 restores the heuristic
// Timeline capture of the TMA decode-attention launches: launch i writes slot i of buf [slots][1024][8]
// (global-timer ns per CTA, see decode_attn.cu); null stops it.
void paged_decode_trace(unsigned long long* buf, int slots);
// ``decode_step``: the kernel before this one in the stream wrote, of this cache, at most the row of each
// sequence's last position (seq_lens[b] - 1) and nothing of bt / seq_lens. Pages before a sequence's last
// one are then loaded before the programmatic-dependent-launch wait, under that kernel's tail.
// ``ctr``: with more splits than one cluster holds, [kDecodeCtrs] zeroed counters let the last split of each
// (sequence, KV head) merge the partials in the same kernel (and leave the counter zero again); null runs
// paged_decode_combine after the kernel instead.
constexpr int kDecodeCtrs = 1 << 16;
void paged_decode_tma(const bf16* q, const bf16* kc, const bf16* vc, int n_cache_pages, const int* bt,
                      const int* seq_lens, bf16* o, float* part, int B, int Hq, int Hkv, int hd, int page,
                      int max_pages, int n_split, float scale, int* err, cudaStream_t st, bool decode_step = false,
                      unsigned* ctr = nullptr);
void paged_decode_combine(const float* part, bf16* o, int B, int Hq, int hd, int n_split, cudaStream_t st);
void kv_write(const bf16* k, const bf16* v, bf16* kc, bf16* vc, const int64_t* slots, int n, int Hkv, int hd, int page,
              cudaStream_t st);
}  // namespace meshy
