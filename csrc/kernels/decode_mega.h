// Whole-step persistent decode kernel ("megakernel") for dense decoders.
//
// One cooperative launch of one CTA per SM runs a complete decode step of a
// Llama/Qwen-style dense decoder for up to kMegaMaxRows running sequences:
// embedding, every layer (RMSNorm -> QKV -> RoPE/KV-cache write -> paged
// attention -> o_proj + residual -> RMSNorm -> gate/up + SwiGLU -> down +
// residual) and the final RMSNorm. The LM head / sampler runs after it.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace meshy {

using bf16 = __nv_bfloat16;

constexpr int kMegaMaxRows = 64;   // running sequences per step (MMA N <= 64)
constexpr int kMegaHeadDim = 128;  // head_dim (one 128-row weight tile = one head)
constexpr int kMegaPage = 64;      // KV page size in tokens
constexpr int kMegaMaxSplit = 32;  // split-K factor cap of a GEMM phase

// Per-layer small tensors (device pointers); the big matrices come in through 3-D tensor maps.
struct MegaLayer {
  const bf16* attn_norm;  // [D]
  const bf16* bqkv;       // [qkv_dim] or null
  const bf16* q_norm;     // [hd] or null
  const bf16* k_norm;     // [hd] or null
  const bf16* mlp_norm;   // [D]
  const bf16* pad0;
  const bf16* pad1;
  const bf16* pad2;
};

// One GEMM phase: T 128-row weight tiles, KB 64-wide k-blocks, s-way split-K (s <= KB).
struct MegaGemm {
  int T, KB, s;
};

struct MegaArgs {
  int n_layers, D, Hq, Hkv, F, qkv_dim, q_dim;
  int B, MP;          // running rows, padded rows (16 / 32 / 64)
  float eps;          // RMSNorm epsilon
  float qk_scale_log2;  // softmax scale * log2(e)
  const float* inv_freq;  // [hd / 2]
  const MegaLayer* layers;
  const bf16* embed;       // [V, D]
  const bf16* final_norm;  // [D]
  // decode state (written by the previous step's bookkeeping kernel)
  const int64_t* tok;
  const int* pos;
  const int* seq_lens;
  const int64_t* slot;
  const int* block_table;
  int max_pages;     // block_table row stride
  int n_cache_pages;  // pages per layer per K/V in the cache tensor [L, 2, n_pages, Hkv, 64, hd]
  bf16* kv;           // cache base
  // workspaces (zero-initialised once; kept consistent by the kernel)
  float* x;        // [D][MP]   residual stream, feature-major
  bf16* xg;        // [MP][D]   bf16(x * gain of the next norm), token-major (TMA X operand)
  float* sumsq;    // [2][MP]   sum of squares of x per row (0: attention norm, 1: MLP norm)
  float* acc;      // [max(qkv_dim, 2F)][MP] split-K accumulator, reset by the tile finalisers
  bf16* q;         // [MP][Hq][hd]
  float* apart;    // [grid][2][16][hd + 2] attention partials
  bf16* ao;        // [MP][q_dim] attention output (TMA X operand of o_proj)
  bf16* act;       // [MP][F]     SwiGLU output (TMA X operand of down_proj)
  bf16* h;         // [B][D]      final normed hidden (LM head input)
  unsigned* ctr;   // [kMegaCtrTiles] tile counters, [kMegaCtrAttn] attention counters, barrier, exit
  int* err;
  MegaGemm g_qkv, g_o, g_gu, g_dn;
  // optional timeline: [phase][cta][8] global-timer ns: start and end of each phase's work, and markers
  // (GEMM: all stages landed, accumulator ready; attention: first / last page landed, last page
  // computed, piece merged, piece counter returned, pieces combined)
  unsigned long long* trace;
  int flags;  // bit 0: always take the split-K path for gate/up (no direct SwiGLU epilogue)
};

constexpr int kMegaCtrTiles = 1024;
constexpr int kMegaCtrAttn = 1024;
constexpr int kMegaCtrWords = kMegaCtrTiles + kMegaCtrAttn + 64;

// Launch one decode step. Tensor maps: the four weight matrices as 3-D maps over (k, row, layer),
// the three X operands as 2-D maps over [MP][K], the KV cache as one 2-D map over its 128-wide rows.
void mega_decode_launch(const MegaArgs& a, const CUtensorMap& m_qkv, const CUtensorMap& m_o,
                        const CUtensorMap& m_gu, const CUtensorMap& m_dn, const CUtensorMap& m_xg,
                        const CUtensorMap& m_ao, const CUtensorMap& m_act, const CUtensorMap& m_kv, int grid,
                        cudaStream_t st);
int mega_grid();                  // CTAs of one launch (one per SM)
size_t mega_apart_floats(int grid);  // size of the attention-partials workspace

}  // namespace meshy
