// Host interface of the tcgen05 GEMM (gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../include/common.cuh"

namespace meshy {

enum Epilogue : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_ACC_F32 = 2, EPI_LSE = 3, EPI_DLOGITS = 4 };
// Grouped (mixture-of-experts) GEMMs over token rows sorted by group, each group's segment padded to a
// multiple of 128 rows (device offsets grp_off[0..grp_n]):
//   GRP_M  out[seg_g] = A[seg_g] . op(B_g)^T   (forward and data gradient; B = [grp_n] matrices at a
//          stride of grp_stride elements; M = rows allocated, units past grp_off[grp_n] do nothing)
//   GRP_K  out[g] += A[seg_g]^T . B[seg_g]      (weight gradient; A and B MN-major with the token rows as
//          K; out = [grp_n * grp_rows, N] fp32, M = grp_rows per group)
enum GroupMode : int { GRP_NONE = 0, GRP_M = 1, GRP_K = 2 };

struct GemmProblem {
  const void* A = nullptr;  // bf16
  const void* B = nullptr;  // bf16
  int64_t lda = 0, ldb = 0;
  bool a_mn = false, b_mn = false;
  int M = 0, N = 0, K = 0;
  int epi = EPI_STORE;
  void* out = nullptr;
  int ldo = 0;
  int out_f32 = 0;
  const bf16* bias = nullptr;
  const bf16* residual = nullptr;
  int ldr = 0;
  bf16* aux = nullptr;
  int ld_aux = 0;
  float* ws = nullptr;        // split-K fp32 workspace [M, N], kept zero between calls
  int64_t ws_cap = 0;
  int* counters = nullptr;    // split-K per-tile arrival counters, kept zero
  int64_t counters_cap = 0;
  const int64_t* labels = nullptr;
  float* partial = nullptr;   // LSE partials [M, n_tiles, 8]
  const float* row_lse = nullptr;
  const float* row_g = nullptr;
  float inv_temp = 1.f;
  uint64_t seed = 0;
  const int64_t* step_ptr = nullptr;
  int gumbel = 0;
  int* err = nullptr;         // device error word
  int force_bn = 0;           // 0 = heuristic
  int max_split = 0;          // 0 = heuristic
  int force_cs = 0;           // small-M path: cluster split-K size (0 = heuristic)
  const bf16* norm_w = nullptr;  // small-M path: fused input RMSNorm gain (A is the raw stream)
  float norm_eps = 1e-6f;
  // small-M path, RMSNorm split across two GEMMs (decode). A residual GEMM (out = A W^T + residual)
  // also writes xg_out = bf16(bf16(out) * g_next) and, per 128-row output tile t and row m, the sum of
  // squares of the rounded outputs into part_out[t * kSmallPartLd + m]. The next GEMM takes xg as its
  // A operand and scales output row m by rsqrt(sum_t part_in[t * kSmallPartLd + m] / norm_d + norm_eps):
  //   W (g * x) * rstd == W RMSNorm(x).
  bf16* xg_out = nullptr;
  const bf16* g_next = nullptr;
  float* part_out = nullptr;
  const float* part_in = nullptr;
  int part_t = 0;
  float norm_d = 0.f;
  // small-M path, fused QKV epilogue (decode): every 128-row tile is one head of head_dim 128 in the
  // fused [Hq | Hkv | Hkv] layout. Output rows are rounded to bf16 (+bias), q/k heads get the optional
  // per-head RMSNorm (qn / kn) and rotate-half RoPE at rope_pos, q heads go to q_out [M, Hq, 128],
  // k / v heads straight into the paged caches kc / vc ([pages, Hkv, 64, 128]) at slots[m].
  bf16* q_out = nullptr;
  const int* rope_pos = nullptr;
  const float* inv_freq = nullptr;
  const bf16* qn = nullptr;
  const bf16* kn = nullptr;
  bf16* kc = nullptr;
  bf16* vc = nullptr;
  const int64_t* slots = nullptr;
  int hq = 0, hkv = 0;
  // grouped problems (see GroupMode)
  int grp_mode = GRP_NONE;
  const int* grp_off = nullptr;
  int grp_n = 0;
  int64_t grp_stride = 0;   // GRP_M: elements between consecutive groups' B matrices
};
constexpr int kSmallPartLd = 256;

void gemm_launch(const GemmProblem& g, cudaStream_t stream);

// Small-M (decode) path, gemm_small.cu: TN problems with M <= kSmallMaxM and a
// STORE or SwiGLU epilogue run with swapped operands and cluster split-K.
constexpr int kSmallMaxM = 256;
constexpr int kSmallMaxCluster = 16;  // above 8 the kernel opts in to non-portable cluster sizes
bool gemm_small_eligible(const GemmProblem& g);
// Whether the small-M path can also fuse the input RMSNorm for this problem.
bool gemm_small_norm_eligible(const GemmProblem& g);
// Whether the small-M path can prepare the next RMSNorm (xg_out / part_out) for this residual GEMM.
bool gemm_small_prep_eligible(const GemmProblem& g);
// Whether the small-M path can run the fused QKV + RoPE + KV-cache epilogue (q_out ...).
bool gemm_small_rope_eligible(const GemmProblem& g);
// Fused LM-head sampler on the small-M path: EPI_LSE with Gumbel noise (no labels), M <= 64, any
// vocabulary size; writes gemm_small_lse_parts(N) partials per token row ([M][parts][8], the layout
// lse_merge reads). With part_in the rows of A are prepared RMSNorm inputs (see above).
bool gemm_small_lse_eligible(const GemmProblem& g);
int gemm_small_lse_parts(int N);
void gemm_small_launch(const GemmProblem& g, cudaStream_t stream);
// enabled: 1/0 (-1 keeps); force_cs: cluster size override, 0 = heuristic (-1 keeps)
void gemm_small_config(int enabled, int force_cs);
// Diagnostics: while ``buf`` is set, the next ``slots`` small-M launches record their timelines into
// buf[slot][160][8] (global-timer ns per CTA, see SmallArgs::trace); null stops recording.
void gemm_small_trace(unsigned long long* buf, int slots);
CUtensorMap make_map_bf16(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int bi, int bo);
CUtensorMap make_map_bf16_3d(const void* ptr, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes,
                             int64_t stride2_bytes, int b0, int b1);
int gemm_n_tiles(int N, int bn);

}  // namespace meshy
