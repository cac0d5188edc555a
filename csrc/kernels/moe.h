// Mixture-of-experts routing kernels (moe.cu). All sizes that depend on the routing stay on the device.
#pragma once
#include <cuda_runtime.h>

#include "../include/common.cuh"

namespace meshy {

// Router: probs = softmax(logits) [T, E] fp32; top-k experts [T, k] int32 and weights [T, k] fp32
// (renormalised over the k picks when ``norm``). E <= 256, k <= 32.
void moe_route(const bf16* logits, int T, int E, int k, bool norm, float* probs, float* weights, int* experts,
               cudaStream_t st);
// d logits [T, E] (bf16) from d weights [T, k].
void moe_route_bwd(const float* dw, const float* probs, const float* weights, const int* experts, int T, int E, int k,
                   bool norm, bf16* dlogits, cudaStream_t st);
// Plan + gather of n = T * k assignments: cnt[E], off[E + 1] (128-aligned segment starts), slot_of[n]
// (row of each assignment), row_src[rows_cap] (assignment of each row, -1 for padding), and, when xp is
// given, xp[row] = x[assignment / k] with zero padding rows.
void moe_plan(const int* experts, int n, int k, int E, int* cnt, int* off, int* slot_of, int* row_src, const bf16* x,
              int D, bf16* xp, int rows_cap, int* err, cudaStream_t st);
// Zero the padding rows of every segment of a [rows, C] bf16 buffer.
void moe_zero_pad(const int* off, const int* cnt, int E, bf16* buf, int C, cudaStream_t st);
// out[t] = sum_j w[t, j] * y[slot_of[t * k + j]] (w == nullptr: plain sum); y has ``rows`` rows and slots
// outside them are skipped.
void moe_combine(const bf16* y, int rows, const int* slot_of, const float* w, int T, int k, int D, bf16* out,
                 cudaStream_t st);
// dy[slot_of[t * k + j]] = w[t, j] * dout[t]; dw[t, j] = <dout[t], y[slot_of[t * k + j]]>.
void moe_combine_bwd(const bf16* dout, const bf16* y, int rows, const int* slot_of, const float* w, int T, int k,
                     int D, bf16* dy, float* dw, cudaStream_t st);

}  // namespace meshy
