// Small fused kernels of the training step and the decode loop:
//   sq_norm          sum of squares of the flat fp32 gradient (grad-norm clip)
//   adamw_flat       AdamW on flat fp32 buffers + clip + bf16 recast (+ mirror)
//   ppo_loss_fused   PPO/GRPO per-token loss, its analytic d/d(new_lp), and all
//                    diagnostic sums in one pass
//   gae_scan         segmented reverse linear recurrence (GAE / returns)
//   lse_merge        merge of the LM-head kernel's per-tile partials
//   decode_advance   per-row bookkeeping after a decode step
#include "../include/common.cuh"
#include "misc.h"

namespace meshy {

template <int NTHREADS>
__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < NTHREADS / 32) ? sh[threadIdx.x] : 0.f;
  if (w == 0) v = warp_sum(v);
  __syncthreads();
  return v;
}

__global__ void sq_norm_kernel(const float* __restrict__ x, long long n, float* __restrict__ out) {
  __shared__ float sh[32];
  float acc = 0.f;
  long long n4 = n / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(x)[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long long i = n4 * 4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    acc += x[i] * x[i];
  acc = block_sum<256>(acc, sh);
  if (threadIdx.x == 0) atomicAdd(out, acc);
}

void sq_norm(const float* x, long long n, float* out, cudaStream_t st) {
  sq_norm_kernel<<<148 * 4, 256, 0, st>>>(x, n, out);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ out, bf16* __restrict__ mirror,
                             const float* __restrict__ norm, long long n, float max_norm, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2) {
  float coef = 1.f;
  if (max_norm > 0.f) {
    float nrm = *norm;
    coef = fminf(1.f, max_norm / (nrm + 1e-6f));
  }
  const float step = lr / bc1, inv_bc2 = 1.f / bc2, decay = 1.f - lr * wd;
  long long i4 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (long long i = i4 * 4; i < n; i += (long long)gridDim.x * blockDim.x * 4) {
    if (i + 4 <= n) {
      float4 pp = *reinterpret_cast<float4*>(p + i), gg = *reinterpret_cast<const float4*>(g + i);
      float4 mm = *reinterpret_cast<float4*>(m + i), vv = *reinterpret_cast<float4*>(v + i);
      float* P = &pp.x; float* G = &gg.x; float* Mv = &mm.x; float* Vv = &vv.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float gk = G[k] * coef;
        Mv[k] = b1 * Mv[k] + (1.f - b1) * gk;
        Vv[k] = b2 * Vv[k] + (1.f - b2) * gk * gk;
        P[k] = P[k] * decay - step * Mv[k] / (sqrtf(Vv[k] * inv_bc2) + eps);
      }
      *reinterpret_cast<float4*>(p + i) = pp;
      *reinterpret_cast<float4*>(m + i) = mm;
      *reinterpret_cast<float4*>(v + i) = vv;
      uint2 packed = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
      if (out) *reinterpret_cast<uint2*>(out + i) = packed;
      if (mirror) *reinterpret_cast<uint2*>(mirror + i) = packed;
    } else {
      for (long long k = i; k < n; ++k) {
        float gk = g[k] * coef;
        m[k] = b1 * m[k] + (1.f - b1) * gk;
        v[k] = b2 * v[k] + (1.f - b2) * gk * gk;
        p[k] = p[k] * decay - step * m[k] / (sqrtf(v[k] * inv_bc2) + eps);
        if (out) out[k] = __float2bfloat16(p[k]);
        if (mirror) mirror[k] = __float2bfloat16(p[k]);
      }
    }
  }
}

void adamw_flat(float* p, const float* g, float* m, float* v, bf16* out, bf16* mirror, const float* norm, long long n,
                float max_norm, float lr, float b1, float b2, float eps, float wd, int step, cudaStream_t st) {
  float bc1 = 1.f - powf(b1, (float)step), bc2 = 1.f - powf(b2, (float)step);
  long long threads = (n + 3) / 4;
  int grid = (int)std::min<long long>((threads + 255) / 256, 148 * 16);
  adamw_kernel<<<grid, 256, 0, st>>>(p, g, m, v, out, mirror, norm, n, max_norm, lr, b1, b2, eps, wd, bc1, bc2);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── PPO loss ──────────────────────────────────────────────────────────────
// sums layout (15): loss, total_loss, positive_lm_loss, tis_ratio_sum, ratio_sum,
// clip_sum, tis_masked_sum, token_count, ppo_kl_sum, log_ratio_abs_sum,
// ess_sum(0), doc_count(0), train_rollout_kl_sum, train_rollout_logdiff_abs_sum,
// entropy_sum.   seg [n_slots, 3]: sum r*mask, sum r^2*mask, (unused).
constexpr int kSums = 15;

__global__ void ppo_loss_kernel(const float* __restrict__ new_lp, const float* __restrict__ old_lp,
                                const float* __restrict__ adv, const float* __restrict__ mask,
                                const float* __restrict__ roll, const float* __restrict__ inv,
                                const float* __restrict__ posw, const float* __restrict__ ent,
                                const int64_t* __restrict__ doc, float* __restrict__ grad, float* __restrict__ sums,
                                float* __restrict__ seg, long long T, float lo, float hi, int use_tis, int use_icepop,
                                float tmin, float tmax, float pcoef, int train_old) {
  __shared__ float sh[32];
  float acc[kSums];
#pragma unroll
  for (int i = 0; i < kSums; ++i) acc[i] = 0.f;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < T; t += (long long)gridDim.x * blockDim.x) {
    const float mk = mask[t];
    const float nl = new_lp[t], ol = old_lp[t];
    const float lr = nl - ol;
    const float r = __expf(lr);
    const float a = adv[t];
    const float rc = fminf(fmaxf(r, 1.f - lo), 1.f + hi);
    const float un = r * a, cl = rc * a;
    const bool inr = (r >= 1.f - lo) && (r <= 1.f + hi);
    float pg = -fminf(un, cl);
    float d_un = r * a, d_cl = inr ? r * a : 0.f;
    float dpg = -(un < cl ? d_un : (cl < un ? d_cl : 0.5f * (d_un + d_cl)));
    float tis_r = r;
    bool tis_keep = true;
    if (use_icepop) {
      tis_r = __expf(ol - roll[t]);
      tis_keep = (tis_r >= tmin) && (tis_r <= tmax);
      float w = tis_keep ? tis_r : 0.f;
      pg = tis_keep ? pg * w : 0.f;
      dpg = tis_keep ? dpg * w : 0.f;
    } else if (use_tis) {
      tis_keep = (r >= tmin) && (r <= tmax);
      pg = tis_keep ? pg : 0.f;
      dpg = tis_keep ? dpg : 0.f;
    }
    const float w_inv = inv[t];
    float pos_term = 0.f, dpos = 0.f;
    if (posw) {
      pos_term = -nl * posw[t] * mk;
      dpos = -posw[t] * mk;
    }
    const float pg_loss = pg * mk * w_inv;
    const float pos_loss = pos_term * w_inv;
    grad[t] = (dpg * mk + pcoef * dpos) * w_inv;
    acc[0] += pg_loss;
    acc[1] += pg_loss + pcoef * pos_loss;
    acc[2] += pos_loss;
    acc[3] += tis_r * mk;
    acc[4] += r * mk;
    acc[5] += ((r < 1.f - lo) || (r > 1.f + hi)) ? mk : 0.f;
    acc[6] += tis_keep ? 0.f : mk;
    acc[7] += mk;
    acc[8] += -lr * mk;
    acc[9] += fabsf(lr) * mk;
    if (roll) {
      float tl = train_old ? ol : nl;
      float dd = fminf(fmaxf(roll[t] - tl, -10.f), 10.f);
      float k3 = __expf(dd) - dd - 1.f;
      if (!isfinite(k3)) k3 = 0.f;
      float ad = fabsf(roll[t] - tl);
      if (!isfinite(ad)) ad = 0.f;
      acc[12] += k3 * mk;
      acc[13] += ad * mk;
    }
    if (ent) acc[14] += ent[t] * mk;
    if (mk != 0.f) {
      long long d = doc[t];
      atomicAdd(&seg[d * 3 + 0], r * mk);
      atomicAdd(&seg[d * 3 + 1], r * r * mk);
    }
  }
#pragma unroll
  for (int i = 0; i < kSums; ++i) {
    float v = block_sum<256>(acc[i], sh);
    if (threadIdx.x == 0 && v != 0.f) atomicAdd(&sums[i], v);
  }
}

void ppo_loss_fused(const float* new_lp, const float* old_lp, const float* adv, const float* mask, const float* roll,
                    const float* inv, const float* posw, const float* ent, const int64_t* doc, float* grad, float* sums,
                    float* seg, long long T, float lo, float hi, int use_tis, int use_icepop, float tmin, float tmax,
                    float pcoef, int train_old, cudaStream_t st) {
  if (T == 0) return;
  int grid = (int)std::min<long long>((T + 255) / 256, 148 * 2);
  ppo_loss_kernel<<<grid, 256, 0, st>>>(new_lp, old_lp, adv, mask, roll, inv, posw, ent, doc, grad, sums, seg, T, lo,
                                        hi, use_tis, use_icepop, tmin, tmax, pcoef, train_old);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── GAE scan ──────────────────────────────────────────────────────────────
// A_t = x_t + d_t A_{t+1} per row (d already carries gamma*lambda*cont); zero
// where !valid.  One block per row: each thread reduces its chunk to an affine
// map A_start = X + D A_end, a right-to-left exclusive scan of the maps gives
// every chunk its incoming A_end, then each chunk is replayed.
__global__ void gae_scan_kernel(const float* __restrict__ x, const float* __restrict__ d,
                                const float* __restrict__ valid, float* __restrict__ out, int S) {
  __shared__ float Xs[1024], Ds[1024], In[1024];
  const int row = blockIdx.x;
  const int n = blockDim.x;
  const int chunk = (S + n - 1) / n;
  const int s0 = threadIdx.x * chunk, s1 = min(S, s0 + chunk);
  const float* xr = x + (size_t)row * S;
  const float* dr = d + (size_t)row * S;
  const float* vr = valid + (size_t)row * S;
  float X = 0.f, D = 1.f;
  for (int t = s1 - 1; t >= s0; --t) {
    float xv = vr[t] > 0.f ? xr[t] : 0.f;
    X = xv + dr[t] * X;
    D = dr[t] * D;
  }
  Xs[threadIdx.x] = X;
  Ds[threadIdx.x] = D;
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.f;  // A at the end of the row
    for (int c = n - 1; c >= 0; --c) {
      In[c] = acc;
      acc = Xs[c] + Ds[c] * acc;
    }
  }
  __syncthreads();
  float A = In[threadIdx.x];
  float* orow = out + (size_t)row * S;
  for (int t = s1 - 1; t >= s0; --t) {
    float xv = vr[t] > 0.f ? xr[t] : 0.f;
    A = xv + dr[t] * A;
    orow[t] = vr[t] > 0.f ? A : 0.f;
  }
}

void gae_scan(const float* x, const float* d, const float* valid, float* out, int rows, int S, cudaStream_t st) {
  if (rows == 0 || S == 0) return;
  int threads = std::min(1024, std::max(32, ((S + 31) / 32) * 32));
  gae_scan_kernel<<<rows, threads, 0, st>>>(x, d, valid, out, S);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── LM-head partial merge ─────────────────────────────────────────────────
// One warp merges the n_tiles partials (max, sum, sum p*z, target z, best, z of best, index) of a row:
// log-sum-exp l, sum p*z / sum p (for the entropy) and the Gumbel-max winner over all tiles.
struct RowMerge {
  float l, pz_s, bestz;
  int besti;
};

__device__ __forceinline__ RowMerge merge_row(const float* __restrict__ pr, int n_tiles, int lane) {
  float M = -INFINITY;
  for (int t = lane; t < n_tiles; t += 32) M = fmaxf(M, pr[t * 8]);
  M = warp_max(M);
  float S = 0.f, PZ = 0.f, best = -INFINITY, bestz = 0.f;
  int besti = 0x7fffffff;
  for (int t = lane; t < n_tiles; t += 32) {
    const float* q = pr + t * 8;
    float f = (q[0] == -INFINITY) ? 0.f : __expf(q[0] - M);
    S += q[1] * f;
    PZ += q[2] * f;
    int bi = __float_as_int(q[6]);
    if (bi >= 0 && (q[4] > best || (q[4] == best && bi < besti))) {
      best = q[4];
      besti = bi;
      bestz = q[5];
    }
  }
  S = warp_sum(S);
  PZ = warp_sum(PZ);
  for (int o = 16; o > 0; o >>= 1) {
    float ob = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    float oz = __shfl_xor_sync(0xffffffffu, bestz, o);
    if (ob > best || (ob == best && oi < besti)) {
      best = ob;
      besti = oi;
      bestz = oz;
    }
  }
  return RowMerge{M + logf(S), PZ / S, bestz, besti};
}

__global__ void lse_merge_kernel(const float* __restrict__ part, int n_tiles, int bn, const int64_t* __restrict__ labels,
                                 float* __restrict__ lp, float* __restrict__ lse, float* __restrict__ ent,
                                 int64_t* __restrict__ tok, float* __restrict__ tok_lp, int rows) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  pdl_wait();
  pdl_trigger();
  if (row >= rows) return;
  const float* pr = part + (size_t)row * n_tiles * 8;
  const RowMerge r = merge_row(pr, n_tiles, lane);
  if (lane == 0) {
    const float l = r.l;
    if (lse) lse[row] = l;
    if (ent) ent[row] = l - r.pz_s;
    if (lp && labels) {
      int64_t y = labels[row];
      int t = (int)(y / bn);
      float tgt = (y >= 0 && t < n_tiles) ? pr[t * 8 + 3] : -INFINITY;
      lp[row] = tgt - l;
    }
    if (tok) {
      tok[row] = r.besti;
      tok_lp[row] = r.bestz - l;
    }
  }
}

void lse_merge(const float* part, int n_tiles, int bn, const int64_t* labels, float* lp, float* lse, float* ent,
               int64_t* tok, float* tok_lp, int rows, cudaStream_t st) {
  if (rows == 0) return;
  launch_pdl(lse_merge_kernel, dim3((rows + 7) / 8), dim3(256), 0, st, part, n_tiles, bn, labels, lp, lse, ent, tok,
             tok_lp, rows);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── decode row advance ────────────────────────────────────────────────────
__global__ void decode_advance_kernel(const int64_t* __restrict__ tok, const float* __restrict__ lp,
                                      int64_t* __restrict__ tok_in, int* __restrict__ pos, int* __restrict__ seq_lens,
                                      int* __restrict__ gen, const int* __restrict__ max_new, int* __restrict__ done,
                                      int64_t* __restrict__ slot, const int* __restrict__ bt, const int* __restrict__ req,
                                      int64_t* __restrict__ out_tok, float* __restrict__ out_lp,
                                      const int64_t* __restrict__ eos, int n_eos, int B, int max_pages, int cap,
                                      int page) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  if (i >= B || done[i]) return;
  int r = req[i], g = gen[i];
  int64_t t = tok[i];
  if (g < cap) {
    out_tok[(size_t)r * cap + g] = t;
    out_lp[(size_t)r * cap + g] = lp[i];
  }
  g += 1;
  gen[i] = g;
  tok_in[i] = t;
  bool fin = g >= max_new[i];
  for (int e = 0; e < n_eos; ++e) fin |= (t == eos[e]);
  done[i] = fin ? 1 : 0;
  int p = pos[i] + 1;
  pos[i] = p;
  seq_lens[i] = seq_lens[i] + 1;
  int pi = p / page;
  slot[i] = (pi < max_pages) ? (int64_t)bt[(size_t)i * max_pages + pi] * page + p % page : 0;
}

void decode_advance(const int64_t* tok, const float* lp, int64_t* tok_in, int* pos, int* seq_lens, int* gen,
                    const int* max_new, int* done, int64_t* slot, const int* bt, const int* req, int64_t* out_tok,
                    float* out_lp, const int64_t* eos, int n_eos, int B, int max_pages, int cap, int page,
                    cudaStream_t st) {
  if (B == 0) return;
  launch_pdl(decode_advance_kernel, dim3((B + 127) / 128), dim3(128), 0, st, tok, lp, tok_in, pos, seq_lens, gen,
             max_new, done, slot, bt, req, out_tok, out_lp, eos, n_eos, B, max_pages, cap, page);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

// ─── sampler merge + decode row advance (one kernel) ───────────────────────
// One warp per running row: merges the LM-head sampler partials into the sampled token and its
// log-probability, then advances the row exactly as decode_advance_kernel does. Thread 0 of block 0
// bumps the step counter that keys the sampler's noise (the sampler kernel has completed: pdl_wait).
__global__ void sample_advance_kernel(const float* __restrict__ part, int n_parts, int64_t* __restrict__ tok_in,
                                      int* __restrict__ pos, int* __restrict__ seq_lens, int* __restrict__ gen,
                                      const int* __restrict__ max_new, int* __restrict__ done,
                                      int64_t* __restrict__ slot, const int* __restrict__ bt,
                                      const int* __restrict__ req, int64_t* __restrict__ out_tok,
                                      float* __restrict__ out_lp, const int64_t* __restrict__ eos, int n_eos, int B,
                                      int max_pages, int cap, int page, int64_t* __restrict__ step) {
  const int i = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  pdl_wait();
  pdl_trigger();
  if (step && blockIdx.x == 0 && threadIdx.x == 0) *step += 1;
  if (i >= B || done[i]) return;
  const RowMerge r = merge_row(part + (size_t)i * n_parts * 8, n_parts, lane);
  if (lane != 0) return;
  const int q = req[i];
  int g = gen[i];
  const int64_t t = r.besti;
  if (g < cap) {
    out_tok[(size_t)q * cap + g] = t;
    out_lp[(size_t)q * cap + g] = r.bestz - r.l;
  }
  g += 1;
  gen[i] = g;
  tok_in[i] = t;
  bool fin = g >= max_new[i];
  for (int e = 0; e < n_eos; ++e) fin |= (t == eos[e]);
  done[i] = fin ? 1 : 0;
  const int p = pos[i] + 1;
  pos[i] = p;
  seq_lens[i] = seq_lens[i] + 1;
  const int pi = p / page;
  slot[i] = (pi < max_pages) ? (int64_t)bt[(size_t)i * max_pages + pi] * page + p % page : 0;
}

void sample_advance(const float* part, int n_parts, int64_t* tok_in, int* pos, int* seq_lens, int* gen,
                    const int* max_new, int* done, int64_t* slot, const int* bt, const int* req, int64_t* out_tok,
                    float* out_lp, const int64_t* eos, int n_eos, int B, int max_pages, int cap, int page,
                    int64_t* step, cudaStream_t st) {
  if (B == 0) return;
  launch_pdl(sample_advance_kernel, dim3((B + 7) / 8), dim3(256), 0, st, part, n_parts, tok_in, pos, seq_lens, gen,
             max_new, done, slot, bt, req, out_tok, out_lp, eos, n_eos, B, max_pages, cap, page, step);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
