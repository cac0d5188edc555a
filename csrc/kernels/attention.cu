// Attention kernels.
//
//   fa_fwd        causal GQA flash attention over packed documents (cu_seqlens),
//                 online softmax in the exp2 domain, writes O and the natural
//                 log-sum-exp per (head, token);
//   fa_bwd_prep   D_i = rowsum(dO ⊙ O);
//   fa_bwd_dkdv   per key block: recompute P^T, accumulate dV = P^T dO and
//                 dK = dS^T Q over every query head of the GQA group;
//   fa_bwd_dq     per query block: recompute P, dS, accumulate dQ = dS K;
//   paged_decode  split-KV decode attention over the paged KV cache; the
//                 GQA heads of one KV head form the MMA rows so K/V stream once;
//   kv_write      scatter new K/V rows into cache pages.
//
// Tiles are 64 queries x 64 keys; each of the 4 warps owns 16 rows.  The
// matrix products use the warp-synchronous bf16 MMA (m16n8k16) with ldmatrix
// from XOR-swizzled shared memory and cp.async double buffering.
#include "../include/common.cuh"
#include "attention.h"

namespace meshy {

namespace {

constexpr int BQ = 64, BKV = 64, NT = 128;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int HD>
__device__ __forceinline__ int swz(int row, int col) {  // element offset in a [rows][HD] swizzled tile
  constexpr int CH = HD / 8;
  int ch = (col >> 3) ^ (row & 7 & (CH - 1));
  return row * HD + ch * 8 + (col & 7);
}

// rows [r0, r0+64) of a [T, H, HD] tensor (head h) → swizzled smem; rows >= rend are zero
template <int HD>
__device__ __forceinline__ void load_tile(bf16* sm, const bf16* g, int r0, int rend, int H, int h) {
  constexpr int CH = HD / 8;
  for (int i = threadIdx.x; i < 64 * CH; i += NT) {
    int r = i / CH, c = (i % CH) * 8;
    int gr = r0 + r;
    bool ok = gr < rend;
    const bf16* src = g + ((size_t)(ok ? gr : 0) * H + h) * HD + c;
    cp_async16(sm + swz<HD>(r, c), src, ok);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const bf16* p) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const bf16* p) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A fragment (16x16) at (r0, c0) of a swizzled [rows][HD] tile
template <int HD>
__device__ __forceinline__ void frag_a(uint32_t* a, const bf16* sm, int r0, int c0) {
  int l = threadIdx.x % 32;
  int r = r0 + (l % 8) + 8 * ((l / 8) % 2), c = c0 + 8 * (l / 16);
  ldsm_x4(a[0], a[1], a[2], a[3], sm + swz<HD>(r, c));
}
// B fragments for two n-tiles (n0, n0+8) with k in [c0, c0+16): tile stored [n][k] (row = n)
template <int HD>
__device__ __forceinline__ void frag_b_nk(uint32_t* b, const bf16* sm, int n0, int c0) {
  int l = threadIdx.x % 32;
  int r = n0 + (l % 8) + 8 * (l / 16), c = c0 + 8 * ((l / 8) % 2);
  ldsm_x4(b[0], b[1], b[2], b[3], sm + swz<HD>(r, c));  // b[0],b[1]: tile n0; b[2],b[3]: tile n0+8
}
// B fragments for two n-tiles (n0, n0+8) with k in [k0, k0+16): tile stored [k][n] (row = k)
template <int HD>
__device__ __forceinline__ void frag_b_kn(uint32_t* b, const bf16* sm, int k0, int n0) {
  int l = threadIdx.x % 32;
  int r = k0 + (l % 8) + 8 * ((l / 8) % 2), c = n0 + 8 * (l / 16);
  ldsm_x4_t(b[0], b[1], b[2], b[3], sm + swz<HD>(r, c));
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

}  // namespace

// ═══════════════════════════════ forward ═══════════════════════════════════
template <int HD>
__global__ void __launch_bounds__(NT) fa_fwd_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                    const bf16* __restrict__ V, const int* __restrict__ cu,
                                                    const int* __restrict__ cu_k, const int* __restrict__ q_off,
                                                    bf16* __restrict__ O, float* __restrict__ LSE, int T, int max_blocks,
                                                    int Hq, int Hkv, float scale) {
  extern __shared__ __align__(128) uint8_t smraw[];
  bf16* Qs = reinterpret_cast<bf16*>(smraw);
  bf16* Ks = Qs + BQ * HD;
  bf16* Vs = Ks + 2 * BKV * HD;
  const int doc = blockIdx.x / max_blocks;
  const int qb = max_blocks - 1 - blockIdx.x % max_blocks;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int s = cu[doc], e = cu[doc + 1], L = e - s;
  // key document (the query document itself unless a separate key stream is given) and the
  // position of the first query inside it: query i attends keys [0, qo + i]
  const int ks = cu_k ? cu_k[doc] : s, ke = cu_k ? cu_k[doc + 1] : e, Lk = ke - ks;
  const int qo = q_off ? q_off[doc] : 0;
  const int q0 = qb * BQ;
  if (q0 >= L) return;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float sl2 = scale * kLog2e;

  load_tile<HD>(Qs, Q, s + q0, e, Hq, h);
  load_tile<HD>(Ks, K, ks, ke, Hkv, hk);
  load_tile<HD>(Vs, V, ks, ke, Hkv, hk);
  cp_commit();
  const int n_kb = max(0, min((Lk + BKV - 1) / BKV, (qo + q0 + BQ - 1) / BKV + 1));

  uint32_t qf[HD / 16][4];
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int row_a = q0 + warp * 16 + lane / 4;  // doc-relative query rows of this thread
  const int row_b = row_a + 8;

  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      load_tile<HD>(Ks + (buf ^ 1) * BKV * HD, K, ks + (kb + 1) * BKV, ke, Hkv, hk);
      load_tile<HD>(Vs + (buf ^ 1) * BKV * HD, V, ks + (kb + 1) * BKV, ke, Hkv, hk);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) frag_a<HD>(qf[kk], Qs, warp * 16, kk * 16);
    }
    const bf16* Kb = Ks + buf * BKV * HD;
    const bf16* Vb = Vs + buf * BKV * HD;
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b[4];
        frag_b_nk<HD>(b, Kb, j * 8, kk * 16);
        mma16816(sc[j], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b[0], b[1]);
        mma16816(sc[j + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b[2], b[3]);
      }
    }
    // scale, mask, online softmax (2 rows per thread)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        int key = kb * BKV + j * 8 + 2 * (lane % 4) + (t & 1);
        int row = (t < 2) ? row_a : row_b;
        float v = sc[j][t] * sl2;
        if (key > row + qo || key >= Lk) v = -INFINITY;
        sc[j][t] = v;
        mx[t >> 1] = fmaxf(mx[t >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], mnew[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(m_r[r], mx[r]);
      alpha[r] = (mnew[r] == -INFINITY) ? 1.f : exp2f(m_r[r] - mnew[r]);
      m_r[r] = mnew[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        int r = t >> 1;
        float p = (mnew[r] == -INFINITY) ? 0.f : exp2f(sc[j][t] - mnew[r]);
        sc[j][t] = p;
        rs[r] += p;
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      pf[kk][0] = pack_bf16x2(sc[2 * kk][0], sc[2 * kk][1]);
      pf[kk][1] = pack_bf16x2(sc[2 * kk][2], sc[2 * kk][3]);
      pf[kk][2] = pack_bf16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
      pf[kk][3] = pack_bf16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t b[4];
        frag_b_kn<HD>(b, Vb, kk * 16, i * 8);
        mma16816(o[i], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b[0], b[1]);
        mma16816(o[i + 1], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b[2], b[3]);
      }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int row = r == 0 ? row_a : row_b;
    if (row >= L) continue;
    float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    bf16* orow = O + ((size_t)(s + row) * Hq + h) * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      int c = i * 8 + 2 * (lane % 4);
      *reinterpret_cast<uint32_t*>(orow + c) = pack_bf16x2(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
    }
    if (lane % 4 == 0) LSE[(size_t)h * T + s + row] = (l_r[r] > 0.f) ? (m_r[r] * kLn2 + logf(l_r[r])) : -INFINITY;
  }
}

// ═══════════════════════════════ backward ══════════════════════════════════
__global__ void fa_bwd_prep_kernel(const bf16* __restrict__ O, const bf16* __restrict__ dO, float* __restrict__ Dv,
                                   int T, int Hq, int HD) {
  // one warp per (token, head); Dv layout [Hq, T]
  long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (w >= (long long)T * Hq) return;
  int t = (int)(w / Hq), h = (int)(w % Hq);
  int lane = threadIdx.x % 32;
  const bf16* o = O + ((size_t)t * Hq + h) * HD;
  const bf16* g = dO + ((size_t)t * Hq + h) * HD;
  float acc = 0.f;
  for (int c = lane * 2; c < HD; c += 64) {
    float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(o + c));
    float2 b = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(g + c));
    acc += a.x * b.x + a.y * b.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) Dv[(size_t)h * T + t] = acc;
}

// dK, dV for one key block of one KV head; loops over the GQA q heads and
// the causal query blocks.  Warp w owns keys [16w, 16w+16) of the block.
template <int HD>
__global__ void __launch_bounds__(NT) fa_bwd_dkdv_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                         const bf16* __restrict__ V, const bf16* __restrict__ dO,
                                                         const float* __restrict__ LSE, const float* __restrict__ Dv,
                                                         const int* __restrict__ cu, const int* __restrict__ cu_k,
                                                         const int* __restrict__ q_off, bf16* __restrict__ dK,
                                                         bf16* __restrict__ dV, int T, int max_blocks, int Hq, int Hkv,
                                                         float scale) {
  extern __shared__ __align__(128) uint8_t smraw[];
  bf16* Ks = reinterpret_cast<bf16*>(smraw);
  bf16* Vs = Ks + BKV * HD;
  bf16* Qs = Vs + BKV * HD;       // 2 buffers
  bf16* dOs = Qs + 2 * BQ * HD;   // 2 buffers
  float* lse_s = reinterpret_cast<float*>(dOs + 2 * BQ * HD);  // 2 x 64
  float* d_s = lse_s + 2 * BQ;                                  // 2 x 64
  const int doc = blockIdx.x / max_blocks;
  const int kb = blockIdx.x % max_blocks;
  const int hk = blockIdx.y;
  const int rep = Hq / Hkv;
  const int s = cu[doc], e = cu[doc + 1], L = e - s;
  const int ks = cu_k ? cu_k[doc] : s, ke = cu_k ? cu_k[doc + 1] : e, Lk = ke - ks;
  const int qo = q_off ? q_off[doc] : 0;
  const int k0 = kb * BKV;
  if (k0 >= Lk) return;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float sl2 = scale * kLog2e;
  load_tile<HD>(Ks, K, ks + k0, ke, Hkv, hk);
  load_tile<HD>(Vs, V, ks + k0, ke, Hkv, hk);
  cp_commit();

  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i)
#pragma unroll
    for (int t = 0; t < 4; ++t) dk[i][t] = dv[i][t] = 0.f;

  const int n_qb = (L + BQ - 1) / BQ;
  const int qb_first = min(n_qb, max(0, k0 - qo) / BQ);  // causal: query positions >= keys
  const int n_iter = rep * (n_qb - qb_first);
  auto issue = [&](int it, int buf) {
    int hh = hk * rep + it / (n_qb - qb_first);
    int qb = qb_first + it % (n_qb - qb_first);
    load_tile<HD>(Qs + buf * BQ * HD, Q, s + qb * BQ, e, Hq, hh);
    load_tile<HD>(dOs + buf * BQ * HD, dO, s + qb * BQ, e, Hq, hh);
    for (int i = threadIdx.x; i < BQ; i += NT) {
      int qrow = qb * BQ + i;
      bool ok = qrow < L;
      lse_s[buf * BQ + i] = ok ? LSE[(size_t)hh * T + s + qrow] : 0.f;
      d_s[buf * BQ + i] = ok ? Dv[(size_t)hh * T + s + qrow] : 0.f;
    }
  };
  issue(0, 0);
  cp_commit();
  const int key_a = k0 + warp * 16 + lane / 4;  // doc-relative keys of this thread's rows (S^T rows)
  const int key_b = key_a + 8;
  for (int it = 0; it < n_iter; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_iter) {
      issue(it + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int qb = qb_first + it % (n_qb - qb_first);
    const bf16* Qb = Qs + buf * BQ * HD;
    const bf16* dOb = dOs + buf * BQ * HD;
    const float* lse_b = lse_s + buf * BQ;
    const float* d_b = d_s + buf * BQ;
    // S^T = K Q^T (16 keys x 64 queries), dP^T = V dO^T
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int t = 0; t < 4; ++t) st[j][t] = dpt[j][t] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t kf[4], vf[4];
      frag_a<HD>(kf, Ks, warp * 16, kk * 16);
      frag_a<HD>(vf, Vs, warp * 16, kk * 16);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b[4];
        frag_b_nk<HD>(b, Qb, j * 8, kk * 16);
        mma16816(st[j], kf[0], kf[1], kf[2], kf[3], b[0], b[1]);
        mma16816(st[j + 1], kf[0], kf[1], kf[2], kf[3], b[2], b[3]);
        frag_b_nk<HD>(b, dOb, j * 8, kk * 16);
        mma16816(dpt[j], vf[0], vf[1], vf[2], vf[3], b[0], b[1]);
        mma16816(dpt[j + 1], vf[0], vf[1], vf[2], vf[3], b[2], b[3]);
      }
    }
    // P^T and dS^T
    uint32_t pf[4][4], dsf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        int ql = j * 8 + 2 * (lane % 4) + (t & 1);  // query within block
        int qrow = qb * BQ + ql;
        int key = (t < 2) ? key_a : key_b;
        float p = 0.f;
        if (qrow < L && key <= qrow + qo && key < Lk) p = exp2f(st[j][t] * sl2 - lse_b[ql] * kLog2e);
        st[j][t] = p;
        dpt[j][t] = p * (dpt[j][t] - d_b[ql]);
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      pf[kk][0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
      pf[kk][1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
      pf[kk][2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pf[kk][3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      dsf[kk][0] = pack_bf16x2(dpt[2 * kk][0], dpt[2 * kk][1]);
      dsf[kk][1] = pack_bf16x2(dpt[2 * kk][2], dpt[2 * kk][3]);
      dsf[kk][2] = pack_bf16x2(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      dsf[kk][3] = pack_bf16x2(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
    }
    // dV += P^T dO ; dK += dS^T Q   (k = queries)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t b[4];
        frag_b_kn<HD>(b, dOb, kk * 16, i * 8);
        mma16816(dv[i], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b[0], b[1]);
        mma16816(dv[i + 1], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b[2], b[3]);
        frag_b_kn<HD>(b, Qb, kk * 16, i * 8);
        mma16816(dk[i], dsf[kk][0], dsf[kk][1], dsf[kk][2], dsf[kk][3], b[0], b[1]);
        mma16816(dk[i + 1], dsf[kk][0], dsf[kk][1], dsf[kk][2], dsf[kk][3], b[2], b[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int key = r == 0 ? key_a : key_b;
    if (key >= Lk) continue;
    bf16* dkr = dK + ((size_t)(ks + key) * Hkv + hk) * HD;
    bf16* dvr = dV + ((size_t)(ks + key) * Hkv + hk) * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      int c = i * 8 + 2 * (lane % 4);
      *reinterpret_cast<uint32_t*>(dkr + c) = pack_bf16x2(dk[i][2 * r] * scale, dk[i][2 * r + 1] * scale);
      *reinterpret_cast<uint32_t*>(dvr + c) = pack_bf16x2(dv[i][2 * r], dv[i][2 * r + 1]);
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(NT) fa_bwd_dq_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                       const bf16* __restrict__ V, const bf16* __restrict__ dO,
                                                       const float* __restrict__ LSE, const float* __restrict__ Dv,
                                                       const int* __restrict__ cu, const int* __restrict__ cu_k,
                                                       const int* __restrict__ q_off, bf16* __restrict__ dQ, int T,
                                                       int max_blocks, int Hq, int Hkv, float scale) {
  extern __shared__ __align__(128) uint8_t smraw[];
  bf16* Qs = reinterpret_cast<bf16*>(smraw);
  bf16* dOs = Qs + BQ * HD;
  bf16* Ks = dOs + BQ * HD;  // 2 buffers
  bf16* Vs = Ks + 2 * BKV * HD;
  const int doc = blockIdx.x / max_blocks;
  const int qb = max_blocks - 1 - blockIdx.x % max_blocks;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int s = cu[doc], e = cu[doc + 1], L = e - s;
  const int ks = cu_k ? cu_k[doc] : s, ke = cu_k ? cu_k[doc + 1] : e, Lk = ke - ks;
  const int qo = q_off ? q_off[doc] : 0;
  const int q0 = qb * BQ;
  if (q0 >= L) return;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float sl2 = scale * kLog2e;
  load_tile<HD>(Qs, Q, s + q0, e, Hq, h);
  load_tile<HD>(dOs, dO, s + q0, e, Hq, h);
  load_tile<HD>(Ks, K, ks, ke, Hkv, hk);
  load_tile<HD>(Vs, V, ks, ke, Hkv, hk);
  cp_commit();
  const int row_a = q0 + warp * 16 + lane / 4, row_b = row_a + 8;
  const float lse_a = row_a < L ? LSE[(size_t)h * T + s + row_a] * kLog2e : 0.f;
  const float lse_b = row_b < L ? LSE[(size_t)h * T + s + row_b] * kLog2e : 0.f;
  const float d_a = row_a < L ? Dv[(size_t)h * T + s + row_a] : 0.f;
  const float d_b = row_b < L ? Dv[(size_t)h * T + s + row_b] : 0.f;
  const int n_kb = max(0, min((Lk + BKV - 1) / BKV, (qo + q0 + BQ - 1) / BKV + 1));
  uint32_t qf[HD / 16][4];
  float dq[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      load_tile<HD>(Ks + (buf ^ 1) * BKV * HD, K, ks + (kb + 1) * BKV, ke, Hkv, hk);
      load_tile<HD>(Vs + (buf ^ 1) * BKV * HD, V, ks + (kb + 1) * BKV, ke, Hkv, hk);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) frag_a<HD>(qf[kk], Qs, warp * 16, kk * 16);
    }
    const bf16* Kb = Ks + buf * BKV * HD;
    const bf16* Vb = Vs + buf * BKV * HD;
    float sc[8][4], dp[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int t = 0; t < 4; ++t) sc[j][t] = dp[j][t] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t gf[4];
      frag_a<HD>(gf, dOs, warp * 16, kk * 16);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b[4];
        frag_b_nk<HD>(b, Kb, j * 8, kk * 16);
        mma16816(sc[j], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b[0], b[1]);
        mma16816(sc[j + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b[2], b[3]);
        frag_b_nk<HD>(b, Vb, j * 8, kk * 16);
        mma16816(dp[j], gf[0], gf[1], gf[2], gf[3], b[0], b[1]);
        mma16816(dp[j + 1], gf[0], gf[1], gf[2], gf[3], b[2], b[3]);
      }
    }
    uint32_t dsf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        int key = kb * BKV + j * 8 + 2 * (lane % 4) + (t & 1);
        int row = t < 2 ? row_a : row_b;
        float p = 0.f;
        if (row < L && key <= row + qo && key < Lk) p = exp2f(sc[j][t] * sl2 - (t < 2 ? lse_a : lse_b));
        dp[j][t] = p * (dp[j][t] - (t < 2 ? d_a : d_b));
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      dsf[kk][0] = pack_bf16x2(dp[2 * kk][0], dp[2 * kk][1]);
      dsf[kk][1] = pack_bf16x2(dp[2 * kk][2], dp[2 * kk][3]);
      dsf[kk][2] = pack_bf16x2(dp[2 * kk + 1][0], dp[2 * kk + 1][1]);
      dsf[kk][3] = pack_bf16x2(dp[2 * kk + 1][2], dp[2 * kk + 1][3]);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t b[4];
        frag_b_kn<HD>(b, Kb, kk * 16, i * 8);
        mma16816(dq[i], dsf[kk][0], dsf[kk][1], dsf[kk][2], dsf[kk][3], b[0], b[1]);
        mma16816(dq[i + 1], dsf[kk][0], dsf[kk][1], dsf[kk][2], dsf[kk][3], b[2], b[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int row = r == 0 ? row_a : row_b;
    if (row >= L) continue;
    bf16* g = dQ + ((size_t)(s + row) * Hq + h) * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      int c = i * 8 + 2 * (lane % 4);
      *reinterpret_cast<uint32_t*>(g + c) = pack_bf16x2(dq[i][2 * r] * scale, dq[i][2 * r + 1] * scale);
    }
  }
}

// ═══════════════════════════════ decode ════════════════════════════════════
// One CTA per (sequence, kv head, split).  The rep = Hq/Hkv query heads are the
// MMA rows (padded to 16).  Each warp takes 16 keys of every 64-key page, keeps
// its own online softmax; the four warp states are merged in shared memory.
// With n_split > 1 the CTA writes (m, l, O) to ``part`` and
// paged_decode_combine_kernel merges the splits.
template <int HD>
__global__ void __launch_bounds__(NT) paged_decode_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ Kc,
                                                          const bf16* __restrict__ Vc, const int* __restrict__ bt,
                                                          const int* __restrict__ seq_lens, bf16* __restrict__ O,
                                                          float* __restrict__ part, int Hq, int Hkv, int page,
                                                          int max_pages, int n_split, float scale) {
  extern __shared__ __align__(128) uint8_t smraw[];
  bf16* Qs = reinterpret_cast<bf16*>(smraw);            // 16 x HD
  bf16* Ks = Qs + 16 * HD;                                // 2 x 64 x HD
  bf16* Vs = Ks + 2 * 64 * HD;
  float* red = reinterpret_cast<float*>(Vs + 2 * 64 * HD);  // merge scratch
  const int b = blockIdx.x, hk = blockIdx.y, sp = blockIdx.z;
  const int rep = Hq / Hkv;
  const int L = seq_lens[b];
  // never read past the row's block table, whatever seq_lens says
  const int n_pages = min((L + page - 1) / page, max_pages);
  const int per = (n_pages + n_split - 1) / n_split;
  const int p0 = sp * per, p1 = min(n_pages, p0 + per);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float sl2 = scale * kLog2e;
  // Q rows (rep heads) → smem, rows >= rep zero
  for (int i = threadIdx.x; i < 16 * HD / 8; i += NT) {
    int r = i / (HD / 8), c = (i % (HD / 8)) * 8;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < rep) val = *reinterpret_cast<const uint4*>(Q + ((size_t)b * Hq + hk * rep + r) * HD + c);
    *reinterpret_cast<uint4*>(Qs + swz<HD>(r, c)) = val;
  }
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  auto issue = [&](int pi, int buf) {
    int pg = bt[(size_t)b * max_pages + pi];
    const bf16* kp = Kc + ((size_t)pg * Hkv + hk) * page * HD;
    const bf16* vp = Vc + ((size_t)pg * Hkv + hk) * page * HD;
    for (int i = threadIdx.x; i < 64 * HD / 8; i += NT) {
      int r = i / (HD / 8), c = (i % (HD / 8)) * 8;
      bool ok = r < page;
      cp_async16(Ks + buf * 64 * HD + swz<HD>(r, c), kp + (size_t)(ok ? r : 0) * HD + c, ok);
      cp_async16(Vs + buf * 64 * HD + swz<HD>(r, c), vp + (size_t)(ok ? r : 0) * HD + c, ok);
    }
  };
  if (p0 < p1) {
    issue(p0, 0);
    cp_commit();
  }
  __syncthreads();
  uint32_t qf[HD / 16][4];
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) frag_a<HD>(qf[kk], Qs, 0, kk * 16);
  for (int pi = p0; pi < p1; ++pi) {
    const int buf = (pi - p0) & 1;
    if (pi + 1 < p1) {
      issue(pi + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const bf16* Kb = Ks + buf * 64 * HD;
    const bf16* Vb = Vs + buf * 64 * HD;
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t bb[4];
      frag_b_nk<HD>(bb, Kb, warp * 16, kk * 16);
      mma16816(sc[0], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], bb[0], bb[1]);
      mma16816(sc[1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], bb[2], bb[3]);
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        int key = pi * page + warp * 16 + j * 8 + 2 * (lane % 4) + (t & 1);
        float v = (key < L && warp * 16 + j * 8 + 2 * (lane % 4) + (t & 1) < page) ? sc[j][t] * sl2 : -INFINITY;
        sc[j][t] = v;
        mx[t >> 1] = fmaxf(mx[t >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], mnew[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(m_r[r], mx[r]);
      alpha[r] = (mnew[r] == -INFINITY) ? 1.f : exp2f(m_r[r] - mnew[r]);
      m_r[r] = mnew[r];
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float p = (mnew[t >> 1] == -INFINITY) ? 0.f : exp2f(sc[j][t] - mnew[t >> 1]);
        sc[j][t] = p;
        rs[t >> 1] += p;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    uint32_t pf0 = pack_bf16x2(sc[0][0], sc[0][1]), pf1 = pack_bf16x2(sc[0][2], sc[0][3]);
    uint32_t pf2 = pack_bf16x2(sc[1][0], sc[1][1]), pf3 = pack_bf16x2(sc[1][2], sc[1][3]);
#pragma unroll
    for (int i = 0; i < HD / 8; i += 2) {
      uint32_t bb[4];
      frag_b_kn<HD>(bb, Vb, warp * 16, i * 8);
      mma16816(o[i], pf0, pf1, pf2, pf3, bb[0], bb[1]);
      mma16816(o[i + 1], pf0, pf1, pf2, pf3, bb[2], bb[3]);
    }
    __syncthreads();
  }
  // merge the 4 warps: rows lane/4 (< 8 real rows; row+8 only if rep > 8)
  // red layout: [4 warps][16 rows] m, l  then [4 warps][16 rows][HD] o
  float* rm = red;
  float* rl = red + 64;
  float* ro = red + 128;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int row = lane / 4 + 8 * r;
    if (lane % 4 == 0) {
      rm[warp * 16 + row] = m_r[r];
      rl[warp * 16 + row] = l_r[r];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      int c = i * 8 + 2 * (lane % 4);
      ro[(warp * 16 + row) * HD + c] = o[i][2 * r];
      ro[(warp * 16 + row) * HD + c + 1] = o[i][2 * r + 1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < rep * HD; idx += NT) {
    int row = idx / HD, c = idx % HD;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, rm[w * 16 + row]);
    float Ls = 0.f, acc = 0.f;
    for (int w = 0; w < 4; ++w) {
      float mw = rm[w * 16 + row];
      float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      Ls += rl[w * 16 + row] * f;
      acc += ro[(w * 16 + row) * HD + c] * f;
    }
    const int h = hk * rep + row;
    if (n_split == 1) {
      O[((size_t)b * Hq + h) * HD + c] = __float2bfloat16(Ls > 0.f ? acc / Ls : 0.f);
    } else {
      float* pp = part + (((size_t)b * Hq + h) * n_split + sp) * (HD + 2);
      pp[c] = acc;
      if (c == 0) {
        pp[HD] = M;
        pp[HD + 1] = Ls;
      }
    }
  }
}

__global__ void paged_decode_combine_kernel(const float* __restrict__ part, bf16* __restrict__ O, int Hq, int HD,
                                            int n_split) {
  const int bh = blockIdx.x;  // b * Hq + h
  const float* pp = part + (size_t)bh * n_split * (HD + 2);
  float M = -INFINITY;
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, pp[s * (HD + 2) + HD]);
  for (int c = threadIdx.x; c < HD; c += blockDim.x) {
    float Ls = 0.f, acc = 0.f;
    for (int s = 0; s < n_split; ++s) {
      float ms = pp[s * (HD + 2) + HD];
      float f = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
      Ls += pp[s * (HD + 2) + HD + 1] * f;
      acc += pp[s * (HD + 2) + c] * f;
    }
    O[(size_t)bh * HD + c] = __float2bfloat16(Ls > 0.f ? acc / Ls : 0.f);
  }
}

__global__ void kv_write_kernel(const bf16* __restrict__ k, const bf16* __restrict__ v, bf16* __restrict__ kc,
                                bf16* __restrict__ vc, const int64_t* __restrict__ slots, int n, int Hkv, int HD,
                                int page) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  int per = Hkv * HD / 8;
  if (idx >= (long long)n * per) return;
  int t = (int)(idx / per), r = (int)(idx % per);
  int h = r / (HD / 8), c = (r % (HD / 8)) * 8;
  int64_t slot = slots[t];
  int64_t pg = slot / page, off = slot % page;
  size_t dst = (((size_t)pg * Hkv + h) * page + off) * HD + c;
  size_t src = ((size_t)t * Hkv + h) * HD + c;
  *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(k + src);
  *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(v + src);
}

// ═══════════════════════════════ host ══════════════════════════════════════
template <typename F>
static void set_smem(F f, int bytes) {
  MESHY_CUDA_CHECK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

void flash_attn_fwd(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, bf16* o, float* lse, int T,
                    int max_seqlen, int Hq, int Hkv, int hd, float scale, cudaStream_t st, const int* cu_k,
                    const int* q_off, int Tk, int* err) {
  MESHY_CHECK(hd == 64 || hd == 128, "flash_attn: head_dim must be 64 or 128");
  MESHY_CHECK(Hq % Hkv == 0, "flash_attn: Hq must be a multiple of Hkv");
  if (hd == 128 && flash_attn_tc_enabled()) {
    flash_attn_fwd_tc(q, k, v, cu, n_docs, o, lse, T, Tk < 0 ? T : Tk, max_seqlen, Hq, Hkv, scale, st, cu_k, q_off,
                      err);
    return;
  }
  int mb = (max_seqlen + BQ - 1) / BQ;
  dim3 grid(n_docs * mb, Hq);
  if (n_docs * mb == 0) return;
  if (hd == 128) {
    int sm = (BQ + 4 * BKV) * 128 * 2;
    set_smem(fa_fwd_kernel<128>, sm);
    fa_fwd_kernel<128><<<grid, NT, sm, st>>>(q, k, v, cu, cu_k, q_off, o, lse, T, mb, Hq, Hkv, scale);
  } else {
    int sm = (BQ + 4 * BKV) * 64 * 2;
    set_smem(fa_fwd_kernel<64>, sm);
    fa_fwd_kernel<64><<<grid, NT, sm, st>>>(q, k, v, cu, cu_k, q_off, o, lse, T, mb, Hq, Hkv, scale);
  }
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void flash_attn_bwd(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, const bf16* o,
                    const bf16* dout, const float* lse, float* dvec, bf16* dq, bf16* dk, bf16* dv, int T,
                    int max_seqlen, int Hq, int Hkv, int hd, float scale, cudaStream_t st, const int* cu_k,
                    const int* q_off, int max_seqlen_k, int Tk, int* err) {
  MESHY_CHECK(hd == 64 || hd == 128, "flash_attn: head_dim must be 64 or 128");
  long long warps = (long long)T * Hq;
  if (warps == 0) return;
  fa_bwd_prep_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(o, dout, dvec, T, Hq, hd);
  if (hd == 128 && flash_attn_tc_enabled()) {
    flash_attn_bwd_tc(q, k, v, dout, lse, dvec, cu, n_docs, dq, dk, dv, T, Tk < 0 ? T : Tk, max_seqlen,
                      cu_k ? max_seqlen_k : max_seqlen, Hq, Hkv, scale, st, cu_k, q_off, err);
    return;
  }
  int mb = (max_seqlen + BQ - 1) / BQ;
  int mbk = ((cu_k ? max_seqlen_k : max_seqlen) + BKV - 1) / BKV;
  dim3 g_kv(n_docs * mbk, Hkv), g_q(n_docs * mb, Hq);
  if (hd == 128) {
    int sm1 = (2 * BKV + 4 * BQ) * 128 * 2 + 4 * BQ * 4;
    set_smem(fa_bwd_dkdv_kernel<128>, sm1);
    fa_bwd_dkdv_kernel<128><<<g_kv, NT, sm1, st>>>(q, k, v, dout, lse, dvec, cu, cu_k, q_off, dk, dv, T, mbk, Hq, Hkv,
                                                   scale);
    int sm2 = (2 * BQ + 4 * BKV) * 128 * 2;
    set_smem(fa_bwd_dq_kernel<128>, sm2);
    fa_bwd_dq_kernel<128><<<g_q, NT, sm2, st>>>(q, k, v, dout, lse, dvec, cu, cu_k, q_off, dq, T, mb, Hq, Hkv, scale);
  } else {
    int sm1 = (2 * BKV + 4 * BQ) * 64 * 2 + 4 * BQ * 4;
    set_smem(fa_bwd_dkdv_kernel<64>, sm1);
    fa_bwd_dkdv_kernel<64><<<g_kv, NT, sm1, st>>>(q, k, v, dout, lse, dvec, cu, cu_k, q_off, dk, dv, T, mbk, Hq, Hkv,
                                                  scale);
    int sm2 = (2 * BQ + 4 * BKV) * 64 * 2;
    set_smem(fa_bwd_dq_kernel<64>, sm2);
    fa_bwd_dq_kernel<64><<<g_q, NT, sm2, st>>>(q, k, v, dout, lse, dvec, cu, cu_k, q_off, dq, T, mb, Hq, Hkv, scale);
  }
  MESHY_CUDA_CHECK(cudaGetLastError());
}

int paged_decode_splits(int B, int Hkv, int max_pages) {
  int ctas = B * Hkv;
  int want = (2 * 148 + ctas - 1) / ctas;
  return std::max(1, std::min({want, max_pages, 64}));
}

void paged_decode(const bf16* q, const bf16* kc, const bf16* vc, const int* bt, const int* seq_lens, bf16* o,
                  float* part, int B, int Hq, int Hkv, int hd, int page, int max_pages, int n_split, float scale,
                  cudaStream_t st) {
  MESHY_CHECK(hd == 64 || hd == 128, "paged_decode: head_dim must be 64 or 128");
  MESHY_CHECK(page == 64, "paged_decode: page size must be 64");
  MESHY_CHECK(Hq / Hkv <= 16, "paged_decode: at most 16 query heads per KV head");
  MESHY_CHECK(n_split == 1 || part != nullptr, "paged_decode: split workspace missing");
  dim3 grid(B, Hkv, n_split);
  if (B == 0) return;
  if (hd == 128) {
    int sm = (16 + 4 * 64) * 128 * 2 + (128 + 64 * 128) * 4;
    set_smem(paged_decode_kernel<128>, sm);
    paged_decode_kernel<128><<<grid, NT, sm, st>>>(q, kc, vc, bt, seq_lens, o, part, Hq, Hkv, page, max_pages, n_split,
                                                   scale);
  } else {
    int sm = (16 + 4 * 64) * 64 * 2 + (128 + 64 * 64) * 4;
    set_smem(paged_decode_kernel<64>, sm);
    paged_decode_kernel<64><<<grid, NT, sm, st>>>(q, kc, vc, bt, seq_lens, o, part, Hq, Hkv, page, max_pages, n_split,
                                                  scale);
  }
  if (n_split > 1) paged_decode_combine_kernel<<<B * Hq, 128, 0, st>>>(part, o, Hq, hd, n_split);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void paged_decode_combine(const float* part, bf16* o, int B, int Hq, int hd, int n_split, cudaStream_t st) {
  if (B == 0) return;
  paged_decode_combine_kernel<<<B * Hq, 128, 0, st>>>(part, o, Hq, hd, n_split);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void kv_write(const bf16* k, const bf16* v, bf16* kc, bf16* vc, const int64_t* slots, int n, int Hkv, int hd, int page,
              cudaStream_t st) {
  long long total = (long long)n * Hkv * hd / 8;
  if (total == 0) return;
  kv_write_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(k, v, kc, vc, slots, n, Hkv, hd, page);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
