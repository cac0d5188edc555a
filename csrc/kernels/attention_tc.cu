// Flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), head_dim 128.
//
// Same problem and conventions as fa_fwd_kernel in attention.cu: packed varlen documents
// (cu_seqlens), an optional separate key stream (cu_k) and per-document query offset (q_off) for
// context-parallel chunks, causal masking "key <= q_off + row", GQA, output O [T, Hq, 128] and the
// natural-log LSE [Hq, T].
//
// One CTA computes 128 query rows of one head against 128-key tiles:
//
//   warp 0      TMA producer: Q once; K and V tiles into a two-stage ring (V in the MN-major
//               layout the P.V product reads it in).
//   warp 1      TMEM allocator and single-thread MMA issuer:
//                 S_j = Q K_j^T        (M=128 queries, N=128 keys,  K=128 dims) into S[j % 2]
//                 O  += P_j V_j        (M=128 queries, N=128 dims,  K=128 keys) into O
//               S_{j+1} is issued before P_j is ready, so the tensor core works on the next
//               scores while the softmax warps exponentiate the current ones.
//   warps 2-5   softmax: thread r owns query row r (TMEM lane r). It reads its row of S_j,
//               masks (diagonal and document-end tiles only), keeps a running max and sum,
//               writes bf16 P_j into shared memory in the 128-byte-swizzled K-major layout of an
//               MMA A operand, and at the end reads its row of O, divides by the sum and stores it.
//               One FMA and one ex2 per score. (Two query tiles per CTA with two softmax
//               warpgroups measured slower: both warpgroups ran in step and shared the
//               special-function units while the tensor core waited.)
//
// O stays in TMEM for the whole key sweep. Its rows are rescaled only when a row's running max
// grows by more than 8 (log2 units) over the max its O was accumulated against; otherwise the
// exponentials are taken against the stale max (P <= 2^8, exact after the final division). The
// rescale reads and writes the row through tcgen05.ld / tcgen05.st after the previous P.V product
// has completed.
//
// Every mbarrier wait is bounded; a timed-out wait records an error code and the CTA drains and
// returns.
#include <cuda.h>

#include <cmath>
#include <cstdlib>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "attention.h"
#include "gemm.h"

namespace meshy {

namespace {

constexpr int TBQ = 128, TBK = 128, THD = 128;
constexpr int kFaThreads = 192;
constexpr int kTileBytes = 128 * 128 * 2;  // one 128 x 128 bf16 tile
// shared memory: Q, K[2], V[2], P (1024-aligned), then the barriers
constexpr int kQOff = 0, kKOff = kTileBytes, kVOff = 3 * kTileBytes, kPOff = 5 * kTileBytes;
constexpr int kBarOff = 6 * kTileBytes;
constexpr int kFaSmem = 1024 + kBarOff + 256;
constexpr float kL2e = 1.4426950408889634f;
constexpr float kLn2f = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.f;  // log2 units

// 2^x on the special-function unit (the hardware instruction; inputs here are <= 0 or -inf).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kFaThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                     const __grid_constant__ CUtensorMap mapV, const int* __restrict__ cu,
                     const int* __restrict__ cu_k, const int* __restrict__ q_off, bf16* __restrict__ O,
                     float* __restrict__ LSE, int T, int max_blocks, int Hq, int Hkv, float scale, int* err) {
  extern __shared__ __align__(1024) uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_free = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;
  uint64_t* o_done = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int doc = blockIdx.x / max_blocks;
  const int qb = max_blocks - 1 - blockIdx.x % max_blocks;  // longest causal rows first
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int s = cu[doc], e = cu[doc + 1], L = e - s;
  const int ks = cu_k ? cu_k[doc] : s, ke = cu_k ? cu_k[doc + 1] : e, Lk = ke - ks;
  const int qo = q_off ? q_off[doc] : 0;
  const int q0 = qb * TBQ;
  if (q0 >= L) return;
  const int n_kb = max(0, min((Lk + TBK - 1) / TBK, (qo + q0 + TBQ - 1) / TBK + 1));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapQ);
    tma_prefetch_desc(&mapK);
    tma_prefetch_desc(&mapV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0 at column 0, S1 at 128, O at 256

  if (warp == 0) {
    // ───────────────────────────── TMA producer ─────────────────────────────
    if (lane == 0 && n_kb > 0) {
      mbar_arrive_expect_tx(q_full, kTileBytes);
      for (int c = 0; c < 2; ++c) tma_load_2d(sm + kQOff + c * 16384, &mapQ, q_full, h * THD + c * 64, s + q0);
      int last = -1;
      uint32_t last_par = 0;
      for (int j = 0; j < n_kb; ++j) {
        const int st = j & 1;
        const uint32_t par = (j >> 1) & 1;
        const int row = ks + j * TBK;
        if (!mbar_wait(&k_empty[st], par ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&k_full[st], kTileBytes);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sm + kKOff + st * kTileBytes + c * 16384, &mapK, &k_full[st], hk * THD + c * 64, row);
        if (!mbar_wait(&v_empty[st], par ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&v_full[st], kTileBytes);
        // MN-major B operand: [key block of 64][dim block of 64][64 keys][64 dims]
        for (int kb2 = 0; kb2 < 2; ++kb2)
          for (int c = 0; c < 2; ++c)
            tma_load_2d(sm + kVOff + st * kTileBytes + kb2 * 16384 + c * 8192, &mapV, &v_full[st], hk * THD + c * 64,
                        row + kb2 * 64);
        last = st;
        last_par = par;
      }
      if (*abort_flag && last >= 0) {
        long long t0 = clock64();
        while (!mbar_try_wait(&v_full[last], last_par) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ───────────────────────────── MMA issuer ───────────────────────────────
    if (lane == 0 && n_kb > 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t id_o = idesc_bf16_f32(128, 128, false, true);
      const uint32_t sq = smem_u32(sm + kQOff), sp = smem_u32(sm + kPOff);
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrTimeoutMma);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t par = (j >> 1) & 1;
        if (!mbar_wait(&k_full[st], par, abort_flag, err, kErrTimeoutMma)) return false;
        if (!mbar_wait(&s_free[st], par ^ 1, abort_flag, err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(sm + kKOff + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < THD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_bf16(tmem + st * 128, smem_desc_sw128(sq + off, 16, 1024), smem_desc_sw128(sk + off, 16, 1024), id_s,
                   k > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[st]);
        mma_commit(&k_empty[st]);
        return true;
      };
      // S_{j+1} is issued before P_j is ready: the tensor core computes the next scores while the
      // softmax warps exponentiate the current ones
      if (ok) ok = issue_s(0);
      if (ok && n_kb > 1) ok = issue_s(1);
      for (int j = 0; j < n_kb && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(p_full, j & 1, abort_flag, err, kErrTimeoutMma)) break;
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t sv = smem_u32(sm + kVOff + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < TBK / 16; ++k) {
          const uint32_t a_off = (k >> 2) * 16384 + (k & 3) * 32;
          const uint32_t b_off = (k >> 2) * 16384 + (k & 3) * 2048;
          mma_bf16(tmem + 256, smem_desc_sw128(sp + a_off, 16, 1024), smem_desc_sw128(sv + b_off, 8192, 1024), id_o,
                   (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(o_done);
        mma_commit(&v_empty[st]);
        if (j + 2 < n_kb) ok = issue_s(j + 2);
      }
    }
  } else {
    // ───────────────────────────── softmax warps ────────────────────────────
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // query row of this thread = TMEM lane
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const float sl2 = scale * kL2e;
    const int qpos = qo + q0 + r;  // keys <= qpos are visible to this row
    uint8_t* prow = sm + kPOff + r * 128;
    float m_used = -INFINITY, l = 0.f;  // running max (log2 units, scaled scores) and sum
    bool ok = true;
    float v[128];
    for (int j = 0; j < n_kb && ok; ++j) {
      const int sb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (j >> 1) & 1, abort_flag, err, kErrTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(t_lane + sb * 128 + c * 32, v + c * 32);
      tc_fence_before();
      mbar_arrive(&s_free[sb]);
      const int key0 = j * TBK;
      float mx = -INFINITY;  // max of the raw scores of this row's visible keys
      if (key0 + TBK - 1 > qpos || key0 + TBK > Lk) {
        const int lim = min(qpos + 1, Lk) - key0;  // keys [0, lim) of the tile are visible
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          v[c] = c < lim ? v[c] : -INFINITY;
          mx = fmaxf(mx, v[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) mx = fmaxf(mx, v[c]);
      }
      const float m_new = fmaxf(m_used, mx * sl2);
      const bool need = (m_used == -INFINITY) ? (m_new != -INFINITY) : (m_new > m_used + kRescaleThreshold);
      if (j > 0) {
        // the previous P.V product must be done before P is overwritten (and before O is rescaled)
        ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, abort_flag, err, kErrTimeoutEpilogue));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, need && m_used != -INFINITY)) {
          const float alpha = (need && m_used != -INFINITY) ? ex2(m_used - m_new) : 1.f;
          float ov[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tmem_ld32(t_lane + 256 + c * 32, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(t_lane + 256 + c * 32, ov);
          }
          tc_fence_before();
          l *= alpha;
        }
      }
      if (need) m_used = m_new;
      // p = 2^(score * scale * log2(e) - m_used): one FMA and one ex2 per score (-inf scores give 0)
      const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 128; c += 8) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p0 = ex2(fmaf(v[c + 2 * i], sl2, neg_m));
          const float p1 = ex2(fmaf(v[c + 2 * i + 1], sl2, neg_m));
          rs += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        // 128-byte swizzle of the K-major A tile: 16-byte chunk index XOR (row % 8)
        const int chunk = (c & 63) >> 3;
        *reinterpret_cast<uint4*>(prow + (c >> 6) * 16384 + ((chunk ^ (r & 7)) << 4)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l += rs;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(p_full);
    }
    // epilogue: O row / l
    const bool row_ok = q0 + r < L;
    if (ok && n_kb > 0)
      ok = __all_sync(0xffffffffu, mbar_wait(o_done, (n_kb - 1) & 1, abort_flag, err, kErrTimeoutEpilogue));
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = O + ((size_t)(s + q0 + r) * Hq + h) * THD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        if (n_kb > 0) {
          tmem_ld32(t_lane + 256 + c * 32, ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0.f;
        }
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            *reinterpret_cast<uint4*>(orow + c * 32 + i) =
                make_uint4(pack_bf16x2(ov[i] * inv, ov[i + 1] * inv), pack_bf16x2(ov[i + 2] * inv, ov[i + 3] * inv),
                           pack_bf16x2(ov[i + 4] * inv, ov[i + 5] * inv), pack_bf16x2(ov[i + 6] * inv, ov[i + 7] * inv));
          }
        }
      }
      if (row_ok) LSE[(size_t)h * T + s + q0 + r] = l > 0.f ? (m_used * kLn2f + logf(l)) : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace

bool flash_attn_tc_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESHY_FA_TC");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

void flash_attn_fwd_tc(const bf16* q, const bf16* k, const bf16* v, const int* cu, int n_docs, bf16* o, float* lse,
                       int T, int Tk, int max_seqlen, int Hq, int Hkv, float scale, cudaStream_t st, const int* cu_k,
                       const int* q_off, int* err) {
  MESHY_CHECK(Hq % Hkv == 0, "flash_attn: Hq must be a multiple of Hkv");
  const int mb = (max_seqlen + TBQ - 1) / TBQ;
  if (n_docs * mb == 0 || T == 0 || Tk == 0) return;
  // [T, H * 128] views; K-major tiles: box {64 dims, 128 rows}; V (MN-major operand): box {64, 64}
  CUtensorMap mq = make_map_bf16(q, T, (int64_t)Hq * THD, (int64_t)Hq * THD, 64, 128);
  CUtensorMap mk = make_map_bf16(k, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 128);
  CUtensorMap mv = make_map_bf16(v, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 64);
  static bool attr = false;
  if (!attr) {
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(fa_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem));
    attr = true;
  }
  dim3 grid(n_docs * mb, Hq);
  fa_fwd_tc_kernel<<<grid, kFaThreads, kFaSmem, st>>>(mq, mk, mv, cu, cu_k, q_off, o, lse, T, mb, Hq, Hkv, scale, err);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
