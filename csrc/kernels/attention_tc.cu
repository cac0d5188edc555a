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

// Named barrier with an AND-reduction: every participating thread gets the same answer, so a
// decision to stop is taken by all of them together.
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// 2^x on the special-function unit (the hardware instruction; inputs here are <= 0 or -inf).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Key / value streams of the forward kernel. NP == 1: one local [Tk, Hkv * 128] stream. NP > 1:
// context parallelism over ``cp`` ranks without an all-gather: every rank's local K / V ([rows * 2c, Hkv
// * 128], its head chunk r then its tail chunk 2 cp - 1 - r of every row) is read in place, through the
// rank's peer mapping, by plain (non-multicast) TMA loads; key position p of row ``doc / docs_per_row``
// lives in chunk p / c on rank (chunk < cp ? chunk : 2 cp - 1 - chunk).
template <int NP>
struct FaKV {
  CUtensorMap k[NP], v[NP];
  int cp, chunk, seq, docs_per_row;
};

template <int NP>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ FaKV<NP> kv,
                     const int* __restrict__ cu, const int* __restrict__ cu_k, const int* __restrict__ q_off,
                     bf16* __restrict__ O, float* __restrict__ LSE, int T, int max_blocks, int Hq, int Hkv,
                     float scale, int* err) {
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

  // query-tile-major dispatch, the longest causal rows (highest tile) of every document first
  const int n_docs = gridDim.x / max_blocks;
  const int doc = blockIdx.x % n_docs;
  const int qb = max_blocks - 1 - blockIdx.x / n_docs;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int s = cu[doc], e = cu[doc + 1], L = e - s;
  const int ks = NP > 1 ? 0 : (cu_k ? cu_k[doc] : s);
  const int Lk = NP > 1 ? kv.seq : (cu_k ? cu_k[doc + 1] : e) - ks;
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
    tma_prefetch_desc(&kv.k[0]);
    tma_prefetch_desc(&kv.v[0]);
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
        int row = ks + j * TBK;
        const CUtensorMap* mapK = &kv.k[0];
        const CUtensorMap* mapV = &kv.v[0];
        if constexpr (NP > 1) {
          const int pos = j * TBK, ci = pos / kv.chunk;  // a key tile never straddles two chunks
          const int owner = ci < kv.cp ? ci : 2 * kv.cp - 1 - ci;
          row = (doc / kv.docs_per_row) * 2 * kv.chunk + (ci < kv.cp ? 0 : kv.chunk) + pos % kv.chunk;
          mapK = &kv.k[owner];
          mapV = &kv.v[owner];
        }
        if (!mbar_wait(&k_empty[st], par ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&k_full[st], kTileBytes);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sm + kKOff + st * kTileBytes + c * 16384, mapK, &k_full[st], hk * THD + c * 64, row);
        if (!mbar_wait(&v_empty[st], par ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&v_full[st], kTileBytes);
        // MN-major B operand: [key block of 64][dim block of 64][64 keys][64 dims]
        for (int kb2 = 0; kb2 < 2; ++kb2)
          for (int c = 0; c < 2; ++c)
            tma_load_2d(sm + kVOff + st * kTileBytes + kb2 * 16384 + c * 8192, mapV, &v_full[st], hk * THD + c * 64,
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

// ═════════════════════════════ backward ═════════════════════════════════════
//
// dK / dV: one CTA per 128-key block of one KV head, sweeping the GQA query heads and the causal
// 64-query blocks. Transposed products keep the key rows on the TMEM lanes:
//   S^T = K Q_i^T, dP^T = V dO_i^T            (M=128 keys, N=64 queries, K=128 dims)
//   P^T = 2^(S^T scale log2e - LSE log2e), dS^T = P^T (dP^T - D)   (thread = key row)
//   dV += P^T dO_i, dK += dS^T Q_i           (M=128 keys, N=128 dims, K=64 queries)
// Q_i and dO_i are loaded once in the K-major layout and read as the MN-major B operand of the
// accumulating products through a descriptor with the other leading-dimension stride.
// TMEM: S^T[2] (64 cols each), dP^T[2], dV (128), dK (128).
constexpr int kBQ = 64;                   // query block of the dK/dV kernel
constexpr int kQdoBytes = 64 * 128 * 2;   // one 64-row Q or dO tile
constexpr int kPdsBytes = 128 * 64 * 2;   // one 128 x 64 P^T or dS^T tile
// shared memory: K, V, {Q, dO}[2], {P^T, dS^T}[2], LSE/D [2][2][64], barriers
constexpr int kBK_K = 0, kBK_V = kTileBytes, kBK_QDO = 2 * kTileBytes;
constexpr int kBK_PDS = kBK_QDO + 2 * 2 * kQdoBytes;
constexpr int kBK_LD = kBK_PDS + 2 * 2 * kPdsBytes;
constexpr int kBK_BAR = kBK_LD + 2 * 2 * 64 * 4;
constexpr int kBKSmem = 1024 + kBK_BAR + 256;

__global__ void __launch_bounds__(kFaThreads, 1)
    fa_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapDO,
                          const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapV,
                          const float* __restrict__ LSE, const float* __restrict__ Dv, const int* __restrict__ cu,
                          const int* __restrict__ cu_k, const int* __restrict__ q_off, bf16* __restrict__ dK,
                          bf16* __restrict__ dV, int T, int max_blocks, int Hq, int Hkv, float scale, int* err) {
  extern __shared__ __align__(1024) uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kBK_BAR);
  uint64_t* kv_full = bars;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;     // [2] S^T and dP^T of a block
  uint64_t* s_free = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;     // [2] P^T and dS^T of a block in shared memory
  uint64_t* p_free = bars + 11;    // [2]
  uint64_t* acc_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* ld_s = reinterpret_cast<float*>(sm + kBK_LD);  // [buf][LSE | D][64]

  // key tile kb of a causal document meets the query tiles from kb on, so low kb carries the most work:
  // CTAs are dispatched key-tile-major (every document's tile 0 first), the heaviest first, so the last wave
  // holds the light tiles
  const int n_docs = gridDim.x / max_blocks;
  const int doc = blockIdx.x % n_docs;
  const int kb = blockIdx.x / n_docs;
  const int hk = blockIdx.y, rep = Hq / Hkv;
  const int s = cu[doc], e = cu[doc + 1], L = e - s;
  const int ks = cu_k ? cu_k[doc] : s, ke = cu_k ? cu_k[doc + 1] : e, Lk = ke - ks;
  const int qo = q_off ? q_off[doc] : 0;
  const int k0 = kb * TBK;
  if (k0 >= Lk) return;
  // query blocks that see any key of this block: query q sees key k iff k <= qo + q
  const int n_qb = (L + kBQ - 1) / kBQ;
  const int qb0 = min(n_qb, max(0, k0 - qo) / kBQ);
  const int per_head = n_qb - qb0;
  const int n_blk = rep * per_head;  // (head, query block) pairs, head-major
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(acc_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapQ);
    tma_prefetch_desc(&mapDO);
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
  const uint32_t tmem = *tmem_slot;  // S^T[b] at 64 b, dP^T[b] at 128 + 64 b, dV at 256, dK at 384

  if (warp == 0) {
    // ───────────────────────────── TMA producer ─────────────────────────────
    if (lane == 0 && n_blk > 0) {
      mbar_arrive_expect_tx(kv_full, 2 * kTileBytes);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(sm + kBK_K + c * 16384, &mapK, kv_full, hk * THD + c * 64, ks + k0);
        tma_load_2d(sm + kBK_V + c * 16384, &mapV, kv_full, hk * THD + c * 64, ks + k0);
      }
      for (int n = 0; n < n_blk; ++n) {
        const int st = n & 1;
        const int h = hk * rep + n / per_head, qb = qb0 + n % per_head;
        if (!mbar_wait(&qdo_empty[st], ((n >> 1) & 1) ^ 1, abort_flag, err, 101)) break;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * kQdoBytes);
        uint8_t* dst = sm + kBK_QDO + st * 2 * kQdoBytes;
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(dst + c * 8192, &mapQ, &qdo_full[st], h * THD + c * 64, s + qb * kBQ);
          tma_load_2d(dst + kQdoBytes + c * 8192, &mapDO, &qdo_full[st], h * THD + c * 64, s + qb * kBQ);
        }
      }
    }
  } else if (warp == 1) {
    // ───────────────────────────── MMA issuer ───────────────────────────────
    if (lane == 0 && n_blk > 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(128, 64, false, false);   // K-major Q / dO as B
      constexpr uint32_t id_a = idesc_bf16_f32(128, 128, false, true);   // MN-major Q / dO as B
      const uint32_t sk = smem_u32(sm + kBK_K), sv = smem_u32(sm + kBK_V);
      bool ok = mbar_wait(kv_full, 0, abort_flag, err, 103);
      auto issue_s = [&](int n) -> bool {
        const int st = n & 1;
        if (!mbar_wait(&qdo_full[st], (n >> 1) & 1, abort_flag, err, 104)) return false;
        if (!mbar_wait(&s_free[st], ((n >> 1) & 1) ^ 1, abort_flag, err, 105)) return false;
        tc_fence_after();
        const uint32_t sq = smem_u32(sm + kBK_QDO + st * 2 * kQdoBytes), sdo = sq + kQdoBytes;
#pragma unroll
        for (int k = 0; k < THD / 16; ++k) {
          const uint32_t a_off = (k >> 2) * 16384 + (k & 3) * 32;
          const uint32_t b_off = (k >> 2) * 8192 + (k & 3) * 32;
          mma_bf16(tmem + st * 64, smem_desc_sw128(sk + a_off, 16, 1024), smem_desc_sw128(sq + b_off, 16, 1024), id_s,
                   k > 0 ? 1u : 0u);
          mma_bf16(tmem + 128 + st * 64, smem_desc_sw128(sv + a_off, 16, 1024), smem_desc_sw128(sdo + b_off, 16, 1024),
                   id_s, k > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n_blk > 1) ok = issue_s(1);
      for (int n = 0; n < n_blk && ok; ++n) {
        const int st = n & 1;
        if (!mbar_wait(&p_full[st], (n >> 1) & 1, abort_flag, err, 106)) break;
        tc_fence_after();
        const uint32_t sq = smem_u32(sm + kBK_QDO + st * 2 * kQdoBytes), sdo = sq + kQdoBytes;
        const uint32_t spt = smem_u32(sm + kBK_PDS + st * 2 * kPdsBytes), sdst = spt + kPdsBytes;
#pragma unroll
        for (int k = 0; k < kBQ / 16; ++k) {
          const uint32_t a_off = (k & 3) * 32;    // K-major P^T / dS^T: 64 queries = one 128-byte row
          const uint32_t b_off = (k & 3) * 2048;  // MN-major dO / Q: 16 query rows
          const uint32_t acc = (n > 0 || k > 0) ? 1u : 0u;
          mma_bf16(tmem + 256, smem_desc_sw128(spt + a_off, 16, 1024), smem_desc_sw128(sdo + b_off, 8192, 1024), id_a,
                   acc);
          mma_bf16(tmem + 384, smem_desc_sw128(sdst + a_off, 16, 1024), smem_desc_sw128(sq + b_off, 8192, 1024), id_a,
                   acc);
        }
        mma_commit(&p_free[st]);
        mma_commit(&qdo_empty[st]);
        if (n + 2 < n_blk) ok = issue_s(n + 2);
      }
      if (ok) mma_commit(acc_done);
    }
  } else {
    // ───────────────────────────── compute warps ────────────────────────────
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // key row of this thread = TMEM lane
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const float sl2 = scale * kL2e;
    const int key = k0 + r;
    const int ept = threadIdx.x - 64;  // 0..127
    bool ok = true;
    for (int n = 0; n < n_blk && ok; ++n) {
      const int st = n & 1;
      const int h = hk * rep + n / per_head, qb = qb0 + n % per_head;
      const int qrow0 = qb * kBQ;
      // LSE and D of the block's 64 queries (buffer st; the block two back has finished with it)
      float* lse_b = ld_s + st * 128;
      float* d_b = lse_b + 64;
      if (ept < 64) {
        const int q = qrow0 + ept;
        lse_b[ept] = q < L ? LSE[(size_t)h * T + s + q] * kL2e : INFINITY;
        d_b[ept] = q < L ? Dv[(size_t)h * T + s + q] : 0.f;
      }
      named_bar_sync(1, 128);
      ok = bar_and(1, 128, mbar_wait(&s_full[st], (n >> 1) & 1, abort_flag, err, 107));
      if (!ok) break;
      tc_fence_after();
      float sv[64], dp[64];
      tmem_ld32(t_lane + st * 64, sv);
      tmem_ld32(t_lane + st * 64 + 32, sv + 32);
      tmem_ld32(t_lane + 128 + st * 64, dp);
      tmem_ld32(t_lane + 128 + st * 64 + 32, dp + 32);
      tc_fence_before();
      mbar_arrive(&s_free[st]);
      // the products of the block two back must be done with this P^T / dS^T buffer
      if (n >= 2) {
        ok = bar_and(1, 128, mbar_wait(&p_free[st], ((n >> 1) & 1) ^ 1, abort_flag, err, 108));
        if (!ok) break;
      }
      // visible: key <= qo + q, key < Lk, q < L (q = qrow0 + c)
      const bool full = key < Lk && key <= qo + qrow0 && qrow0 + kBQ <= L;
      const int cmin = key - qo - qrow0;  // first visible column
      uint8_t* ptrow = sm + kBK_PDS + st * 2 * kPdsBytes + r * 128;
      uint8_t* dsrow = ptrow + kPdsBytes;
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        uint32_t pk[4], dk4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c0 = c + 2 * i;
          float p0 = ex2(fmaf(sv[c0], sl2, -lse_b[c0]));
          float p1 = ex2(fmaf(sv[c0 + 1], sl2, -lse_b[c0 + 1]));
          if (!full) {
            if (key >= Lk || c0 < cmin) p0 = 0.f;
            if (key >= Lk || c0 + 1 < cmin) p1 = 0.f;
          }
          pk[i] = pack_bf16x2(p0, p1);
          dk4[i] = pack_bf16x2(p0 * (dp[c0] - d_b[c0]), p1 * (dp[c0 + 1] - d_b[c0 + 1]));
        }
        const int chunk = c >> 3;
        const int off = (chunk ^ (r & 7)) << 4;
        *reinterpret_cast<uint4*>(ptrow + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(dsrow + off) = make_uint4(dk4[0], dk4[1], dk4[2], dk4[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&p_full[st]);
    }
    // epilogue: dV and scale * dK rows of this key
    if (ok && n_blk > 0) ok = bar_and(1, 128, mbar_wait(acc_done, 0, abort_flag, err, 109));
    if (ok) {
      // tcgen05.ld is warp-collective: every lane loads, only rows of real keys are stored
      tc_fence_after();
      const bool key_ok = key < Lk;
      bf16* dvrow = dV + ((size_t)(ks + key) * Hkv + hk) * THD;
      bf16* dkrow = dK + ((size_t)(ks + key) * Hkv + hk) * THD;
      for (int which = 0; which < 2; ++which) {
        bf16* dst = which ? dkrow : dvrow;
        const float mul = which ? scale : 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          if (n_blk > 0) {
            tmem_ld32(t_lane + 256 + which * 128 + c * 32, ov);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = 0.f;
          }
          if (key_ok) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(dst + c * 32 + i) = make_uint4(
                  pack_bf16x2(ov[i] * mul, ov[i + 1] * mul), pack_bf16x2(ov[i + 2] * mul, ov[i + 3] * mul),
                  pack_bf16x2(ov[i + 4] * mul, ov[i + 5] * mul), pack_bf16x2(ov[i + 6] * mul, ov[i + 7] * mul));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// dQ: one CTA per 128-query block of one head, sweeping the causal 64-key blocks:
//   S = Q K_j^T, dP = dO V_j^T                (M=128 queries, N=64 keys, K=128 dims)
//   dS = P (dP - D), P = 2^(S scale log2e - LSE log2e)            (thread = query row)
//   dQ += dS K_j                              (M=128 queries, N=128 dims, K=64 keys)
// TMEM: S[2] (64 cols), dP[2], dQ (128).
constexpr int kBKq = 64;                  // key block of the dQ kernel
constexpr int kKvBytes = 64 * 128 * 2;    // one 64-row K or V tile
constexpr int kDsBytes = 128 * 64 * 2;    // one 128 x 64 dS tile
constexpr int kDQ_Q = 0, kDQ_DO = kTileBytes, kDQ_KV = 2 * kTileBytes;
constexpr int kDQ_DS = kDQ_KV + 2 * 2 * kKvBytes;
constexpr int kDQ_BAR = kDQ_DS + 2 * kDsBytes;
constexpr int kDQSmem = 1024 + kDQ_BAR + 256;

__global__ void __launch_bounds__(kFaThreads, 1)
    fa_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapDO,
                        const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapV,
                        const float* __restrict__ LSE, const float* __restrict__ Dv, const int* __restrict__ cu,
                        const int* __restrict__ cu_k, const int* __restrict__ q_off, bf16* __restrict__ dQ, int T,
                        int max_blocks, int Hq, int Hkv, float scale, int* err) {
  extern __shared__ __align__(1024) uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kDQ_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;    // [2] dS in shared memory
  uint64_t* p_free = bars + 11;   // [2]
  uint64_t* acc_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int n_docs = gridDim.x / max_blocks;  // query-tile-major, longest causal rows first (as the forward)
  const int doc = blockIdx.x % n_docs;
  const int qb = max_blocks - 1 - blockIdx.x / n_docs;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int s = cu[doc], e = cu[doc + 1], L = e - s;
  const int ks = cu_k ? cu_k[doc] : s, ke = cu_k ? cu_k[doc + 1] : e, Lk = ke - ks;
  const int qo = q_off ? q_off[doc] : 0;
  const int q0 = qb * TBQ;
  if (q0 >= L) return;
  const int n_kb = max(0, min((Lk + kBKq - 1) / kBKq, (qo + q0 + TBQ - 1) / kBKq + 1));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(acc_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapQ);
    tma_prefetch_desc(&mapDO);
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
  const uint32_t tmem = *tmem_slot;  // S[b] at 64 b, dP[b] at 128 + 64 b, dQ at 256

  if (warp == 0) {
    if (lane == 0 && n_kb > 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(sm + kDQ_Q + c * 16384, &mapQ, q_full, h * THD + c * 64, s + q0);
        tma_load_2d(sm + kDQ_DO + c * 16384, &mapDO, q_full, h * THD + c * 64, s + q0);
      }
      for (int j = 0; j < n_kb; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, abort_flag, err, 111)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kKvBytes);
        uint8_t* dst = sm + kDQ_KV + st * 2 * kKvBytes;
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(dst + c * 8192, &mapK, &kv_full[st], hk * THD + c * 64, ks + j * kBKq);
          tma_load_2d(dst + kKvBytes + c * 8192, &mapV, &kv_full[st], hk * THD + c * 64, ks + j * kBKq);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_kb > 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(128, 64, false, false);
      constexpr uint32_t id_a = idesc_bf16_f32(128, 128, false, true);
      const uint32_t sq = smem_u32(sm + kDQ_Q), sdo = smem_u32(sm + kDQ_DO);
      bool ok = mbar_wait(q_full, 0, abort_flag, err, 113);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1, abort_flag, err, 114)) return false;
        if (!mbar_wait(&s_free[st], ((j >> 1) & 1) ^ 1, abort_flag, err, 115)) return false;
        tc_fence_after();
        const uint32_t skk = smem_u32(sm + kDQ_KV + st * 2 * kKvBytes), svv = skk + kKvBytes;
#pragma unroll
        for (int k = 0; k < THD / 16; ++k) {
          const uint32_t a_off = (k >> 2) * 16384 + (k & 3) * 32;
          const uint32_t b_off = (k >> 2) * 8192 + (k & 3) * 32;
          mma_bf16(tmem + st * 64, smem_desc_sw128(sq + a_off, 16, 1024), smem_desc_sw128(skk + b_off, 16, 1024), id_s,
                   k > 0 ? 1u : 0u);
          mma_bf16(tmem + 128 + st * 64, smem_desc_sw128(sdo + a_off, 16, 1024), smem_desc_sw128(svv + b_off, 16, 1024),
                   id_s, k > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n_kb > 1) ok = issue_s(1);
      for (int j = 0; j < n_kb && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&p_full[st], (j >> 1) & 1, abort_flag, err, 116)) break;
        tc_fence_after();
        const uint32_t skk = smem_u32(sm + kDQ_KV + st * 2 * kKvBytes);
        const uint32_t sds = smem_u32(sm + kDQ_DS + st * kDsBytes);
#pragma unroll
        for (int k = 0; k < kBKq / 16; ++k)
          mma_bf16(tmem + 256, smem_desc_sw128(sds + (k & 3) * 32, 16, 1024),
                   smem_desc_sw128(skk + (k & 3) * 2048, 8192, 1024), id_a, (j > 0 || k > 0) ? 1u : 0u);
        mma_commit(&p_free[st]);
        mma_commit(&kv_empty[st]);
        if (j + 2 < n_kb) ok = issue_s(j + 2);
      }
      if (ok) mma_commit(acc_done);
    }
  } else {
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // query row = TMEM lane
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const float sl2 = scale * kL2e;
    const int row = q0 + r;
    const bool row_ok = row < L;
    const int qpos = qo + row;
    const float lse2 = row_ok ? LSE[(size_t)h * T + s + row] * kL2e : INFINITY;
    const float dval = row_ok ? Dv[(size_t)h * T + s + row] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kb && ok; ++j) {
      const int st = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[st], (j >> 1) & 1, abort_flag, err, 117));
      if (!ok) break;
      tc_fence_after();
      float sv[64], dp[64];
      tmem_ld32(t_lane + st * 64, sv);
      tmem_ld32(t_lane + st * 64 + 32, sv + 32);
      tmem_ld32(t_lane + 128 + st * 64, dp);
      tmem_ld32(t_lane + 128 + st * 64 + 32, dp + 32);
      tc_fence_before();
      mbar_arrive(&s_free[st]);
      if (j >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&p_free[st], ((j >> 1) & 1) ^ 1, abort_flag, err, 118));
        if (!ok) break;
      }
      const int key0 = j * kBKq;
      const bool full = row_ok && key0 + kBKq - 1 <= qpos && key0 + kBKq <= Lk;
      const int lim = min(qpos + 1, Lk) - key0;  // visible keys [0, lim) of this block
      uint8_t* dsrow = sm + kDQ_DS + st * kDsBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        uint32_t d4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c0 = c + 2 * i;
          float p0 = ex2(fmaf(sv[c0], sl2, -lse2));
          float p1 = ex2(fmaf(sv[c0 + 1], sl2, -lse2));
          if (!full) {
            if (!row_ok || c0 >= lim) p0 = 0.f;
            if (!row_ok || c0 + 1 >= lim) p1 = 0.f;
          }
          d4[i] = pack_bf16x2(p0 * (dp[c0] - dval), p1 * (dp[c0 + 1] - dval));
        }
        *reinterpret_cast<uint4*>(dsrow + (((c >> 3) ^ (r & 7)) << 4)) = make_uint4(d4[0], d4[1], d4[2], d4[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&p_full[st]);
    }
    if (ok && n_kb > 0) ok = __all_sync(0xffffffffu, mbar_wait(acc_done, 0, abort_flag, err, 119));
    if (ok) {
      // tcgen05.ld is warp-collective: every lane loads, only rows of real queries are stored
      tc_fence_after();
      bf16* dqrow = dQ + ((size_t)(s + row) * Hq + h) * THD;
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
          for (int i = 0; i < 32; i += 8)
            *reinterpret_cast<uint4*>(dqrow + c * 32 + i) = make_uint4(
                pack_bf16x2(ov[i] * scale, ov[i + 1] * scale), pack_bf16x2(ov[i + 2] * scale, ov[i + 3] * scale),
                pack_bf16x2(ov[i + 4] * scale, ov[i + 5] * scale), pack_bf16x2(ov[i + 6] * scale, ov[i + 7] * scale));
        }
      }
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
  FaKV<1> kv{};
  kv.k[0] = make_map_bf16(k, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 128);
  kv.v[0] = make_map_bf16(v, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 64);
  static bool attr = false;
  if (!attr) {
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(fa_fwd_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem));
    attr = true;
  }
  dim3 grid(n_docs * mb, Hq);
  fa_fwd_tc_kernel<1><<<grid, kFaThreads, kFaSmem, st>>>(mq, kv, cu, cu_k, q_off, o, lse, T, mb, Hq, Hkv, scale, err);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

void flash_attn_fwd_tc_cp(const bf16* q, const bf16* const* k_ranks, const bf16* const* v_ranks, int cp, int rows,
                          int chunk, const int* cu, int n_docs, int docs_per_row, const int* q_off, bf16* o, float* lse,
                          int T, int max_seqlen, int Hq, int Hkv, float scale, cudaStream_t st, int* err) {
  MESHY_CHECK(Hq % Hkv == 0, "flash_attn_cp: Hq must be a multiple of Hkv");
  MESHY_CHECK(cp >= 1 && cp <= kFaMaxCp, "flash_attn_cp: 1 to 8 context-parallel ranks");
  MESHY_CHECK(chunk % TBK == 0, "flash_attn_cp: the chunk length must be a multiple of 128 tokens");
  const int mb = (max_seqlen + TBQ - 1) / TBQ;
  if (n_docs * mb == 0 || T == 0) return;
  CUtensorMap mq = make_map_bf16(q, T, (int64_t)Hq * THD, (int64_t)Hq * THD, 64, 128);
  FaKV<kFaMaxCp> kv{};
  const int64_t local = (int64_t)rows * 2 * chunk;
  for (int r = 0; r < cp; ++r) {
    kv.k[r] = make_map_bf16(k_ranks[r], local, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 128);
    kv.v[r] = make_map_bf16(v_ranks[r], local, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 64);
  }
  kv.cp = cp;
  kv.chunk = chunk;
  kv.seq = 2 * cp * chunk;
  kv.docs_per_row = docs_per_row;
  static bool attr = false;
  if (!attr) {
    MESHY_CUDA_CHECK(
        cudaFuncSetAttribute(fa_fwd_tc_kernel<kFaMaxCp>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem));
    attr = true;
  }
  dim3 grid(n_docs * mb, Hq);
  fa_fwd_tc_kernel<kFaMaxCp>
      <<<grid, kFaThreads, kFaSmem, st>>>(mq, kv, cu, nullptr, q_off, o, lse, T, mb, Hq, Hkv, scale, err);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy

namespace meshy {

void flash_attn_bwd_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* dout, const float* lse,
                       const float* dvec, const int* cu, int n_docs, bf16* dq, bf16* dk, bf16* dv, int T, int Tk,
                       int max_seqlen, int max_seqlen_k, int Hq, int Hkv, float scale, cudaStream_t st,
                       const int* cu_k, const int* q_off, int* err) {
  if (T == 0 || Tk == 0 || n_docs == 0) return;
  CUtensorMap mq128 = make_map_bf16(q, T, (int64_t)Hq * THD, (int64_t)Hq * THD, 64, 128);
  CUtensorMap mdo128 = make_map_bf16(dout, T, (int64_t)Hq * THD, (int64_t)Hq * THD, 64, 128);
  CUtensorMap mq64 = make_map_bf16(q, T, (int64_t)Hq * THD, (int64_t)Hq * THD, 64, 64);
  CUtensorMap mdo64 = make_map_bf16(dout, T, (int64_t)Hq * THD, (int64_t)Hq * THD, 64, 64);
  CUtensorMap mk128 = make_map_bf16(k, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 128);
  CUtensorMap mv128 = make_map_bf16(v, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 128);
  CUtensorMap mk64 = make_map_bf16(k, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 64);
  CUtensorMap mv64 = make_map_bf16(v, Tk, (int64_t)Hkv * THD, (int64_t)Hkv * THD, 64, 64);
  static bool attr = false;
  if (!attr) {
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(fa_bwd_dkdv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBKSmem));
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(fa_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDQSmem));
    attr = true;
  }
  const int mbk = ((cu_k ? max_seqlen_k : max_seqlen) + TBK - 1) / TBK;
  const int mbq = (max_seqlen + TBQ - 1) / TBQ;
  fa_bwd_dkdv_tc_kernel<<<dim3(n_docs * mbk, Hkv), kFaThreads, kBKSmem, st>>>(
      mq64, mdo64, mk128, mv128, lse, dvec, cu, cu_k, q_off, dk, dv, T, mbk, Hq, Hkv, scale, err);
  MESHY_CUDA_CHECK(cudaGetLastError());
  fa_bwd_dq_tc_kernel<<<dim3(n_docs * mbq, Hq), kFaThreads, kDQSmem, st>>>(
      mq128, mdo128, mk64, mv64, lse, dvec, cu, cu_k, q_off, dq, T, mbq, Hq, Hkv, scale, err);
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
