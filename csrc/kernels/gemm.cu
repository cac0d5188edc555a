// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M, N] = op(A)[M, K] · op(B)[N, K]^T      (bf16 in, fp32 accumulate in TMEM)
//
// op(A) is K-major ([M, K] row-major) or MN-major ([K, M] row-major); same for B
// with [N, K] / [K, N].  That covers forward (TN), dgrad (B MN-major) and wgrad
// (both MN-major) without transposing anything in memory.
//
// Roles (192 threads):
//   warp 0   — TMA producer: 128-byte-swizzled tiles of A (128 x 64) and B
//              (BN x 64) into a STAGES-deep shared-memory ring;
//   warp 1   — allocates TMEM (2 accumulators x BN fp32 columns) and issues
//              tcgen05.mma (M=128, N=BN, K=16) from one thread; tcgen05.commit
//              frees smem stages and publishes finished accumulators;
//   warps 2-5 — epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//              lanes 32*(w%4)..+31), fused epilogue, global stores.
// The two TMEM accumulators let the epilogue of tile i overlap the MMAs of
// tile i+1.  Work units (m-tile, n-tile, k-split) are strided over a grid of
// at most one CTA per SM.
//
// Fused epilogues:
//   STORE    out = acc (+bias[n]) (+residual[m,n]), bf16 or fp32; with split-K
//            the partials go through an fp32 workspace and the last CTA of a
//            tile applies the epilogue (and re-zeroes the workspace);
//   SWIGLU   gate/up columns interleaved in blocks of 64: out = silu(g)*u,
//            optional store of the pre-activation for backward;
//   ACC_F32  out_f32 += acc (weight-gradient accumulation);
//   LSE      per (row, n-tile) partials of log-sum-exp, sum p*z, target logit
//            and a Gumbel-max sample (fused LM-head log-prob / sampler);
//   DLOGITS  dz = g_row * (onehot(label) - exp(z - lse_row)), bf16.
//
// Every mbarrier wait is bounded (sm100.cuh): a stuck pipeline sets an error
// code in ``err`` and the CTA returns after releasing its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "gemm.h"

namespace meshy {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int A_TILE_BYTES = BM * BK * 2;

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks, split_k, kb_per_split, total_units;
  int epi;
  void* out;
  int ldo;
  int out_f32;
  const bf16* bias;
  const bf16* residual;
  int ldr;
  bf16* aux;
  int ld_aux;
  float* ws;
  int* counters;
  const int64_t* labels;
  float* partial;
  const float* row_lse;
  const float* row_g;
  float inv_temp;
  uint64_t seed;
  const int64_t* step_ptr;
  int gumbel;
  int* err;
  // 1: the epilogue stages each 128-row x 128-byte slice of the tile in shared memory and writes it with one
  // TMA store (bf16 output; SwiGLU output and pre-activations) or TMA reduce-add (fp32 accumulation), so
  // the global writes are whole lines instead of one 16-byte piece per row and lane
  int tma_out;
  // grouped problems (mixture-of-experts): grp_off[0..grp_n] are device row offsets, multiples of 128, of
  // each group's segment of the token rows. GRP_M: the segment rows of A are multiplied by the group's own
  // B (a 3-D tensor map, group = outermost coordinate); units past grp_off[grp_n] are skipped. GRP_K: the
  // contraction runs over the group's segment rows (A and B MN-major) into output rows
  // [g * grp_rows, (g + 1) * grp_rows); empty groups are skipped.
  const int* grp_off;
  int grp_n;
  int grp_mode;
  int grp_rows;
};

template <int BN>
struct Cfg {
  static constexpr int B_TILE_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int STG_BYTES = BM * 128;  // one epilogue staging buffer: 128 rows x 128 bytes
  static constexpr int STG_OFF = STAGES * STAGE_BYTES + 1024;  // after the barriers, 1024-aligned for the swizzle
  static constexpr int SMEM_BYTES = 1024 /*align*/ + STG_OFF + 2 * STG_BYTES;
};

// Named barrier 1 over the four epilogue warps with an AND of ``v``: every thread gets the same answer.
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// ─── epilogue through shared memory + TMA store ─────────────────────────────
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               :
               : "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];"
               :
               : "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}

// The four epilogue warps write one 128 x 128-byte slice (row r = TMEM lane, 128-byte swizzle) into staging
// buffer ``sb`` and one thread sends it with a TMA store (or reduce-add) at (c0, r0). A buffer is reused two
// slices later, after the store that read it has finished reading.
struct Stager {
  uint8_t* stg;
  int sb;
  template <bool REDUCE>
  __device__ __forceinline__ void put(const uint4* row16, int r, const CUtensorMap* map, int c0, int r0, int et) {
    if (et == 0) bulk_wait_read1();
    named_bar_sync(1, 128);
    uint8_t* buf = stg + sb * (BM * 128);
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(buf + r * 128 + ((j ^ (r & 7)) << 4)) = row16[j];
    fence_async_smem();
    named_bar_sync(1, 128);
    if (et == 0) {
      if (REDUCE) tma_reduce_add_2d(map, buf, c0, r0);
      else tma_store_2d(map, buf, c0, r0);
      bulk_commit();
    }
    sb ^= 1;
  }
};

__device__ __forceinline__ void unit_coords(const GemmArgs& p, int u, int& mt, int& nt, int& ks) {
  ks = u % p.split_k;
  int t = u / p.split_k;
  // grouped raster: 8 m-tiles per group walk the n dimension together (L2 reuse of B)
  constexpr int G = 8;
  int group = t / (G * p.n_tiles);
  int first_m = group * G;
  int gm = min(G, p.m_tiles - first_m);
  int r = t - group * G * p.n_tiles;
  mt = first_m + r % gm;
  nt = r / gm;
}

// One work unit of a CTA: its tile, its k-block range, the first output row, and (grouped) its group.
struct Unit {
  int mt, nt, ks, kb0, kb1, row0, grp;
};

// Every role of the CTA resolves units the same way and skips the same ones (no work: a grouped problem
// is launched for its largest possible size).
__device__ __forceinline__ bool resolve_unit(const GemmArgs& p, int u, Unit& w) {
  if (p.grp_mode == GRP_K) {
    const int per = p.m_tiles * p.n_tiles;
    w.grp = u / per;
    const int r = u - w.grp * per;
    w.mt = r % p.m_tiles;
    w.nt = r / p.m_tiles;
    w.ks = 0;
    w.kb0 = p.grp_off[w.grp] / BK;
    w.kb1 = p.grp_off[w.grp + 1] / BK;
    w.row0 = w.grp * p.grp_rows + w.mt * BM;
    return w.kb1 > w.kb0;
  }
  unit_coords(p, u, w.mt, w.nt, w.ks);
  w.kb0 = w.ks * p.kb_per_split;
  w.kb1 = min(p.k_blocks, w.kb0 + p.kb_per_split);
  w.row0 = w.mt * BM;
  w.grp = 0;
  if (p.grp_mode == GRP_M) {
    if (w.row0 >= p.grp_off[p.grp_n]) return false;
    // owner of rows [row0, row0 + 128): the last group whose segment starts at or before row0 (segments are
    // 128-aligned, so a tile never spans two groups; empty groups before it share its start)
    int lo = 0, hi = p.grp_n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.grp_off[mid] <= w.row0) lo = mid;
      else hi = mid - 1;
    }
    w.grp = lo;
  }
  return true;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapAux, GemmArgs p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapA);
    tma_prefetch_desc(&mapB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ───────────────────────────── TMA producer ─────────────────────────────
    if (lane == 0) {
      pdl_wait();  // the A operand comes from the kernel before
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0, last_stage = 0;
      uint32_t last_phase = 0;
      for (int u = blockIdx.x; u < p.total_units && !*abort_flag; u += gridDim.x) {
        Unit w;
        if (!resolve_unit(p, u, w)) continue;
        const int mt = w.mt, nt = w.nt;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + A_TILE_BYTES;
          if (!A_MN) {
            tma_load_2d(sa, &mapA, &full[stage], kb * BK, mt * BM);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(sa + j * 8192, &mapA, &full[stage], mt * BM + 64 * j, kb * BK);
          }
          if (p.grp_mode == GRP_M) {
            if (!B_MN) {
              tma_load_3d(sb, &mapB, &full[stage], kb * BK, nt * BN, w.grp);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_3d(sb + j * 8192, &mapB, &full[stage], nt * BN + 64 * j, kb * BK, w.grp);
            }
          } else if (!B_MN) {
            tma_load_2d(sb, &mapB, &full[stage], kb * BK, nt * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &mapB, &full[stage], nt * BN + 64 * j, kb * BK);
          }
          issued++;
          last_stage = stage;
          last_phase = phase;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag && issued) {
        // let the copies already in flight land before the CTA can exit
        long long t0 = clock64();
        while (!mbar_try_wait(&full[last_stage], last_phase) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ───────────────────────────── MMA issuer ───────────────────────────────
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
      if (p.grp_mode) pdl_wait();  // the group offsets come from the kernel before
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool any = false;
      for (int u = blockIdx.x; u < p.total_units && !*abort_flag; u += gridDim.x) {
        Unit w;
        if (!resolve_unit(p, u, w)) continue;
        const int kb0 = w.kb0, kb1 = w.kb1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + A_TILE_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad, bd;
            if (!A_MN) ad = smem_desc_sw128(sa + k * 32, 16, 1024);
            else ad = smem_desc_sw128(sa + k * 2048, 8192, 1024);
            if (!B_MN) bd = smem_desc_sw128(sb + k * 32, 16, 1024);
            else bd = smem_desc_sw128(sb + k * 2048, 8192, 1024);
            mma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          any = true;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (any) {
        // all MMAs retired before TMEM can be released
        mma_commit(drain);
        long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ───────────────────────────── epilogue ─────────────────────────────────
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    const int et = threadIdx.x - 64;  // 0..127
    Stager stager{smem + C::STG_OFF, 0};
    pdl_wait();  // residual / labels / workspace may come from the kernels before
    pdl_trigger();
    for (int u = blockIdx.x; u < p.total_units; u += gridDim.x) {
      Unit w_;
      if (!resolve_unit(p, u, w_)) continue;
      const int mt = w_.mt, nt = w_.nt;
      const int r0 = w_.row0;  // first output row of the tile
      if (!epi_all(mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue))) break;
      tc_fence_after();
      const int row = r0 + q * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      const int n0 = nt * BN;
      float v[32];

      if (p.tma_out && p.epi == EPI_ACC_F32) {
        // fp32 accumulation: 32-column slices, reduce-added by TMA
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(t_row + c * 32, v);
          if (n0 + c * 32 >= p.N) break;  // uniform over the warps
          uint4 r16[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            r16[j] = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]), __float_as_uint(v[4 * j + 2]),
                                __float_as_uint(v[4 * j + 3]));
          stager.put<true>(r16, q * 32 + lane, &mapC, n0 + c * 32, r0, et);
        }
      } else if (p.tma_out && p.epi == EPI_STORE) {
        // bf16 output: 64-column slices (+bias, +residual), stored by TMA (rows >= M / columns >= N clipped)
        for (int c = 0; c < BN / 64; ++c) {
          float w[64];
          tmem_ld32(t_row + c * 64, w);
          tmem_ld32(t_row + c * 64 + 32, w + 32);
          const int col0 = n0 + c * 64;
          if (col0 >= p.N) break;  // uniform over the warps
          const int ncol = min(64, p.N - col0);
          if (p.bias) {
#pragma unroll
            for (int i = 0; i < 64; ++i) w[i] += (i < ncol) ? __bfloat162float(p.bias[col0 + i]) : 0.f;
          }
          if (p.residual && row_ok) {
            const bf16* rr = p.residual + (size_t)row * p.ldr + col0;
            if (ncol == 64) {
#pragma unroll
              for (int i = 0; i < 64; i += 8) {
                uint4 x = *reinterpret_cast<const uint4*>(rr + i);
                float2 a0 = unpack_bf16x2(x.x), a1 = unpack_bf16x2(x.y), a2 = unpack_bf16x2(x.z),
                       a3 = unpack_bf16x2(x.w);
                w[i] += a0.x; w[i + 1] += a0.y; w[i + 2] += a1.x; w[i + 3] += a1.y;
                w[i + 4] += a2.x; w[i + 5] += a2.y; w[i + 6] += a3.x; w[i + 7] += a3.y;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 64; ++i)
                if (i < ncol) w[i] += __bfloat162float(rr[i]);
            }
          }
          uint4 r16[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            r16[j] = make_uint4(pack_bf16x2(w[8 * j], w[8 * j + 1]), pack_bf16x2(w[8 * j + 2], w[8 * j + 3]),
                                pack_bf16x2(w[8 * j + 4], w[8 * j + 5]), pack_bf16x2(w[8 * j + 6], w[8 * j + 7]));
          stager.put<false>(r16, q * 32 + lane, &mapC, col0, r0, et);
        }
      } else if (p.tma_out && p.epi == EPI_DLOGITS) {
        // d logits = g * (onehot(label) - softmax), 64-column slices stored by TMA
        const float lse = row_ok ? p.row_lse[row] : 0.f;
        const float gr = row_ok ? p.row_g[row] : 0.f;
        const int64_t label = row_ok ? p.labels[row] : -1;
        for (int c = 0; c < BN / 64; ++c) {
          float w[64];
          tmem_ld32(t_row + c * 64, w);
          tmem_ld32(t_row + c * 64 + 32, w + 32);
          const int col0 = n0 + c * 64;
          if (col0 >= p.N) break;  // uniform over the warps
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const float pr = __expf(w[i] - lse);
            w[i] = gr * (((int64_t)(col0 + i) == label ? 1.f : 0.f) - pr);
          }
          uint4 r16[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            r16[j] = make_uint4(pack_bf16x2(w[8 * j], w[8 * j + 1]), pack_bf16x2(w[8 * j + 2], w[8 * j + 3]),
                                pack_bf16x2(w[8 * j + 4], w[8 * j + 5]), pack_bf16x2(w[8 * j + 6], w[8 * j + 7]));
          stager.put<false>(r16, q * 32 + lane, &mapC, col0, r0, et);
        }
      } else if (p.tma_out && p.epi == EPI_SWIGLU) {
        // columns [128j, 128j+64) are gate, [128j+64, 128j+128) the matching up rows -> 64 SwiGLU columns
        for (int j = 0; j < BN / 128; ++j) {
          const int gcol = n0 + j * 128;
          if (gcol >= p.N) break;  // uniform over the warps
          uint4 act[8], hg[8], hu[8];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float g[32];
            tmem_ld32(t_row + j * 128 + h * 32, g);
            tmem_ld32(t_row + j * 128 + 64 + h * 32, v);
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float a[8];
#pragma unroll
              for (int t = 0; t < 8; ++t) {
                // round the pre-activations to bf16 first so forward and the
                // backward recompute (from the stored bf16 h) agree exactly
                float gg = __bfloat162float(__float2bfloat16(g[i + t]));
                float uu = __bfloat162float(__float2bfloat16(v[i + t]));
                a[t] = silu(gg) * uu;
              }
              act[h * 4 + i / 8] = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                                              pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
              hg[h * 4 + i / 8] = make_uint4(pack_bf16x2(g[i], g[i + 1]), pack_bf16x2(g[i + 2], g[i + 3]),
                                             pack_bf16x2(g[i + 4], g[i + 5]), pack_bf16x2(g[i + 6], g[i + 7]));
              hu[h * 4 + i / 8] = make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                                             pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
            }
          }
          stager.put<false>(act, q * 32 + lane, &mapC, n0 / 2 + j * 64, r0, et);
          if (p.aux) {
            stager.put<false>(hg, q * 32 + lane, &mapAux, gcol, r0, et);
            stager.put<false>(hu, q * 32 + lane, &mapAux, gcol + 64, r0, et);
          }
        }
      } else if (p.epi == EPI_STORE || p.epi == EPI_ACC_F32) {
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(t_row + c * 32, v);
          const int col0 = n0 + c * 32;
          if (!row_ok || col0 >= p.N) continue;
          const int ncol = min(32, p.N - col0);
          if (p.split_k > 1 && p.epi == EPI_STORE) {
            float* w = p.ws + (size_t)row * p.N + col0;
            if (ncol == 32 && (p.N % 4) == 0) {
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                atomicAdd(reinterpret_cast<float4*>(w + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
            } else {
              for (int i = 0; i < ncol; ++i) atomicAdd(w + i, v[i]);
            }
            continue;
          }
          if (p.epi == EPI_ACC_F32) {
            float* o = reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + col0;
            if (p.split_k > 1) {
              if (ncol == 32 && (p.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                  atomicAdd(reinterpret_cast<float4*>(o + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
              } else {
                for (int i = 0; i < ncol; ++i) atomicAdd(o + i, v[i]);
              }
            } else if (ncol == 32 && (p.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0) {
#pragma unroll
              for (int i = 0; i < 32; i += 4) {
                float4 x = *reinterpret_cast<float4*>(o + i);
                x.x += v[i]; x.y += v[i + 1]; x.z += v[i + 2]; x.w += v[i + 3];
                *reinterpret_cast<float4*>(o + i) = x;
              }
            } else {
              for (int i = 0; i < ncol; ++i) o[i] += v[i];
            }
            continue;
          }
          if (p.bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += (i < ncol) ? __bfloat162float(p.bias[col0 + i]) : 0.f;
          }
          if (p.residual) {
            const bf16* r = p.residual + (size_t)row * p.ldr + col0;
            if (ncol == 32) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 x = *reinterpret_cast<const uint4*>(r + i);
                float2 a0 = unpack_bf16x2(x.x), a1 = unpack_bf16x2(x.y), a2 = unpack_bf16x2(x.z),
                       a3 = unpack_bf16x2(x.w);
                v[i] += a0.x; v[i + 1] += a0.y; v[i + 2] += a1.x; v[i + 3] += a1.y;
                v[i + 4] += a2.x; v[i + 5] += a2.y; v[i + 6] += a3.x; v[i + 7] += a3.y;
              }
            } else {
              for (int i = 0; i < ncol; ++i) v[i] += __bfloat162float(r[i]);
            }
          }
          if (p.out_f32) {
            float* o = reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + col0;
            for (int i = 0; i < ncol; ++i) o[i] = v[i];
          } else {
            bf16* o = reinterpret_cast<bf16*>(p.out) + (size_t)row * p.ldo + col0;
            if (ncol == 32) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 x = make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                                     pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
                *reinterpret_cast<uint4*>(o + i) = x;
              }
            } else {
              for (int i = 0; i < ncol; ++i) o[i] = __float2bfloat16(v[i]);
            }
          }
        }
      } else if (p.epi == EPI_SWIGLU) {
        // columns [128j, 128j+64) are gate, [128j+64, 128j+128) the matching up rows
        for (int j = 0; j < BN / 128; ++j) {
          for (int h = 0; h < 2; ++h) {
            float g[32];
            tmem_ld32(t_row + j * 128 + h * 32, g);
            tmem_ld32(t_row + j * 128 + 64 + h * 32, v);
            const int gcol = n0 + j * 128 + h * 32;
            if (!row_ok || gcol >= p.N) continue;
            const int ocol = n0 / 2 + j * 64 + h * 32;
            bf16* o = reinterpret_cast<bf16*>(p.out) + (size_t)row * p.ldo + ocol;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float a[8];
#pragma unroll
              for (int t = 0; t < 8; ++t) {
                // round the pre-activations to bf16 first so forward and the
                // backward recompute (from the stored bf16 h) agree exactly
                float gg = __bfloat162float(__float2bfloat16(g[i + t]));
                float uu = __bfloat162float(__float2bfloat16(v[i + t]));
                a[t] = silu(gg) * uu;
              }
              *reinterpret_cast<uint4*>(o + i) = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                                                            pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
            }
            if (p.aux) {
              bf16* hg = p.aux + (size_t)row * p.ld_aux + gcol;
              bf16* hu = hg + 64;
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                *reinterpret_cast<uint4*>(hg + i) =
                    make_uint4(pack_bf16x2(g[i], g[i + 1]), pack_bf16x2(g[i + 2], g[i + 3]),
                               pack_bf16x2(g[i + 4], g[i + 5]), pack_bf16x2(g[i + 6], g[i + 7]));
                *reinterpret_cast<uint4*>(hu + i) =
                    make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                               pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
              }
            }
          }
        }
      } else if (p.epi == EPI_LSE) {
        float m = -INFINITY, s = 0.f, pz = 0.f, tgt = 0.f, best = -INFINITY, bestz = 0.f;
        int besti = -1;
        const int64_t label = (row_ok && p.labels) ? p.labels[row] : -1;
        const uint64_t step = p.step_ptr ? (uint64_t)*p.step_ptr : 0ull;
        const uint2 key = make_uint2((uint32_t)p.seed, (uint32_t)(p.seed >> 32) ^ (uint32_t)step);
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(t_row + c * 32, v);
          const int col0 = n0 + c * 32;
          float cm = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = (col0 + i < p.N) ? v[i] * p.inv_temp : -INFINITY;
            cm = fmaxf(cm, v[i]);
          }
          if (cm > m) {
            float sc = __expf(m - cm);
            s *= sc;
            pz *= sc;
            m = cm;
          }
          if (m == -INFINITY) continue;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float e = __expf(v[i] - m);
            s += e;
            pz += (v[i] == -INFINITY) ? 0.f : e * v[i];
          }
          if (label >= col0 && label < col0 + 32) tgt = v[label - col0];
          if (p.gumbel) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              uint4 r = Philox::gen(make_uint4((uint32_t)(col0 + i), (uint32_t)row, (uint32_t)(step >> 32), 0x5A3Du),
                                    key);
              uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                float z = v[i + t];
                if (z == -INFINITY) continue;
                float gsc = z + gumbel(rr[t]);
                if (gsc > best) {
                  best = gsc;
                  besti = col0 + i + t;
                  bestz = z;
                }
              }
            }
          }
        }
        if (row_ok) {
          float* o = p.partial + ((size_t)row * p.n_tiles + nt) * 8;
          *reinterpret_cast<float4*>(o) = make_float4(m, s, pz, tgt);
          *reinterpret_cast<float4*>(o + 4) = make_float4(best, bestz, __int_as_float(besti), 0.f);
        }
      } else if (p.epi == EPI_DLOGITS) {
        const float lse = row_ok ? p.row_lse[row] : 0.f;
        const float g = row_ok ? p.row_g[row] : 0.f;
        const int64_t label = row_ok ? p.labels[row] : -1;
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(t_row + c * 32, v);
          const int col0 = n0 + c * 32;
          if (!row_ok || col0 >= p.N) continue;
          const int ncol = min(32, p.N - col0);
          bf16* o = reinterpret_cast<bf16*>(p.out) + (size_t)row * p.ldo + col0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float pr = __expf(v[i] - lse);
            v[i] = g * (((int64_t)(col0 + i) == label ? 1.f : 0.f) - pr);
          }
          if (ncol == 32) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(o + i) = make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                                                            pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
          } else {
            for (int i = 0; i < ncol; ++i) o[i] = __float2bfloat16(v[i]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }

      if (p.split_k > 1 && p.epi == EPI_STORE) {
        // last CTA to finish this tile applies the epilogue from the workspace
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          int tile = mt * p.n_tiles + nt;
          int prev = atomicAdd(&p.counters[tile], 1);
          *last_flag = (prev == p.split_k - 1) ? 1 : 0;
          if (*last_flag) p.counters[tile] = 0;
          __threadfence();
        }
        named_bar_sync(1, 128);
        if (*last_flag && row_ok) {
          // the whole row slice is read with independent 16-byte loads before anything is
          // written back, so the fix-up costs a few L2 round trips, not one per column
          for (int col0 = n0; col0 < min(n0 + BN, p.N); col0 += 32) {
            const int ncol = min(32, p.N - col0);
            float* w = p.ws + (size_t)row * p.N + col0;
            const bool vec = ncol == 32 && (p.N % 4) == 0;
            if (vec) {
#pragma unroll
              for (int i = 0; i < 32; i += 4) {
                float4 x = __ldcg(reinterpret_cast<const float4*>(w + i));
                v[i] = x.x; v[i + 1] = x.y; v[i + 2] = x.z; v[i + 3] = x.w;
              }
#pragma unroll
              for (int i = 0; i < 32; i += 4) __stcg(reinterpret_cast<float4*>(w + i), make_float4(0.f, 0.f, 0.f, 0.f));
            } else {
              for (int i = 0; i < ncol; ++i) v[i] = __ldcg(w + i);
              for (int i = 0; i < ncol; ++i) __stcg(w + i, 0.f);
            }
            if (p.bias)
              for (int i = 0; i < ncol; ++i) v[i] += __bfloat162float(p.bias[col0 + i]);
            if (p.residual)
              for (int i = 0; i < ncol; ++i) v[i] += __bfloat162float(p.residual[(size_t)row * p.ldr + col0 + i]);
            if (p.out_f32) {
              float* o = reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + col0;
              for (int i = 0; i < ncol; ++i) o[i] = v[i];
            } else {
              bf16* o = reinterpret_cast<bf16*>(p.out) + (size_t)row * p.ldo + col0;
              if (vec && (p.ldo % 8) == 0) {
#pragma unroll
                for (int i = 0; i < 32; i += 8)
                  *reinterpret_cast<uint4*>(o + i) =
                      make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                                 pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
              } else {
                for (int i = 0; i < ncol; ++i) o[i] = __float2bfloat16(v[i]);
              }
            }
          }
        }
        named_bar_sync(1, 128);
      }
    }
    if (p.tma_out && et == 0) bulk_wait_all();  // staged stores complete before the CTA leaves
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ════════════════════════════════ host side ══════════════════════════════════

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESHY_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    MESHY_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    MESHY_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  int64_t rows, cols, ld;
  int bi, bo;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && bi == o.bi && bo == o.bo;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = reinterpret_cast<size_t>(k.ptr);
    h ^= (size_t)k.rows * 0x9E3779B97F4A7C15ull + (size_t)k.cols * 0xC2B2AE3D27D4EB4Full + (size_t)k.ld +
         ((size_t)k.bi << 40) + ((size_t)k.bo << 50);
    return h;
  }
};

// 2-D bf16 row-major [rows, cols] (row stride ld elements), box {bi, bo}, 128B swizzle.
CUtensorMap make_map_bf16(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int bi, int bo) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{ptr, rows, cols, ld, bi, bo};
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  MESHY_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base address must be 16-byte aligned");
  MESHY_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)bi, (cuuint32_t)bo};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MESHY_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, map);
  return map;
}

// 3-D bf16 [d2][d1][d0] (d0 contiguous; strides of d1 and d2 in bytes), box {b0, b1, 1}, 128B swizzle.
// Used for per-layer weight matrices that sit at a uniform stride in one flat buffer.
CUtensorMap make_map_bf16_3d(const void* ptr, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes,
                             int64_t stride2_bytes, int b0, int b1) {
  MESHY_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base address must be 16-byte aligned");
  MESHY_CHECK(stride1_bytes % 16 == 0 && stride2_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)stride1_bytes, (cuuint64_t)stride2_bytes};
  cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MESHY_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed (" + std::to_string((int)r) + ")");
  return map;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    MESHY_CUDA_CHECK(cudaGetDevice(&dev));
    MESHY_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN>
static void launch_t(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mx,
                     const GemmArgs& a, int grid, cudaStream_t st) {
  using C = Cfg<BN>;
  auto k = gemm_kernel<BN, A_MN, B_MN>;
  static bool attr_set = false;
  if (!attr_set) {
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    attr_set = true;
  }
  launch_pdl(k, dim3(grid), dim3(kThreads), C::SMEM_BYTES, st, ma, mb, mc, mx, a);
}

template <int BN>
static void launch_bn(bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                      const CUtensorMap& mx, const GemmArgs& a, int grid, cudaStream_t st) {
  if (!a_mn && !b_mn) launch_t<BN, false, false>(ma, mb, mc, mx, a, grid, st);
  else if (!a_mn && b_mn) launch_t<BN, false, true>(ma, mb, mc, mx, a, grid, st);
  else if (a_mn && !b_mn) launch_t<BN, true, false>(ma, mb, mc, mx, a, grid, st);
  else launch_t<BN, true, true>(ma, mb, mc, mx, a, grid, st);
}

// fp32 [rows, cols] (row stride ld elements), box {bi, bo}, 128-byte swizzle: TMA reduce-add target.
static CUtensorMap make_map_f32(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int bi, int bo) {
  MESHY_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (ld * 4) % 16 == 0, "TMA: 16-byte aligned rows");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)bi, (cuuint32_t)bo};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MESHY_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp32) failed (" + std::to_string((int)r) + ")");
  return map;
}

static bool gemm_tma_out_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESHY_GEMM_TMA_OUT");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

static void gemm_grouped_launch(const GemmProblem& g, cudaStream_t stream);

void gemm_launch(const GemmProblem& g, cudaStream_t stream) {
  MESHY_CHECK(g.M > 0 && g.N > 0 && g.K > 0, "empty GEMM");
  if (g.grp_mode != GRP_NONE) {
    gemm_grouped_launch(g, stream);
    return;
  }
  if (g.force_bn == 0 && gemm_small_eligible(g)) {
    gemm_small_launch(g, stream);
    return;
  }
  // the epilogue writes 16-byte vectors of a row (and reads the residual that way)
  MESHY_CHECK((reinterpret_cast<uintptr_t>(g.out) & 15) == 0 && (g.ldo * (g.out_f32 ? 4 : 2)) % 16 == 0,
              "gemm: output rows must start on 16-byte boundaries");
  MESHY_CHECK(!g.residual || ((reinterpret_cast<uintptr_t>(g.residual) & 15) == 0 && (g.ldr * 2) % 16 == 0),
              "gemm: residual rows must start on 16-byte boundaries");
  int BN = g.force_bn;
  const int sms = num_sms();
  const int m_tiles = (g.M + BM - 1) / BM;
  if (BN == 0) {
    if (g.epi == EPI_SWIGLU) BN = 256;
    else if (m_tiles * ((g.N + 255) / 256) >= sms && g.N >= 256) BN = 256;
    else if (g.N >= 128) BN = 128;
    else BN = 64;
  }
  MESHY_CHECK(g.epi != EPI_SWIGLU || (g.N % 128 == 0), "SwiGLU GEMM needs N % 128 == 0");
  GemmArgs a{};
  a.M = g.M; a.N = g.N; a.K = g.K;
  a.m_tiles = m_tiles;
  a.n_tiles = (g.N + BN - 1) / BN;
  a.k_blocks = (g.K + BK - 1) / BK;
  int split = 1;
  const int tiles = a.m_tiles * a.n_tiles;
  if ((g.epi == EPI_STORE && g.ws != nullptr) || g.epi == EPI_ACC_F32) {
    // (splitting weight-gradient GEMMs further, to fill whole waves of the persistent grid, measured no
    // faster on the 1.5B training step: 3086 vs 3083 ms)
    if (tiles * 2 <= sms && a.k_blocks >= 4) {
      split = std::min(a.k_blocks / 2, (sms + tiles - 1) / tiles);
      split = std::max(1, std::min(split, 32));
    }
  }
  if (g.max_split > 0) split = std::min(split, g.max_split);
  a.kb_per_split = (a.k_blocks + split - 1) / split;
  a.split_k = (a.k_blocks + a.kb_per_split - 1) / a.kb_per_split;
  a.total_units = tiles * a.split_k;
  a.epi = g.epi;
  a.out = g.out; a.ldo = g.ldo; a.out_f32 = g.out_f32;
  a.bias = g.bias; a.residual = g.residual; a.ldr = g.ldr;
  a.aux = g.aux; a.ld_aux = g.ld_aux;
  a.ws = g.ws; a.counters = g.counters;
  MESHY_CHECK(a.split_k == 1 || g.epi != EPI_STORE || (g.ws && g.counters &&
                                                        (int64_t)a.m_tiles * a.n_tiles <= g.counters_cap &&
                                                        (int64_t)g.M * g.N <= g.ws_cap),
              "split-K workspace too small");
  a.labels = g.labels; a.partial = g.partial; a.row_lse = g.row_lse; a.row_g = g.row_g;
  a.inv_temp = g.inv_temp; a.seed = g.seed; a.step_ptr = g.step_ptr; a.gumbel = g.gumbel;
  a.err = g.err;
  // tensor maps: K-major operand [rows, K] box {64, rows_box}; MN-major [K, mn] box {64, 64}
  CUtensorMap ma = g.a_mn ? make_map_bf16(g.A, g.K, g.M, g.lda, 64, 64) : make_map_bf16(g.A, g.M, g.K, g.lda, 64, BM);
  CUtensorMap mb = g.b_mn ? make_map_bf16(g.B, g.K, g.N, g.ldb, 64, 64) : make_map_bf16(g.B, g.N, g.K, g.ldb, 64, BN);
  // TMA-store epilogue: 128-row x 128-byte slices of the output (and of the SwiGLU pre-activations)
  CUtensorMap mc = ma, mx = ma;
  a.tma_out = 0;
  if (gemm_tma_out_enabled() && (a.split_k == 1 || g.epi == EPI_ACC_F32)) {
    const bool aux_ok = g.aux == nullptr || ((reinterpret_cast<uintptr_t>(g.aux) & 15) == 0 && (g.ld_aux * 2) % 16 == 0);
    if (g.epi == EPI_STORE && !g.out_f32 && g.aux == nullptr) {
      mc = make_map_bf16(g.out, g.M, g.N, g.ldo, 64, BM);
      a.tma_out = 1;
    } else if (g.epi == EPI_ACC_F32) {
      mc = make_map_f32(g.out, g.M, g.N, g.ldo, 32, BM);
      a.tma_out = 1;
    } else if (g.epi == EPI_DLOGITS && !g.out_f32) {
      mc = make_map_bf16(g.out, g.M, g.N, g.ldo, 64, BM);
      a.tma_out = 1;
    } else if (g.epi == EPI_SWIGLU && !g.out_f32 && aux_ok) {
      mc = make_map_bf16(g.out, g.M, g.N / 2, g.ldo, 64, BM);
      if (g.aux) mx = make_map_bf16(g.aux, g.M, g.N, g.ld_aux, 64, BM);
      a.tma_out = 1;
    }
  }
  int grid = std::min(a.total_units, sms);
  switch (BN) {
    case 256: launch_bn<256>(g.a_mn, g.b_mn, ma, mb, mc, mx, a, grid, stream); break;
    case 128: launch_bn<128>(g.a_mn, g.b_mn, ma, mb, mc, mx, a, grid, stream); break;
    default: launch_bn<64>(g.a_mn, g.b_mn, ma, mb, mc, mx, a, grid, stream); break;
  }
}

// Grouped problems: one persistent launch sized for the largest possible row count; the group offsets are
// read on the device, so nothing here waits for the routing.
static void gemm_grouped_launch(const GemmProblem& g, cudaStream_t stream) {
  MESHY_CHECK(g.grp_off != nullptr && g.grp_n > 0, "grouped GEMM: group offsets missing");
  MESHY_CHECK((reinterpret_cast<uintptr_t>(g.out) & 15) == 0 && (g.ldo * (g.out_f32 ? 4 : 2)) % 16 == 0,
              "grouped GEMM: output rows must start on 16-byte boundaries");
  MESHY_CHECK(g.bias == nullptr && g.residual == nullptr, "grouped GEMM: no bias / residual epilogue");
  const int sms = num_sms();
  GemmArgs a{};
  a.N = g.N;
  a.K = g.K;
  a.grp_off = g.grp_off;
  a.grp_n = g.grp_n;
  a.grp_mode = g.grp_mode;
  a.epi = g.epi;
  a.out = g.out; a.ldo = g.ldo; a.out_f32 = g.out_f32;
  a.aux = g.aux; a.ld_aux = g.ld_aux;
  a.err = g.err;
  a.split_k = 1;
  int BN = g.force_bn;
  CUtensorMap ma, mb, mc, mx;
  if (g.grp_mode == GRP_M) {
    MESHY_CHECK(!g.a_mn && g.M % BM == 0, "GRP_M: A K-major with a row count padded to 128");
    MESHY_CHECK(g.epi == EPI_STORE || g.epi == EPI_SWIGLU, "GRP_M: store or SwiGLU epilogue");
    MESHY_CHECK(!g.out_f32, "GRP_M: bf16 output");
    if (BN == 0) BN = (g.epi == EPI_SWIGLU || g.N >= 256) ? 256 : (g.N >= 128 ? 128 : 64);
    MESHY_CHECK(g.epi != EPI_SWIGLU || g.N % 128 == 0, "GRP_M SwiGLU: N % 128 == 0");
    MESHY_CHECK(g.N % BN == 0 || g.epi == EPI_STORE, "GRP_M: N must be a multiple of the tile width");
    a.M = g.M;
    a.m_tiles = g.M / BM;
    a.n_tiles = (g.N + BN - 1) / BN;
    a.k_blocks = (g.K + BK - 1) / BK;
    a.kb_per_split = a.k_blocks;
    a.total_units = a.m_tiles * a.n_tiles;
    ma = make_map_bf16(g.A, g.M, g.K, g.lda, 64, BM);
    MESHY_CHECK((g.grp_stride * 2) % 16 == 0 && (g.ldb * 2) % 16 == 0, "GRP_M: B strides must be 16-byte multiples");
    if (!g.b_mn)  // B_g = [N, K] row-major (row stride ldb), groups grp_stride apart
      mb = make_map_bf16_3d(g.B, g.K, g.N, g.grp_n, g.ldb * 2, g.grp_stride * 2, 64, BN);
    else          // B_g = [K, N] row-major
      mb = make_map_bf16_3d(g.B, g.N, g.K, g.grp_n, g.ldb * 2, g.grp_stride * 2, 64, 64);
    mc = mx = ma;
    a.tma_out = 0;
    if (gemm_tma_out_enabled()) {
      const bool aux_ok = g.aux == nullptr || ((reinterpret_cast<uintptr_t>(g.aux) & 15) == 0 && (g.ld_aux * 2) % 16 == 0);
      if (g.epi == EPI_STORE) {
        mc = make_map_bf16(g.out, g.M, g.N, g.ldo, 64, BM);
        a.tma_out = 1;
      } else if (aux_ok) {
        mc = make_map_bf16(g.out, g.M, g.N / 2, g.ldo, 64, BM);
        if (g.aux) mx = make_map_bf16(g.aux, g.M, g.N, g.ld_aux, 64, BM);
        a.tma_out = 1;
      }
    }
  } else {
    MESHY_CHECK(g.grp_mode == GRP_K && g.a_mn && g.b_mn, "GRP_K: A and B MN-major (token rows as K)");
    MESHY_CHECK(g.epi == EPI_ACC_F32 && g.out_f32, "GRP_K: fp32 accumulation");
    MESHY_CHECK(g.M % BM == 0, "GRP_K: rows per group must be a multiple of 128");
    if (BN == 0) BN = g.N >= 256 ? 256 : (g.N >= 128 ? 128 : 64);
    a.M = g.M * g.grp_n;
    a.grp_rows = g.M;
    a.m_tiles = g.M / BM;
    a.n_tiles = (g.N + BN - 1) / BN;
    a.k_blocks = (g.K + BK - 1) / BK;
    a.kb_per_split = a.k_blocks;
    a.total_units = g.grp_n * a.m_tiles * a.n_tiles;
    ma = make_map_bf16(g.A, g.K, g.M, g.lda, 64, 64);
    mb = make_map_bf16(g.B, g.K, g.N, g.ldb, 64, 64);
    mx = ma;
    a.tma_out = gemm_tma_out_enabled() ? 1 : 0;
    mc = a.tma_out ? make_map_f32(g.out, (int64_t)g.M * g.grp_n, g.N, g.ldo, 32, BM) : ma;
  }
  const int grid = std::min(a.total_units, sms);
  switch (BN) {
    case 256: launch_bn<256>(g.a_mn, g.b_mn, ma, mb, mc, mx, a, grid, stream); break;
    case 128: launch_bn<128>(g.a_mn, g.b_mn, ma, mb, mc, mx, a, grid, stream); break;
    default: launch_bn<64>(g.a_mn, g.b_mn, ma, mb, mc, mx, a, grid, stream); break;
  }
}

int gemm_n_tiles(int N, int bn) { return (N + bn - 1) / bn; }

}  // namespace meshy
