// Whole-step persistent decode kernel for dense decoders on sm_100a.
//
// At decode batch sizes every linear streams its weights once and is bound by
// HBM; run as ~9 kernels per layer the step is dominated by per-kernel ramp
// and drain (each launch re-fills the memory pipeline from empty). Here one
// cooperative launch of one CTA per SM runs the whole step as a sequence of
// phases separated by grid barriers:
//
//   EMBED | per layer: QKV, ATTN, OPROJ, GATEUP, DOWN | FINAL
//
// and the weight stream never stops: the TMA producer of every CTA walks the
// whole step's schedule and loads the NEXT phase's weight tiles into free
// ring stages while the current phase is still computing. Only the small
// activation tiles (and the KV pages) wait for the grid barrier.
//
// Roles (192 threads): warp 0 lane 0 = TMA producer; warp 1 = TMEM allocator
// and single-thread tcgen05.mma issuer; warps 2-5 = epilogue (thread f owns
// TMEM lane / weight row f of a tile) and, in the attention phase, the four
// consumer warps.
//
// GEMMs use swapped operands: MMA M = 128 weight rows, MMA N = MP padded
// tokens, fp32 accumulators in TMEM (two buffers). Each phase's T tiles x KB
// k-blocks are split s ways along K so that T*s items cover the SMs; partial
// sums go to fp32 global accumulators with vector atomics and the last CTA to
// finish a tile (a counter per tile) finalises it:
//   QKV    bias, RoPE (+ QK-norm), q -> q buffer, k/v -> paged KV cache;
//   OPROJ  residual stream x += o_proj(attn): round to bf16, write the next
//          norm's input xg = bf16(x * gain) and add the per-row sum of squares;
//   GATEUP SwiGLU -> act (directly from TMEM when the phase is not split);
//   DOWN   like OPROJ, for the next layer's attention norm (or the final norm).
// RMSNorm is thereby split into a sum of squares accumulated by the producer
// of x and a per-row scale rstd applied in the consumer's epilogue:
//   W (g * x) * rstd  ==  W (RMSNorm(x)),  rstd = 1 / sqrt(mean(x^2) + eps).
//
// Attention is stream-K over (row, KV head, 64-token page) units: the units
// of all running rows are dealt out in equal contiguous ranges, each CTA keeps
// one online-softmax state per contiguous piece, pieces of a row/head that
// span several CTAs are merged by the last of them (a counter per row/head).
// K/V pages arrive by TMA; scores and P.V use m16n8k16 MMAs with the GQA
// query heads of one KV head as the 16 rows.
//
// Every wait is bounded (mbarriers, tile/piece counters, grid barriers): on a
// timeout the kernel records an error code, every CTA gives up at its next
// wait, and the host reads the code and resets the counters.
#include <cuda.h>

#include <cmath>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "decode_mega.h"
#include "gemm.h"

namespace meshy {

namespace {

constexpr int kThreads = 192;
constexpr int kStages = 5;
constexpr int kStageBytes = 32768;                 // W tile (16 KB) + X tile (<= 8 KB), or K + V page
constexpr int kWBytes = 128 * 64 * 2;              // 128 rows x 64 k bf16
constexpr int kRingBytes = kStages * kStageBytes;  // 160 KB
constexpr int kMergeFloats = 128 + 4 * 16 * 128;   // attention merge (also finaliser scratch)
constexpr int kMergeBytes = kMergeFloats * 4;
constexpr int kQsBytes = 16 * 128 * 2;
constexpr int kMaxSeg = kMegaMaxRows * 8;          // rows x KV heads
constexpr int kSegBytes = (kMaxSeg + 8) * 4;
constexpr int kMiscBytes = 1280;  // barriers, flags, rstd[64], pos[64], slot[64]
constexpr int kSmemBytes = 1024 + kRingBytes + kMergeBytes + kQsBytes + kSegBytes + kMiscBytes;
constexpr int kPartRow = kMegaHeadDim + 4;  // o[128], m, l, pad (rows of whole float4s)

enum Kind : int { K_EMBED = 0, K_QKV, K_ATTN, K_O, K_GU, K_DN, K_FINAL };

__device__ __forceinline__ int phase_kind(int p, int L) {
  if (p == 0) return K_EMBED;
  if (p == 1 + 5 * L) return K_FINAL;
  return K_QKV + (p - 1) % 5;
}
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float round_bf(float v) { return __bfloat162float(__float2bfloat16(v)); }
__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void fence_proxy_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }


// Arrive on the grid barrier (one thread per CTA, after the CTA's writes of the phase are fenced).
__device__ __forceinline__ void gbar_arrive(unsigned* bar) {
  __threadfence();
  fence_proxy_global();
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

__device__ __noinline__ void record_timeout(unsigned* dbg, int site, int cta, int p, int x, int y);
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until ``target`` CTAs arrived: one thread per CTA polls with relaxed loads and a short
// back-off, then an acquire fence orders the data reads that follow. Gives up (false) after
// kWaitCycles, when the CTA aborted, or when any CTA recorded an error.
__device__ bool gbar_wait(const unsigned* bar, unsigned target, volatile int* abort, int* err, unsigned* dbg) {
  long long t0 = clock64();
  int spins = 0;
  while ((int)(ld_relaxed(bar) - target) < 0) {
    __nanosleep(32);
    if (*abort) return false;
    if ((++spins & 63) == 0) {
      if (*reinterpret_cast<volatile int*>(err)) {
        *abort = 1;
        return false;
      }
      if (clock64() - t0 > kWaitCycles) {
        *abort = 1;
        atomicCAS(err, 0, (int)kErrTimeoutPeer);
        record_timeout(dbg, 16, (int)blockIdx.x, (int)target, (int)threadIdx.x, (int)ld_relaxed(bar));
        return false;
      }
    }
  }
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  fence_proxy_global();
  return true;
}

// Where a wait gave up: the first CTA to time out records (site, cta, phase, x, y, barrier count) in
// words [8, 14) after the grid barrier, for the host to read back.
__device__ __noinline__ void record_timeout(unsigned* dbg, int site, int cta, int p, int x, int y) {
  if (atomicCAS(dbg, 0u, (unsigned)site) == 0u) {
    dbg[1] = (unsigned)cta;
    dbg[2] = (unsigned)p;
    dbg[3] = (unsigned)x;
    dbg[4] = (unsigned)y;
    dbg[5] = *reinterpret_cast<volatile unsigned*>(dbg - 8);
    __threadfence();
  }
}

// mbar_wait that also records the site of its own timeout.
__device__ __forceinline__ bool mwait(uint64_t* b, uint32_t phase, volatile int* abort, int* err, int code,
                                      unsigned* dbg, int site, int cta, int p, int x) {
  if (mbar_try_wait(b, phase)) return true;
  long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(b, phase)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort = 1;
      atomicCAS(err, 0, code);
      record_timeout(dbg, site, cta, p, x, (int)phase);
      return false;
    }
  }
}

// Element offset of (row r, column c) in a [64, 128] bf16 tile stored as two 128-byte-swizzled
// [64][64] boxes (the TMA SWIZZLE_128B layout).
__device__ __forceinline__ int sw128(int r, int c) {
  return (c >> 6) * (64 * 64) + r * 64 + ((((c & 63) >> 3) ^ (r & 7)) << 3) + (c & 7);
}
__device__ __forceinline__ void ldsm4(uint32_t* d, const bf16* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm4t(uint32_t* d, const bf16* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Named barrier with an AND-reduction of ``v`` over the participating threads: every thread gets
// the same answer, so a decision to stop is taken by all of them together (no thread left waiting
// at a later barrier for one that stopped).
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

struct Sched {
  // stream-K attention schedule, identical in every role of every CTA
  int U;       // total units
  int n_att;   // CTAs that take attention units
  const int* seg;  // [n_seg + 1] unit prefix over (row, KV head)
  int n_seg;
  __device__ int range(int c) const { return (int)((long long)c * U / n_att); }
  __device__ int cta_of(int u) const { return (int)(((long long)(u + 1) * n_att + U - 1) / U) - 1; }
};

struct Gsel {
  MegaGemm g;
  const CUtensorMap* mw;
  const CUtensorMap* mx;
  int K;  // row length of the weight (elements)
};

__device__ __forceinline__ Gsel gemm_of(int kind, const MegaArgs& a, const CUtensorMap* mq, const CUtensorMap* mo,
                                        const CUtensorMap* mg, const CUtensorMap* md, const CUtensorMap* mxg,
                                        const CUtensorMap* mao, const CUtensorMap* mact) {
  if (kind == K_QKV) return {a.g_qkv, mq, mxg, a.D};
  if (kind == K_O) return {a.g_o, mo, mao, a.q_dim};
  if (kind == K_GU) return {a.g_gu, mg, mxg, a.D};
  return {a.g_dn, md, mact, a.F};
}

// k-block of the j-th stage of an item. The start is rotated per item so that concurrent CTAs read
// different column ranges of their weight rows (all CTAs sweeping the same offset of rows a few KB
// apart concentrate the traffic on a few memory channels).
__device__ __forceinline__ int kb_at(int item, int kb0, int kb1, int j) {
  const int nk = kb1 - kb0;
  return kb0 + (j + item * 5) % nk;
}

__device__ __forceinline__ void item_range(const MegaGemm& g, int item, int& tile, int& kb0, int& kb1) {
  tile = item / g.s;
  const int r = item % g.s;
  kb0 = r * g.KB / g.s;
  kb1 = (r + 1) * g.KB / g.s;
}

// Row [0, B) of a [*, MP] fp32 workspace (L2, written by other CTAs) into registers, float4 at a time.
template <int MP>
__device__ __forceinline__ void ldcg_row(const float* p, float* v, int B) {
#pragma unroll
  for (int t = 0; t < MP; t += 4) {
    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < B) q = __ldcg(reinterpret_cast<const float4*>(p + t));
    v[t] = q.x;
    v[t + 1] = q.y;
    v[t + 2] = q.z;
    v[t + 3] = q.w;
  }
}
template <int MP>
__device__ __forceinline__ void stcg_row(float* p, const float* v, int B) {
#pragma unroll
  for (int t = 0; t < MP; t += 4)
    if (t < B) __stcg(reinterpret_cast<float4*>(p + t), make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]));
}
template <int MP>
__device__ __forceinline__ void zero_row(float* p, int B) {
#pragma unroll
  for (int t = 0; t < MP; t += 4)
    if (t < B) __stcg(reinterpret_cast<float4*>(p + t), make_float4(0.f, 0.f, 0.f, 0.f));
}

template <int MP>
__device__ __forceinline__ void tmem_load_row(uint32_t taddr, float* v) {
#pragma unroll
  for (int c = 0; c < MP; c += 16) tmem_ld16(taddr + c, v + c);
}

template <int MP>
__global__ void __launch_bounds__(kThreads, 1)
    mega_decode_kernel(const __grid_constant__ CUtensorMap m_qkv, const __grid_constant__ CUtensorMap m_o,
                       const __grid_constant__ CUtensorMap m_gu, const __grid_constant__ CUtensorMap m_dn,
                       const __grid_constant__ CUtensorMap m_xg, const __grid_constant__ CUtensorMap m_ao,
                       const __grid_constant__ CUtensorMap m_act, const __grid_constant__ CUtensorMap m_kv,
                       const MegaArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* merge = reinterpret_cast<float*>(ring + kRingBytes);
  bf16* Qs = reinterpret_cast<bf16*>(ring + kRingBytes + kMergeBytes);
  int* seg = reinterpret_cast<int*>(ring + kRingBytes + kMergeBytes + kQsBytes);
  uint8_t* misc = ring + kRingBytes + kMergeBytes + kQsBytes + kSegBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_flag = abort_flag + 1;
  volatile int* passed_s = abort_flag + 2;  // highest grid barrier this CTA's poller has seen complete
  float* rstd_s = reinterpret_cast<float*>(misc + 256);      // [64]
  int* pos_s = reinterpret_cast<int*>(misc + 512);           // [64] positions of this step's tokens
  int64_t* slot_s = reinterpret_cast<int64_t*>(misc + 768);  // [64] their KV-cache slots

  constexpr uint32_t kTmemCols = MP * 2 < 32 ? 32 : MP * 2;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n = gridDim.x, c = blockIdx.x;
  const int L = a.n_layers;
  const int n_ph = 2 + 5 * L;
  unsigned* bar = a.ctr + kMegaCtrTiles + kMegaCtrAttn;
  unsigned* exit_ctr = bar + 1;
  unsigned* dbg = bar + 8;
  unsigned* tile_ctr = a.ctr;
  unsigned* attn_ctr = a.ctr + kMegaCtrTiles;
  const int rep = a.Hq / a.Hkv;

  if (threadIdx.x == 0) {
    // A stage is released by two arrivals: its consumer (tcgen05.commit of the MMA warp for weight
    // stages, the attention warps for KV pages) and the role that skips it (the epilogue group for
    // weight stages, the MMA warp for KV pages). A role that skipped stages without observing them
    // could fall two mbarrier phases behind, and a parity wait would then match a stale phase.
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    *abort_flag = 0;
    *passed_s = -1;
    fence_mbar_init();
    tma_prefetch_desc(&m_qkv);
    tma_prefetch_desc(&m_o);
    tma_prefetch_desc(&m_gu);
    tma_prefetch_desc(&m_dn);
    tma_prefetch_desc(&m_xg);
    tma_prefetch_desc(&m_ao);
    tma_prefetch_desc(&m_act);
    tma_prefetch_desc(&m_kv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  for (int t = threadIdx.x; t < a.B; t += kThreads) {
    pos_s[t] = a.pos[t];
    slot_s[t] = a.slot[t];
  }
  // stream-K attention schedule: unit prefix over (row, KV head) segments
  const int n_seg = a.B * a.Hkv;
  for (int s = threadIdx.x; s < n_seg; s += kThreads) {
    const int Ls = a.seq_lens[s / a.Hkv];
    seg[s + 1] = (Ls + kMegaPage - 1) / kMegaPage;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    seg[0] = 0;
    for (int s = 0; s < n_seg; ++s) seg[s + 1] += seg[s];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  Sched sc;
  sc.U = seg[n_seg];
  // about four 64-token pages per attention CTA: more CTAs stream the cache faster, fewer merge in
  // fewer pieces
  sc.n_att = max(1, min(n, (sc.U + 3) / 4));
  sc.seg = seg;
  sc.n_seg = n_seg;

  if (warp == 0) {
    // ─────────────────────────────── TMA producer ───────────────────────────────
    if (lane == 0) {
      int stage = 0;
      uint32_t eph = 0;
      int passed = -1;  // highest grid barrier known complete
      struct Pend {
        int stage, kind, c0, c1, bar;
        const CUtensorMap* map;
      };
      Pend pend[kStages];
      int np = 0;
      int last_stage = -1;
      uint32_t last_phase = 0;
      int cur_p = 0;
      bool ok = true;
      auto wait_bar = [&](int k) -> bool {
        // the epilogue group's poller publishes each completed grid barrier in shared memory
        if (k <= passed) return true;
        long long t0 = clock64();
        while (*passed_s < k) {
          __nanosleep(64);
          if (*abort_flag) return false;
          if (clock64() - t0 > kWaitCycles) {
            *abort_flag = 1;
            atomicCAS(a.err, 0, (int)kErrTimeoutProducer);
            record_timeout(dbg, 19, c, k, *passed_s, 0);
            return false;
          }
        }
        __threadfence_block();
        fence_proxy_global();
        passed = k;
        return true;
      };
      auto issue = [&](const Pend& q) {
        uint8_t* dst = ring + q.stage * kStageBytes;
        if (q.kind == K_ATTN) {
          // c0 = K row, c1 = V row of the page in the [rows, 128] cache view
          tma_load_2d(dst, &m_kv, &full[q.stage], 0, q.c0);
          tma_load_2d(dst + 8192, &m_kv, &full[q.stage], 64, q.c0);
          tma_load_2d(dst + 16384, &m_kv, &full[q.stage], 0, q.c1);
          tma_load_2d(dst + 16384 + 8192, &m_kv, &full[q.stage], 64, q.c1);
        } else {
          tma_load_2d(dst + kWBytes, q.map, &full[q.stage], q.c0, 0);
        }
      };
      auto flush = [&]() -> bool {
        for (int i = 0; i < np; ++i) {
          if (!wait_bar(pend[i].bar)) return false;
          issue(pend[i]);
        }
        np = 0;
        return true;
      };
      auto next_stage = [&]() -> bool {
        // issue parked X / page loads as soon as their barrier has passed (one poll, no wait)
        if (np && *passed_s >= pend[0].bar) {
          if (!flush()) return false;
        }
        if (np && !mbar_try_wait(&empty[stage], eph ^ 1)) {
          if (!flush()) return false;
        }
        return mwait(&empty[stage], eph ^ 1, abort_flag, a.err, kErrTimeoutProducer, dbg, 11, c, cur_p, stage);
      };
      auto advance = [&]() {
        last_stage = stage;
        last_phase = eph;
        if (++stage == kStages) {
          stage = 0;
          eph ^= 1;
        }
      };
      for (int p = 0; p < n_ph && ok; ++p) {
        const int kind = phase_kind(p, L);
        const int layer = (p - 1) / 5;
        cur_p = p;
        if (kind == K_QKV || kind == K_O || kind == K_GU || kind == K_DN) {
          const Gsel gs = gemm_of(kind, a, &m_qkv, &m_o, &m_gu, &m_dn, &m_xg, &m_ao, &m_act);
          for (int item = c; item < gs.g.T * gs.g.s && ok; item += n) {
            int tile, kb0, kb1;
            item_range(gs.g, item, tile, kb0, kb1);
            for (int j = 0; j < kb1 - kb0; ++j) {
              const int kb = kb_at(item, kb0, kb1, j);
              if (!next_stage()) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&full[stage], kWBytes + MP * 128);
              tma_load_3d(ring + stage * kStageBytes, gs.mw, &full[stage], kb * 64, tile * 128, layer);
              Pend q{stage, kind, kb * 64, 0, p - 1, gs.mx};
              if (p - 1 <= passed && np == 0)
                issue(q);
              else
                pend[np++] = q;
              advance();
            }
          }
        } else if (kind == K_ATTN && c < sc.n_att) {
          const int u0 = sc.range(c), u1 = sc.range(c + 1);
          int s = 0;
          while (s < n_seg && sc.seg[s + 1] <= u0) ++s;
          for (int u = u0; u < u1 && ok; ++u) {
            while (sc.seg[s + 1] <= u) ++s;
            const int b = s / a.Hkv, hk = s % a.Hkv;
            const int pi = u - sc.seg[s];
            const int pg = a.block_table[(size_t)b * a.max_pages + pi];
            const int rowk = (((layer * 2 + 0) * a.n_cache_pages + pg) * a.Hkv + hk) * kMegaPage;
            const int rowv = (((layer * 2 + 1) * a.n_cache_pages + pg) * a.Hkv + hk) * kMegaPage;
            if (!next_stage()) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], 4 * 8192);
            Pend q{stage, K_ATTN, rowk, rowv, p - 1, nullptr};
            if (p - 1 <= passed && np == 0)
              issue(q);
            else
              pend[np++] = q;
            advance();
          }
        }
      }
      if (ok) ok = flush();
      if (!ok && last_stage >= 0) {
        // let loads already issued land before the CTA exits
        long long t0 = clock64();
        while (!mbar_try_wait(&full[last_stage], last_phase) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ─────────────────────────────── MMA issuer ─────────────────────────────────
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, MP, false, false);
      int stage = 0;
      uint32_t fph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int p = 0; p < n_ph && ok; ++p) {
        const int kind = phase_kind(p, L);
        if (kind == K_QKV || kind == K_O || kind == K_GU || kind == K_DN) {
          const Gsel gs = gemm_of(kind, a, &m_qkv, &m_o, &m_gu, &m_dn, &m_xg, &m_ao, &m_act);
          for (int item = c; item < gs.g.T * gs.g.s && ok; item += n) {
            int tile, kb0, kb1;
            item_range(gs.g, item, tile, kb0, kb1);
            if (!mwait(&tempty[acc], aph ^ 1, abort_flag, a.err, kErrTimeoutMma, dbg, 12, c, p, acc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * MP;
            for (int j = 0; j < kb1 - kb0; ++j) {
              if (!mwait(&full[stage], fph, abort_flag, a.err, kErrTimeoutMma, dbg, 13, c, p, stage)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t sw = smem_u32(ring + stage * kStageBytes);
              const uint32_t sx = sw + kWBytes;
#pragma unroll
              for (int k = 0; k < 4; ++k)
                mma_bf16(d_tmem, smem_desc_sw128(sw + k * 32, 16, 1024), smem_desc_sw128(sx + k * 32, 16, 1024),
                         idesc, (j > 0 || k > 0) ? 1u : 0u);
              mma_commit(&empty[stage]);
              if (++stage == kStages) {
                stage = 0;
                fph ^= 1;
              }
            }
            if (!ok) break;
            mma_commit(&tfull[acc]);
            if (++acc == 2) {
              acc = 0;
              aph ^= 1;
            }
          }
        } else if (kind == K_ATTN && c < sc.n_att) {
          // the attention warps consume these stages; observe each one land and release our share
          const int cnt = sc.range(c + 1) - sc.range(c);
          for (int i = 0; i < cnt && ok; ++i) {
            if (!mwait(&full[stage], fph, abort_flag, a.err, kErrTimeoutMma, dbg, 17, c, p, stage)) {
              ok = false;
              break;
            }
            mbar_arrive(&empty[stage]);
            if (++stage == kStages) {
              stage = 0;
              fph ^= 1;
            }
          }
        }
      }
    }
  } else {
    // ──────────────────────── epilogue / attention warps ─────────────────────────
    const int wq = warp & 3;
    const int f = wq * 32 + lane;  // TMEM lane = weight row within a tile
    const uint32_t t_lane = tmem_base + ((uint32_t)(wq * 32) << 16);
    int stage = 0;
    uint32_t fph = 0;
    int acc = 0;
    uint32_t aph = 0;
    bool ok = true;
    auto sync_epi = [&]() { named_bar_sync(1, 128); };
    auto phase_wait = [&](int k) -> bool {
      // grid barrier k complete (one thread spins, the others wait at the named barrier)
      bool r = true;
      if (f == 0) {
        r = gbar_wait(bar, (unsigned)((k + 1) * n), abort_flag, a.err, dbg);
        if (r) *passed_s = k;
      }
      return bar_and(1, 128, r && !*abort_flag);
    };
    auto load_rstd = [&](int which) {
      if (f < MP) {
        const float s2 = f < a.B ? __ldcg(a.sumsq + which * MP + f) : 0.f;
        rstd_s[f] = rsqrtf(s2 / (float)a.D + a.eps);
      }
      sync_epi();
    };
    // last of the s contributors of counter ``ctr``? (every thread of the epilogue group calls this)
    auto last_arrival = [&](unsigned* ctr, unsigned expected) -> bool {
      sync_epi();
      if (f == 0) {
        __threadfence();
        const unsigned old = atomicAdd(ctr, 1u);
        *s_flag = (old == expected - 1) ? 1 : 0;
        if (old == expected - 1) *ctr = 0;  // reset for the next phase that uses it
      }
      sync_epi();
      const bool last = *s_flag != 0;
      if (last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
      return last;
    };

    for (int p = 0; p < n_ph && ok; ++p) {
      const int kind = phase_kind(p, L);
      const int layer = (p - 1) / 5;
      if (p > 0 && !phase_wait(p - 1)) {
        ok = false;
        break;
      }
      if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8] = gtimer();
      if (kind == K_EMBED) {
        if (c < a.B) {
          const int t = c;
          const int64_t id = a.tok[t];
          const bf16* g0 = a.layers[0].attn_norm;
          float ss = 0.f;
          for (int n0 = 0; n0 < a.D; n0 += 128 * 16) {
            // sixteen independent row loads in flight per thread, then the stores
            float ev[16], gv[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int nn = n0 + u * 128 + f;
              ev[u] = nn < a.D ? bf2f(a.embed[(size_t)id * a.D + nn]) : 0.f;
              gv[u] = nn < a.D ? bf2f(g0[nn]) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int nn = n0 + u * 128 + f;
              if (nn < a.D) {
                a.x[(size_t)nn * MP + t] = ev[u];
                a.xg[(size_t)t * a.D + nn] = __float2bfloat16(ev[u] * gv[u]);
                ss += ev[u] * ev[u];
              }
            }
          }
          ss = warp_sum(ss);
          if (lane == 0) merge[wq] = ss;
          sync_epi();
          if (f == 0) a.sumsq[t] = merge[0] + merge[1] + merge[2] + merge[3];
        } else if (c == n - 1) {
          if (f < MP) a.sumsq[MP + f] = 0.f;
        }
      } else if (kind == K_FINAL) {
        load_rstd(0);
        const bf16* gF = a.final_norm;
        for (int i0 = c * 128 + f; i0 < a.B * a.D; i0 += n * 128 * 8) {
          float xv[8], gv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int idx = i0 + u * n * 128;
            xv[u] = 0.f;
            gv[u] = 0.f;
            if (idx < a.B * a.D) {
              const int t = idx / a.D, nn = idx % a.D;
              xv[u] = __ldcg(a.x + (size_t)nn * MP + t);
              gv[u] = bf2f(gF[nn]);
            }
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int idx = i0 + u * n * 128;
            if (idx < a.B * a.D) a.h[idx] = __float2bfloat16(xv[u] * rstd_s[idx / a.D] * gv[u]);
          }
        }
      } else if (kind == K_ATTN) {
        if (c == 0 && f < MP) a.sumsq[MP + f] = 0.f;  // MLP-norm sums of this layer start from zero
        if (c < sc.n_att) {
          const int u0 = sc.range(c), u1 = sc.range(c + 1);
          int s = 0;
          while (s < n_seg && sc.seg[s + 1] <= u0) ++s;
          const MegaLayer& lay = a.layers[layer];
          (void)lay;
          uint32_t qf[8][4];
          float o[16][4];
          float m_r[2], l_r[2];
          int L_b = 0;
          for (int u = u0; u < u1 && ok; ++u) {
            while (sc.seg[s + 1] <= u) ++s;
            const int b = s / a.Hkv, hk = s % a.Hkv;
            const int pi = u - sc.seg[s];
            const bool first = (u == u0) || (u == sc.seg[s]);
            const bool lastu = (u == u1 - 1) || (u == sc.seg[s + 1] - 1);
            if (first) {
              L_b = a.seq_lens[b];
              sync_epi();  // previous piece's ldmatrix reads of Qs are done
              uint4 qv[2];
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2) {
                const int i = f + h2 * 128, r = i / 16, cc = (i % 16) * 8;
                qv[h2] = make_uint4(0, 0, 0, 0);
                if (r < rep)
                  qv[h2] = __ldcg(reinterpret_cast<const uint4*>(a.q + ((size_t)b * a.Hq + hk * rep + r) * kMegaHeadDim +
                                                                 cc));
              }
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2) {
                const int i = f + h2 * 128, r = i / 16, cc = (i % 16) * 8;
                const int ch = (cc >> 3) ^ (r & 7);
                *reinterpret_cast<uint4*>(Qs + r * kMegaHeadDim + ch * 8) = qv[h2];
              }
              sync_epi();
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const int r = (lane % 8) + 8 * ((lane / 8) % 2), cc = kk * 16 + 8 * (lane / 16);
                ldsm4(qf[kk], Qs + r * kMegaHeadDim + (((cc >> 3) ^ (r & 7)) << 3));
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
              m_r[0] = m_r[1] = -INFINITY;
              l_r[0] = l_r[1] = 0.f;
            }
            if (!bar_and(1, 128, mwait(&full[stage], fph, abort_flag, a.err, kErrTimeoutEpilogue, dbg, 14, c, p,
                                       stage))) {
              ok = false;
              break;
            }
            if (a.trace && f == 0 && u == u0) a.trace[((size_t)p * n + c) * 8 + 2] = gtimer();
            if (a.trace && f == 0 && u == u1 - 1) a.trace[((size_t)p * n + c) * 8 + 3] = gtimer();
            const bf16* Kb = reinterpret_cast<const bf16*>(ring + stage * kStageBytes);
            const bf16* Vb = reinterpret_cast<const bf16*>(ring + stage * kStageBytes + 16384);
            float scr[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              uint32_t bb[4];
              const int r = wq * 16 + (lane % 8) + 8 * (lane / 16), cc = kk * 16 + 8 * ((lane / 8) % 2);
              ldsm4(bb, Kb + sw128(r, cc));
              mma_16816(scr[0], qf[kk], bb[0], bb[1]);
              mma_16816(scr[1], qf[kk], bb[2], bb[3]);
            }
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const int key = pi * kMegaPage + wq * 16 + j * 8 + 2 * (lane % 4) + (t & 1);
                const float v = key < L_b ? scr[j][t] * a.qk_scale_log2 : -INFINITY;
                scr[j][t] = v;
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
                const float pv = (mnew[t >> 1] == -INFINITY) ? 0.f : exp2f(scr[j][t] - mnew[t >> 1]);
                scr[j][t] = pv;
                rs[t >> 1] += pv;
              }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
              rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
              l_r[r] = l_r[r] * alpha[r] + rs[r];
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              o[i][0] *= alpha[0];
              o[i][1] *= alpha[0];
              o[i][2] *= alpha[1];
              o[i][3] *= alpha[1];
            }
            const uint32_t pf[4] = {pack_bf16x2(scr[0][0], scr[0][1]), pack_bf16x2(scr[0][2], scr[0][3]),
                                    pack_bf16x2(scr[1][0], scr[1][1]), pack_bf16x2(scr[1][2], scr[1][3])};
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              uint32_t bb[4];
              const int r = wq * 16 + (lane % 8) + 8 * ((lane / 8) % 2), cc = i * 8 + 8 * (lane / 16);
              ldsm4t(bb, Vb + sw128(r, cc));
              mma_16816(o[i], pf, bb[0], bb[1]);
              mma_16816(o[i + 1], pf, bb[2], bb[3]);
            }
            sync_epi();  // all four warps are done with the stage
            if (a.trace && f == 0 && u == u1 - 1) a.trace[((size_t)p * n + c) * 8 + 4] = gtimer();
            if (f == 0) mbar_arrive(&empty[stage]);
            if (++stage == kStages) {
              stage = 0;
              fph ^= 1;
            }
            if (!lastu) continue;

            // ── end of a piece: merge the four warps (rows lane/4 and lane/4 + 8) ──
            float* rm = merge;
            float* rl = merge + 64;
            float* ro = merge + 128;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              const int row = lane / 4 + 8 * r;
              if (lane % 4 == 0) {
                rm[wq * 16 + row] = m_r[r];
                rl[wq * 16 + row] = l_r[r];
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int cc = i * 8 + 2 * (lane % 4);
                ro[(wq * 16 + row) * kMegaHeadDim + cc] = o[i][2 * r];
                ro[(wq * 16 + row) * kMegaHeadDim + cc + 1] = o[i][2 * r + 1];
              }
            }
            sync_epi();
            const int s0 = sc.seg[s], s1 = sc.seg[s + 1];
            const bool whole = (s0 >= u0) && (s1 <= u1);
            const int slot = (s0 <= u0) ? 0 : 1;
            float* mypart = a.apart + ((size_t)c * 2 + slot) * 16 * kPartRow;
            for (int row = 0; row < rep; ++row) {
              float M = -INFINITY;
              for (int w = 0; w < 4; ++w) M = fmaxf(M, rm[w * 16 + row]);
              float Ls = 0.f, accv = 0.f;
              for (int w = 0; w < 4; ++w) {
                const float mw = rm[w * 16 + row];
                const float fw = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
                Ls += rl[w * 16 + row] * fw;
                accv += ro[(w * 16 + row) * kMegaHeadDim + f] * fw;
              }
              if (whole) {
                a.ao[(size_t)b * a.q_dim + (hk * rep + row) * kMegaHeadDim + f] =
                    __float2bfloat16(Ls > 0.f ? accv / Ls : 0.f);
              } else {
                mypart[row * kPartRow + f] = accv;
                if (f == 0) {
                  mypart[row * kPartRow + kMegaHeadDim] = M;
                  mypart[row * kPartRow + kMegaHeadDim + 1] = Ls;
                }
              }
            }
            if (a.trace && f == 0 && u == u1 - 1) a.trace[((size_t)p * n + c) * 8 + 5] = gtimer();
            if (!whole) {
              const int c_first = sc.cta_of(s0), c_last = sc.cta_of(s1 - 1);
              const unsigned expected = (unsigned)(c_last - c_first + 1);
              const bool lastc = last_arrival(&attn_ctr[s], expected);
              if (a.trace && f == 0 && u == u1 - 1) a.trace[((size_t)p * n + c) * 8 + 6] = gtimer();
              if (lastc) {
                // Merge the pieces a chunk of contributors at a time: the chunk's partial rows are
                // staged in shared memory with independent float4 loads (one L2 round trip per
                // chunk instead of one per contributor and row), then folded into a running
                // (max, sum, o) per row.
                const int nc = c_last - c_first + 1;
                const int ch = max(1, min(nc, (kMergeFloats / kPartRow) / rep));
                constexpr int kV4 = kPartRow / 4;
                float runM[16], runL[16], runO[16];
#pragma unroll
                for (int row = 0; row < 16; ++row) {
                  runM[row] = -INFINITY;
                  runL[row] = 0.f;
                  runO[row] = 0.f;
                }
                float* stg = merge;  // [ch][rep][kPartRow]
                for (int c0 = 0; c0 < nc; c0 += ch) {
                  const int cn = min(ch, nc - c0);
                  sync_epi();  // previous chunk consumed
                  const int total = cn * rep * kV4;
                  for (int i0 = 0; i0 < total; i0 += 128 * 8) {
                    // eight independent loads in flight per thread, then the stores
                    float4 q4[8];
#pragma unroll
                    for (int u8 = 0; u8 < 8; ++u8) {
                      const int i = i0 + u8 * 128 + f;
                      q4[u8] = make_float4(0.f, 0.f, 0.f, 0.f);
                      if (i < total) {
                        const int k4 = i % kV4, row = (i / kV4) % rep, j = i / (kV4 * rep);
                        const int cc = c_first + c0 + j;
                        const int sl = (s0 <= sc.range(cc)) ? 0 : 1;
                        q4[u8] = __ldcg(reinterpret_cast<const float4*>(
                            a.apart + ((size_t)cc * 2 + sl) * 16 * kPartRow + row * kPartRow + k4 * 4));
                      }
                    }
#pragma unroll
                    for (int u8 = 0; u8 < 8; ++u8) {
                      const int i = i0 + u8 * 128 + f;
                      if (i < total) {
                        const int k4 = i % kV4, row = (i / kV4) % rep, j = i / (kV4 * rep);
                        *reinterpret_cast<float4*>(stg + (j * rep + row) * kPartRow + k4 * 4) = q4[u8];
                      }
                    }
                  }
                  sync_epi();
                  if (a.trace && f == 0 && c0 == 0) a.trace[((size_t)p * n + c) * 8 + 4] = gtimer();
#pragma unroll
                  for (int row = 0; row < 16; ++row) {
                    if (row >= rep) break;
                    float M = runM[row];
                    for (int j = 0; j < cn; ++j) M = fmaxf(M, stg[(j * rep + row) * kPartRow + kMegaHeadDim]);
                    const float r0 = (runM[row] == -INFINITY) ? 0.f : exp2f(runM[row] - M);
                    float Ls = runL[row] * r0, accv = runO[row] * r0;
                    for (int j = 0; j < cn; ++j) {
                      const float* pp = stg + (j * rep + row) * kPartRow;
                      const float mw = pp[kMegaHeadDim];
                      const float fw = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
                      Ls += pp[kMegaHeadDim + 1] * fw;
                      accv += pp[f] * fw;
                    }
                    runM[row] = M;
                    runL[row] = Ls;
                    runO[row] = accv;
                  }
                }
#pragma unroll
                for (int row = 0; row < 16; ++row) {
                  if (row >= rep) break;
                  a.ao[(size_t)b * a.q_dim + (hk * rep + row) * kMegaHeadDim + f] =
                      __float2bfloat16(runL[row] > 0.f ? runO[row] / runL[row] : 0.f);
                }
                if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8 + 7] = gtimer();
              }
            }
            sync_epi();  // the merge buffers are reused by the next piece
          }
        }
      } else {
        // ───────────── GEMM phase epilogue (QKV / OPROJ / GATEUP / DOWN) ─────────────
        const Gsel gs = gemm_of(kind, a, &m_qkv, &m_o, &m_gu, &m_dn, &m_xg, &m_ao, &m_act);
        const MegaLayer& lay = a.layers[layer];
        if (kind == K_QKV) load_rstd(0);
        if (kind == K_GU) {
          load_rstd(1);
          if (c == 0 && f < MP) a.sumsq[f] = 0.f;  // attention-norm sums of the next layer start from zero
        }
        for (int item = c; item < gs.g.T * gs.g.s && ok; item += n) {
          int tile, kb0, kb1;
          item_range(gs.g, item, tile, kb0, kb1);
          // the MMA warp consumes this item's ring stages: observe each one land and release our share
          bool staged = true;
          for (int kb = kb0; kb < kb1; ++kb) {
            if (f == 0 && staged) {
              staged = mwait(&full[stage], fph, abort_flag, a.err, kErrTimeoutEpilogue, dbg, 18, c, p, stage);
              if (staged) mbar_arrive(&empty[stage]);
            }
            if (++stage == kStages) {
              stage = 0;
              fph ^= 1;
            }
          }
          if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8 + 2] = gtimer();
          if (!bar_and(1, 128, staged && mwait(&tfull[acc], aph, abort_flag, a.err, kErrTimeoutEpilogue, dbg, 15, c,
                                               p, acc))) {
            ok = false;
            break;
          }
          if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8 + 3] = gtimer();
          tc_fence_after();
          float v[MP];
          tmem_load_row<MP>(t_lane + acc * MP, v);
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
          if (++acc == 2) {
            acc = 0;
            aph ^= 1;
          }
          const int nrow = tile * 128 + f;
          if (kind == K_GU && gs.g.s == 1 && !(a.flags & 1)) {
            // direct SwiGLU: rows [0, 64) of the tile are gate, [64, 128) the matching up rows
            float* ex = merge;  // [64][MP + 1] (padded: no bank conflicts)
            if (f >= 64) {
#pragma unroll
              for (int t = 0; t < MP; ++t)
                if (t < a.B) ex[(f - 64) * (MP + 1) + t] = v[t];
            }
            sync_epi();
            if (f < 64) {
              const int col = tile * 64 + f;
#pragma unroll
              for (int t = 0; t < MP; ++t) {
                if (t < a.B) {
                  const float gg = round_bf(v[t] * rstd_s[t]);
                  const float uu = round_bf(ex[f * (MP + 1) + t] * rstd_s[t]);
                  a.act[(size_t)t * a.F + col] = __float2bfloat16(silu(gg) * uu);
                }
              }
            }
            sync_epi();
            continue;
          }
          // split-K partial -> fp32 accumulator (QKV / split GATEUP: acc; OPROJ / DOWN: residual x)
          float* dst = (kind == K_QKV || kind == K_GU) ? a.acc : a.x;
          float* drow = dst + (size_t)nrow * MP;
#pragma unroll
          for (int t = 0; t < MP; t += 4) {
            if (t + 4 <= a.B) {
              atomicAdd(reinterpret_cast<float4*>(drow + t), make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]));
            } else if (t < a.B) {
#pragma unroll
              for (int i = 0; i < 3; ++i)
                if (t + i < a.B) atomicAdd(drow + t + i, v[t + i]);
            }
          }
          if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8 + 4] = gtimer();
          const bool lastt = last_arrival(&tile_ctr[tile], (unsigned)gs.g.s);
          if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8 + 5] = gtimer();
          if (!lastt) continue;

          // ── tile finaliser (this CTA completed the tile) ──
          if (kind == K_QKV) {
            float* sm = merge;  // [MP][128] pre-rotation values, then per-row rstd of the head norm
            float* hrs = merge + 64 * 128;
            const float bias = lay.bqkv ? bf2f(lay.bqkv[nrow]) : 0.f;
            ldcg_row<MP>(a.acc + (size_t)nrow * MP, v, a.B);
            zero_row<MP>(a.acc + (size_t)nrow * MP, a.B);
#pragma unroll
            for (int t = 0; t < MP; ++t)
              if (t < a.B) sm[t * 128 + f] = round_bf(v[t] * rstd_s[t] + bias);
            const int Hqk = a.Hq + a.Hkv;
            if (tile >= Hqk) {
              const int hk = tile - Hqk;
              for (int tt = 0; tt < a.B; ++tt) {
                const int64_t sl = slot_s[tt];
                const size_t row = ((size_t)((layer * 2 + 1) * a.n_cache_pages + sl / kMegaPage) * a.Hkv + hk) *
                                       kMegaPage + (size_t)(sl % kMegaPage);
                a.kv[row * kMegaHeadDim + f] = __float2bfloat16(sm[tt * 128 + f]);
              }
            } else {
              sync_epi();
              const bool is_q = tile < a.Hq;
              const bf16* nw = is_q ? lay.q_norm : lay.k_norm;
              if (nw) {
                for (int tt = wq; tt < a.B; tt += 4) {
                  float ss = 0.f;
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    const float e = sm[tt * 128 + lane * 4 + i];
                    ss += e * e;
                  }
                  ss = warp_sum(ss);
                  if (lane == 0) hrs[tt] = rsqrtf(ss / (float)kMegaHeadDim + a.eps);
                }
                sync_epi();
              }
              const int partner = f ^ 64;
              const float inv = a.inv_freq[f & 63];
              const float w_me = nw ? bf2f(nw[f]) : 1.f, w_pa = nw ? bf2f(nw[partner]) : 1.f;
              for (int tt = 0; tt < a.B; ++tt) {
                float x0 = sm[tt * 128 + f], x1 = sm[tt * 128 + partner];
                if (nw) {
                  x0 = round_bf(x0 * hrs[tt] * w_me);
                  x1 = round_bf(x1 * hrs[tt] * w_pa);
                }
                float sn, cs;
                sincosf((float)pos_s[tt] * inv, &sn, &cs);
                const float out = (f < 64) ? x0 * cs - x1 * sn : x0 * cs + x1 * sn;
                if (is_q) {
                  a.q[((size_t)tt * a.Hq + tile) * kMegaHeadDim + f] = __float2bfloat16(out);
                } else {
                  const int hk = tile - a.Hq;
                  const int64_t sl = slot_s[tt];
                  const size_t row = ((size_t)((layer * 2 + 0) * a.n_cache_pages + sl / kMegaPage) * a.Hkv + hk) *
                                         kMegaPage + (size_t)(sl % kMegaPage);
                  a.kv[row * kMegaHeadDim + f] = __float2bfloat16(out);
                }
              }
            }
            sync_epi();
          } else if (kind == K_GU) {
            // split gate/up: SwiGLU from the completed accumulator
            float* ex = merge;
            ldcg_row<MP>(a.acc + (size_t)nrow * MP, v, a.B);
            zero_row<MP>(a.acc + (size_t)nrow * MP, a.B);
            if (f >= 64) {
#pragma unroll
              for (int t = 0; t < MP; ++t)
                if (t < a.B) ex[(f - 64) * (MP + 1) + t] = v[t];
            }
            sync_epi();
            if (f < 64) {
              const int col = tile * 64 + f;
#pragma unroll
              for (int t = 0; t < MP; ++t) {
                if (t < a.B) {
                  const float gg = round_bf(v[t] * rstd_s[t]);
                  const float uu = round_bf(ex[f * (MP + 1) + t] * rstd_s[t]);
                  a.act[(size_t)t * a.F + col] = __float2bfloat16(silu(gg) * uu);
                }
              }
            }
            sync_epi();
          } else {
            // residual stream rows of this tile are final: round, write the next norm's input, add sums
            const bf16* gnext = kind == K_O ? lay.mlp_norm
                                            : (layer + 1 < L ? a.layers[layer + 1].attn_norm : a.final_norm);
            const float gn = bf2f(gnext[nrow]);
            float* red = merge;  // [4][MP]
            ldcg_row<MP>(a.x + (size_t)nrow * MP, v, a.B);
#pragma unroll
            for (int t = 0; t < MP; ++t) v[t] = round_bf(v[t]);
            stcg_row<MP>(a.x + (size_t)nrow * MP, v, a.B);
#pragma unroll
            for (int t = 0; t < MP; ++t) {
              if (t < a.B) {
                a.xg[(size_t)t * a.D + nrow] = __float2bfloat16(v[t] * gn);
                const float ps = warp_sum(v[t] * v[t]);
                if (lane == 0) red[wq * MP + t] = ps;
              }
            }
            sync_epi();
            if (f < a.B)
              atomicAdd(a.sumsq + (kind == K_O ? MP : 0) + f, red[f] + red[MP + f] + red[2 * MP + f] + red[3 * MP + f]);
            sync_epi();
          }
          if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8 + 6] = gtimer();
        }
      }
      // phase done: publish this CTA's writes and arrive on the grid barrier
      if (!ok) break;
      fence_proxy_global();  // this thread's generic writes before the other CTAs' TMA reads of them
      sync_epi();
      if (a.trace && f == 0) a.trace[((size_t)p * n + c) * 8 + 1] = gtimer();
      if (f == 0) gbar_arrive(bar);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(exit_ctr, 1u);
    if (prev == (unsigned)n - 1) {
      // every CTA has left every wait: reset the grid barrier for the next launch
      atomicExch(bar, 0u);
      atomicExch(exit_ctr, 0u);
    }
  }
}

}  // namespace

int mega_grid() {
  static int n = 0;
  if (!n) {
    int dev;
    MESHY_CUDA_CHECK(cudaGetDevice(&dev));
    MESHY_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

size_t mega_apart_floats(int grid) { return (size_t)grid * 2 * 16 * kPartRow; }

template <int MP>
static void launch_mp(const MegaArgs& a, const CUtensorMap& m_qkv, const CUtensorMap& m_o, const CUtensorMap& m_gu,
                      const CUtensorMap& m_dn, const CUtensorMap& m_xg, const CUtensorMap& m_ao,
                      const CUtensorMap& m_act, const CUtensorMap& m_kv, int grid, cudaStream_t st) {
  auto k = mega_decode_kernel<MP>;
  static bool attr = false;
  if (!attr) {
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    int blocks = 0;
    MESHY_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, kThreads, kSmemBytes));
    MESHY_CHECK(blocks >= 1, "mega decode kernel does not fit on an SM");
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers need it
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  MESHY_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, m_qkv, m_o, m_gu, m_dn, m_xg, m_ao, m_act, m_kv, a));
}

void mega_decode_launch(const MegaArgs& a, const CUtensorMap& m_qkv, const CUtensorMap& m_o,
                        const CUtensorMap& m_gu, const CUtensorMap& m_dn, const CUtensorMap& m_xg,
                        const CUtensorMap& m_ao, const CUtensorMap& m_act, const CUtensorMap& m_kv, int grid,
                        cudaStream_t st) {
  MESHY_CHECK(a.B >= 1 && a.B <= a.MP && a.MP <= kMegaMaxRows, "mega decode: 1 <= B <= MP <= 64");
  MESHY_CHECK(grid >= 1 && grid <= 256, "mega decode: at most 256 CTAs (barrier flag lines)");
  MESHY_CHECK(a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= 16 && a.Hkv <= 8, "mega decode: GQA group <= 16, Hkv <= 8");
  MESHY_CHECK(a.D % 128 == 0 && a.F % 64 == 0 && a.q_dim % 128 == 0, "mega decode: dims must tile by 128 / 64");
  for (const MegaGemm* g : {&a.g_qkv, &a.g_o, &a.g_gu, &a.g_dn})
    MESHY_CHECK(g->s >= 1 && g->s <= g->KB && g->s <= kMegaMaxSplit && g->T <= kMegaCtrTiles,
                "mega decode: bad GEMM split");
  switch (a.MP) {
    case 16:
      launch_mp<16>(a, m_qkv, m_o, m_gu, m_dn, m_xg, m_ao, m_act, m_kv, grid, st);
      break;
    case 32:
      launch_mp<32>(a, m_qkv, m_o, m_gu, m_dn, m_xg, m_ao, m_act, m_kv, grid, st);
      break;
    case 64:
      launch_mp<64>(a, m_qkv, m_o, m_gu, m_dn, m_xg, m_ao, m_act, m_kv, grid, st);
      break;
    default:
      MESHY_CHECK(false, "mega decode: MP must be 16, 32 or 64");
  }
  MESHY_CUDA_CHECK(cudaGetLastError());
}

}  // namespace meshy
