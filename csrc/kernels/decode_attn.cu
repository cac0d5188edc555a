// Split-KV paged decode attention with TMA page loads and a cluster reduction.
//
// One CTA per (sequence b, KV head hk, split sp). The rep = Hq/Hkv query
// heads of a KV head form the rows of a 16-row MMA tile, so every K/V page is
// read once for the whole GQA group.
//
//   warp 4     producer: reads the block table and brings each 64-token page
//              of K and V (one [64, HD] bf16 tile each, contiguous in the
//              cache) into a STAGES-deep shared-memory ring with 2-D TMA
//              tiles (128-byte swizzle), completing on an mbarrier;
//   warps 0-3  consumers: warp w scores keys [16w, 16w+16) of every page
//              against the query rows (m16n8k16 bf16 MMA, ldmatrix from the
//              swizzled tile), keeps an online softmax in the exp2 domain and
//              accumulates P·V; the four warp states merge in shared memory.
//
// The n_split CTAs of one (b, hk) form a thread-block cluster along z. Each
// writes its merged (max, sum, O) to its own shared memory; after a cluster
// barrier every CTA combines a disjoint slice of the output across all splits
// through distributed shared memory and writes bf16 O. No global partials and
// no second kernel. Above kMaxClusterSplits splits the CTAs write partials to
// a caller-provided fp32 buffer and paged_decode_combine_kernel merges them.
//
// Every mbarrier wait is bounded; a CTA that gives up records an error code
// and still reaches both cluster barriers.
#include <cuda.h>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "attention.h"
#include "gemm.h"

namespace meshy {

namespace {

constexpr int kPage = 64;
constexpr int kThreadsDec = 160;

template <int HD>
struct DCfg {
  static constexpr int TILE_BYTES = kPage * HD * 2;   // one K or V page of one head
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // K + V
  static constexpr int STAGES = HD == 128 ? 3 : 4;
  static constexpr int Q_BYTES = 16 * HD * 2;
  static constexpr int MERGE_BYTES = (128 + 4 * 16 * HD) * 4;   // rm, rl, ro of the 4 warps
  static constexpr int RED_BYTES = (32 + 16 * HD) * 4;           // cm, cl, co of this CTA
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static_assert(MERGE_BYTES + RED_BYTES <= RING_BYTES, "merge buffers alias the stage ring");
  static constexpr int SMEM_BYTES = RING_BYTES + Q_BYTES + 1024 + 256;
};

// Element offset of (row r, column c) in a [64, HD] tile stored as HD/64
// 128-byte-swizzled [64 rows][64 cols] boxes (the TMA SWIZZLE_128B layout).
__device__ __forceinline__ int sw128(int r, int c) {
  return (c >> 6) * (64 * 64) + r * 64 + ((((c & 63) >> 3) ^ (r & 7)) << 3) + (c & 7);
}

__device__ __forceinline__ void ldsm4(uint32_t* d, const bf16* p) {
  uint32_t a = smem_u32(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t* d, const bf16* p) {
  uint32_t a = smem_u32(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a));
}
__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr float kLog2eD = 1.4426950408889634f;

template <int HD, bool CLUSTER>
__global__ void __launch_bounds__(kThreadsDec) paged_decode_tma_kernel(
    const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapV, const bf16* __restrict__ Q,
    const int* __restrict__ bt, const int* __restrict__ seq_lens, bf16* __restrict__ O, float* __restrict__ part,
    int Hq, int Hkv, int max_pages, int n_split, float scale, int* err, int early, unsigned* __restrict__ ctr,
    unsigned long long* __restrict__ trace) {
  using C = DCfg<HD>;
  extern __shared__ __align__(1024) uint8_t smraw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  bf16* Qs = reinterpret_cast<bf16*>(ring + C::RING_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + C::RING_BYTES + C::Q_BYTES);
  uint64_t* empty = full + C::STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + C::STAGES);

  const int b = blockIdx.x, hk = blockIdx.y, sp = blockIdx.z;
  const int rep = Hq / Hkv;
  // optional timeline, [CTA][8] global-timer ns: entry, past the dependency wait, Q staged, first page
  // consumed (warp 0), last page consumed (warp 0), CTA merge done, cluster merge done, exit
  unsigned long long* tr =
      trace ? trace + (((size_t)b * gridDim.y + hk) * gridDim.z + sp) * 8 : nullptr;
#define DEC_TRACE(k)                                     \
  do {                                                   \
    if (tr && threadIdx.x == 0) tr[(k)] = globaltimer_ns(); \
  } while (0)
  DEC_TRACE(0);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float sl2 = scale * kLog2eD;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapK);
    tma_prefetch_desc(&mapV);
  }
  // Decode step (``early``): the kernel before wrote only each sequence's newest K/V row, and the lengths
  // and block table are older, so everything but the Q rows and the last page may be read before the
  // wait; the producer starts the ring on the split's complete pages under that kernel's tail.
  if (!early) pdl_wait();
  const int L = seq_lens[b];
  const int n_pages = (L + kPage - 1) / kPage;
  const int per = (n_pages + n_split - 1) / n_split;
  const int p0 = min(n_pages, sp * per), p1 = min(n_pages, p0 + per);
  int npre = 0;
  if (early) {
    __syncthreads();  // barriers initialised
    npre = max(0, min(min(p1, n_pages - 1) - p0, C::STAGES));
    if (warp == 4 && lane == 0) {
      for (int j = 0; j < npre; ++j) {
        const int row = (bt[(size_t)b * max_pages + p0 + j] * Hkv + hk) * kPage;
        uint8_t* sk = ring + j * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[j], C::STAGE_BYTES);
#pragma unroll
        for (int h = 0; h < HD / 64; ++h) {
          tma_load_2d(sk + h * 8192, &mapK, &full[j], h * 64, row);
          tma_load_2d(sk + C::TILE_BYTES + h * 8192, &mapV, &full[j], h * 64, row);
        }
      }
    }
    pdl_wait();  // Q and the newest K/V rows come from the kernel before
  }
  DEC_TRACE(1);
  pdl_trigger();
  // query rows of this GQA group → Qs[16][HD] (XOR swizzle of 16-byte chunks), rows >= rep zero
  for (int i = threadIdx.x; i < 16 * HD / 8; i += kThreadsDec) {
    int r = i / (HD / 8), c = (i % (HD / 8)) * 8;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < rep) val = *reinterpret_cast<const uint4*>(Q + ((size_t)b * Hq + hk * rep + r) * HD + c);
    int ch = (c >> 3) ^ (r & 7);
    *reinterpret_cast<uint4*>(Qs + r * HD + ch * 8) = val;
  }
  __syncthreads();
  DEC_TRACE(2);

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  if (warp == 4) {
    // ───────────────────────────── producer ─────────────────────────────
    if (lane == 0) {
      int stage = npre % C::STAGES;
      uint32_t phase = npre == C::STAGES ? 1u : 0u;
      int issued = npre, last_stage = npre > 0 ? npre - 1 : 0;
      uint32_t last_phase = 0;
      for (int pi = p0 + npre; pi < p1; ++pi) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        const int pg = bt[(size_t)b * max_pages + pi];
        const int row = (pg * Hkv + hk) * kPage;
        mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
        uint8_t* sk = ring + stage * C::STAGE_BYTES;
#pragma unroll
        for (int h = 0; h < HD / 64; ++h) {
          tma_load_2d(sk + h * 8192, &mapK, &full[stage], h * 64, row);
          tma_load_2d(sk + C::TILE_BYTES + h * 8192, &mapV, &full[stage], h * 64, row);
        }
        issued++;
        last_stage = stage;
        last_phase = phase;
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (*abort_flag && issued) {
        long long t0 = clock64();
        while (!mbar_try_wait(&full[last_stage], last_phase) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ───────────────────────────── consumers ────────────────────────────
    uint32_t qf[HD / 16][4];
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      int r = (lane % 8) + 8 * ((lane / 8) % 2), c = kk * 16 + 8 * (lane / 16);
      ldsm4(qf[kk], Qs + r * HD + (((c >> 3) ^ (r & 7)) << 3));
    }
    int stage = 0;
    uint32_t phase = 0;
    for (int pi = p0; pi < p1; ++pi) {
      if (!mbar_wait(&full[stage], phase, abort_flag, err, kErrTimeoutMma)) break;
      const bf16* Kb = reinterpret_cast<const bf16*>(ring + stage * C::STAGE_BYTES);
      const bf16* Vb = reinterpret_cast<const bf16*>(ring + stage * C::STAGE_BYTES + C::TILE_BYTES);
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t bb[4];
        int r = warp * 16 + (lane % 8) + 8 * (lane / 16), c = kk * 16 + 8 * ((lane / 8) % 2);
        ldsm4(bb, Kb + sw128(r, c));
        mma_16816(sc[0], qf[kk], bb[0], bb[1]);
        mma_16816(sc[1], qf[kk], bb[2], bb[3]);
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          int key = pi * kPage + warp * 16 + j * 8 + 2 * (lane % 4) + (t & 1);
          float v = key < L ? sc[j][t] * sl2 : -INFINITY;
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
          float pv = (mnew[t >> 1] == -INFINITY) ? 0.f : exp2f(sc[j][t] - mnew[t >> 1]);
          sc[j][t] = pv;
          rs[t >> 1] += pv;
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
      uint32_t pf[4] = {pack_bf16x2(sc[0][0], sc[0][1]), pack_bf16x2(sc[0][2], sc[0][3]),
                        pack_bf16x2(sc[1][0], sc[1][1]), pack_bf16x2(sc[1][2], sc[1][3])};
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t bb[4];
        int r = warp * 16 + (lane % 8) + 8 * ((lane / 8) % 2), c = i * 8 + 8 * (lane / 16);
        ldsm4t(bb, Vb + sw128(r, c));
        mma_16816(o[i], pf, bb[0], bb[1]);
        mma_16816(o[i + 1], pf, bb[2], bb[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (pi == p0) DEC_TRACE(3);
      if (++stage == C::STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    DEC_TRACE(4);
  }
  __syncthreads();  // every page consumed: the stage ring is free for the merge buffers

  // merge the 4 consumer warps. Every warp holds the same (row, column) positions per lane, for its own
  // tokens: all four leave their fragments in shared memory (float4 per lane and column octet) with their
  // row maxima and sums, then warp w combines the four for its quarter of the columns (octets i in
  // [w HD/32, (w + 1) HD/32)) and writes the CTA's state for rows < rep.
  constexpr int IQ = HD / 32;  // column octets per warp
  float* rm = reinterpret_cast<float*>(ring);
  float* rl = rm + 64;
  float* ro = rm + 128;
  float* cm = rm + 128 + 4 * 16 * HD;  // this CTA's merged state
  float* cl = cm + 16;
  float* co = cm + 32;
  if (warp < 4) {
    if (lane % 4 == 0) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        rm[warp * 16 + lane / 4 + 8 * r] = m_r[r];
        rl[warp * 16 + lane / 4 + 8 * r] = l_r[r];
      }
    }
    // [warp][i][lane] float4: consecutive lanes hit consecutive 16-byte words (no bank conflicts)
    float4* dst = reinterpret_cast<float4*>(ro) + warp * (HD / 8) * 32 + lane;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) dst[i * 32] = make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
  }
  __syncthreads();
  if (warp < 4) {
    float f[4][2], Mr[2], Lr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = lane / 4 + 8 * r;
      float mw[4], lw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        mw[w] = rm[w * 16 + row];
        lw[w] = rl[w * 16 + row];
      }
      Mr[r] = fmaxf(fmaxf(mw[0], mw[1]), fmaxf(mw[2], mw[3]));
      Lr[r] = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        f[w][r] = (mw[w] == -INFINITY) ? 0.f : exp2f(mw[w] - Mr[r]);
        Lr[r] += lw[w] * f[w][r];
      }
    }
    float4 x[4][IQ];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float4* src = reinterpret_cast<const float4*>(ro) + (w * (HD / 8) + warp * IQ) * 32 + lane;
#pragma unroll
      for (int k = 0; k < IQ; ++k) x[w][k] = src[k * 32];
    }
#pragma unroll
    for (int k = 0; k < IQ; ++k) {
      const int i = warp * IQ + k;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int r = t >> 1, row = lane / 4 + 8 * r;
        if (row >= rep) continue;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) acc += (&x[w][k].x)[t] * f[w][r];
        const int c = i * 8 + 2 * (lane % 4) + (t & 1);
        const int h = hk * rep + row;
        if (n_split == 1) {
          O[((size_t)b * Hq + h) * HD + c] = __float2bfloat16(Lr[r] > 0.f ? acc / Lr[r] : 0.f);
        } else if (CLUSTER) {
          co[row * HD + c] = acc;
        } else {
          part[(((size_t)b * Hq + h) * n_split + sp) * (HD + 2) + c] = acc;
        }
      }
    }
    if (warp == 0 && lane % 4 == 0 && n_split > 1) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = lane / 4 + 8 * r;
        if (row >= rep) continue;
        if (CLUSTER) {
          cm[row] = Mr[r];
          cl[row] = Lr[r];
        } else {
          float* pp = part + (((size_t)b * Hq + hk * rep + row) * n_split + sp) * (HD + 2);
          pp[HD] = Mr[r];
          pp[HD + 1] = Lr[r];
        }
      }
    }
  }
  DEC_TRACE(5);
  if constexpr (!CLUSTER) {
    if (n_split > 1 && ctr != nullptr) {
      // the last split of (b, hk) to finish merges all splits' partials (no second kernel); it resets
      // the counter for the next launch
      volatile int* last_s = reinterpret_cast<volatile int*>(abort_flag) + 1;
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) *last_s = atomicAdd(&ctr[b * Hkv + hk], 1u) == (unsigned)(n_split - 1);
      __syncthreads();
      if (*last_s) {
        __threadfence();
        float* fm = reinterpret_cast<float*>(ring);  // [16][64]: split maxima, then their weights
        float* fl = fm + 16 * 64;                    // [16]: merged sums
        for (int i = threadIdx.x; i < rep * n_split; i += kThreadsDec) {
          const int row = i / n_split, sp2 = i % n_split;
          fm[row * 64 + sp2] = __ldcg(part + (((size_t)b * Hq + hk * rep + row) * n_split + sp2) * (HD + 2) + HD);
        }
        __syncthreads();
        if (threadIdx.x < rep) {
          const int row = threadIdx.x;
          const float* pr = part + ((size_t)b * Hq + hk * rep + row) * n_split * (HD + 2);
          float M = -INFINITY;
          for (int t = 0; t < n_split; ++t) M = fmaxf(M, fm[row * 64 + t]);
          float Ls = 0.f;
          for (int t = 0; t < n_split; ++t) {
            const float ms = fm[row * 64 + t];
            const float f = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
            Ls += __ldcg(pr + t * (HD + 2) + HD + 1) * f;
            fm[row * 64 + t] = f;
          }
          fl[row] = Ls;
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < rep * HD; idx += kThreadsDec) {
          const int row = idx / HD, c = idx % HD;
          const float* pr = part + ((size_t)b * Hq + hk * rep + row) * n_split * (HD + 2);
          float acc = 0.f;
          for (int t = 0; t < n_split; ++t) acc += __ldcg(pr + t * (HD + 2) + c) * fm[row * 64 + t];
          const float Ls = fl[row];
          O[((size_t)b * Hq + hk * rep + row) * HD + c] = __float2bfloat16(Ls > 0.f ? acc / Ls : 0.f);
        }
        if (threadIdx.x == 0) ctr[b * Hkv + hk] = 0u;
      }
    }
  }
  if constexpr (CLUSTER) {
    if (n_split > 1) {
      __syncwarp();
      cluster_sync_all();
      const uint32_t base_m = smem_u32(cm), base_l = smem_u32(cl), base_o = smem_u32(co);
      for (int idx = sp * kThreadsDec + threadIdx.x; idx < rep * HD; idx += n_split * kThreadsDec) {
        int row = idx / HD, c = idx % HD;
        // every peer's (m, l, o) is loaded before any of them is used, so the DSMEM round trips overlap
        float ms[kMaxClusterSplits], ls[kMaxClusterSplits], os[kMaxClusterSplits];
#pragma unroll
        for (int r = 0; r < kMaxClusterSplits; ++r) {
          if (r < n_split) {
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ms[r]) : "r"(mapa_shared(base_m + row * 4, r)));
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ls[r]) : "r"(mapa_shared(base_l + row * 4, r)));
            asm volatile("ld.shared::cluster.f32 %0, [%1];"
                         : "=f"(os[r])
                         : "r"(mapa_shared(base_o + (row * HD + c) * 4, r)));
          }
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kMaxClusterSplits; ++r)
          if (r < n_split) M = fmaxf(M, ms[r]);
        float Ls = 0.f, acc = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxClusterSplits; ++r) {
          if (r < n_split) {
            const float f = (ms[r] == -INFINITY) ? 0.f : exp2f(ms[r] - M);
            Ls += ls[r] * f;
            acc += os[r] * f;
          }
        }
        O[((size_t)b * Hq + hk * rep + row) * HD + c] = __float2bfloat16(Ls > 0.f ? acc / Ls : 0.f);
      }
      DEC_TRACE(6);
      __syncwarp();
      cluster_sync_all();
    }
  }
  DEC_TRACE(7);
#undef DEC_TRACE
}

// Timeline capture (tests / benchmarks): launch i writes slot i of [slots][kDecTraceCtas][8].
constexpr int kDecTraceCtas = 1024;
unsigned long long* g_dec_trace = nullptr;
int g_dec_trace_slots = 0, g_dec_trace_next = 0;

template <int HD, bool CLUSTER>
void launch_dec(const CUtensorMap& mk, const CUtensorMap& mv, const bf16* q, const int* bt, const int* seq_lens,
                bf16* o, float* part, int B, int Hq, int Hkv, int max_pages, int n_split, float scale, int* err,
                bool early, unsigned* ctr, cudaStream_t st) {
  using C = DCfg<HD>;
  auto k = paged_decode_tma_kernel<HD, CLUSTER>;
  unsigned long long* trace = nullptr;
  const size_t ctas = (size_t)B * Hkv * n_split;
  if (g_dec_trace && g_dec_trace_next < g_dec_trace_slots && ctas <= (size_t)kDecTraceCtas)
    trace = g_dec_trace + (size_t)(g_dec_trace_next++) * kDecTraceCtas * 8;
  static bool attr_set = false;
  if (!attr_set) {
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    if (CLUSTER) MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B, Hkv, n_split);
  cfg.blockDim = dim3(kThreadsDec, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = CLUSTER ? n_split : 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  MESHY_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, mk, mv, q, bt, seq_lens, o, part, Hq, Hkv, max_pages, n_split, scale,
                                      err, early ? 1 : 0, ctr, trace));
}

}  // namespace

// Largest cluster of decode CTAs the device can place (16 needs a non-portable cluster size; if the
// occupancy query finds no room for one, stay at the portable 8).
static int dec_max_cluster() {
  static int n = 0;
  if (!n) {
    auto k = paged_decode_tma_kernel<128, true>;
    using C = DCfg<128>;
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, kMaxClusterSplits);
    cfg.blockDim = dim3(kThreadsDec, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = kMaxClusterSplits;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, k, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      c = 0;
    }
    n = c > 0 ? kMaxClusterSplits : 8;
  }
  return n;
}

int paged_decode_max_cluster() { return dec_max_cluster(); }

void paged_decode_trace(unsigned long long* buf, int slots) {
  g_dec_trace = buf;
  g_dec_trace_slots = buf ? slots : 0;
  g_dec_trace_next = 0;
}

static int g_force_splits = 0;
void paged_decode_force_splits(int n) { g_force_splits = n < 0 ? 0 : n; }

int paged_decode_tma_splits(int B, int Hkv, int max_pages) {
  if (g_force_splits > 0) return std::min(g_force_splits, 64);
  // at most two CTAs per SM are resident (100 KB of shared memory each at head_dim 128), so
  // aim for one wave of them; stay within a cluster (no partial buffer) unless that leaves
  // most SMs idle
  const int slots = 2 * 148;
  const int ctas = std::max(1, B * Hkv);
  int want = std::max(1, slots / ctas);
  // Merging more splits than one cluster holds (partials through global memory) costs more than the SMs a
  // cluster-capped grid leaves idle, unless every split would still walk many pages (measured on B200,
  // 1-16 rows, 2k-8k tokens: 8 cluster splits beat 16-64 global splits in every case). 16-CTA clusters
  // pay off only for a tiny grid over long contexts (1 row x 8k: 12.0 us vs 14.6 us per layer); with
  // 8 or more rows they place poorly (8 rows x 4k: 28 us vs 15 us), so the cap stays at 8 there.
  int cap = 8;
  const int cl = dec_max_cluster();
  if (cl > 8 && ctas * cl <= 64 && max_pages >= 4 * cl) cap = cl;
  if (want > cap && (max_pages + cap - 1) / cap <= 48) want = cap;
  return std::max(1, std::min({want, max_pages, 64}));
}

void paged_decode_tma(const bf16* q, const bf16* kc, const bf16* vc, int n_cache_pages, const int* bt,
                      const int* seq_lens, bf16* o, float* part, int B, int Hq, int Hkv, int hd, int page,
                      int max_pages, int n_split, float scale, int* err, cudaStream_t st, bool decode_step,
                      unsigned* ctr) {
  MESHY_CHECK(hd == 64 || hd == 128, "paged_decode: head_dim must be 64 or 128");
  MESHY_CHECK(page == kPage, "paged_decode: page size must be 64");
  MESHY_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "paged_decode: at most 16 query heads per KV head");
  MESHY_CHECK(n_split >= 1, "paged_decode: n_split must be >= 1");
  const bool cluster = n_split <= dec_max_cluster();
  MESHY_CHECK(cluster || part != nullptr, "paged_decode: more than 8 splits need a partial buffer");
  if (B == 0) return;
  const int64_t rows = (int64_t)n_cache_pages * Hkv * kPage;
  CUtensorMap mk = make_map_bf16(kc, rows, hd, hd, 64, kPage);
  CUtensorMap mv = make_map_bf16(vc, rows, hd, hd, 64, kPage);
  const bool early = decode_step && pdl_enabled();
  if (cluster || (int64_t)B * Hkv > kDecodeCtrs) ctr = nullptr;
  if (hd == 128) {
    if (cluster)
      launch_dec<128, true>(mk, mv, q, bt, seq_lens, o, part, B, Hq, Hkv, max_pages, n_split, scale, err, early, ctr,
                            st);
    else
      launch_dec<128, false>(mk, mv, q, bt, seq_lens, o, part, B, Hq, Hkv, max_pages, n_split, scale, err, early, ctr,
                             st);
  } else {
    if (cluster)
      launch_dec<64, true>(mk, mv, q, bt, seq_lens, o, part, B, Hq, Hkv, max_pages, n_split, scale, err, early, ctr,
                           st);
    else
      launch_dec<64, false>(mk, mv, q, bt, seq_lens, o, part, B, Hq, Hkv, max_pages, n_split, scale, err, early, ctr,
                            st);
  }
  if (!cluster && ctr == nullptr) paged_decode_combine(part, o, B, Hq, hd, n_split, st);
}

}  // namespace meshy
