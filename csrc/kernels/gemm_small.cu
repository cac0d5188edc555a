// Small-M GEMM for sm_100a (decode-time linears):
//
//   out[M, N] = X[M, K] · W[N, K]^T (+bias[n]) (+residual[m, n]),  M <= 256
//
// At decode M is the number of running sequences (8-256) while N and K are
// model dimensions, so the op streams the weight once and is bound by HBM.
// With the regular 128-row MMA tile the token dimension would fill at most
// half of the M=128 MMA, and the few N tiles of a narrow projection (QKV,
// o_proj, down_proj: 12-16 tiles of 128) would leave most SMs idle.  Here the
// operands are swapped: the MMA computes D^T[n, m] = W[n, :] · X[m, :]^T with
// the weight rows as the 128-lane MMA M dimension and the (padded) token count
// MP as the MMA N dimension, so every MMA is full and the accumulator is only
// MP TMEM columns wide.
//
// Two schedules:
//  * split-K over a thread-block cluster (n_tiles <= #SMs): cluster (cs,1,1)
//    of CTAs shares one 128-row weight tile and splits K cs ways.  Each CTA
//    drains its fp32 partial from TMEM into its own shared memory; after a
//    cluster barrier every CTA sums a disjoint set of token columns across all
//    cs partials through distributed shared memory (ld.shared::cluster) and
//    applies the epilogue.  No global workspace, no atomics, no second kernel.
//  * persistent (n_tiles > #SMs, e.g. a 152k-row LM head): one CTA per SM
//    walks the N tiles with two TMEM accumulators, so the epilogue of one tile
//    overlaps the MMAs of the next.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator + single
// thread MMA issuer, warps 2-5 epilogue (warp w owns TMEM lanes 32*(w%4)...).
// Every mbarrier wait is bounded; on a timeout the kernel records an error
// code and still reaches both cluster barriers, so no CTA of a cluster waits
// on one that left.
#include <cuda.h>

#include <cstdlib>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "gemm.h"

namespace meshy {

namespace {

constexpr int SBK = 64;
constexpr int kSmallThreads = 192;
constexpr int W_TILE_BYTES = 128 * SBK * 2;

struct SmallArgs {
  int M, N, K;
  int n_tiles, k_blocks, kb_per, cs;
  int stages;  // depth of the shared-memory stage ring of this launch (<= SCfg::STAGES)
  int early_arrive;  // closing cluster barrier: arrive once the partials are read (1) or after the epilogue (0)
  int epi;
  void* out;
  int ldo;
  int out_f32;
  const bf16* bias;
  const bf16* residual;
  int ldr;
  int* err;
  // fused input RMSNorm: X is the raw residual stream; every row is scaled by its own rstd and the
  // gain before the MMA reads it (null: X is used as is)
  const bf16* norm_w;
  float norm_eps;
  const bf16* x_raw;
  int ldx;
  // RMSNorm split across GEMMs (see GemmProblem): producer outputs / consumer row scale
  bf16* xg_out;
  const bf16* g_next;
  float* part_out;
  const float* part_in;
  int part_t;
  float norm_d;
  // fused QKV epilogue (see GemmProblem)
  bf16* q_out;
  const int* rope_pos;
  const float* inv_freq;
  const bf16* qn;
  const bf16* kn;
  bf16* kc;
  bf16* vc;
  const int64_t* slots;
  int hq, hkv;
  // fused LM-head sampler (EPI_LSE, persistent schedule): per CTA and token row, the log-sum-exp
  // partial and the Gumbel-max winner of the CTA's vocabulary tiles -> partial[m][gridDim.x][8]
  float* partial;
  float inv_temp;
  uint64_t seed;
  const int64_t* step_ptr;
  // optional timeline of this launch, [gridDim.x][8] global-timer ns: entry, producer past the dependency
  // wait, first stage landed at the MMA, last MMA committed, accumulator ready at the epilogue, partials
  // exchanged (first cluster barrier), epilogue done, exit
  unsigned long long* trace;
};

#define SMALL_TRACE(k)                                                   \
  do {                                                                   \
    if (p.trace) p.trace[(size_t)blockIdx.x * 8 + (k)] = globaltimer_ns(); \
  } while (0)

template <int MP, bool PERSIST>
struct SCfg {
  static constexpr int X_TILE_BYTES = MP * SBK * 2;
  static constexpr int STAGE_BYTES = W_TILE_BYTES + X_TILE_BYTES;
  static constexpr int STAGES_FIT = (192 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int N_ACC = PERSIST ? 2 : 1;
  static constexpr int TMEM_COLS = (N_ACC * MP < 32) ? 32 : N_ACC * MP;
  static constexpr int RED_BYTES = 128 * MP * 4;
  static constexpr int BAR_BYTES = 512;
  // after the barriers: rstd [MP], 16 floats of cross-warp sums, then the QKV epilogue's row exchange
  // [4][128] or the sampler's cross-warp statistics [4][MP][5]
  static constexpr int XCH_FLOATS = (MP <= 64 && 20 * MP > 4 * 128) ? 20 * MP : 4 * 128;
  static constexpr int FIXED_BYTES = 1024 + BAR_BYTES + (MP + 16 + XCH_FLOATS) * 4;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + FIXED_BYTES;
  // the split-K partials alias the ring after the K loop: the ring is never shallower than this
  static constexpr int RED_STAGES = (RED_BYTES + STAGE_BYTES - 1) / STAGE_BYTES;
  // deepest ring with which two CTAs fit in one SM's 228 KB (1 KB of it reserved per CTA)
  static constexpr int PAIR_STAGES_FIT = (113 * 1024 - FIXED_BYTES) / STAGE_BYTES;
  static constexpr int PAIR_STAGES = PAIR_STAGES_FIT < RED_STAGES ? RED_STAGES : PAIR_STAGES_FIT;
  static_assert(RED_BYTES <= STAGES * STAGE_BYTES, "reduction buffer must fit in the stage ring");
  static_assert(STAGES <= 8, "the barrier block holds 8 stages");
  static_assert(TMEM_COLS <= 512, "TMEM holds 512 columns");
  static constexpr int smem_bytes(int stages) { return stages * STAGE_BYTES + FIXED_BYTES; }
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// Load 32 (or 16 for MP == 16) accumulator columns starting at ``col`` for this thread's TMEM lane.
template <int MP>
__device__ __forceinline__ void ld_cols(uint32_t taddr, float* v) {
  if constexpr (MP == 16) tmem_ld16(taddr, v);
  else tmem_ld32(taddr, v);
}

__device__ __forceinline__ void store_val(const SmallArgs& p, int m, int n, float x) {
  if (p.bias) x += __bfloat162float(p.bias[n]);
  if (p.residual) x += __bfloat162float(p.residual[(size_t)m * p.ldr + n]);
  if (p.out_f32) reinterpret_cast<float*>(p.out)[(size_t)m * p.ldo + n] = x;
  else reinterpret_cast<bf16*>(p.out)[(size_t)m * p.ldo + n] = __float2bfloat16(x);
}

// Fused input RMSNorm, run by the four epilogue warps while the producer and MMA warps stream the
// K loop.  First every row's rstd = rsqrt(mean(x^2) + eps) -- one warp per row, summed in the same
// order as rmsnorm_fwd_kernel (lane l owns 8-element chunks l, l+32, ...; pairs accumulated in
// order; xor-butterfly warp sum), so the result is bitwise that of the unfused op.  Then, stage by
// stage, the landed X tile is rewritten in place as bf16((x * rstd) * g) and handed to the MMA
// (generic-proxy writes fenced to the async proxy before the arrive).
template <int MP>
__device__ __forceinline__ void norm_stages(const SmallArgs& p, uint8_t* smem, uint64_t* full, uint64_t* normed,
                                            float* rstd_s, int kb0, int kb1, volatile int* abort_flag) {
  using C = SCfg<MP, false>;
  const int ew = (threadIdx.x / 32) - 2;  // 0..3
  const int lane = threadIdx.x % 32;
  const int et = threadIdx.x - 64;        // 0..127
  for (int m = ew; m < MP; m += 4) {
    float ss = 0.f;
    if (m < p.M) {
      const bf16* xr = p.x_raw + (size_t)m * p.ldx;
      for (int c = lane * 8; c < p.K; c += 32 * 8) {
        uint4 u = *reinterpret_cast<const uint4*>(xr + c);
        uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 f = unpack_bf16x2(uu[t]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) rstd_s[m] = (m < p.M) ? rsqrtf(ss / p.K + p.norm_eps) : 0.f;
  }
  named_bar_sync(1, 128);
  int stage = 0;
  uint32_t phase = 0;
  for (int kb = kb0; kb < kb1; ++kb) {
    if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrTimeoutEpilogue)) return;
    bf16* xs = reinterpret_cast<bf16*>(smem + stage * C::STAGE_BYTES + W_TILE_BYTES);
    for (int i = et; i < MP * 8; i += 128) {
      const int m = i >> 3, pc = i & 7;
      const int lc = pc ^ (m & 7);  // 128-byte swizzle: physical 16-byte chunk -> logical
      const int k = kb * SBK + lc * 8;
      uint4* ptr = reinterpret_cast<uint4*>(xs + m * 64 + pc * 8);
      uint4 u = *ptr;
      uint4 o = make_uint4(0, 0, 0, 0);
      if (m < p.M && k < p.K) {
        const float rs = rstd_s[m];
        const uint4 gu = *reinterpret_cast<const uint4*>(p.norm_w + k);
        uint32_t uu[4] = {u.x, u.y, u.z, u.w}, gg[4] = {gu.x, gu.y, gu.z, gu.w}, oo[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 x = unpack_bf16x2(uu[t]), g = unpack_bf16x2(gg[t]);
          oo[t] = pack_bf16x2(x.x * rs * g.x, x.y * rs * g.y);
        }
        o = make_uint4(oo[0], oo[1], oo[2], oo[3]);
      }
      *ptr = o;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&normed[stage]);
    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1;
    }
  }
}

// ─── fused LM-head sampler (EPI_LSE) ─────────────────────────────────────────
// Statistics of a set of logits z_n (one token row): max, sum exp(z - max), and the Gumbel-max winner
// (largest z_n + g_n, its z_n and its vocabulary index n). Two sets combine exactly, in any order.
struct LseSt {
  float mx, s, best, bz;
  int bi;
};

__device__ __forceinline__ LseSt lse_comb(const LseSt& a, const LseSt& b) {
  LseSt r;
  const float hi = fmaxf(a.mx, b.mx), lo = fminf(a.mx, b.mx);
  const float e = (hi == -INFINITY) ? 0.f : __expf(lo - hi);
  r.mx = hi;
  r.s = (a.mx >= b.mx) ? a.s + b.s * e : a.s * e + b.s;
  // ties go to the smaller index; -1 (no winner) compares as the largest unsigned index
  const bool tb = b.best > a.best || (b.best == a.best && (unsigned)b.bi < (unsigned)a.bi);
  r.best = tb ? b.best : a.best;
  r.bz = tb ? b.bz : a.bz;
  r.bi = tb ? b.bi : a.bi;
  return r;
}

__device__ __forceinline__ LseSt lse_shfl(const LseSt& a, int o) {
  LseSt r;
  r.mx = __shfl_xor_sync(0xffffffffu, a.mx, o);
  r.s = __shfl_xor_sync(0xffffffffu, a.s, o);
  r.best = __shfl_xor_sync(0xffffffffu, a.best, o);
  r.bz = __shfl_xor_sync(0xffffffffu, a.bz, o);
  r.bi = __shfl_xor_sync(0xffffffffu, a.bi, o);
  return r;
}

// One halving step of the warp reduce-scatter: the lane keeps the upper or lower half of its C
// statistics (by lane bit C/2) and folds in the partner's copy of the same half.
template <int C>
__device__ __forceinline__ void lse_halve(LseSt* S, int lane) {
  if constexpr (C > 1) {
    constexpr int h = C / 2;
    const bool up = (lane & h) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const LseSt keep = up ? S[i + h] : S[i];
      const LseSt send = up ? S[i] : S[i + h];
      S[i] = lse_comb(keep, lse_shfl(send, h));
    }
    lse_halve<h>(S, lane);
  }
}

// Reduce-scatter over the warp: lane l holds logits z[0..CH) and perturbed logits zg of its vocabulary
// row n for CH token columns; afterwards it holds the warp's statistics (32 vocabulary rows) of token
// column l % CH. 31 combines and ~80 shuffles per lane instead of a full reduction per column.
template <int CH>
__device__ __forceinline__ LseSt lse_warp_scatter(const float* z, const float* zg, int n, int lane) {
  constexpr int H = CH / 2;
  LseSt S[H];
  const bool up = (lane & H) != 0;
#pragma unroll
  for (int i = 0; i < H; ++i) {
    // first step on single logits: only z and z + g cross lanes (the partner's row is n ^ H)
    const float kz = up ? z[i + H] : z[i], kg = up ? zg[i + H] : zg[i];
    const float sz = up ? z[i] : z[i + H], sg = up ? zg[i] : zg[i + H];
    const float rz = __shfl_xor_sync(0xffffffffu, sz, H), rg = __shfl_xor_sync(0xffffffffu, sg, H);
    const LseSt a{kz, kz == -INFINITY ? 0.f : 1.f, kg, kz, n};
    const LseSt b{rz, rz == -INFINITY ? 0.f : 1.f, rg, rz, n ^ H};
    S[i] = lse_comb(a, b);
  }
  lse_halve<H>(S, lane);
  LseSt r = S[0];
  if constexpr (CH < 32) r = lse_comb(r, lse_shfl(r, CH));  // lanes l and l + CH hold the same column
  return r;
}

// Persistent-schedule epilogue of the sampler. Every tile: logits z = acc * rstd[m] / T of the tile's
// 128 vocabulary rows (TMEM lanes) for each token column m, Gumbel noise from Philox-4x32-10 keyed by
// (seed, step) with counter (n, m & ~3, step >> 32, tag) -- one call covers four token columns of a
// row -- and the warp reduce-scatter above; each lane folds its column into running statistics. At
// the end the four warps combine through shared memory and thread m writes the CTA's partial
// (max, sum, 0, 0, best, z of best, index, 0) of row m, the layout lse_merge reads.
template <int MP>
__device__ __forceinline__ void lse_epilogue(const SmallArgs& p, uint32_t t_lane, uint64_t* tfull, uint64_t* tempty,
                                             volatile int* abort_flag, const float* sc, float* red, int first,
                                             int stride) {
  constexpr int CH = MP < 32 ? MP : 32;
  constexpr int NC = MP / CH;
  const int lane = threadIdx.x % 32, q = (threadIdx.x / 32) & 3, f = q * 32 + lane;
  const uint64_t step = p.step_ptr ? (uint64_t)*p.step_ptr : 0ull;
  const uint2 key = make_uint2((uint32_t)p.seed, (uint32_t)(p.seed >> 32) ^ (uint32_t)step);
  LseSt run[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) run[c] = LseSt{-INFINITY, 0.f, -INFINITY, 0.f, -1};
  int acc = 0;
  uint32_t acc_phase = 0;
  for (int nt = first; nt < p.n_tiles; nt += stride) {
    if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue)) break;
    tc_fence_after();
    const int n = nt * 128 + f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float v[32];
      ld_cols<MP>(t_lane + acc * MP + c * CH, v);
      if (c == NC - 1) {  // the accumulator is in registers: hand it back to the MMA warp
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      }
      if (c * CH >= p.M) continue;  // warp-uniform
      float z[CH], zg[CH];
#pragma unroll
      for (int i = 0; i < CH; i += 4) {
        const int m0 = c * CH + i;
        uint4 r = make_uint4(0u, 0u, 0u, 0u);
        if (m0 < p.M)  // warp-uniform: no noise for padding columns
          r = Philox::gen(make_uint4((uint32_t)n, (uint32_t)m0, (uint32_t)(step >> 32), 0x6B1Fu), key);
        const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int m = m0 + t;
          const float zz = (n < p.N && m < p.M) ? v[i + t] * sc[m] : -INFINITY;
          z[i + t] = zz;
          zg[i + t] = zz == -INFINITY ? -INFINITY : zz + gumbel(rr[t]);
        }
      }
      run[c] = lse_comb(run[c], lse_warp_scatter<CH>(z, zg, n, lane));
    }
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1;
    }
  }
  // combine the four warps: red[w][MP][5]
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (lane < CH) {
      float* o = red + ((size_t)q * MP + c * CH + lane) * 5;
      o[0] = run[c].mx;
      o[1] = run[c].s;
      o[2] = run[c].best;
      o[3] = run[c].bz;
      o[4] = __int_as_float(run[c].bi);
    }
  }
  named_bar_sync(1, 128);
  const int m = threadIdx.x - 64;
  if (m < p.M) {
    LseSt t{-INFINITY, 0.f, -INFINITY, 0.f, -1};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* o = red + ((size_t)w * MP + m) * 5;
      t = lse_comb(t, LseSt{o[0], o[1], o[2], o[3], __float_as_int(o[4])});
    }
    float* o = p.partial + ((size_t)m * gridDim.x + blockIdx.x) * 8;
    *reinterpret_cast<float4*>(o) = make_float4(t.mx, t.s, 0.f, 0.f);
    *reinterpret_cast<float4*>(o + 4) = make_float4(t.best, t.bz, __int_as_float(t.bi), 0.f);
  }
}

template <int MP, bool PERSIST>
__global__ void __launch_bounds__(kSmallThreads, 2)
    gemm_small_kernel(const __grid_constant__ CUtensorMap mapW, const __grid_constant__ CUtensorMap mapX,
                      SmallArgs p) {
  using C = SCfg<MP, PERSIST>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::STAGE_BYTES);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* normed = drain + 1;  // [STAGES]: X tile of the stage normalised (fused RMSNorm)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(normed + S);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* rstd_s = reinterpret_cast<float*>(smem + S * C::STAGE_BYTES + C::BAR_BYTES);
  const bool fuse_norm = p.norm_w != nullptr;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = PERSIST ? 0u : cluster_ctarank();
  const int first = blockIdx.x / p.cs, stride = gridDim.x / p.cs;
  const int kb0 = (int)rank * p.kb_per, kb1 = min(p.k_blocks, kb0 + p.kb_per);
  const bool has_k = kb1 > kb0;

  if (threadIdx.x == 0) {
    SMALL_TRACE(0);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    for (int s = 0; s < S; ++s) mbar_init(&normed[s], 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapW);
    tma_prefetch_desc(&mapX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Epilogue operands of the first row group this CTA reduces (group ``rank``: rows 4 rank .. 4 rank + 3),
  // loaded by the epilogue warps while the MMAs run so the epilogue after the reduction issues no
  // dependent global loads: bias / gain of the output row, residual rows, RoPE position and cache slot.
  float pre_bias = 0.f, pre_gain = 0.f, pre_freq = 0.f;
  float pre_res[4] = {0.f, 0.f, 0.f, 0.f};
  int pre_pos[4] = {0, 0, 0, 0};
  int64_t pre_slot[4] = {0, 0, 0, 0};

  if (warp == 0) {
    // ─────────────────────────────── TMA producer ───────────────────────────────
    if (lane == 0 && has_k) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0, last_stage = 0;
      uint32_t last_phase = 0;
      // The weights do not depend on the kernel before this one: under programmatic dependent
      // launch the first STAGES weight tiles stream in while that kernel finishes; the activation
      // tiles of those stages follow once it has completed.
      const int npre = first < p.n_tiles ? min(kb1 - kb0, S) : 0;
      for (int j = 0; j < npre; ++j) {
        mbar_arrive_expect_tx(&full[j], C::STAGE_BYTES);
        tma_load_2d(smem + j * C::STAGE_BYTES, &mapW, &full[j], (kb0 + j) * SBK, first * 128);
      }
      pdl_wait();
      SMALL_TRACE(1);
      for (int j = 0; j < npre; ++j)
        tma_load_2d(smem + j * C::STAGE_BYTES + W_TILE_BYTES, &mapX, &full[j], (kb0 + j) * SBK, 0);
      if (npre > 0) {
        issued = npre;
        last_stage = npre - 1;
        last_phase = 0;
        stage = npre % S;
        phase = (npre == S) ? 1u : 0u;
      }
      for (int nt = first; nt < p.n_tiles && !*abort_flag; nt += stride) {
        for (int kb = (nt == first ? kb0 + npre : kb0); kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          uint8_t* sw = smem + stage * C::STAGE_BYTES;
          tma_load_2d(sw, &mapW, &full[stage], kb * SBK, nt * 128);
          tma_load_2d(sw + W_TILE_BYTES, &mapX, &full[stage], kb * SBK, 0);
          issued++;
          last_stage = stage;
          last_phase = phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      pdl_trigger();
      if (*abort_flag && issued) {
        long long t0 = clock64();
        while (!mbar_try_wait(&full[last_stage], last_phase) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ─────────────────────────────── MMA issuer ─────────────────────────────────
    if (lane == 0 && has_k) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, MP, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool any = false;
      for (int nt = first; nt < p.n_tiles && !*abort_flag; nt += stride) {
        if (PERSIST && !mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * MP;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(fuse_norm ? &normed[stage] : &full[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          if (!any) SMALL_TRACE(2);
          tc_fence_after();
          const uint32_t sw = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sx = sw + W_TILE_BYTES;
#pragma unroll
          for (int k = 0; k < SBK / 16; ++k) {
            mma_bf16(d_tmem, smem_desc_sw128(sw + k * 32, 16, 1024), smem_desc_sw128(sx + k * 32, 16, 1024), idesc,
                     (kb > kb0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          any = true;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (PERSIST && ++acc == C::N_ACC) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (any) {
        SMALL_TRACE(3);
        mma_commit(drain);
        long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ─────────────────────────────── epilogue ───────────────────────────────────
    pdl_wait();  // bias / residual / output may be touched by the kernels before
    if (!PERSIST && fuse_norm && has_k) norm_stages<MP>(p, smem, full, normed, rstd_s, kb0, kb1, abort_flag);
    const bool lse = PERSIST && p.epi == EPI_LSE;
    if (p.part_in || lse) {
      // rows of X were bf16(g * x): their RMSNorm scale from the producer GEMM's per-tile partial sums
      // (the sampler also folds in 1 / temperature)
      for (int m = threadIdx.x - 64; m < MP; m += 128) {
        float r = 1.f;
        if (p.part_in) {
          float ss = 0.f;
          if (m < p.M)
            for (int t = 0; t < p.part_t; ++t) ss += p.part_in[(size_t)t * kSmallPartLd + m];
          r = m < p.M ? rsqrtf(ss / p.norm_d + p.norm_eps) : 0.f;
        }
        rstd_s[m] = lse ? r * p.inv_temp : r;
      }
      named_bar_sync(1, 128);
    }
    const int q = warp & 3;
    const int f = q * 32 + lane;  // weight row within the tile = TMEM lane
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    constexpr int CH = MP < 32 ? MP : 32;
    if constexpr (PERSIST) {
      if (lse) {
        if constexpr (MP <= 64)
          lse_epilogue<MP>(p, t_lane, tfull, tempty, abort_flag, rstd_s, rstd_s + MP + 16, first, stride);
      } else {
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int nt = first; nt < p.n_tiles; nt += stride) {
          if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue)) break;
          tc_fence_after();
          const int n = nt * 128 + f;
          float v[32];
#pragma unroll 1
          for (int c = 0; c < MP / CH; ++c) {
            ld_cols<MP>(t_lane + acc * MP + c * CH, v);
            if (n < p.N) {
#pragma unroll
              for (int i = 0; i < CH; ++i) {
                const int m = c * CH + i;
                if (m < p.M) store_val(p, m, n, p.part_in ? v[i] * rstd_s[m] : v[i]);
              }
            }
          }
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
          if (++acc == C::N_ACC) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
    } else {
      if (p.epi != EPI_SWIGLU && 4 * (int)rank < p.M) {
        const int n = first * 128 + f;
        if (n < p.N) {
          if (p.bias) pre_bias = __bfloat162float(p.bias[n]);
          if (p.q_out) {
            const bf16* nw = first < p.hq ? p.qn : (first < p.hq + p.hkv ? p.kn : nullptr);
            pre_gain = nw ? __bfloat162float(nw[f]) : 0.f;
            pre_freq = p.inv_freq[f & 63];
          } else if (p.part_out) {
            pre_gain = __bfloat162float(p.g_next[n]);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = 4 * (int)rank + i;
            if (m < p.M) {
              if (p.residual) pre_res[i] = __bfloat162float(p.residual[(size_t)m * p.ldr + n]);
              if (p.q_out) {
                pre_pos[i] = p.rope_pos[m];
                pre_slot[i] = p.slots[m];
              }
            }
          }
        }
      }
      // drain this CTA's partial into the (now idle) stage ring: layout [MP/4][128][4] fp32
      float* red = reinterpret_cast<float*>(smem);
      bool ok = true;
      if (has_k) {
        ok = mbar_wait(&tfull[0], 0, abort_flag, p.err, kErrTimeoutEpilogue);
        tc_fence_after();
      }
      if (threadIdx.x == 64) SMALL_TRACE(4);
      float v[32];
#pragma unroll 1
      for (int c = 0; c < MP / CH; ++c) {
        if (has_k && ok) {
          ld_cols<MP>(t_lane + c * CH, v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < CH; i += 4) {
          const int g = (c * CH + i) / 4;
          *reinterpret_cast<float4*>(red + ((size_t)g * 128 + f) * 4) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
      tc_fence_before();
    }
  }

  if constexpr (!PERSIST) {
    __syncwarp();
    cluster_sync_all();  // every partial of the cluster is in shared memory
    if (threadIdx.x == 64) SMALL_TRACE(5);
    if (warp >= 2) {
      const int q = warp & 3;
      const int f = q * 32 + lane;
      const int nt = first;
      const uint32_t red_addr = smem_u32(smem);
      const bool swiglu = p.epi == EPI_SWIGLU;
      constexpr int G = MP / 4;
      // The closing cluster barrier only guards the peers' reads of this CTA's partials. With early_arrive a warp
      // arrives as soon as its last group's partials are summed and waits only before the CTA exits, so the
      // epilogue runs inside the barrier interval (the loop bounds are warp-uniform); otherwise every warp
      // arrives after its epilogue.
      int g_last = -1;
      for (int g = (int)rank; g < G && 4 * g < p.M && !(swiglu && f >= 64); g += p.cs) g_last = g;
      if (!p.early_arrive) g_last = -2;  // arrive after the epilogue instead (below)
      if (g_last == -1) cluster_arrive();
      for (int g = (int)rank; g < G; g += p.cs) {
        if (4 * g >= p.M) break;
        if (swiglu && f >= 64) break;
        const bool pf = g == (int)rank;  // operands prefetched for this group
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = make_float4(0.f, 0.f, 0.f, 0.f);
        const uint32_t off_a = red_addr + (uint32_t)((g * 128 + f) * 16);
        const uint32_t off_b = red_addr + (uint32_t)((g * 128 + f + 64) * 16);
        // issue the peers' loads before summing, so the DSMEM latency is paid once (all peers at once
        // for a plain output, in batches of four when SwiGLU pairs two rows); a CTA alone on its tile reads
        // its partial straight from its own shared memory
        if (p.cs == 1) {
          const float4* red = reinterpret_cast<const float4*>(smem);
          a = red[g * 128 + f];
          if (swiglu) b = red[g * 128 + f + 64];
        } else if (!swiglu) {
          float4 xa[kSmallMaxCluster];
#pragma unroll
          for (int j = 0; j < kSmallMaxCluster; ++j)
            if (j < p.cs) xa[j] = ld_dsmem_f4(mapa_shared(off_a, (uint32_t)j));
#pragma unroll
          for (int j = 0; j < kSmallMaxCluster; ++j) {
            if (j < p.cs) {
              a.x += xa[j].x; a.y += xa[j].y; a.z += xa[j].z; a.w += xa[j].w;
            }
          }
        }
        for (int r0 = 0; swiglu && p.cs > 1 && r0 < p.cs; r0 += 4) {
          float4 xa[4], xb[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (r0 + j < p.cs) {
              xa[j] = ld_dsmem_f4(mapa_shared(off_a, (uint32_t)(r0 + j)));
              if (swiglu) xb[j] = ld_dsmem_f4(mapa_shared(off_b, (uint32_t)(r0 + j)));
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (r0 + j < p.cs) {
              a.x += xa[j].x; a.y += xa[j].y; a.z += xa[j].z; a.w += xa[j].w;
              if (swiglu) { b.x += xb[j].x; b.y += xb[j].y; b.z += xb[j].z; b.w += xb[j].w; }
            }
          }
        }
        float av[4] = {a.x, a.y, a.z, a.w};
        float bv[4] = {b.x, b.y, b.z, b.w};
        if (g == g_last) cluster_arrive();  // every read of a peer's shared memory by this warp is done
        if (p.part_in) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float rs = 4 * g + i < p.M ? rstd_s[4 * g + i] : 0.f;
            av[i] *= rs;
            bv[i] *= rs;
          }
        }
        if (p.q_out) {
          // one head per tile: bias, bf16 rounding, (per-head RMSNorm), RoPE, then q out / K,V to cache
          const int n = nt * 128 + f;
          const int hqk = p.hq + p.hkv;
          float y[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float t = av[i];
            if (p.bias) t += pf ? pre_bias : __bfloat162float(p.bias[n]);
            y[i] = __bfloat162float(__float2bfloat16(t));
          }
          if (nt >= hqk) {  // V head: into the cache as is
            const int hk = nt - hqk;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int m = 4 * g + i;
              if (m < p.M) {
                const int64_t sl = pf ? pre_slot[i] : p.slots[m];
                p.vc[(((size_t)(sl / 64) * p.hkv + hk) * 64 + (size_t)(sl % 64)) * 128 + f] = __float2bfloat16(y[i]);
              }
            }
          } else {
            float* xch = rstd_s + MP + 16;  // [4 rows][128] pre-rotation values, then [4] head-norm scales
            const bool is_q = nt < p.hq;
            const bf16* nw = is_q ? p.qn : p.kn;
            if (nw) {
              float* red4 = rstd_s + MP;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float s4 = warp_sum(y[i] * y[i]);
                if (lane == 0) red4[q * 4 + i] = s4;
              }
              named_bar_sync(1, 128);
              const float w = pf ? pre_gain : __bfloat162float(nw[f]);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float ss = red4[i] + red4[4 + i] + red4[8 + i] + red4[12 + i];
                y[i] = __bfloat162float(__float2bfloat16(y[i] * rsqrtf(ss / 128.f + p.norm_eps) * w));
              }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) xch[i * 128 + f] = y[i];
            named_bar_sync(1, 128);
            const float inv = pf ? pre_freq : p.inv_freq[f & 63];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int m = 4 * g + i;
              if (m < p.M) {
                const float yp = xch[i * 128 + (f ^ 64)];
                float sn, cs;
                sincosf((float)(pf ? pre_pos[i] : p.rope_pos[m]) * inv, &sn, &cs);
                const float o = (f < 64) ? y[i] * cs - yp * sn : y[i] * cs + yp * sn;
                if (is_q) {
                  p.q_out[((size_t)m * p.hq + nt) * 128 + f] = __float2bfloat16(o);
                } else {
                  const int64_t sl = pf ? pre_slot[i] : p.slots[m];
                  p.kc[(((size_t)(sl / 64) * p.hkv + (nt - p.hq)) * 64 + (size_t)(sl % 64)) * 128 + f] =
                      __float2bfloat16(o);
                }
              }
            }
            named_bar_sync(1, 128);  // xch is reused by the next row group
          }
        } else if (!swiglu && p.part_out) {
          // residual GEMM preparing the next RMSNorm (N is a multiple of 128: every lane owns a row)
          const int n = nt * 128 + f;
          const float gn = pf ? pre_gain : __bfloat162float(p.g_next[n]);
          float sq[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = 4 * g + i;
            sq[i] = 0.f;
            if (m < p.M) {
              float y = av[i];
              if (p.bias) y += pf ? pre_bias : __bfloat162float(p.bias[n]);
              if (p.residual) y += pf ? pre_res[i] : __bfloat162float(p.residual[(size_t)m * p.ldr + n]);
              const bf16 yb = __float2bfloat16(y);
              reinterpret_cast<bf16*>(p.out)[(size_t)m * p.ldo + n] = yb;
              const float yr = __bfloat162float(yb);
              p.xg_out[(size_t)m * p.ldo + n] = __float2bfloat16(yr * gn);
              sq[i] = yr * yr;
            }
          }
          float* red4 = rstd_s + MP;  // [4 warps][4 rows]
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float s4 = warp_sum(sq[i]);
            if (lane == 0) red4[q * 4 + i] = s4;
          }
          named_bar_sync(1, 128);
          if (f < 4 && 4 * g + f < p.M)
            p.part_out[(size_t)nt * kSmallPartLd + 4 * g + f] = red4[f] + red4[4 + f] + red4[8 + f] + red4[12 + f];
          named_bar_sync(1, 128);
        } else if (!swiglu) {
          const int n = nt * 128 + f;
          if (n < p.N) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int m = 4 * g + i;
              if (m >= p.M) continue;
              if (!pf) {
                store_val(p, m, n, av[i]);
                continue;
              }
              float x = av[i];
              if (p.bias) x += pre_bias;
              if (p.residual) x += pre_res[i];
              if (p.out_f32) reinterpret_cast<float*>(p.out)[(size_t)m * p.ldo + n] = x;
              else reinterpret_cast<bf16*>(p.out)[(size_t)m * p.ldo + n] = __float2bfloat16(x);
            }
          }
        } else {
          // rows [128 nt, 128 nt + 64) are gate, the next 64 the matching up rows
          const int n = nt * 64 + f;
          bf16* o = reinterpret_cast<bf16*>(p.out);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = 4 * g + i;
            if (m >= p.M) break;
            // round the pre-activations to bf16 as the regular GEMM epilogue does
            float gg = __bfloat162float(__float2bfloat16(av[i]));
            float uu = __bfloat162float(__float2bfloat16(bv[i]));
            o[(size_t)m * p.ldo + n] = __float2bfloat16(silu_f(gg) * uu);
          }
        }
      }
    }
    if (threadIdx.x == 64) SMALL_TRACE(6);
    __syncwarp();
    if (warp < 2 || !p.early_arrive) cluster_arrive();
    cluster_wait();  // no CTA leaves while a peer may still read its shared memory
    if (threadIdx.x == 64) SMALL_TRACE(7);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev;
    MESHY_CUDA_CHECK(cudaGetDevice(&dev));
    MESHY_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

// Pair-sized rings (MESHY_GEMM_SMALL_PAIR, default on; read once).
bool pair_rings() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESHY_GEMM_SMALL_PAIR");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Ring depth of a launch. A split-K CTA never needs more stages than its k-blocks, and with a ring small
// enough for two CTAs per SM (registers allow two: __launch_bounds__(192, 2)) the next kernel of a decode
// chain becomes resident under programmatic dependent launch and streams its weights while this one
// finishes. The persistent schedule (LM head) keeps the full ring.
template <int MP, bool PERSIST>
int ring_stages(int kb_per) {
  using C = SCfg<MP, PERSIST>;
  if (PERSIST) return C::STAGES;
  const int cap = pair_rings() ? std::min(C::STAGES, C::PAIR_STAGES) : C::STAGES;
  return std::max(C::RED_STAGES, std::min(cap, kb_per));
}

template <int MP, bool PERSIST>
void launch_small(const CUtensorMap& mw, const CUtensorMap& mx, const SmallArgs& args, int grid, int cs,
                  cudaStream_t st) {
  using C = SCfg<MP, PERSIST>;
  SmallArgs a = args;
  a.stages = ring_stages<MP, PERSIST>(a.kb_per);
  // early arrival (MESHY_GEMM_SMALL_EARLY_ARRIVE=1) measured 1-4 % slower at 16-64 rows on the same box (its
  // release fence stalls the epilogue warps), and ~1 % faster at 1 row: off by default
  static const int early = [] {
    const char* e = std::getenv("MESHY_GEMM_SMALL_EARLY_ARRIVE");
    return (e && e[0] == '1') ? 1 : 0;
  }();
  a.early_arrive = early;
  auto k = gemm_small_kernel<MP, PERSIST>;
  static bool attr_set = false;
  if (!attr_set) {
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kSmallThreads, 1, 1);
  cfg.dynamicSmemBytes = C::smem_bytes(a.stages);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  MESHY_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, mw, mx, a));
}

// How many clusters of ``cs`` CTAs of this kernel can be resident at once (GPC limits).
template <int MP>
int max_active_clusters(int cs) {
  using C = SCfg<MP, false>;
  static int cache[kSmallMaxCluster + 1] = {};
  if (cache[cs]) return cache[cs];
  auto k = gemm_small_kernel<MP, false>;
  MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
  MESHY_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs * 64, 1, 1);
  cfg.blockDim = dim3(kSmallThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    n = sm_count() / cs;
  }
  cache[cs] = n;
  return n;
}

int max_clusters_mp(int MP, int cs) {
  switch (MP) {
    case 16: return max_active_clusters<16>(cs);
    case 32: return max_active_clusters<32>(cs);
    case 64: return max_active_clusters<64>(cs);
    case 128: return max_active_clusters<128>(cs);
    default: return max_active_clusters<256>(cs);
  }
}

template <bool PERSIST>
void launch_mp(int MP, const CUtensorMap& mw, const CUtensorMap& mx, const SmallArgs& a, int grid, int cs,
               cudaStream_t st) {
  switch (MP) {
    case 16: launch_small<16, PERSIST>(mw, mx, a, grid, cs, st); break;
    case 32: launch_small<32, PERSIST>(mw, mx, a, grid, cs, st); break;
    case 64: launch_small<64, PERSIST>(mw, mx, a, grid, cs, st); break;
    case 128: launch_small<128, PERSIST>(mw, mx, a, grid, cs, st); break;
    default: launch_small<256, PERSIST>(mw, mx, a, grid, cs, st); break;
  }
}

// Process-wide switches (tests and the op benchmark compare schedules with them).
int g_small_enabled = -1;  // -1: from MESHY_GEMM_SMALL_M (default on)
int g_small_force_cs = 0;
// Timeline capture: launch i writes trace slot i of [slots][kSmallTraceCtas][8] until the slots run out.
constexpr int kSmallTraceCtas = 160;
unsigned long long* g_trace = nullptr;
int g_trace_slots = 0, g_trace_next = 0;

bool small_enabled() {
  if (g_small_enabled < 0) {
    const char* e = std::getenv("MESHY_GEMM_SMALL_M");
    g_small_enabled = (e && e[0] == '0') ? 0 : 1;
  }
  return g_small_enabled == 1;
}

}  // namespace

void gemm_small_trace(unsigned long long* buf, int slots) {
  g_trace = buf;
  g_trace_slots = buf ? slots : 0;
  g_trace_next = 0;
}

void gemm_small_config(int enabled, int force_cs) {
  if (enabled >= 0) g_small_enabled = enabled ? 1 : 0;
  if (force_cs >= 0) g_small_force_cs = force_cs;
}

bool gemm_small_eligible(const GemmProblem& g) {
  if (!small_enabled()) return false;
  if (g.a_mn || g.b_mn || g.M > kSmallMaxM || g.M <= 0) return false;
  if (g.epi != EPI_STORE && g.epi != EPI_SWIGLU) return false;
  const int n_tiles = (g.N + 127) / 128;
  if (g.epi == EPI_SWIGLU) {
    // above 128 tokens the regular 128 x 256 tiling fills its MMA and wins
    if (g.aux != nullptr || g.N % 128 != 0 || g.out_f32 || g.M > 128 || n_tiles > sm_count()) return false;
  }
  // the persistent schedule stores 2-byte scalars per token column; above 64 tokens the
  // regular tiling writes the output faster
  if (n_tiles > sm_count() && g.M > 64) return false;
  return true;
}

bool gemm_small_norm_eligible(const GemmProblem& g) {
  if (!gemm_small_eligible(g)) return false;
  const int n_tiles = (g.N + 127) / 128;
  return n_tiles <= sm_count() && g.K % 8 == 0 && g.lda % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(g.A) & 15) == 0;
}

bool gemm_small_prep_eligible(const GemmProblem& g) {
  if (!gemm_small_eligible(g) || g.epi != EPI_STORE || g.out_f32) return false;
  const int n_tiles = (g.N + 127) / 128;
  return g.N % 128 == 0 && n_tiles <= sm_count() && n_tiles <= kSmallPartLd && g.M <= kSmallPartLd;
}

bool gemm_small_rope_eligible(const GemmProblem& g) {
  if (!gemm_small_eligible(g) || g.epi != EPI_STORE || g.out_f32) return false;
  const int n_tiles = (g.N + 127) / 128;
  return g.hq > 0 && g.hkv > 0 && g.N == (g.hq + 2 * g.hkv) * 128 && n_tiles <= sm_count();
}

bool gemm_small_lse_eligible(const GemmProblem& g) {
  return small_enabled() && g.epi == EPI_LSE && g.gumbel && g.labels == nullptr &&
         !g.a_mn && !g.b_mn && g.M >= 1 && g.M <= 64 && g.K % 8 == 0 && g.lda % 8 == 0 && g.ldb % 8 == 0 &&
         g.norm_w == nullptr && g.part_out == nullptr && g.q_out == nullptr;
}

int gemm_small_lse_parts(int N) { return std::max(1, std::min(sm_count(), (N + 127) / 128)); }

void gemm_small_launch(const GemmProblem& g, cudaStream_t st) {
  const bool lse = g.epi == EPI_LSE;
  MESHY_CHECK(lse ? gemm_small_lse_eligible(g) : gemm_small_eligible(g), "gemm_small: problem not eligible");
  MESHY_CHECK(!lse || g.partial != nullptr, "gemm_small: the sampler needs a partial buffer");
  MESHY_CHECK(g.part_out == nullptr || (gemm_small_prep_eligible(g) && g.xg_out && g.g_next),
              "gemm_small: norm preparation needs a STORE epilogue, N a multiple of 128, xg_out and g_next");
  MESHY_CHECK(g.part_in == nullptr || (g.part_t > 0 && g.norm_d > 0.f && g.norm_w == nullptr),
              "gemm_small: norm scale needs part_t, norm_d and no fused input norm");
  MESHY_CHECK(g.q_out == nullptr || (gemm_small_rope_eligible(g) && g.part_out == nullptr && g.norm_w == nullptr &&
                                     g.rope_pos && g.inv_freq && g.kc && g.vc && g.slots),
              "gemm_small: fused QKV epilogue needs N = (Hq + 2 Hkv) * 128, positions, caches and slots");
  MESHY_CHECK(g.norm_w == nullptr || gemm_small_norm_eligible(g), "gemm_small: fused RMSNorm not eligible");
  MESHY_CHECK(g.norm_w == nullptr || (reinterpret_cast<uintptr_t>(g.norm_w) & 15) == 0,
              "gemm_small: RMSNorm gain must be 16-byte aligned");
  const int MP = g.M <= 16 ? 16 : g.M <= 32 ? 32 : g.M <= 64 ? 64 : g.M <= 128 ? 128 : 256;
  SmallArgs a{};
  a.M = g.M; a.N = g.N; a.K = g.K;
  a.n_tiles = (g.N + 127) / 128;
  a.k_blocks = (g.K + SBK - 1) / SBK;
  a.epi = g.epi;
  a.out = g.out; a.ldo = g.ldo; a.out_f32 = g.out_f32;
  a.bias = g.bias; a.residual = g.residual; a.ldr = g.ldr;
  a.err = g.err;
  a.norm_w = g.norm_w;
  a.norm_eps = g.norm_eps;
  a.x_raw = static_cast<const bf16*>(g.A);
  a.ldx = (int)g.lda;
  a.xg_out = g.xg_out;
  a.g_next = g.g_next;
  a.part_out = g.part_out;
  a.part_in = g.part_in;
  a.part_t = g.part_t;
  a.norm_d = g.norm_d;
  a.q_out = g.q_out;
  a.rope_pos = g.rope_pos;
  a.inv_freq = g.inv_freq;
  a.qn = g.qn;
  a.kn = g.kn;
  a.kc = g.kc;
  a.vc = g.vc;
  a.slots = g.slots;
  a.hq = g.hq;
  a.hkv = g.hkv;
  a.partial = g.partial;
  a.inv_temp = g.inv_temp;
  a.seed = g.seed;
  a.step_ptr = g.step_ptr;
  a.trace = nullptr;
  if (g_trace && g_trace_next < g_trace_slots) a.trace = g_trace + (size_t)(g_trace_next++) * kSmallTraceCtas * 8;
  const int sms = sm_count();
  CUtensorMap mw = make_map_bf16(g.B, g.N, g.K, g.ldb, SBK, 128);
  CUtensorMap mx = make_map_bf16(g.A, g.M, g.K, g.lda, SBK, MP);
  if (lse) {
    // persistent: every CTA walks its vocabulary tiles and writes one partial per token row
    a.cs = 1;
    a.kb_per = a.k_blocks;
    launch_mp<true>(MP, mw, mx, a, gemm_small_lse_parts(g.N), 1, st);
  } else if (a.n_tiles <= sms) {
    // largest split whose clusters all fit in one wave (clusters are placed per GPC, so fewer
    // than sms / cs of them may be resident)
    int cs = 1;
    for (int c = std::min(kSmallMaxCluster, a.k_blocks); c >= 2; --c) {
      if (a.n_tiles * c <= sms && a.n_tiles <= max_clusters_mp(MP, c)) {
        cs = c;
        break;
      }
    }
    const int want = g.force_cs > 0 ? g.force_cs : g_small_force_cs;
    if (want > 0) cs = std::max(1, std::min({want, kSmallMaxCluster, a.k_blocks}));
    a.kb_per = (a.k_blocks + cs - 1) / cs;
    cs = (a.k_blocks + a.kb_per - 1) / a.kb_per;  // every rank gets at least one k-block
    a.cs = cs;
    launch_mp<false>(MP, mw, mx, a, a.n_tiles * cs, cs, st);
  } else {
    a.cs = 1;
    a.kb_per = a.k_blocks;
    launch_mp<true>(MP, mw, mx, a, sms, 1, st);
  }
}

}  // namespace meshy
