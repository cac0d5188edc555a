// Python bindings of the kernel library (module ``meshy_b200._C``).
//
// Every entry point takes preallocated output tensors, checks shapes/dtypes
// and launches on the current PyTorch CUDA stream, so all of them can be
// captured in CUDA graphs.  Persistent scratch (split-K workspace and
// counters, the device error word) is owned here and sized on first use.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "kernels/attention.h"
#include "kernels/decode_mega.h"
#include "kernels/elementwise.h"
#include "kernels/gemm.h"
#include "kernels/misc.h"
#include "kernels/ep.h"
#include "kernels/moe.h"
#include "kernels/symm.h"

using torch::Tensor;
using namespace meshy;

namespace {

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_BF16(t) TORCH_CHECK((t).scalar_type() == at::kBFloat16, #t " must be bfloat16")
#define CHECK_F32(t) TORCH_CHECK((t).scalar_type() == at::kFloat, #t " must be float32")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")

std::atomic<int64_t> g_launches{0};
// Every entry point counts the kernels it launches (graph replays are counted
// by the caller from the capture-time count).
cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }
inline void count(int n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

template <typename T>
T* ptr(const Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <typename T>
T* optr(const c10::optional<Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

struct DeviceScratch {
  Tensor ws, counters, err;
};
std::mutex g_mu;
DeviceScratch& scratch(int64_t ws_elems, int64_t n_counters) {
  static DeviceScratch per_dev[64];
  int dev = at::cuda::current_device();
  std::lock_guard<std::mutex> g(g_mu);
  DeviceScratch& s = per_dev[dev];
  auto opts = torch::TensorOptions().device(torch::kCUDA, dev);
  if (!s.err.defined()) s.err = torch::zeros({1}, opts.dtype(torch::kInt32));
  if (!s.ws.defined() || s.ws.numel() < ws_elems) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    MESHY_CUDA_CHECK(cudaStreamIsCapturing(cur_stream(), &cap));
    TORCH_CHECK(cap == cudaStreamCaptureStatusNone,
                "split-K workspace must be sized before CUDA graph capture (run the shape once uncaptured)");
    s.ws = torch::zeros({std::max<int64_t>(ws_elems, 16 << 20)}, opts.dtype(torch::kFloat));
  }
  if (!s.counters.defined() || s.counters.numel() < n_counters)
    s.counters = torch::zeros({std::max<int64_t>(n_counters, 1 << 16)}, opts.dtype(torch::kInt32));
  return s;
}

// out[M,N] (=|+=) op(a) · op(b)^T
void gemm(Tensor a, Tensor b, Tensor out, bool a_mn, bool b_mn, c10::optional<Tensor> bias,
          c10::optional<Tensor> residual, c10::optional<Tensor> aux, int64_t epi, bool accumulate, int64_t block) {
  CHECK_CUDA(a);
  CHECK_BF16(a);
  CHECK_BF16(b);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm expects 2-D tensors");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm operands must be row-major");
  const c10::cuda::CUDAGuard guard(a.device());
  GemmProblem g;
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.lda = a.stride(0);
  g.ldb = b.stride(0);
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.M = a_mn ? a.size(1) : a.size(0);
  g.K = a_mn ? a.size(0) : a.size(1);
  g.N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == g.K, "gemm: K mismatch");
  if (g.M == 0 || g.N == 0) return;
  if (g.K == 0) {
    if (!accumulate) out.zero_();
    return;
  }
  g.out = out.data_ptr();
  g.ldo = out.stride(0);
  g.out_f32 = out.scalar_type() == at::kFloat;
  g.epi = (int)epi;
  if (epi == EPI_STORE && accumulate) {
    TORCH_CHECK(g.out_f32, "accumulating GEMM needs an fp32 output");
    g.epi = EPI_ACC_F32;
  }
  if (g.epi == EPI_SWIGLU) {
    TORCH_CHECK(block == 64, "fused SwiGLU epilogue expects interleave block 64");
    TORCH_CHECK(out.size(1) * 2 == g.N, "swiglu out must be [M, N/2]");
  } else {
    TORCH_CHECK(out.size(0) == g.M && out.size(1) == g.N, "gemm: out shape mismatch");
  }
  g.bias = optr<bf16>(bias);
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(residual->stride(1) == 1, "residual must be row-major");
    g.residual = ptr<bf16>(*residual);
    g.ldr = residual->stride(0);
  }
  if (aux.has_value() && aux->defined()) {
    g.aux = ptr<bf16>(*aux);
    g.ld_aux = aux->stride(0);
  }
  const int m_tiles = (g.M + 127) / 128;
  if (g.epi == EPI_STORE && m_tiles <= 4) {
    int64_t need = (int64_t)g.M * g.N;
    auto& s = scratch(need, (int64_t)m_tiles * ((g.N + 63) / 64));
    g.ws = ptr<float>(s.ws);
    g.ws_cap = s.ws.numel();
    g.counters = ptr<int>(s.counters);
    g.counters_cap = s.counters.numel();
  }
  g.err = ptr<int>(scratch(0, 0).err);
  gemm_launch(g, cur_stream());
  count();
}

// Decode-time fused RMSNorm -> linear (optionally SwiGLU): out = epi(rmsnorm(x; w_norm, eps) . W^T (+bias)).
// Returns false (and does nothing) when the problem is not eligible for the fused small-M path.
// Decode-time RMSNorm split across two small-M GEMMs (returns false when the problem is not eligible,
// in which case the caller uses the unfused ops).
//  * prep:  out = x W^T + residual, xg = bf16(out * g_next), part[t, m] = sum of out^2 over tile t's rows
//  * scaled: out = epi(rstd[m] * (xg W^T) + bias), rstd from part (part_t tiles, model dim norm_d)
bool gemm_norm_prep(Tensor x, Tensor w, Tensor residual, Tensor out, Tensor xg, Tensor g_next, Tensor part) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1, "gemm_norm_prep: row-major");
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.numel() >= (int64_t)((w.size(0) + 127) / 128) * kSmallPartLd,
              "gemm_norm_prep: part must be fp32 [n_tiles, 256]");
  TORCH_CHECK(xg.stride(0) == out.stride(0) && residual.size(1) == w.size(0), "gemm_norm_prep: layouts");
  const c10::cuda::CUDAGuard guard(x.device());
  GemmProblem g;
  g.A = x.data_ptr();
  g.B = w.data_ptr();
  g.lda = x.stride(0);
  g.ldb = w.stride(0);
  g.M = x.size(0);
  g.K = x.size(1);
  g.N = w.size(0);
  g.out = out.data_ptr();
  g.ldo = out.stride(0);
  g.epi = EPI_STORE;
  g.residual = ptr<bf16>(residual);
  g.ldr = residual.stride(0);
  g.xg_out = ptr<bf16>(xg);
  g.g_next = ptr<bf16>(g_next);
  g.part_out = ptr<float>(part);
  g.err = ptr<int>(scratch(0, 0).err);
  if (g.M == 0 || !gemm_small_prep_eligible(g)) return false;
  gemm_small_launch(g, cur_stream());
  count();
  return true;
}

bool gemm_norm_scaled(Tensor xg, Tensor w, Tensor out, c10::optional<Tensor> bias, Tensor part, int64_t part_t,
                      double norm_d, double eps, int64_t epi, int64_t block) {
  CHECK_CUDA(xg);
  CHECK_BF16(xg);
  CHECK_BF16(w);
  TORCH_CHECK(xg.dim() == 2 && w.dim() == 2 && xg.stride(1) == 1 && w.stride(1) == 1, "gemm_norm_scaled: row-major");
  const c10::cuda::CUDAGuard guard(xg.device());
  GemmProblem g;
  g.A = xg.data_ptr();
  g.B = w.data_ptr();
  g.lda = xg.stride(0);
  g.ldb = w.stride(0);
  g.M = xg.size(0);
  g.K = xg.size(1);
  g.N = w.size(0);
  g.out = out.data_ptr();
  g.ldo = out.stride(0);
  g.epi = (int)epi;
  if (g.epi == EPI_SWIGLU) TORCH_CHECK(block == 64 && out.size(1) * 2 == g.N, "gemm_norm_scaled: swiglu out [M, N/2]");
  g.bias = optr<bf16>(bias);
  g.part_in = ptr<float>(part);
  g.part_t = (int)part_t;
  g.norm_d = (float)norm_d;
  g.norm_eps = (float)eps;
  g.err = ptr<int>(scratch(0, 0).err);
  if (g.M == 0 || g.M > kSmallPartLd || !gemm_small_eligible(g)) return false;
  gemm_small_launch(g, cur_stream());
  count();
  return true;
}

Tensor inv_freq_table(int64_t hd, double theta, const torch::Device& dev);

// Decode QKV projection with the rope / KV-cache epilogue: q [M, Hq, 128] out, K and V rows written
// into the paged caches at ``slots``. With ``part`` the input is a prepared RMSNorm input (see
// gemm_norm_scaled). Returns false when not eligible.
bool gemm_qkv_rope(Tensor x, Tensor w, c10::optional<Tensor> bias, c10::optional<Tensor> part, int64_t part_t,
                   double norm_d, double eps, Tensor pos, c10::optional<Tensor> qn, c10::optional<Tensor> kn,
                   Tensor q_out, Tensor kc, Tensor vc, Tensor slots, double theta, int64_t Hq, int64_t Hkv) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1, "gemm_qkv_rope: row-major");
  TORCH_CHECK(pos.scalar_type() == at::kInt && slots.scalar_type() == at::kLong, "gemm_qkv_rope: int32 pos, int64 slots");
  TORCH_CHECK(kc.dim() == 4 && kc.size(2) == 64 && kc.size(3) == 128 && kc.is_contiguous() && vc.is_contiguous(),
              "gemm_qkv_rope: caches [pages, Hkv, 64, 128]");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() >= x.size(0) * Hq * 128, "gemm_qkv_rope: q_out [M, Hq, 128]");
  const c10::cuda::CUDAGuard guard(x.device());
  GemmProblem g;
  g.A = x.data_ptr();
  g.B = w.data_ptr();
  g.lda = x.stride(0);
  g.ldb = w.stride(0);
  g.M = x.size(0);
  g.K = x.size(1);
  g.N = w.size(0);
  g.out = q_out.data_ptr();
  g.ldo = (int)g.N;
  g.epi = EPI_STORE;
  g.bias = optr<bf16>(bias);
  if (part.has_value() && part->defined()) {
    g.part_in = ptr<float>(*part);
    g.part_t = (int)part_t;
    g.norm_d = (float)norm_d;
  }
  g.norm_eps = (float)eps;
  Tensor inv = inv_freq_table(128, theta, x.device());
  g.q_out = ptr<bf16>(q_out);
  g.rope_pos = ptr<int>(pos);
  g.inv_freq = ptr<float>(inv);
  g.qn = optr<bf16>(qn);
  g.kn = optr<bf16>(kn);
  g.kc = ptr<bf16>(kc);
  g.vc = ptr<bf16>(vc);
  g.slots = ptr<int64_t>(slots);
  g.hq = (int)Hq;
  g.hkv = (int)Hkv;
  g.err = ptr<int>(scratch(0, 0).err);
  if (g.M == 0 || g.M > kSmallPartLd || !gemm_small_rope_eligible(g)) return false;
  gemm_small_launch(g, cur_stream());
  count();
  return true;
}

bool gemm_norm(Tensor x, Tensor norm_w, double eps, Tensor w, Tensor out, c10::optional<Tensor> bias,
               c10::optional<Tensor> residual, int64_t epi, int64_t block) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(norm_w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1, "gemm_norm: row-major 2-D");
  const c10::cuda::CUDAGuard guard(x.device());
  GemmProblem g;
  g.A = x.data_ptr();
  g.B = w.data_ptr();
  g.lda = x.stride(0);
  g.ldb = w.stride(0);
  g.M = x.size(0);
  g.K = x.size(1);
  g.N = w.size(0);
  TORCH_CHECK(w.size(1) == g.K && norm_w.numel() == g.K, "gemm_norm: K mismatch");
  g.out = out.data_ptr();
  g.ldo = out.stride(0);
  g.out_f32 = out.scalar_type() == at::kFloat;
  g.epi = (int)epi;
  if (g.epi == EPI_SWIGLU) TORCH_CHECK(block == 64 && out.size(1) * 2 == g.N, "gemm_norm: swiglu out [M, N/2]");
  g.bias = optr<bf16>(bias);
  if (residual.has_value() && residual->defined()) {
    g.residual = ptr<bf16>(*residual);
    g.ldr = residual->stride(0);
  }
  g.norm_w = ptr<bf16>(norm_w);
  g.norm_eps = (float)eps;
  g.err = ptr<int>(scratch(0, 0).err);
  if (g.M == 0 || !gemm_small_norm_eligible(g)) return false;
  gemm_small_launch(g, cur_stream());
  count();
  return true;
}

void swiglu_bwd_(Tensor h, Tensor ga, Tensor dh, int64_t block) {
  CHECK_CONTIG(h);
  CHECK_CONTIG(ga);
  const c10::cuda::CUDAGuard guard(h.device());
  swiglu_bwd(ptr<bf16>(h), ptr<bf16>(ga), ptr<bf16>(dh), h.size(0), (int)ga.size(1), (int)block, cur_stream());
  count();
}

void rmsnorm_fwd_(Tensor x, Tensor w, Tensor y, Tensor rstd, double eps) {
  CHECK_CONTIG(x);
  CHECK_BF16(x);
  const c10::cuda::CUDAGuard guard(x.device());
  rmsnorm_fwd(ptr<bf16>(x), ptr<bf16>(w), ptr<bf16>(y), ptr<float>(rstd), (int)x.size(0), (int)x.size(1), (float)eps,
              cur_stream());
  count();
}

void rmsnorm_bwd_(Tensor gy, Tensor x, Tensor w, Tensor rstd, Tensor gx, Tensor gw) {
  CHECK_CONTIG(gy);
  CHECK_F32(gw);
  const c10::cuda::CUDAGuard guard(x.device());
  rmsnorm_bwd(ptr<bf16>(gy), ptr<bf16>(x), ptr<bf16>(w), ptr<float>(rstd), ptr<bf16>(gx), ptr<float>(gw),
              (int)x.size(0), (int)x.size(1), cur_stream());
  count();
}

Tensor inv_freq_table(int64_t hd, double theta, const torch::Device& dev) {
  static std::mutex mu;
  static std::map<std::tuple<int64_t, double, int>, Tensor> cache;
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_tuple(hd, theta, (int)dev.index());
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  // HF convention: inv_freq = 1 / theta^(arange(0, hd, 2) / hd), fp32
  auto ar = torch::arange(0, hd, 2, torch::kInt64).to(torch::kFloat) / (float)hd;
  auto inv = 1.0 / torch::pow(torch::tensor((float)theta), ar);
  // expand to per-dim table: entry i (i < hd/2) holds inv_freq[i]
  Tensor t = inv.to(torch::kFloat).to(dev);
  cache.emplace(key, t);
  return t;
}

void qkv_rope_fwd_(Tensor qkv, Tensor pos, c10::optional<Tensor> qn, c10::optional<Tensor> kn, Tensor q, Tensor k,
                   Tensor v, double theta, double eps) {
  CHECK_CONTIG(qkv);
  TORCH_CHECK(pos.scalar_type() == at::kInt, "positions must be int32");
  const c10::cuda::CUDAGuard guard(qkv.device());
  int T = q.size(0), Hq = q.size(1), hd = q.size(2), Hkv = k.size(1);
  Tensor inv = inv_freq_table(hd, theta, qkv.device());
  qkv_rope_fwd(ptr<bf16>(qkv), ptr<int>(pos), optr<bf16>(qn), optr<bf16>(kn), ptr<float>(inv), ptr<bf16>(q), ptr<bf16>(k),
               ptr<bf16>(v), T, Hq, Hkv, hd, (float)eps, cur_stream());
  count();
}

// decode / prefill: rope'd q out, K and V straight into the paged cache (and optionally k / v tensors)
void qkv_rope_cache_(Tensor qkv, Tensor pos, c10::optional<Tensor> qn, c10::optional<Tensor> kn, Tensor q,
                     c10::optional<Tensor> k, c10::optional<Tensor> v, Tensor kc, Tensor vc, Tensor slots, double theta,
                     double eps) {
  CHECK_CONTIG(qkv);
  CHECK_CONTIG(kc);
  CHECK_CONTIG(vc);
  TORCH_CHECK(pos.scalar_type() == at::kInt, "positions must be int32");
  TORCH_CHECK(slots.scalar_type() == at::kLong, "slot map must be int64");
  const c10::cuda::CUDAGuard guard(qkv.device());
  int T = q.size(0), Hq = q.size(1), hd = q.size(2), Hkv = kc.size(1);
  Tensor inv = inv_freq_table(hd, theta, qkv.device());
  qkv_rope_fwd(ptr<bf16>(qkv), ptr<int>(pos), optr<bf16>(qn), optr<bf16>(kn), ptr<float>(inv), ptr<bf16>(q),
               optr<bf16>(k), optr<bf16>(v), T, Hq, Hkv, hd, (float)eps, cur_stream(), ptr<bf16>(kc), ptr<bf16>(vc),
               ptr<int64_t>(slots), (int)kc.size(2));
  count();
}

void qkv_rope_bwd_(Tensor qkv, Tensor pos, c10::optional<Tensor> qn, c10::optional<Tensor> kn, Tensor gq, Tensor gk,
                   Tensor gv, Tensor gqkv, c10::optional<Tensor> gqn, c10::optional<Tensor> gkn, double theta,
                   double eps) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  int T = gq.size(0), Hq = gq.size(1), hd = gq.size(2), Hkv = gk.size(1);
  Tensor inv = inv_freq_table(hd, theta, qkv.device());
  qkv_rope_bwd(ptr<bf16>(qkv), ptr<int>(pos), optr<bf16>(qn), optr<bf16>(kn), ptr<float>(inv), ptr<bf16>(gq),
               ptr<bf16>(gk), ptr<bf16>(gv), ptr<bf16>(gqkv), optr<float>(gqn), optr<float>(gkn), T, Hq, Hkv, hd,
               (float)eps, cur_stream());
  count();
}

void flash_attn_fwd_(Tensor q, Tensor k, Tensor v, Tensor cu, Tensor out, Tensor lse, int64_t max_seqlen,
                     double scale) {
  CHECK_CONTIG(q);
  CHECK_CONTIG(k);
  CHECK_CONTIG(v);
  TORCH_CHECK(cu.scalar_type() == at::kInt, "cu_seqlens must be int32");
  const c10::cuda::CUDAGuard guard(q.device());
  flash_attn_fwd(ptr<bf16>(q), ptr<bf16>(k), ptr<bf16>(v), ptr<int>(cu), (int)cu.numel() - 1, ptr<bf16>(out),
                 ptr<float>(lse), (int)q.size(0), (int)max_seqlen, (int)q.size(1), (int)k.size(1), (int)q.size(2),
                 (float)scale, cur_stream(), nullptr, nullptr, (int)k.size(0), ptr<int>(scratch(0, 0).err));
  count();
}

void flash_attn_bwd_(Tensor q, Tensor k, Tensor v, Tensor cu, Tensor out, Tensor gout, Tensor lse, Tensor gq,
                     Tensor gk, Tensor gv, int64_t max_seqlen, double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  Tensor dvec = torch::empty({q.size(1), q.size(0)}, q.options().dtype(torch::kFloat));
  flash_attn_bwd(ptr<bf16>(q), ptr<bf16>(k), ptr<bf16>(v), ptr<int>(cu), (int)cu.numel() - 1, ptr<bf16>(out),
                 ptr<bf16>(gout), ptr<float>(lse), ptr<float>(dvec), ptr<bf16>(gq), ptr<bf16>(gk), ptr<bf16>(gv),
                 (int)q.size(0), (int)max_seqlen, (int)q.size(1), (int)k.size(1), (int)q.size(2), (float)scale,
                 cur_stream(), nullptr, nullptr, 0, (int)k.size(0), ptr<int>(scratch(0, 0).err));
  count(3);
}

// Query chunks against a separate key stream (context parallelism): doc d = queries cu_q[d]..cu_q[d+1] at key
// positions q_off[d].., keys cu_k[d]..cu_k[d+1].
void flash_attn_fwd_kv_(Tensor q, Tensor k, Tensor v, Tensor cu_q, Tensor cu_k, Tensor q_off, Tensor out, Tensor lse,
                        int64_t max_seqlen_q, double scale) {
  CHECK_CONTIG(q);
  CHECK_CONTIG(k);
  CHECK_CONTIG(v);
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && cu_k.scalar_type() == at::kInt && q_off.scalar_type() == at::kInt,
              "cu_q / cu_k / q_off must be int32");
  TORCH_CHECK(cu_q.numel() == cu_k.numel() && q_off.numel() == cu_q.numel() - 1, "cu_q / cu_k / q_off sizes");
  const c10::cuda::CUDAGuard guard(q.device());
  flash_attn_fwd(ptr<bf16>(q), ptr<bf16>(k), ptr<bf16>(v), ptr<int>(cu_q), (int)cu_q.numel() - 1, ptr<bf16>(out),
                 ptr<float>(lse), (int)q.size(0), (int)max_seqlen_q, (int)q.size(1), (int)k.size(1), (int)q.size(2),
                 (float)scale, cur_stream(), ptr<int>(cu_k), ptr<int>(q_off), (int)k.size(0),
                 ptr<int>(scratch(0, 0).err));
  count();
}

// Context-parallel attention forward that reads every CP rank's K / V in place (no all-gather):
// ``k_ptrs`` / ``v_ptrs`` are the device addresses, in this process, of each rank's local [rows * 2 chunk,
// Hkv, 128] K / V buffers (peer mappings of symmetric memory; this rank's own at index rank).
void flash_attn_fwd_cp_peer(Tensor q, std::vector<int64_t> k_ptrs, std::vector<int64_t> v_ptrs, int64_t rows,
                            int64_t chunk, int64_t hkv, Tensor cu_q, Tensor q_off, int64_t docs_per_row, Tensor out,
                            Tensor lse, int64_t max_seqlen_q, double scale) {
  CHECK_CONTIG(q);
  TORCH_CHECK(q.size(2) == 128, "flash_attn_fwd_cp_peer: head_dim 128");
  TORCH_CHECK(k_ptrs.size() == v_ptrs.size() && !k_ptrs.empty() && (int)k_ptrs.size() <= kFaMaxCp,
              "flash_attn_fwd_cp_peer: 1 to 8 ranks");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && q_off.scalar_type() == at::kInt && q_off.numel() == cu_q.numel() - 1,
              "cu_q / q_off: int32, one offset per query document");
  const c10::cuda::CUDAGuard guard(q.device());
  const bf16* kr[kFaMaxCp];
  const bf16* vr[kFaMaxCp];
  for (size_t r = 0; r < k_ptrs.size(); ++r) {
    kr[r] = reinterpret_cast<const bf16*>(k_ptrs[r]);
    vr[r] = reinterpret_cast<const bf16*>(v_ptrs[r]);
  }
  flash_attn_fwd_tc_cp(ptr<bf16>(q), kr, vr, (int)k_ptrs.size(), (int)rows, (int)chunk, ptr<int>(cu_q),
                       (int)cu_q.numel() - 1, (int)docs_per_row, ptr<int>(q_off), ptr<bf16>(out), ptr<float>(lse),
                       (int)q.size(0), (int)max_seqlen_q, (int)q.size(1), (int)hkv, (float)scale, cur_stream(),
                       ptr<int>(scratch(0, 0).err));
  count();
}

void flash_attn_bwd_kv_(Tensor q, Tensor k, Tensor v, Tensor cu_q, Tensor cu_k, Tensor q_off, Tensor out, Tensor gout,
                        Tensor lse, Tensor gq, Tensor gk, Tensor gv, int64_t max_seqlen_q, int64_t max_seqlen_k,
                        double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  Tensor dvec = torch::empty({q.size(1), q.size(0)}, q.options().dtype(torch::kFloat));
  flash_attn_bwd(ptr<bf16>(q), ptr<bf16>(k), ptr<bf16>(v), ptr<int>(cu_q), (int)cu_q.numel() - 1, ptr<bf16>(out),
                 ptr<bf16>(gout), ptr<float>(lse), ptr<float>(dvec), ptr<bf16>(gq), ptr<bf16>(gk), ptr<bf16>(gv),
                 (int)q.size(0), (int)max_seqlen_q, (int)q.size(1), (int)k.size(1), (int)q.size(2), (float)scale,
                 cur_stream(), ptr<int>(cu_k), ptr<int>(q_off), (int)max_seqlen_k, (int)k.size(0),
                 ptr<int>(scratch(0, 0).err));
  count(3);
}

constexpr int kLseBN = 256;

// lp = z[label] - lse, lse, entropy — no [T, V] logits in memory
void lmhead_logprob_fwd(Tensor h, Tensor w, Tensor labels, Tensor lp, Tensor lse, c10::optional<Tensor> ent) {
  CHECK_CONTIG(h);
  CHECK_BF16(h);
  const c10::cuda::CUDAGuard guard(h.device());
  const int T = h.size(0), V = w.size(0), D = h.size(1);
  const int n_tiles = (V + kLseBN - 1) / kLseBN;
  const int chunk = 8192;
  Tensor part = torch::empty({std::min(T, chunk), n_tiles, 8}, h.options().dtype(torch::kFloat));
  for (int s = 0; s < T; s += chunk) {
    int n = std::min(chunk, T - s);
    GemmProblem g;
    g.A = h.data_ptr<at::BFloat16>() + (int64_t)s * D;
    g.B = w.data_ptr();
    g.lda = D;
    g.ldb = w.stride(0);
    g.M = n;
    g.N = V;
    g.K = D;
    g.epi = EPI_LSE;
    g.labels = labels.data_ptr<int64_t>() + s;
    g.partial = ptr<float>(part);
    g.force_bn = kLseBN;
    g.err = ptr<int>(scratch(0, 0).err);
    gemm_launch(g, cur_stream());
    lse_merge(ptr<float>(part), n_tiles, kLseBN, labels.data_ptr<int64_t>() + s, ptr<float>(lp) + s,
              ptr<float>(lse) + s, ent.has_value() && ent->defined() ? ptr<float>(*ent) + s : nullptr, nullptr, nullptr,
              n, cur_stream());
    count(2);
  }
}

// dz[t, v] = g[t] * (onehot(label) - softmax)  (bf16)
void lmhead_dlogits(Tensor h, Tensor w, Tensor labels, Tensor lse, Tensor glp, Tensor dz) {
  const c10::cuda::CUDAGuard guard(h.device());
  GemmProblem g;
  g.A = h.data_ptr();
  g.B = w.data_ptr();
  g.lda = h.stride(0);
  g.ldb = w.stride(0);
  g.M = h.size(0);
  g.N = w.size(0);
  g.K = h.size(1);
  g.epi = EPI_DLOGITS;
  g.out = dz.data_ptr();
  g.ldo = dz.stride(0);
  g.labels = labels.data_ptr<int64_t>();
  g.row_lse = ptr<float>(lse);
  g.row_g = ptr<float>(glp);
  g.err = ptr<int>(scratch(0, 0).err);
  gemm_launch(g, cur_stream());
  count();
}

// fused LM head + Gumbel-max categorical sample + log-prob of the sample
void lmhead_sample(Tensor h, Tensor w, Tensor tok, Tensor lp, double temperature, int64_t seed,
                   c10::optional<Tensor> step) {
  CHECK_CONTIG(h);
  const c10::cuda::CUDAGuard guard(h.device());
  const int B = h.size(0), V = w.size(0);
  const int n_tiles = (V + kLseBN - 1) / kLseBN;
  Tensor part = torch::empty({B, n_tiles, 8}, h.options().dtype(torch::kFloat));
  GemmProblem g;
  g.A = h.data_ptr();
  g.B = w.data_ptr();
  g.lda = h.stride(0);
  g.ldb = w.stride(0);
  g.M = B;
  g.N = V;
  g.K = h.size(1);
  g.epi = EPI_LSE;
  g.partial = ptr<float>(part);
  g.inv_temp = (float)(1.0 / temperature);
  g.seed = (uint64_t)seed;
  g.step_ptr = optr<int64_t>(step);
  g.gumbel = 1;
  g.force_bn = kLseBN;
  g.err = ptr<int>(scratch(0, 0).err);
  gemm_launch(g, cur_stream());
  lse_merge(ptr<float>(part), n_tiles, kLseBN, nullptr, nullptr, nullptr, nullptr, ptr<int64_t>(tok), ptr<float>(lp), B,
            cur_stream());
  count(2);
}

// One decode step's sampling and bookkeeping in two kernels: the LM head with the Gumbel-max sampler
// in its epilogue on the small-M path (optionally on a prepared RMSNorm input: h = bf16(g * x) with
// the per-tile sums of squares ``part``), then the partial merge fused with the row advance (and
// step += 1). Returns false when the small-M sampler cannot take the problem.
bool decode_sample_advance(Tensor h, Tensor w, c10::optional<Tensor> part, int64_t part_t, double norm_d, double eps,
                           double temperature, int64_t seed, Tensor step, Tensor tok_in, Tensor pos, Tensor seq_lens,
                           Tensor gen, Tensor max_new, Tensor done, Tensor slot, Tensor bt, Tensor req,
                           Tensor out_tok, Tensor out_lp, Tensor eos, int64_t page) {
  CHECK_CUDA(h);
  CHECK_BF16(h);
  CHECK_BF16(w);
  TORCH_CHECK(h.dim() == 2 && w.dim() == 2 && h.stride(1) == 1 && w.stride(1) == 1, "decode_sample_advance: row-major");
  TORCH_CHECK(step.scalar_type() == at::kLong, "decode_sample_advance: int64 step");
  if (!(temperature > 0.0)) return false;
  const c10::cuda::CUDAGuard guard(h.device());
  GemmProblem g;
  g.A = h.data_ptr();
  g.B = w.data_ptr();
  g.lda = h.stride(0);
  g.ldb = w.stride(0);
  g.M = h.size(0);
  g.K = h.size(1);
  g.N = w.size(0);
  g.epi = EPI_LSE;
  g.gumbel = 1;
  g.inv_temp = (float)(1.0 / temperature);
  g.seed = (uint64_t)seed;
  g.step_ptr = ptr<int64_t>(step);
  if (part.has_value() && part->defined()) {
    g.part_in = ptr<float>(*part);
    g.part_t = (int)part_t;
    g.norm_d = (float)norm_d;
    g.norm_eps = (float)eps;
  }
  g.err = ptr<int>(scratch(0, 0).err);
  if (g.M == 0 || !gemm_small_lse_eligible(g)) return false;
  const int parts = gemm_small_lse_parts(g.N);
  Tensor pbuf = torch::empty({g.M, parts, 8}, h.options().dtype(torch::kFloat));
  g.partial = ptr<float>(pbuf);
  gemm_small_launch(g, cur_stream());
  sample_advance(ptr<float>(pbuf), parts, ptr<int64_t>(tok_in), ptr<int>(pos), ptr<int>(seq_lens), ptr<int>(gen),
                 ptr<int>(max_new), ptr<int>(done), ptr<int64_t>(slot), ptr<int>(bt), ptr<int>(req),
                 ptr<int64_t>(out_tok), ptr<float>(out_lp), eos.numel() ? ptr<int64_t>(eos) : nullptr,
                 (int)eos.numel(), g.M, (int)bt.size(1), (int)out_tok.size(1), (int)page, ptr<int64_t>(step),
                 cur_stream());
  count(2);
  return true;
}

// The small-M sampler alone (tokens and log-probs out), for tests and benchmarks of the kernel.
bool lmhead_sample_small(Tensor h, Tensor w, c10::optional<Tensor> part, int64_t part_t, double norm_d, double eps,
                         Tensor tok, Tensor lp, double temperature, int64_t seed, c10::optional<Tensor> step) {
  CHECK_CUDA(h);
  CHECK_BF16(h);
  CHECK_BF16(w);
  TORCH_CHECK(h.dim() == 2 && w.dim() == 2 && h.stride(1) == 1 && w.stride(1) == 1, "lmhead_sample_small: row-major");
  if (!(temperature > 0.0)) return false;
  const c10::cuda::CUDAGuard guard(h.device());
  GemmProblem g;
  g.A = h.data_ptr();
  g.B = w.data_ptr();
  g.lda = h.stride(0);
  g.ldb = w.stride(0);
  g.M = h.size(0);
  g.K = h.size(1);
  g.N = w.size(0);
  g.epi = EPI_LSE;
  g.gumbel = 1;
  g.inv_temp = (float)(1.0 / temperature);
  g.seed = (uint64_t)seed;
  g.step_ptr = optr<int64_t>(step);
  if (part.has_value() && part->defined()) {
    g.part_in = ptr<float>(*part);
    g.part_t = (int)part_t;
    g.norm_d = (float)norm_d;
    g.norm_eps = (float)eps;
  }
  g.err = ptr<int>(scratch(0, 0).err);
  if (g.M == 0 || !gemm_small_lse_eligible(g)) return false;
  const int parts = gemm_small_lse_parts(g.N);
  Tensor pbuf = torch::empty({g.M, parts, 8}, h.options().dtype(torch::kFloat));
  g.partial = ptr<float>(pbuf);
  gemm_small_launch(g, cur_stream());
  lse_merge(ptr<float>(pbuf), parts, 128, nullptr, nullptr, nullptr, nullptr, ptr<int64_t>(tok), ptr<float>(lp), g.M,
            cur_stream());
  count(2);
  return true;
}

void embedding_fwd_(Tensor ids, Tensor w, Tensor out) {
  const c10::cuda::CUDAGuard guard(w.device());
  TORCH_CHECK(ids.scalar_type() == at::kLong, "ids must be int64");
  embedding_fwd(ptr<int64_t>(ids), ptr<bf16>(w), ptr<bf16>(out), ids.numel(), (int)w.size(1), w.size(0), cur_stream());
  count();
}

void embedding_bwd_(Tensor ids, Tensor g, Tensor gw) {
  const c10::cuda::CUDAGuard guard(g.device());
  embedding_bwd(ptr<int64_t>(ids), ptr<bf16>(g), ptr<float>(gw), ids.numel(), (int)gw.size(1), gw.size(0),
                cur_stream());
  count();
}

void sq_norm_(Tensor x, Tensor out) {
  CHECK_F32(x);
  const c10::cuda::CUDAGuard guard(x.device());
  sq_norm(ptr<float>(x), x.numel(), ptr<float>(out), cur_stream());
  count();
}

void adamw_flat_(Tensor p, Tensor g, Tensor m, Tensor v, c10::optional<Tensor> out, c10::optional<Tensor> mirror,
                 Tensor norm, double max_norm, double lr, double b1, double b2, double eps, double wd, int64_t step) {
  const c10::cuda::CUDAGuard guard(p.device());
  adamw_flat(ptr<float>(p), ptr<float>(g), ptr<float>(m), ptr<float>(v), optr<bf16>(out), optr<bf16>(mirror),
             ptr<float>(norm), p.numel(), (float)max_norm, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd,
             (int)step, cur_stream());
  count();
}

void ppo_loss_fused_(Tensor new_lp, Tensor old_lp, Tensor adv, Tensor mask, c10::optional<Tensor> roll, Tensor inv,
                     c10::optional<Tensor> posw, c10::optional<Tensor> ent, Tensor doc, Tensor grad, Tensor sums,
                     Tensor seg, double lo, double hi, int64_t use_tis, int64_t use_icepop, double tmin, double tmax,
                     double pcoef, int64_t train_old) {
  const c10::cuda::CUDAGuard guard(new_lp.device());
  TORCH_CHECK(new_lp.is_contiguous() && old_lp.is_contiguous(), "log-probs must be contiguous");
  ppo_loss_fused(ptr<float>(new_lp), ptr<float>(old_lp), ptr<float>(adv), ptr<float>(mask), optr<float>(roll),
                 ptr<float>(inv), optr<float>(posw), optr<float>(ent), ptr<int64_t>(doc), ptr<float>(grad),
                 ptr<float>(sums), ptr<float>(seg), new_lp.numel(), (float)lo, (float)hi, (int)use_tis,
                 (int)use_icepop, (float)tmin, (float)tmax, (float)pcoef, (int)train_old, cur_stream());
  count();
}

void gae_scan_(Tensor x, Tensor d, Tensor valid, Tensor out) {
  const c10::cuda::CUDAGuard guard(x.device());
  gae_scan(ptr<float>(x), ptr<float>(d), ptr<float>(valid), ptr<float>(out), (int)x.size(0), (int)x.size(1),
           cur_stream());
  count();
}

void kv_write_(Tensor k, Tensor v, Tensor kc, Tensor vc, Tensor slots) {
  const c10::cuda::CUDAGuard guard(k.device());
  CHECK_CONTIG(k);
  CHECK_CONTIG(v);
  kv_write(ptr<bf16>(k), ptr<bf16>(v), ptr<bf16>(kc), ptr<bf16>(vc), ptr<int64_t>(slots), (int)k.size(0),
           (int)k.size(1), (int)k.size(2), (int)kc.size(2), cur_stream());
  count();
}

void paged_attention_(Tensor q, Tensor kc, Tensor vc, Tensor bt, Tensor seq_lens, Tensor out, double scale,
                      c10::optional<Tensor> workspace, bool decode_step) {
  const c10::cuda::CUDAGuard guard(q.device());
  CHECK_CONTIG(q);
  CHECK_CONTIG(kc);
  CHECK_CONTIG(vc);
  TORCH_CHECK(bt.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "block table / lens must be int32");
  const int B = q.size(0), Hq = q.size(1), hd = q.size(2), Hkv = kc.size(1), page = kc.size(2);
  const int max_pages = bt.size(1);
  const int n_split = paged_decode_tma_splits(B, Hkv, max_pages);
  Tensor part;
  const int max_cluster = paged_decode_max_cluster();
  if (n_split > max_cluster) {
    int64_t need = (int64_t)B * Hq * n_split * (hd + 2);
    if (workspace.has_value() && workspace->defined() && workspace->numel() >= need) part = *workspace;
    else part = torch::empty({need}, q.options().dtype(torch::kFloat));
  }
  // split counters of the in-kernel merge: zeroed once per device, left zero by every launch
  static Tensor ctrs[64];
  Tensor ctr;
  {
    std::lock_guard<std::mutex> g(g_mu);
    Tensor& c = ctrs[q.get_device()];
    if (!c.defined()) c = torch::zeros({kDecodeCtrs}, q.options().dtype(torch::kInt32));
    ctr = c;
  }
  paged_decode_tma(ptr<bf16>(q), ptr<bf16>(kc), ptr<bf16>(vc), (int)kc.size(0), ptr<int>(bt), ptr<int>(seq_lens),
                   ptr<bf16>(out), part.defined() ? ptr<float>(part) : nullptr, B, Hq, Hkv, hd, page, max_pages,
                   n_split, (float)scale, ptr<int>(scratch(0, 0).err), cur_stream(), decode_step,
                   reinterpret_cast<unsigned*>(ctr.data_ptr<int>()));
  count(n_split > max_cluster && (int64_t)B * Hkv > kDecodeCtrs ? 2 : 1);
}

void decode_advance_(Tensor tok, Tensor lp, Tensor tok_in, Tensor pos, Tensor seq_lens, Tensor gen, Tensor max_new,
                     Tensor done, Tensor slot, Tensor bt, Tensor req, Tensor out_tok, Tensor out_lp, Tensor eos,
                     int64_t page) {
  const c10::cuda::CUDAGuard guard(tok.device());
  decode_advance(ptr<int64_t>(tok), ptr<float>(lp), ptr<int64_t>(tok_in), ptr<int>(pos), ptr<int>(seq_lens),
                 ptr<int>(gen), ptr<int>(max_new), ptr<int>(done), ptr<int64_t>(slot), ptr<int>(bt), ptr<int>(req),
                 ptr<int64_t>(out_tok), ptr<float>(out_lp), eos.numel() ? ptr<int64_t>(eos) : nullptr,
                 (int)eos.numel(), (int)tok.size(0), (int)bt.size(1), (int)out_tok.size(1), (int)page, cur_stream());
  count();
}

void cast_copy(Tensor src, Tensor dst) {
  const c10::cuda::CUDAGuard guard(src.device());
  TORCH_CHECK(src.numel() == dst.numel(), "cast_copy: size mismatch");
  if (src.scalar_type() == at::kFloat && dst.scalar_type() == at::kBFloat16) {
    cast_f32_bf16(ptr<float>(src), ptr<bf16>(dst), src.numel(), cur_stream());
    count();
  } else {
    dst.copy_(src);
  }
}

// ─── symmetric peer memory ────────────────────────────────────────────────────
// ─── mixture of experts ─────────────────────────────────────────────────────
void moe_route_(Tensor logits, int64_t k, bool norm, Tensor probs, Tensor weights, Tensor experts) {
  CHECK_CUDA(logits);
  CHECK_BF16(logits);
  CHECK_CONTIG(logits);
  CHECK_F32(probs);
  CHECK_F32(weights);
  TORCH_CHECK(experts.scalar_type() == at::kInt, "experts must be int32");
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(probs.numel() == (int64_t)T * E && weights.numel() == (int64_t)T * k && experts.numel() == (int64_t)T * k,
              "moe_route: shape mismatch");
  const c10::cuda::CUDAGuard guard(logits.device());
  moe_route(ptr<bf16>(logits), T, E, (int)k, norm, ptr<float>(probs), ptr<float>(weights), ptr<int>(experts),
            cur_stream());
  count();
}

void moe_route_bwd_(Tensor dw, Tensor probs, Tensor weights, Tensor experts, bool norm, Tensor dlogits) {
  CHECK_CUDA(dw);
  CHECK_F32(dw);
  CHECK_CONTIG(dw);
  CHECK_BF16(dlogits);
  const int T = probs.size(0), E = probs.size(1), k = weights.size(1);
  TORCH_CHECK(dlogits.numel() == (int64_t)T * E && dw.numel() == (int64_t)T * k, "moe_route_bwd: shape mismatch");
  const c10::cuda::CUDAGuard guard(dw.device());
  moe_route_bwd(ptr<float>(dw), ptr<float>(probs), ptr<float>(weights), ptr<int>(experts), T, E, k, norm,
                ptr<bf16>(dlogits), cur_stream());
  count();
}

void moe_plan_(Tensor experts, Tensor cnt, Tensor off, Tensor slot_of, Tensor row_src, c10::optional<Tensor> x,
               c10::optional<Tensor> xp) {
  CHECK_CUDA(experts);
  CHECK_CONTIG(experts);
  TORCH_CHECK(experts.scalar_type() == at::kInt && cnt.scalar_type() == at::kInt && off.scalar_type() == at::kInt &&
                  slot_of.scalar_type() == at::kInt && row_src.scalar_type() == at::kInt,
              "moe_plan: int32 index tensors");
  const int E = cnt.numel();
  TORCH_CHECK(off.numel() == E + 1, "moe_plan: off must have E + 1 entries");
  const int n = experts.numel(), k = experts.size(-1);
  TORCH_CHECK(slot_of.numel() == n, "moe_plan: slot_of must have one entry per assignment");
  const int rows_cap = row_src.numel();
  int D = 0;
  if (xp.has_value() && xp->defined()) {
    TORCH_CHECK(x.has_value() && x->defined(), "moe_plan: xp needs x");
    CHECK_BF16(*x);
    CHECK_BF16(*xp);
    CHECK_CONTIG(*x);
    CHECK_CONTIG(*xp);
    D = x->size(1);
    TORCH_CHECK(xp->size(0) == rows_cap && xp->size(1) == D && x->size(0) * k == n, "moe_plan: x / xp shapes");
  }
  const c10::cuda::CUDAGuard guard(experts.device());
  moe_plan(ptr<int>(experts), n, k, E, ptr<int>(cnt), ptr<int>(off), ptr<int>(slot_of), ptr<int>(row_src),
           D ? ptr<bf16>(*x) : nullptr, D ? D : 8, D ? ptr<bf16>(*xp) : nullptr, rows_cap, ptr<int>(scratch(0, 0).err),
           cur_stream());
  count(2);
}

void moe_zero_pad_(Tensor off, Tensor cnt, Tensor buf) {
  CHECK_CUDA(buf);
  CHECK_BF16(buf);
  CHECK_CONTIG(buf);
  const c10::cuda::CUDAGuard guard(buf.device());
  moe_zero_pad(ptr<int>(off), ptr<int>(cnt), cnt.numel(), ptr<bf16>(buf), buf.size(1), cur_stream());
  count();
}

void moe_combine_(Tensor y, Tensor slot_of, c10::optional<Tensor> w, Tensor out) {
  CHECK_CUDA(y);
  CHECK_BF16(y);
  CHECK_BF16(out);
  CHECK_CONTIG(y);
  CHECK_CONTIG(out);
  const int T = out.size(0), D = out.size(1);
  const int k = slot_of.numel() / std::max(T, 1);
  TORCH_CHECK(y.size(1) == D && slot_of.numel() == (int64_t)T * k, "moe_combine: shapes");
  const c10::cuda::CUDAGuard guard(y.device());
  moe_combine(ptr<bf16>(y), y.size(0), ptr<int>(slot_of), optr<float>(w), T, k, D, ptr<bf16>(out), cur_stream());
  count();
}

void moe_combine_bwd_(Tensor dout, Tensor y, Tensor slot_of, Tensor w, Tensor dy, Tensor dw) {
  CHECK_CUDA(dout);
  CHECK_BF16(dout);
  CHECK_CONTIG(dout);
  CHECK_BF16(dy);
  CHECK_F32(dw);
  const int T = dout.size(0), D = dout.size(1), k = w.size(1);
  TORCH_CHECK(dy.size(1) == D && y.size(1) == D && slot_of.numel() == (int64_t)T * k, "moe_combine_bwd: shapes");
  const c10::cuda::CUDAGuard guard(dout.device());
  moe_combine_bwd(ptr<bf16>(dout), ptr<bf16>(y), y.size(0), ptr<int>(slot_of), ptr<float>(w), T, k, D,
                  ptr<bf16>(dy), ptr<float>(dw), cur_stream());
  count();
}

// Grouped GEMM over 128-aligned token segments (off [G + 1] on the device):
//   mode 1 (GRP_M): out[seg_g] = a[seg_g] . op(b[g])^T, a [rows, K], b [G, N, K] (or [G, K, N] with b_mn),
//                   epilogue store or SwiGLU (out [rows, N / 2], optional pre-activation aux [rows, N]);
//   mode 2 (GRP_K): out[g] += a[seg_g]^T . b[seg_g], a [rows, M], b [rows, N], out [G * M, N] fp32.
void gemm_grouped(Tensor a, Tensor b, Tensor out, Tensor off, int64_t mode, bool b_mn, int64_t epi,
                  c10::optional<Tensor> aux) {
  CHECK_CUDA(a);
  CHECK_BF16(a);
  CHECK_BF16(b);
  CHECK_CONTIG(a);
  CHECK_CONTIG(b);
  CHECK_CONTIG(out);
  TORCH_CHECK(off.scalar_type() == at::kInt, "gemm_grouped: int32 offsets");
  const c10::cuda::CUDAGuard guard(a.device());
  GemmProblem g;
  g.grp_mode = (int)mode;
  g.grp_off = ptr<int>(off);
  g.grp_n = off.numel() - 1;
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.out = out.data_ptr();
  g.ldo = out.stride(0);
  g.out_f32 = out.scalar_type() == at::kFloat;
  g.err = ptr<int>(scratch(0, 0).err);
  if (mode == GRP_M) {
    TORCH_CHECK(b.dim() == 3 && b.size(0) == g.grp_n, "GRP_M: b must be [G, N, K] / [G, K, N]");
    g.a_mn = false;
    g.b_mn = b_mn;
    g.M = a.size(0);
    g.K = a.size(1);
    g.lda = a.stride(0);
    g.N = b_mn ? b.size(2) : b.size(1);
    TORCH_CHECK((b_mn ? b.size(1) : b.size(2)) == g.K, "GRP_M: K mismatch");
    g.ldb = b.stride(1);
    g.grp_stride = b.stride(0);
    g.epi = (int)epi;
    if (epi == EPI_SWIGLU) {
      TORCH_CHECK(out.size(0) == g.M && out.size(1) * 2 == g.N, "GRP_M SwiGLU: out [rows, N / 2]");
      if (aux.has_value() && aux->defined()) {
        CHECK_BF16(*aux);
        TORCH_CHECK(aux->size(0) == g.M && aux->size(1) == g.N, "GRP_M SwiGLU: aux [rows, N]");
        g.aux = ptr<bf16>(*aux);
        g.ld_aux = aux->stride(0);
      }
    } else {
      TORCH_CHECK(epi == EPI_STORE && out.size(0) == g.M && out.size(1) == g.N, "GRP_M: out [rows, N]");
    }
  } else {
    TORCH_CHECK(mode == GRP_K, "gemm_grouped: mode 1 (GRP_M) or 2 (GRP_K)");
    TORCH_CHECK(b.dim() == 2 && a.size(0) == b.size(0), "GRP_K: a [rows, M], b [rows, N]");
    g.a_mn = true;
    g.b_mn = true;
    g.K = a.size(0);
    g.M = a.size(1);
    g.N = b.size(1);
    g.lda = a.stride(0);
    g.ldb = b.stride(0);
    g.epi = EPI_ACC_F32;
    TORCH_CHECK(g.out_f32 && out.size(0) == (int64_t)g.M * g.grp_n && out.size(1) == g.N, "GRP_K: out [G * M, N] fp32");
  }
  if (g.M == 0 || g.N == 0 || g.K == 0) return;
  gemm_launch(g, cur_stream());
  count();
}

void filtered_sample_(Tensor logits, double temperature, int64_t top_k, double top_p, int64_t seed,
                      c10::optional<Tensor> step, Tensor tok, Tensor lp) {
  CHECK_CUDA(logits);
  CHECK_F32(logits);
  CHECK_CONTIG(logits);
  TORCH_CHECK(tok.scalar_type() == at::kLong && lp.scalar_type() == at::kFloat, "tok int64, lp fp32");
  const c10::cuda::CUDAGuard guard(logits.device());
  filtered_sample(ptr<float>(logits), logits.size(0), logits.size(1), (float)temperature, (int)top_k, (float)top_p,
                  (uint64_t)seed, optr<int64_t>(step), ptr<int64_t>(tok), ptr<float>(lp), cur_stream());
  count();
}

void value_head_fwd_(Tensor h, Tensor w, Tensor b, Tensor ret, Tensor mask, c10::optional<Tensor> old, double clip,
                     double inv_denom, Tensor v, Tensor dv, Tensor num) {
  CHECK_CUDA(h);
  CHECK_BF16(h);
  CHECK_CONTIG(h);
  CHECK_F32(w);
  const int T = h.size(0), D = h.size(1);
  TORCH_CHECK(w.numel() == D && ret.numel() == T && mask.numel() == T && v.numel() == T && dv.numel() == T,
              "value_head_fwd: shapes");
  const c10::cuda::CUDAGuard guard(h.device());
  value_head_fwd(ptr<bf16>(h), ptr<float>(w), ptr<float>(b), T, D, ptr<float>(ret), ptr<float>(mask), optr<float>(old),
                 (float)clip, (float)inv_denom, ptr<float>(v), ptr<float>(dv), ptr<float>(num), cur_stream());
  count();
}

void value_head_bwd_(Tensor h, Tensor w, Tensor dv, Tensor dh, Tensor dw, Tensor db) {
  CHECK_CUDA(h);
  CHECK_BF16(h);
  CHECK_BF16(dh);
  CHECK_F32(dw);
  const c10::cuda::CUDAGuard guard(h.device());
  value_head_bwd(ptr<bf16>(h), ptr<float>(w), ptr<float>(dv), h.size(0), h.size(1), ptr<bf16>(dh), ptr<float>(dw),
                 ptr<float>(db), cur_stream());
  count();
}

void topk_logprobs_(Tensor z, int64_t k, Tensor ids, Tensor lp, c10::optional<Tensor> lse) {
  CHECK_CUDA(z);
  CHECK_F32(z);
  TORCH_CHECK(z.dim() == 2 && z.stride(1) == 1, "topk_logprobs: z [T, V] row-major");
  const int T = z.size(0);
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.numel() == (int64_t)T * k,
              "topk_logprobs: ids [T, K] int64");
  TORCH_CHECK(lp.scalar_type() == at::kFloat && lp.is_contiguous() && lp.numel() == (int64_t)T * k,
              "topk_logprobs: lp [T, K] fp32");
  TORCH_CHECK(!lse || (lse->scalar_type() == at::kFloat && lse->numel() == T), "topk_logprobs: lse [T] fp32");
  const c10::cuda::CUDAGuard guard(z.device());
  topk_logprobs(ptr<float>(z), z.stride(0), T, z.size(1), (int)k, ptr<int64_t>(ids), ptr<float>(lp), optr<float>(lse),
                cur_stream());
  count();
}

void gather_logprobs_(Tensor h, Tensor w, Tensor ids, Tensor lse, Tensor lp) {
  CHECK_CUDA(h);
  CHECK_BF16(h);
  CHECK_BF16(w);
  TORCH_CHECK(h.dim() == 2 && w.dim() == 2 && h.stride(1) == 1 && w.stride(1) == 1 && h.size(1) == w.size(1),
              "gather_logprobs: h [T, D], w [V, D] row-major");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == h.size(0),
              "gather_logprobs: ids [T, K] int64");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == h.size(0), "gather_logprobs: lse [T] fp32");
  TORCH_CHECK(lp.scalar_type() == at::kFloat && lp.is_contiguous() && lp.numel() == ids.numel(),
              "gather_logprobs: lp [T, K] fp32");
  const c10::cuda::CUDAGuard guard(h.device());
  gather_logprobs(ptr<bf16>(h), h.stride(0), ptr<bf16>(w), w.stride(0), h.size(0), h.size(1), w.size(0),
                  ptr<int64_t>(ids), ids.size(1), ptr<float>(lse), ptr<float>(lp), cur_stream());
  count();
}

void scatter_add_rows_(Tensor dz, Tensor ids, Tensor g) {
  CHECK_CUDA(dz);
  CHECK_BF16(dz);
  TORCH_CHECK(dz.dim() == 2 && dz.stride(1) == 1, "scatter_add_rows: dz [T, V] row-major");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == dz.size(0),
              "scatter_add_rows: ids [T, K] int64");
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && g.numel() == ids.numel(),
              "scatter_add_rows: g [T, K] fp32");
  const c10::cuda::CUDAGuard guard(dz.device());
  scatter_add_rows(ptr<bf16>(dz), dz.stride(0), dz.size(0), dz.size(1), ptr<int64_t>(ids), ptr<float>(g),
                   ids.size(1), cur_stream());
  count();
}

// ─── expert parallelism over peer memory ────────────────────────────────────
using ull = unsigned long long;
const ull* tab(const Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kLong && t.is_cuda(), "peer pointer tables are int64 CUDA tensors");
  return reinterpret_cast<const ull*>(t.data_ptr());
}
const ull* otab(const c10::optional<Tensor>& t) { return (t.has_value() && t->defined()) ? tab(*t) : nullptr; }

void ep_dispatch_(Tensor rows, int64_t row_div, Tensor experts, Tensor slot_of, Tensor off, Tensor cnt,
                  int64_t e_local, int64_t rank, int64_t world, int64_t cap, Tensor recv_x,
                  c10::optional<Tensor> recv_meta, c10::optional<Tensor> recv_idx, c10::optional<Tensor> recv_cnt) {
  CHECK_CUDA(rows);
  CHECK_BF16(rows);
  CHECK_CONTIG(rows);
  TORCH_CHECK(off.numel() == world + 1 && cnt.numel() == world, "ep_dispatch: owner plan of world entries");
  TORCH_CHECK(rows.size(0) * row_div >= experts.numel(), "ep_dispatch: too few rows");
  const c10::cuda::CUDAGuard guard(rows.device());
  EpDispatchArgs a;
  a.rows = ptr<bf16>(rows);
  a.row_div = (int)row_div;
  a.experts = ptr<int>(experts);
  a.n = experts.numel();
  a.slot_of = ptr<int>(slot_of);
  a.off = ptr<int>(off);
  a.cnt = ptr<int>(cnt);
  a.e_local = (int)e_local;
  a.rank = (int)rank;
  a.world = (int)world;
  a.cap = (int)cap;
  a.D = rows.size(1);
  a.recv_x = tab(recv_x);
  a.recv_meta = otab(recv_meta);
  a.recv_idx = otab(recv_idx);
  a.recv_cnt = otab(recv_cnt);
  ep_dispatch(a, cur_stream());
  count();
}

void ep_recv_ids_(Tensor meta, Tensor cnt, int64_t world, int64_t cap, int64_t e_local, Tensor ids) {
  CHECK_CUDA(meta);
  TORCH_CHECK(meta.numel() >= world * cap && ids.numel() >= world * cap, "ep_recv_ids: sizes");
  const c10::cuda::CUDAGuard guard(meta.device());
  ep_recv_ids(ptr<int>(meta), ptr<int>(cnt), (int)world, (int)cap, (int)e_local, ptr<int>(ids), cur_stream());
  count();
}

void ep_return_(Tensor y, Tensor ids, Tensor slot_of, Tensor idx, int64_t world, int64_t cap, int64_t n_src_cap,
                Tensor ret) {
  CHECK_CUDA(y);
  CHECK_BF16(y);
  CHECK_CONTIG(y);
  TORCH_CHECK(ids.numel() >= world * cap && slot_of.numel() >= world * cap && idx.numel() >= world * cap,
              "ep_return: sizes");
  const c10::cuda::CUDAGuard guard(y.device());
  ep_return(ptr<bf16>(y), y.size(0), ptr<int>(ids), ptr<int>(slot_of), ptr<int>(idx), (int)world, (int)cap,
            (int)n_src_cap, y.size(1), tab(ret), cur_stream());
  count();
}

void gather_rows_(Tensor row_src, Tensor off, Tensor src, Tensor dst) {
  CHECK_CUDA(src);
  CHECK_BF16(src);
  CHECK_BF16(dst);
  CHECK_CONTIG(src);
  CHECK_CONTIG(dst);
  TORCH_CHECK(src.size(1) == dst.size(1) && row_src.numel() >= dst.size(0), "gather_rows: shapes");
  const c10::cuda::CUDAGuard guard(src.device());
  gather_rows(ptr<int>(row_src), ptr<int>(off) + (off.numel() - 1), ptr<bf16>(src), src.size(0), src.size(1),
              ptr<bf16>(dst), dst.size(0), cur_stream());
  count();
}

int64_t symm_alloc_(int64_t nbytes) {
  const c10::cuda::CUDAGuard guard(at::cuda::current_device());
  return reinterpret_cast<int64_t>(symm_malloc((size_t)nbytes));
}
void symm_free_(int64_t p) { symm_free(reinterpret_cast<void*>(p)); }
pybind11::bytes symm_export_(int64_t p) { return pybind11::bytes(symm_export(reinterpret_cast<void*>(p))); }
int64_t symm_import_(pybind11::bytes h) { return reinterpret_cast<int64_t>(symm_import(std::string(h))); }
void symm_close_(int64_t p) { symm_close(reinterpret_cast<void*>(p)); }

// A tensor view of ``numel`` elements at ``ptr + offset_bytes`` (no ownership: the heap object keeps the memory).
Tensor symm_view_(int64_t ptr, int64_t offset_bytes, int64_t numel, c10::ScalarType dtype) {
  auto opts = torch::TensorOptions().device(torch::kCUDA, at::cuda::current_device()).dtype(dtype);
  return torch::from_blob(reinterpret_cast<char*>(ptr) + offset_bytes, {numel}, opts);
}

void symm_barrier_(Tensor flag_ptrs, int64_t rank, int64_t world, int64_t epoch, double timeout_s) {
  TORCH_CHECK(flag_ptrs.scalar_type() == at::kLong && flag_ptrs.is_cuda(), "flag_ptrs: int64 CUDA tensor");
  symm_barrier(reinterpret_cast<const unsigned long long*>(flag_ptrs.data_ptr()), (int)rank, (int)world,
               (unsigned)epoch, timeout_s, ptr<int>(scratch(0, 0).err), cur_stream());
  count();
}

void fsdp_gather_(Tensor ptrs, int64_t off_bytes, int64_t bytes, Tensor dst) {
  TORCH_CHECK(ptrs.scalar_type() == at::kLong && ptrs.is_cuda(), "ptrs: int64 CUDA tensor");
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous() && dst.numel() * dst.element_size() >= ptrs.numel() * bytes,
              "fsdp_gather: dst holds world x bytes");
  const c10::cuda::CUDAGuard guard(dst.device());
  fsdp_gather(reinterpret_cast<const unsigned long long*>(ptrs.data_ptr()), off_bytes, bytes, (int)ptrs.numel(),
              dst.data_ptr(), cur_stream());
  count();
}

void fsdp_reduce_(Tensor ptrs, int64_t off_bytes, int64_t n, int64_t rank, Tensor dst) {
  TORCH_CHECK(ptrs.scalar_type() == at::kLong && ptrs.is_cuda(), "ptrs: int64 CUDA tensor");
  CHECK_F32(dst);
  TORCH_CHECK(dst.is_contiguous() && dst.numel() >= n, "fsdp_reduce: dst holds n fp32");
  const c10::cuda::CUDAGuard guard(dst.device());
  fsdp_reduce(reinterpret_cast<const unsigned long long*>(ptrs.data_ptr()), off_bytes, n, (int)rank,
              (int)ptrs.numel(), ptr<float>(dst), cur_stream());
  count();
}

void symm_dp_adamw_(Tensor grad_ptrs, c10::optional<Tensor> master_ptrs, c10::optional<Tensor> compute_ptrs,
                    Tensor flag_ptrs,
                    Tensor slot_ptrs, Tensor master_local, Tensor grad_local, Tensor exp_avg, Tensor exp_avg_sq,
                    Tensor scalars, int64_t rank, int64_t world, int64_t lo, int64_t hi, int64_t epoch, double max_norm,
                    double lr, double b1, double b2, double eps, double wd, int64_t step, double timeout_s) {
  TORCH_CHECK(scalars.scalar_type() == at::kFloat && scalars.numel() >= 2, "scalars: fp32 [2] (sumsq, norm)");
  TORCH_CHECK(exp_avg.numel() >= hi - lo && exp_avg_sq.numel() >= hi - lo,
              "symm_dp_adamw: the moments are this rank's shard [lo, hi)");
  SymmAdamWArgs a;
  auto tab = [](const Tensor& t) { return reinterpret_cast<const unsigned long long*>(t.data_ptr()); };
  a.grad_ptrs = tab(grad_ptrs);
  a.master_ptrs = master_ptrs.has_value() && master_ptrs->defined() ? tab(*master_ptrs) : nullptr;
  a.compute_ptrs = compute_ptrs.has_value() && compute_ptrs->defined() ? tab(*compute_ptrs) : nullptr;
  TORCH_CHECK(a.master_ptrs || a.compute_ptrs, "symm_dp_adamw: a sharded master needs the bf16 compute table");
  a.flag_ptrs = tab(flag_ptrs);
  a.slot_ptrs = tab(slot_ptrs);
  a.master_local = ptr<float>(master_local);
  a.local_grad = ptr<float>(grad_local);
  a.exp_avg = ptr<float>(exp_avg);
  a.exp_avg_sq = ptr<float>(exp_avg_sq);
  a.sumsq = ptr<float>(scalars);
  a.norm = ptr<float>(scalars) + 1;
  a.err = ptr<int>(scratch(0, 0).err);
  a.rank = (int)rank;
  a.world = (int)world;
  a.lo = lo;
  a.hi = hi;
  a.epoch = (unsigned)epoch;
  a.max_norm = (float)max_norm;
  a.lr = (float)lr;
  a.b1 = (float)b1;
  a.b2 = (float)b2;
  a.eps = (float)eps;
  a.wd = (float)wd;
  a.step = (int)step;
  a.timeout_s = timeout_s;
  symm_dp_adamw_step(a, cur_stream());
  count(5);
}

// Whole-step decode kernel. ``table``: int64 [L, 8] device table of per-layer pointers
// (attn_norm, bqkv, q_norm, k_norm, mlp_norm, 0, 0, 0); ``w*0``: layer 0's matrices, the other
// layers at ``layer_stride`` elements; ``ws``: [x, xg, sumsq, acc, q, apart, ao, act, h, ctr];
// ``gemm``: (T, KB, s) of QKV, o_proj, gate/up, down.
void mega_decode_(Tensor table, Tensor wqkv0, Tensor wo0, Tensor w130, Tensor w20, int64_t layer_stride, Tensor embed,
                  Tensor final_norm, Tensor kv, Tensor tok, Tensor pos, Tensor seq_lens, Tensor slot,
                  Tensor block_table, std::vector<Tensor> ws, int64_t B, int64_t MP, int64_t Hq, int64_t Hkv,
                  double eps, double scale, double theta, std::vector<int64_t> gemm, int64_t grid,
                  c10::optional<Tensor> trace) {
  TORCH_CHECK(ws.size() == 10 && gemm.size() == 12, "mega_decode: 10 workspaces and 4 x (T, KB, s)");
  TORCH_CHECK(tok.scalar_type() == at::kLong && slot.scalar_type() == at::kLong, "tok / slot must be int64");
  TORCH_CHECK(pos.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  block_table.scalar_type() == at::kInt, "pos / seq_lens / block_table must be int32");
  TORCH_CHECK(kv.dim() == 6 && kv.size(4) == kMegaPage && kv.size(5) == kMegaHeadDim, "kv: [L, 2, pages, Hkv, 64, 128]");
  const c10::cuda::CUDAGuard guard(kv.device());
  const int L = (int)kv.size(0);
  const int D = (int)embed.size(1);
  const int qkv_dim = (int)wqkv0.size(0), q_dim = (int)wo0.size(1), F = (int)w20.size(1);
  TORCH_CHECK(wqkv0.size(1) == D && wo0.size(0) == D && w130.size(0) == 2 * F && w130.size(1) == D && w20.size(0) == D,
              "mega_decode: weight shapes");
  TORCH_CHECK(table.size(0) == L && table.size(1) == 8, "mega_decode: layer table [L, 8]");
  MegaArgs a = {};
  a.n_layers = L;
  a.D = D;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.F = F;
  a.qkv_dim = qkv_dim;
  a.q_dim = q_dim;
  a.B = (int)B;
  a.MP = (int)MP;
  a.eps = (float)eps;
  a.qk_scale_log2 = (float)(scale * 1.4426950408889634);
  Tensor inv = inv_freq_table(kMegaHeadDim, theta, kv.device());
  a.inv_freq = ptr<float>(inv);
  a.layers = reinterpret_cast<const MegaLayer*>(table.data_ptr());
  a.embed = ptr<bf16>(embed);
  a.final_norm = ptr<bf16>(final_norm);
  a.tok = ptr<int64_t>(tok);
  a.pos = ptr<int>(pos);
  a.seq_lens = ptr<int>(seq_lens);
  a.slot = ptr<int64_t>(slot);
  a.block_table = ptr<int>(block_table);
  a.max_pages = (int)block_table.size(1);
  a.n_cache_pages = (int)kv.size(2);
  a.kv = ptr<bf16>(kv);
  a.x = ptr<float>(ws[0]);
  a.xg = ptr<bf16>(ws[1]);
  a.sumsq = ptr<float>(ws[2]);
  a.acc = ptr<float>(ws[3]);
  a.q = ptr<bf16>(ws[4]);
  a.apart = ptr<float>(ws[5]);
  a.ao = ptr<bf16>(ws[6]);
  a.act = ptr<bf16>(ws[7]);
  a.h = ptr<bf16>(ws[8]);
  a.ctr = reinterpret_cast<unsigned*>(ws[9].data_ptr());
  a.err = ptr<int>(scratch(0, 0).err);
  a.flags = std::getenv("MESHY_MEGA_FLAGS") ? std::atoi(std::getenv("MESHY_MEGA_FLAGS")) : 0;
  a.trace = trace.has_value() && trace->defined() ? reinterpret_cast<unsigned long long*>(trace->data_ptr()) : nullptr;
  if (a.trace) TORCH_CHECK(trace->numel() >= (int64_t)(2 + 5 * L) * grid * 8, "mega_decode: trace buffer too small");
  TORCH_CHECK(ws[9].numel() >= kMegaCtrWords, "mega_decode: counter workspace too small");
  TORCH_CHECK(ws[5].numel() >= (int64_t)mega_apart_floats((int)grid), "mega_decode: partials workspace too small");
  MegaGemm* gs[4] = {&a.g_qkv, &a.g_o, &a.g_gu, &a.g_dn};
  for (int i = 0; i < 4; ++i) *gs[i] = {(int)gemm[3 * i], (int)gemm[3 * i + 1], (int)gemm[3 * i + 2]};
  const int64_t ls = layer_stride * 2;  // bytes
  CUtensorMap m_qkv = make_map_bf16_3d(wqkv0.data_ptr(), D, qkv_dim, L, (int64_t)D * 2, ls, 64, 128);
  CUtensorMap m_o = make_map_bf16_3d(wo0.data_ptr(), q_dim, D, L, (int64_t)q_dim * 2, ls, 64, 128);
  CUtensorMap m_gu = make_map_bf16_3d(w130.data_ptr(), D, 2 * F, L, (int64_t)D * 2, ls, 64, 128);
  CUtensorMap m_dn = make_map_bf16_3d(w20.data_ptr(), F, D, L, (int64_t)F * 2, ls, 64, 128);
  CUtensorMap m_xg = make_map_bf16(ws[1].data_ptr(), MP, D, D, 64, (int)MP);
  CUtensorMap m_ao = make_map_bf16(ws[6].data_ptr(), MP, q_dim, q_dim, 64, (int)MP);
  CUtensorMap m_act = make_map_bf16(ws[7].data_ptr(), MP, F, F, 64, (int)MP);
  const int64_t kv_rows = kv.numel() / kMegaHeadDim;
  TORCH_CHECK(kv_rows < (int64_t)1 << 31, "mega_decode: KV cache too large for 32-bit TMA row coordinates");
  CUtensorMap m_kv = make_map_bf16(kv.data_ptr(), kv_rows, kMegaHeadDim, kMegaHeadDim, 64, kMegaPage);
  mega_decode_launch(a, m_qkv, m_o, m_gu, m_dn, m_xg, m_ao, m_act, m_kv, (int)grid, cur_stream());
  count();
}

int64_t mega_grid_() { return mega_grid(); }
int64_t mega_apart_floats_(int64_t grid) { return (int64_t)mega_apart_floats((int)grid); }
int64_t mega_ctr_words_() { return kMegaCtrWords; }

int64_t device_error() {
  auto& s = scratch(0, 0);
  return s.err.item<int>();
}
void clear_device_error() { scratch(0, 0).err.zero_(); }
int64_t launch_count() { return g_launches.load(); }

}  // namespace

namespace meshy {
void register_vmm(pybind11::module_& m);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  meshy::register_vmm(m);
  m.doc() = "meshy_b200 sm_100a kernel library";
  m.def("gemm", &gemm, "tcgen05 GEMM with fused epilogues");
  m.def("mega_decode", &mega_decode_, "one decode step of a dense decoder in one persistent cooperative kernel",
        pybind11::arg("table"), pybind11::arg("wqkv0"), pybind11::arg("wo0"), pybind11::arg("w130"), pybind11::arg("w20"),
        pybind11::arg("layer_stride"), pybind11::arg("embed"), pybind11::arg("final_norm"), pybind11::arg("kv"),
        pybind11::arg("tok"), pybind11::arg("pos"), pybind11::arg("seq_lens"), pybind11::arg("slot"),
        pybind11::arg("block_table"), pybind11::arg("ws"), pybind11::arg("B"), pybind11::arg("MP"), pybind11::arg("Hq"),
        pybind11::arg("Hkv"), pybind11::arg("eps"), pybind11::arg("scale"), pybind11::arg("theta"), pybind11::arg("gemm"),
        pybind11::arg("grid"), pybind11::arg("trace") = pybind11::none());
  m.def("mega_grid", &mega_grid_);
  m.def("mega_apart_floats", &mega_apart_floats_);
  m.def("mega_ctr_words", &mega_ctr_words_);

  m.def("gemm_norm_prep", &gemm_norm_prep, "decode: residual GEMM that also prepares the next RMSNorm");
  m.def("gemm_norm_scaled", &gemm_norm_scaled, "decode: GEMM on a prepared RMSNorm input, rows scaled by rstd");
  m.def("gemm_qkv_rope", &gemm_qkv_rope, "decode: QKV GEMM with RoPE / QK-norm and the KV-cache write fused");
  m.def("gemm_norm", &gemm_norm, "decode: fused input RMSNorm + small-M GEMM (returns False if not eligible)");
  m.def("paged_decode_trace",
        [](c10::optional<Tensor> buf) {
          if (buf && buf->defined()) {
            TORCH_CHECK(buf->scalar_type() == at::kLong && buf->is_cuda() && buf->dim() == 3 && buf->size(-1) == 8 &&
                            buf->size(-2) == 1024,
                        "paged_decode_trace: int64 [slots, 1024, 8]");
            paged_decode_trace(reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>()), (int)buf->size(0));
          } else {
            paged_decode_trace(nullptr, 0);
          }
        },
        "record per-CTA timelines of the decode-attention launches (None stops)", py::arg("buf") = py::none());
  m.def("gemm_small_trace",
        [](c10::optional<Tensor> buf) {
          if (buf.has_value() && buf->defined()) {
            TORCH_CHECK(buf->scalar_type() == at::kLong && buf->is_contiguous() && buf->size(-1) == 8 &&
                            buf->size(-2) == 160, "gemm_small_trace: int64 [slots, 160, 8]");
            gemm_small_trace(reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>()), (int)buf->size(0));
          } else {
            gemm_small_trace(nullptr, 0);
          }
        },
        "record the timelines of the next small-M GEMM launches into int64 [slots, 160, 8] (None: stop)");
  m.def("gemm_small_config", [](int64_t enabled, int64_t cluster) { gemm_small_config((int)enabled, (int)cluster); },
        "small-M GEMM switches: enabled (1/0, -1 keep), cluster split-K size (0 auto, -1 keep)");
  m.def("swiglu_bwd", &swiglu_bwd_);
  m.def("filtered_sample", &filtered_sample_, "top-k / top-p / temperature sampling over fp32 logits");
  m.def("value_head_fwd", &value_head_fwd_, "critic value head + clipped value loss (values, dL/dv, loss sum)");
  m.def("value_head_bwd", &value_head_bwd_, "critic value head backward: dh, dw, db");
  m.def("topk_logprobs", &topk_logprobs_, "K largest fp32 logits per row (sorted), log-probabilities, lse");
  m.def("gather_logprobs", &gather_logprobs_, "log-probabilities of given ids from hidden rows and the LM head");
  m.def("scatter_add_rows", &scatter_add_rows_, "dz[t, ids[t, k]] += g[t, k] on bf16 logit gradients");
  m.def("moe_route", &moe_route_, "router softmax + top-k (+ renormalisation)");
  m.def("moe_route_bwd", &moe_route_bwd_, "router backward: d logits from d weights");
  m.def("moe_plan", &moe_plan_, "device-side expert plan: counts, 128-aligned offsets, slots, gather");
  m.def("moe_zero_pad", &moe_zero_pad_, "zero the padding rows of every expert segment");
  m.def("moe_combine", &moe_combine_, "weighted gather-sum of expert outputs per token");
  m.def("moe_combine_bwd", &moe_combine_bwd_, "combine backward: expert-row gradients and routing-weight gradients");
  m.def("gemm_grouped", &gemm_grouped, "grouped tcgen05 GEMM over 128-aligned expert segments");
  m.def("ep_dispatch", &ep_dispatch_, "expert-parallel dispatch: P2P stores of token rows into the owners' regions");
  m.def("ep_recv_ids", &ep_recv_ids_, "received rows -> local expert ids (-1 past each source's count)");
  m.def("ep_return", &ep_return_, "expert-parallel return: P2P stores of expert rows into the sources' buffers");
  m.def("gather_rows", &gather_rows_, "dst[r] = src[row_src[r]] up to the plan's end (zero padding rows)");
  m.def("rmsnorm_fwd", &rmsnorm_fwd_);
  m.def("rmsnorm_bwd", &rmsnorm_bwd_);
  m.def("qkv_rope_fwd", &qkv_rope_fwd_);
  m.def("qkv_rope_bwd", &qkv_rope_bwd_);
  m.def("qkv_rope_cache", &qkv_rope_cache_, "QK-norm + RoPE with K/V written straight into the paged cache");
  m.def("flash_attn_fwd", &flash_attn_fwd_);
  m.def("flash_attn_bwd", &flash_attn_bwd_);
  m.def("flash_attn_fwd_kv", &flash_attn_fwd_kv_, "causal attention of query chunks against a separate key stream");
  m.def("flash_attn_bwd_kv", &flash_attn_bwd_kv_);
  m.def("flash_attn_fwd_cp_peer", &flash_attn_fwd_cp_peer,
        "context-parallel attention forward reading every rank's K/V in place over NVLink (no all-gather)");
  m.def("lmhead_logprob_fwd", &lmhead_logprob_fwd);
  m.def("lmhead_dlogits", &lmhead_dlogits);
  m.def("lmhead_sample", &lmhead_sample);
  m.def("lmhead_sample_small", &lmhead_sample_small,
        "small-M LM-head sampler (<= 64 rows); returns false when not eligible");
  m.def("decode_sample_advance", &decode_sample_advance,
        "decode step tail: small-M LM-head sampler + merge fused with the row advance; false when not eligible");
  m.def("embedding_fwd", &embedding_fwd_);
  m.def("embedding_bwd", &embedding_bwd_);
  m.def("sq_norm", &sq_norm_);
  m.def("adamw_flat", &adamw_flat_);
  m.def("ppo_loss_fused", &ppo_loss_fused_);
  m.def("gae_scan", &gae_scan_);
  m.def("kv_write", &kv_write_);
  m.def("paged_attention", &paged_attention_, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_table"), py::arg("seq_lens"), py::arg("out"), py::arg("scale"), py::arg("workspace"),
        py::arg("decode_step") = false,
        "paged decode attention; decode_step: the kernel before wrote only each sequence's newest K/V row");
  m.def("paged_decode_force_splits", [](int64_t n) { paged_decode_force_splits((int)n); },
        "decode attention split count override (0 = heuristic); for tests and benchmarks");
  m.def("decode_advance", &decode_advance_);
  m.def("cast_copy", &cast_copy);
  m.def("symm_alloc", &symm_alloc_, "cudaMalloc a symmetric-heap buffer (zeroed); returns the pointer");
  m.def("symm_free", &symm_free_);
  m.def("symm_export", &symm_export_, "CUDA IPC handle bytes of a symmetric-heap buffer");
  m.def("symm_import", &symm_import_, "map a peer's symmetric-heap buffer; returns the local pointer");
  m.def("symm_close", &symm_close_);
  m.def("symm_view", &symm_view_, "non-owning tensor view into a symmetric-heap buffer");
  m.def("symm_barrier", &symm_barrier_, "device barrier over the ranks' flag arrays (bounded wait)");
  m.def("fsdp_gather", &fsdp_gather_, "gather every rank's shard of a symmetric region (peer loads)");
  m.def("fsdp_reduce", &fsdp_reduce_, "this rank's shard of the sum of the ranks' fp32 regions (peer loads)");
  m.def("symm_dp_adamw", &symm_dp_adamw_,
        "fused DP optimiser step over NVLink: reduce-scatter + grad norm + AdamW + all-gather by P2P stores");
  m.def("device_error", &device_error);
  m.def("clear_device_error", &clear_device_error);
  m.def("launch_count", &launch_count, "kernels launched by this library so far (host-side count)");
}
