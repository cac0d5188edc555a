// Allocation-free variant of split-KV paged decode attention (no counterpart
// in the reference framework; the contract is in decode_noalloc.h).
//
// The split-KV decode kernels write per-split (m, l, O) partials that a second
// kernel merges.  Here those partials live in a file-scope device array
// instead of a buffer the caller or torch allocates.  Host code cannot use the
// array's name as a device address (in host code it names a host-side shadow
// symbol), so the first call on each device asks the runtime for the real
// device address once and caches it per device ordinal.
//
// Nothing in the array has to start at zero: every split CTA writes all of
// its partial slots (an empty split writes m = -inf, l = 0, O = 0) before the
// merge kernel of the same call reads them, so leftovers from an earlier call
// are never read.
#include <cuda_runtime.h>

#include <exception>
#include <mutex>
#include <string>

#include "../include/common.cuh"
#include "attention.h"
#include "decode_noalloc.h"

namespace {

constexpr size_t kScratchFloats = MESHY_PAGED_DECODE_NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_paged_decode_scratch[kScratchFloats];

std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};
thread_local std::string g_last_error;

int fail(const std::string& msg, int code) {
  g_last_error = msg;
  return code;
}

// Device address of the scratch array on the current device (looked up once).
int scratch_ptr(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(std::string("cudaGetDevice failed: ") + cudaGetErrorString(e), 2);
  if (dev < 0 || dev >= kMaxDevices) return fail("device ordinal out of range", 2);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_paged_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e), 2);
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

size_t need_floats(int batch, int n_q_heads, int head_dim, int n_split) {
  if (n_split <= 1) return 0;
  return (size_t)batch * n_q_heads * n_split * (head_dim + 2);
}

}  // namespace

extern "C" size_t meshy_paged_decode_noalloc_scratch_need(int batch, int n_q_heads, int head_dim, int n_split) {
  return need_floats(batch, n_q_heads, head_dim, n_split) * sizeof(float);
}

extern "C" size_t meshy_paged_decode_noalloc_scratch_capacity(void) { return MESHY_PAGED_DECODE_NOALLOC_SCRATCH_BYTES; }

extern "C" const char* meshy_noalloc_last_error(void) { return g_last_error.c_str(); }

extern "C" int meshy_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                          const int* block_table, const int* seq_lens, void* out, int batch,
                                          int n_q_heads, int n_kv_heads, int head_dim, int page_size, int max_pages,
                                          int n_split, float scale, void* stream) {
  g_last_error.clear();
  if (batch < 0 || n_q_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || max_pages <= 0 || n_split < 0)
    return fail("invalid size argument", 1);
  if (n_q_heads % n_kv_heads != 0) return fail("n_q_heads must be a multiple of n_kv_heads", 1);
  if (page_size != 64) return fail("page_size must be 64 (got " + std::to_string(page_size) + ")", 1);
  if (head_dim != 64 && head_dim != 128)
    return fail("head_dim must be 64 or 128 (got " + std::to_string(head_dim) + ")", 1);
  if (n_q_heads / n_kv_heads > 16) return fail("at most 16 query heads per KV head", 1);
  if (batch == 0) return 0;
  if (!q || !k_cache || !v_cache || !block_table || !seq_lens || !out) return fail("null pointer argument", 1);
  int splits = n_split;
  if (splits == 0) {
    splits = meshy::paged_decode_splits(batch, n_kv_heads, max_pages);
    while (splits > 1 && need_floats(batch, n_q_heads, head_dim, splits) > kScratchFloats) --splits;
  } else if (need_floats(batch, n_q_heads, head_dim, splits) > kScratchFloats) {
    return fail("split partials need " + std::to_string(need_floats(batch, n_q_heads, head_dim, splits) * 4) +
                    " bytes of scratch; the fixed scratch array holds " +
                    std::to_string(MESHY_PAGED_DECODE_NOALLOC_SCRATCH_BYTES) + " bytes",
                3);
  }
  float* part = nullptr;
  int rc = scratch_ptr(&part);
  if (rc) return rc;
  try {
    meshy::paged_decode(static_cast<const meshy::bf16*>(q), static_cast<const meshy::bf16*>(k_cache),
                        static_cast<const meshy::bf16*>(v_cache), block_table, seq_lens,
                        static_cast<meshy::bf16*>(out), splits > 1 ? part : nullptr, batch, n_q_heads, n_kv_heads, head_dim, page_size,
                        max_pages, splits, scale, static_cast<cudaStream_t>(stream));
  } catch (const std::exception& ex) {
    return fail(ex.what(), 4);
  }
  return 0;
}
