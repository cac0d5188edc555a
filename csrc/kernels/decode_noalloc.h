// Allocation-free entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference framework: it is an
// addition of this library for callers that cannot allocate device memory.
// Such callers include a C or C++ host that embeds the kernels without
// PyTorch (so it has no caching allocator to borrow from), a serving process
// that has already handed nearly all of HBM to its KV-cache pool, and a
// latency-critical decode loop where cudaMalloc's implicit device
// synchronisation is not acceptable.
//
// It runs the split-KV decode kernels of meshy::paged_decode, whose regular
// entry point takes the partial buffer from the caller.  This one uses a fixed
// file-scope device array of MESHY_PAGED_DECODE_NOALLOC_SCRATCH_BYTES instead;
// every GPU that loads the library keeps that array until the process exits.
// (``meshy_b200._C.paged_attention`` computes the same op with the TMA /
// cluster-reduction kernel of decode_attn.cu.)
//
// Contract:
//  * All pointers are device pointers on the current device; ``stream`` is a
//    cudaStream_t (may be null for the legacy default stream).
//  * q [batch, n_q_heads, head_dim] bf16; k_cache / v_cache
//    [n_pages, n_kv_heads, page_size, head_dim] bf16; block_table
//    [batch, max_pages] int32; seq_lens [batch] int32; out like q.
//  * Layout preconditions, checked before anything is launched (return code
//    1 and a message otherwise): page_size == 64, head_dim 64 or 128,
//    n_q_heads a multiple of n_kv_heads with at most 16 query heads per KV
//    head.
//  * Each row reads at most max_pages block-table entries, however large its
//    seq_lens value.  The kernel does not know the cache's page count, so the
//    caller guarantees that every block-table entry a row reads (the first
//    ceil(seq_lens[b] / page_size) of row b, capped at max_pages) is a valid
//    page index of k_cache / v_cache.
//  * n_split = 0 picks the split count automatically (capped so the partials
//    fit the array); n_split > 0 is used as given and a request whose
//    partials do not fit is rejected with an error.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress; make that first call before any stream capture.
//  * Every call shares the one array: calls that can overlap on the GPU (on
//    different streams, or from different host threads) race and must be
//    serialised by the caller.
//  * Returns 0 on success and a non-zero code otherwise;
//    meshy_noalloc_last_error() then describes the failure (per host thread).
//  * Calls no cudaMalloc, cudaFree or other allocating routine.
#pragma once
#include <cstddef>

#ifdef __cplusplus
extern "C" {
#endif

// Size of the file-scope scratch array (fp32 split partials), in bytes.
#define MESHY_PAGED_DECODE_NOALLOC_SCRATCH_BYTES (8u << 20)

int meshy_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                               const int* seq_lens, void* out, int batch, int n_q_heads, int n_kv_heads,
                               int head_dim, int page_size, int max_pages, int n_split, float scale, void* stream);

// Bytes of scratch one call with these sizes needs (0 when n_split == 1).
size_t meshy_paged_decode_noalloc_scratch_need(int batch, int n_q_heads, int head_dim, int n_split);

// Capacity of the scratch array in bytes.
size_t meshy_paged_decode_noalloc_scratch_capacity(void);

// Message of the last failed call on this host thread ("" if none).
const char* meshy_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
