// Expert-parallel token exchange over NVLink peer memory (ep.cu).
#pragma once
#include <cuda_runtime.h>

#include "../include/common.cuh"

namespace meshy {

struct EpDispatchArgs {
  const bf16* rows = nullptr;  // source rows; assignment i sends rows[i / row_div]
  int row_div = 1;
  const int* experts = nullptr;  // [n] global expert id of each assignment
  int n = 0;
  const int* slot_of = nullptr;  // owner plan of the assignments (moe_plan over owner ids)
  const int* off = nullptr;      // [world + 1]
  const int* cnt = nullptr;      // [world]
  int e_local = 1, rank = 0, world = 1, cap = 0, D = 0;
  const unsigned long long* recv_x = nullptr;     // [world] peer tables of the receive regions
  const unsigned long long* recv_meta = nullptr;  // (null: rows only)
  const unsigned long long* recv_idx = nullptr;
  const unsigned long long* recv_cnt = nullptr;
};

void ep_dispatch(const EpDispatchArgs& a, cudaStream_t st);
// ids[s * cap + p] = local expert id of received row p of source s, -1 past that source's count.
void ep_recv_ids(const int* meta, const int* cnt, int world, int cap, int e_local, int* ids, cudaStream_t st);
// For every valid received row i: ret[src(i)][idx[i]] = y[slot_of[i]] (P2P store into the source's buffer).
void ep_return(const bf16* y, int y_rows, const int* ids, const int* slot_of, const int* idx, int world, int cap,
               int n_src_cap, int D, const unsigned long long* ret, cudaStream_t st);
// dst[r] = src[row_src[r]] for r < *off_end (row_src < 0: zero row).
void gather_rows(const int* row_src, const int* off_end, const bf16* src, int src_rows, int D, bf16* dst, int rows,
                 cudaStream_t st);

}  // namespace meshy
