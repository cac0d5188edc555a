// Expert-parallel token exchange over NVLink peer memory (sm_100a).
//
// Expert e lives on EP rank e / E_local. Every rank keeps, in symmetric memory mapped by all its peers,
// one receive region per source rank: recv_x[src][cap][D] rows, recv_meta[src][cap] (local expert id of
// each row), recv_idx[src][cap] (the row's assignment index t * k + j at the source) and recv_cnt[src].
// A source places its assignments for owner o at the positions given by its owner plan (the same
// device-side stable plan the local expert layer uses, over owner ids): position = slot - off[o].
//
//   dispatch   one warp per assignment copies its token row (16-byte vectors) straight into the owner's
//              region with plain st.global to the peer pointer; block 0 publishes the per-owner counts;
//   barrier    symm_barrier (release/acquire flags, bounded spin) -- afterwards every owner holds all
//              rows sent to it;
//   recv ids   the owner turns its regions into one id list (-1 past each source's count) for the plan of
//              its local experts; the grouped tcgen05 GEMMs then run on its own memory only;
//   return     one warp per received row writes the expert output back into the source's return buffer at
//              the row's assignment index (P2P store); a second barrier completes the exchange.
//
// The backward pass runs the same two exchanges in the same directions (gradients of the returned rows go
// out, gradients of the token rows come back). No TMA and no multicast touch peer memory; every wait is
// the bounded barrier of symm.cu.
#include <cuda_runtime.h>

#include "../include/common.cuh"
#include "../include/sm100.cuh"
#include "ep.h"

namespace meshy {

namespace {

__global__ void ep_dispatch_kernel(const bf16* __restrict__ rows, int row_div, const int* __restrict__ experts, int n,
                                   const int* __restrict__ slot_of, const int* __restrict__ off,
                                   const int* __restrict__ cnt, int e_local, int rank, int world, int cap, int D,
                                   const unsigned long long* __restrict__ recv_x,
                                   const unsigned long long* __restrict__ recv_meta,
                                   const unsigned long long* __restrict__ recv_idx,
                                   const unsigned long long* __restrict__ recv_cnt) {
  pdl_wait();
  if (blockIdx.x == 0 && threadIdx.x < world && recv_cnt) {
    int* c = reinterpret_cast<int*>(recv_cnt[threadIdx.x]);
    c[rank] = cnt[threadIdx.x];
  }
  const int warps = blockDim.x / 32;
  const int i = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (i >= n) return;
  const int e = experts[i];
  const int o = e / e_local;
  if (e < 0 || o >= world) return;
  const int pos = slot_of[i] - off[o];
  if (pos < 0 || pos >= cap) return;
  const size_t row = (size_t)rank * cap + pos;
  const uint4* src = reinterpret_cast<const uint4*>(rows + (size_t)(i / row_div) * D);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(recv_x[o]) + row * D);
  for (int v = lane; v < D / 8; v += 32) dst[v] = src[v];
  if (lane == 0) {
    if (recv_meta) reinterpret_cast<int*>(recv_meta[o])[row] = e - o * e_local;
    if (recv_idx) reinterpret_cast<int*>(recv_idx[o])[row] = i;
  }
}

__global__ void ep_recv_ids_kernel(const int* __restrict__ meta, const int* __restrict__ cnt, int world, int cap,
                                   int e_local, int* __restrict__ ids) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= world * cap) return;
  const int s = i / cap, p = i - s * cap;
  const int c = cnt[s];
  int id = -1;
  if (p < c && c <= cap) {
    id = meta[i];
    if (id < 0 || id >= e_local) id = -1;
  }
  ids[i] = id;
}

__global__ void ep_return_kernel(const bf16* __restrict__ y, int y_rows, const int* __restrict__ ids,
                                 const int* __restrict__ slot_of, const int* __restrict__ idx, int world, int cap,
                                 int n_src_cap, int D, const unsigned long long* __restrict__ ret) {
  pdl_wait();
  const int warps = blockDim.x / 32;
  const int i = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (i >= world * cap || ids[i] < 0) return;
  const int s = i / cap;
  const int r = slot_of[i];
  const int a = idx[i];
  if (r < 0 || r >= y_rows || a < 0 || a >= n_src_cap) return;
  const uint4* src = reinterpret_cast<const uint4*>(y + (size_t)r * D);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(ret[s]) + (size_t)a * D);
  for (int v = lane; v < D / 8; v += 32) dst[v] = src[v];
}

// dst[row] = src[row_src[row]] for rows below off[E] (row_src = -1: zero row); one warp per row.
__global__ void gather_rows_kernel(const int* __restrict__ row_src, const int* __restrict__ off_end,
                                   const bf16* __restrict__ src, int src_rows, int D, bf16* __restrict__ dst,
                                   int rows) {
  pdl_wait();
  const int warps = blockDim.x / 32;
  const int r = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= rows || r >= *off_end) return;
  const int s = row_src[r];
  uint4* d = reinterpret_cast<uint4*>(dst + (size_t)r * D);
  if (s < 0 || s >= src_rows) {
    for (int v = lane; v < D / 8; v += 32) d[v] = make_uint4(0, 0, 0, 0);
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(src + (size_t)s * D);
    for (int v = lane; v < D / 8; v += 32) d[v] = p[v];
  }
}

}  // namespace

void ep_dispatch(const EpDispatchArgs& a, cudaStream_t st) {
  MESHY_CHECK(a.D % 8 == 0, "ep_dispatch: D must be a multiple of 8");
  MESHY_CHECK(a.n <= a.cap, "ep_dispatch: more assignments than the receive regions hold");
  MESHY_CHECK(a.world <= 1024, "ep_dispatch: EP group too large");
  const int threads = 256, warps = threads / 32;
  const int grid = std::max(1, (a.n + warps - 1) / warps);
  launch_pdl(ep_dispatch_kernel, dim3(grid), dim3(threads), 0, st, a.rows, a.row_div, a.experts, a.n, a.slot_of,
             a.off, a.cnt, a.e_local, a.rank, a.world, a.cap, a.D, a.recv_x, a.recv_meta, a.recv_idx, a.recv_cnt);
}

void ep_recv_ids(const int* meta, const int* cnt, int world, int cap, int e_local, int* ids, cudaStream_t st) {
  const int n = world * cap;
  launch_pdl(ep_recv_ids_kernel, dim3((n + 255) / 256), dim3(256), 0, st, meta, cnt, world, cap, e_local, ids);
}

void ep_return(const bf16* y, int y_rows, const int* ids, const int* slot_of, const int* idx, int world, int cap,
               int n_src_cap, int D, const unsigned long long* ret, cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0, "ep_return: D must be a multiple of 8");
  const int threads = 256, warps = threads / 32;
  const int n = world * cap;
  launch_pdl(ep_return_kernel, dim3((n + warps - 1) / warps), dim3(threads), 0, st, y, y_rows, ids, slot_of, idx,
             world, cap, n_src_cap, D, ret);
}

void gather_rows(const int* row_src, const int* off_end, const bf16* src, int src_rows, int D, bf16* dst, int rows,
                 cudaStream_t st) {
  MESHY_CHECK(D % 8 == 0, "gather_rows: D must be a multiple of 8");
  const int threads = 256, warps = threads / 32;
  launch_pdl(gather_rows_kernel, dim3((rows + warps - 1) / warps), dim3(threads), 0, st, row_src, off_end, src,
             src_rows, D, dst, rows);
}

}  // namespace meshy
