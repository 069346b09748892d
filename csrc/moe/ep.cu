// Expert-parallel token movement over NVLink peer memory (sm_100a).
//
// One launch moves a list of row blocks between this GPU's memory and its peers'
// symmetric (CUDA-IPC) buffers: block b copies `nrows` rows of `row_bytes` bytes from
// src_table[src_rank[b]] + src_row[b] * src_ld to dst_table[dst_rank[b]] + dst_row[b] *
// dst_ld. With the source in a peer's buffer this is the dispatch pull (P2P loads of the
// tokens routed to this rank's experts); with the destination in a peer's buffer it is
// the combine push (P2P stores of expert outputs back to the token's rank). Rows are
// moved as 16-byte vectors, a warp per row stripe, all blocks of all peers in one grid
// (block list prefix-summed on the host), so the copies to / from every peer overlap.
// Plain 16-byte vector loads and stores through the NVLink mapping (no TMA).
//
// Replaces the reference's single-device token scatter / gather (layers/kernels/
// moe_kernels.py:45-148, never distributed) with the cross-GPU form of the same step.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>

#include "../common/tma.h"
#include "moe.h"

namespace ddb {
namespace {

__device__ __forceinline__ int find_block(const int* __restrict__ row_prefix, int nblocks, long r) {
  int lo = 0, hi = nblocks - 1;  // largest b with row_prefix[b] <= r
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (row_prefix[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(256) ep_copy_rows_kernel(EpCopyArgs a) {
  const int lanes_per_row = a.row_bytes / 16;
  const long total_vec = a.total_rows * lanes_per_row;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < total_vec; i += static_cast<long>(gridDim.x) * 256) {
    const long r = i / lanes_per_row;
    const int c = static_cast<int>(i % lanes_per_row);
    const int b = find_block(a.row_prefix, a.nblocks, r);
    const long k = r - a.row_prefix[b];
    const int* blk = a.blocks + 4 * b;   // 4-byte aligned only: plain loads
    const void* sb = a.src_table != nullptr ? a.src_table[blk[0]] : a.src_local;
    void* db = a.dst_table != nullptr ? a.dst_table[blk[2]] : a.dst_local;
    const char* src = reinterpret_cast<const char*>(sb) + (blk[1] + k) * a.src_ld + c * 16;
    char* dst = reinterpret_cast<char*>(db) + (blk[3] + k) * a.dst_ld + c * 16;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
}

}  // namespace

void ep_copy_rows(const EpCopyArgs& a, cudaStream_t stream) {
  if (a.total_rows <= 0 || a.nblocks <= 0) return;
  if (a.row_bytes % 16 != 0 || a.src_ld % 16 != 0 || a.dst_ld % 16 != 0)
    throw std::runtime_error("ep_copy_rows: rows and strides must be multiples of 16 bytes");
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const long vec = a.total_rows * (a.row_bytes / 16);
  const int grid = static_cast<int>(std::min<long>((vec + 255) / 256, 8L * num_sms(dev)));
  ep_copy_rows_kernel<<<std::max(grid, 1), 256, 0, stream>>>(a);
  count_launch();
  check_cuda(cudaGetLastError(), "ep_copy_rows_kernel launch");
}

}  // namespace ddb
