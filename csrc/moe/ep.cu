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
#include <type_traits>

#include "../common/ptx.cuh"
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

constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxChunks = 8;  // rows of up to 8 x 256 bf16 = 2048 columns

// Row helpers and kernels are instantiated for C 256-column chunks per row (C = 4 for
// d <= 1024, else 8): the per-lane row buffers and fp32 accumulators take C x 8 registers,
// so narrow rows keep more warps resident.
// Load one bf16 row (d columns, d % 8 == 0, d <= 2048) into registers: lane holds chunks
// i * 256 + lane * 8 .. + 8.
template <int C>
__device__ __forceinline__ void load_row(const __nv_bfloat16* row, int d, int lane, uint4 (&v)[C]) {
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = i * 256 + lane * 8;
    if (c < d) v[i] = ld_global_v4(row + c);
  }
}

template <int C>
__device__ __forceinline__ void store_row(__nv_bfloat16* row, int d, int lane, const uint4 (&v)[C]) {
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = i * 256 + lane * 8;
    if (c < d) st_global_v4(row + c, v[i].x, v[i].y, v[i].z, v[i].w);
  }
}

template <int C>
__device__ __forceinline__ void axpy_row(float (&acc)[C][8], float w, const __nv_bfloat16* row, int d,
                                         int lane) {
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = i * 256 + lane * 8;
    if (c < d) {
      const uint4 y = ld_global_v4(row + c);
      const uint32_t yw[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16(yw[q]);
        acc[i][2 * q] += w * f.x;
        acc[i][2 * q + 1] += w * f.y;
      }
    }
  }
}

template <int C>
__device__ __forceinline__ void store_acc(__nv_bfloat16* row, int d, int lane, const float (&acc)[C][8]) {
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = i * 256 + lane * 8;
    if (c < d)
      st_global_v4(row + c, pack_bf16(acc[i][0], acc[i][1]), pack_bf16(acc[i][2], acc[i][3]),
                   pack_bf16(acc[i][4], acc[i][5]), pack_bf16(acc[i][6], acc[i][7]));
  }
}

// One warp per unique row: z = sum_j w_j src[slot_j] -> the source's return buffer.
template <int C>
__global__ void __launch_bounds__(256) ep_owner_scatter_sum_kernel(EpOwnerArgs a, const __nv_bfloat16* src,
                                                                   long ld_src, bool weighted,
                                                                   __nv_bfloat16* const* peer_ret) {
  const int lane = threadIdx.x & 31;
  const long u = blockIdx.x * 8L + (threadIdx.x >> 5);
  if (u >= *a.n_uniq) return;
  const int* m = a.meta + u * (2 + a.k);
  const int s = m[0], t = m[1];
  int sl = -1;
  float wj = 0.f;
  if (lane < a.k) {
    sl = m[2 + lane];
    wj = weighted ? a.meta_w[u * a.k + lane] : 1.f;
  }
  const unsigned mask = __ballot_sync(kFull, lane < a.k && sl >= 0);
  float acc[C][8];
#pragma unroll
  for (int i = 0; i < C; ++i)
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[i][q] = 0.f;
  for (unsigned mm = mask; mm; mm &= mm - 1) {
    const int j = __ffs(mm) - 1;
    const int slj = __shfl_sync(kFull, sl, j);
    const float w = __shfl_sync(kFull, wj, j);
    axpy_row(acc, w, src + static_cast<long>(slj) * ld_src, a.d, lane);
  }
  store_acc(peer_ret[s] + (static_cast<long>(a.rank) * a.N + t) * a.d, a.d, lane, acc);
}

// Source push. One warp per token; owners of the token's experts found by lanes < k. Block
// counters aggregate the positions so each owner counter takes one atomic per block.
template <int C>
__global__ void __launch_bounds__(256) ep_push_rows_kernel(EpPushArgs a) {
  __shared__ int s_cnt[32], s_base[32];
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const bool fwd = a.smeta != nullptr;
  const bool live = t < a.N;
  int e = -1, o = -1;
  float w = 0.f;
  if (live && lane < a.k) {
    e = a.idx[static_cast<long>(t) * a.k + lane];
    w = a.w ? a.w[static_cast<long>(t) * a.k + lane] : 0.f;
    o = e / a.El;
  }
  // owner set of the token as a bitmask over ranks (every lane reaches the same collective)
  bool routed = false;  // gradient mode: lane o's owner received this token
  if (!fwd && live && lane < a.world) routed = a.pos[static_cast<long>(t) * a.world + lane] >= 0;
  const unsigned owners = fwd ? __reduce_or_sync(kFull, o >= 0 ? (1u << o) : 0u) : __ballot_sync(kFull, routed);
  int myp = -1;  // lane o: this token's position at owner o
  if (fwd) {
    if (threadIdx.x < 32) s_cnt[threadIdx.x] = 0;
    __syncthreads();
    if (live && lane < a.world && ((owners >> lane) & 1)) myp = atomicAdd(&s_cnt[lane], 1);
    __syncthreads();
    if (threadIdx.x < a.world) s_base[threadIdx.x] = s_cnt[threadIdx.x] ? atomicAdd(&a.cnt[threadIdx.x], s_cnt[threadIdx.x]) : 0;
    __syncthreads();
    if (myp >= 0) myp += s_base[lane];
    if (live && lane < a.world) a.pos[static_cast<long>(t) * a.world + lane] = myp;
  } else if (live && lane < a.world) {
    myp = a.pos[static_cast<long>(t) * a.world + lane];
  }
  if (!live) return;
  uint4 v[C];
  load_row(a.rows + static_cast<long>(t) * a.ld_rows, a.d, lane, v);
  for (unsigned mm = owners; mm; mm &= mm - 1) {
    const int ow = __ffs(mm) - 1;
    const long r = static_cast<long>(a.rank) * a.N + __shfl_sync(kFull, myp, ow);
    store_row(a.stage[ow] + r * a.d, a.d, lane, v);
    if (fwd) {
      int* m = a.smeta[ow] + r * (1 + 2 * a.k);
      if (lane == 0) m[0] = t;
      if (lane < a.k) {
        const bool here = o == ow;
        m[1 + lane] = here ? e : -1;
        m[1 + a.k + lane] = __float_as_int(here ? w : 0.f);
      }
    }
  }
}

// Owner fan-out of the staged rows into the local experts' segments (local copies).
template <int C>
__global__ void __launch_bounds__(256) ep_owner_fanout_kernel(EpFanoutArgs a) {
  __shared__ int s_cnt[256], s_base[256];
  const int lane = threadIdx.x & 31;
  const int u = blockIdx.x * 8 + (threadIdx.x >> 5);
  const bool live = u < a.total;
  for (int i = threadIdx.x; i < a.El; i += 256) s_cnt[i] = 0;
  if (blockIdx.x == 0 && threadIdx.x == 0) *a.n_uniq = a.total;
  __syncthreads();
  // source of u: the last s with prefix[s] <= u (prefix[0] = 0)
  const bool le = live && lane < a.world && a.prefix[lane] <= u;
  const unsigned lemask = __ballot_sync(kFull, le);
  const int s = lemask ? 31 - __clz(lemask) : 0;
  const long R = static_cast<long>(s) * a.N + (live ? u - a.prefix[s] : 0);
  const int* rec = a.smeta + R * (1 + 2 * a.k);
  int e = -1, loc = -1;
  float w = 0.f;
  if (live && lane < a.k) {
    e = rec[1 + lane];
    w = __int_as_float(rec[1 + a.k + lane]);
    if (e >= 0) loc = atomicAdd(&s_cnt[e - a.lo], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.El; i += 256)
    s_base[i] = s_cnt[i] ? atomicAdd(&a.cursor[i], s_cnt[i]) : 0;
  __syncthreads();
  if (!live) return;
  const int slot = e >= 0 ? a.seg_start[e - a.lo] + s_base[e - a.lo] + loc : -1;
  int* m = a.meta + static_cast<long>(u) * (2 + a.k);
  if (lane == 0) {
    m[0] = s;
    m[1] = rec[0];
    a.urow[u] = static_cast<int>(R);
  }
  if (lane < a.k) {
    m[2 + lane] = slot;
    a.meta_w[static_cast<long>(u) * a.k + lane] = e >= 0 ? w : 0.f;
  }
  uint4 v[C];
  load_row(a.stage + R * a.d, a.d, lane, v);
  for (unsigned mm = __ballot_sync(kFull, slot >= 0); mm; mm &= mm - 1) {
    const int j = __ffs(mm) - 1;
    store_row(a.xr + static_cast<long>(__shfl_sync(kFull, slot, j)) * a.ld_xr, a.d, lane, v);
  }
}

// One warp per unique row: read dout once; dy[slot_j] = w_j dout; dw_j = dout . y[slot_j]
// stored into the source's dw buffer.
template <int C>
__global__ void __launch_bounds__(256) ep_owner_grad_gather_kernel(EpOwnerArgs a, const __nv_bfloat16* y,
                                                                   long ld_y, __nv_bfloat16* dy, long ld_dy,
                                                                   float* const* peer_dw) {
  const int lane = threadIdx.x & 31;
  const long u = blockIdx.x * 8L + (threadIdx.x >> 5);
  if (u >= *a.n_uniq) return;
  const int* m = a.meta + u * (2 + a.k);
  const int s = m[0], t = m[1];
  int sl = -1;
  float wj = 0.f;
  if (lane < a.k) {
    sl = m[2 + lane];
    wj = a.meta_w[u * a.k + lane];
  }
  const unsigned mask = __ballot_sync(kFull, lane < a.k && sl >= 0);
  uint4 g[C];
  load_row(a.local_rows ? a.local_rows + static_cast<long>(a.urow[u]) * a.d
                        : a.peer_rows[s] + static_cast<long>(t) * a.d,
           a.d, lane, g);
  for (unsigned mm = mask; mm; mm &= mm - 1) {
    const int j = __ffs(mm) - 1;
    const int slj = __shfl_sync(kFull, sl, j);
    const float w = __shfl_sync(kFull, wj, j);
    const __nv_bfloat16* yr = y + static_cast<long>(slj) * ld_y;
    __nv_bfloat16* dr = dy + static_cast<long>(slj) * ld_dy;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = i * 256 + lane * 8;
      if (c < a.d) {
        const uint4 yv = ld_global_v4(yr + c);
        const uint32_t gw[4] = {g[i].x, g[i].y, g[i].z, g[i].w}, yw[4] = {yv.x, yv.y, yv.z, yv.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 fg = unpack_bf16(gw[q]), fy = unpack_bf16(yw[q]);
          dot += fg.x * fy.x + fg.y * fy.y;
          o[q] = pack_bf16(w * fg.x, w * fg.y);
        }
        st_global_v4(dr + c, o[0], o[1], o[2], o[3]);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(kFull, dot, off);
    if (lane == 0) peer_dw[s][static_cast<long>(t) * a.k + j] = dot;
  }
}

// One warp per local token: residual + the partial rows of every owner it routed to
// (+ gated shared-expert rows).
template <int C>
__global__ void __launch_bounds__(256) ep_source_reduce_kernel(EpSourceArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= a.N) return;
  unsigned bits = 0;
  if (lane < a.k) bits = 1u << (a.idx[static_cast<long>(t) * a.k + lane] / a.El);
  const unsigned owners = __reduce_or_sync(kFull, bits);
  float acc[C][8];
  if (a.residual) {
    uint4 r[C];
    load_row(a.residual + static_cast<long>(t) * a.ld_res, a.d, lane, r);
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const uint32_t rw[4] = {r[i].x, r[i].y, r[i].z, r[i].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16(rw[q]);
        acc[i][2 * q] = f.x;
        acc[i][2 * q + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < C; ++i)
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[i][q] = 0.f;
  }
  for (unsigned mm = owners; mm; mm &= mm - 1) {
    const int o = __ffs(mm) - 1;
    axpy_row(acc, 1.f, a.ret + (static_cast<long>(o) * a.N + t) * a.d, a.d, lane);
  }
  for (int sh = 0; sh < a.ns; ++sh) {
    const float gsh = a.shared_w ? a.shared_w[static_cast<long>(t) * a.ns + sh] : 1.f;
    const int sl = a.slot_s[static_cast<long>(t) * a.ns + sh];
    axpy_row(acc, gsh, a.ys + static_cast<long>(sl) * a.ld_ys, a.d, lane);
  }
  store_acc(a.out + static_cast<long>(t) * a.ld_out, a.d, lane, acc);
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

namespace ddb {
namespace {
// run f with the chunk count for rows of d columns as a compile-time constant
template <typename F>
void launch_c(int d, F f) {
  if (d <= 1024)
    f(std::integral_constant<int, 4>{});
  else
    f(std::integral_constant<int, 8>{});
}
void check_owner(const EpOwnerArgs& a) {
  if (a.d % 8 != 0 || a.d > 256 * kMaxChunks) throw std::runtime_error("ep: d % 8 == 0 and d <= 2048");
  if (a.k > 32 || a.k < 1) throw std::runtime_error("ep: 1 <= k <= 32");
  if (a.world > 32) throw std::runtime_error("ep: at most 32 ranks");
}
}  // namespace

void ep_push_rows(const EpPushArgs& a, cudaStream_t s) {
  if (a.d % 8 != 0 || a.d > 256 * kMaxChunks) throw std::runtime_error("ep: d % 8 == 0 and d <= 2048");
  if (a.k > 32 || a.k < 1 || a.world > 32 || a.world < 1) throw std::runtime_error("ep: k <= 32, world <= 32");
  if (a.N == 0) return;
  launch_c(a.d, [&](auto c) { ep_push_rows_kernel<decltype(c)::value><<<(a.N + 7) / 8, 256, 0, s>>>(a); });
  count_launch();
  check_cuda(cudaGetLastError(), "ep_push_rows launch");
}

void ep_owner_fanout(const EpFanoutArgs& a, cudaStream_t s) {
  if (a.d % 8 != 0 || a.d > 256 * kMaxChunks) throw std::runtime_error("ep: d % 8 == 0 and d <= 2048");
  if (a.k > 32 || a.world > 32 || a.El > 256) throw std::runtime_error("ep: k <= 32, world <= 32, El <= 256");
  if (a.total <= 0) {
    check_cuda(cudaMemsetAsync(a.n_uniq, 0, sizeof(int), s), "ep fanout n_uniq");
    return;
  }
  launch_c(a.d, [&](auto c) { ep_owner_fanout_kernel<decltype(c)::value><<<(a.total + 7) / 8, 256, 0, s>>>(a); });
  count_launch();
  check_cuda(cudaGetLastError(), "ep_owner_fanout launch");
}

void ep_owner_grad_gather(const EpOwnerArgs& a, const __nv_bfloat16* y, long ld_y, __nv_bfloat16* dy,
                          long ld_dy, float* const* peer_dw, cudaStream_t s) {
  check_owner(a);
  if (a.cap == 0) return;
  launch_c(a.d, [&](auto c) {
    ep_owner_grad_gather_kernel<decltype(c)::value><<<(a.cap + 7) / 8, 256, 0, s>>>(a, y, ld_y, dy, ld_dy, peer_dw);
  });
  count_launch();
  check_cuda(cudaGetLastError(), "ep_owner_grad_gather launch");
}

void ep_owner_scatter_sum(const EpOwnerArgs& a, const __nv_bfloat16* src, long ld_src, bool weighted,
                          __nv_bfloat16* const* peer_ret, cudaStream_t s) {
  check_owner(a);
  if (a.cap == 0) return;
  launch_c(a.d, [&](auto c) {
    ep_owner_scatter_sum_kernel<decltype(c)::value><<<(a.cap + 7) / 8, 256, 0, s>>>(a, src, ld_src, weighted, peer_ret);
  });
  count_launch();
  check_cuda(cudaGetLastError(), "ep_owner_scatter_sum launch");
}

void ep_source_reduce(const EpSourceArgs& a, cudaStream_t s) {
  if (a.d % 8 != 0 || a.d > 256 * kMaxChunks) throw std::runtime_error("ep: d % 8 == 0 and d <= 2048");
  if (a.N == 0) return;
  launch_c(a.d, [&](auto c) { ep_source_reduce_kernel<decltype(c)::value><<<(a.N + 7) / 8, 256, 0, s>>>(a); });
  count_launch();
  check_cuda(cudaGetLastError(), "ep_source_reduce launch");
}

}  // namespace ddb
