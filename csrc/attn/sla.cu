// Sparse-linear attention (SLA) support kernels for sm_100a: routing and the linear branch.
//
// Routing (reference layers/sla.py:61-137 re-designed as top-k over mean-pooled blocks):
//   sla_pool_kernel   mean of q and k over each 64-token block -> qm, km [B,H,nb,64] fp32
//   sla_route_kernel  per (b, h): block scores qm.km/sqrt(64), block validity
//                     (frame-causal / token-causal / none), diagonal forced, top-k per
//                     query block; emits the selection bits, the linear-branch block
//                     matrix W = valid & ~selected (bf16, for the batched GEMM), the
//                     forward pair lists (per 128-query tile, the union of its two blocks'
//                     selections paired into 128-key tiles, 4-bit half masks) and the
//                     backward lists (per 128-key tile, the query blocks that selected
//                     it, paired into 128-query units).
// Linear branch (phi = elu + 1; reference layers/sla.py:333-357 per block pair, here over
// all allowed-but-unselected blocks at once), per-block products on the tensor cores in
// sla_tc.cu:
//   sla_kv_state   per key block j: [phi(K_j)^T V_j | sum phi(K_j)] -> KVz [.., 4160] bf16
//   (tcgen05 batched GEMM) state_i = sum_j W_ij KVz_j             (drivedit_b200.ops.gemm)
//   sla_lin_out    per query block: o = phi(q) S / (phi(q).z + eps), saves den
//   sla_lin_bwd_q  per query block: dq (+=), dS/dz for the transposed GEMM
//   (tcgen05 batched GEMM) dKVz_j = sum_i W_ij dSz_i
//   sla_lin_bwd_kv per key block: dk, dv (+=)
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "sla.h"

namespace ddb {
namespace {

constexpr int D = 64;


// ------------------------------------------------------------------ pooling
__global__ void __launch_bounds__(256) sla_pool_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                       long ld, int T, int H, int nb,
                                                       float* __restrict__ qm,
                                                       float* __restrict__ km) {
  const int blk = blockIdx.x % nb;
  const int b = blockIdx.x / nb;
  const int dm = H * D;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  for (int c2 = threadIdx.x; c2 < dm; c2 += 256) {  // one bf16 pair of q and of k each
    const int c = (c2 % (dm / 2)) * 2;
    const int which = c2 / (dm / 2);               // 0: q, 1: k  (first/second half)
    const __nv_bfloat16* src = qkv + row0 * ld + which * dm + c;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
    for (int t = 0; t < 64; ++t) {
      float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + t * ld));
      s0 += f.x;
      s1 += f.y;
    }
    const int h = c / D, d = c % D;
    float* dst = (which == 0 ? qm : km) + ((static_cast<long>(b) * H + h) * nb + blk) * D + d;
    dst[0] = s0 * (1.f / 64.f);
    dst[1] = s1 * (1.f / 64.f);
  }
}

// ------------------------------------------------------------------ routing
__device__ __forceinline__ bool block_valid(int i, int j, int causal, int bpf) {
  if (causal == 1) return (j / bpf) <= (i / bpf);
  if (causal == 2) return j <= i;
  return true;
}

// one CTA per (b, h); nb <= 256 (multiple of 32). 32 warps per CTA: there are only B*H
// CTAs, so each one's query-block rows are spread over as many warps as a CTA holds.
constexpr int kRouteThreads = 1024;
__global__ void __launch_bounds__(kRouteThreads) sla_route_kernel(SlaRouteArgs a) {
  extern __shared__ float sm[];
  const int nb = a.nb;
  const int words = (nb + 31) / 32;
  float* sq = sm;                       // [nb][D]
  float* sk = sq + nb * D;              // [nb][D + 1] (padded: conflict-free column reads)
  uint32_t* sel = reinterpret_cast<uint32_t*>(sk + nb * (D + 1));  // [nb][words]
  const int bh = blockIdx.x;
  const float* qm = a.qm + static_cast<long>(bh) * nb * D;
  const float* km = a.km + static_cast<long>(bh) * nb * D;
  for (int i = threadIdx.x; i < nb * D; i += kRouteThreads) {
    sq[i] = qm[i];
    sk[(i / D) * (D + 1) + i % D] = km[i];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = rsqrtf(static_cast<float>(D));
  constexpr int MAXS = 8;  // nb / 32 <= 8
  for (int i = warp; i < nb; i += kRouteThreads / 32) {
    float sc[MAXS];
#pragma unroll
    for (int s = 0; s < MAXS; ++s) {
      const int j = s * 32 + lane;
      sc[s] = -INFINITY;
      if (s < words && j < nb) {
        float acc = 0.f;
#pragma unroll 16
        for (int d = 0; d < D; ++d) acc += sq[i * D + d] * sk[j * (D + 1) + d];
        if (block_valid(i, j, a.causal, a.bpf))
          sc[s] = (a.always_diag && j == i) ? INFINITY : acc * scale;
      }
    }
    uint32_t chosen[MAXS];
#pragma unroll
    for (int s = 0; s < MAXS; ++s) chosen[s] = 0;
    for (int r = 0; r < a.topk; ++r) {
      float best = -INFINITY;
      int bi = -1;
#pragma unroll
      for (int s = 0; s < MAXS; ++s)
        if (sc[s] > best) {
          best = sc[s];
          bi = s * 32 + lane;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi >= 0 && (bi < 0 || oi < bi))) {
          best = ob;
          bi = oi;
        }
      }
      if (best == -INFINITY || bi < 0) break;  // fewer allowed blocks than k
      if ((bi & 31) == lane) {
        sc[bi >> 5] = -INFINITY;
        chosen[bi >> 5] = 1;
      }
    }
#pragma unroll
    for (int s = 0; s < MAXS; ++s) {
      if (s < words) {
        const uint32_t w = __ballot_sync(0xffffffffu, chosen[s] != 0);
        if (lane == 0) sel[i * words + s] = w;
        const int j = s * 32 + lane;
        const bool lin = block_valid(i, j, a.causal, a.bpf) && !chosen[s];
        if (a.wlin && j < nb)
          a.wlin[(static_cast<long>(bh) * nb + i) * nb + j] = __float2bfloat16(lin ? 1.f : 0.f);
      }
    }
  }
  __syncthreads();
  if (a.sel_bits)
    for (int i = threadIdx.x; i < nb * words; i += kRouteThreads)
      a.sel_bits[static_cast<long>(bh) * nb * words + i] = sel[i];
  const int nt = nb / 2;
  auto bit = [&](int row, int col) -> uint32_t { return (sel[row * words + (col >> 5)] >> (col & 31)) & 1u; };
  // forward lists: per query tile t, its union of selected key blocks, paired
  for (int t = threadIdx.x; t < nt; t += kRouteThreads) {
    const long li = static_cast<long>(bh) * nt + t;
    int n = 0, pending = -1;
    for (int j = 0; j < nb; ++j) {
      const uint32_t lo = bit(2 * t, j), hi = bit(2 * t + 1, j);
      if (!(lo | hi)) continue;
      if (pending < 0) {
        pending = j;
      } else {
        const uint32_t m = bit(2 * t, pending) | (lo << 1) | (bit(2 * t + 1, pending) << 2) | (hi << 3);
        if (n < a.max_pairs) {
          a.pair_blocks[li * a.max_pairs + n] = pending | (j << 16);
          a.pair_mask[li * a.max_pairs + n] = static_cast<uint8_t>(m);
        }
        ++n;
        pending = -1;
      }
    }
    if (pending >= 0) {
      const uint32_t m = bit(2 * t, pending) | (bit(2 * t + 1, pending) << 2);
      if (n < a.max_pairs) {
        a.pair_blocks[li * a.max_pairs + n] = pending | (pending << 16);
        a.pair_mask[li * a.max_pairs + n] = static_cast<uint8_t>(m);
      }
      ++n;
    }
    a.pair_count[li] = min(n, a.max_pairs);
  }
  // backward lists: per key tile t (blocks 2t, 2t+1), the query blocks that selected
  // either key block, ascending and paired two at a time into 128-query units (any two
  // blocks, not only neighbours, so a unit wastes at most its key-half masking); an odd
  // last block is paired with itself with its second half masked off
  for (int t = threadIdx.x; t < nt; t += kRouteThreads) {
    const long li = static_cast<long>(bh) * nt + t;
    int n = 0, pending = -1;
    uint32_t pending_m = 0;
    for (int i = 0; i < nb; ++i) {
      const uint32_t m = bit(i, 2 * t) | (bit(i, 2 * t + 1) << 1);
      if (!m) continue;
      if (pending < 0) {
        pending = i;
        pending_m = m;
      } else {
        a.kv_qtiles[li * nt + n] = pending | (i << 16);
        a.kv_qmask[li * nt + n] = static_cast<uint8_t>(pending_m | (m << 2));
        ++n;
        pending = -1;
      }
    }
    if (pending >= 0) {
      a.kv_qtiles[li * nt + n] = pending | (pending << 16);
      a.kv_qmask[li * nt + n] = static_cast<uint8_t>(pending_m);
      ++n;
    }
    a.kv_count[li] = n;
  }
}

}  // namespace

void sla_pool(const __nv_bfloat16* qkv, long ld, int B, int T, int H, float* qm, float* km,
              cudaStream_t s) {
  const int nb = T / 64;
  sla_pool_kernel<<<B * nb, 256, 0, s>>>(qkv, ld, T, H, nb, qm, km);
  count_launch();
}

void sla_route(const SlaRouteArgs& a, int BH, cudaStream_t s) {
  if (a.nb % 2 != 0 || a.nb > 256 || a.nb < 2)
    throw std::runtime_error("sla_route: blocks per sequence must be even and <= 256");
  const int smem = a.nb * D * 4 + a.nb * (D + 1) * 4 + a.nb * ((a.nb + 31) / 32) * 4;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(sla_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    200 * 1024),
               "cudaFuncSetAttribute(sla_route)");
    attr = true;
  }
  sla_route_kernel<<<BH, kRouteThreads, smem, s>>>(a);
  count_launch();
}

}  // namespace ddb
