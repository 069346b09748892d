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
//                     backward lists (per 128-key tile, the query tiles that selected it).
// Linear branch (phi = elu + 1; reference layers/sla.py:333-357 per block pair, here over
// all allowed-but-unselected blocks at once):
//   sla_kv_state_kernel  per key block j: [phi(K_j)^T V_j | sum phi(K_j)] -> KVz [.., 4160] bf16
//   (tcgen05 batched GEMM) state_i = sum_j W_ij KVz_j             (drivedit_b200.ops.gemm)
//   sla_lin_out_kernel   per query block: o = phi(q) S / (phi(q).z + eps), saves den
//   sla_lin_bwd_q_kernel per query block: dq (+=), dS/dz for the transposed GEMM
//   (tcgen05 batched GEMM) dKVz_j = sum_i W_ij dSz_i
//   sla_lin_bwd_kv_kernel per key block: dk, dv (+=)
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "sla.h"

namespace ddb {
namespace {

constexpr int D = 64;
constexpr int NZ = D * D + D;  // 4160: KV state + normaliser row

__device__ __forceinline__ float phi(float x) { return x > 0.f ? x + 1.f : __expf(x); }
__device__ __forceinline__ float dphi(float x) { return x > 0.f ? 1.f : __expf(x); }

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

// one CTA per (b, h); nb <= 256 (multiple of 32)
__global__ void __launch_bounds__(256) sla_route_kernel(SlaRouteArgs a) {
  extern __shared__ float sm[];
  const int nb = a.nb;
  const int words = (nb + 31) / 32;
  float* sq = sm;                       // [nb][D]
  float* sk = sq + nb * D;              // [nb][D + 1] (padded: conflict-free column reads)
  uint32_t* sel = reinterpret_cast<uint32_t*>(sk + nb * (D + 1));  // [nb][words]
  const int bh = blockIdx.x;
  const float* qm = a.qm + static_cast<long>(bh) * nb * D;
  const float* km = a.km + static_cast<long>(bh) * nb * D;
  for (int i = threadIdx.x; i < nb * D; i += 256) {
    sq[i] = qm[i];
    sk[(i / D) * (D + 1) + i % D] = km[i];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = rsqrtf(static_cast<float>(D));
  constexpr int MAXS = 8;  // nb / 32 <= 8
  for (int i = warp; i < nb; i += 8) {
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
    for (int i = threadIdx.x; i < nb * words; i += 256)
      a.sel_bits[static_cast<long>(bh) * nb * words + i] = sel[i];
  const int nt = nb / 2;
  auto bit = [&](int row, int col) -> uint32_t { return (sel[row * words + (col >> 5)] >> (col & 31)) & 1u; };
  // forward lists: per query tile t, its union of selected key blocks, paired
  for (int t = threadIdx.x; t < nt; t += 256) {
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
  // backward lists: per key tile t (blocks 2t, 2t+1), the query tiles that selected it
  for (int t = threadIdx.x; t < nt; t += 256) {
    const long li = static_cast<long>(bh) * nt + t;
    int n = 0;
    for (int i = 0; i < nt; ++i) {
      const uint32_t m = bit(2 * i, 2 * t) | (bit(2 * i, 2 * t + 1) << 1) |
                         (bit(2 * i + 1, 2 * t) << 2) | (bit(2 * i + 1, 2 * t + 1) << 3);
      if (m) {
        a.kv_qtiles[li * nt + n] = i;
        a.kv_qmask[li * nt + n] = static_cast<uint8_t>(m);
        ++n;
      }
    }
    a.kv_count[li] = n;
  }
}

// ------------------------------------------------------------------ linear branch
// Loads a [64 tokens x 64] bf16 head block into fp32 shared memory (optionally phi'd).
__device__ __forceinline__ void load_block(float* dst, const __nv_bfloat16* src, long ld,
                                           bool apply_phi) {
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    const int t = i >> 3, c = (i & 7) * 8;
    uint4 u = ld_global_v4(src + t * ld + c);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(w[j]);
      dst[t * 65 + c + 2 * j] = apply_phi ? phi(f.x) : f.x;
      dst[t * 65 + c + 2 * j + 1] = apply_phi ? phi(f.y) : f.y;
    }
  }
}

// KVz_j = [phi(K_j)^T V_j (d-major), sum_t phi(K_j)[t, :]] as bf16
__global__ void __launch_bounds__(256) sla_kv_state_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                           long ld, int T, int H, int nb,
                                                           __nv_bfloat16* __restrict__ kvz) {
  __shared__ float fk[64 * 65], vv[64 * 65];
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const int dm = H * D;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  load_block(fk, qkv + row0 * ld + dm + h * D, ld, true);
  load_block(vv, qkv + row0 * ld + 2 * dm + h * D, ld, false);
  __syncthreads();
  const int d = threadIdx.x >> 2;
  const int e0 = (threadIdx.x & 3) * 16;
  float acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
  float zs = 0.f;
  for (int t = 0; t < 64; ++t) {
    const float k = fk[t * 65 + d];
    zs += k;
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] += k * vv[t * 65 + e0 + e];
  }
  __nv_bfloat16* out = kvz + (static_cast<long>(bh) * nb + blk) * NZ;
#pragma unroll
  for (int e = 0; e < 16; e += 8)
    st_global_v4(out + d * D + e0 + e, pack_bf16(acc[e], acc[e + 1]), pack_bf16(acc[e + 2], acc[e + 3]),
                 pack_bf16(acc[e + 4], acc[e + 5]), pack_bf16(acc[e + 6], acc[e + 7]));
  if ((threadIdx.x & 3) == 0) out[D * D + d] = __float2bfloat16(zs);
}

// o_i = phi(Q_i) S_i / (phi(Q_i) . z_i + eps); state rows come from the batched GEMM (fp32)
__global__ void __launch_bounds__(256) sla_lin_out_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                          long ld, int T, int H, int nb,
                                                          const float* __restrict__ state,
                                                          __nv_bfloat16* __restrict__ o, long ldo,
                                                          float* __restrict__ den_out, float eps) {
  __shared__ float fq[64 * 65], st[64 * 65], z[64], den[64];
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  load_block(fq, qkv + row0 * ld + h * D, ld, true);
  const float* S = state + (static_cast<long>(bh) * nb + blk) * NZ;
  for (int i = threadIdx.x; i < D * D; i += 256) st[(i / D) * 65 + i % D] = S[i];
  if (threadIdx.x < D) z[threadIdx.x] = S[D * D + threadIdx.x];
  __syncthreads();
  if (threadIdx.x < 64) {
    float s = 0.f;
    for (int d = 0; d < D; ++d) s += fq[threadIdx.x * 65 + d] * z[d];
    den[threadIdx.x] = s + eps;
    den_out[static_cast<long>(bh) * T + blk * 64 + threadIdx.x] = s + eps;
  }
  __syncthreads();
  const int t = threadIdx.x >> 2;
  const int e0 = (threadIdx.x & 3) * 16;
  float acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
  for (int d = 0; d < D; ++d) {
    const float q = fq[t * 65 + d];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] += q * st[d * 65 + e0 + e];
  }
  const float inv = 1.f / den[t];
  __nv_bfloat16* dst = o + (row0 + t) * ldo + h * D + e0;
#pragma unroll
  for (int e = 0; e < 16; e += 8)
    st_global_v4(dst + e, pack_bf16(acc[e] * inv, acc[e + 1] * inv),
                 pack_bf16(acc[e + 2] * inv, acc[e + 3] * inv),
                 pack_bf16(acc[e + 4] * inv, acc[e + 5] * inv),
                 pack_bf16(acc[e + 6] * inv, acc[e + 7] * inv));
}

// Backward, query side. dnum = do/den, dden = -(do.o)/den,
// dphi(q) = dnum S^T + dden z, dS = phi(q)^T dnum, dz = phi(q)^T dden; dq += dphi(q)*phi'(q).
__global__ void __launch_bounds__(256) sla_lin_bwd_q_kernel(
    const __nv_bfloat16* __restrict__ qkv, long ld, int T, int H, int nb,
    const float* __restrict__ state, const __nv_bfloat16* __restrict__ o, long ldo,
    const __nv_bfloat16* __restrict__ dout, long lddo, const float* __restrict__ den_in,
    __nv_bfloat16* __restrict__ dsz, __nv_bfloat16* __restrict__ dqkv, long lddq) {
  extern __shared__ float dyn[];
  float* fq = dyn;
  float* st = fq + 64 * 65;
  float* dn = st + 64 * 65;
  float* z = dn + 64 * 65;
  float* dd = z + 64;
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  const float* S = state + (static_cast<long>(bh) * nb + blk) * NZ;
  load_block(fq, qkv + row0 * ld + h * D, ld, true);
  for (int i = threadIdx.x; i < D * D; i += 256) st[(i / D) * 65 + i % D] = S[i];
  if (threadIdx.x < D) z[threadIdx.x] = S[D * D + threadIdx.x];
  // dnum and dden per token (one warp-quarter per token: 4 threads x 16 columns)
  {
    const int t = threadIdx.x >> 2, e0 = (threadIdx.x & 3) * 16;
    const float den = den_in[static_cast<long>(bh) * T + blk * 64 + t];
    const __nv_bfloat16* dr = dout + (row0 + t) * lddo + h * D + e0;
    const __nv_bfloat16* orow = o + (row0 + t) * ldo + h * D + e0;
    float part = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float g = __bfloat162float(dr[e]);
      part += g * __bfloat162float(orow[e]);
      dn[t * 65 + e0 + e] = g / den;
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if ((threadIdx.x & 3) == 0) dd[t] = -part / den;
  }
  __syncthreads();
  // dq for this block's rows
  {
    const int t = threadIdx.x >> 2, d0 = (threadIdx.x & 3) * 16;
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = dd[t] * z[d0 + j];
    for (int e = 0; e < D; ++e) {
      const float g = dn[t * 65 + e];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] += g * st[(d0 + j) * 65 + e];
    }
    __nv_bfloat16* qrow = dqkv + (row0 + t) * lddq + h * D + d0;
    const __nv_bfloat16* qin = qkv + (row0 + t) * ld + h * D + d0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float x = __bfloat162float(qin[j]);
      qrow[j] = __float2bfloat16(__bfloat162float(qrow[j]) + acc[j] * dphi(x));
    }
  }
  // dS = phi(q)^T dnum, dz = phi(q)^T dden  -> bf16 rows for the transposed GEMM
  {
    const int d = threadIdx.x >> 2, e0 = (threadIdx.x & 3) * 16;
    float acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0.f;
    float zacc = 0.f;
    for (int t = 0; t < 64; ++t) {
      const float q = fq[t * 65 + d];
      zacc += q * dd[t];
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] += q * dn[t * 65 + e0 + e];
    }
    __nv_bfloat16* out = dsz + (static_cast<long>(bh) * nb + blk) * NZ;
#pragma unroll
    for (int e = 0; e < 16; e += 8)
      st_global_v4(out + d * D + e0 + e, pack_bf16(acc[e], acc[e + 1]), pack_bf16(acc[e + 2], acc[e + 3]),
                   pack_bf16(acc[e + 4], acc[e + 5]), pack_bf16(acc[e + 6], acc[e + 7]));
    if ((threadIdx.x & 3) == 0) out[D * D + d] = __float2bfloat16(zacc);
  }
}

// Backward, key side: dphi(K_j) = V_j dKV_j^T + dz_j, dV_j = phi(K_j) dKV_j; dk, dv (+=).
__global__ void __launch_bounds__(256) sla_lin_bwd_kv_kernel(
    const __nv_bfloat16* __restrict__ qkv, long ld, int T, int H, int nb,
    const float* __restrict__ dkvz, __nv_bfloat16* __restrict__ dqkv, long lddq) {
  extern __shared__ float dyn[];
  float* fk = dyn;
  float* vv = fk + 64 * 65;
  float* g = vv + 64 * 65;
  float* dz = g + 64 * 65;
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const int dm = H * D;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  load_block(fk, qkv + row0 * ld + dm + h * D, ld, true);
  load_block(vv, qkv + row0 * ld + 2 * dm + h * D, ld, false);
  const float* G = dkvz + (static_cast<long>(bh) * nb + blk) * NZ;
  for (int i = threadIdx.x; i < D * D; i += 256) g[(i / D) * 65 + i % D] = G[i];
  if (threadIdx.x < D) dz[threadIdx.x] = G[D * D + threadIdx.x];
  __syncthreads();
  const int t = threadIdx.x >> 2, c0 = (threadIdx.x & 3) * 16;
  float ak[16], av[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    ak[j] = dz[c0 + j];
    av[j] = 0.f;
  }
  for (int x = 0; x < D; ++x) {
    const float v = vv[t * 65 + x];   // dphi(k)[t, d] += V[t, x] G[d, x]
    const float k = fk[t * 65 + x];   // dV[t, e] += phi(k)[t, x] G[x, e]
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      ak[j] += v * g[(c0 + j) * 65 + x];
      av[j] += k * g[x * 65 + c0 + j];
    }
  }
  __nv_bfloat16* krow = dqkv + (row0 + t) * lddq + dm + h * D + c0;
  __nv_bfloat16* vrow = dqkv + (row0 + t) * lddq + 2 * dm + h * D + c0;
  const __nv_bfloat16* kin = qkv + (row0 + t) * ld + dm + h * D + c0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float x = __bfloat162float(kin[j]);
    krow[j] = __float2bfloat16(__bfloat162float(krow[j]) + ak[j] * dphi(x));
    vrow[j] = __float2bfloat16(__bfloat162float(vrow[j]) + av[j]);
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
  sla_route_kernel<<<BH, 256, smem, s>>>(a);
  count_launch();
}

void sla_kv_state(const __nv_bfloat16* qkv, long ld, int B, int T, int H, __nv_bfloat16* kvz,
                  cudaStream_t s) {
  const int nb = T / 64;
  sla_kv_state_kernel<<<B * H * nb, 256, 0, s>>>(qkv, ld, T, H, nb, kvz);
  count_launch();
}

void sla_lin_out(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                 __nv_bfloat16* o, long ldo, float* den, float eps, cudaStream_t s) {
  const int nb = T / 64;
  sla_lin_out_kernel<<<B * H * nb, 256, 0, s>>>(qkv, ld, T, H, nb, state, o, ldo, den, eps);
  count_launch();
}

void sla_lin_bwd_q(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                   const __nv_bfloat16* o, long ldo, const __nv_bfloat16* dout, long lddo,
                   const float* den, __nv_bfloat16* dsz, __nv_bfloat16* dqkv, long lddq,
                   cudaStream_t s) {
  const int nb = T / 64;
  constexpr int smem = (3 * 64 * 65 + 128) * 4;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(sla_lin_bwd_q_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "cudaFuncSetAttribute(sla_lin_bwd_q)");
    attr = true;
  }
  sla_lin_bwd_q_kernel<<<B * H * nb, 256, smem, s>>>(qkv, ld, T, H, nb, state, o, ldo, dout, lddo,
                                                   den, dsz, dqkv, lddq);
  count_launch();
}

void sla_lin_bwd_kv(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* dkvz,
                    __nv_bfloat16* dqkv, long lddq, cudaStream_t s) {
  const int nb = T / 64;
  constexpr int smem = (3 * 64 * 65 + 64) * 4;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(sla_lin_bwd_kv_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "cudaFuncSetAttribute(sla_lin_bwd_kv)");
    attr = true;
  }
  sla_lin_bwd_kv_kernel<<<B * H * nb, 256, smem, s>>>(qkv, ld, T, H, nb, dkvz, dqkv, lddq);
  count_launch();
}

}  // namespace ddb
