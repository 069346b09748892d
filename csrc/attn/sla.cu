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
// The 64 x 64 x 64 products below use 4 x 4 register tiles: operands are staged in shared
// memory "reduction-major" ([k][m], [k][n], rows padded to LDP floats) so each step of the
// reduction is one broadcast float4 of A, one float4 of B and 16 FMAs per thread.
constexpr int LDP = 68;        // padded row (floats); keeps float4 alignment
constexpr int TILE_F = 64 * LDP;

// Stage a [64 tokens x 64] bf16 head block as fp32: `rowmajor` -> dst[t][c], else dst[c][t].
__device__ __forceinline__ void stage_block(float* dst, const __nv_bfloat16* src, long ld,
                                            bool apply_phi, bool rowmajor) {
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    const int t = i >> 3, c = (i & 7) * 8;
    uint4 u = ld_global_v4(src + t * ld + c);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(w[j]);
      const float a = apply_phi ? phi(f.x) : f.x;
      const float b = apply_phi ? phi(f.y) : f.y;
      if (rowmajor) {
        dst[t * LDP + c + 2 * j] = a;
        dst[t * LDP + c + 2 * j + 1] = b;
      } else {
        dst[(c + 2 * j) * LDP + t] = a;
        dst[(c + 2 * j + 1) * LDP + t] = b;
      }
    }
  }
}

// Stage a dense fp32 [64 x 64] matrix (row stride 64): dst[r][c] or, transposed, dst[c][r].
__device__ __forceinline__ void stage_f32(float* dst, const float* src, bool transpose) {
  for (int i = threadIdx.x; i < 64 * 16; i += blockDim.x) {
    const int r = i >> 4, c = (i & 15) * 4;
    const float4 v = *reinterpret_cast<const float4*>(src + r * 64 + c);
    if (!transpose) {
      *reinterpret_cast<float4*>(dst + r * LDP + c) = v;
    } else {
      dst[c * LDP + r] = v.x;
      dst[(c + 1) * LDP + r] = v.y;
      dst[(c + 2) * LDP + r] = v.z;
      dst[(c + 3) * LDP + r] = v.w;
    }
  }
}

// acc[i][j] += sum_k AT[k][m0 + i] * B[k][n0 + j], thread (ty, tx) = (tid / 16, tid % 16)
__device__ __forceinline__ void mm64(float (&acc)[4][4], const float* AT, const float* B, int m0,
                                     int n0) {
#pragma unroll 8
  for (int k = 0; k < 64; ++k) {
    const float4 a = *reinterpret_cast<const float4*>(AT + k * LDP + m0);
    const float4 b = *reinterpret_cast<const float4*>(B + k * LDP + n0);
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
  }
}

__device__ __forceinline__ void zero44(float (&a)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) a[i][j] = 0.f;
}

// KVz_j = [phi(K_j)^T V_j (d-major), sum_t phi(K_j)[t, :]] as bf16
__global__ void __launch_bounds__(256) sla_kv_state_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                           long ld, int T, int H, int nb,
                                                           __nv_bfloat16* __restrict__ kvz) {
  extern __shared__ float dyn[];
  float* fk = dyn;            // [t][d]
  float* vv = fk + TILE_F;    // [t][e]
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const int dm = H * D;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  stage_block(fk, qkv + row0 * ld + dm + h * D, ld, true, true);
  stage_block(vv, qkv + row0 * ld + 2 * dm + h * D, ld, false, true);
  __syncthreads();
  const int m0 = (threadIdx.x >> 4) * 4, n0 = (threadIdx.x & 15) * 4;
  float acc[4][4];
  zero44(acc);
  mm64(acc, fk, vv, m0, n0);  // KV[d][e] = sum_t fk[t][d] v[t][e]
  __nv_bfloat16* out = kvz + (static_cast<long>(bh) * nb + blk) * NZ;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint2 w = make_uint2(pack_bf16(acc[i][0], acc[i][1]), pack_bf16(acc[i][2], acc[i][3]));
    *reinterpret_cast<uint2*>(out + (m0 + i) * D + n0) = w;
  }
  if (threadIdx.x < 64) {
    float zs = 0.f;
    for (int t = 0; t < 64; ++t) zs += fk[t * LDP + threadIdx.x];
    out[D * D + threadIdx.x] = __float2bfloat16(zs);
  }
}

// o_i = phi(Q_i) S_i / (phi(Q_i) . z_i + eps); state rows come from the batched GEMM (fp32)
__global__ void __launch_bounds__(256) sla_lin_out_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                          long ld, int T, int H, int nb,
                                                          const float* __restrict__ state,
                                                          __nv_bfloat16* __restrict__ o, long ldo,
                                                          float* __restrict__ den_out, float eps) {
  extern __shared__ float dyn[];
  float* fqT = dyn;              // [d][t]
  float* st = fqT + TILE_F;      // [d][e]
  float* z = st + TILE_F;        // [64]
  float* den = z + 64;           // [64]
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  const float* S = state + (static_cast<long>(bh) * nb + blk) * NZ;
  stage_block(fqT, qkv + row0 * ld + h * D, ld, true, false);
  stage_f32(st, S, false);
  if (threadIdx.x < D) z[threadIdx.x] = S[D * D + threadIdx.x];
  __syncthreads();
  if (threadIdx.x < 64) {
    float s = 0.f;
    for (int d = 0; d < D; ++d) s += fqT[d * LDP + threadIdx.x] * z[d];
    den[threadIdx.x] = s + eps;
    den_out[static_cast<long>(bh) * T + blk * 64 + threadIdx.x] = s + eps;
  }
  __syncthreads();
  const int m0 = (threadIdx.x >> 4) * 4, n0 = (threadIdx.x & 15) * 4;
  float acc[4][4];
  zero44(acc);
  mm64(acc, fqT, st, m0, n0);  // num[t][e] = sum_d fq[t][d] S[d][e]
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float inv = 1.f / den[m0 + i];
    uint2 w = make_uint2(pack_bf16(acc[i][0] * inv, acc[i][1] * inv),
                         pack_bf16(acc[i][2] * inv, acc[i][3] * inv));
    *reinterpret_cast<uint2*>(o + (row0 + m0 + i) * ldo + h * D + n0) = w;
  }
}

// Backward, query side. dnum = do/den, dden = -(do.o)/den,
// dphi(q) = dnum S^T + dden z, dS = phi(q)^T dnum, dz = phi(q)^T dden; dq += dphi(q)*phi'(q).
__global__ void __launch_bounds__(256) sla_lin_bwd_q_kernel(
    const __nv_bfloat16* __restrict__ qkv, long ld, int T, int H, int nb,
    const float* __restrict__ state, const __nv_bfloat16* __restrict__ o, long ldo,
    const __nv_bfloat16* __restrict__ dout, long lddo, const float* __restrict__ den_in,
    __nv_bfloat16* __restrict__ dsz, __nv_bfloat16* __restrict__ dqkv, long lddq) {
  extern __shared__ float dyn[];
  float* fq = dyn;               // [t][d]
  float* stT = fq + TILE_F;      // [e][d]
  float* dn = stT + TILE_F;      // [t][e]
  float* dnT = dn + TILE_F;      // [e][t]
  float* z = dnT + TILE_F;       // [64]
  float* dd = z + 64;            // [64]
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  const float* S = state + (static_cast<long>(bh) * nb + blk) * NZ;
  stage_block(fq, qkv + row0 * ld + h * D, ld, true, true);
  stage_f32(stT, S, true);
  if (threadIdx.x < D) z[threadIdx.x] = S[D * D + threadIdx.x];
  {  // dnum and dden: 4 threads per token, 16 columns each
    const int t = threadIdx.x >> 2, e0 = (threadIdx.x & 3) * 16;
    const float den = den_in[static_cast<long>(bh) * T + blk * 64 + t];
    const __nv_bfloat16* dr = dout + (row0 + t) * lddo + h * D + e0;
    const __nv_bfloat16* orow = o + (row0 + t) * ldo + h * D + e0;
    float part = 0.f;
#pragma unroll
    for (int e = 0; e < 16; e += 8) {
      uint4 gu = ld_global_v4(dr + e), ou = ld_global_v4(orow + e);
      uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w}, ow[4] = {ou.x, ou.y, ou.z, ou.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 g = unpack_bf16(gw[j]), ov = unpack_bf16(ow[j]);
        part += g.x * ov.x + g.y * ov.y;
        const int c = e0 + e + 2 * j;
        dn[t * LDP + c] = g.x / den;
        dn[t * LDP + c + 1] = g.y / den;
        dnT[c * LDP + t] = g.x / den;
        dnT[(c + 1) * LDP + t] = g.y / den;
      }
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if ((threadIdx.x & 3) == 0) dd[t] = -part / den;
  }
  __syncthreads();
  const int m0 = (threadIdx.x >> 4) * 4, n0 = (threadIdx.x & 15) * 4;
  {  // dq[t][d] = (sum_e dn[t][e] S[d][e] + dd[t] z[d]) * phi'(q[t][d])
    float acc[4][4];
    zero44(acc);
    mm64(acc, dnT, stT, m0, n0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const long r = row0 + m0 + i;
      __nv_bfloat16* qrow = dqkv + r * lddq + h * D + n0;
      const __nv_bfloat16* qin = qkv + r * ld + h * D + n0;
      const uint2 qv = *reinterpret_cast<const uint2*>(qin);
      const uint2 cur = *reinterpret_cast<const uint2*>(qrow);
      const float2 q01 = unpack_bf16(qv.x), q23 = unpack_bf16(qv.y);
      const float2 c01 = unpack_bf16(cur.x), c23 = unpack_bf16(cur.y);
      const float qx[4] = {q01.x, q01.y, q23.x, q23.y}, cx[4] = {c01.x, c01.y, c23.x, c23.y};
      float out[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        out[j] = cx[j] + (acc[i][j] + dd[m0 + i] * z[n0 + j]) * dphi(qx[j]);
      *reinterpret_cast<uint2*>(qrow) = make_uint2(pack_bf16(out[0], out[1]), pack_bf16(out[2], out[3]));
    }
  }
  {  // dS[d][e] = sum_t fq[t][d] dn[t][e]; dz[d] = sum_t fq[t][d] dd[t]
    float acc[4][4];
    zero44(acc);
    mm64(acc, fq, dn, m0, n0);
    __nv_bfloat16* out = dsz + (static_cast<long>(bh) * nb + blk) * NZ;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint2*>(out + (m0 + i) * D + n0) =
          make_uint2(pack_bf16(acc[i][0], acc[i][1]), pack_bf16(acc[i][2], acc[i][3]));
    if (threadIdx.x < 64) {
      float zacc = 0.f;
      for (int t = 0; t < 64; ++t) zacc += fq[t * LDP + threadIdx.x] * dd[t];
      out[D * D + threadIdx.x] = __float2bfloat16(zacc);
    }
  }
}

// Backward, key side: dphi(K_j) = V_j dKV_j^T + dz_j, dV_j = phi(K_j) dKV_j; dk, dv (+=).
__global__ void __launch_bounds__(256) sla_lin_bwd_kv_kernel(
    const __nv_bfloat16* __restrict__ qkv, long ld, int T, int H, int nb,
    const float* __restrict__ dkvz, __nv_bfloat16* __restrict__ dqkv, long lddq) {
  extern __shared__ float dyn[];
  float* vT = dyn;               // [e][t]
  float* gT = vT + TILE_F;       // [e][d]
  float* fkT = gT + TILE_F;      // [d][t]
  float* g = fkT + TILE_F;       // [d][e]
  float* dz = g + TILE_F;        // [64]
  const int blk = blockIdx.x % nb;
  const int bh = blockIdx.x / nb;
  const int b = bh / H, h = bh % H;
  const int dm = H * D;
  const long row0 = static_cast<long>(b) * T + blk * 64;
  const float* G = dkvz + (static_cast<long>(bh) * nb + blk) * NZ;
  stage_block(fkT, qkv + row0 * ld + dm + h * D, ld, true, false);
  stage_block(vT, qkv + row0 * ld + 2 * dm + h * D, ld, false, false);
  stage_f32(g, G, false);
  stage_f32(gT, G, true);
  if (threadIdx.x < D) dz[threadIdx.x] = G[D * D + threadIdx.x];
  __syncthreads();
  const int m0 = (threadIdx.x >> 4) * 4, n0 = (threadIdx.x & 15) * 4;
  float ak[4][4], av[4][4];
  zero44(ak);
  zero44(av);
  mm64(ak, vT, gT, m0, n0);   // dphi(k)[t][d] = sum_e V[t][e] G[d][e]
  mm64(av, fkT, g, m0, n0);   // dV[t][e] = sum_d phi(k)[t][d] G[d][e]
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long r = row0 + m0 + i;
    __nv_bfloat16* krow = dqkv + r * lddq + dm + h * D + n0;
    __nv_bfloat16* vrow = dqkv + r * lddq + 2 * dm + h * D + n0;
    const uint2 kin = *reinterpret_cast<const uint2*>(qkv + r * ld + dm + h * D + n0);
    const uint2 kc = *reinterpret_cast<const uint2*>(krow);
    const uint2 vc = *reinterpret_cast<const uint2*>(vrow);
    const float2 k01 = unpack_bf16(kin.x), k23 = unpack_bf16(kin.y);
    const float2 a01 = unpack_bf16(kc.x), a23 = unpack_bf16(kc.y);
    const float2 b01 = unpack_bf16(vc.x), b23 = unpack_bf16(vc.y);
    const float kx[4] = {k01.x, k01.y, k23.x, k23.y};
    const float kcur[4] = {a01.x, a01.y, a23.x, a23.y}, vcur[4] = {b01.x, b01.y, b23.x, b23.y};
    float ko[4], vo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ko[j] = kcur[j] + (ak[i][j] + dz[n0 + j]) * dphi(kx[j]);
      vo[j] = vcur[j] + av[i][j];
    }
    *reinterpret_cast<uint2*>(krow) = make_uint2(pack_bf16(ko[0], ko[1]), pack_bf16(ko[2], ko[3]));
    *reinterpret_cast<uint2*>(vrow) = make_uint2(pack_bf16(vo[0], vo[1]), pack_bf16(vo[2], vo[3]));
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
  constexpr int smem = 2 * TILE_F * 4;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(sla_kv_state_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "cudaFuncSetAttribute(sla_kv_state)");
    attr = true;
  }
  sla_kv_state_kernel<<<B * H * nb, 256, smem, s>>>(qkv, ld, T, H, nb, kvz);
  count_launch();
}

void sla_lin_out(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                 __nv_bfloat16* o, long ldo, float* den, float eps, cudaStream_t s) {
  const int nb = T / 64;
  constexpr int smem = (2 * TILE_F + 128) * 4;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(sla_lin_out_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "cudaFuncSetAttribute(sla_lin_out)");
    attr = true;
  }
  sla_lin_out_kernel<<<B * H * nb, 256, smem, s>>>(qkv, ld, T, H, nb, state, o, ldo, den, eps);
  count_launch();
}

void sla_lin_bwd_q(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                   const __nv_bfloat16* o, long ldo, const __nv_bfloat16* dout, long lddo,
                   const float* den, __nv_bfloat16* dsz, __nv_bfloat16* dqkv, long lddq,
                   cudaStream_t s) {
  const int nb = T / 64;
  constexpr int smem = (4 * TILE_F + 128) * 4;
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
  constexpr int smem = (4 * TILE_F + 64) * 4;
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
