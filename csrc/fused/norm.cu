// Fused AdaLN-modulated RMSNorm, forward and backward (sm_100a).
//
//   h = rmsnorm(x) * w * (1 + scale[g]) + shift[g],   g = row / rows_per_group
//
// The per-group (per-frame) modulation comes from the AdaLN projection of the
// conditioning (reference layers/nn_helpers.py:92-139 applied per frame). One warp owns
// one row; each lane holds d/32 contiguous-by-8 bf16 elements in registers, so x is
// read once and h written once (HBM-bound). The backward kernel also accumulates the
// norm-weight and modulation gradients (column sums over each group's rows) and can add
// the residual-stream gradient, so a block's backward needs no separate add.
#include <cuda_bf16.h>
#include <cstdint>

#include "../common/ptx.cuh"
#include "fused.h"
#include "../common/tma.h"

namespace ddb {
namespace {

template <int VEC>  // VEC = d / 256 (8 bf16 per 16-byte access, 32 lanes)
__global__ void __launch_bounds__(256) adaln_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
    const float* __restrict__ mod, long ld_mod, int scale_off, int shift_off,
    int rows_per_group, __nv_bfloat16* __restrict__ h, float* __restrict__ rstd_out, int M,
    float eps) {
  constexpr int D = VEC * 256;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const __nv_bfloat16* xr = x + static_cast<long>(row) * D;
  float v[VEC][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    uint4 u = ld_global_v4(xr + (i * 32 + lane) * 8);
    uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(wd[j]);
      v[i][2 * j] = f.x;
      v[i][2 * j + 1] = f.y;
      ss += f.x * f.x + f.y * f.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = r;
  const float* mg = mod + static_cast<long>(row / rows_per_group) * ld_mod;
  __nv_bfloat16* hr = h + static_cast<long>(row) * D;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; j += 4) {
      float4 wv = __ldg(reinterpret_cast<const float4*>(w + c + j));
      float4 sc = __ldg(reinterpret_cast<const float4*>(mg + scale_off + c + j));
      float4 sh = __ldg(reinterpret_cast<const float4*>(mg + shift_off + c + j));
      o[j + 0] = v[i][j + 0] * r * wv.x * (1.f + sc.x) + sh.x;
      o[j + 1] = v[i][j + 1] * r * wv.y * (1.f + sc.y) + sh.y;
      o[j + 2] = v[i][j + 2] * r * wv.z * (1.f + sc.z) + sh.z;
      o[j + 3] = v[i][j + 3] * r * wv.w * (1.f + sc.w) + sh.w;
    }
    st_global_v4(hr + c, pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]),
                 pack_bf16(o[6], o[7]));
  }
}

// Backward. Each CTA (8 warps) walks `rows_per_cta` rows that all belong to one group,
// keeping per-lane column partials of dw, dscale, dshift in registers.
template <int VEC>
__global__ void __launch_bounds__(256) adaln_bwd_kernel(
    const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ x,
    const float* __restrict__ rstd, const float* __restrict__ w, const float* __restrict__ mod,
    long ld_mod, int scale_off, int shift_off, int rows_per_group, int rows_per_cta,
    const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ dw, float* __restrict__ dmod, long ld_dmod, int M) {
  constexpr int D = VEC * 256;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row0 = blockIdx.x * rows_per_cta;
  const int g = row0 / rows_per_group;
  const float* mg = mod + static_cast<long>(g) * ld_mod;
  float pw[VEC][8], psc[VEC][8], psh[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) pw[i][j] = psc[i][j] = psh[i][j] = 0.f;

  for (int row = row0 + warp; row < min(row0 + rows_per_cta, M); row += 8) {
    const float r = rstd[row];
    const __nv_bfloat16* xr = x + static_cast<long>(row) * D;
    const __nv_bfloat16* gr = dh + static_cast<long>(row) * D;
    float n[VEC][8], dn[VEC][8];
    float dot = 0.f;
    // the residual gradient is loaded with x and dh so a row costs one memory round trip
    const __nv_bfloat16* rr = dres ? dres + static_cast<long>(row) * D : nullptr;
    uint4 ures[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) ures[i] = rr ? ld_global_v4(rr + (i * 32 + lane) * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 8;
      uint4 ux = ld_global_v4(xr + c);
      uint4 ug = ld_global_v4(gr + c);
      uint32_t wx[4] = {ux.x, ux.y, ux.z, ux.w};
      uint32_t wg[4] = {ug.x, ug.y, ug.z, ug.w};
      float xv[8], gv[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 a = unpack_bf16(wx[j]);
        float2 b = unpack_bf16(wg[j]);
        xv[2 * j] = a.x;
        xv[2 * j + 1] = a.y;
        gv[2 * j] = b.x;
        gv[2 * j + 1] = b.y;
      }
#pragma unroll
      for (int j = 0; j < 8; j += 4) {
        float4 wv = __ldg(reinterpret_cast<const float4*>(w + c + j));
        float4 sc = __ldg(reinterpret_cast<const float4*>(mg + scale_off + c + j));
        float wa[4] = {wv.x, wv.y, wv.z, wv.w};
        float sa[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float nn = xv[j + q] * r;
          const float y = nn * wa[q];
          const float gg = gv[j + q];
          psh[i][j + q] += gg;
          psc[i][j + q] += gg * y;
          const float dy = gg * (1.f + sa[q]);
          pw[i][j + q] += dy * nn;
          const float d_n = dy * wa[q];
          n[i][j + q] = nn;
          dn[i][j + q] = d_n;
          dot += d_n * nn;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot /= D;
    __nv_bfloat16* dxr = dx + static_cast<long>(row) * D;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 8;
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = r * (dn[i][j] - n[i][j] * dot);
      if (rr) {
        const uint4 u = ures[i];
        uint32_t wr[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = unpack_bf16(wr[j]);
          o[2 * j] += f.x;
          o[2 * j + 1] += f.y;
        }
      }
      st_global_v4(dxr + c, pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]),
                   pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
    }
  }
  // reduce the 8 warps' column partials through shared memory, 256 columns at a time
  __shared__ float red[8][256];
  float* dmg = dmod + static_cast<long>(g) * ld_dmod;
  auto reduce_store = [&](float (&p)[VEC][8], float* dst) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = p[i][j];
      __syncthreads();
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) s += red[k][threadIdx.x];
      atomicAdd(dst + i * 256 + threadIdx.x, s);
      __syncthreads();
    }
  };
  if (dw) reduce_store(pw, dw);
  reduce_store(psc, dmg + scale_off);
  reduce_store(psh, dmg + shift_off);
}

}  // namespace

void adaln_rmsnorm_fwd(const AdaLNArgs& a, cudaStream_t s) {
  count_launch();
  const int grid = (a.M + 7) / 8;
  switch (a.D) {
#define CASE(V)                                                                                  \
  case V * 256:                                                                                  \
    adaln_fwd_kernel<V><<<grid, 256, 0, s>>>(a.x, a.w, a.mod, a.ld_mod, a.scale_off, a.shift_off, \
                                             a.rows_per_group, a.h, a.rstd, a.M, a.eps);         \
    break;
    CASE(1) CASE(2) CASE(3) CASE(4) CASE(6) CASE(8)
#undef CASE
    default:
      throw std::runtime_error("adaln_rmsnorm_fwd: unsupported width");
  }
}

void adaln_rmsnorm_bwd(const AdaLNArgs& a, cudaStream_t s) {
  count_launch();
  // rows per CTA: the largest divisor of rows_per_group up to 64, so a CTA never
  // straddles two groups
  int rpc = a.rows_per_group < 64 ? a.rows_per_group : 64;
  while (a.rows_per_group % rpc) --rpc;
  const int grid = (a.M + rpc - 1) / rpc;
  switch (a.D) {
#define CASE(V)                                                                                   \
  case V * 256:                                                                                   \
    adaln_bwd_kernel<V><<<grid, 256, 0, s>>>(a.dh, a.x, a.rstd, a.w, a.mod, a.ld_mod, a.scale_off, \
                                             a.shift_off, a.rows_per_group, rpc, a.dres, a.dx,    \
                                             a.dw, a.dmod, a.ld_dmod, a.M);                       \
    break;
    CASE(1) CASE(2) CASE(3) CASE(4)
#undef CASE
    default:
      throw std::runtime_error("adaln_rmsnorm_bwd: unsupported width");
  }
}

}  // namespace ddb
