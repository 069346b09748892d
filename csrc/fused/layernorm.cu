// LayerNorm forward / backward over rows of a bf16 matrix (sm_100a).
//
//   y = (x - mean) * rstd * w + b            (w, b optional: plain normalisation)
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = dy * w
//   dw += sum_rows dy * xhat,  db += sum_rows dy
//
// One warp per row, each lane holding D/32 elements (8 per 16-byte access) in registers:
// x is read once and y written once. Statistics are two-pass in registers (mean first,
// then the centred sum of squares), so no E[x^2] - E[x]^2 cancellation. The backward
// keeps per-lane column partials of dw / db over the CTA's rows and adds them with one
// fp32 atomic per column per CTA.
//
// Replaces the reference's Triton normalisation kernels (training/kernels/
// fused_normalize.py:20-191: normalise fwd/bwd and affine LayerNorm) and nn.LayerNorm in
// the V-JEPA / ViT teacher blocks (core/vjepa_backbone.py:92-131).
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "fused.h"

namespace ddb {
namespace {

template <int VEC>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, int lane, float (&v)[VEC][8]) {
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    uint4 u = ld_global_v4(p + (i * 32 + lane) * 8);
    uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(wd[j]);
      v[i][2 * j] = f.x;
      v[i][2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

template <int VEC>
__global__ void __launch_bounds__(256) ln_fwd_kernel(LayerNormArgs a) {
  constexpr int D = VEC * 256;
  const int lane = threadIdx.x & 31;
  const long row = static_cast<long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= a.M) return;
  float v[VEC][8];
  load_row<VEC>(a.x + row * D, lane, v);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) s += v[i][j];
  const float mean = warp_sum(s) / D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float c = v[i][j] - mean;
      q += c * c;
    }
  const float rstd = rsqrtf(warp_sum(q) / D + a.eps);
  if (lane == 0) {
    if (a.mean) a.mean[row] = mean;
    if (a.rstd) a.rstd[row] = rstd;
  }
  __nv_bfloat16* yr = a.y + row * D;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t = (v[i][j] - mean) * rstd;
      if (a.w) t *= __ldg(a.w + c + j);
      if (a.b) t += __ldg(a.b + c + j);
      o[j] = t;
    }
    st_global_v4(yr + c, pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]),
                 pack_bf16(o[6], o[7]));
  }
}

template <int VEC>
__global__ void __launch_bounds__(256) ln_bwd_kernel(LayerNormArgs a, int rows_per_cta) {
  constexpr int D = VEC * 256;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long row0 = static_cast<long>(blockIdx.x) * rows_per_cta;
  const long row1 = min(row0 + rows_per_cta, static_cast<long>(a.M));
  float pw[VEC][8], pb[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) pw[i][j] = pb[i][j] = 0.f;
  for (long row = row0 + warp; row < row1; row += 8) {
    const float mean = a.mean[row], rstd = a.rstd[row];
    float xv[VEC][8], gv[VEC][8];
    load_row<VEC>(a.x + row * D, lane, xv);
    load_row<VEC>(a.dy + row * D, lane, gv);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = (xv[i][j] - mean) * rstd;
        const float dy = gv[i][j];
        pw[i][j] += dy * xh;
        pb[i][j] += dy;
        const float g = a.w ? dy * __ldg(a.w + c + j) : dy;
        xv[i][j] = xh;
        gv[i][j] = g;
        s1 += g;
        s2 += g * xh;
      }
    }
    s1 = warp_sum(s1) / D;
    s2 = warp_sum(s2) / D;
    __nv_bfloat16* dxr = a.dx + row * D;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 8;
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rstd * (gv[i][j] - s1 - xv[i][j] * s2);
      st_global_v4(dxr + c, pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]),
                   pack_bf16(o[6], o[7]));
    }
  }
  // column partials: reduce the 8 warps in shared memory, one atomic per column
  __shared__ float red[8][256];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      float* dst = which == 0 ? a.dw : a.db;
      __syncthreads();
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = which == 0 ? pw[i][j] : pb[i][j];
      __syncthreads();
      if (dst != nullptr) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
        // element threadIdx.x of this 256-chunk = lane l*8+j of chunk i -> column
        const int l = threadIdx.x >> 3, j = threadIdx.x & 7;
        atomicAdd(dst + (i * 32 + l) * 8 + j, t);
      }
    }
  }
}

template <template <int> class K, typename... Args>
void dispatch_vec(int vec, dim3 grid, cudaStream_t st, Args... args) {
  switch (vec) {
#define DDB_V(V)                                   \
  case V:                                          \
    K<V>::launch(grid, st, args...);               \
    return;
    DDB_V(1) DDB_V(2) DDB_V(3) DDB_V(4) DDB_V(5) DDB_V(6) DDB_V(8)
#undef DDB_V
    default:
      throw std::runtime_error("layernorm: D must be 256 * {1,2,3,4,5,6,8}");
  }
}

template <int V>
struct FwdL {
  static void launch(dim3 g, cudaStream_t st, LayerNormArgs a) {
    ln_fwd_kernel<V><<<g, 256, 0, st>>>(a);
  }
};
template <int V>
struct BwdL {
  static void launch(dim3 g, cudaStream_t st, LayerNormArgs a, int rpc) {
    ln_bwd_kernel<V><<<g, 256, 0, st>>>(a, rpc);
  }
};

}  // namespace

void layernorm_fwd(const LayerNormArgs& a, cudaStream_t stream) {
  if (a.D % 256 != 0) throw std::runtime_error("layernorm: D must be a multiple of 256");
  if (a.M <= 0) return;
  dispatch_vec<FwdL>(a.D / 256, dim3(static_cast<unsigned>((a.M + 7) / 8)), stream, a);
  count_launch();
  check_cuda(cudaGetLastError(), "ln_fwd_kernel launch");
}

void layernorm_bwd(const LayerNormArgs& a, cudaStream_t stream) {
  if (a.D % 256 != 0) throw std::runtime_error("layernorm: D must be a multiple of 256");
  if (a.M <= 0) return;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const long want = 4L * num_sms(dev);
  const int rpc = static_cast<int>(std::max<long>(8, (a.M + want - 1) / want));
  const unsigned grid = static_cast<unsigned>((a.M + rpc - 1) / rpc);
  dispatch_vec<BwdL>(a.D / 256, dim3(grid), stream, a, rpc);
  count_launch();
  check_cuda(cudaGetLastError(), "ln_bwd_kernel launch");
}

}  // namespace ddb
