// Flat-buffer AdamW (+ bf16 compute-copy write), casts, squared norm, rotary rotation.
//
// AdamW follows torch.optim.AdamW (decoupled decay, bias-corrected moments) applied to a
// flat fp32 buffer: one read of grad/master/m/v and one write of master/m/v/bf16 copy
// per element, 4 elements per thread access. The clip multiplier is a device scalar so
// gradient clipping needs no host synchronisation.
#include <cuda_bf16.h>
#include <cstdint>

#include "../common/ptx.cuh"
#include "fused.h"
#include "../common/tma.h"

namespace ddb {
namespace {

__global__ void __launch_bounds__(256) adamw_kernel(AdamWArgs a) {
  const float clip = a.clip ? *a.clip : 1.f;
  const float gs = a.grad_scale * clip;
  const float step = a.lr / a.bc1;
  const float inv_bc2 = 1.f / a.bc2;
  const long n4 = a.n / 4;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n4; i += static_cast<long>(gridDim.x) * 256) {
    float4 p = reinterpret_cast<float4*>(a.master)[i];
    float4 g = reinterpret_cast<const float4*>(a.grad)[i];
    float4 m = reinterpret_cast<float4*>(a.m)[i];
    float4 v = reinterpret_cast<float4*>(a.v)[i];
    float pa[4] = {p.x, p.y, p.z, p.w}, ga[4] = {g.x, g.y, g.z, g.w};
    float ma[4] = {m.x, m.y, m.z, m.w}, va[4] = {v.x, v.y, v.z, v.w};
    const bool decay = (4 * i) < a.decay_end;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gg = ga[j] * gs;
      ma[j] = a.b1 * ma[j] + (1.f - a.b1) * gg;
      va[j] = a.b2 * va[j] + (1.f - a.b2) * gg * gg;
      if (decay) pa[j] *= (1.f - a.lr * a.wd);
      pa[j] -= step * ma[j] / (sqrtf(va[j] * inv_bc2) + a.eps);
    }
    reinterpret_cast<float4*>(a.master)[i] = make_float4(pa[0], pa[1], pa[2], pa[3]);
    reinterpret_cast<float4*>(a.m)[i] = make_float4(ma[0], ma[1], ma[2], ma[3]);
    reinterpret_cast<float4*>(a.v)[i] = make_float4(va[0], va[1], va[2], va[3]);
    if (a.compute) {
      uint2 o = make_uint2(pack_bf16(pa[0], pa[1]), pack_bf16(pa[2], pa[3]));
      reinterpret_cast<uint2*>(a.compute)[i] = o;
    }
  }
}

__global__ void cast_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long n4) {
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n4; i += static_cast<long>(gridDim.x) * 256) {
    float4 p = reinterpret_cast<const float4*>(src)[i];
    reinterpret_cast<uint2*>(dst)[i] = make_uint2(pack_bf16(p.x, p.y), pack_bf16(p.z, p.w));
  }
}

__global__ void sq_norm_kernel(const float* __restrict__ x, long n4, float* out) {
  float s = 0.f;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n4; i += static_cast<long>(gridDim.x) * 256) {
    float4 p = reinterpret_cast<const float4*>(x)[i];
    s += p.x * p.x + p.y * p.y + p.z * p.z + p.w * p.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += red[k];
    atomicAdd(out, t);
  }
}

// One thread per (row, 8-column chunk) of the rotated region.
__global__ void rope_rotate_kernel(__nv_bfloat16* x, long ld, int M, int rot_cols,
                                   const float2* __restrict__ tab, int head_dim, int rows_per_seq,
                                   int pos_offset, bool inverse) {
  const int chunks = rot_cols / 8;
  const long idx = blockIdx.x * 256L + threadIdx.x;
  if (idx >= static_cast<long>(M) * chunks) return;
  const int row = static_cast<int>(idx / chunks);
  const int c = static_cast<int>(idx % chunks) * 8;
  const int pos = row % rows_per_seq + pos_offset;
  const float2* t = tab + static_cast<long>(pos) * (head_dim / 2) + (c % head_dim) / 2;
  __nv_bfloat16* p = x + static_cast<long>(row) * ld + c;
  uint4 u = ld_global_v4(p);
  uint32_t w[4] = {u.x, u.y, u.z, u.w};
  const float sgn = inverse ? -1.f : 1.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = unpack_bf16(w[j]);
    float2 cs = __ldg(t + j);
    const float sn = sgn * cs.y;
    w[j] = pack_bf16(f.x * cs.x - f.y * sn, f.x * sn + f.y * cs.x);
  }
  st_global_v4(p, w[0], w[1], w[2], w[3]);
}

int grid_for(long n4) {
  long g = (n4 + 255) / 256;
  return static_cast<int>(g < 148L * 16 ? (g < 1 ? 1 : g) : 148L * 16);
}

}  // namespace

void adamw_flat(const AdamWArgs& a, cudaStream_t s) {
  if (a.n % 4 != 0) throw std::runtime_error("adamw_flat: length must be a multiple of 4");
  count_launch();
  adamw_kernel<<<grid_for(a.n / 4), 256, 0, s>>>(a);
}

void cast_f32_bf16(const float* src, __nv_bfloat16* dst, long n, cudaStream_t s) {
  if (n % 4 != 0) throw std::runtime_error("cast_f32_bf16: length must be a multiple of 4");
  count_launch();
  cast_kernel<<<grid_for(n / 4), 256, 0, s>>>(src, dst, n / 4);
}

void sq_norm_f32(const float* x, long n, float* out, cudaStream_t s) {
  if (n % 4 != 0) throw std::runtime_error("sq_norm_f32: length must be a multiple of 4");
  count_launch();
  sq_norm_kernel<<<grid_for(n / 4), 256, 0, s>>>(x, n / 4, out);
}

void rope_rotate_bf16(__nv_bfloat16* x, long ld, int M, int rot_cols, const float2* tab,
                      int head_dim, int rows_per_seq, int pos_offset, bool inverse,
                      cudaStream_t s) {
  const long n = static_cast<long>(M) * (rot_cols / 8);
  count_launch();
  rope_rotate_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, s>>>(
      x, ld, M, rot_cols, tab, head_dim, rows_per_seq, pos_offset, inverse);
}

}  // namespace ddb
