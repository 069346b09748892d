// GroupNorm (+ SiLU) for channels-last video activations [B, P, C], P = T*H*W.
//
// Forward:  pre = (x - mean_g) * rstd_g * w_c + b_c,  y = silu(pre) (or pre)
// Backward: with dpre = dy * silu'(pre) and xhat = (x - mean) * rstd,
//           dx = rstd * (w*dpre - mean_g(w*dpre) - xhat * mean_g(w*dpre*xhat)),
//           dw_c = sum dpre*xhat, db_c = sum dpre.
// Statistics are reduced per channel with fp32 block partials and fp64 atomics, then
// folded into groups by a tiny finalize kernel, so E[x^2] - E[x]^2 does not cancel in
// fp32 over ~10^6-element groups. Vectorised 8 channels (16 bytes) per thread.
//
// Replaces nn.GroupNorm(min(32, C), C) + F.silu of the reference VAE blocks
// (models/vae3d.py:239-285 ResidualBlock3D, :693-694 / :818-819 norm_out).
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "groupnorm.h"

namespace ddb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = ld_global_v4(p);
  uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = unpack_bf16(w[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  st_global_v4(p, pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
               pack_bf16(v[6], v[7]));
}

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

// Per-channel sums over a chunk of rows -> fp64 atomics into acc[b][c][2].
// Mode 0: (x, x^2). Mode 1 (backward): (dpre, dpre * xhat).
template <int MODE>
__global__ void __launch_bounds__(kThreads) gn_reduce_kernel(GroupNormArgs a, int rows_per_block) {
  extern __shared__ float red[];  // [rows_per_iter][C][2]
  const int tpr = a.C / 8;
  const int rpi = kThreads / tpr;
  const int lr = threadIdx.x / tpr;
  const int cv = (threadIdx.x % tpr) * 8;
  const int b = blockIdx.y;
  const long r0 = static_cast<long>(blockIdx.x) * rows_per_block;
  const long r1 = std::min<long>(a.P, r0 + rows_per_block);
  float s[8], q[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = q[j] = 0.f;
  float w[8], bb[8], mean = 0.f, rstd = 0.f;
  if (MODE == 1 && lr < rpi) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      w[j] = a.w[cv + j];
      bb[j] = a.b ? a.b[cv + j] : 0.f;
    }
  }
  if (lr < rpi) {
    for (long r = r0 + lr; r < r1; r += rpi) {
      const long off = (static_cast<long>(b) * a.P + r) * a.C + cv;
      float x[8];
      load8(a.x + off, x);
      if constexpr (MODE == 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          s[j] += x[j];
          q[j] += x[j] * x[j];
        }
      } else {
        float dy[8];
        load8(a.dy + off, dy);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int g = (cv + j) / (a.C / a.G);
          mean = a.stats[(b * a.G + g) * 2];
          rstd = a.stats[(b * a.G + g) * 2 + 1];
          const float xh = (x[j] - mean) * rstd;
          float dp = dy[j];
          if (a.silu) {
            const float pre = xh * w[j] + bb[j];
            const float sg = sigm(pre);
            dp *= sg * (1.f + pre * (1.f - sg));
          }
          s[j] += dp;
          q[j] += dp * xh;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      red[(lr * a.C + cv + j) * 2] = s[j];
      red[(lr * a.C + cv + j) * 2 + 1] = q[j];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < a.C; c += kThreads) {
    double ts = 0.0, tq = 0.0;
    for (int l = 0; l < rpi; ++l) {
      ts += red[(l * a.C + c) * 2];
      tq += red[(l * a.C + c) * 2 + 1];
    }
    atomicAdd(a.acc + (static_cast<long>(b) * a.C + c) * 2, ts);
    atomicAdd(a.acc + (static_cast<long>(b) * a.C + c) * 2 + 1, tq);
  }
}

// forward: per (b, g) mean and rstd
__global__ void gn_finalize_kernel(GroupNormArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.B * a.G) return;
  const int b = i / a.G, g = i % a.G;
  const int cpg = a.C / a.G;
  double s = 0.0, q = 0.0;
  for (int c = g * cpg; c < (g + 1) * cpg; ++c) {
    s += a.acc[(static_cast<long>(b) * a.C + c) * 2];
    q += a.acc[(static_cast<long>(b) * a.C + c) * 2 + 1];
  }
  const double n = static_cast<double>(a.P) * cpg;
  const double m = s / n;
  const double var = std::max(q / n - m * m, 0.0);
  a.stats[i * 2] = static_cast<float>(m);
  a.stats[i * 2 + 1] = rsqrtf(static_cast<float>(var) + a.eps);
}

// backward: per (b, g) c1 = mean(w * dpre), c2 = mean(w * dpre * xhat)
__global__ void gn_bwd_finalize_kernel(GroupNormArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.B * a.G) return;
  const int b = i / a.G, g = i % a.G;
  const int cpg = a.C / a.G;
  double s = 0.0, q = 0.0;
  for (int c = g * cpg; c < (g + 1) * cpg; ++c) {
    s += a.w[c] * a.acc[(static_cast<long>(b) * a.C + c) * 2];
    q += a.w[c] * a.acc[(static_cast<long>(b) * a.C + c) * 2 + 1];
  }
  const double n = static_cast<double>(a.P) * cpg;
  a.coef[i * 2] = static_cast<float>(s / n);
  a.coef[i * 2 + 1] = static_cast<float>(q / n);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads) gn_apply_kernel(GroupNormArgs a) {
  const long nvec = static_cast<long>(a.B) * a.P * (a.C / 8);
  const int cpg = a.C / a.G;
  for (long i = blockIdx.x * static_cast<long>(kThreads) + threadIdx.x; i < nvec;
       i += static_cast<long>(gridDim.x) * kThreads) {
    const int cv = static_cast<int>(i % (a.C / 8)) * 8;
    const long row = i / (a.C / 8);
    const int b = static_cast<int>(row / a.P);
    const long off = row * a.C + cv;
    float x[8], o[8];
    load8(a.x + off, x);
    if constexpr (MODE == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int g = (cv + j) / cpg;
        const float m = a.stats[(b * a.G + g) * 2], rs = a.stats[(b * a.G + g) * 2 + 1];
        float p = (x[j] - m) * rs * a.w[cv + j] + (a.b ? a.b[cv + j] : 0.f);
        o[j] = a.silu ? p * sigm(p) : p;
      }
      store8(a.y + off, o);
    } else {
      float dy[8];
      load8(a.dy + off, dy);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int g = (cv + j) / cpg;
        const float m = a.stats[(b * a.G + g) * 2], rs = a.stats[(b * a.G + g) * 2 + 1];
        const float xh = (x[j] - m) * rs;
        const float wj = a.w[cv + j];
        float dp = dy[j];
        if (a.silu) {
          const float pre = xh * wj + (a.b ? a.b[cv + j] : 0.f);
          const float sg = sigm(pre);
          dp *= sg * (1.f + pre * (1.f - sg));
        }
        o[j] = rs * (wj * dp - a.coef[(b * a.G + g) * 2] - xh * a.coef[(b * a.G + g) * 2 + 1]);
      }
      store8(a.dx + off, o);
    }
  }
}

void check(const GroupNormArgs& a) {
  if (a.C % 8 != 0 || a.C / 8 > kThreads || a.G <= 0 || a.C % a.G != 0)
    throw std::runtime_error("groupnorm: C must be a multiple of 8, <= 2048, divisible by G");
}

int reduce_blocks_per_batch(const GroupNormArgs& a, int& rows_per_block) {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const int want = std::max(1, 4 * num_sms(dev) / std::max(1, a.B));
  rows_per_block = static_cast<int>(std::max<long>(16, (a.P + want - 1) / want));
  return static_cast<int>((a.P + rows_per_block - 1) / rows_per_block);
}

template <int MODE>
void launch_reduce(const GroupNormArgs& a, cudaStream_t st) {
  int rpb = 0;
  const int nb = reduce_blocks_per_batch(a, rpb);
  const int rpi = kThreads / (a.C / 8);
  const size_t smem = static_cast<size_t>(rpi) * a.C * 2 * sizeof(float);
  auto kern = gn_reduce_kernel<MODE>;
  if (smem > 48 * 1024)
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)),
               "cudaFuncSetAttribute(gn reduce)");
  kern<<<dim3(nb, a.B), kThreads, smem, st>>>(a, rpb);
  count_launch();
  check_cuda(cudaGetLastError(), "gn_reduce_kernel launch");
}

template <int MODE>
void launch_apply(const GroupNormArgs& a, cudaStream_t st) {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const long nvec = static_cast<long>(a.B) * a.P * (a.C / 8);
  const int grid = static_cast<int>(std::min<long>((nvec + kThreads - 1) / kThreads,
                                                   8L * num_sms(dev)));
  gn_apply_kernel<MODE><<<std::max(grid, 1), kThreads, 0, st>>>(a);
  count_launch();
  check_cuda(cudaGetLastError(), "gn_apply_kernel launch");
}

}  // namespace

void groupnorm_fwd(const GroupNormArgs& a, cudaStream_t st) {
  check(a);
  check_cuda(cudaMemsetAsync(a.acc, 0, sizeof(double) * a.B * a.C * 2, st), "memset acc");
  launch_reduce<0>(a, st);
  gn_finalize_kernel<<<(a.B * a.G + 127) / 128, 128, 0, st>>>(a);
  count_launch();
  check_cuda(cudaGetLastError(), "gn_finalize_kernel launch");
  launch_apply<0>(a, st);
}

void groupnorm_bwd(const GroupNormArgs& a, cudaStream_t st) {
  check(a);
  check_cuda(cudaMemsetAsync(a.acc, 0, sizeof(double) * a.B * a.C * 2, st), "memset acc");
  launch_reduce<1>(a, st);
  gn_bwd_finalize_kernel<<<(a.B * a.G + 127) / 128, 128, 0, st>>>(a);
  count_launch();
  check_cuda(cudaGetLastError(), "gn_bwd_finalize_kernel launch");
  launch_apply<1>(a, st);
}

}  // namespace ddb
