// Fused AdaLN-modulated RMSNorm, forward and backward (sm_100a).
//
//   h = rmsnorm(x) * w * (1 + scale[g]) + shift[g],   g = row / rows_per_group
//
// The per-group (per-frame) modulation comes from the AdaLN projection of the
// conditioning (reference layers/nn_helpers.py:92-139 applied per frame). One warp owns
// one row at a time; each lane holds d/32 contiguous-by-8 bf16 elements, so x is read
// once and h written once (HBM-bound). The backward kernel also accumulates the
// norm-weight and modulation gradients (column sums over each group's rows) and can add
// the residual-stream gradient, so a block's backward needs no separate add.
#include <cuda_bf16.h>
#include <cstdint>

#include "../common/ptx.cuh"
#include "fused.h"
#include "../common/tma.h"

namespace ddb {
namespace {

// rows per CTA: the largest divisor of the group size up to `cap`, so a CTA's rows all
// belong to one group (one set of modulation vectors)
__host__ __device__ inline int rows_per_cta_for(int rows_per_group, int cap) {
  int r = rows_per_group < cap ? rows_per_group : cap;
  while (rows_per_group % r) --r;
  return r;
}

// Forward. A CTA (8 warps) takes up to 64 rows of one group; each lane first folds the
// group's modulation into two per-column vectors (a = w * (1 + scale), b = shift) for its
// columns, so a row needs only its x: h = x * rstd * a + b. Warps walk rows 8 apart and
// load the next row before reducing the current one (two rows in flight per warp).
template <int VEC>  // VEC = d / 256 (8 bf16 per 16-byte access, 32 lanes)
__global__ void __launch_bounds__(256, VEC <= 4 ? 2 : 1) adaln_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
    const float* __restrict__ mod, long ld_mod, int scale_off, int shift_off,
    int rows_per_group, int rows_per_cta, __nv_bfloat16* __restrict__ h,
    float* __restrict__ rstd_out, int M, float eps) {
  constexpr int D = VEC * 256;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row0 = blockIdx.x * rows_per_cta;
  const int row_end = min(row0 + rows_per_cta, M);
  if (row0 >= M) return;
  const float* mg = mod + static_cast<long>(row0 / rows_per_group) * ld_mod;
  float av[VEC][8], bv[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
#pragma unroll
    for (int j = 0; j < 8; j += 4) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w + c + j));
      const float4 sc = __ldg(reinterpret_cast<const float4*>(mg + scale_off + c + j));
      const float4 sh = __ldg(reinterpret_cast<const float4*>(mg + shift_off + c + j));
      av[i][j] = wv.x * (1.f + sc.x);
      av[i][j + 1] = wv.y * (1.f + sc.y);
      av[i][j + 2] = wv.z * (1.f + sc.z);
      av[i][j + 3] = wv.w * (1.f + sc.w);
      bv[i][j] = sh.x;
      bv[i][j + 1] = sh.y;
      bv[i][j + 2] = sh.z;
      bv[i][j + 3] = sh.w;
    }
  }
  uint4 cur[VEC], nxt[VEC];
  int row = row0 + warp;
  if (row < row_end) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) cur[i] = ld_global_v4(x + static_cast<long>(row) * D + (i * 32 + lane) * 8);
  }
  for (; row < row_end; row += 8) {
    const int rn = row + 8;
    if (rn < row_end) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) nxt[i] = ld_global_v4(x + static_cast<long>(rn) * D + (i * 32 + lane) * 8);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const uint32_t wd[4] = {cur[i].x, cur[i].y, cur[i].z, cur[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16(wd[j]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / D + eps);
    if (lane == 0 && rstd_out) rstd_out[row] = r;
    __nv_bfloat16* hr = h + static_cast<long>(row) * D;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const uint32_t wd[4] = {cur[i].x, cur[i].y, cur[i].z, cur[i].w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16(wd[j]);
        o[j] = pack_bf16(fmaf(f.x * r, av[i][2 * j], bv[i][2 * j]),
                         fmaf(f.y * r, av[i][2 * j + 1], bv[i][2 * j + 1]));
      }
      st_global_v4(hr + (i * 32 + lane) * 8, o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) cur[i] = nxt[i];
  }
}

// Backward. A CTA (8 warps) takes up to 128 rows of one group in chunks of CH rows. The
// chunk's x and dh rows (contiguous) arrive in shared memory by two bulk copies
// (double-buffered, the next chunk in flight while this one is processed). Phase A:
// each warp turns its rows into dx (+ the residual gradient) from shared memory. Phase
// B: each thread owns D/256 columns and accumulates, over the chunk's rows, the two
// column sums every parameter gradient is made of, S1 = sum dh and S2 = sum dh * n
// (n = x * rstd): d shift = S1, d scale = w * S2, d w = (1 + scale) * S2. Nothing
// per-column lives in registers across rows except these 2 * D/256 sums.
template <int VEC>
struct AdaLNBwdCfg {
  static constexpr int D = VEC * 256;
  static constexpr int CH = VEC <= 3 ? 16 : 8;       // rows per chunk
  static constexpr int BUF = CH * D * 2;             // bytes of one tensor's chunk
  static constexpr int SMEM = 2 * 2 * BUF + 2 * CH * 4 + 64;  // 2 buffers x (x, dh), rstd, barriers
};

template <int VEC>
__global__ void __launch_bounds__(256, VEC <= 3 ? 2 : 1) adaln_bwd_kernel(
    const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ x,
    const float* __restrict__ rstd, const float* __restrict__ w, const float* __restrict__ mod,
    long ld_mod, int scale_off, int shift_off, int rows_per_group, int rows_per_cta,
    const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ dw, float* __restrict__ dmod, long ld_dmod, int M, int* status) {
  using Cfg = AdaLNBwdCfg<VEC>;
  constexpr int D = Cfg::D;
  constexpr int CH = Cfg::CH;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* bx = smem;                     // [2][CH][D] bf16 x
  uint8_t* bg = smem + 2 * Cfg::BUF;      // [2][CH][D] bf16 dh
  float* rs = reinterpret_cast<float*>(smem + 4 * Cfg::BUF);  // [2][CH] rstd
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 4 * Cfg::BUF + 2 * CH * 4 + 16);  // 2

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row0 = blockIdx.x * rows_per_cta;
  const int row_end = min(row0 + rows_per_cta, M);
  const int g = row0 / rows_per_group;
  const float* mg = mod + static_cast<long>(g) * ld_mod;
  const int nchunks = row0 < M ? (row_end - row0 + CH - 1) / CH : 0;

  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  // thread 0: bulk copies of chunk c's x and dh rows (and its rstd) into buffer c & 1
  auto issue = [&](int c) {
    const int r0 = row0 + c * CH;
    const int n = min(CH, row_end - r0);
    const uint32_t bytes = static_cast<uint32_t>(n) * D * 2;
    uint64_t* bar = &full[c & 1];
    fence_proxy_async_smem();  // the buffer's earlier generic-proxy reads come first
    mbar_arrive_expect_tx(bar, 2 * bytes);
    bulk_load(bx + (c & 1) * Cfg::BUF, x + static_cast<long>(r0) * D, bytes, bar);
    bulk_load(bg + (c & 1) * Cfg::BUF, dh + static_cast<long>(r0) * D, bytes, bar);
  };
  if (threadIdx.x == 0 && nchunks > 0) issue(0);

  // per-lane folded modulation for phase A: dn = dh * w * (1 + scale)
  float a2[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
#pragma unroll
    for (int j = 0; j < 8; j += 4) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w + c + j));
      const float4 sc = __ldg(reinterpret_cast<const float4*>(mg + scale_off + c + j));
      a2[i][j] = wv.x * (1.f + sc.x);
      a2[i][j + 1] = wv.y * (1.f + sc.y);
      a2[i][j + 2] = wv.z * (1.f + sc.z);
      a2[i][j + 3] = wv.w * (1.f + sc.w);
    }
  }
  float s1[VEC], s2[VEC];  // phase B column sums of column threadIdx.x + 256 i
#pragma unroll
  for (int i = 0; i < VEC; ++i) s1[i] = s2[i] = 0.f;

  bool ok = true;
  for (int c = 0; c < nchunks; ++c) {
    const int r0 = row0 + c * CH;
    const int n = min(CH, row_end - r0);
    if (threadIdx.x == 0 && c + 1 < nchunks) issue(c + 1);  // its buffer was freed below
    if (threadIdx.x < CH) rs[(c & 1) * CH + threadIdx.x] = threadIdx.x < n ? rstd[r0 + threadIdx.x] : 0.f;
    // bounded wait (all threads); on expiry record the status and stop (uniformly: the
    // block-wide vote is also the barrier that publishes the chunk's rstd)
    long long t0 = clock64();
    bool landed = mbar_try_wait(&full[c & 1], (c >> 1) & 1);
    while (!landed && clock64() - t0 < kSpinLimitCycles) landed = mbar_try_wait(&full[c & 1], (c >> 1) & 1);
    if (__syncthreads_or(!landed)) {
      if (threadIdx.x == 0) {
        if (status) atomicCAS(status, 0, kStatusTimeoutProducer);
        // the next chunk's copies, if issued, land before the CTA exits (bounded)
        if (c + 1 < nchunks) {
          t0 = clock64();
          while (!mbar_try_wait(&full[(c + 1) & 1], ((c + 1) >> 1) & 1) &&
                 clock64() - t0 < kSpinLimitCycles / 8) {
          }
        }
      }
      ok = false;
      break;
    }
    const uint32_t sx = smem_u32(bx + (c & 1) * Cfg::BUF);
    const uint32_t sg = smem_u32(bg + (c & 1) * Cfg::BUF);
    const float* rc = rs + (c & 1) * CH;
    // ---- phase A: dx rows (warp per row)
    for (int k = warp; k < n; k += 8) {
      const float r = rc[k];
      const long row = r0 + k;
      float nv[VEC][8], dn[VEC][8];
      float dot = 0.f;
      uint4 ures[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i)
        ures[i] = dres ? ld_global_v4(dres + row * D + (i * 32 + lane) * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const uint32_t off = static_cast<uint32_t>((k * D + (i * 32 + lane) * 8) * 2);
        uint4 ux, ug;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(ux.x), "=r"(ux.y), "=r"(ux.z), "=r"(ux.w) : "r"(sx + off));
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(ug.x), "=r"(ug.y), "=r"(ug.z), "=r"(ug.w) : "r"(sg + off));
        const uint32_t wx[4] = {ux.x, ux.y, ux.z, ux.w};
        const uint32_t wg[4] = {ug.x, ug.y, ug.z, ug.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fx = unpack_bf16(wx[j]);
          const float2 fg = unpack_bf16(wg[j]);
          nv[i][2 * j] = fx.x * r;
          nv[i][2 * j + 1] = fx.y * r;
          dn[i][2 * j] = fg.x * a2[i][2 * j];
          dn[i][2 * j + 1] = fg.y * a2[i][2 * j + 1];
          dot = fmaf(dn[i][2 * j], nv[i][2 * j], dot);
          dot = fmaf(dn[i][2 * j + 1], nv[i][2 * j + 1], dot);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      dot *= 1.f / D;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        float o8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o8[j] = r * (dn[i][j] - nv[i][j] * dot);
        if (dres) {
          const uint32_t wr[4] = {ures[i].x, ures[i].y, ures[i].z, ures[i].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack_bf16(wr[j]);
            o8[2 * j] += f.x;
            o8[2 * j + 1] += f.y;
          }
        }
        st_global_v4(dx + row * D + (i * 32 + lane) * 8, pack_bf16(o8[0], o8[1]),
                     pack_bf16(o8[2], o8[3]), pack_bf16(o8[4], o8[5]), pack_bf16(o8[6], o8[7]));
      }
    }
    // ---- phase B: column sums (thread per column, rows of the chunk)
    const __nv_bfloat16* cx = reinterpret_cast<const __nv_bfloat16*>(bx + (c & 1) * Cfg::BUF);
    const __nv_bfloat16* cg = reinterpret_cast<const __nv_bfloat16*>(bg + (c & 1) * Cfg::BUF);
    for (int k = 0; k < n; ++k) {
      const float r = rc[k];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int col = threadIdx.x + 256 * i;
        const float gg = __bfloat162float(cg[k * D + col]);
        s1[i] += gg;
        s2[i] = fmaf(gg, __bfloat162float(cx[k * D + col]) * r, s2[i]);
      }
    }
    __syncthreads();  // buffer c & 1 and its rstd slots are free for chunk c + 2
  }
  if (!ok) return;
  float* dmg = dmod + static_cast<long>(g) * ld_dmod;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int col = threadIdx.x + 256 * i;
    atomicAdd(dmg + shift_off + col, s1[i]);
    atomicAdd(dmg + scale_off + col, w[col] * s2[i]);
    if (dw) atomicAdd(dw + col, (1.f + mg[scale_off + col]) * s2[i]);
  }
}

}  // namespace

void adaln_rmsnorm_fwd(const AdaLNArgs& a, cudaStream_t s) {
  count_launch();
  const int rpc = rows_per_cta_for(a.rows_per_group, 64);
  const int grid = (a.M + rpc - 1) / rpc;
  switch (a.D) {
#define CASE(V)                                                                                   \
  case V * 256:                                                                                   \
    adaln_fwd_kernel<V><<<grid, 256, 0, s>>>(a.x, a.w, a.mod, a.ld_mod, a.scale_off, a.shift_off, \
                                             a.rows_per_group, rpc, a.h, a.rstd, a.M, a.eps);    \
    break;
    CASE(1) CASE(2) CASE(3) CASE(4) CASE(6) CASE(8)
#undef CASE
    default:
      throw std::runtime_error("adaln_rmsnorm_fwd: unsupported width");
  }
}

void adaln_rmsnorm_bwd(const AdaLNArgs& a, cudaStream_t s) {
  count_launch();
  // rows per CTA: the largest divisor of rows_per_group up to 128, so a CTA never
  // straddles two groups
  const int rpc = rows_per_cta_for(a.rows_per_group, 128);
  const int grid = (a.M + rpc - 1) / rpc;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  int* status = device_status(dev);
  switch (a.D) {
#define CASE(V)                                                                                   \
  case V * 256: {                                                                                 \
    static bool attr = false;                                                                     \
    if (!attr) {                                                                                  \
      check_cuda(cudaFuncSetAttribute(adaln_bwd_kernel<V>,                                        \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,                \
                                      AdaLNBwdCfg<V>::SMEM),                                      \
                 "cudaFuncSetAttribute(adaln_bwd)");                                              \
      attr = true;                                                                                \
    }                                                                                             \
    adaln_bwd_kernel<V><<<grid, 256, AdaLNBwdCfg<V>::SMEM, s>>>(                                  \
        a.dh, a.x, a.rstd, a.w, a.mod, a.ld_mod, a.scale_off, a.shift_off, a.rows_per_group, rpc, \
        a.dres, a.dx, a.dw, a.dmod, a.ld_dmod, a.M, status);                                      \
    break;                                                                                        \
  }
    CASE(1) CASE(2) CASE(3) CASE(4) CASE(6) CASE(8)
#undef CASE
    default:
      throw std::runtime_error("adaln_rmsnorm_bwd: unsupported width");
  }
}

}  // namespace ddb
