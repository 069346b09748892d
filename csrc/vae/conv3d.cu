// Causal 3-D convolution for the video VAE as a persistent implicit GEMM on tcgen05.
//
// Activations are channels-last [B, T, H, W, C]. A forward output tile is 128 output
// positions of one (b, t) frame laid out as an hbox x wbox patch (wbox * hbox = 128) by
// 128 output channels. The K loop walks (tap, 64-channel chunk); for each step the A
// tile is ONE 5-D TMA box {64 ch, wbox, hbox, 1, 1} of the input at the tap-shifted
// coordinate. Causal temporal padding and spatial zero padding are never materialised:
// a box that starts before 0 or runs past the end is zero-filled by the TMA unit. The
// channel coordinate (the innermost, x) is always a multiple of 64, so every copy
// starts on a 128-byte boundary. B tiles are 128 x 64 slices of the weights
// [Cout, kt*kh*kw*Cin] (tap-major, channels fastest).
//
// The weight gradient uses the same machinery with K = output positions: A = dy
// ([pos][cout], cout contiguous: an MN-major operand), B = the tap-shifted input
// ([pos][cin], MN-major), 64 positions per K step; position ranges are split over CTAs
// and reduced into an fp32 dw with vector reductions.
//
// Roles (192 threads, 1 CTA/SM): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2-5 epilogue (TMEM lane quadrant = warp % 4); 6-stage ring, double-buffered
// 2 x 128-column accumulator. Every wait is bounded (status word + abort flag).
//
// Replaces the cuDNN nn.Conv3d inside CausalConv3d (reference models/vae3d.py:119-173)
// used by ResidualBlock3D, Downsample3D (after a space-to-depth rewrite) and
// CausalConvTranspose3d's convolution (:176-232).
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "conv3d.h"

namespace ddb {
namespace {

constexpr int BM = 128;  // rows of one MMA (one M sub-tile)
constexpr int BN = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int B_BYTES = BN * BK * 2;

// MT M sub-tiles (128 rows each) share every B tile: MT = 2 halves the shared-memory
// fill traffic per FLOP (48 KB per 2 x 128x128x64 MMAs instead of 32 KB per one), which
// is what keeps the tensor pipe fed from L2 at 128-wide N.
template <int MT>
struct ConvCfg {
  static constexpr int A_BYTES = MT * BM * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = MT == 2 ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * MT * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
};

struct ConvSched {
  int tiles_n, tiles_m, total;
  int tiles_w, tiles_h, To;
  int wbox, hbox;
  int kblocks;      // forward: taps * Cin/64; wgrad: position chunks
  int splits, kb_per_split;
  int cchunks;      // Cin / 64 (forward) or Cin / 128 (wgrad n tiles per tap)
  int kw, kh;
  // tile -> (m index, n index, k range)
  __device__ __forceinline__ void decode(int t, int& mi, int& ni, int& kb0, int& kb1) const {
    ni = t % tiles_n;
    t /= tiles_n;
    mi = t % tiles_m;
    const int split = t / tiles_m;
    kb0 = split * kb_per_split;
    kb1 = min(kblocks, kb0 + kb_per_split);
  }
  // position tile index -> (b, t, h0, w0)
  __device__ __forceinline__ void pos(int p, int& b, int& t, int& h0, int& w0) const {
    const int wt = p % tiles_w;
    p /= tiles_w;
    const int ht = p % tiles_h;
    p /= tiles_h;
    t = p % To;
    b = p / To;
    h0 = ht * hbox;
    w0 = wt * wbox;
  }
};

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

template <bool WG, int MT>
__global__ void __launch_bounds__(kThreads, 1)
    conv3d_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const Conv3dArgs args,
                     const ConvSched sched, int* status) {
  // forward: A = input patch (K-major), B = weights (K-major)
  // wgrad:   A = dy patch (MN-major over cout), B = input patch (MN-major over cin)
  using Cfg = ConvCfg<MT>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int STAGE_BYTES = Cfg::STAGE_BYTES;
  constexpr int TMEM_COLS = Cfg::TMEM_COLS;
  constexpr uint32_t IDESC = make_idesc_bf16(BM, BN, WG, WG);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < sched.total && ok; t += gridDim.x) {
        int mi, ni, kb0, kb1;
        sched.decode(t, mi, ni, kb0, kb1);
        int b = 0, to = 0, h0 = 0, w0 = 0, dt = 0, dh = 0, dw = 0, c0 = 0;
        if constexpr (!WG) {
          sched.pos(mi, b, to, h0, w0);
        } else {
          const int tap = ni / sched.cchunks;
          c0 = (ni % sched.cchunks) * 128;
          dw = tap % sched.kw;
          dh = (tap / sched.kw) % sched.kh;
          dt = tap / (sched.kw * sched.kh);
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          if constexpr (!WG) {
            const int tap = kb / sched.cchunks;
            const int cc = (kb % sched.cchunks) * BK;
            const int kx = tap % sched.kw;
            const int ky = (tap / sched.kw) % sched.kh;
            const int kz = tap / (sched.kw * sched.kh);
            tma_load_5d(sa, &tmA, &full[stage], cc, w0 + kx - args.pw, h0 + ky - args.ph,
                        to + kz - args.pt, b);
            tma_load_2d(sb, &tmB, &full[stage], kb * BK, ni * BN);
          } else {
            sched.pos(kb, b, to, h0, w0);
            const int m0 = mi * BM * MT;
#pragma unroll
            for (int c = 0; c < 2 * MT; ++c)
              tma_load_5d(sa + c * 8192, &tmA, &full[stage], m0 + 64 * c, w0, h0, to, b);
            tma_load_5d(sb, &tmB, &full[stage], c0, w0 + dw - args.pw, h0 + dh - args.ph,
                        to + dt - args.pt, b);
            tma_load_5d(sb + 8192, &tmB, &full[stage], c0 + 64, w0 + dw - args.pw,
                        h0 + dh - args.ph, to + dt - args.pt, b);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        record_status(status, kStatusTimeoutProducer);
        *abort_flag = 1;
        int s = stage, ph = phase;
        for (int i = 0; i < min(issued, STAGES); ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          long long t0 = clock64();
          while (!mbar_try_wait(&full[s], ph) && clock64() - t0 < kSpinLimitCycles / 8) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool any = false;
      for (int t = blockIdx.x; t < sched.total && ok; t += gridDim.x) {
        int mi, ni, kb0, kb1;
        sched.decode(t, mi, ni, kb0, kb1);
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * MT * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t db = WG ? make_sw128_desc(sb + kk * 2048, 8192, 1024)
                             : make_sw128_desc(sb + kk * 32, 16, 1024);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              // sub-tile mt: rows [128 mt, 128 mt + 128) of the A tile (16 KB apart)
              const uint32_t am = sa + mt * (BM * BK * 2);
              uint64_t da = WG ? make_sw128_desc(am + kk * 2048, 8192, 1024)
                               : make_sw128_desc(am + kk * 32, 16, 1024);
              mma_bf16_ss(d_tmem + mt * BN, da, db, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
            }
          }
          any = true;
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
        if (++buf == 2) {
          buf = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) {
        record_status(status, kStatusTimeoutMma);
        *abort_flag = 1;
      }
      if (any) {
        mma_commit(drain_bar);
        long long t0 = clock64();
        while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < kSpinLimitCycles / 8) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    int buf = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < sched.total; t += gridDim.x) {
      int mi, ni, kb0, kb1;
      sched.decode(t, mi, ni, kb0, kb1);
      if (!mbar_wait(&acc_full[buf], acc_phase, abort_flag)) {
        if (lane == 0) record_status(status, kStatusTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tlane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * MT * BN;
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const uint32_t tbase = tlane + mt * BN;
        const int rr_row = mt * BM + r;  // row within the MT*128-row tile
        if constexpr (!WG) {
          int b, to, h0, w0;
          sched.pos(mi, b, to, h0, w0);
          const int h = h0 + rr_row / sched.wbox;
          const int w = w0 + rr_row % sched.wbox;
          const bool row_ok = h < args.Ho && w < args.Wo;
          const long orow = ((static_cast<long>(b) * args.To + to) * args.Ho + h) * args.Wo + w;
          const int n0 = ni * BN;
          const bool vec_ok = (args.Cout & 7) == 0;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            uint32_t rr[32];
            tmem_ld32(tbase + c, rr);
            tmem_wait_ld();
            const int col0 = n0 + c;
            if (!row_ok || col0 >= args.Cout) continue;
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(rr[i]);
            const int ncol = min(32, args.Cout - col0);
            if (args.bias != nullptr)
              for (int i = 0; i < ncol; ++i) v[i] += __ldg(args.bias + col0 + i);
            __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(args.y) + orow * args.Cout + col0;
            const __nv_bfloat16* res =
                args.residual == nullptr
                    ? nullptr
                    : reinterpret_cast<const __nv_bfloat16*>(args.residual) + orow * args.Cout + col0;
            if (vec_ok && ncol == 32) {
              if (res != nullptr) {
#pragma unroll
                for (int i = 0; i < 32; i += 8) {
                  uint4 cv = ld_global_v4(res + i);
                  uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    float2 f = unpack_bf16(cw[j]);
                    v[i + 2 * j] += f.x;
                    v[i + 2 * j + 1] += f.y;
                  }
                }
              }
#pragma unroll
              for (int i = 0; i < 32; i += 8)
                st_global_v4(y + i, pack_bf16(v[i], v[i + 1]), pack_bf16(v[i + 2], v[i + 3]),
                             pack_bf16(v[i + 4], v[i + 5]), pack_bf16(v[i + 6], v[i + 7]));
            } else {
              for (int i = 0; i < ncol; ++i) {
                float o = v[i];
                if (res != nullptr) o += __bfloat162float(res[i]);
                y[i] = __float2bfloat16(o);
              }
            }
          }
        } else {
          // dw[cout = m0 + row, tap * Cin + c0 + col]
          const int tap = ni / sched.cchunks;
          const int c0 = (ni % sched.cchunks) * 128;
          const int row = mi * BM * MT + rr_row;
          const long K = static_cast<long>(sched.kw) * sched.kh * args.kt * args.Cin;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            uint32_t rr[32];
            tmem_ld32(tbase + c, rr);
            tmem_wait_ld();
            if (row >= args.Cout || c0 + c >= args.Cin) continue;
            float* d = args.dw + row * K + static_cast<long>(tap) * args.Cin + c0 + c;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              red_add_v4_f32(d + i, __uint_as_float(rr[i]), __uint_as_float(rr[i + 1]),
                             __uint_as_float(rr[i + 2]), __uint_as_float(rr[i + 3]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (++buf == 2) {
        buf = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// patch geometry: wbox * hbox = positions per tile (wbox a power of two, 8..256, hbox
// <= 256), chosen to minimise the padded output area ceil(Wo/wbox)*wbox *
// ceil(Ho/hbox)*hbox; ties go to the wider patch (longer contiguous TMA rows)
void patch_dims(int Wo, int Ho, int positions, int& wbox, int& hbox) {
  long best = -1;
  for (int wb = std::min(positions, 256); wb >= 8; wb /= 2) {
    const int hb = positions / wb;
    if (hb > 256) break;
    const long area = static_cast<long>((Wo + wb - 1) / wb) * wb * ((Ho + hb - 1) / hb) * hb;
    if (best < 0 || area < best) {
      best = area;
      wbox = wb;
      hbox = hb;
    }
  }
}

CUtensorMap act_map(const void* base, int B, int T, int H, int W, int C, int wbox, int hbox) {
  const uint64_t dims[5] = {static_cast<uint64_t>(C), static_cast<uint64_t>(W),
                            static_cast<uint64_t>(H), static_cast<uint64_t>(T),
                            static_cast<uint64_t>(B)};
  const uint64_t es = 2;
  const uint64_t strides[4] = {C * es, static_cast<uint64_t>(W) * C * es,
                               static_cast<uint64_t>(H) * W * C * es,
                               static_cast<uint64_t>(T) * H * W * C * es};
  const uint32_t box[5] = {64, static_cast<uint32_t>(wbox), static_cast<uint32_t>(hbox), 1, 1};
  return make_tmap_nd(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 5, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

template <bool WG, int MT>
void launch(const CUtensorMap& tA, const CUtensorMap& tB, const Conv3dArgs& a,
            const ConvSched& s, cudaStream_t stream) {
  static bool attr_set = false;
  constexpr int SMEM_BYTES = ConvCfg<MT>::SMEM_BYTES;
  auto kern = conv3d_tc_kernel<WG, MT>;
  if (!attr_set) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES),
               "cudaFuncSetAttribute(conv3d smem)");
    attr_set = true;
  }
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  int grid = num_sms(dev);
  if (a.max_ctas > 0) grid = std::min(grid, a.max_ctas);
  grid = std::max(1, std::min(grid, s.total));
  kern<<<grid, kThreads, SMEM_BYTES, stream>>>(tA, tB, a, s, device_status(dev));
  count_launch();
  check_cuda(cudaGetLastError(), "conv3d_tc_kernel launch");
}

void check_common(const Conv3dArgs& a) {
  if (a.Cin % 64 != 0) throw std::runtime_error("conv3d: Cin must be a multiple of 64");
  if (a.B <= 0 || a.T <= 0 || a.H <= 0 || a.W <= 0 || a.To <= 0 || a.Ho <= 0 || a.Wo <= 0 ||
      a.Cout <= 0 || a.kt <= 0 || a.kh <= 0 || a.kw <= 0)
    throw std::runtime_error("conv3d: empty or invalid extents");
}

}  // namespace

void conv3d_fwd(const Conv3dArgs& a, cudaStream_t stream) {
  check_common(a);
  if (a.x == nullptr || a.w == nullptr || a.y == nullptr)
    throw std::runtime_error("conv3d_fwd: null operand");
  ConvSched s{};
  constexpr int MT = 2;
  patch_dims(a.Wo, a.Ho, BM * MT, s.wbox, s.hbox);
  s.tiles_w = (a.Wo + s.wbox - 1) / s.wbox;
  s.tiles_h = (a.Ho + s.hbox - 1) / s.hbox;
  s.To = a.To;
  s.tiles_m = a.B * a.To * s.tiles_h * s.tiles_w;
  s.tiles_n = (a.Cout + BN - 1) / BN;
  s.cchunks = a.Cin / BK;
  s.kw = a.kw;
  s.kh = a.kh;
  s.kblocks = a.kt * a.kh * a.kw * s.cchunks;
  s.splits = 1;
  s.kb_per_split = s.kblocks;
  s.total = s.tiles_m * s.tiles_n;
  const CUtensorMap tA = act_map(a.x, a.B, a.T, a.H, a.W, a.Cin, s.wbox, s.hbox);
  const long K = static_cast<long>(a.kt) * a.kh * a.kw * a.Cin;
  const CUtensorMap tB = make_tmap_2d(a.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, a.Cout,
                                      K * 2, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  launch<false, MT>(tA, tB, a, s, stream);
}

void conv3d_wgrad(const Conv3dArgs& a, cudaStream_t stream) {
  check_common(a);
  if (a.x == nullptr || a.dy == nullptr || a.dw == nullptr)
    throw std::runtime_error("conv3d_wgrad: null operand");
  if (a.Cin % 128 != 0 || a.Cout % 64 != 0)
    throw std::runtime_error("conv3d_wgrad: needs Cin % 128 == 0 and Cout % 64 == 0");
  ConvSched s{};
  patch_dims(a.Wo, a.Ho, BK, s.wbox, s.hbox);
  const int MT = a.Cout >= 256 ? 2 : 1;
  s.tiles_w = (a.Wo + s.wbox - 1) / s.wbox;
  s.tiles_h = (a.Ho + s.hbox - 1) / s.hbox;
  s.To = a.To;
  s.tiles_m = (a.Cout + BM * MT - 1) / (BM * MT);
  s.cchunks = a.Cin / 128;
  s.tiles_n = a.kt * a.kh * a.kw * s.cchunks;
  s.kw = a.kw;
  s.kh = a.kh;
  s.kblocks = a.B * a.To * s.tiles_h * s.tiles_w;  // 64-position chunks
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const int sms = num_sms(dev);
  int splits = a.splits;
  if (splits <= 0) {
    // enough work items for ~2 waves, at least 8 K steps per item
    const int tiles = s.tiles_m * s.tiles_n;
    splits = std::max(1, std::min((2 * sms + tiles - 1) / tiles, s.kblocks / 8));
  }
  s.kb_per_split = (s.kblocks + splits - 1) / splits;
  s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;
  s.total = s.tiles_m * s.tiles_n * s.splits;
  const CUtensorMap tA = act_map(a.dy, a.B, a.To, a.Ho, a.Wo, a.Cout, s.wbox, s.hbox);
  const CUtensorMap tB = act_map(a.x, a.B, a.T, a.H, a.W, a.Cin, s.wbox, s.hbox);
  if (MT == 2)
    launch<true, 2>(tA, tB, a, s, stream);
  else
    launch<true, 1>(tA, tB, a, s, stream);
}

}  // namespace ddb
