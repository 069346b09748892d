// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M,N] = A[M,K] * B[N,K]^T, bf16 operands, fp32 accumulation in TMEM.
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: streams 128x64 A and BNx64 B tiles into a STAGES-deep
//               shared-memory ring (128-byte swizzle), one mbarrier pair per slot.
//   warp 1      owns TMEM (2 x BN fp32 columns, double-buffered accumulator) and issues
//               tcgen05.mma (M=128, N=BN, K=16) from one thread; tcgen05.commit frees
//               ring slots and hands finished accumulators to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, fused elementwise op; bf16
//               outputs go through a per-warp [32 rows x 64 cols] shared-memory box
//               (128-byte swizzle) and a TMA store, so every row segment leaves as full
//               lines instead of 32 scattered 16-byte stores per instruction; fp32
//               outputs use 16-byte stores or vector reductions (split-K).
// Tiles are walked persistently (n fastest, so concurrent CTAs share the A panel in L2);
// the epilogue of tile i overlaps the MMAs of tile i+1.
//
// CTA-pair mode (PAIR, clusters of 2 on two SMs, cta_group::2): a tile is 256 x BN; each
// CTA loads its own 128 rows of A and half (BN/2 rows) of B into its own shared memory
// with plain TMA loads that count on the even CTA's `full` barrier; the even CTA issues
// one M=256 MMA per K step, which reads A and B from both CTAs, and each CTA's TMEM
// receives its 128 rows of D. Per FLOP a CTA then stages and reads a third less
// operand data than in 128 x 256 single-CTA tiles (the B half instead of all of B).
// The even CTA's MMA commits free the ring slots and hand accumulators to the epilogue
// of both CTAs; the odd CTA's epilogue warps release the accumulator on the even CTA's
// barrier. No load is multicast. Before a CTA of a pair exits it waits for the last
// arrive its peer sends to each of its barriers. Pairs are opt-in (see gemm()).
//
// Replaces every nn.Linear of the reference (layers/mha.py:307-308, layers/mlp.py:112-114,
// layers/moe.py:54-56) and carries the SwiGLU (layers/mlp.py:131-155), rotary
// (layers/rope_v2.py:95-148) and residual epilogues.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "gemm.h"

namespace ddb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

// Epilogue staging per epilogue warp (bf16-output kernels only), each double-buffered:
//   D  box [32 rows x 64 cols] bf16, 128-byte swizzle       (TMA store)
//   D2 box [32 rows x 32 cols] bf16, unswizzled 64-byte rows (TMA store, SwiGLU activation)
//   C  box [32 rows x 64 cols] bf16, 128-byte swizzle       (TMA load of the residual / gu)
constexpr int kOutBoxD = 32 * 128;
constexpr int kOutBoxD2 = 32 * 64;
constexpr int kOffD2 = 4 * 2 * kOutBoxD;
constexpr int kOffC = kOffD2 + 4 * 2 * kOutBoxD2;
constexpr int kOutStage = kOffC + 4 * 2 * kOutBoxD;

// Shared-memory layouts: fp32 outputs (no boxes), bf16 outputs (D boxes only), and
// bf16 outputs with a second output or a C operand (all boxes, one operand stage fewer).
enum GemmLayout : int { kLayF32 = 0, kLayOut = 1, kLayOutC = 2 };

template <int BN, int LAY, bool PAIR = false>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;  // a pair CTA holds half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OUT_BYTES = LAY == kLayOutC ? kOutStage : (LAY == kLayOut ? kOffD2 : 0);
  static constexpr int PAIR_STAGES = (232448 - 1280 - OUT_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = PAIR ? (PAIR_STAGES > 8 ? 8 : PAIR_STAGES)
                                     : (LAY == kLayOutC ? ((BN == 256) ? 3 : 4) : ((BN == 256) ? 4 : 6));
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int OFF_OUT = STAGES * STAGE_BYTES;   // epilogue boxes
  static constexpr int OFF_BAR = OFF_OUT + OUT_BYTES;    // mbarriers, TMEM slot, abort flag
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// TMA maps of the bf16 epilogue: D {cols, rows, batch} with [64 x 32] boxes, D2 with
// [32 x 32] boxes, C (residual / gu) with [64 x 32] boxes. use == 0: plain global stores;
// use_c == 0: C read with plain loads.
struct OutMaps {
  CUtensorMap d;
  CUtensorMap d2;
  CUtensorMap c;
  int use;
  int use_c;
};

// Per-warp output staging; rows are the warp's 32 TMEM lanes (row `lane` of each box).
// Box k of the warp uses buffer k & 1.
struct OutStage {
  uint32_t base_d, base_d2, base_c;  // shared addresses of this warp's buffer 0
  uint64_t* cbar;                    // 2 mbarriers: C box loaded
  int k = 0;                         // output boxes flushed so far
  int kc = 0;                        // C boxes requested so far
  __device__ __forceinline__ uint32_t box_d() const { return base_d + (k & 1) * kOutBoxD; }
  __device__ __forceinline__ uint32_t box_d2() const { return base_d2 + (k & 1) * kOutBoxD2; }
  // wait until the store that last used this buffer (two boxes ago) has read it
  __device__ __forceinline__ void acquire(int lane) const {
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    __syncwarp();
  }
  // 32 bf16 columns (16 packed pairs) into half `h` of the 64-column D box
  __device__ __forceinline__ void put_d(int lane, int h, const uint32_t (&p)[16]) const {
    const uint32_t b = box_d() + lane * 128;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      st_shared_v4(b + (((h * 4 + i) ^ (lane & 7)) << 4), p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
  }
  __device__ __forceinline__ void put_d2(int lane, const uint32_t (&p)[16]) const {
    const uint32_t b = box_d2() + lane * 64;
#pragma unroll
    for (int i = 0; i < 4; ++i) st_shared_v4(b + i * 16, p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
  }
  // hand the filled D box (and the D2 box when `d2`) to TMA as one bulk group; rows /
  // columns past the tensor's extent are clipped by the copy
  __device__ __forceinline__ void flush(int lane, const OutMaps& om, int col, int row0, int bt, bool d2,
                                        int col2) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(&om.d, box_d(), col, row0, bt);
      if (d2) tma_store_3d(&om.d2, box_d2(), col2, row0, bt);
      tma_store_commit();
    }
    ++k;
  }
  // request C box kc (columns col.., rows row0.., batch bt) into buffer kc & 1; the buffer's
  // previous box was consumed by this warp before (program order + __syncwarp)
  __device__ __forceinline__ void load_c(int lane, const OutMaps& om, int col, int row0, int bt) {
    fence_proxy_async_smem();  // this warp's reads of the buffer precede the TMA write
    __syncwarp();
    if (lane == 0) {
      uint64_t* bar = &cbar[kc & 1];
      mbar_arrive_expect_tx(bar, kOutBoxD);
      tma_load_3d_s(base_c + (kc & 1) * kOutBoxD, &om.c, bar, col, row0, bt);
    }
    ++kc;
  }
  // wait for C box `idx` (bounded) and return its shared address
  __device__ __forceinline__ bool wait_c(int idx, volatile int* abort_flag, uint32_t& addr) const {
    addr = base_c + (idx & 1) * kOutBoxD;
    return mbar_wait(&cbar[idx & 1], (idx >> 1) & 1, abort_flag);
  }
};

// 8 bf16 of row `lane`, 16-byte chunk `chunk` of a 128-byte-swizzled [32 x 64] box
__device__ __forceinline__ uint4 box_chunk(uint32_t box, int lane, int chunk) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(box + lane * 128 + ((chunk ^ (lane & 7)) << 4)));
  return v;
}

struct Sched {
  int tiles_m, tiles_n, kblocks, kb_per_split, splits, total, M;
  int bm;  // rows per tile: 128, or 256 for CTA pairs
  int grouped;
  const int* g_tile_expert;
  const int* g_tile_row;
  const int* g_total_mtiles;
  const int* g_kstart;
  const int* g_kend;
  // tile t -> (batch bt, row m0, column tile n0, k-block range); n fastest.
  // Returns false for tiles that carry no work (grouped tables).
  __device__ __forceinline__ bool decode(int t, int& m0, int& n0, int& kb0, int& kb1,
                                         int& bt) const {
    int n_idx = t % tiles_n;
    t /= tiles_n;
    n0 = n_idx;  // scaled by BN by the caller
    if (grouped == 1) {
      if (t >= __ldg(g_total_mtiles)) return false;
      bt = __ldg(g_tile_expert + t);
      m0 = __ldg(g_tile_row + t);
      kb0 = 0;
      kb1 = kblocks;
      return true;
    }
    int m_idx = t % tiles_m;
    t /= tiles_m;
    int split = t % splits;
    bt = t / splits;
    m0 = m_idx * bm;
    if (grouped == 2) {
      kb0 = __ldg(g_kstart + bt);
      kb1 = __ldg(g_kend + bt);
      return kb1 > kb0;
    }
    kb0 = split * kb_per_split;
    kb1 = min(kblocks, kb0 + kb_per_split);
    return true;
  }
};

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

// ---------------------------------------------------------------- fused weight all-gather
constexpr long kGatherPieceElems = 8192;  // 16 KB of bf16 per gather work item
constexpr int kGatherRows = 128;          // rows of B per readiness counter

__device__ __forceinline__ int gather_pieces(const GemmArgs& a, int g) {
  const long rows = min(kGatherRows, a.N - g * kGatherRows);
  return static_cast<int>((rows * a.K + kGatherPieceElems - 1) / kGatherPieceElems);
}

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epilogue warps (128 threads, named barrier 1): copy the peer-owned pieces of this CTA's
// gather items into the local copy of B, then count each finished item on its row group.
__device__ void gather_weight_pieces(const GemmArgs& a, int tid) {
  const int groups = (a.N + kGatherRows - 1) / kGatherRows;
  const int ppg = static_cast<int>((static_cast<long>(kGatherRows) * a.K + kGatherPieceElems - 1) /
                                   kGatherPieceElems);
  const long total = static_cast<long>(groups) * ppg;
  const long n_elems = static_cast<long>(a.N) * a.K;
  uint4* local = reinterpret_cast<uint4*>(const_cast<void*>(a.B));
  for (long item = blockIdx.x; item < total; item += gridDim.x) {
    const int g = static_cast<int>(item / ppg);
    const int q = static_cast<int>(item % ppg);
    // the last row group may hold fewer pieces; the same for all 128 threads, so the
    // named barrier below stays uniform, and only real pieces are counted
    if (q >= gather_pieces(a, g)) continue;
    const long group_end = min(n_elems, static_cast<long>(g + 1) * kGatherRows * a.K);
    long e = static_cast<long>(g) * kGatherRows * a.K + q * kGatherPieceElems;
    const long e_end = min(group_end, e + kGatherPieceElems);
    while (e < e_end) {  // split the piece at shard (owner) boundaries
      const long flat = a.gb_elem0 + e;
      const int owner = static_cast<int>(flat / a.gb_shard);
      const long seg_end = min(e_end, (owner + 1) * a.gb_shard - a.gb_elem0);
      if (owner != a.gb_rank) {
        const uint4* src = reinterpret_cast<const uint4*>(a.gb_peers[owner]);
        for (long v = e / 8 + tid; v < seg_end / 8; v += 128) local[v] = src[v];
      }
      e = seg_end;
    }
    __threadfence();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (tid == 0) {
      fence_proxy_async_global();
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.gb_counters + g) : "memory");
    }
  }
}

// ---------------------------------------------------------------- epilogue ops
template <int EPI>
__device__ __forceinline__ void epi_chunk32(const GemmArgs& a, int row, int col0,
                                            const uint32_t (&r)[32], const OutStage* st = nullptr,
                                            int lane = 0, int h = 0, uint32_t cbox = 0) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);

  if constexpr (EPI == kEpiF32Atomic) {
    float* d = reinterpret_cast<float*>(a.D) + static_cast<long>(row) * a.ldd + col0;
#pragma unroll
    for (int i = 0; i < 32; i += 4) red_add_v4_f32(d + i, v[i], v[i + 1], v[i + 2], v[i + 3]);
    return;
  } else {
    if (a.bias != nullptr) {
      const float4* b4 = reinterpret_cast<const float4*>(a.bias + col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 b = __ldg(b4 + i);
        v[4 * i] += b.x;
        v[4 * i + 1] += b.y;
        v[4 * i + 2] += b.z;
        v[4 * i + 3] += b.w;
      }
    }
    if constexpr (EPI == kEpiF32) {
      float* d = reinterpret_cast<float*>(a.D) + static_cast<long>(row) * a.ldd + col0;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        st_global_v4(d + i, __float_as_uint(v[i]), __float_as_uint(v[i + 1]),
                     __float_as_uint(v[i + 2]), __float_as_uint(v[i + 3]));
      return;
    } else {
      if constexpr (EPI == kEpiRope) {
        if (col0 < a.rope_cols) {
          const int pos = (row % a.rope_rows_per_seq) + a.rope_pos_offset;
          const int half = a.rope_head_dim >> 1;
          const int p0 = (col0 % a.rope_head_dim) >> 1;
          const float2* tab = a.rope_tab + static_cast<long>(pos) * half + p0;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float2 cs = __ldg(tab + i);
            float x0 = v[2 * i], x1 = v[2 * i + 1];
            v[2 * i] = x0 * cs.x - x1 * cs.y;
            v[2 * i + 1] = x0 * cs.y + x1 * cs.x;
          }
        }
      }
      if constexpr (EPI == kEpiGateResidual) {
        const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(a.gate) +
                                 static_cast<long>(row / a.gate_rows_per_group) * a.ldg + col0;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 gv = ld_global_v4(g + i);
          uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 f = unpack_bf16(gw[j]);
            v[i + 2 * j] *= f.x;
            v[i + 2 * j + 1] *= f.y;
          }
        }
      }
      if constexpr (EPI == kEpiGelu) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.5f * v[i] * (1.f + erff(v[i] * 0.70710678118654752f));
      }
      if (a.C != nullptr && (EPI == kEpiBf16 || EPI == kEpiGateResidual)) {
        const __nv_bfloat16* c =
            reinterpret_cast<const __nv_bfloat16*>(a.C) + static_cast<long>(row) * a.ldc + col0;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          // C from the TMA-loaded box (columns h*32.. of it) or straight from global memory
          uint4 cv = cbox ? box_chunk(cbox, lane, h * 4 + i / 8) : ld_global_v4(c + i);
          uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 f = unpack_bf16(cw[j]);
            v[i + 2 * j] += f.x;
            v[i + 2 * j + 1] += f.y;
          }
        }
      }
      if (st != nullptr) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
        st->put_d(lane, h, pk);
        return;
      }
      __nv_bfloat16* d;
      if (EPI == kEpiBf16 && a.d_peers != nullptr) {  // reduce-scatter: P2P store to the row's owner
        const int owner = row / a.d_rows_per_peer;
        const long lrow = static_cast<long>(a.d_slot) * a.d_rows_per_peer + row % a.d_rows_per_peer;
        d = reinterpret_cast<__nv_bfloat16*>(a.d_peers[owner]) + lrow * a.ldd + col0;
      } else {
        d = reinterpret_cast<__nv_bfloat16*>(a.D) + static_cast<long>(row) * a.ldd + col0;
      }
#pragma unroll
      for (int i = 0; i < 32; i += 8)
        st_global_v4(d + i, pack_bf16(v[i], v[i + 1]), pack_bf16(v[i + 2], v[i + 3]),
                     pack_bf16(v[i + 4], v[i + 5]), pack_bf16(v[i + 6], v[i + 7]));
    }
  }
}

// SwiGLU forward: accumulator columns come in groups of 64: 32 gate then 32 up.
__device__ __forceinline__ void epi_swiglu(const GemmArgs& a, int row, int col0,
                                           const uint32_t (&rg)[32], const uint32_t (&ru)[32],
                                           const OutStage* st = nullptr, int lane = 0) {
  __nv_bfloat16* gu =
      reinterpret_cast<__nv_bfloat16*>(a.D) + static_cast<long>(row) * a.ldd + col0;
  __nv_bfloat16* act =
      reinterpret_cast<__nv_bfloat16*>(a.D2) + static_cast<long>(row) * a.ldd2 + (col0 >> 1);
  float g[32], u[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    // round through bf16 so the saved pre-activation and the activation agree exactly
    g[i] = __bfloat162float(__float2bfloat16(__uint_as_float(rg[i])));
    u[i] = __bfloat162float(__float2bfloat16(__uint_as_float(ru[i])));
  }
  if (st != nullptr) {
    uint32_t pg[16], pu[16], ph[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      pg[i] = pack_bf16(g[2 * i], g[2 * i + 1]);
      pu[i] = pack_bf16(u[2 * i], u[2 * i + 1]);
      ph[i] = pack_bf16(silu_f(g[2 * i]) * u[2 * i], silu_f(g[2 * i + 1]) * u[2 * i + 1]);
    }
    st->put_d(lane, 0, pg);
    st->put_d(lane, 1, pu);
    st->put_d2(lane, ph);
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    st_global_v4(gu + i, pack_bf16(g[i], g[i + 1]), pack_bf16(g[i + 2], g[i + 3]),
                 pack_bf16(g[i + 4], g[i + 5]), pack_bf16(g[i + 6], g[i + 7]));
    st_global_v4(gu + 32 + i, pack_bf16(u[i], u[i + 1]), pack_bf16(u[i + 2], u[i + 3]),
                 pack_bf16(u[i + 4], u[i + 5]), pack_bf16(u[i + 6], u[i + 7]));
  }
  float h[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) h[i] = silu_f(g[i]) * u[i];
#pragma unroll
  for (int i = 0; i < 32; i += 8)
    st_global_v4(act + i, pack_bf16(h[i], h[i + 1]), pack_bf16(h[i + 2], h[i + 3]),
                 pack_bf16(h[i + 4], h[i + 5]), pack_bf16(h[i + 6], h[i + 7]));
}

// SwiGLU backward: acc = dA for activation columns [col0, col0+32), which map to the
// gate columns 2*col0 + [0,32) and up columns 2*col0 + 32 + [0,32) of gu.
__device__ __forceinline__ void epi_dswiglu(const GemmArgs& a, int row, int col0,
                                            const uint32_t (&r)[32], const OutStage* st = nullptr,
                                            int lane = 0, uint32_t cbox = 0) {
  const __nv_bfloat16* gu = reinterpret_cast<const __nv_bfloat16*>(a.C) +
                            static_cast<long>(row) * a.ldc + 2 * col0;
  __nv_bfloat16* dgu =
      reinterpret_cast<__nv_bfloat16*>(a.D) + static_cast<long>(row) * a.ldd + 2 * col0;
  float g[32], u[32];
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    // gate columns are chunks 0-3 of the C box, up columns chunks 4-7
    uint4 gv = cbox ? box_chunk(cbox, lane, i / 8) : ld_global_v4(gu + i);
    uint4 uv = cbox ? box_chunk(cbox, lane, 4 + i / 8) : ld_global_v4(gu + 32 + i);
    uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 fg = unpack_bf16(gw[j]);
      float2 fu = unpack_bf16(uw[j]);
      g[i + 2 * j] = fg.x;
      g[i + 2 * j + 1] = fg.y;
      u[i + 2 * j] = fu.x;
      u[i + 2 * j + 1] = fu.y;
    }
  }
  float dg[32], du[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float da = __uint_as_float(r[i]);
    float s = 1.f / (1.f + __expf(-g[i]));
    float sl = g[i] * s;
    du[i] = da * sl;
    dg[i] = da * u[i] * s * (1.f + g[i] * (1.f - s));
  }
  if (st != nullptr) {
    uint32_t pg[16], pu[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      pg[i] = pack_bf16(dg[2 * i], dg[2 * i + 1]);
      pu[i] = pack_bf16(du[2 * i], du[2 * i + 1]);
    }
    st->put_d(lane, 0, pg);
    st->put_d(lane, 1, pu);
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    st_global_v4(dgu + i, pack_bf16(dg[i], dg[i + 1]), pack_bf16(dg[i + 2], dg[i + 3]),
                 pack_bf16(dg[i + 4], dg[i + 5]), pack_bf16(dg[i + 6], dg[i + 7]));
    st_global_v4(dgu + 32 + i, pack_bf16(du[i], du[i + 1]), pack_bf16(du[i + 2], du[i + 3]),
                 pack_bf16(du[i + 4], du[i + 5]), pack_bf16(du[i + 6], du[i + 7]));
  }
}

// Per-peer A maps of the all-gather-fused form (unused entries are never read).
struct PeerMaps {
  CUtensorMap m[kMaxGemmPeers];
};

// ---------------------------------------------------------------- kernel
template <int BN, bool A_MN, bool B_MN, int EPI, int LAY, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const GemmArgs args,
                   const Sched sched, int* status, const __grid_constant__ PeerMaps pmA,
                   const __grid_constant__ OutMaps om) {
  constexpr bool kBf16Out = LAY != kLayF32;
  using Cfg = GemmCfg<BN, LAY, PAIR>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = make_idesc_bf16(PAIR ? 2 * BM : BM, BN, A_MN, B_MN);
  // CTA pairs: rank in the pair, tiles walked per cluster, this CTA's rows of a tile
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const int t_begin = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int t_step = PAIR ? static_cast<int>(nclusters_x()) : static_cast<int>(gridDim.x);
  const int m_off = static_cast<int>(crank) * BM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint64_t* cin_bar = drain_bar + 1;  // 4 epilogue warps x 2 C buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cin_bar + 8);
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
      mbar_init(&acc_empty[b], PAIR ? 8 : 4);  // pairs: both CTAs' epilogue warps
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&cin_bar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int p = 0; p < args.a_npeers; ++p) tma_prefetch_desc(&pmA.m[p]);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // pairs: both CTAs' barriers are initialised before either CTA signals the other's
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      uint64_t ready = 0;  // row groups (< 64) whose gathered B this CTA has acquired
      for (int t = t_begin; t < sched.total && ok; t += t_step) {
        int m0, nt, kb0, kb1, bt;
        if (!sched.decode(t, m0, nt, kb0, kb1, bt)) continue;
        const int n0 = nt * BN;
        if (args.gb_world > 1) {  // this tile's B rows must have landed locally
          const int g_end = min((n0 + BN + kGatherRows - 1) / kGatherRows,
                                (args.N + kGatherRows - 1) / kGatherRows);
          for (int g = n0 / kGatherRows; g < g_end && ok; ++g) {
            if (g < 64 && ((ready >> g) & 1)) continue;
            const unsigned target = args.gb_epoch * static_cast<unsigned>(gather_pieces(args, g));
            const long long t0 = clock64();
            while (static_cast<int>(ld_acquire_gpu_u32(args.gb_counters + g) - target) < 0) {
              if (*abort_flag || clock64() - t0 > kSpinLimitCycles) {
                ok = false;
                break;
              }
              __nanosleep(64);
            }
            if (g < 64) ready |= 1ull << g;
          }
          fence_proxy_async_global();  // generic-proxy stores of the gather -> TMA reads
          if (!ok) break;
        }
        const int ab = sched.grouped ? 0 : bt;        // A batch coordinate
        const int bb = sched.grouped == 2 ? 0 : bt;   // B batch coordinate
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          if constexpr (PAIR) {
            // both CTAs' bytes count on the even CTA's barrier (its MMA reads both)
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
            const int ma = m0 + m_off;
            const int nb0 = n0 + static_cast<int>(crank) * (BN / 2);
            if constexpr (A_MN) {
              tma_load_3d_pair(sa, &tmA, fb, ma, kb * BK, ab);
              tma_load_3d_pair(sa + 8192, &tmA, fb, ma + 64, kb * BK, ab);
            } else {
              tma_load_3d_pair(sa, &tmA, fb, kb * BK, ma, ab);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int c = 0; c < BN / 128; ++c)
                tma_load_3d_pair(sb + c * 8192, &tmB, fb, nb0 + c * 64, kb * BK, bb);
            } else {
              tma_load_3d_pair(sb, &tmB, fb, kb * BK, nb0, bb);
            }
            ++issued;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          if constexpr (A_MN) {
            tma_load_3d(sa, &tmA, &full[stage], m0, kb * BK, ab);
            tma_load_3d(sa + 8192, &tmA, &full[stage], m0 + 64, kb * BK, ab);
          } else if (args.a_npeers > 0) {  // all-gather fused: rows of peer m0 / rows_per_peer
            tma_load_3d(sa, &pmA.m[m0 / args.a_rows_per_peer], &full[stage], kb * BK,
                        m0 % args.a_rows_per_peer, 0);
          } else {
            tma_load_3d(sa, &tmA, &full[stage], kb * BK, m0, ab);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(sb + c * 8192, &tmB, &full[stage], n0 + c * 64, kb * BK, bb);
          } else {
            tma_load_3d(sb, &tmB, &full[stage], kb * BK, n0, bb);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if constexpr (PAIR) {
        // the even CTA's MMA commits release this CTA's stages through the cluster; wait
        // for the last release of every stage used, so that no arrive from the peer can
        // land in this CTA's shared memory after it exits (where the next kernel's CTA
        // may already own it)
        if (ok) {
          int s = stage, ph = phase;
          for (int i = 0; i < min(issued, STAGES); ++i) {
            if (--s < 0) {
              s = STAGES - 1;
              ph ^= 1;
            }
            long long t0 = clock64();
            while (!mbar_try_wait(&empty[s], ph) && clock64() - t0 < kSpinLimitCycles / 8) {
            }
          }
        }
      }
      if (!ok) {
        record_status(status, kStatusTimeoutProducer);
        *abort_flag = 1;
        // let copies already in flight land before the CTA exits (bounded); a pair's
        // copies all count on the even CTA's barriers
        int s = stage, ph = phase;
        for (int i = 0; i < ((PAIR && crank != 0) ? 0 : min(issued, STAGES)); ++i) {
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
    // (pairs: the even CTA issues for both; the odd CTA's MMA warp only owns its TMEM)
    if (lane == 0 && crank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool any = false;
      int tiles = 0;
      // signal an mbarrier of this CTA (and, for pairs, the same one of the odd CTA)
      auto commit_both = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          mma_commit_pair(smem_u32(bar));
          mma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          mma_commit(bar);
        }
      };
      for (int t = t_begin; t < sched.total && ok; t += t_step) {
        int m0, nt, kb0, kb1, bt;
        if (!sched.decode(t, m0, nt, kb0, kb1, bt)) continue;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t da = A_MN ? make_sw128_desc(sa + kk * 2048, 8192, 1024)
                               : make_sw128_desc(sa + kk * 32, 16, 1024);
            uint64_t db = B_MN ? make_sw128_desc(sb + kk * 2048, 8192, 1024)
                               : make_sw128_desc(sb + kk * 32, 16, 1024);
            if constexpr (PAIR)
              mma_bf16_ss_pair(d_tmem, da, db, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
            else
              mma_bf16_ss(d_tmem, da, db, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          any = true;
          commit_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        commit_both(&acc_full[buf]);
        ++tiles;
        if (++buf == 2) {
          buf = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) {
        record_status(status, kStatusTimeoutMma);
        *abort_flag = 1;
      } else if (PAIR) {
        // the odd CTA's epilogue releases the accumulators with remote arrives: take the
        // last release of each buffer used before this CTA can exit
        int b = buf, ph = acc_phase;
        for (int i = 0; i < min(tiles, 2); ++i) {
          if (--b < 0) {
            b = 1;
            ph ^= 1;
          }
          long long t0 = clock64();
          while (!mbar_try_wait(&acc_empty[b], ph) && clock64() - t0 < kSpinLimitCycles / 8) {
          }
        }
      }
      if (any) {
        // all MMAs of this thread complete before TMEM is released
        if constexpr (PAIR)
          mma_commit_pair(smem_u32(drain_bar));
        else
          mma_commit(drain_bar);
        long long t0 = clock64();
        while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < kSpinLimitCycles / 8) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    const bool tma_out = kBf16Out && om.use != 0;
    const bool tma_c = LAY == kLayOutC && tma_out && om.use_c != 0;
    const int ew = warp - 2;
    OutStage ost;
    ost.base_d = smem_u32(smem + Cfg::OFF_OUT + ew * 2 * kOutBoxD);
    ost.base_d2 = smem_u32(smem + Cfg::OFF_OUT + kOffD2 + ew * 2 * kOutBoxD2);
    ost.base_c = smem_u32(smem + Cfg::OFF_OUT + kOffC + ew * 2 * kOutBoxD);
    ost.cbar = cin_bar + 2 * ew;
    int c_done = 0;  // C boxes consumed
    int buf = 0;
    uint32_t acc_phase = 0;
    // Epilogues that read a bf16 operand C (residual, or gu for dSwiGLU) pull this thread's
    // C row segment of a tile into L2 one tile ahead, while the MMAs of that tile run, so
    // the row-per-thread reads of C hit L2 instead of waiting on DRAM.
    auto prefetch_c = [&](int tp) {
      if constexpr (EPI == kEpiDSwiGLU || EPI == kEpiBf16 || EPI == kEpiGateResidual) {
        if (args.C == nullptr || tp >= sched.total) return;
        int pm0, pnt, pk0, pk1, pbt;
        if (!sched.decode(tp, pm0, pnt, pk0, pk1, pbt)) return;
        pm0 += m_off;
        if (pm0 + row_in_tile >= args.M) return;
        const long prow = (sched.grouped == 1 ? 0 : static_cast<long>(pbt) * args.M) + pm0 + row_in_tile;
        const int c0 = (EPI == kEpiDSwiGLU ? 2 : 1) * pnt * BN;
        const int ncols = min((EPI == kEpiDSwiGLU ? 2 : 1) * BN,
                              (EPI == kEpiDSwiGLU ? 2 * args.N : args.N) - c0);
        const char* base = reinterpret_cast<const char*>(args.C) + (prow * args.ldc + c0) * 2;
        for (int off = 0; off < ncols * 2; off += 128)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
      }
    };
    if (args.gb_world > 1) gather_weight_pieces(args, threadIdx.x - 64);
    prefetch_c(t_begin);
    for (int t = t_begin; t < sched.total; t += t_step) {
      int m0, nt, kb0, kb1, bt;
      if (!sched.decode(t, m0, nt, kb0, kb1, bt)) continue;
      m0 += m_off;  // this CTA's rows of a pair tile
      const int n0 = nt * BN;
      prefetch_c(t + t_step);
      // TMA loads of this tile's C boxes (two in flight), issued before the accumulator
      // is ready: DSwiGLU reads one 64-column gu box per 32 accumulator columns, the
      // residual epilogues one box per 64 columns
      const int box_row_c = m0 + quad * 32;
      const int box_bt_c = sched.grouped == 1 ? 0 : bt;
      constexpr int kCStep = EPI == kEpiDSwiGLU ? 32 : 64;  // accumulator columns per C box
      const int n_cbox = tma_c ? (min(BN, args.N - n0) + kCStep - 1) / kCStep : 0;
      const int c_first = ost.kc;
      auto c_col = [&](int i) { return (EPI == kEpiDSwiGLU ? 2 : 1) * (n0 + i * kCStep); };
      for (int i = 0; i < min(2, n_cbox); ++i) ost.load_c(lane, om, c_col(i), box_row_c, box_bt_c);
      bool c_ok = true;
      // wait for C box i of this tile; request box i + 2 once box i has been read
      auto c_box = [&](int i, uint32_t& addr) {
        if (!ost.wait_c(c_first + i, abort_flag, addr)) {
          if (lane == 0) record_status(status, kStatusTimeoutEpilogue);
          *abort_flag = 1;
          c_ok = false;
        }
      };
      auto c_release = [&](int i) {
        ++c_done;
        if (i + 2 < n_cbox) ost.load_c(lane, om, c_col(i + 2), box_row_c, box_bt_c);
      };
      if (!mbar_wait(&acc_full[buf], acc_phase, abort_flag)) {
        if (lane == 0) record_status(status, kStatusTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      // batches are stacked row-wise in D (and C): global row = bt * M + row; grouped
      // row tiles address the permuted buffer directly
      const bool row_ok = m0 + row_in_tile < args.M;
      const int row = (sched.grouped == 1 ? 0 : bt * args.M) + m0 + row_in_tile;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN;
      // TMA box coordinates: rows within the batch, batch index (grouped: one buffer)
      const int box_row = m0 + quad * 32;
      const int box_bt = sched.grouped == 1 ? 0 : bt;
      if constexpr (EPI == kEpiSwiGLU) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          uint32_t rg[32], ru[32];
          tmem_ld32(tbase + c, rg);
          tmem_ld32(tbase + c + 32, ru);
          tmem_wait_ld();
          if (n0 + c >= args.N) continue;
          if (tma_out) {
            ost.acquire(lane);  // rows past M: nothing read, the store clips them
            if (row_ok) epi_swiglu(args, row, n0 + c, rg, ru, &ost, lane);
            ost.flush(lane, om, n0 + c, box_row, box_bt, true, (n0 + c) >> 1);
          } else if (row_ok) {
            epi_swiglu(args, row, n0 + c, rg, ru);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
          tmem_wait_ld();
          if (n0 + c >= args.N) continue;
          if constexpr (EPI == kEpiDSwiGLU) {
            if (tma_out) {  // 32 activation-gradient columns -> one 64-column box of dgu
              uint32_t cb = 0;
              if (tma_c) c_box(c >> 5, cb);
              if (!c_ok) break;
              ost.acquire(lane);
              if (row_ok) epi_dswiglu(args, row, n0 + c, r, &ost, lane, cb);
              if (tma_c) {
                __syncwarp();
                c_release(c >> 5);
              }
              ost.flush(lane, om, 2 * (n0 + c), box_row, box_bt, false, 0);
            } else if (row_ok) {
              epi_dswiglu(args, row, n0 + c, r);
            }
          } else if (tma_out) {  // two 32-column chunks fill one 64-column box
            const int h = (c >> 5) & 1;
            uint32_t cb = 0;
            if (tma_c) {
              c_box(c >> 6, cb);
              if (!c_ok) break;
            }
            if (h == 0) ost.acquire(lane);
            if (row_ok) epi_chunk32<EPI>(args, row, n0 + c, r, &ost, lane, h, cb);
            const bool last = h == 1 || n0 + c + 32 >= args.N;
            if (tma_c && last) {
              __syncwarp();
              c_release(c >> 6);
            }
            if (last) ost.flush(lane, om, n0 + c - 32 * h, box_row, box_bt, false, 0);
          } else if (row_ok) {
            epi_chunk32<EPI>(args, row, n0 + c, r);
          }
        }
      }
      if (!c_ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && crank != 0)
          mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[buf]), 0));
        else
          mbar_arrive(&acc_empty[buf]);
      }
      if (++buf == 2) {
        buf = 0;
        acc_phase ^= 1;
      }
    }
    if (tma_out && lane == 0) tma_store_wait_all();  // boxes read and stores complete
    // C boxes requested but not consumed (an aborted tile) land before the CTA exits
    for (int i = c_done; i < ost.kc; ++i) {
      long long t0 = clock64();
      while (!mbar_try_wait(&ost.cbar[i & 1], (i >> 1) & 1) && clock64() - t0 < kSpinLimitCycles / 8) {
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // pairs: the even CTA's MMAs (which write the odd CTA's TMEM and read its shared
  // memory) are drained before either CTA releases TMEM or exits
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host launch
template <int BN, bool A_MN, bool B_MN, int EPI, int LAY, bool PAIR>
void launch_lay(const GemmArgs& a, const Sched& s, int grid, cudaStream_t stream, int* status) {
  using Cfg = GemmCfg<BN, LAY, PAIR>;
  static bool attr_set = false;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, EPI, LAY, PAIR>;
  if (!attr_set) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::SMEM_BYTES),
               "cudaFuncSetAttribute(gemm smem)");
    attr_set = true;
  }
  CUtensorMap tA, tB;
  // batch extents of the operand maps (grouped: A is one permuted buffer; in the
  // weight-gradient form neither operand is batched, only D is)
  const int nba = a.grouped ? 1 : a.batch;
  const int nbb = a.grouped == 2 ? 1 : a.batch;
  const long sa = nba > 1 ? a.stride_a : (A_MN ? a.lda * a.K : a.lda * a.M);
  const long sb = nbb > 1 ? a.stride_b : (B_MN ? a.ldb * a.K : a.ldb * a.N);
  if (A_MN)
    tA = make_tmap_3d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, nba, a.lda * 2,
                      sa * 2, 64, 64, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    tA = make_tmap_3d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.M, nba, a.lda * 2,
                      sa * 2, 64, BM, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  if (B_MN)
    tB = make_tmap_3d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, nbb, a.ldb * 2,
                      sb * 2, 64, 64, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    tB = make_tmap_3d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.N, nbb, a.ldb * 2,
                      sb * 2, 64, PAIR ? BN / 2 : BN, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  PeerMaps pm;
  std::memset(&pm, 0, sizeof(pm));
  if (a.a_npeers > 0) {
    if (A_MN || a.batch > 1 || a.grouped) throw std::runtime_error("gemm: peer A needs K-major, unbatched A");
    if (a.a_npeers > kMaxGemmPeers || a.a_rows_per_peer % BM != 0 ||
        static_cast<long>(a.a_rows_per_peer) * a.a_npeers != a.M)
      throw std::runtime_error("gemm: peer A rows must be a multiple of 128 per peer and cover M");
    for (int p = 0; p < a.a_npeers; ++p)
      pm.m[p] = make_tmap_3d(a.a_peer_ptrs[p], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.a_rows_per_peer, 1,
                             a.lda * 2, a.lda * 2 * a.a_rows_per_peer, 64, BM, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (a.d_peers != nullptr && (EPI != kEpiBf16 || a.C != nullptr || a.bias != nullptr || a.d_rows_per_peer <= 0))
    throw std::runtime_error("gemm: the reduce-scatter store needs the plain bf16 epilogue");
  OutMaps om;
  std::memset(&om, 0, sizeof(om));
  constexpr bool kBf16Out = LAY != kLayF32;
  auto aligned = [](const void* p, long ld) {
    return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ld % 8 == 0;
  };
  if (kBf16Out && a.d_peers == nullptr && a.grouped != 2 && aligned(a.D, a.ldd) &&
      (EPI != kEpiSwiGLU || aligned(a.D2, a.ldd2))) {
    const int nbd = a.grouped == 1 ? 1 : a.batch;
    const long dcols = EPI == kEpiDSwiGLU ? 2L * a.N : a.N;
    om.d = make_tmap_3d(a.D, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dcols, a.M, nbd, a.ldd * 2,
                        static_cast<uint64_t>(a.M) * a.ldd * 2, 64, 32, 1, CU_TENSOR_MAP_SWIZZLE_128B);
    if (EPI == kEpiSwiGLU)
      om.d2 = make_tmap_3d(a.D2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N / 2, a.M, nbd, a.ldd2 * 2,
                           static_cast<uint64_t>(a.M) * a.ldd2 * 2, 32, 32, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    om.use = 1;
    if (LAY == kLayOutC && (EPI == kEpiDSwiGLU || EPI == kEpiBf16 || EPI == kEpiGateResidual) &&
        aligned(a.C, a.ldc)) {
      om.c = make_tmap_3d(a.C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dcols, a.M, nbd, a.ldc * 2,
                          static_cast<uint64_t>(a.M) * a.ldc * 2, 64, 32, 1, CU_TENSOR_MAP_SWIZZLE_128B);
      om.use_c = 1;
    }
  }
  if constexpr (PAIR) {
    // clusters of two CTAs (grid = 2 x clusters)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_cuda(cudaLaunchKernelEx(&cfg, kern, tA, tB, a, s, status, pm, om),
               "gemm_tc_kernel (CTA pairs) launch");
  } else {
    kern<<<grid, kThreads, Cfg::SMEM_BYTES, stream>>>(tA, tB, a, s, status, pm, om);
  }
  count_launch();
  check_cuda(cudaGetLastError(), "gemm_tc_kernel launch");
}

// Clusters of two 1-CTA-per-SM GEMM CTAs that can be resident at once on this device
// (SMs pair up inside a GPC, so this can be below half the SM count).
int pair_clusters(int dev) {
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 0;
  if (cached[dev] == 0) {
    using Cfg = GemmCfg<256, kLayOut, true>;
    auto kern = gemm_tc_kernel<256, false, false, kEpiBf16, kLayOut, true>;
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES),
               "cudaFuncSetAttribute(gemm pair smem)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms(dev), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = -1;  // pairs unavailable
    }
    cached[dev] = n;
  }
  return cached[dev];
}

// layout by epilogue: fp32 outputs need no boxes; SwiGLU (second output), dSwiGLU and
// residual epilogues with a C operand take all boxes; other bf16 outputs the D boxes only
template <int BN, bool A_MN, bool B_MN, int EPI, bool PAIR>
void launch_p(const GemmArgs& a, const Sched& s, int grid, cudaStream_t stream, int* status) {
  if constexpr (EPI == kEpiF32 || EPI == kEpiF32Atomic) {
    launch_lay<BN, A_MN, B_MN, EPI, kLayF32, PAIR>(a, s, grid, stream, status);
  } else if constexpr (EPI == kEpiSwiGLU || EPI == kEpiDSwiGLU) {
    launch_lay<BN, A_MN, B_MN, EPI, kLayOutC, PAIR>(a, s, grid, stream, status);
  } else if constexpr (EPI == kEpiBf16 || EPI == kEpiGateResidual) {
    if (a.C != nullptr)
      launch_lay<BN, A_MN, B_MN, EPI, kLayOutC, PAIR>(a, s, grid, stream, status);
    else
      launch_lay<BN, A_MN, B_MN, EPI, kLayOut, PAIR>(a, s, grid, stream, status);
  } else {
    launch_lay<BN, A_MN, B_MN, EPI, kLayOut, PAIR>(a, s, grid, stream, status);
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
void launch(const GemmArgs& a, const Sched& s, int grid, cudaStream_t stream, int* status) {
  if (s.bm == 2 * BM)
    launch_p<BN, A_MN, B_MN, EPI, true>(a, s, grid, stream, status);
  else
    launch_p<BN, A_MN, B_MN, EPI, false>(a, s, grid, stream, status);
}

template <int BN>
void dispatch_bn(const GemmArgs& a, int epi, const Sched& s, int grid, cudaStream_t st,
                 int* status) {
  const int mode = (a.a_mn_major ? 2 : 0) | (a.b_mn_major ? 1 : 0);
#define DDB_CASE(E)                                                             \
  case E:                                                                       \
    if (mode == 0) return launch<BN, false, false, E>(a, s, grid, st, status);  \
    if (mode == 1) return launch<BN, false, true, E>(a, s, grid, st, status);   \
    break;
  switch (epi) {
    DDB_CASE(kEpiBf16)
    DDB_CASE(kEpiDSwiGLU)
    case kEpiF32:
      if (mode == 0) return launch<BN, false, false, kEpiF32>(a, s, grid, st, status);
      if (mode == 1) return launch<BN, false, true, kEpiF32>(a, s, grid, st, status);
      if (mode == 3) return launch<BN, true, true, kEpiF32>(a, s, grid, st, status);
      break;
    case kEpiF32Atomic:
      if (mode == 0) return launch<BN, false, false, kEpiF32Atomic>(a, s, grid, st, status);
      if (mode == 3) return launch<BN, true, true, kEpiF32Atomic>(a, s, grid, st, status);
      break;
    case kEpiSwiGLU:
      if (mode == 0) return launch<BN, false, false, kEpiSwiGLU>(a, s, grid, st, status);
      break;
    case kEpiRope:
      if (mode == 0) return launch<BN, false, false, kEpiRope>(a, s, grid, st, status);
      break;
    case kEpiGateResidual:
      if (mode == 0) return launch<BN, false, false, kEpiGateResidual>(a, s, grid, st, status);
      break;
    case kEpiGelu:
      if (mode == 0) return launch<BN, false, false, kEpiGelu>(a, s, grid, st, status);
      break;
    default:
      break;
  }
#undef DDB_CASE
  throw std::runtime_error("gemm: unsupported epilogue/major combination (epi=" +
                           std::to_string(epi) + ", mode=" + std::to_string(mode) + ")");
}

int g_pair_mode = -1;

}  // namespace

int gemm_set_pair_mode(int mode) {
  const int prev = g_pair_mode;
  g_pair_mode = mode < 0 ? -1 : (mode > 0 ? 1 : 0);
  return prev;
}

void gemm(const GemmArgs& a_in, int epi, cudaStream_t stream) {
  GemmArgs a = a_in;
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
  if (a.N % 32 != 0) throw std::runtime_error("gemm: N must be a multiple of 32");
  if (epi == kEpiSwiGLU && a.N % 64 != 0)
    throw std::runtime_error("gemm: SwiGLU needs N % 64 == 0");
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const int sms = num_sms(dev);
  const int kblocks = (a.K + BK - 1) / BK;
  const long nbatch = (a.grouped == 0 && a.batch > 1) ? a.batch : 1;
  // CTA pairs (256-row tiles over two SMs) for plain GEMMs: not for grouped tables, the
  // peer-memory operand forms, or problems of one 128-row tile
  // Pairs are opt-in (DDB_GEMM_PAIRS=1 lets the cost model choose them, gemm_set_pair_mode(1)
  // forces them): intermittent launch failures and TMEM-leak errors appeared in long
  // training runs once pairs were on by default; the cause is not pinned down.
  static const bool pairs_env = std::getenv("DDB_GEMM_PAIRS") != nullptr &&
                                std::getenv("DDB_GEMM_NO_PAIRS") == nullptr;
  const bool pairs_on = g_pair_mode == 1 || (g_pair_mode == -1 && pairs_env);
  const int clusters = (pairs_on && a.grouped == 0 && a.a_npeers == 0 && a.d_peers == nullptr &&
                        a.gb_world <= 1 && a.M > BM) ? pair_clusters(dev) : 0;
  // Estimated time of a (pair, BN, split-K) choice: waves of persistent tiles x tile work
  // at a relative efficiency. Operand bytes staged and read from shared memory per FLOP
  // set it: a 128-wide single-CTA tile reads A twice as often per FLOP as a 256-wide one
  // (~0.8 of it); a 256 x 256 CTA-pair tile stages a third less than a 128 x 256
  // single-CTA tile (taken as ~1.15 of it). The SwiGLU epilogues are bound by their own
  // memory traffic, where pairs gain nothing (measured), so they stay single-CTA.
  const bool epi_bound = (epi == kEpiSwiGLU || epi == kEpiDSwiGLU) && g_pair_mode != 1;
  auto est = [&](bool pr, int bn_c, int sp) -> double {
    const long tm = (a.M + (pr ? 2 * BM : BM) - 1) / (pr ? 2 * BM : BM);
    const long units = pr ? clusters : sms;
    const long items = tm * ((a.N + bn_c - 1) / bn_c) * sp * nbatch;
    const long waves = (items + units - 1) / units;
    const long kb = (kblocks + sp - 1) / sp;
    const double eff = pr ? (epi_bound ? 0.0 : (bn_c == 256 ? 1.15 : 0.95))
                          : (bn_c == 256 ? 1.0 : 0.8);
    if (eff == 0.0) return 1e300;
    return static_cast<double>(waves) * bn_c * kb / eff;
  };
  // split K (fp32-accumulating epilogue only) while it strictly shortens the estimate
  auto best_splits = [&](bool pr, int bn_c) {
    int sp = 1;
    if (epi == kEpiF32Atomic) {
      // deterministic mode: one writer per output element, so the fp32 accumulation
      // does not depend on the arrival order of split-K partial sums
      if (deterministic()) return 1;
      if (a.splits > 0) return a.splits;
      while (kblocks / (sp * 2) >= 8 && est(pr, bn_c, sp * 2) < est(pr, bn_c, sp)) sp *= 2;
    }
    return sp;
  };
  // tile shape (pair or not, width) and split-K chosen together
  bool pair = false;
  int bn = a.bn;
  {
    double best = 1e300;
    const bool wide_ok = a.N >= 256 && !(a.N % 256 != 0 && a.N < 512);
    for (int pr = (clusters > 0 && g_pair_mode == 1) ? 1 : 0; pr < (clusters > 0 ? 2 : 1); ++pr)
      for (int bn_c : {128, 256}) {
        if (a.bn != 0 && bn_c != a.bn) continue;
        if (a.bn == 0 && bn_c == 256 && !wide_ok) continue;
        const double e = est(pr != 0, bn_c, best_splits(pr != 0, bn_c));
        // ties: the wider tile of the same kind; a pair only when strictly faster
        if (e < best || (e == best && bn_c == 256 && bn != 256 && (pr != 0) == pair)) {
          best = e;
          pair = pr != 0;
          bn = bn_c;
        }
      }
    if (bn == 0) bn = 128;
  }
  Sched s;
  s.bm = pair ? 2 * BM : BM;
  s.tiles_m = static_cast<int>((a.M + s.bm - 1) / s.bm);
  s.tiles_n = (a.N + bn - 1) / bn;
  s.kblocks = kblocks;
  const int splits = best_splits(pair, bn);
  s.kb_per_split = (s.kblocks + splits - 1) / splits;
  s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;
  s.M = a.M;
  s.grouped = a.grouped;
  s.g_tile_expert = a.grp_tile_expert;
  s.g_tile_row = a.grp_tile_row;
  s.g_total_mtiles = a.grp_total_mtiles;
  s.g_kstart = a.grp_kstart;
  s.g_kend = a.grp_kend;
  if (a.grouped == 1) {
    s.splits = 1;
    s.total = a.grp_max_mtiles * s.tiles_n;
  } else if (a.grouped == 2) {
    s.splits = 1;
    s.total = s.tiles_m * s.tiles_n * a.batch;
  } else {
    s.total = s.tiles_m * s.tiles_n * s.splits * (a.batch > 1 ? a.batch : 1);
  }
  if (a.gb_world > 1) {
    if (a.b_mn_major || a.batch > 1 || a.grouped || a.ldb != a.K || a.K % 8 != 0)
      throw std::runtime_error("gemm: the fused weight gather needs an unbatched K-major B with ldb == K");
    if (a.gb_world > kMaxGemmPeers || a.gb_rank < 0 || a.gb_rank >= a.gb_world ||
        a.gb_peers[a.gb_rank] != a.B || a.gb_counters == nullptr || a.gb_epoch == 0 ||
        a.gb_shard <= 0 || a.gb_shard % 8 != 0 || a.gb_elem0 % 8 != 0 ||
        a.gb_elem0 + static_cast<long>(a.N) * a.K > a.gb_shard * a.gb_world)
      throw std::runtime_error("gemm: bad fused weight-gather arguments");
    for (int r = 0; r < a.gb_world; ++r)
      if (a.gb_peers[r] == nullptr || (reinterpret_cast<uintptr_t>(a.gb_peers[r]) & 15) != 0)
        throw std::runtime_error("gemm: weight-gather peer pointers must be 16-byte aligned");
  }
  if (a.batch > 1 && ((a.grouped == 0 && a.stride_a % 8 != 0) ||
                      (a.grouped != 2 && a.stride_b % 8 != 0)))
    throw std::runtime_error("gemm: batch strides must be multiples of 8 elements");
  int grid = s.total < sms ? s.total : sms;
  if (a.max_ctas > 0 && grid > a.max_ctas) grid = a.max_ctas;
  if (pair) {  // two CTAs per cluster, one cluster per pair tile at most
    int nc = s.total < clusters ? s.total : clusters;
    if (a.max_ctas > 0 && nc > a.max_ctas / 2) nc = a.max_ctas / 2 > 0 ? a.max_ctas / 2 : 1;
    grid = 2 * nc;
  }
  int* status = device_status(dev);
  if (bn == 256)
    dispatch_bn<256>(a, epi, s, grid, stream, status);
  else
    dispatch_bn<128>(a, epi, s, grid, stream, status);
}

}  // namespace ddb
