// SLA linear branch on the tensor cores (tcgen05), sm_100a.
//
// The linear branch of sparse-linear attention (phi = elu + 1; reference
// layers/sla.py:333-357) needs, per 64-token block, 64 x 64 x 64 products: the key-side
// state phi(K)^T V, the query-side output phi(Q) S, and in backward dnum S^T, phi(Q)^T dnum,
// V G^T and phi(K) G (S / G: the block's fp32 state or state gradient from the batched
// GEMM over blocks). One CTA takes two consecutive blocks: the two 64 x 64 A tiles stack
// into one M = 128 operand, and the product runs once with each block's B tile (M=128,
// N=64, K=64: D1 = A B1, D2 = A B2); rows 0-63 of D1 and rows 64-127 of D2 are the two
// blocks' results. Every operand is a 64 x 64 bf16 tile stored row-major in shared memory
// with the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r & 7)); whether a tile
// is read K-major or MN-major is the descriptor's choice, so no operand is transposed.
//
// Threads: 128 (thread r owns TMEM lane / output row r). Thread 0 issues the MMAs; all
// threads stage operands, wait on one mbarrier (bounded) and run the epilogue. The small
// per-row reductions (normaliser sums) stay on the CUDA cores in fp32.
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "sla.h"

namespace ddb {
namespace {

constexpr int D = 64;
constexpr int NZ = D * D + D;   // per-block state: [64 x 64] + normaliser row
constexpr int TILE = 8192;      // 64 x 64 bf16
constexpr int kThreads = 128;
constexpr uint32_t IDESC_KK = make_idesc_bf16(128, 64, false, false);  // A K-major, B K-major
constexpr uint32_t IDESC_KM = make_idesc_bf16(128, 64, false, true);   // A K-major, B MN-major
constexpr uint32_t IDESC_MM = make_idesc_bf16(128, 64, true, true);    // A MN-major, B MN-major

__device__ __forceinline__ float phi(float x) { return x > 0.f ? x + 1.f : __expf(x); }
__device__ __forceinline__ float dphi(float x) { return x > 0.f ? 1.f : __expf(x); }

// 8 bf16 at (row r, 16-byte chunk c8) of a swizzled tile
__device__ __forceinline__ void tile_put(uint32_t tile, int r, int c8, uint32_t a, uint32_t b, uint32_t c,
                                         uint32_t d) {
  st_shared_v4(tile + r * 128 + ((c8 ^ (r & 7)) << 4), a, b, c, d);
}
__device__ __forceinline__ uint4 tile_get(uint32_t tile, int r, int c8) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(tile + r * 128 + ((c8 ^ (r & 7)) << 4)));
  return v;
}

// Staging is split into a load phase (all of a tile's 16-byte pieces of this thread in
// flight at once, plain loads the compiler may batch) and a store phase, so a CTA pays
// one memory latency per batch of tiles instead of one per piece.
struct RowTile {
  uint4 u[4];  // pieces i = threadIdx.x + 128 * j: row i >> 3, 16-byte chunk i & 7
};
__device__ __forceinline__ void load_rows(RowTile& t, const __nv_bfloat16* src, long ld) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + kThreads * j;
    t.u[j] = *reinterpret_cast<const uint4*>(src + (i >> 3) * ld + (i & 7) * 8);
  }
}
// [64 tokens x 64] bf16 rows -> swizzled tile, phi applied or not
__device__ __forceinline__ void store_rows(uint32_t tile, const RowTile& t, bool apply_phi) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + kThreads * j;
    const uint4 u = t.u[j];
    if (!apply_phi) {
      tile_put(tile, i >> 3, i & 7, u.x, u.y, u.z, u.w);
    } else {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16(w[q]);
        o[q] = pack_bf16(phi(f.x), phi(f.y));
      }
      tile_put(tile, i >> 3, i & 7, o[0], o[1], o[2], o[3]);
    }
  }
}
struct F32Tile {
  float4 a[4], b[4];
};
// dense fp32 [64 x 64] (row stride 64)
__device__ __forceinline__ void load_f32(F32Tile& t, const float* src) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + kThreads * j;
    t.a[j] = *reinterpret_cast<const float4*>(src + (i >> 3) * 64 + (i & 7) * 8);
    t.b[j] = *reinterpret_cast<const float4*>(src + (i >> 3) * 64 + (i & 7) * 8 + 4);
  }
}
__device__ __forceinline__ void store_f32(uint32_t tile, const F32Tile& t) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + kThreads * j;
    tile_put(tile, i >> 3, i & 7, pack_bf16(t.a[j].x, t.a[j].y), pack_bf16(t.a[j].z, t.a[j].w),
             pack_bf16(t.b[j].x, t.b[j].y), pack_bf16(t.b[j].z, t.b[j].w));
  }
}
// one 128-byte row segment (64 bf16) of a token as 8 plain 16-byte loads
__device__ __forceinline__ void load_row64(uint4 (&u)[8], const __nv_bfloat16* p) {
#pragma unroll
  for (int c8 = 0; c8 < 8; ++c8) u[c8] = *reinterpret_cast<const uint4*>(p + c8 * 8);
}

// Shared-memory descriptors of a tile pair stacked along M (tile 1 at +TILE) or of one tile.
__device__ __forceinline__ uint64_t desc_k(uint32_t tile, int kk) { return make_sw128_desc(tile + kk * 32, 16, 1024); }
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile, int kk) {
  return make_sw128_desc(tile + kk * 2048, TILE, 1024);
}

// D1 = A B1, D2 = A B2 (K = 64 in four K = 16 steps); a_mn / b_mn choose the descriptors.
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint32_t a, uint32_t b1, uint32_t b2, bool a_mn,
                                         bool b_mn, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t da = a_mn ? desc_mn(a, kk) : desc_k(a, kk);
    mma_bf16_ss(d_tmem, da, b_mn ? desc_mn(b1, kk) : desc_k(b1, kk), idesc, kk > 0 ? 1u : 0u);
    mma_bf16_ss(d_tmem + 64, da, b_mn ? desc_mn(b2, kk) : desc_k(b2, kk), idesc, kk > 0 ? 1u : 0u);
  }
}

// CTA prologue / epilogue shared by the four kernels: TMEM allocation, one mbarrier.
struct TcCta {
  uint32_t tmem;
  uint64_t* bar;
  volatile int* abort_flag;
};

__device__ __forceinline__ TcCta tc_setup(uint8_t* smem_tail, uint32_t cols) {
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_tail);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(slot + 1);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(slot, cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return TcCta{*slot, bar, abort_flag};
}

// operands written by all threads -> visible to the tensor core; thread 0 then issues
__device__ __forceinline__ void operands_ready() {
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// wait for the MMAs (bounded); false on timeout (recorded in the status word)
__device__ __forceinline__ bool wait_mma(const TcCta& c, int* status, uint32_t phase = 0) {
  if (!mbar_wait(c.bar, phase, c.abort_flag)) {
    if (status) atomicCAS(status, 0, kStatusTimeoutEpilogue);
    *c.abort_flag = 1;
    return false;
  }
  tc_fence_after();
  return true;
}

__device__ __forceinline__ void tc_teardown(const TcCta& c, uint32_t cols) {
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    tmem_dealloc(c.tmem, cols);
  }
}

// The second product of the backward kernels reuses the first one's TMEM columns once
// every thread has read them (128 columns per CTA keep four CTAs per SM).
__device__ __forceinline__ void tmem_reads_done() {
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// Row r of the result: D1 for the first block's rows, D2 (64 columns further) for the second.
__device__ __forceinline__ void tmem_row64(uint32_t tmem, uint32_t (&v)[64]) {
  const int r = threadIdx.x;
  const uint32_t base = tmem + (static_cast<uint32_t>((r >> 5) * 32) << 16) + (r >> 6) * 64;
  uint32_t a[32], b[32];
  tmem_ld32(base, a);
  tmem_ld32(base + 32, b);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = a[i];
    v[32 + i] = b[i];
  }
}

constexpr int SMEM_TAIL = 64;

// ------------------------------------------------------------------ kernels
// KVz_j = [phi(K_j)^T V_j (row d), sum_t phi(K_j)[t][d]] as bf16. M = d: A = [phi(K_1) |
// phi(K_2)] read MN-major (tiles [t][d]), B_j = V_j [t][e] MN-major.
__global__ void __launch_bounds__(kThreads) sla_kv_state_tc(const __nv_bfloat16* __restrict__ qkv, long ld,
                                                            int T, int H, int nbp,
                                                            __nv_bfloat16* __restrict__ kvz, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t s0 = smem_u32(smem);
  if (s0 & 1023) {  // swizzled tiles need a 1024-byte aligned window
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadArgument);
    return;
  }
  const uint32_t tA = s0, tB1 = s0 + 2 * TILE, tB2 = s0 + 3 * TILE;
  const int pr = blockIdx.x % nbp, bh = blockIdx.x / nbp, b = bh / H, h = bh % H;
  const int dm = H * D, nb = 2 * nbp;
  const long row0 = static_cast<long>(b) * T + pr * 128;
  TcCta c = tc_setup(smem + 4 * TILE, 128);
  {
    RowTile k1, k2, v1, v2;
    load_rows(k1, qkv + row0 * ld + dm + h * D, ld);
    load_rows(k2, qkv + (row0 + 64) * ld + dm + h * D, ld);
    load_rows(v1, qkv + row0 * ld + 2 * dm + h * D, ld);
    load_rows(v2, qkv + (row0 + 64) * ld + 2 * dm + h * D, ld);
    store_rows(tA, k1, true);
    store_rows(tA + TILE, k2, true);
    store_rows(tB1, v1, false);
    store_rows(tB2, v2, false);
  }
  operands_ready();
  if (threadIdx.x == 0) {
    mma_pair(c.tmem, tA, tB1, tB2, true, true, IDESC_MM);
    mma_commit(c.bar);
  }
  // normaliser z_j[d] = sum_t phi(k[t][d]) over the staged phi(K) tile (thread r: block
  // r >> 6, feature r & 63), fp32 sums
  const int r = threadIdx.x, blk = r >> 6, dd = r & 63;
  float z = 0.f;
  for (int t = 0; t < 64; ++t) {
    const uint4 u = tile_get(tA + blk * TILE, t, dd >> 3);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    const float2 f = unpack_bf16(w[(dd & 7) >> 1]);
    z += (dd & 1) ? f.y : f.x;
  }
  if (wait_mma(c, status)) {
    uint32_t v[64];
    tmem_row64(c.tmem, v);
    __nv_bfloat16* out = kvz + (static_cast<long>(bh) * nb + 2 * pr + blk) * NZ;
#pragma unroll
    for (int e = 0; e < 64; e += 8)
      st_global_v4(out + dd * D + e, pack_bf16(__uint_as_float(v[e]), __uint_as_float(v[e + 1])),
                   pack_bf16(__uint_as_float(v[e + 2]), __uint_as_float(v[e + 3])),
                   pack_bf16(__uint_as_float(v[e + 4]), __uint_as_float(v[e + 5])),
                   pack_bf16(__uint_as_float(v[e + 6]), __uint_as_float(v[e + 7])));
    out[D * D + dd] = __float2bfloat16(z);
  }
  tc_teardown(c, 128);
}

// o = phi(Q) S / (phi(Q) . z + eps). M = t: A = phi(Q) tiles K-major, B_j = S_j [d][e]
// MN-major (bf16 copy of the fp32 state).
__global__ void __launch_bounds__(kThreads) sla_lin_out_tc(const __nv_bfloat16* __restrict__ qkv, long ld,
                                                           int T, int H, int nbp, const float* __restrict__ state,
                                                           __nv_bfloat16* __restrict__ o, long ldo,
                                                           float* __restrict__ den_out, float eps, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t s0 = smem_u32(smem);
  if (s0 & 1023) {  // swizzled tiles need a 1024-byte aligned window
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadArgument);
    return;
  }
  const uint32_t tA = s0, tB1 = s0 + 2 * TILE, tB2 = s0 + 3 * TILE;
  float* zs = reinterpret_cast<float*>(smem + 4 * TILE + SMEM_TAIL);  // [2][64]
  const int pr = blockIdx.x % nbp, bh = blockIdx.x / nbp, b = bh / H, h = bh % H;
  const int nb = 2 * nbp;
  const long row0 = static_cast<long>(b) * T + pr * 128;
  const float* S1 = state + (static_cast<long>(bh) * nb + 2 * pr) * NZ;
  const float* S2 = S1 + NZ;
  TcCta c = tc_setup(smem + 4 * TILE, 128);
  {
    RowTile q1, q2;
    F32Tile f1, f2;
    load_rows(q1, qkv + row0 * ld + h * D, ld);
    load_rows(q2, qkv + (row0 + 64) * ld + h * D, ld);
    load_f32(f1, S1);
    load_f32(f2, S2);
    if (threadIdx.x < 64) {
      zs[threadIdx.x] = S1[D * D + threadIdx.x];
      zs[64 + threadIdx.x] = S2[D * D + threadIdx.x];
    }
    store_rows(tA, q1, true);
    store_rows(tA + TILE, q2, true);
    store_f32(tB1, f1);
    store_f32(tB2, f2);
  }
  operands_ready();
  if (threadIdx.x == 0) {
    mma_pair(c.tmem, tA, tB1, tB2, false, true, IDESC_KM);
    mma_commit(c.bar);
  }
  // den[t] = phi(q[t]) . z + eps from the staged bf16 phi(q) row, fp32 sums
  const int r = threadIdx.x, blk = r >> 6;
  float den = eps;
#pragma unroll
  for (int c8 = 0; c8 < 8; ++c8) {
    const uint4 u = tile_get(tA + blk * TILE, r & 63, c8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16(w[j]);
      den += f.x * zs[blk * 64 + c8 * 8 + 2 * j] + f.y * zs[blk * 64 + c8 * 8 + 2 * j + 1];
    }
  }
  den_out[static_cast<long>(bh) * T + pr * 128 + r] = den;
  if (wait_mma(c, status)) {
    uint32_t v[64];
    tmem_row64(c.tmem, v);
    const float inv = 1.f / den;
    __nv_bfloat16* orow = o + (row0 + r) * ldo + h * D;
#pragma unroll
    for (int e = 0; e < 64; e += 8)
      st_global_v4(orow + e, pack_bf16(__uint_as_float(v[e]) * inv, __uint_as_float(v[e + 1]) * inv),
                   pack_bf16(__uint_as_float(v[e + 2]) * inv, __uint_as_float(v[e + 3]) * inv),
                   pack_bf16(__uint_as_float(v[e + 4]) * inv, __uint_as_float(v[e + 5]) * inv),
                   pack_bf16(__uint_as_float(v[e + 6]) * inv, __uint_as_float(v[e + 7]) * inv));
  }
  tc_teardown(c, 128);
}

// Backward, query side. dnum = do / den, dden = -(do . o) / den;
//   (a) dphi(q)[t][d] = sum_e dnum[t][e] S[d][e] (+ dden[t] z[d]): A = dnum tiles K-major,
//       B_j = S_j K-major (rows d);
//   (b) dS_j[d][e] = sum_t phi(q)[t][d] dnum[t][e]: A = phi(Q) tiles MN-major, B_j = dnum_j
//       MN-major; dz_j[d] = sum_t phi(q)[t][d] dden[t] on the CUDA cores.
// dq += dphi(q) * phi'(q); dS, dz -> dsz (bf16) for the transposed batched GEMM.
__global__ void __launch_bounds__(kThreads) sla_lin_bwd_q_tc(
    const __nv_bfloat16* __restrict__ qkv, long ld, int T, int H, int nbp, const float* __restrict__ state,
    const __nv_bfloat16* __restrict__ o, long ldo, const __nv_bfloat16* __restrict__ dout, long lddo,
    const float* __restrict__ den_in, __nv_bfloat16* __restrict__ dsz, __nv_bfloat16* __restrict__ dqkv,
    long lddq, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t s0 = smem_u32(smem);
  if (s0 & 1023) {  // swizzled tiles need a 1024-byte aligned window
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadArgument);
    return;
  }
  const uint32_t tQ = s0, tN = s0 + 2 * TILE, tS1 = s0 + 4 * TILE, tS2 = s0 + 5 * TILE;
  float* zs = reinterpret_cast<float*>(smem + 6 * TILE + SMEM_TAIL);  // [2][64]
  float* dds = zs + 128;                                              // [128] dden
  const int pr = blockIdx.x % nbp, bh = blockIdx.x / nbp, b = bh / H, h = bh % H;
  const int nb = 2 * nbp;
  const long row0 = static_cast<long>(b) * T + pr * 128;
  const float* S1 = state + (static_cast<long>(bh) * nb + 2 * pr) * NZ;
  const float* S2 = S1 + NZ;
  TcCta c = tc_setup(smem + 6 * TILE, 128);
  {
    RowTile q1, q2;
    F32Tile f1, f2;
    load_rows(q1, qkv + row0 * ld + h * D, ld);
    load_rows(q2, qkv + (row0 + 64) * ld + h * D, ld);
    load_f32(f1, S1);
    load_f32(f2, S2);
    if (threadIdx.x < 64) {
      zs[threadIdx.x] = S1[D * D + threadIdx.x];
      zs[64 + threadIdx.x] = S2[D * D + threadIdx.x];
    }
    store_rows(tQ, q1, true);
    store_rows(tQ + TILE, q2, true);
    store_f32(tS1, f1);
    store_f32(tS2, f2);
  }
  {  // thread r: token r's dnum row (tile) and dden
    const int r = threadIdx.x;
    const float den = den_in[static_cast<long>(bh) * T + pr * 128 + r];
    const float inv = 1.f / den;
    uint4 gall[8], oall[8];
    load_row64(gall, dout + (row0 + r) * lddo + h * D);
    load_row64(oall, o + (row0 + r) * ldo + h * D);
    float part = 0.f;
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      const uint4 gu = gall[c8], ou = oall[c8];
      const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w}, ow[4] = {ou.x, ou.y, ou.z, ou.w};
      uint32_t pk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 g = unpack_bf16(gw[j]), ov = unpack_bf16(ow[j]);
        part += g.x * ov.x + g.y * ov.y;
        pk[j] = pack_bf16(g.x * inv, g.y * inv);
      }
      tile_put(tN + (r >> 6) * TILE, r & 63, c8, pk[0], pk[1], pk[2], pk[3]);
    }
    dds[r] = -part * inv;
  }
  operands_ready();
  if (threadIdx.x == 0) {
    mma_pair(c.tmem, tN, tS1, tS2, false, false, IDESC_KK);  // (a)
    mma_commit(c.bar);
  }
  const int r = threadIdx.x, blk = r >> 6, dd = r & 63;
  // dz_j[d] = sum_t phi(q)[t][d] dden[t] for block blk, feature dd (fp32 over bf16 phi)
  // this token's q and dq rows for the epilogue, in flight while the MMAs run
  __nv_bfloat16* qrow = dqkv + (row0 + r) * lddq + h * D;
  uint4 qall[8], call[8];
  load_row64(qall, qkv + (row0 + r) * ld + h * D);
  load_row64(call, qrow);
  float dzp[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains over t
#pragma unroll 8
  for (int t = 0; t < 64; ++t) {
    const uint4 u = tile_get(tQ + blk * TILE, t, dd >> 3);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    const float2 f = unpack_bf16(w[(dd & 7) >> 1]);
    dzp[t & 3] += ((dd & 1) ? f.y : f.x) * dds[blk * 64 + t];
  }
  const float dz = (dzp[0] + dzp[1]) + (dzp[2] + dzp[3]);
  if (wait_mma(c, status)) {
    uint32_t v[64];
    tmem_row64(c.tmem, v);  // (a): row r = token r, column d
    {
      const float ddn = dds[r];
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const uint4 qv = qall[c8], cv = call[c8];
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w}, cw[4] = {cv.x, cv.y, cv.z, cv.w};
        uint32_t ow[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int d0 = c8 * 8 + 2 * j;
          const float2 q = unpack_bf16(qw[j]), cur = unpack_bf16(cw[j]);
          const float g0 = (__uint_as_float(v[d0]) + ddn * zs[blk * 64 + d0]) * dphi(q.x);
          const float g1 = (__uint_as_float(v[d0 + 1]) + ddn * zs[blk * 64 + d0 + 1]) * dphi(q.y);
          ow[j] = pack_bf16(cur.x + g0, cur.y + g1);
        }
        st_global_v4(qrow + c8 * 8, ow[0], ow[1], ow[2], ow[3]);
      }
    }
  }
  tmem_reads_done();
  if (threadIdx.x == 0 && !*c.abort_flag) {
    mma_pair(c.tmem, tQ, tN, tN + TILE, true, true, IDESC_MM);  // (b) into the same columns
    mma_commit(c.bar);
  }
  if (!*c.abort_flag && wait_mma(c, status, 1)) {
    uint32_t v[64];
    tmem_row64(c.tmem, v);  // (b): row r = (block r >> 6, feature r & 63), column e
    __nv_bfloat16* out = dsz + (static_cast<long>(bh) * nb + 2 * pr + blk) * NZ;
#pragma unroll
    for (int e = 0; e < 64; e += 8)
      st_global_v4(out + dd * D + e, pack_bf16(__uint_as_float(v[e]), __uint_as_float(v[e + 1])),
                   pack_bf16(__uint_as_float(v[e + 2]), __uint_as_float(v[e + 3])),
                   pack_bf16(__uint_as_float(v[e + 4]), __uint_as_float(v[e + 5])),
                   pack_bf16(__uint_as_float(v[e + 6]), __uint_as_float(v[e + 7])));
    out[D * D + dd] = __float2bfloat16(dz);
  }
  tc_teardown(c, 128);
}

// Backward, key side. (a) dphi(K)[t][d] = sum_e V[t][e] G[d][e] (+ dz[d]): A = V tiles
// K-major, B_j = G_j K-major; (b) dV[t][e] = sum_d phi(K)[t][d] G[d][e]: A = phi(K) tiles
// K-major, B_j = G_j MN-major. dk += dphi(K) * phi'(k), dv += dV.
__global__ void __launch_bounds__(kThreads) sla_lin_bwd_kv_tc(const __nv_bfloat16* __restrict__ qkv, long ld,
                                                              int T, int H, int nbp, const float* __restrict__ dkvz,
                                                              __nv_bfloat16* __restrict__ dqkv, long lddq,
                                                              int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t s0 = smem_u32(smem);
  if (s0 & 1023) {  // swizzled tiles need a 1024-byte aligned window
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadArgument);
    return;
  }
  const uint32_t tV = s0, tK = s0 + 2 * TILE, tG1 = s0 + 4 * TILE, tG2 = s0 + 5 * TILE;
  float* dzs = reinterpret_cast<float*>(smem + 6 * TILE + SMEM_TAIL);  // [2][64]
  const int pr = blockIdx.x % nbp, bh = blockIdx.x / nbp, b = bh / H, h = bh % H;
  const int dm = H * D, nb = 2 * nbp;
  const long row0 = static_cast<long>(b) * T + pr * 128;
  const float* G1 = dkvz + (static_cast<long>(bh) * nb + 2 * pr) * NZ;
  const float* G2 = G1 + NZ;
  TcCta c = tc_setup(smem + 6 * TILE, 128);
  {
    RowTile v1, v2, k1, k2;
    load_rows(v1, qkv + row0 * ld + 2 * dm + h * D, ld);
    load_rows(v2, qkv + (row0 + 64) * ld + 2 * dm + h * D, ld);
    load_rows(k1, qkv + row0 * ld + dm + h * D, ld);
    load_rows(k2, qkv + (row0 + 64) * ld + dm + h * D, ld);
    store_rows(tV, v1, false);
    store_rows(tV + TILE, v2, false);
    store_rows(tK, k1, true);
    store_rows(tK + TILE, k2, true);
  }
  {
    F32Tile g1, g2;
    load_f32(g1, G1);
    load_f32(g2, G2);
    if (threadIdx.x < 64) {
      dzs[threadIdx.x] = G1[D * D + threadIdx.x];
      dzs[64 + threadIdx.x] = G2[D * D + threadIdx.x];
    }
    store_f32(tG1, g1);
    store_f32(tG2, g2);
  }
  operands_ready();
  if (threadIdx.x == 0) {
    mma_pair(c.tmem, tV, tG1, tG2, false, false, IDESC_KK);  // (a)
    mma_commit(c.bar);
  }
  const int r = threadIdx.x, blk = r >> 6;
  // this token's k and dk rows for the epilogue, in flight while the MMAs run
  __nv_bfloat16* krow = dqkv + (row0 + r) * lddq + dm + h * D;
  uint4 kall[8], call[8];
  load_row64(kall, qkv + (row0 + r) * ld + dm + h * D);
  load_row64(call, krow);
  if (wait_mma(c, status)) {
    uint32_t v[64];
    tmem_row64(c.tmem, v);
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      const uint4 kv = kall[c8], cv = call[c8];
      const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w}, cw[4] = {cv.x, cv.y, cv.z, cv.w};
      uint32_t ow[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d0 = c8 * 8 + 2 * j;
        const float2 k = unpack_bf16(kw[j]), cur = unpack_bf16(cw[j]);
        ow[j] = pack_bf16(cur.x + (__uint_as_float(v[d0]) + dzs[blk * 64 + d0]) * dphi(k.x),
                          cur.y + (__uint_as_float(v[d0 + 1]) + dzs[blk * 64 + d0 + 1]) * dphi(k.y));
      }
      st_global_v4(krow + c8 * 8, ow[0], ow[1], ow[2], ow[3]);
    }
  }
  tmem_reads_done();
  if (threadIdx.x == 0 && !*c.abort_flag) {
    mma_pair(c.tmem, tK, tG1, tG2, false, true, IDESC_KM);  // (b) into the same columns
    mma_commit(c.bar);
  }
  if (!*c.abort_flag && wait_mma(c, status, 1)) {
    uint32_t v[64];
    tmem_row64(c.tmem, v);
    __nv_bfloat16* vrow = dqkv + (row0 + r) * lddq + 2 * dm + h * D;
    uint4 vall[8];
    load_row64(vall, vrow);
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      const uint4 cv = vall[c8];
      const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
      uint32_t ow[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e0 = c8 * 8 + 2 * j;
        const float2 cur = unpack_bf16(cw[j]);
        ow[j] = pack_bf16(cur.x + __uint_as_float(v[e0]), cur.y + __uint_as_float(v[e0 + 1]));
      }
      st_global_v4(vrow + c8 * 8, ow[0], ow[1], ow[2], ow[3]);
    }
  }
  tc_teardown(c, 128);
}

template <typename K>
void set_smem(K kern, int bytes) {
  check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
             "cudaFuncSetAttribute(sla tc)");
}

int* status_word() {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  return device_status(dev);
}

constexpr int SMEM4 = 4 * TILE + SMEM_TAIL + 512 * 4;
constexpr int SMEM6 = 6 * TILE + SMEM_TAIL + 512 * 4;

void check_blocks(int T) {
  if (T % 128 != 0) throw std::runtime_error("sla linear branch: tokens per sequence must be a multiple of 128");
}

}  // namespace

void sla_kv_state(const __nv_bfloat16* qkv, long ld, int B, int T, int H, __nv_bfloat16* kvz, cudaStream_t s) {
  check_blocks(T);
  static bool attr = false;
  if (!attr) {
    set_smem(sla_kv_state_tc, SMEM4);
    attr = true;
  }
  const int nbp = T / 128;
  sla_kv_state_tc<<<B * H * nbp, kThreads, SMEM4, s>>>(qkv, ld, T, H, nbp, kvz, status_word());
  count_launch();
  check_cuda(cudaGetLastError(), "sla_kv_state launch");
}

void sla_lin_out(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                 __nv_bfloat16* o, long ldo, float* den, float eps, cudaStream_t s) {
  check_blocks(T);
  static bool attr = false;
  if (!attr) {
    set_smem(sla_lin_out_tc, SMEM4);
    attr = true;
  }
  const int nbp = T / 128;
  sla_lin_out_tc<<<B * H * nbp, kThreads, SMEM4, s>>>(qkv, ld, T, H, nbp, state, o, ldo, den, eps,
                                                      status_word());
  count_launch();
  check_cuda(cudaGetLastError(), "sla_lin_out launch");
}

void sla_lin_bwd_q(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                   const __nv_bfloat16* o, long ldo, const __nv_bfloat16* dout, long lddo,
                   const float* den, __nv_bfloat16* dsz, __nv_bfloat16* dqkv, long lddq, cudaStream_t s) {
  check_blocks(T);
  static bool attr = false;
  if (!attr) {
    set_smem(sla_lin_bwd_q_tc, SMEM6);
    attr = true;
  }
  const int nbp = T / 128;
  sla_lin_bwd_q_tc<<<B * H * nbp, kThreads, SMEM6, s>>>(qkv, ld, T, H, nbp, state, o, ldo, dout, lddo, den,
                                                        dsz, dqkv, lddq, status_word());
  count_launch();
  check_cuda(cudaGetLastError(), "sla_lin_bwd_q launch");
}

void sla_lin_bwd_kv(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* dkvz,
                    __nv_bfloat16* dqkv, long lddq, cudaStream_t s) {
  check_blocks(T);
  static bool attr = false;
  if (!attr) {
    set_smem(sla_lin_bwd_kv_tc, SMEM6);
    attr = true;
  }
  const int nbp = T / 128;
  sla_lin_bwd_kv_tc<<<B * H * nbp, kThreads, SMEM6, s>>>(qkv, ld, T, H, nbp, dkvz, dqkv, lddq, status_word());
  count_launch();
  check_cuda(cudaGetLastError(), "sla_lin_bwd_kv launch");
}

}  // namespace ddb
