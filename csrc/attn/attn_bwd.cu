// tcgen05 flash-attention backward, d_head = 64, for sm_100a (KV-stationary).
//
// One CTA = one (batch, head, 128-key tile = two adjacent 64-key blocks); it walks the
// 128-query units that can see its keys: the 128-query tiles of all later frames
// (frame-causal), or for SLA the query blocks that selected one of its two key blocks,
// two 64-query blocks per unit in any combination (routing lists `kv_qtiles`), so a unit
// carries no query block that selected neither key block. Per query unit, with the key
// tile's K and V resident in shared memory:
//
//   S^T  = K Q^T      (M=128 keys, N=128 queries, K=64)        TMEM cols [  0,128)
//   dP^T = V dO^T     (M=128, N=128, K=64)                      TMEM cols [128,256)
//   softmax warps (one thread per key row): P^T = exp2(S^T*scale*log2e - lse) -> TMEM
//                 cols [448,512) as bf16 pairs; dS^T = scale * P^T (dP^T - delta) ->
//                 shared memory (bf16, 128-byte swizzle)
//   dV  += P^T dO     (M=128, N=64, K=128 queries; A read from TMEM) TMEM cols [256,320)
//   dK  += dS^T Q     (M=128, N=64, K=128)                      TMEM cols [320,384)
//   dQ   = dS K       (M=128 queries, N=64, K=128 keys; dS^T read MN-major)
//                                                               TMEM cols [384,448)
//   dQ warps: TMEM -> the tile's dS^T buffer (free once dQ is computed; fp32, two
//             128-byte swizzled boxes) -> one TMA reduce-add into the fp32 dQ
//             accumulator, so the accumulation bypasses the load/store pipe the softmax
//             warps use.
// Q / dO (+ lse / delta) stream through 3 stages; keeping P^T out of shared memory pays
// for the third stage and halves the shared-memory reads of the dV MMA.
// After the last query tile dK and dV go to global memory (bf16).
//
// Roles: warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 softmax/dS (two warps per TMEM lane
// quarter: warps 2-5 take queries 0-63 of the tile, warps 6-9 queries 64-127, so two
// softmax warps share each SM sub-partition), warps 10-13 dQ.
#include <cuda.h>
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "attn.h"

namespace ddb {
namespace {

constexpr int kThreads = 448;
constexpr int NS = 3;                          // Q / dO stages
constexpr int TILE = 16384;
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + TILE;
constexpr int OFF_Q = OFF_V + TILE;            // NS stages
constexpr int OFF_DO = OFF_Q + NS * TILE;      // NS stages
constexpr int OFF_DST = OFF_DO + NS * TILE;    // 2 buffers x 2 chunks (dS^T, then dQ staging)
constexpr int OFF_VEC = OFF_DST + 4 * TILE;    // per stage: lse[128], delta[128]
constexpr int OFF_BAR = OFF_VEC + NS * 1024;
// no alignment slack: the dynamic shared window of a CTA without static shared memory
// starts 1024-byte aligned; the kernel checks this and reports a status code otherwise.
constexpr int SMEM_BYTES = OFF_BAR + 256;
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320, C_DQ = 384, C_PT = 448;
constexpr uint32_t IDESC_SS = make_idesc_bf16(128, 128, false, false);
constexpr uint32_t IDESC_GRAD = make_idesc_bf16(128, 64, false, true);  // A K-major, B MN-major
constexpr uint32_t IDESC_DQ = make_idesc_bf16(128, 64, true, true);     // both MN-major

// first query (within the sample) whose key limit exceeds key index k
__device__ __forceinline__ int first_query_seeing(const AttnArgs& a, int k) {
  if (a.causal == kCausalFrame) {
    const int ka = k + a.kv_pos_offset;
    return (ka / a.tpf) * a.tpf - a.q_pos_offset;
  }
  if (a.causal == kCausalToken) return k + a.kv_pos_offset - a.q_pos_offset;
  return 0;
}


// trace slot: [role (0 producer, 1 mma, 2 softmax, 3 dq)][event < 8][pair < 64]
#define DDB_TRACE(role, ev, j)                                                      \
  do {                                                                              \
    if (g.trace && blockIdx.x == g.trace_cta && (j) < 64)                           \
      g.trace[((role) * 8 + (ev)) * 64 + (j)] = clock64();                          \
  } while (0)

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const AttnBwdArgs g, int n_kvtiles,
                    int n_qtiles, int* status) {
  const AttnArgs& a = g.f;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;            // NS
  uint64_t* qd_empty = bars + 1 + NS;      // NS
  uint64_t* s_full = bars + 1 + 2 * NS;
  uint64_t* s_free = s_full + 1;
  uint64_t* ds_full = s_full + 2;   // 2 buffers: P^T (TMEM) and dS^T (smem) of the tile written
  uint64_t* ds_empty = s_full + 4;  // 2 buffers: all gradient MMAs of the tile done
  uint64_t* dq_full = s_full + 6;
  uint64_t* dq_free = s_full + 7;
  uint64_t* drain = s_full + 8;
  uint64_t* ds_free = s_full + 9;   // 2 buffers: dS^T buffer free again (dQ staging read)
  uint64_t* dq_staged = s_full + 11;  // the 4 dQ warps' rows are in shared memory
  uint64_t* pt_tfree = s_full + 12;   // P^T in TMEM consumed by the dV MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_staged + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if ((smem_u32(smem_raw) & 1023) != 0) {
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadArgument);
    return;
  }

  const int warp = warp_id();
  const int lane = lane_id();
  const int kt = blockIdx.x % n_kvtiles;
  const int bh = blockIdx.x / n_kvtiles;
  const int b = bh / a.H;
  const int h = bh % a.H;
  const int k0 = kt * 128;
  const bool sparse = g.kv_count != nullptr;
  const long list_idx = static_cast<long>(bh) * n_kvtiles + kt;
  int nq, qt_first = 0;
  if (sparse) {
    nq = min(g.kv_count[list_idx], g.max_q);
  } else {
    const int fq = max(0, first_query_seeing(a, k0));
    qt_first = fq / 128;
    nq = fq < a.Tq ? n_qtiles - qt_first : 0;
    if (k0 >= a.S) nq = 0;
  }
  // the unit's two 64-query blocks, qa | qb << 16; a list entry naming a block past the
  // queries is recorded in the status word and clamped (no access leaves the tensors)
  const int n_qblocks = (a.Tq + 63) / 64;
  auto qpair_of = [&](int j) -> int {
    if (sparse) {
      const int qp = g.kv_qtiles[list_idx * g.max_q + j];
      int qa = qp & 0xffff, qb = (qp >> 16) & 0xffff;
      if (qa >= n_qblocks || qb >= n_qblocks) {
        if (threadIdx.x == 0) record_bad_index(status, list_idx);
        qa = min(qa, n_qblocks - 1);
        qb = min(qb, n_qblocks - 1);
      }
      return qa | (qb << 16);
    }
    const int qt = qt_first + j;
    return (2 * qt) | ((2 * qt + 1) << 16);
  };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(&ds_full[0], 8);
    mbar_init(&ds_full[1], 8);
    mbar_init(&ds_free[0], 1);
    mbar_init(&ds_free[1], 1);
    mbar_init(dq_staged, 4);
    mbar_init(pt_tfree, 1);
    mbar_init(&ds_empty[0], 1);
    mbar_init(&ds_empty[1], 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      const int krow = static_cast<int>(b * a.kv_rows_per_b) + k0;
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      tma_load_2d(smem + OFF_K, &tmK, kv_full, a.k_col + h * 64, krow);
      tma_load_2d(smem + OFF_K + 8192, &tmK, kv_full, a.k_col + h * 64, krow + 64);
      tma_load_2d(smem + OFF_V, &tmV, kv_full, a.v_col + h * 64, krow);
      tma_load_2d(smem + OFF_V + 8192, &tmV, kv_full, a.v_col + h * 64, krow + 64);
      bool ok = true;
      int issued = 0;
      for (int j = 0; j < nq; ++j) {
        const int s = j % NS;
        if (!mbar_wait(&qd_empty[s], ((j / NS) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        DDB_TRACE(0, 0, j);
        const int qp = qpair_of(j);
        const int qa = qp & 0xffff, qb = (qp >> 16) & 0xffff;
        const int rowb = static_cast<int>(b * a.q_rows_per_b);
        uint8_t* sq = smem + OFF_Q + s * TILE;
        uint8_t* sd = smem + OFF_DO + s * TILE;
        uint8_t* sv = smem + OFF_VEC + s * 1024;
        // lse / delta of the two blocks: 64 floats (256 bytes, 16-byte aligned) each
        const long va = static_cast<long>(bh) * a.Tq + qa * 64;
        const long vb = static_cast<long>(bh) * a.Tq + qb * 64;
        mbar_arrive_expect_tx(&qd_full[s], 2 * TILE + 1024);
        tma_load_2d(sq, &tmQ, &qd_full[s], a.q_col + h * 64, rowb + qa * 64);
        tma_load_2d(sq + 8192, &tmQ, &qd_full[s], a.q_col + h * 64, rowb + qb * 64);
        tma_load_2d(sd, &tmDO, &qd_full[s], g.do_col + h * 64, rowb + qa * 64);
        tma_load_2d(sd + 8192, &tmDO, &qd_full[s], g.do_col + h * 64, rowb + qb * 64);
        bulk_load(sv, a.lse + va, 256, &qd_full[s]);
        bulk_load(sv + 256, a.lse + vb, 256, &qd_full[s]);
        bulk_load(sv + 512, g.delta + va, 256, &qd_full[s]);
        bulk_load(sv + 768, g.delta + vb, 256, &qd_full[s]);
        ++issued;
      }
      if (!ok) {
        if (status) atomicCAS(status, 0, kStatusTimeoutProducer);
        *abort_flag = 1;
      }
      long long t0 = clock64();
      while (!mbar_try_wait(kv_full, 0) && clock64() - t0 < kSpinLimitCycles / 8) {
      }
      for (int j = max(0, issued - NS); j < issued; ++j) {
        t0 = clock64();
        while (!mbar_try_wait(&qd_full[j % NS], (j / NS) & 1) &&
               clock64() - t0 < kSpinLimitCycles / 8) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(kv_full, 0, abort_flag);
      const uint32_t aK = smem_u32(smem + OFF_K);
      const uint32_t aV = smem_u32(smem + OFF_V);
      auto issue_grads = [&](int i) -> bool {
        const int pb = i & 1;  // dS^T buffer
        const uint32_t aDST = smem_u32(smem + OFF_DST + pb * 2 * TILE);
        if (!mbar_wait(&ds_full[pb], (i >> 1) & 1, abort_flag)) return false;
        DDB_TRACE(1, 3, i);
        if (i > 0 && !mbar_wait(dq_free, (i - 1) & 1, abort_flag)) return false;
        DDB_TRACE(1, 4, i);
        tc_fence_after();
        const int s = i % NS;
        const uint32_t aQ = smem_u32(smem + OFF_Q + s * TILE);
        const uint32_t aDO = smem_u32(smem + OFF_DO + s * TILE);
        if (!(g.debug_flags & 8)) {
          // dV += P^T dO: A = P^T straight from TMEM (keys = lanes, 16 queries per 8
          // columns), B = dO [queries][dh] read MN-major
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ts(tmem + C_DV, tmem + C_PT + kk * 8, make_sw128_desc(aDO + kk * 2048, 8192, 1024),
                        IDESC_GRAD, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(pt_tfree);
        if (!(g.debug_flags & 8)) {
          // dK += dS^T Q
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * TILE + (kk & 3) * 32;
            mma_bf16_ss(tmem + C_DK, make_sw128_desc(aDST + off, 16, 1024),
                        make_sw128_desc(aQ + kk * 2048, 8192, 1024), IDESC_GRAD,
                        (i > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&qd_empty[s]);  // Q and dO of this stage are no longer read
        if (!(g.debug_flags & 8))
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // K = 128 keys: dQ = dS K
          // A = dS^T tile read MN-major: queries contiguous in 64-wide chunks (LBO =
          // chunk distance), keys as rows; B = K [keys][dh] MN-major.
          mma_bf16_ss(tmem + C_DQ, make_sw128_desc(aDST + kk * 2048, TILE, 1024),
                      make_sw128_desc(aK + kk * 2048, 8192, 1024), IDESC_DQ, kk > 0 ? 1u : 0u);
        }
        mma_commit(&ds_empty[pb]);
        mma_commit(dq_full);
        DDB_TRACE(1, 5, i);
        return true;
      };
      for (int j = 0; j < nq && ok; ++j) {
        const int s = j % NS;
        if (!mbar_wait(&qd_full[s], (j / NS) & 1, abort_flag)) {
          ok = false;
          break;
        }
        DDB_TRACE(1, 0, j);
        if (j > 0 && !mbar_wait(s_free, (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        DDB_TRACE(1, 1, j);
        tc_fence_after();
        const uint32_t aQ = smem_u32(smem + OFF_Q + s * TILE);
        const uint32_t aDO = smem_u32(smem + OFF_DO + s * TILE);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16_ss(tmem + C_S, make_sw128_desc(aK + kk * 32, 16, 1024),
                      make_sw128_desc(aQ + kk * 32, 16, 1024), IDESC_SS, kk > 0 ? 1u : 0u);
          mma_bf16_ss(tmem + C_DP, make_sw128_desc(aV + kk * 32, 16, 1024),
                      make_sw128_desc(aDO + kk * 32, 16, 1024), IDESC_SS, kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full);
        DDB_TRACE(1, 2, j);
        if (j > 0 && !issue_grads(j - 1)) ok = false;
      }
      if (ok && nq > 0) ok = issue_grads(nq - 1);
      if (!ok) {
        if (status) atomicCAS(status, 0, kStatusTimeoutMma);
        *abort_flag = 1;
      }
      mma_commit(drain);
      long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kSpinLimitCycles / 8) {
      }
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax / dS warps
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // this warp's 64 query columns of the tile
    const int r = quad * 32 + lane;    // key row within the tile
    const int key = k0 + r;
    const int khalf = r >> 6;
    const float sl2 = a.scale * 1.4426950408889634f;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t swz = r & 7;
    // this key is visible to every query q >= qmin (masks are monotone in the query);
    // keys past the sequence end are visible to none
    const int qmin = (key < a.S) ? (sparse ? 0 : first_query_seeing(a, key)) : (1 << 30);
    bool ok = true;
    for (int j = 0; j < nq; ++j) {
      const int s = j % NS;
      const int pb = j & 1;
      // first query of the unit; only the dense (adjacent-block) masks read it
      const int q0 = (qpair_of(j) & 0xffff) * 64;
      const float* s_lse = reinterpret_cast<const float*>(smem + OFF_VEC + s * 1024);
      const float* s_delta = s_lse + 128;
      const int bits = sparse ? g.kv_qmask[list_idx * g.max_q + j] : 0xF;
      if (!mbar_wait(s_full, j & 1, abort_flag)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) DDB_TRACE(2, 0, j);
      if (!mbar_wait(&qd_full[s], (j / NS) & 1, abort_flag)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) DDB_TRACE(2, 1, j);
      tc_fence_after();
      const uint32_t ds_base = smem_u32(smem + OFF_DST + pb * 2 * TILE) + r * 128;
#pragma unroll 1
      for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
        uint32_t rs[32], rp[32];
        tmem_ld32(trow + C_S + c0, rs);
        tmem_ld32(trow + C_DP + c0, rp);
        tmem_wait_ld();
        if (warp == 2 && lane == 0 && j < 8) DDB_TRACE(2, 3 + ((c0 & 63) >> 5), j);
        if ((c0 & 63) == 32) {  // this warp's S^T / dP^T columns are all read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(s_free);
        }
        const bool half_on = (bits >> ((c0 >> 6) * 2 + khalf)) & 1;
        float p[32], ds[32];
        if (g.debug_flags & 2) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            p[c] = __uint_as_float(rs[c]);
            ds[c] = __uint_as_float(rp[c]);
          }
        } else if (__all_sync(0xffffffffu, half_on && q0 + c0 >= qmin)) {
          // every query of the chunk sees every key of the warp: no per-element mask;
          // dS = P * (scale * dP - scale * delta) as one FFMA and one FMUL
#pragma unroll
          for (int c4 = 0; c4 < 32; c4 += 4) {
            // lse / delta of 4 queries as broadcast 16-byte loads
            const float4 l4 = *reinterpret_cast<const float4*>(s_lse + c0 + c4);
            const float4 d4 = *reinterpret_cast<const float4*>(s_delta + c0 + c4);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
            const float nsd[4] = {-a.scale * d4.x, -a.scale * d4.y, -a.scale * d4.z, -a.scale * d4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c = c4 + e;
              const float pv = exp2f(__uint_as_float(rs[c]) * sl2 - lv[e]);
              p[c] = pv;
              ds[c] = pv * fmaf(a.scale, __uint_as_float(rp[c]), nsd[e]);
            }
          }
        } else {
#pragma unroll
          for (int c4 = 0; c4 < 32; c4 += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(s_lse + c0 + c4);
            const float4 d4 = *reinterpret_cast<const float4*>(s_delta + c0 + c4);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c = c4 + e;
              const bool vis = half_on && (q0 + c0 + c >= qmin);
              const float pv = vis ? exp2f(__uint_as_float(rs[c]) * sl2 - lv[e]) : 0.f;
              p[c] = pv;
              ds[c] = pv * (__uint_as_float(rp[c]) - dv[e]) * a.scale;
            }
          }
        }
        // P^T (bf16 pairs) -> TMEM for the dV MMA, once the previous tile's dV is done
        if ((c0 & 63) == 0 && j > 0) {
          if (!mbar_wait(pt_tfree, (j - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(p[2 * i], p[2 * i + 1]);
          tmem_st16(trow + C_PT + (c0 >> 1), pk);
        }
        // dS^T (bf16) -> shared memory for the dK and dQ MMAs, once the buffer's previous
        // contents (tile j - 2's dS^T, then its dQ staging) have been read
        if ((c0 & 63) == 0 && !mbar_wait(&ds_free[pb], ((j >> 1) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const int ch = c0 >> 6;
        if (!(g.debug_flags & 4))
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = ((c0 & 63) >> 3) + u4;
          const int c = u4 * 8;
          const uint32_t off = ch * TILE + ((u ^ swz) << 4);
          st_shared_v4(ds_base + off, pack_bf16(ds[c], ds[c + 1]),
                       pack_bf16(ds[c + 2], ds[c + 3]), pack_bf16(ds[c + 4], ds[c + 5]),
                       pack_bf16(ds[c + 6], ds[c + 7]));
        }
      }
      if (!ok) break;
      if (warp == 2 && lane == 0) DDB_TRACE(2, 2, j);
      tmem_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[pb]);
    }
    if (!ok) {
      if (lane == 0 && status) atomicCAS(status, 0, kStatusTimeoutEpilogue);
      *abort_flag = 1;
    }
    // final dK (warps of half 0) and dV (half 1), bf16, once the last gradient MMAs are done
    const uint32_t c_src = half == 0 ? C_DK : C_DV;
    const long grow = b * a.kv_rows_per_b + key;
    __nv_bfloat16* drow = half == 0
                              ? reinterpret_cast<__nv_bfloat16*>(g.dk) + grow * g.lddk + g.dk_col + h * 64
                              : reinterpret_cast<__nv_bfloat16*>(g.dv) + grow * g.lddv + g.dv_col + h * 64;
    if (ok && nq > 0 && mbar_wait(&ds_empty[(nq - 1) & 1], ((nq - 1) >> 1) & 1, abort_flag)) {
      tc_fence_after();
      uint32_t rv[2][32];
      tmem_ld32(trow + c_src, rv[0]);
      tmem_ld32(trow + c_src + 32, rv[1]);
      tmem_wait_ld();
      if (key < a.S) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int c = 0; c < 32; c += 8)
            st_global_v4(drow + hh * 32 + c,
                         pack_bf16(__uint_as_float(rv[hh][c]), __uint_as_float(rv[hh][c + 1])),
                         pack_bf16(__uint_as_float(rv[hh][c + 2]), __uint_as_float(rv[hh][c + 3])),
                         pack_bf16(__uint_as_float(rv[hh][c + 4]), __uint_as_float(rv[hh][c + 5])),
                         pack_bf16(__uint_as_float(rv[hh][c + 6]), __uint_as_float(rv[hh][c + 7])));
      }
    } else if (nq == 0 && key < a.S) {
      // keys nobody attends to get zero gradients
#pragma unroll
      for (int c = 0; c < 64; c += 8) st_global_v4(drow + c, 0, 0, 0, 0);
    }
  } else {
    // ------------------------------------------------------------ dQ warps
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the tile
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const bool issuer = warp == 10 && lane == 0;
    bool ok = true;
    for (int j = 0; j < nq; ++j) {
      const int pb = j & 1;
      if (!mbar_wait(dq_full, j & 1, abort_flag)) {
        ok = false;
        break;
      }
      if (issuer) DDB_TRACE(3, 0, j);
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld32(trow + C_DQ, v[0]);
      tmem_ld32(trow + C_DQ + 32, v[1]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      // The tile's dS^T buffer is free: every MMA that read it completed before dq_full.
      // Stage dQ there as two [128 rows][32 fp32] boxes, 128-byte swizzled (16-byte chunk
      // c of row r at chunk c ^ (r & 7)), then one thread adds both boxes into the
      // accumulator with TMA and frees the buffer once the reads are done.
      uint8_t* stage = smem + OFF_DST + pb * 2 * TILE;
      if (!(g.debug_flags & 1)) {
        const uint32_t sbase = smem_u32(stage) + r * 128;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            st_shared_v4(sbase + hh * TILE + ((c ^ (r & 7)) << 4), v[hh][4 * c], v[hh][4 * c + 1],
                         v[hh][4 * c + 2], v[hh][4 * c + 3]);
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_staged);
      bool staged = true;
      if (issuer) {
        staged = mbar_wait(dq_staged, j & 1, abort_flag);
        if (staged && !(g.debug_flags & 1)) {
          // rows 0-63 of the staged boxes belong to block qa, rows 64-127 to block qb;
          // a half whose mask is empty (odd last block) adds nothing
          const int qp = qpair_of(j);
          const int bits = sparse ? g.kv_qmask[list_idx * g.max_q + j] : 0xF;
          const int rowb = static_cast<int>(b * a.q_rows_per_b);
#pragma unroll
          for (int qh = 0; qh < 2; ++qh) {
            if (!((bits >> (2 * qh)) & 3)) continue;
            const int row0 = rowb + ((qp >> (16 * qh)) & 0xffff) * 64;
            tma_reduce_add_2d(&tmDQ, stage + qh * 8192, h * 64, row0);
            tma_reduce_add_2d(&tmDQ, stage + TILE + qh * 8192, h * 64 + 32, row0);
          }
          tma_store_commit();
          tma_store_wait_read();
        }
        mbar_arrive(&ds_free[pb]);
      }
      // warp-uniform exit (the next iteration's TMEM loads are warp-collective)
      if (warp == 10 && !__shfl_sync(0xffffffffu, staged, 0)) {
        ok = false;
        break;
      }
    }
    if (issuer) tma_store_wait_all();
    if (!ok) {
      if (lane == 0 && status) atomicCAS(status, 0, kStatusTimeoutEpilogue);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// delta[b,h,t] = sum over the head's 64 columns of dO * O (one warp per row)
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ o, long ldo, int o_col,
                             const __nv_bfloat16* __restrict__ dout, long lddo, int do_col,
                             float* __restrict__ delta, int B, int H, int Tq, long rows_per_b) {
  const int lane = threadIdx.x & 31;
  const long row = blockIdx.x * 8L + (threadIdx.x >> 5);
  if (row >= static_cast<long>(B) * Tq) return;
  const int b = static_cast<int>(row / Tq);
  const int t = static_cast<int>(row % Tq);
  const long grow = b * rows_per_b + t;
  const int chunks = H * 8;
  for (int base = 0; base < chunks; base += 32) {
    const int c = base + lane;
    float s = 0.f;
    if (c < chunks) {
      uint4 ov = ld_global_v4(o + grow * ldo + o_col + c * 8);
      uint4 dv = ld_global_v4(dout + grow * lddo + do_col + c * 8);
      uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
      uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 a = unpack_bf16(ow[j]);
        float2 d = unpack_bf16(dw[j]);
        s += a.x * d.x + a.y * d.y;
      }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if ((lane & 7) == 0 && c < chunks) {
      const int hh = c / 8;
      delta[(static_cast<long>(b) * H + hh) * Tq + t] = s;
    }
  }
}

// dq (bf16) = dq_acc, rotated back by the rotary table when given
__global__ void dq_finalize_kernel(const float* __restrict__ acc, long ld_acc,
                                   __nv_bfloat16* __restrict__ dq, long lddq, int dq_col, int rows,
                                   int H, const float2* __restrict__ tab, int rows_per_seq,
                                   int pos_offset) {
  const long idx = blockIdx.x * 256L + threadIdx.x;
  const int chunks = H * 8;
  if (idx >= static_cast<long>(rows) * chunks) return;
  const int row = static_cast<int>(idx / chunks);
  const int c = static_cast<int>(idx % chunks) * 8;
  const float* src = acc + row * ld_acc + c;
  float4 x0 = *reinterpret_cast<const float4*>(src);
  float4 x1 = *reinterpret_cast<const float4*>(src + 4);
  float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  if (tab) {
    const int pos = row % rows_per_seq + pos_offset;
    const float2* t = tab + static_cast<long>(pos) * 32 + (c % 64) / 2;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 cs = __ldg(t + j);
      const float a0 = v[2 * j], a1 = v[2 * j + 1];
      v[2 * j] = a0 * cs.x + a1 * cs.y;
      v[2 * j + 1] = -a0 * cs.y + a1 * cs.x;
    }
  }
  st_global_v4(dq + row * lddq + dq_col + c, pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]),
               pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
}

}  // namespace

namespace {
void launch_bwd(const AttnBwdArgs& g, int* status, cudaStream_t stream) {
  const AttnArgs& a = g.f;
  const long q_rows = a.q_rows_total > 0 ? a.q_rows_total : a.B * a.q_rows_per_b;
  const long kv_rows = a.kv_rows_total > 0 ? a.kv_rows_total : a.B * a.kv_rows_per_b;
  if (g.ld_dqacc % 4 != 0 || (reinterpret_cast<uintptr_t>(g.dq_acc) & 15) != 0)
    throw std::runtime_error("attn_bwd: the dQ accumulator needs 16-byte aligned rows");
  CUtensorMap tQ = make_tmap_2d(a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.ldq, q_rows, a.ldq * 2,
                                64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tK = make_tmap_2d(a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.ldk, kv_rows,
                                a.ldk * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tV = make_tmap_2d(a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.ldv, kv_rows,
                                a.ldv * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tDO = make_tmap_2d(g.dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.lddo, q_rows,
                                 g.lddo * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  // dQ reduce-add boxes: 32 fp32 columns x 64 rows (one query block)
  CUtensorMap tDQ = make_tmap_2d(g.dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.ld_dqacc, a.B * a.q_rows_per_b,
                                 g.ld_dqacc * 4, 32, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  const int n_kvtiles = (a.S + 127) / 128;
  const int n_qtiles = (a.Tq + 127) / 128;
  attn_bwd_kernel<<<a.B * a.H * n_kvtiles, kThreads, SMEM_BYTES, stream>>>(
      tQ, tK, tV, tDO, tDQ, g, n_kvtiles, n_qtiles, status);
  count_launch();
  check_cuda(cudaGetLastError(), "attn_bwd_kernel launch");
}
}  // namespace

void attn_bwd(const AttnBwdArgs& g, cudaStream_t stream) {
  const AttnArgs& a = g.f;
  if (a.B <= 0 || a.H <= 0 || a.S <= 0) return;
  if (a.Tq % 128 != 0) throw std::runtime_error("attn_bwd: queries per sample must be a multiple of 128");
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES),
               "cudaFuncSetAttribute(attn_bwd)");
    attr = true;
  }
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  launch_bwd(g, device_status(dev), stream);
}

void attn_bwd_delta(const void* o, long ldo, int o_col, const void* dout, long lddo, int do_col,
                    float* delta, int B, int H, int Tq, long rows_per_b, cudaStream_t s) {
  const long rows = static_cast<long>(B) * Tq;
  delta_kernel<<<static_cast<int>((rows + 7) / 8), 256, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(o), ldo, o_col,
      reinterpret_cast<const __nv_bfloat16*>(dout), lddo, do_col, delta, B, H, Tq, rows_per_b);
  count_launch();
}

void attn_dq_finalize(const float* dq_acc, long ld_acc, void* dq, long lddq, int dq_col, int rows,
                      int H, const float2* rope_tab, int rows_per_seq, int pos_offset,
                      cudaStream_t s) {
  const long n = static_cast<long>(rows) * H * 8;
  dq_finalize_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, s>>>(
      dq_acc, ld_acc, reinterpret_cast<__nv_bfloat16*>(dq), lddq, dq_col, rows, H, rope_tab,
      rows_per_seq, pos_offset);
  count_launch();
}

}  // namespace ddb

namespace ddb {

// The attn_bwd launch with the bounded-wait status word supplied by the caller instead
// of the per-device word (whose first use allocates it).
void attn_bwd_with_status(const AttnBwdArgs& g, int* status, cudaStream_t stream) {
  const AttnArgs& a = g.f;
  if (a.B <= 0 || a.H <= 0 || a.S <= 0) return;
  if (a.Tq % 128 != 0) throw std::runtime_error("attn_bwd: queries per sample must be a multiple of 128");
  check_cuda(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  SMEM_BYTES),
             "cudaFuncSetAttribute(attn_bwd)");
  launch_bwd(g, status, stream);
}

}  // namespace ddb
