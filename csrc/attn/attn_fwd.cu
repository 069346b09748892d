// tcgen05 flash-attention forward, d_head = 64, for sm_100a.
//
// One CTA = one (batch, head, 128-query tile). Roles (192 threads, 2 CTAs per SM):
//   warp 0     TMA: Q tile once (two 64-row boxes), then K and V tiles of 128 keys made of
//              two independent 64-key blocks (so SLA can pair any two selected blocks)
//              into 3-stage rings, K one tile ahead of V.
//   warp 1     TMEM owner + MMA issuer: S = Q K^T (M=128, N=128, K=64) into TMEM
//              columns [0,128), O += P V (M=128, N=64, K=128; A = P read from TMEM
//              columns [192,256)) into columns [128,192).
//   warps 2-5  softmax: one thread per query row reads its S row from TMEM, applies the
//              mask, keeps the running max / sum (log2 domain), rescales its O row in
//              TMEM when the max moves by more than 2^8, writes P (bf16 pairs) to TMEM,
//              and finally normalises O.
// The S MMA of tile j+1 overlaps the softmax of tile j; the second resident CTA of the
// SM (112 KB of shared memory each) overlaps the rest.
//
// Masks: frame-causal (all keys of frames <= the query's frame), token-causal, none;
// KV-cache attention via absolute query/key position offsets; block-sparse SLA via a
// per-tile list of 64-key block pairs with a 4-bit (query half x key half) mask.
//
// Split-KV: when batch x heads x query tiles would leave SMs idle (rollout at batch 1:
// 12 heads x 16 tiles of a 4-frame chunk against a 36-frame window), `kv_splits` CTAs
// share each query tile's key tiles; each writes its normalised fp32 O and its lse, and
// attn_split_merge_kernel combines them (O = sum 2^(lse_i - lse) O_i).
// Semantics oracle: layers/attention.py attention_reference (reference layers/mha.py:88-116
// with fp32 softmax), layers/sla.py sla_sparse_reference.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "attn.h"

namespace ddb {
namespace {

constexpr int kThreads = 192;
constexpr float kRescaleLog2 = 8.f;
constexpr int NS = 3;
constexpr int TILE_BYTES = 16384;  // 128 rows x 64 bf16
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;
constexpr int OFF_V = OFF_K + NS * TILE_BYTES;
constexpr int OFF_BAR = OFF_V + NS * TILE_BYTES;
// No alignment slack: the dynamic shared window of a CTA without static shared memory
// starts 1024-byte aligned (checked below). With the slack two CTAs (2 x (113 KB + 1 KB
// reserved)) would not fit the SM's 228 KB and only one would be resident.
constexpr int SMEM_BYTES = OFF_BAR + 256;
static_assert(2 * (SMEM_BYTES + 1024) <= 233472, "two CTAs per SM");
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t S_COL = 0;
constexpr uint32_t O_COL = 128;
constexpr uint32_t P_COL = 192;  // P as bf16 pairs: 128 keys in 64 columns
constexpr uint32_t IDESC_S = make_idesc_bf16(128, 128, false, false);
constexpr uint32_t IDESC_PV = make_idesc_bf16(128, 64, false, true);

// Optional clock64 trace of one CTA for pipeline studies: slot [role][event < 8][tile < 64]
// (role 0 producer, 1 MMA issuer, 2 softmax warp 2). Off unless attn_fwd_set_trace was given
// a buffer of 3 * 8 * 64 int64.
struct FwdTrace {
  long long* buf;
  int cta;
};
__device__ __forceinline__ void fwd_trace(const FwdTrace& t, int role, int ev, int j) {
  if (t.buf && blockIdx.x == t.cta && j < 64) t.buf[(role * 8 + ev) * 64 + j] = clock64();
}

__device__ __forceinline__ int row_limit(const AttnArgs& a, int q_local) {
  int lim = a.S;
  const int qa = a.q_pos_offset + q_local;
  if (a.causal == kCausalFrame) {
    lim = min(lim, (qa / a.tpf + 1) * a.tpf - a.kv_pos_offset);
  } else if (a.causal == kCausalToken) {
    lim = min(lim, qa + 1 - a.kv_pos_offset);
  }
  return max(lim, 0);
}


__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnArgs a, int n_qtiles,
                    int* status, const FwdTrace tr) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem_raw) & 1023) != 0) {
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadArgument);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  // K and V stages are released separately: K_j as soon as S_j is computed, V_j after PV_j,
  // so the K load of a later tile does not wait for the previous P V product.
  uint64_t* k_full = bars + 1;            // NS
  uint64_t* k_empty = bars + 1 + NS;      // NS
  uint64_t* v_full = bars + 1 + 2 * NS;   // NS
  uint64_t* v_empty = bars + 1 + 3 * NS;  // NS
  uint64_t* s_full = bars + 1 + 4 * NS;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = s_full + 3;
  uint64_t* drain = s_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int splits = a.kv_splits > 1 ? a.kv_splits : 1;
  const int split = blockIdx.x % splits;
  const int item = blockIdx.x / splits;
  const int qt = n_qtiles - 1 - (item % n_qtiles);  // heavy (late) tiles first
  const int bh = item / n_qtiles;
  const int b = bh / a.H;
  const int h = bh % a.H;
  const int q0 = qt * 128;
  const bool sparse = a.pair_count != nullptr;
  const long list_idx = static_cast<long>(bh) * n_qtiles + qt;
  int ntiles;
  int j0 = 0;  // first key tile of this CTA (split-KV: its share of the tile's key range)
  if (sparse) {
    ntiles = min(a.pair_count[list_idx], a.max_pairs);
  } else {
    const int lim = row_limit(a, min(q0 + 127, a.Tq - 1));
    ntiles = (lim + 127) / 128;
    if (splits > 1) {
      const int per = (ntiles + splits - 1) / splits;
      j0 = min(ntiles, split * per);
      ntiles = min(ntiles, j0 + per) - j0;
    }
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
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
  uint8_t* sQ = smem + OFF_Q;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int qrow = static_cast<int>(b * a.q_rows_per_b) + q0;
      const int qcol = a.q_col + h * 64;
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, qcol, qrow);
      tma_load_2d(sQ + 8192, &tmQ, q_full, qcol, qrow + 64);
      const int krow0 = static_cast<int>(b * a.kv_rows_per_b);
      int issued_k = 0, issued_v = 0;
      // one 128-key tile of K (is_v false) or V into its stage, once the stage is free
      auto load_tile = [&](int j, bool is_v) -> bool {
        const int s = j % NS;
        uint64_t* empty = is_v ? &v_empty[s] : &k_empty[s];
        uint64_t* full = is_v ? &v_full[s] : &k_full[s];
        if (!mbar_wait(empty, ((j / NS) & 1) ^ 1, abort_flag)) return false;
        fwd_trace(tr, 0, is_v ? 1 : 0, j);
        int b0 = 2 * (j0 + j), b1 = 2 * (j0 + j) + 1;
        if (sparse) {
          const int packed = a.pair_blocks[list_idx * a.max_pairs + j];
          b0 = packed & 0xffff;
          b1 = (packed >> 16) & 0xffff;
          const int nkb = (a.S + 63) / 64;  // a block past the keys: recorded, clamped
          if (b0 >= nkb || b1 >= nkb) {
            record_bad_index(status, list_idx);
            b0 = min(b0, nkb - 1);
            b1 = min(b1, nkb - 1);
          }
        }
        uint8_t* dst = smem + (is_v ? OFF_V : OFF_K) + s * TILE_BYTES;
        const CUtensorMap* tm = is_v ? &tmV : &tmK;
        const int col = (is_v ? a.v_col : a.k_col) + h * 64;
        mbar_arrive_expect_tx(full, TILE_BYTES);
        tma_load_2d(dst, tm, full, col, krow0 + b0 * 64);
        tma_load_2d(dst + 8192, tm, full, col, krow0 + b1 * 64);
        if (is_v) ++issued_v; else ++issued_k;
        return true;
      };
      // K runs one tile ahead of V: K_{j+1} needs only S_{j-1} done, V_j needs PV_{j-2}
      bool ok = ntiles == 0 || load_tile(0, false);
      for (int j = 0; j < ntiles && ok; ++j) {
        if (j + 1 < ntiles) ok = load_tile(j + 1, false);
        if (ok) ok = load_tile(j, true);
      }
      if (!ok) {
        if (status) atomicCAS(status, 0, kStatusTimeoutProducer);
        *abort_flag = 1;
      }
      // loads still in flight land before the CTA can retire (bounded)
      long long t0 = clock64();
      while (!mbar_try_wait(q_full, 0) && clock64() - t0 < kSpinLimitCycles / 8) {
      }
      for (int j = max(0, issued_k - NS); j < issued_k; ++j) {
        t0 = clock64();
        while (!mbar_try_wait(&k_full[j % NS], (j / NS) & 1) &&
               clock64() - t0 < kSpinLimitCycles / 8) {
        }
      }
      for (int j = max(0, issued_v - NS); j < issued_v; ++j) {
        t0 = clock64();
        while (!mbar_try_wait(&v_full[j % NS], (j / NS) & 1) &&
               clock64() - t0 < kSpinLimitCycles / 8) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag);
      const uint32_t aQ = smem_u32(sQ);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(p_full, i & 1, abort_flag)) return false;
        if (!mbar_wait(&v_full[i % NS], (i / NS) & 1, abort_flag)) return false;
        fwd_trace(tr, 1, 2, i);
        tc_fence_after();
        const uint32_t aV = smem_u32(smem + OFF_V + (i % NS) * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // A = P from TMEM: 16 keys per 8 columns
          const uint64_t db = make_sw128_desc(aV + kk * 2048, 8192, 1024);
          mma_bf16_ts(tmem + O_COL, tmem + P_COL + kk * 8, db, IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&v_empty[i % NS]);
        mma_commit(o_done);
        return true;
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        const int s = j % NS;
        if (!mbar_wait(&k_full[s], (j / NS) & 1, abort_flag)) {
          ok = false;
          break;
        }
        fwd_trace(tr, 1, 0, j);
        if (j > 0 && !mbar_wait(s_free, (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        fwd_trace(tr, 1, 1, j);
        tc_fence_after();
        const uint32_t aK = smem_u32(smem + OFF_K + s * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16_ss(tmem + S_COL, make_sw128_desc(aQ + kk * 32, 16, 1024),
                      make_sw128_desc(aK + kk * 32, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        mma_commit(&k_empty[s]);
        mma_commit(s_full);
        if (j > 0 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && ntiles > 0) ok = issue_pv(ntiles - 1);
      if (!ok) {
        if (status) atomicCAS(status, 0, kStatusTimeoutMma);
        *abort_flag = 1;
      }
      mma_commit(drain);
      long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kSpinLimitCycles / 8) {
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int q_local = q0 + r;
    const bool row_ok = q_local < a.Tq;
    const int lim = row_ok ? row_limit(a, q_local) : 0;
    const int qhalf = r >> 6;
    const float sl2 = a.scale * 1.4426950408889634f;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!mbar_wait(s_full, j & 1, abort_flag)) {
        ok = false;
        break;
      }
      const bool tw = warp == 2 && lane == 0;
      if (tw) fwd_trace(tr, 2, 0, j);
      tc_fence_after();
      float sf[128];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(trow + S_COL + 0, r0);
        tmem_ld32(trow + S_COL + 32, r1);
        tmem_ld32(trow + S_COL + 64, r2);
        tmem_ld32(trow + S_COL + 96, r3);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sf[c] = __uint_as_float(r0[c]);
          sf[32 + c] = __uint_as_float(r1[c]);
          sf[64 + c] = __uint_as_float(r2[c]);
          sf[96 + c] = __uint_as_float(r3[c]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      if (tw) fwd_trace(tr, 2, 1, j);
      if (sparse) {
        const int bits = a.pair_mask[list_idx * a.max_pairs + j];
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
          if (!((bits >> (qhalf * 2 + kh)) & 1)) {
#pragma unroll
            for (int c = 0; c < 64; ++c) sf[kh * 64 + c] = -INFINITY;
          }
        }
        if (!row_ok) {
#pragma unroll
          for (int c = 0; c < 128; ++c) sf[c] = -INFINITY;
        }
      } else if ((j0 + j) * 128 + 128 > lim) {
        const int base = (j0 + j) * 128;
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (base + c >= lim) sf[c] = -INFINITY;
      }
      // row max and row sum as 8 independent chains (a single 128-long chain of dependent
      // max/add instructions would be latency-bound with two softmax warps per SMSP)
      float mp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mp[i] = sf[i];
#pragma unroll
      for (int c = 8; c < 128; ++c) mp[c & 7] = fmaxf(mp[c & 7], sf[c]);
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      // The running max moves only when a score exceeds it by more than 2^8 (log2 units):
      // exponentials stay <= 256, and most tiles skip the O rescale in TMEM.
      const float mx2 = mx * sl2;
      float alpha = 1.f;
      if (mx2 > m + kRescaleLog2) {
        alpha = exp2f(m - mx2);
        m = mx2;
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      // exponentials packed to bf16 pairs as they are made (P lives in 64 registers)
      float sp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        const float p0 = exp2f(sf[c] * sl2 - m_use);
        const float p1 = exp2f(sf[c + 1] * sl2 - m_use);
        sp[c & 7] += p0;
        sp[(c + 1) & 7] += p1;
        pk[c >> 1] = pack_bf16(p0, p1);
      }
      const float sum = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      l = l * alpha + sum;
      if (tw) fwd_trace(tr, 2, 2, j);
      if (j > 0) {
        if (!mbar_wait(o_done, (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        if (tw) fwd_trace(tr, 2, 3, j);
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 64; c += 16) {
            uint32_t ov[16];
            tmem_ld16(trow + O_COL + c, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st16(trow + O_COL + c, ov);
          }
          tmem_wait_st();
        }
      }
      // P (bf16 pairs) -> TMEM columns [P_COL, P_COL + 64), the A operand of the PV MMA
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t q[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) q[i] = pk[ch * 16 + i];
        tmem_st16(trow + P_COL + ch * 16, q);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (tw) fwd_trace(tr, 2, 4, j);
    }
    if (!ok) {
      if (lane == 0 && status) atomicCAS(status, 0, kStatusTimeoutEpilogue);
      *abort_flag = 1;
    }
    float ov[64];
    if (ok && ntiles > 0 && mbar_wait(o_done, (ntiles - 1) & 1, abort_flag)) {
      tc_fence_after();
      uint32_t o0[32], o1[32];
      tmem_ld32(trow + O_COL, o0);
      tmem_ld32(trow + O_COL + 32, o1);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        ov[c] = __uint_as_float(o0[c]);
        ov[32 + c] = __uint_as_float(o1[c]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < 64; ++c) ov[c] = 0.f;
    }
    if (row_ok && splits > 1) {
      // this split's normalised O (fp32) and lse; attn_split_merge_kernel combines them
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const long prow = static_cast<long>(split) * a.B * a.Tq + static_cast<long>(b) * a.Tq + q_local;
      float* op = a.o_part + prow * (a.H * 64) + h * 64;
#pragma unroll
      for (int c = 0; c < 64; c += 4)
        st_global_v4(op + c, __float_as_uint(ov[c] * inv), __float_as_uint(ov[c + 1] * inv),
                     __float_as_uint(ov[c + 2] * inv), __float_as_uint(ov[c + 3] * inv));
      a.lse_part[(static_cast<long>(split) * a.B * a.H + bh) * a.Tq + q_local] =
          l > 0.f ? m + __log2f(l) : -INFINITY;
    } else if (row_ok) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.o) +
                            (b * a.q_rows_per_b + q_local) * a.ldo + a.o_col + h * 64;
#pragma unroll
      for (int c = 0; c < 64; c += 8)
        st_global_v4(orow + c, pack_bf16(ov[c] * inv, ov[c + 1] * inv),
                     pack_bf16(ov[c + 2] * inv, ov[c + 3] * inv),
                     pack_bf16(ov[c + 4] * inv, ov[c + 5] * inv),
                     pack_bf16(ov[c + 6] * inv, ov[c + 7] * inv));
      if (a.lse) a.lse[static_cast<long>(bh) * a.Tq + q_local] = l > 0.f ? m + __log2f(l) : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

FwdTrace g_fwd_trace{nullptr, 0};

// Split-KV merge: one warp per (query row, head); lane i holds columns 2i, 2i+1.
__global__ void __launch_bounds__(256) attn_split_merge_kernel(const AttnArgs a) {
  const int lane = threadIdx.x & 31;
  const long item = blockIdx.x * 8L + (threadIdx.x >> 5);
  const long rows = static_cast<long>(a.B) * a.Tq;
  if (item >= rows * a.H) return;
  const int h = static_cast<int>(item % a.H);
  const long r = item / a.H;  // b * Tq + q
  const int b = static_cast<int>(r / a.Tq);
  const int q = static_cast<int>(r % a.Tq);
  const long bh = static_cast<long>(b) * a.H + h;
  const int splits = a.kv_splits;
  float mx = -INFINITY;
  for (int i = 0; i < splits; ++i)
    mx = fmaxf(mx, a.lse_part[(static_cast<long>(i) * a.B * a.H + bh) * a.Tq + q]);
  float o0 = 0.f, o1 = 0.f, wsum = 0.f;
  if (mx != -INFINITY) {
    for (int i = 0; i < splits; ++i) {
      const float li = a.lse_part[(static_cast<long>(i) * a.B * a.H + bh) * a.Tq + q];
      const float wi = exp2f(li - mx);  // 0 for an empty split (lse = -inf)
      const float2 v = *reinterpret_cast<const float2*>(
          a.o_part + (static_cast<long>(i) * rows + r) * (a.H * 64) + h * 64 + 2 * lane);
      o0 += wi * v.x;
      o1 += wi * v.y;
      wsum += wi;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.o) +
                        (b * a.q_rows_per_b + q) * a.ldo + a.o_col + h * 64;
  *reinterpret_cast<uint32_t*>(orow + 2 * lane) = pack_bf16(o0 * inv, o1 * inv);
  if (a.lse && lane == 0) a.lse[bh * a.Tq + q] = wsum > 0.f ? mx + __log2f(wsum) : -INFINITY;
}

}  // namespace

int attn_fwd_kv_splits(const AttnArgs& a) {
  if (a.pair_count != nullptr || a.B <= 0 || a.H <= 0 || a.Tq <= 0) return 1;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const long slots = 2L * num_sms(dev);  // two forward CTAs per SM
  const long ctas = static_cast<long>(a.B) * a.H * ((a.Tq + 127) / 128);
  if (ctas >= slots) return 1;
  // key tiles of the last (longest) query tile; a split keeps at least 4 of them
  int lim = a.S;
  const int qa = a.q_pos_offset + a.Tq - 1;
  if (a.causal == kCausalFrame) lim = std::min(lim, (qa / a.tpf + 1) * a.tpf - a.kv_pos_offset);
  else if (a.causal == kCausalToken) lim = std::min(lim, qa + 1 - a.kv_pos_offset);
  const int tiles = (std::max(lim, 0) + 127) / 128;
  // time ~ waves x key tiles per split: the fewest splits with the smallest estimate
  int best = 1;
  double best_t = 1.0;
  for (int s = 2; s <= 8 && tiles / s >= 4; ++s) {
    const double t = static_cast<double>((ctas * s + slots - 1) / slots) / s;
    if (t < best_t - 1e-9) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

void attn_fwd_split_scratch(const AttnArgs& a, int splits, long* o_part_elems, long* lse_part_elems) {
  *o_part_elems = static_cast<long>(splits) * a.B * a.Tq * a.H * 64;
  *lse_part_elems = static_cast<long>(splits) * a.B * a.H * a.Tq;
}

void attn_fwd_set_trace(long long* buf, int cta) { g_fwd_trace = FwdTrace{buf, cta}; }

void attn_fwd(const AttnArgs& a, cudaStream_t stream) {
  if (a.B <= 0 || a.H <= 0 || a.Tq <= 0) return;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES),
               "cudaFuncSetAttribute(attn_fwd)");
    attr = true;
  }
  const long q_rows = a.q_rows_total > 0 ? a.q_rows_total : a.B * a.q_rows_per_b;
  const long kv_rows = a.kv_rows_total > 0 ? a.kv_rows_total : a.B * a.kv_rows_per_b;
  CUtensorMap tQ = make_tmap_2d(a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.ldq, q_rows, a.ldq * 2,
                                64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tK = make_tmap_2d(a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.ldk, kv_rows,
                                a.ldk * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tV = make_tmap_2d(a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.ldv, kv_rows,
                                a.ldv * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  const int n_qtiles = (a.Tq + 127) / 128;
  const int splits = a.kv_splits > 1 ? a.kv_splits : 1;
  if (splits > 1 && (a.pair_count != nullptr || a.o_part == nullptr || a.lse_part == nullptr))
    throw std::runtime_error("attn_fwd: split-KV needs dense/causal mode and both scratch buffers");
  const int grid = a.B * a.H * n_qtiles * splits;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  attn_fwd_kernel<<<grid, kThreads, SMEM_BYTES, stream>>>(tQ, tK, tV, a, n_qtiles,
                                                          device_status(dev), g_fwd_trace);
  count_launch();
  check_cuda(cudaGetLastError(), "attn_fwd_kernel launch");
  if (splits > 1) {
    const long items = static_cast<long>(a.B) * a.Tq * a.H;
    attn_split_merge_kernel<<<static_cast<int>((items + 7) / 8), 256, 0, stream>>>(a);
    count_launch();
    check_cuda(cudaGetLastError(), "attn_split_merge_kernel launch");
  }
}

}  // namespace ddb
