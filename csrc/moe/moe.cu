// DeepSeek-style MoE FFN support kernels for sm_100a (routing, permutation, combine).
//
// The FFN of a block runs as grouped tcgen05 GEMMs (csrc/gemm, grouped scheduling) over a
// permuted token buffer in which every expert owns a segment padded to 128 rows. Shared
// experts are the last `ns` "experts"; every token is routed to them with the softmax
// shared-gate weight, so they go through exactly the same dispatch / GEMM / combine path.
//
//   moe_route     per token: p = softmax(logits[:E] + bias); top-k; renormalise;
//                 shared gates g = softmax(logits[E:E+ns]); expert counts and the per-
//                 expert probability sums (aux load-balance loss) by block reduction
//   moe_plan      per expert: padded segment starts, row-tile tables for the grouped GEMM,
//                 k-block ranges for the grouped weight gradients
//   moe_dispatch  copies each (token, route) row into its expert segment; zeroes padding
//   moe_combine   out[t] = residual[t] + sum_j w[t,j] * y[slot(t,j)]
//   moe_combine_bwd  dy[slot(t,j)] = w[t,j] dout[t];  dw[t,j] = dout[t] . y[slot(t,j)]
//   moe_unpermute dx[t] = sum_j dx_perm[slot(t,j)]
// Under expert parallelism the routed rows (j < k) and the shared-expert rows (j >= k) live
// in different buffers (a compact send / return buffer in peer-mapped memory, and the
// local shared-expert segments); every kernel then takes the second buffer for j >= k.
// Semantics: reference layers/moe.py:73-228 (Router), :231-424 (MoEFFN).
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "moe.h"

namespace ddb {
namespace {

constexpr int kMaxE = 256;

// One warp per token. logits row: [E routed | ns shared | pad].
__global__ void __launch_bounds__(256) moe_route_kernel(MoeRouteArgs a) {
  __shared__ float s_psum[kMaxE];
  __shared__ int s_cnt[kMaxE];
  for (int e = threadIdx.x; e < a.E; e += 256) {
    s_psum[e] = 0.f;
    s_cnt[e] = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int tok = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (tok < a.N) {
    const float* lg = a.logits + static_cast<long>(tok) * a.ld_logits;
    constexpr int PER = kMaxE / 32;
    float v[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      v[i] = e < a.E ? lg[e] + (a.bias ? a.bias[e] : 0.f) : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      v[i] = (i * 32 + lane) < a.E ? __expf(v[i] - mx) : 0.f;
      sum += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      v[i] *= inv;
      const int e = i * 32 + lane;
      if (e < a.E) {
        if (a.probs) a.probs[static_cast<long>(tok) * a.E + e] = v[i];
        atomicAdd(&s_psum[e], v[i]);
      }
    }
    // top-k (ties -> lower expert index)
    float cand[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) cand[i] = ((i * 32 + lane) < a.E) ? v[i] : -1.f;
    float wsum = 0.f;
    for (int r = 0; r < a.k; ++r) {
      float best = -1.f;
      int bi = kMaxE;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (cand[i] > best) {
          best = cand[i];
          bi = i * 32 + lane;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
      }
      if ((bi & 31) == lane) cand[bi >> 5] = -1.f;
      wsum += best;
      if (lane == 0) {
        a.topk_idx[static_cast<long>(tok) * a.k + r] = bi;
        a.topk_w[static_cast<long>(tok) * a.k + r] = best;
        atomicAdd(&s_cnt[bi], 1);
      }
    }
    if (lane < a.k) {
      const long o = static_cast<long>(tok) * a.k + lane;
      a.topk_w[o] = a.topk_w[o] / (wsum + 1e-8f);
    }
    // shared-expert gates: softmax over the ns shared logits
    if (a.ns > 0 && lane == 0) {
      float m2 = -INFINITY;
      for (int s = 0; s < a.ns; ++s) m2 = fmaxf(m2, lg[a.E + s]);
      float z = 0.f;
      for (int s = 0; s < a.ns; ++s) z += __expf(lg[a.E + s] - m2);
      for (int s = 0; s < a.ns; ++s)
        a.shared_w[static_cast<long>(tok) * a.ns + s] = __expf(lg[a.E + s] - m2) / z;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += 256) {
    if (s_psum[e] != 0.f) atomicAdd(a.psum + e, s_psum[e]);
    if (s_cnt[e]) atomicAdd(a.counts + e, s_cnt[e]);
  }
}

// Deterministic mode: psum[e] = sum over tokens of probs[t, e] in a fixed order (each
// thread a fixed stride of rows, then a fixed-shape tree), replacing the route kernel's
// float atomics whose rounding depends on arrival order.
__global__ void __launch_bounds__(256) moe_psum_fixed_kernel(const float* __restrict__ probs, int N,
                                                             int E, float* __restrict__ psum) {
  __shared__ float part[256];
  const int e = blockIdx.x;
  float acc = 0.f;
  for (int t = threadIdx.x; t < N; t += 256) acc += probs[static_cast<long>(t) * E + e];
  part[threadIdx.x] = acc;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) psum[e] = part[0];
}

// One block: segment layout for E routed + ns shared experts.
__global__ void moe_plan_kernel(const int* __restrict__ counts, int E, int ns, int N,
                                int* __restrict__ seg_start, int* __restrict__ seg_count,
                                int* __restrict__ tile_expert, int* __restrict__ tile_row,
                                int* __restrict__ total_mtiles, int* __restrict__ kstart,
                                int* __restrict__ kend, int* __restrict__ cursor, int max_mtiles) {
  if (threadIdx.x != 0) return;
  int row = 0, nt = 0;
  for (int e = 0; e < E + ns; ++e) {
    const int c = e < E ? counts[e] : N;
    seg_start[e] = row;
    seg_count[e] = c;
    cursor[e] = 0;
    kstart[e] = row / 64;
    kend[e] = (row + ((c + 63) / 64) * 64) / 64;
    const int tiles = (c + 127) / 128;
    for (int i = 0; i < tiles && nt < max_mtiles; ++i, ++nt) {
      tile_expert[nt] = e;
      tile_row[nt] = row + i * 128;
    }
    row += tiles * 128;
  }
  *total_mtiles = nt;
}

// Deterministic slot assignment (one block per routed expert): the routes to expert e
// get the rows of e's segment in (token, route) order, a stable counting sort, so the
// permuted layout and every reduction over it repeat bit for bit.
__global__ void __launch_bounds__(1024) moe_slots_stable_kernel(const int* __restrict__ topk_idx,
                                                                long NK, int k, int R,
                                                                const int* __restrict__ seg_start,
                                                                int* __restrict__ slot_of) {
  __shared__ int warp_cnt[32];
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int base = seg_start[e];
  for (long c0 = 0; c0 < NK; c0 += blockDim.x) {
    const long i = c0 + threadIdx.x;
    const bool mine = i < NK && topk_idx[i] == e;
    const unsigned m = __ballot_sync(0xffffffffu, mine);
    if (lane == 0) warp_cnt[w] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int q = 0; q < nw; ++q) {
      const int c = warp_cnt[q];
      before += q < w ? c : 0;
      total += c;
    }
    if (mine) {
      const long t = i / k, j = i % k;
      slot_of[t * R + j] = base + before + __popc(m & ((1u << lane) - 1u));
    }
    base += total;
    __syncthreads();
  }
}

// One warp per (token, route). Routes j < k are the top-k experts, j >= k the shared ones.
// fixed_slots: routed slots already assigned (deterministic mode); check: bounds mode.
__global__ void __launch_bounds__(256) moe_dispatch_kernel(
    const __nv_bfloat16* __restrict__ x, long ldx, int N, int d, int k, int ns, int E,
    const int* __restrict__ topk_idx, const int* __restrict__ seg_start, int* __restrict__ cursor,
    __nv_bfloat16* __restrict__ xp, long ldp, int* __restrict__ slot_of, __nv_bfloat16* __restrict__ xp2,
    long ldp2, int fixed_slots, long xp_rows, long xp2_rows, int check, int* status) {
  const int lane = threadIdx.x & 31;
  const long wi = blockIdx.x * 8L + (threadIdx.x >> 5);
  const int R = k + ns;
  if (wi >= static_cast<long>(N) * R) return;
  const int t = static_cast<int>(wi / R), j = static_cast<int>(wi % R);
  int slot = 0;
  if (lane == 0) {
    if (j < k) {
      const int e = topk_idx[static_cast<long>(t) * k + j];
      if (check && (e < 0 || e >= E)) {
        record_bad_index(status, e);
        slot = -1;
      } else {
        slot = fixed_slots ? slot_of[wi] : seg_start[e] + atomicAdd(cursor + e, 1);
      }
    } else {
      slot = seg_start[E + (j - k)] + t;
    }
    const bool second = xp2 != nullptr && j >= k;
    if (check && slot >= 0 && slot >= (second ? xp2_rows : xp_rows)) {
      record_bad_index(status, slot);
      slot = -1;
    }
    slot_of[wi] = slot;
  }
  slot = __shfl_sync(0xffffffffu, slot, 0);
  if (slot < 0) return;  // bounds mode: the bad route is skipped
  const __nv_bfloat16* src = x + static_cast<long>(t) * ldx;
  __nv_bfloat16* dst = (xp2 != nullptr && j >= k) ? xp2 + static_cast<long>(slot) * ldp2
                                                  : xp + static_cast<long>(slot) * ldp;
  for (int c = lane * 8; c < d; c += 256) {
    const uint4 v = ld_global_v4(src + c);
    st_global_v4(dst + c, v.x, v.y, v.z, v.w);
  }
}

// zero the padding rows of every expert segment (one block per expert)
__global__ void moe_zero_pad_kernel(const int* __restrict__ seg_start,
                                    const int* __restrict__ seg_count, __nv_bfloat16* xp, long ldp,
                                    int d) {
  const int e = blockIdx.x;
  const int c = seg_count[e];
  const int r0 = seg_start[e] + c;
  const int r1 = seg_start[e] + ((c + 127) / 128) * 128;
  for (int r = r0; r < r1; ++r)
    for (int col = threadIdx.x * 8; col < d; col += blockDim.x * 8)
      st_global_v4(xp + static_cast<long>(r) * ldp + col, 0, 0, 0, 0);
}

__device__ __forceinline__ float route_w(const MoeCombineArgs& a, int t, int j) {
  return j < a.k ? a.topk_w[static_cast<long>(t) * a.k + j]
                 : a.shared_w[static_cast<long>(t) * a.ns + (j - a.k)];
}

// bounds mode: slot inside the buffer its route reads (a bad one is recorded and skipped)
__device__ __forceinline__ bool slot_ok(const MoeCombineArgs& a, int j, int slot) {
  const long rows = (a.y2 != nullptr && j >= a.k) ? a.y2_rows : a.y_rows;
  if (slot >= 0 && slot < rows) return true;
  record_bad_index(a.status, slot);
  return false;
}

__device__ __forceinline__ const __nv_bfloat16* y_row(const MoeCombineArgs& a, int j, int slot) {
  return (a.y2 != nullptr && j >= a.k) ? a.y2 + static_cast<long>(slot) * a.ld_y2
                                       : a.y + static_cast<long>(slot) * a.ld_y;
}

// one warp per token; d <= 2048
__global__ void __launch_bounds__(256) moe_combine_kernel(MoeCombineArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= a.N) return;
  const int R = a.k + a.ns;
  for (int c = lane * 8; c < a.d; c += 256) {
    float acc[8];
    if (a.residual) {
      const uint4 r = ld_global_v4(a.residual + static_cast<long>(t) * a.ld_res + c);
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16(rw[q]);
        acc[2 * q] = f.x;
        acc[2 * q + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    }
    for (int j = 0; j < R; ++j) {
      const float w = route_w(a, t, j);
      const int slot = a.slot_of[static_cast<long>(t) * R + j];
      if (a.check && !slot_ok(a, j, slot)) continue;
      const uint4 y = ld_global_v4(y_row(a, j, slot) + c);
      const uint32_t yw[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16(yw[q]);
        acc[2 * q] += w * f.x;
        acc[2 * q + 1] += w * f.y;
      }
    }
    st_global_v4(a.out + static_cast<long>(t) * a.ld_out + c, pack_bf16(acc[0], acc[1]),
                 pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]), pack_bf16(acc[6], acc[7]));
  }
}

// one warp per (token, route)
__global__ void __launch_bounds__(256) moe_combine_bwd_kernel(MoeCombineArgs a,
                                                              const __nv_bfloat16* __restrict__ dout,
                                                              long ld_dout,
                                                              __nv_bfloat16* __restrict__ dy,
                                                              float* __restrict__ dw,
                                                              __nv_bfloat16* __restrict__ dy2) {
  const int lane = threadIdx.x & 31;
  const long wi = blockIdx.x * 8L + (threadIdx.x >> 5);
  const int R = a.k + a.ns;
  if (wi >= static_cast<long>(a.N) * R) return;
  const int t = static_cast<int>(wi / R), j = static_cast<int>(wi % R);
  const float w = route_w(a, t, j);
  const int slot = a.slot_of[wi];
  if (a.check && !slot_ok(a, j, slot)) {
    if (lane == 0) dw[wi] = 0.f;
    return;
  }
  const bool second = a.y2 != nullptr && j >= a.k;
  __nv_bfloat16* dst = second ? dy2 + static_cast<long>(slot) * a.ld_y2 : dy + static_cast<long>(slot) * a.ld_y;
  const __nv_bfloat16* yr = y_row(a, j, slot);
  float dot = 0.f;
  for (int c = lane * 8; c < a.d; c += 256) {
    const uint4 g = ld_global_v4(dout + static_cast<long>(t) * ld_dout + c);
    const uint4 y = ld_global_v4(yr + c);
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, yw[4] = {y.x, y.y, y.z, y.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 fg = unpack_bf16(gw[q]), fy = unpack_bf16(yw[q]);
      dot += fg.x * fy.x + fg.y * fy.y;
      o[q] = pack_bf16(w * fg.x, w * fg.y);
    }
    st_global_v4(dst + c, o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
  if (lane == 0) dw[wi] = dot;
}

// one warp per token: dx[t] = sum_j dxp[slot(t, j)]
__global__ void __launch_bounds__(256) moe_unpermute_kernel(const __nv_bfloat16* __restrict__ dxp,
                                                            long ldp, const int* __restrict__ slot_of,
                                                            int N, int R, int d,
                                                            __nv_bfloat16* __restrict__ dx, long ldx,
                                                            int k, const __nv_bfloat16* __restrict__ dxp2,
                                                            long ldp2, long rows, long rows2, int check,
                                                            int* status) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= N) return;
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < R; ++j) {
      const int slot = slot_of[static_cast<long>(t) * R + j];
      if (check && (slot < 0 || slot >= ((dxp2 != nullptr && j >= k) ? rows2 : rows))) {
        record_bad_index(status, slot);
        continue;
      }
      const __nv_bfloat16* row = (dxp2 != nullptr && j >= k) ? dxp2 + static_cast<long>(slot) * ldp2
                                                             : dxp + static_cast<long>(slot) * ldp;
      const uint4 v = ld_global_v4(row + c);
      const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16(vw[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    st_global_v4(dx + static_cast<long>(t) * ldx + c, pack_bf16(acc[0], acc[1]),
                 pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]), pack_bf16(acc[6], acc[7]));
  }
}

}  // namespace

void moe_route(const MoeRouteArgs& a, cudaStream_t s) {
  if (a.E > kMaxE || a.k > 32 || a.k > a.E) throw std::runtime_error("moe_route: E <= 256, k <= 32");
  moe_route_kernel<<<(a.N + 7) / 8, 256, 0, s>>>(a);
  count_launch();
  if (deterministic() && a.probs != nullptr && a.psum != nullptr) {
    moe_psum_fixed_kernel<<<a.E, 256, 0, s>>>(a.probs, a.N, a.E, a.psum);
    count_launch();
  }
}

void moe_plan(const int* counts, int E, int ns, int N, int* seg_start, int* seg_count,
              int* tile_expert, int* tile_row, int* total_mtiles, int* kstart, int* kend,
              int* cursor, int max_mtiles, cudaStream_t s) {
  moe_plan_kernel<<<1, 32, 0, s>>>(counts, E, ns, N, seg_start, seg_count, tile_expert, tile_row,
                                   total_mtiles, kstart, kend, cursor, max_mtiles);
  count_launch();
}

void moe_dispatch(const __nv_bfloat16* x, long ldx, int N, int d, int k, int ns, int E,
                  const int* topk_idx, const int* seg_start, const int* seg_count, int* cursor,
                  __nv_bfloat16* xp, long ldp, int* slot_of, cudaStream_t s, __nv_bfloat16* xp2,
                  long ldp2, bool zero_routed_pad, long xp_rows, long xp2_rows) {
  if (d % 8 != 0) throw std::runtime_error("moe_dispatch: d % 8");
  const long rows = static_cast<long>(N) * (k + ns);
  const bool det = deterministic() && k > 0 && E > 0;
  const bool check = check_bounds();
  if (check && (xp_rows <= 0 || (xp2 != nullptr && xp2_rows <= 0)))
    throw std::runtime_error("moe_dispatch: bounds checking needs the buffer extents");
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (det) {  // routed slots by a stable counting sort, then the copies
    moe_slots_stable_kernel<<<E, 1024, 0, s>>>(topk_idx, static_cast<long>(N) * k, k, k + ns,
                                               seg_start, slot_of);
    count_launch();
  }
  moe_dispatch_kernel<<<static_cast<int>((rows + 7) / 8), 256, 0, s>>>(
      x, ldx, N, d, k, ns, E, topk_idx, seg_start, cursor, xp, ldp, slot_of, xp2, ldp2, det ? 1 : 0,
      xp_rows, xp2_rows, check ? 1 : 0, check ? device_status(dev) : nullptr);
  count_launch();
  if (xp2 == nullptr && zero_routed_pad) {
    moe_zero_pad(seg_start, seg_count, E + ns, xp, ldp, d, s);
  } else {
    // compact routed rows (zero_routed_pad false) have no padding to clear
    if (zero_routed_pad) moe_zero_pad(seg_start, seg_count, E, xp, ldp, d, s);
    if (ns) moe_zero_pad(seg_start + E, seg_count + E, ns, xp2 ? xp2 : xp, xp2 ? ldp2 : ldp, d, s);
  }
}

void moe_zero_pad(const int* seg_start, const int* seg_count, int nseg, __nv_bfloat16* xp, long ldp,
                  int d, cudaStream_t s) {
  if (nseg <= 0) return;
  moe_zero_pad_kernel<<<nseg, 128, 0, s>>>(seg_start, seg_count, xp, ldp, d);
  count_launch();
}

namespace {
MoeCombineArgs with_checks(const MoeCombineArgs& in) {
  MoeCombineArgs a = in;
  a.check = check_bounds() ? 1 : 0;
  if (a.check) {
    if (a.y_rows <= 0 || (a.y2 != nullptr && a.y2_rows <= 0))
      throw std::runtime_error("moe_combine: bounds checking needs the buffer extents");
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    a.status = device_status(dev);
  }
  return a;
}
}  // namespace

void moe_combine(const MoeCombineArgs& a_in, cudaStream_t s) {
  const MoeCombineArgs a = with_checks(a_in);
  moe_combine_kernel<<<(a.N + 7) / 8, 256, 0, s>>>(a);
  count_launch();
}

void moe_combine_bwd(const MoeCombineArgs& a_in, const __nv_bfloat16* dout, long ld_dout,
                     __nv_bfloat16* dy, float* dw, cudaStream_t s, __nv_bfloat16* dy2) {
  const MoeCombineArgs a = with_checks(a_in);
  const long rows = static_cast<long>(a.N) * (a.k + a.ns);
  if ((a.y2 == nullptr) != (dy2 == nullptr)) throw std::runtime_error("moe_combine_bwd: y2 / dy2");
  moe_combine_bwd_kernel<<<static_cast<int>((rows + 7) / 8), 256, 0, s>>>(a, dout, ld_dout, dy, dw, dy2);
  count_launch();
}

void moe_unpermute(const __nv_bfloat16* dxp, long ldp, const int* slot_of, int N, int R, int d,
                   __nv_bfloat16* dx, long ldx, cudaStream_t s, int k, const __nv_bfloat16* dxp2,
                   long ldp2, long rows, long rows2) {
  const bool check = check_bounds();
  if (check && (rows <= 0 || (dxp2 != nullptr && rows2 <= 0)))
    throw std::runtime_error("moe_unpermute: bounds checking needs the buffer extents");
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  moe_unpermute_kernel<<<(N + 7) / 8, 256, 0, s>>>(dxp, ldp, slot_of, N, R, d, dx, ldx, k, dxp2, ldp2,
                                                   rows, rows2, check ? 1 : 0,
                                                   check ? device_status(dev) : nullptr);
  count_launch();
}

}  // namespace ddb
