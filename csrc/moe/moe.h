// MoE routing / permutation / combine kernels (see moe.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ddb {

struct MoeRouteArgs {
  const float* logits = nullptr;  // [N, ld_logits]: E routed, then ns shared-gate logits
  long ld_logits = 0;
  const float* bias = nullptr;    // [E] load-balancing bias (may be null)
  int N = 0, E = 0, k = 0, ns = 0;
  int* topk_idx = nullptr;        // [N, k]
  float* topk_w = nullptr;        // [N, k] renormalised
  float* shared_w = nullptr;      // [N, ns]
  float* probs = nullptr;         // [N, E] (optional, for the router backward)
  int* counts = nullptr;          // [E] += tokens per expert
  float* psum = nullptr;          // [E] += sum of probabilities
};

struct MoeCombineArgs {
  int N = 0, d = 0, k = 0, ns = 0;
  const float* topk_w = nullptr;
  const float* shared_w = nullptr;
  const int* slot_of = nullptr;        // [N, k + ns]
  const __nv_bfloat16* y = nullptr;    // permuted expert outputs
  long ld_y = 0;
  const __nv_bfloat16* y2 = nullptr;   // shared-expert rows when they live apart (EP); else null
  long ld_y2 = 0;
  const __nv_bfloat16* residual = nullptr;
  long ld_res = 0;
  __nv_bfloat16* out = nullptr;
  long ld_out = 0;
  long y_rows = 0, y2_rows = 0;        // extents of y / y2 (bounds-checking mode)
  int check = 0;                       // bounds-checking mode
  int* status = nullptr;
};

void moe_route(const MoeRouteArgs& a, cudaStream_t s);
void moe_plan(const int* counts, int E, int ns, int N, int* seg_start, int* seg_count,
              int* tile_expert, int* tile_row, int* total_mtiles, int* kstart, int* kend,
              int* cursor, int max_mtiles, cudaStream_t s);
void moe_dispatch(const __nv_bfloat16* x, long ldx, int N, int d, int k, int ns, int E,
                  const int* topk_idx, const int* seg_start, const int* seg_count, int* cursor,
                  __nv_bfloat16* xp, long ldp, int* slot_of, cudaStream_t s,
                  __nv_bfloat16* xp2 = nullptr, long ldp2 = 0, bool zero_routed_pad = true,
                  long xp_rows = 0, long xp2_rows = 0);
void moe_zero_pad(const int* seg_start, const int* seg_count, int nseg, __nv_bfloat16* xp, long ldp,
                  int d, cudaStream_t s);
void moe_combine(const MoeCombineArgs& a, cudaStream_t s);
void moe_combine_bwd(const MoeCombineArgs& a, const __nv_bfloat16* dout, long ld_dout,
                     __nv_bfloat16* dy, float* dw, cudaStream_t s, __nv_bfloat16* dy2 = nullptr);
// routes j >= k read dxp2 (when non-null) instead of dxp
void moe_unpermute(const __nv_bfloat16* dxp, long ldp, const int* slot_of, int N, int R, int d,
                   __nv_bfloat16* dx, long ldx, cudaStream_t s, int k = 0,
                   const __nv_bfloat16* dxp2 = nullptr, long ldp2 = 0, long rows = 0,
                   long rows2 = 0);

// ---- expert parallelism: row-block copies between local and peer (IPC) buffers
struct EpCopyArgs {
  const void* const* src_table = nullptr;  // device array: base pointer per rank; null -> src_local
  void* const* dst_table = nullptr;        // null -> dst_local
  const void* src_local = nullptr;
  void* dst_local = nullptr;
  const int* blocks = nullptr;             // device [nblocks, 4]: src_rank, src_row, dst_rank, dst_row
  const int* row_prefix = nullptr;         // device [nblocks]: first flat row of each block
  int nblocks = 0;
  long total_rows = 0;
  int row_bytes = 0;                       // bytes copied per row (multiple of 16)
  long src_ld = 0, dst_ld = 0;             // row strides in bytes
};
void ep_copy_rows(const EpCopyArgs& a, cudaStream_t stream);

// ---- expert parallelism, one row per (token, owner rank) each way
// Every source pushes each token row ONCE to every rank owning one of its experts
// (ep_push_rows, P2P stores into the owner's staging rows); the owner of experts
// [lo, lo + El) fans its staged rows out into its local expert segments (ep_owner_fanout);
// after the expert GEMMs it sums the token's local expert outputs (weighted) and stores
// that one row into the source's return buffer. Sources add the rows of the owners they
// used. Backward pushes the output-gradient rows to the same staging positions.
struct EpOwnerArgs {
  int world = 0, rank = 0, N = 0, k = 0, d = 0, lo = 0, El = 0;
  const int* const* peer_idx = nullptr;              // [world] -> [N, k] int32 routed expert ids
  const float* const* peer_w = nullptr;              // [world] -> [N, k] fp32 routed weights
  const __nv_bfloat16* const* peer_rows = nullptr;   // [world] -> [N, d] rows (h, or dout)
  const int* seg_start = nullptr;                    // [El] owner-layout segment starts
  int* cursor = nullptr;                             // [El] zeroed
  __nv_bfloat16* xr = nullptr;                       // owner layout rows
  long ld_xr = 0;
  // unique (source, token) rows that route here: [cap] x (2 + k) int32 = (s, t, slot per route
  // or -1) and [cap] x k fp32 weights; count in *n_uniq
  int* meta = nullptr;
  float* meta_w = nullptr;
  int* n_uniq = nullptr;
  int cap = 0;
  // gradient gather from local staging rows (pushed by the sources) instead of peer rows:
  // the dout row of unique row u is local_rows[urow[u]]
  const __nv_bfloat16* local_rows = nullptr;
  const int* urow = nullptr;
};

// Source-side push of token rows to their expert owners (P2P stores). Forward mode
// (smeta != nullptr): each token's row goes once to every rank owning one of its experts,
// into that owner's staging rows [rank * N + p] (p = the token's position among this
// rank's tokens for that owner, from cnt[o]), with a record (t, expert ids on that owner or
// -1, weights) in the owner's staging metadata; pos[t * world + o] = p or -1. Gradient
// mode (smeta == nullptr): the rows go to the same staging positions, read from pos.
struct EpPushArgs {
  int world = 0, rank = 0, N = 0, k = 0, d = 0, El = 0;
  const int* idx = nullptr;            // [N, k]
  const float* w = nullptr;            // [N, k]
  const __nv_bfloat16* rows = nullptr; // [N, d] (h, or dout)
  long ld_rows = 0;
  __nv_bfloat16* const* stage = nullptr;  // [world] -> [world * N, d] staging rows
  int* const* smeta = nullptr;            // [world] -> [world * N, 1 + 2k] records
  int* cnt = nullptr;                     // [world] zeroed: rows pushed to each owner
  int* pos = nullptr;                     // [N, world]
};
void ep_push_rows(const EpPushArgs& a, cudaStream_t s);

// Owner side after the pushes landed: staged rows u in [0, total) (sources in order, row
// u of source s at stage[s * N + u - prefix[s]]) fan out into the local experts' segments
// of xr; meta [total, 2 + k] = (source, token, slot per route or -1), meta_w [total, k],
// *n_uniq = total, urow[u] = staging row.
struct EpFanoutArgs {
  int world = 0, N = 0, k = 0, d = 0, lo = 0, El = 0, total = 0;
  const __nv_bfloat16* stage = nullptr;
  const int* smeta = nullptr;
  const int* prefix = nullptr;  // [world + 1]
  const int* seg_start = nullptr;
  int* cursor = nullptr;
  __nv_bfloat16* xr = nullptr;
  long ld_xr = 0;
  int* meta = nullptr;
  float* meta_w = nullptr;
  int* urow = nullptr;
  int* n_uniq = nullptr;
};
void ep_owner_fanout(const EpFanoutArgs& a, cudaStream_t s);
// backward dispatch: per unique row reads dout once (local staging row urow[u], or the
// source's peer_rows), writes dy[slot] = w dout and
// stores dw = dout . y[slot] into the source's dw buffer (peer_dw[s][t * k + j])
void ep_owner_grad_gather(const EpOwnerArgs& a, const __nv_bfloat16* y, long ld_y, __nv_bfloat16* dy,
                          long ld_dy, float* const* peer_dw, cudaStream_t s);
// owner combine: per unique row z = sum_j (weighted ? w_j : 1) src[slot_j]; stored (bf16) into
// peer_ret[s] + ((rank * N) + t) * d
void ep_owner_scatter_sum(const EpOwnerArgs& a, const __nv_bfloat16* src, long ld_src, bool weighted,
                          __nv_bfloat16* const* peer_ret, cudaStream_t s);
// source combine: out[t] = residual[t] + sum_{owners o of t's experts} ret[o * N + t]
//                          + sum_s g[t, s] shared[slot_of_s[t, s]]   (g = 1 when shared_w null)
struct EpSourceArgs {
  int N = 0, k = 0, d = 0, El = 0, ns = 0;
  const int* idx = nullptr;                 // [N, k]
  const __nv_bfloat16* ret = nullptr;       // [world * N, d]
  const __nv_bfloat16* residual = nullptr;  // [N, d] or null
  long ld_res = 0;
  const float* shared_w = nullptr;          // [N, ns] or null (unit gates)
  const int* slot_s = nullptr;              // [N, ns]
  const __nv_bfloat16* ys = nullptr;        // shared-expert rows
  long ld_ys = 0;
  __nv_bfloat16* out = nullptr;
  long ld_out = 0;
  long y_rows = 0, y2_rows = 0;        // extents of y / y2 (bounds-checking mode)
  int check = 0;                       // bounds-checking mode
  int* status = nullptr;
};
void ep_source_reduce(const EpSourceArgs& a, cudaStream_t s);

}  // namespace ddb
