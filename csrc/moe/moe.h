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
};

void moe_route(const MoeRouteArgs& a, cudaStream_t s);
void moe_plan(const int* counts, int E, int ns, int N, int* seg_start, int* seg_count,
              int* tile_expert, int* tile_row, int* total_mtiles, int* kstart, int* kend,
              int* cursor, int max_mtiles, cudaStream_t s);
void moe_dispatch(const __nv_bfloat16* x, long ldx, int N, int d, int k, int ns, int E,
                  const int* topk_idx, const int* seg_start, const int* seg_count, int* cursor,
                  __nv_bfloat16* xp, long ldp, int* slot_of, cudaStream_t s,
                  __nv_bfloat16* xp2 = nullptr, long ldp2 = 0, bool zero_routed_pad = true);
void moe_zero_pad(const int* seg_start, const int* seg_count, int nseg, __nv_bfloat16* xp, long ldp,
                  int d, cudaStream_t s);
void moe_combine(const MoeCombineArgs& a, cudaStream_t s);
void moe_combine_bwd(const MoeCombineArgs& a, const __nv_bfloat16* dout, long ld_dout,
                     __nv_bfloat16* dy, float* dw, cudaStream_t s, __nv_bfloat16* dy2 = nullptr);
// routes j >= k read dxp2 (when non-null) instead of dxp
void moe_unpermute(const __nv_bfloat16* dxp, long ldp, const int* slot_of, int N, int R, int d,
                   __nv_bfloat16* dx, long ldx, cudaStream_t s, int k = 0,
                   const __nv_bfloat16* dxp2 = nullptr, long ldp2 = 0);

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

}  // namespace ddb
